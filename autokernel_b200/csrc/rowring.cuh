// Persistent, TMA-staged row kernels (see rowring.cu).
#pragma once
#include "ak_common.cuh"

namespace ak {

enum RingOp { RING_SOFTMAX = 2 };

struct RingArgs {
  const void* x;
  void* y;              // softmax output
  int64_t rows, cols, ldx, ldy;
};

// Runs softmax through the ring kernel when the rows qualify (16-byte aligned
// rows of 16-64 KiB).  Returns AK_OK, a negative
// error, or 1 when the caller should use another kernel.
int ring_rowop(int op, int dtype, const RingArgs& a, cudaStream_t s);

}  // namespace ak
