// Host-side interface of the tcgen05 GEMM (gemm_sm100.cu) used by the C ABI.
#pragma once
#include "ak_common.cuh"

namespace ak {

// Rotary embedding applied in the GEMM epilogue to output columns [0, cols): interleaved
// pairs inside head_dim-wide column groups, position = row % T, fp32 cos/sin [T, head_dim / 2].
struct RopeEpilogue {
  const float* cos = nullptr;
  const float* sin = nullptr;
  int T = 1, head_dim = 2, cols = 0;
};

// LM head + cross entropy (MODE_XENT): per-row partials of every 256-column vocab tile.
struct XentEpilogue {
  const int64_t* targets = nullptr;  // [M]
  float* part = nullptr;             // [ceil(N / 256)][M] pairs (max, sum of exp)
  float* tgt = nullptr;              // [M] target logits (written by the tile holding them)
};
constexpr int kXentTileN = 256;

// RMSNorm folded into a K-major GEMM: each output row is scaled by 1 / sqrt(mean + eps) from
// the per-row partial sums of squares rs_in [rs_tiles][M] of the A operand (the norm weight is
// folded into B), and / or the stored outputs' per-row sums of squares are written to
// ss_out [ceil(N / 256)][M] for the next norm.
struct RmsEpilogue {
  const float* rs_in = nullptr;
  int rs_tiles = 0;
  float eps = 0.f;
  float* ss_out = nullptr;
};
constexpr int kRmsTileN = 256;

int tc_gemm_rms(int dtype, bool dual, const void* A, const void* B, const void* B2, void* C,
                int M, int N, int K, int64_t lda, int64_t ldb, int64_t ldc, int act,
                const void* R, int64_t ldr, const RmsEpilogue& rms, const RopeEpilogue& rope,
                cudaStream_t st);

int tc_gemm_xent(int dtype, const void* x, const void* w, int M, int N, int K, int64_t ldx,
                 int64_t ldw, const XentEpilogue& xe, cudaStream_t st);

bool tc_gemm_ok(int dtype, const void* A, const void* B, const void* B2, int64_t K, int64_t lda,
                int64_t ldb, bool b_mn);
int tc_gemm(int dtype, int mode, const void* A, const void* B, const void* B2, void* C, int M,
            int N, int K, int64_t lda, int64_t ldb, int64_t ldc, int act, const void* R,
            int64_t ldr, const RopeEpilogue& rope, cudaStream_t st);

}  // namespace ak
