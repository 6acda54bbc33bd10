// LM head fused with cross entropy: per-row losses of logits = x @ W^T without ever storing
// the logits (models/llama_7b.py's output projection followed by reference.py:58-60).
//
// Pass 1 is the tcgen05 GEMM in MODE_XENT (gemm_sm100.cu): every 128 x 256 tile of logits
// lives only in TMEM; its epilogue rounds the logits to the dtype, reduces each row to a
// (max, sum of exp) pair per 256-column vocab tile and copies out the target logit.  Pass 2
// (this file) merges a row's ceil(vocab / 256) pairs in fixed order:
//   M = max_t m_t,  S = sum_t s_t * exp(m_t - M),  loss = M + log(S) - logit[target].
// For a [65536, 32000] fp16 LM head that replaces a 4.2 GB write and re-read with 66 MB of
// partials.  Rows whose target is ignore_index get loss 0; a target outside [0, vocab)
// gives NaN and raises *bad_target.  Deterministic: no atomics in the sums.
#include "ak_common.cuh"
#include "gemm.cuh"
#include "sm100.cuh"

namespace ak {

__global__ void __launch_bounds__(256) xent_merge_kernel(const float2* part, int tiles,
                                                         const float* tgt,
                                                         const int64_t* targets, int64_t rows,
                                                         int64_t vocab, int64_t ignore_index,
                                                         float* row_loss, float* row_max,
                                                         float* row_tgt, int* bad_target) {
  constexpr float kL2e = 1.4426950408889634f;
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= rows) return;
  float m = -INFINITY;
  for (int t = 0; t < tiles; ++t) m = fmaxf(m, part[(int64_t)t * rows + row].x);
  float s = 0.f;
  for (int t = 0; t < tiles; ++t) {
    const float2 q = part[(int64_t)t * rows + row];
    if (q.x != -INFINITY) s += q.y * sm100::ex2_approx((q.x - m) * kL2e);
  }
  const int64_t tg = targets[row];
  float loss, tl;
  if (tg == ignore_index) {
    loss = 0.f;
    tl = NAN;
  } else if (tg < 0 || tg >= vocab) {
    loss = NAN;
    tl = NAN;
    if (bad_target) atomicExch(bad_target, 1);
  } else {
    tl = tgt[row];
    loss = (m + logf(s)) - tl;
  }
  row_loss[row] = loss;
  if (row_max) row_max[row] = m;
  if (row_tgt) row_tgt[row] = tl;
}

static size_t xent_tiles(int64_t vocab) { return (size_t)((vocab + kXentTileN - 1) / kXentTileN); }

}  // namespace ak

using namespace ak;

extern "C" size_t ak_linear_cross_entropy_workspace_size(int64_t rows, int64_t vocab) {
  if (rows <= 0 || vocab <= 0) return 256;
  return xent_tiles(vocab) * (size_t)rows * sizeof(float2) + (size_t)rows * sizeof(float) + 256;
}

extern "C" int ak_linear_cross_entropy_rows(const void* x, const void* w, const int64_t* targets,
                                            int64_t rows, int64_t vocab, int64_t dim,
                                            int64_t ldx, int64_t ldw, int dtype,
                                            int64_t ignore_index, void* workspace,
                                            size_t ws_bytes, float* row_loss, float* row_max,
                                            float* row_target_logit, int* bad_target,
                                            void* stream) {
  AK_REQUIRE(dtype == AK_F16 || dtype == AK_BF16, AK_ERR_DTYPE,
             "linear_cross_entropy: 16-bit x and weight only (dtype %d)", dtype);
  AK_REQUIRE(rows >= 0 && vocab > 0 && dim > 0, AK_ERR_SHAPE, "bad shape");
  AK_REQUIRE(rows < (1LL << 31) && vocab < (1LL << 31) && dim < (1LL << 31), AK_ERR_SHAPE,
             "dimension exceeds 2^31-1");
  AK_REQUIRE(ldx >= dim && ldw >= dim, AK_ERR_SHAPE, "leading dimension too small");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(x && w && targets && row_loss && workspace, AK_ERR_ARG, "null pointer");
  AK_REQUIRE(ws_bytes >= ak_linear_cross_entropy_workspace_size(rows, vocab), AK_ERR_ARG,
             "workspace of %zu bytes, need %zu", ws_bytes,
             ak_linear_cross_entropy_workspace_size(rows, vocab));
  AK_REQUIRE(tc_gemm_ok(dtype, x, w, nullptr, dim, ldx, ldw, false), AK_ERR_ARG,
             "linear_cross_entropy: x / weight not TMA-describable (16-byte aligned base and "
             "row stride needed)");
  const size_t tiles = xent_tiles(vocab);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  ws += (256 - (reinterpret_cast<uintptr_t>(ws) & 255)) & 255;
  float* part = reinterpret_cast<float*>(ws);
  float* tgt = reinterpret_cast<float*>(ws + tiles * (size_t)rows * sizeof(float2));
  cudaStream_t st = (cudaStream_t)stream;
  XentEpilogue xe;
  xe.targets = targets;
  xe.part = part;
  xe.tgt = tgt;
  int rc = tc_gemm_xent(dtype, x, w, (int)rows, (int)vocab, (int)dim, ldx, ldw, xe, st);
  if (rc) return rc;
  xent_merge_kernel<<<(unsigned)((rows + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const float2*>(part), (int)tiles, tgt, targets, rows, vocab,
      ignore_index, row_loss, row_max, row_target_logit, bad_target);
  return launch_status("linear_cross_entropy");
}
