// C-ABI entry points for the contractions: matmul, fused MLP and attention.
// Each picks the tcgen05 tensor-core kernel when the operands are 16-bit and
// TMA-describable, and the SIMT kernel otherwise (fp32, odd strides).  The
// choice depends only on dtype/shape/alignment, never on the data, so a given
// call is bitwise reproducible.
#include "ak_common.cuh"
#include "attn.cuh"
#include "gemm.cuh"

#include <cstdlib>

namespace ak {
int simt_gemm_any(int dtype, const void* A, const void* B, const void* B2, void* C, int M, int N,
                  int K, int64_t lda, int64_t ldb, int64_t ldc, int b_kmajor, int act,
                  const void* R, int64_t ldr, cudaStream_t s);
int simt_attention_any(int dtype, const void* Q, const void* K, const void* V, void* O,
                       int64_t bh, int Sq, int Sk, int D, int causal, float scale,
                       cudaStream_t s);

// Route every contraction through the SIMT kernels: set by ak_set_force_simt()
// or, at load time, by the environment variable AK_FORCE_SIMT=1.
static int g_force_simt = [] {
  const char* e = getenv("AK_FORCE_SIMT");
  return (e && e[0] == '1') ? 1 : 0;
}();
}  // namespace ak

using namespace ak;

extern "C" void ak_set_force_simt(int on) { g_force_simt = on; }

extern "C" int ak_matmul_add(const void* A, const void* B, void* C, const void* R, int64_t M,
                             int64_t N, int64_t K, int64_t lda, int64_t ldb, int64_t ldc,
                             int64_t ldr, int b_kmajor, int dtype, void* stream) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(M >= 0 && N >= 0 && K >= 0, AK_ERR_SHAPE, "negative shape");
  AK_REQUIRE(M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31), AK_ERR_SHAPE,
             "dimension exceeds 2^31-1");
  AK_REQUIRE(lda >= K && ldc >= N && ldb >= (b_kmajor ? K : N) && (!R || ldr >= N),
             AK_ERR_SHAPE, "leading dimension too small");
  if (M == 0 || N == 0) return AK_OK;
  AK_REQUIRE(A && B && C, AK_ERR_ARG, "null tensor pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (K == 0) {
    // empty contraction: C = R (or 0)
    const size_t es = dtype_size(dtype);
    cudaError_t e = R ? cudaMemcpy2DAsync(C, ldc * es, R, ldr * es, N * es, M,
                                          cudaMemcpyDeviceToDevice, st)
                      : cudaMemset2DAsync(C, ldc * es, 0, N * es, M, st);
    AK_REQUIRE(e == cudaSuccess, AK_ERR_LAUNCH, "empty contraction: %s", cudaGetErrorString(e));
    return AK_OK;
  }
  if (!g_force_simt && tc_gemm_ok(dtype, A, B, nullptr, K, lda, ldb, !b_kmajor) &&
      (b_kmajor || N % 8 == 0))
    return tc_gemm(dtype, b_kmajor ? 0 : 1, A, B, nullptr, C, (int)M, (int)N, (int)K, lda, ldb,
                   ldc, 0, R, ldr, RopeEpilogue(), st);
  return simt_gemm_any(dtype, A, B, nullptr, C, (int)M, (int)N, (int)K, lda, ldb, ldc, b_kmajor,
                       0, R, ldr, st);
}

extern "C" int ak_linear_rope(const void* x, const void* w, void* out, int64_t M, int64_t N,
                              int64_t K, int64_t ldx, int64_t ldo, const float* cos,
                              const float* sin, int64_t T, int64_t head_dim, int64_t rope_cols,
                              int dtype, void* stream) {
  AK_REQUIRE(dtype == AK_F16 || dtype == AK_BF16, AK_ERR_DTYPE,
             "ak_linear_rope: 16-bit inputs only (tensor-core epilogue)");
  AK_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1LL << 31) && N < (1LL << 31) &&
                 K < (1LL << 31),
             AK_ERR_SHAPE, "bad shape");
  AK_REQUIRE(ldx >= K && ldo >= N, AK_ERR_SHAPE, "leading dimension too small");
  AK_REQUIRE(T > 0 && T < (1LL << 31) && head_dim % 32 == 0 && head_dim > 0 &&
                 rope_cols >= 0 && rope_cols <= N && rope_cols % head_dim == 0,
             AK_ERR_SHAPE, "rope: need head_dim a multiple of 32 and rope_cols a multiple of it");
  if (M == 0) return AK_OK;
  AK_REQUIRE(x && w && out && (rope_cols == 0 || (cos && sin)), AK_ERR_ARG, "null pointer");
  AK_REQUIRE(!g_force_simt && tc_gemm_ok(dtype, x, w, nullptr, K, ldx, K, false),
             AK_ERR_UNSUPPORTED, "ak_linear_rope needs TMA-describable operands on sm_100");
  RopeEpilogue rope;
  rope.cos = cos;
  rope.sin = sin;
  rope.T = (int)T;
  rope.head_dim = (int)head_dim;
  rope.cols = (int)rope_cols;
  return tc_gemm(dtype, 0, x, w, nullptr, out, (int)M, (int)N, (int)K, ldx, K, ldo, 0, nullptr,
                 0, rope, (cudaStream_t)stream);
}

extern "C" int ak_matmul(const void* A, const void* B, void* C, int64_t M, int64_t N, int64_t K,
                         int64_t lda, int64_t ldb, int64_t ldc, int b_kmajor, int dtype,
                         void* stream) {
  return ak_matmul_add(A, B, C, nullptr, M, N, K, lda, ldb, ldc, 0, b_kmajor, dtype, stream);
}

extern "C" int ak_mlp_gate_up(const void* x, const void* w_gate, const void* w_up, void* hidden,
                              int64_t M, int64_t D, int64_t H, int activation, int dtype,
                              void* stream) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(activation >= AK_ACT_SILU && activation <= AK_ACT_RELU2, AK_ERR_ARG,
             "unknown activation %d", activation);
  AK_REQUIRE(M >= 0 && D >= 0 && H >= 0 && M < (1LL << 31) && D < (1LL << 31) &&
                 H < (1LL << 31),
             AK_ERR_SHAPE, "bad shape");
  if (M == 0 || H == 0) return AK_OK;
  AK_REQUIRE(x && w_gate && w_up && hidden, AK_ERR_ARG, "null tensor pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (!g_force_simt && D > 0 && tc_gemm_ok(dtype, x, w_gate, w_up, D, D, D, false))
    return tc_gemm(dtype, 2, x, w_gate, w_up, hidden, (int)M, (int)H, (int)D, D, D, H,
                   activation, nullptr, 0, RopeEpilogue(), st);
  return simt_gemm_any(dtype, x, w_gate, w_up, hidden, (int)M, (int)H, (int)D, D, D, H, 1,
                       activation, nullptr, 0, st);
}

extern "C" int ak_fused_mlp(const void* x, const void* w_gate, const void* w_up,
                            const void* w_down, void* hidden, void* out, int64_t M, int64_t D,
                            int64_t H, int activation, int dtype, void* stream) {
  int rc = ak_mlp_gate_up(x, w_gate, w_up, hidden, M, D, H, activation, dtype, stream);
  if (rc) return rc;
  // out[M, D] = hidden[M, H] @ w_down[D, H]^T
  return ak_matmul(hidden, w_down, out, M, D, H, H, H, D, 1, dtype, stream);
}

extern "C" int ak_flash_attention_strided(const void* Q, const void* K, const void* V, void* O,
                                          int64_t B, int64_t H, int64_t Hkv, int64_t Sq,
                                          int64_t Sk, int64_t D, const int64_t* q_strides,
                                          const int64_t* k_strides, const int64_t* v_strides,
                                          const int64_t* o_strides, int causal, float sm_scale,
                                          int dtype, void* stream) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(B >= 0 && H >= 0 && Hkv > 0 && Sq >= 0 && Sk >= 0 && D > 0, AK_ERR_SHAPE,
             "bad shape");
  AK_REQUIRE(H % Hkv == 0, AK_ERR_SHAPE, "query heads %lld not a multiple of kv heads %lld",
             (long long)H, (long long)Hkv);
  AK_REQUIRE(Sq < (1LL << 31) && Sk < (1LL << 31), AK_ERR_SHAPE, "sequence too long");
  if (B == 0 || H == 0 || Sq == 0) return AK_OK;
  AK_REQUIRE(Sk > 0, AK_ERR_SHAPE, "attention over zero keys");
  AK_REQUIRE(Q && K && V && O && q_strides && k_strides && v_strides && o_strides, AK_ERR_ARG,
             "null pointer");
  AttnShape a;
  a.Q = Q; a.K = K; a.V = V; a.O = O;
  a.B = B; a.H = H; a.Hkv = Hkv;
  a.Sq = (int)Sq; a.Sk = (int)Sk; a.D = (int)D;
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = q_strides[i]; a.ks[i] = k_strides[i];
    a.vs[i] = v_strides[i]; a.os[i] = o_strides[i];
  }
  a.causal = causal; a.scale = sm_scale; a.dtype = dtype;
  AK_REQUIRE(!g_force_simt && tc_attention_ok(a), AK_ERR_UNSUPPORTED,
             "strided attention needs 16-bit inputs, head_dim 64 or 128 and 16-byte aligned "
             "strides on sm_100; use ak_flash_attention on contiguous tensors");
  return tc_attention(a, (cudaStream_t)stream);
}

extern "C" int ak_flash_attention(const void* Q, const void* K, const void* V, void* O,
                                  int64_t batch_heads, int64_t Sq, int64_t Sk, int64_t D,
                                  int causal, float sm_scale, int dtype, void* stream) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(batch_heads >= 0 && Sq >= 0 && Sk >= 0 && D > 0, AK_ERR_SHAPE, "bad shape");
  AK_REQUIRE(Sq < (1LL << 31) && Sk < (1LL << 31), AK_ERR_SHAPE, "sequence too long");
  if (batch_heads == 0 || Sq == 0) return AK_OK;
  AK_REQUIRE(Sk > 0, AK_ERR_SHAPE, "attention over zero keys");
  AK_REQUIRE(Q && K && V && O, AK_ERR_ARG, "null tensor pointer");
  cudaStream_t st = (cudaStream_t)stream;
  // contiguous [BH, S, D]: batch = BH, one head per batch entry
  AttnShape a;
  a.Q = Q; a.K = K; a.V = V; a.O = O;
  a.B = batch_heads; a.H = 1; a.Hkv = 1;
  a.Sq = (int)Sq; a.Sk = (int)Sk; a.D = (int)D;
  const int64_t qst[3] = {Sq * D, Sq * D, D}, kst[3] = {Sk * D, Sk * D, D};
  for (int i = 0; i < 3; ++i) {
    a.qs[i] = qst[i]; a.os[i] = qst[i]; a.ks[i] = kst[i]; a.vs[i] = kst[i];
  }
  a.causal = causal; a.scale = sm_scale; a.dtype = dtype;
  if (!g_force_simt && tc_attention_ok(a)) return tc_attention(a, st);
  return simt_attention_any(dtype, Q, K, V, O, batch_heads, (int)Sq, (int)Sk, (int)D, causal,
                            sm_scale, st);
}

// ------------------------------------------------------------------ RMSNorm folded into GEMMs
namespace ak {
// Per-row sums of squares of x [rows, cols] over 256-column tiles: ss[t][row].  One warp per
// (row, tile); the values are read as 16-byte vectors when the row allows it.
template <int DT>
__global__ void __launch_bounds__(256) row_sumsq_kernel(const void* xv, int64_t rows,
                                                        int64_t cols, int64_t ld, float* ss) {
  using E = Elem<DT>;
  using T = typename E::T;
  const int64_t row = (int64_t)blockIdx.y * 8 + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const int64_t c0 = (int64_t)blockIdx.x * kRmsTileN;
  const T* x = reinterpret_cast<const T*>(xv) + row * ld;
  float acc = 0.f;
  const bool vec = (ld % 8 == 0) && aligned16(xv) && c0 + kRmsTileN <= cols;
  if (vec) {
    float f[8];
    load_vec<DT>(x + c0 + lane * 8, f);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc = fmaf(f[j], f[j], acc);
  } else {
    for (int64_t c = c0 + lane; c < min(c0 + kRmsTileN, cols); c += 32) {
      const float f = E::to_f(x[c]);
      acc = fmaf(f, f, acc);
    }
  }
  acc = warp_sum(acc);
  if (lane == 0) ss[(int64_t)blockIdx.x * rows + row] = acc;
}
}  // namespace ak

extern "C" int ak_row_sumsq(const void* x, int64_t rows, int64_t cols, int64_t ld, int dtype,
                            float* ss_out, void* stream) {
  AK_REQUIRE(dtype == AK_F16 || dtype == AK_BF16, AK_ERR_DTYPE, "row_sumsq: 16-bit x only");
  AK_REQUIRE(rows >= 0 && cols > 0 && ld >= cols && rows < (1LL << 31), AK_ERR_SHAPE,
             "bad shape");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(x && ss_out, AK_ERR_ARG, "null pointer");
  cudaStream_t st = (cudaStream_t)stream;
  dim3 grid((unsigned)((cols + kRmsTileN - 1) / kRmsTileN), (unsigned)((rows + 7) / 8));
  if (dtype == AK_BF16)
    row_sumsq_kernel<AK_BF16><<<grid, 256, 0, st>>>(x, rows, cols, ld, ss_out);
  else
    row_sumsq_kernel<AK_F16><<<grid, 256, 0, st>>>(x, rows, cols, ld, ss_out);
  return launch_status("row_sumsq");
}

static int rms_common_checks(const void* x, const void* w, int64_t M, int64_t N, int64_t K,
                             int64_t ldx, int dtype, const float* rs_in, int rs_tiles) {
  AK_REQUIRE(dtype == AK_F16 || dtype == AK_BF16, AK_ERR_DTYPE,
             "RMSNorm-fused GEMM: 16-bit operands only (dtype %d)", dtype);
  AK_REQUIRE(M >= 0 && N > 0 && K > 0 && M < (1LL << 31) && N < (1LL << 31) && K < (1LL << 31),
             AK_ERR_SHAPE, "bad shape");
  AK_REQUIRE(ldx >= K, AK_ERR_SHAPE, "leading dimension too small");
  AK_REQUIRE(!rs_in || rs_tiles > 0, AK_ERR_ARG, "rs_in given without rs_tiles");
  AK_REQUIRE(!g_force_simt && tc_gemm_ok(dtype, x, w, nullptr, K, ldx, K, false), AK_ERR_ARG,
             "RMSNorm-fused GEMM needs the tensor-core path (16-byte aligned operands)");
  return AK_OK;
}

extern "C" int ak_linear_rms(const void* x, const void* w, void* C, const void* R, int64_t M,
                             int64_t N, int64_t K, int64_t ldx, int64_t ldc, int64_t ldr,
                             const float* rs_in, int rs_tiles, float eps, float* ss_out,
                             const float* cos, const float* sin, int64_t T, int64_t head_dim,
                             int64_t rope_cols, int dtype, void* stream) {
  int rc = rms_common_checks(x, w, M, N, K, ldx, dtype, rs_in, rs_tiles);
  if (rc) return rc;
  AK_REQUIRE(ldc >= N && (!R || ldr >= N), AK_ERR_SHAPE, "leading dimension too small");
  if (M == 0) return AK_OK;
  AK_REQUIRE(C, AK_ERR_ARG, "null output");
  RmsEpilogue rms;
  rms.rs_in = rs_in;
  rms.rs_tiles = rs_tiles;
  rms.eps = eps;
  rms.ss_out = ss_out;
  RopeEpilogue rope;
  if (cos) {
    AK_REQUIRE(sin && T > 0 && head_dim > 0 && head_dim % 2 == 0 && rope_cols >= 0 &&
                   rope_cols <= N && rope_cols % head_dim == 0 && T < (1LL << 31),
               AK_ERR_ARG, "bad RoPE epilogue arguments");
    rope.cos = cos;
    rope.sin = sin;
    rope.T = (int)T;
    rope.head_dim = (int)head_dim;
    rope.cols = (int)rope_cols;
  }
  return tc_gemm_rms(dtype, false, x, w, nullptr, C, (int)M, (int)N, (int)K, ldx, K, ldc, 0, R,
                     ldr, rms, rope, (cudaStream_t)stream);
}

extern "C" int ak_mlp_gate_up_rms(const void* x, const void* w_gate, const void* w_up,
                                  void* hidden, int64_t M, int64_t D, int64_t H,
                                  const float* rs_in, int rs_tiles, float eps, int activation,
                                  int dtype, void* stream) {
  int rc = rms_common_checks(x, w_gate, M, H, D, D, dtype, rs_in, rs_tiles);
  if (rc) return rc;
  AK_REQUIRE(activation >= AK_ACT_SILU && activation <= AK_ACT_RELU2, AK_ERR_ARG,
             "unknown activation %d", activation);
  AK_REQUIRE(aligned16(w_up), AK_ERR_ARG, "w_up not 16-byte aligned");
  if (M == 0) return AK_OK;
  AK_REQUIRE(hidden, AK_ERR_ARG, "null output");
  RmsEpilogue rms;
  rms.rs_in = rs_in;
  rms.rs_tiles = rs_tiles;
  rms.eps = eps;
  return tc_gemm_rms(dtype, true, x, w_gate, w_up, hidden, (int)M, (int)H, (int)D, D, D, H,
                     activation, nullptr, 0, rms, RopeEpilogue(), (cudaStream_t)stream);
}
