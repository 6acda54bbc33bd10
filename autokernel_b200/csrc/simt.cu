// SIMT (CUDA-core) kernels for the contractions, used where the tensor-core
// path does not apply:
//   * fp32 inputs (the reference's fp32 tolerance of 1e-4 rules out
//     tf32/bf16 tensor-core arithmetic), and
//   * shapes whose row strides are not 16-byte multiples (K or N not a
//     multiple of 8 in 16-bit types, e.g. the 1023/4097/1537 edge sizes),
//     which TMA cannot describe.
// Accumulation is fp32 in a fixed order; no atomics (bitwise deterministic).
//
//   simt_gemm:  C = A @ op(B) [+ R]  reference.py:10-12 (matmul_ref)
//   simt_dual:  H = act(A @ Wg^T) * (A @ Wu^T)   first half of reference.py:45-55
//   simt_attn:  O = softmax(Q K^T * scale [+ causal mask]) V   reference.py:32-42
#include "ak_common.cuh"
#include "ak_act.cuh"

namespace ak {

constexpr int SB_M = 64, SB_N = 64, SB_K = 16;

// B element (k, n): B is [K, N] row-major (b_kmajor = 0) or [N, K] row-major
// (b_kmajor = 1, i.e. the product is A @ B^T).
template <int DT, bool DUAL>
__global__ void __launch_bounds__(256) simt_gemm_kernel(const void* Av, const void* Bv,
                                                        const void* B2v, void* Cv, int M, int N,
                                                        int K, int64_t lda, int64_t ldb,
                                                        int64_t ldc, int b_kmajor, int act,
                                                        const void* Rv, int64_t ldr) {
  using E = Elem<DT>;
  using T = typename E::T;
  const T* A = reinterpret_cast<const T*>(Av);
  const T* B = reinterpret_cast<const T*>(Bv);
  const T* B2 = reinterpret_cast<const T*>(B2v);
  T* C = reinterpret_cast<T*>(Cv);
  __shared__ float As[SB_K][SB_M + 4];
  __shared__ float Bs[SB_K][SB_N + 4];
  __shared__ float B2s[DUAL ? SB_K : 1][DUAL ? SB_N + 4 : 1];

  const int m0 = blockIdx.y * SB_M, n0 = blockIdx.x * SB_N;
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  float acc[4][4] = {}, acc2[DUAL ? 4 : 1][DUAL ? 4 : 1] = {};

  for (int k0 = 0; k0 < K; k0 += SB_K) {
    for (int i = threadIdx.x; i < SB_M * SB_K; i += 256) {
      const int mm = i / SB_K, kk = i % SB_K;  // consecutive threads walk k: A is K-contiguous
      const int gm = m0 + mm, gk = k0 + kk;
      As[kk][mm] = (gm < M && gk < K) ? E::to_f(A[(int64_t)gm * lda + gk]) : 0.f;
    }
    for (int i = threadIdx.x; i < SB_N * SB_K; i += 256) {
      int nn, kk;
      if (b_kmajor) { nn = i / SB_K; kk = i % SB_K; }
      else { kk = i / SB_N; nn = i % SB_N; }
      const int gn = n0 + nn, gk = k0 + kk;
      const bool ok = gn < N && gk < K;
      const int64_t off = b_kmajor ? (int64_t)gn * ldb + gk : (int64_t)gk * ldb + gn;
      Bs[kk][nn] = ok ? E::to_f(B[off]) : 0.f;
      if (DUAL) B2s[kk][nn] = ok ? E::to_f(B2[off]) : 0.f;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < SB_K; ++kk) {
      float a[4], b[4], b2[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
      if (DUAL) {
#pragma unroll
        for (int j = 0; j < 4; ++j) b2[j] = B2s[kk][tx * 4 + j];
      }
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
          if (DUAL) acc2[i][j] = fmaf(a[i], b2[j], acc2[i][j]);
        }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gm = m0 + ty * 4 + i;
    if (gm >= M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int gn = n0 + tx * 4 + j;
      if (gn >= N) continue;
      float v = acc[i][j];
      if (DUAL) v = swiglu_ref<DT>(act, v, acc2[i][j]);
      if (Rv) v += E::to_f(reinterpret_cast<const T*>(Rv)[(int64_t)gm * ldr + gn]);
      C[(int64_t)gm * ldc + gn] = E::from_f(v);
    }
  }
}

// One warp per query row.  Lane j of the warp scores key (j0 + j) of each
// 32-key chunk; the running max / sum follow the online-softmax recurrence;
// lane l accumulates output columns l, l+32, ... (D <= 256).
template <int DT>
__global__ void __launch_bounds__(128) simt_attn_kernel(const void* Qv, const void* Kv,
                                                        const void* Vv, void* Ov, int Sq, int Sk,
                                                        int D, int causal, float scale) {
  using E = Elem<DT>;
  using T = typename E::T;
  __shared__ float qs[4][256];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t bh = blockIdx.y;
  const int qi = blockIdx.x * 4 + warp;
  if (qi >= Sq) return;
  const T* Q = reinterpret_cast<const T*>(Qv) + (bh * Sq + qi) * (int64_t)D;
  const T* Kb = reinterpret_cast<const T*>(Kv) + bh * Sk * (int64_t)D;
  const T* Vb = reinterpret_cast<const T*>(Vv) + bh * Sk * (int64_t)D;
  T* O = reinterpret_cast<T*>(Ov) + (bh * Sq + qi) * (int64_t)D;
  for (int d = lane; d < D; d += 32) qs[warp][d] = E::to_f(Q[d]);
  __syncwarp();
  float acc[8] = {};
  float m = -INFINITY, l = 0.f;
  const int kend = causal ? min(Sk, qi + 1) : Sk;
  for (int j0 = 0; j0 < kend; j0 += 32) {
    const int j = j0 + lane;
    float s = -INFINITY;
    if (j < kend) {
      const T* kr = Kb + (int64_t)j * D;
      float dot = 0.f;
      for (int d = 0; d < D; ++d) dot = fmaf(qs[warp][d], E::to_f(kr[d]), dot);
      s = dot * scale;
    }
    const float cm = warp_max(s);
    const float mn = fmaxf(m, cm);
    const float alpha = (m == -INFINITY) ? 0.f : __expf(m - mn);
    const float p = (s == -INFINITY) ? 0.f : __expf(s - mn);
    l = l * alpha + warp_sum(p);
#pragma unroll
    for (int t = 0; t < 8; ++t) acc[t] *= alpha;
    const int nj = min(32, kend - j0);
    for (int jj = 0; jj < nj; ++jj) {
      const float pj = __shfl_sync(0xffffffffu, p, jj);
      const T* vr = Vb + (int64_t)(j0 + jj) * D;
#pragma unroll
      for (int t = 0; t < 8; ++t) {
        const int d = lane + 32 * t;
        if (d < D) acc[t] = fmaf(pj, E::to_f(vr[d]), acc[t]);
      }
    }
    m = mn;
  }
  const float inv = 1.f / l;
#pragma unroll
  for (int t = 0; t < 8; ++t) {
    const int d = lane + 32 * t;
    if (d < D) O[d] = E::from_f(acc[t] * inv);
  }
}

template <int DT>
int simt_gemm(const void* A, const void* B, const void* B2, void* C, int M, int N, int K,
              int64_t lda, int64_t ldb, int64_t ldc, int b_kmajor, int act, const void* R,
              int64_t ldr, cudaStream_t s) {
  dim3 grid((N + SB_N - 1) / SB_N, (M + SB_M - 1) / SB_M);
  AK_REQUIRE(grid.y <= 65535u, AK_ERR_SHAPE, "M too large for the SIMT path");
  if (B2) simt_gemm_kernel<DT, true><<<grid, 256, 0, s>>>(A, B, B2, C, M, N, K, lda, ldb, ldc, b_kmajor, act, R, ldr);
  else simt_gemm_kernel<DT, false><<<grid, 256, 0, s>>>(A, B, B2, C, M, N, K, lda, ldb, ldc, b_kmajor, act, R, ldr);
  return launch_status("simt_gemm");
}

int simt_gemm_any(int dtype, const void* A, const void* B, const void* B2, void* C, int M, int N,
                  int K, int64_t lda, int64_t ldb, int64_t ldc, int b_kmajor, int act,
                  const void* R, int64_t ldr, cudaStream_t s) {
  switch (dtype) {
    case AK_F32: return simt_gemm<AK_F32>(A, B, B2, C, M, N, K, lda, ldb, ldc, b_kmajor, act, R, ldr, s);
    case AK_F16: return simt_gemm<AK_F16>(A, B, B2, C, M, N, K, lda, ldb, ldc, b_kmajor, act, R, ldr, s);
    case AK_BF16: return simt_gemm<AK_BF16>(A, B, B2, C, M, N, K, lda, ldb, ldc, b_kmajor, act, R, ldr, s);
  }
  set_error("unsupported dtype %d", dtype);
  return AK_ERR_DTYPE;
}

int simt_attention_any(int dtype, const void* Q, const void* K, const void* V, void* O,
                       int64_t bh, int Sq, int Sk, int D, int causal, float scale,
                       cudaStream_t s) {
  AK_REQUIRE(D <= 256, AK_ERR_SHAPE, "head_dim %d > 256 unsupported", D);
  AK_REQUIRE(bh <= 65535, AK_ERR_SHAPE, "batch*heads %lld > 65535 on the SIMT path",
             (long long)bh);
  dim3 grid((Sq + 3) / 4, (unsigned)bh);
  switch (dtype) {
    case AK_F32: simt_attn_kernel<AK_F32><<<grid, 128, 0, s>>>(Q, K, V, O, Sq, Sk, D, causal, scale); break;
    case AK_F16: simt_attn_kernel<AK_F16><<<grid, 128, 0, s>>>(Q, K, V, O, Sq, Sk, D, causal, scale); break;
    case AK_BF16: simt_attn_kernel<AK_BF16><<<grid, 128, 0, s>>>(Q, K, V, O, Sq, Sk, D, causal, scale); break;
    default: set_error("unsupported dtype %d", dtype); return AK_ERR_DTYPE;
  }
  return launch_status("simt_attention");
}

}  // namespace ak
