// Row-wise normalisation kernels: RMSNorm, LayerNorm and softmax over the
// last dimension of a [rows, cols] view.
//
// Math follows the reference oracle:
//   rmsnorm   y = (x / sqrt(mean(x^2) + eps)) * w          reference.py:26-29
//   layernorm y = (x - mean) * rsqrt(var + eps) * w + b    reference.py:20-23 (F.layer_norm)
//   softmax   y = exp(x - max) / sum(exp(x - max))         reference.py:15-17
// all accumulated in fp32 with fixed-order (deterministic) reductions.  The
// per-element divisions are applied as one reciprocal per row times a multiply
// (at most one extra fp32 rounding, far below every output tolerance), which
// keeps the ALU work under the HBM time.
//
// Fast path: the whole row lives in registers as raw 128-bit vectors, so x is
// read from HBM exactly once and y written once (the algorithmic 2*rows*cols
// bytes).  A warp owns a row when the row is short, a CTA otherwise.  The
// looping fallback handles unaligned rows (odd widths such as 4097 or 50257,
// whose rows do not start on 16-byte boundaries) and rows wider than the
// register budget; it re-reads the row from L2.
#include "ak_common.cuh"
#include "rowring.cuh"

namespace ak {

enum RowOp { OP_RMS = 0, OP_LN = 1, OP_SOFTMAX = 2 };

struct RowArgs {
  const void* x;
  const void* w;
  const void* b;
  void* y;
  int64_t rows, cols, ldx, ldy;
  float eps;
};

template <int DT, int OP, int VPT, bool WARP_ROW>
__global__ void __launch_bounds__(1024) row_reg_kernel(RowArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VEC = E::kVec;
  __shared__ float red[32];

  const int G = WARP_ROW ? 32 : blockDim.x;
  const int t = WARP_ROW ? (threadIdx.x & 31) : threadIdx.x;
  const int64_t row = WARP_ROW ? (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)
                               : (int64_t)blockIdx.x;
  if (WARP_ROW && row >= a.rows) return;  // whole warp exits together

  const int64_t nv = a.cols / VEC;
  const T* xr = reinterpret_cast<const T*>(a.x) + row * a.ldx;
  T* yr = reinterpret_cast<T*>(a.y) + row * a.ldy;

  uint4 raw[VPT];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    int64_t v = t + (int64_t)i * G;
    if (v < nv) raw[i] = __ldcs(reinterpret_cast<const uint4*>(xr) + v);
    else raw[i] = make_uint4(0, 0, 0, 0);
  }
  auto elems = [&](int i, float* f) {
    const T* e = reinterpret_cast<const T*>(&raw[i]);
#pragma unroll
    for (int j = 0; j < VEC; ++j) f[j] = E::to_f(e[j]);
  };
  auto rsum = [&](float v) { return WARP_ROW ? warp_sum(v) : block_sum(v, red); };
  auto rmax = [&](float v) { return WARP_ROW ? warp_max(v) : block_max(v, red); };
  const float n = (float)a.cols;

  float s0 = 0.f, s1 = 0.f;  // row statistics
  float ex[OP == OP_SOFTMAX ? VPT : 1][OP == OP_SOFTMAX ? VEC : 1];
  if (OP == OP_RMS) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[VEC];
      elems(i, f);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc = fmaf(f[j], f[j], acc);
    }
    acc = rsum(acc);
    s0 = 1.0f / sqrtf(acc / n + a.eps);  // 1 / rms
  } else if (OP == OP_LN) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[VEC];
      elems(i, f);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc += f[j];
    }
    const float mean = rsum(acc) / n;
    float var = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (t + (int64_t)i * G < nv) {
        float f[VEC];
        elems(i, f);
#pragma unroll
        for (int j = 0; j < VEC; ++j) {
          float d = f[j] - mean;
          var = fmaf(d, d, var);
        }
      }
    }
    var = rsum(var) / n;
    s0 = mean;
    s1 = rsqrtf(var + a.eps);
  } else {  // softmax: exp(x - max) is computed once and kept in registers
    float m = -INFINITY;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if (t + (int64_t)i * G < nv) {
        float f[VEC];
        elems(i, f);
#pragma unroll
        for (int j = 0; j < VEC; ++j) m = fmaxf(m, f[j]);
      }
    }
    m = rmax(m);
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      float f[VEC];
      elems(i, f);
      const bool ok = t + (int64_t)i * G < nv;
#pragma unroll
      for (int j = 0; j < VEC; ++j) {
        ex[i][j] = ok ? __expf(f[j] - m) : 0.f;
        acc += ex[i][j];
      }
    }
    s0 = m;
    s1 = 1.0f / rsum(acc);
  }
  const T* w = reinterpret_cast<const T*>(a.w);
  const T* b = reinterpret_cast<const T*>(a.b);
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    int64_t v = t + (int64_t)i * G;
    if (v >= nv) continue;
    float f[VEC], o[VEC];
    if (OP != OP_SOFTMAX) elems(i, f);
    if (OP == OP_RMS) {
      float wf[VEC];
      load_vec<DT>(w + v * VEC, wf);
#pragma unroll
      for (int j = 0; j < VEC; ++j) o[j] = (f[j] * s0) * wf[j];
    } else if (OP == OP_LN) {
      float wf[VEC], bf[VEC];
      load_vec<DT>(w + v * VEC, wf);
      load_vec<DT>(b + v * VEC, bf);
#pragma unroll
      for (int j = 0; j < VEC; ++j) o[j] = fmaf((f[j] - s0) * s1, wf[j], bf[j]);
    } else {
#pragma unroll
      for (int j = 0; j < VEC; ++j) o[j] = ex[i][j] * s1;
    }
    store_vec<DT>(yr + v * VEC, o);
  }
}

// Looping fallback: one CTA per row, scalar coalesced accesses, any width
// and any alignment.  Re-reads the row (from L2) once per pass.
template <int DT, int OP>
__global__ void __launch_bounds__(512) row_loop_kernel(RowArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = reinterpret_cast<const T*>(a.x) + row * a.ldx;
  T* yr = reinterpret_cast<T*>(a.y) + row * a.ldy;
  const T* w = reinterpret_cast<const T*>(a.w);
  const T* b = reinterpret_cast<const T*>(a.b);
  const float n = (float)a.cols;

  if (OP == OP_RMS) {
    float acc = 0.f;
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x) {
      float f = E::to_f(xr[c]);
      acc = fmaf(f, f, acc);
    }
    const float inv = 1.0f / sqrtf(block_sum(acc, red) / n + a.eps);
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x)
      yr[c] = E::from_f((E::to_f(xr[c]) * inv) * E::to_f(w[c]));
  } else if (OP == OP_LN) {
    float acc = 0.f;
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x) acc += E::to_f(xr[c]);
    const float mean = block_sum(acc, red) / n;
    float var = 0.f;
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x) {
      float d = E::to_f(xr[c]) - mean;
      var = fmaf(d, d, var);
    }
    const float rstd = rsqrtf(block_sum(var, red) / n + a.eps);
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x)
      yr[c] = E::from_f(fmaf((E::to_f(xr[c]) - mean) * rstd, E::to_f(w[c]), E::to_f(b[c])));
  } else {
    float m = -INFINITY, s = 0.f;
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x) {
      float f = E::to_f(xr[c]);
      if (f > m) {
        s = (m == -INFINITY) ? 0.f : s * __expf(m - f);
        m = f;
      }
      s += __expf(f - m);
    }
    // merge per-thread (m, s) pairs: max first, then rescaled sums
    const float gm = block_max(m, red);
    const float inv = 1.0f / block_sum(m == -INFINITY ? 0.f : s * __expf(m - gm), red);
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x)
      yr[c] = E::from_f(__expf(E::to_f(xr[c]) - gm) * inv);
  }
}

template <int DT, int OP, int VPT>
static void launch_reg(const RowArgs& a, int G, cudaStream_t s) {
  if (G == 32) {
    const int threads = 256;  // 8 rows per CTA
    const int64_t blocks = (a.rows + 7) / 8;
    row_reg_kernel<DT, OP, VPT, true><<<(unsigned)blocks, threads, 0, s>>>(a);
  } else {
    row_reg_kernel<DT, OP, VPT, false><<<(unsigned)a.rows, G, 0, s>>>(a);
  }
}

template <int DT, int OP>
static int run_rowop(const RowArgs& a, cudaStream_t s) {
  constexpr int VEC = Elem<DT>::kVec;
  if (OP == OP_SOFTMAX) {
    // long aligned rows: persistent TMA-staged ring (rowring.cu)
    RingArgs ra{};
    ra.x = a.x; ra.y = a.y;
    ra.rows = a.rows; ra.cols = a.cols; ra.ldx = a.ldx; ra.ldy = a.ldy;
    const int rc = ring_rowop(RING_SOFTMAX, DT, ra, s);
    if (rc != 1) return rc;
  }
  const bool vec_ok = (a.cols % VEC == 0) && (a.ldx % VEC == 0) && (a.ldy % VEC == 0) &&
                      aligned16(a.x) && aligned16(a.y) &&
                      (OP == OP_SOFTMAX || aligned16(a.w)) && (OP != OP_LN || aligned16(a.b));
  const int64_t nv = a.cols / VEC;
  if (vec_ok && nv <= 1024 * 8) {
    // Aim for 4 vectors per thread (enough loads in flight per thread),
    // then round the per-thread count up to a supported template value.
    int64_t g = 32;
    while (g < 1024 && g * 4 < nv) g <<= 1;
    int64_t vpt = (nv + g - 1) / g;
    int V = vpt <= 1 ? 1 : vpt <= 2 ? 2 : vpt <= 4 ? 4 : 8;
    switch (V) {
      case 1: launch_reg<DT, OP, 1>(a, (int)g, s); break;
      case 2: launch_reg<DT, OP, 2>(a, (int)g, s); break;
      case 4: launch_reg<DT, OP, 4>(a, (int)g, s); break;
      default: launch_reg<DT, OP, 8>(a, (int)g, s); break;
    }
  } else {
    int threads = a.cols >= 4096 ? 512 : a.cols >= 1024 ? 256 : 128;
    row_loop_kernel<DT, OP><<<(unsigned)a.rows, threads, 0, s>>>(a);
  }
  return launch_status("rowop");
}

template <int OP>
static int dispatch_rowop(const RowArgs& a, int dtype, cudaStream_t s) {
  switch (dtype) {
    case AK_F32: return run_rowop<AK_F32, OP>(a, s);
    case AK_F16: return run_rowop<AK_F16, OP>(a, s);
    case AK_BF16: return run_rowop<AK_BF16, OP>(a, s);
  }
  set_error("unsupported dtype %d", dtype);
  return AK_ERR_DTYPE;
}

static int check_rows(const void* x, const void* y, int64_t rows, int64_t cols, int64_t ldx,
                      int64_t ldy, int dtype) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(rows >= 0 && cols >= 0, AK_ERR_SHAPE, "negative shape rows=%lld cols=%lld",
             (long long)rows, (long long)cols);
  AK_REQUIRE(rows <= 0x7fffffffLL, AK_ERR_SHAPE, "rows=%lld exceeds 2^31-1", (long long)rows);
  AK_REQUIRE(ldx >= cols && ldy >= cols, AK_ERR_SHAPE, "row stride smaller than cols");
  AK_REQUIRE(rows == 0 || cols == 0 || (x && y), AK_ERR_ARG, "null tensor pointer");
  return AK_OK;
}

}  // namespace ak

using namespace ak;

extern "C" int ak_rmsnorm(const void* x, const void* w, void* y, int64_t rows, int64_t cols,
                          int64_t ldx, int64_t ldy, float eps, int dtype, void* stream) {
  int rc = check_rows(x, y, rows, cols, ldx, ldy, dtype);
  if (rc) return rc;
  if (rows == 0 || cols == 0) return AK_OK;
  AK_REQUIRE(w, AK_ERR_ARG, "rmsnorm: null weight");
  RowArgs a{x, w, nullptr, y, rows, cols, ldx, ldy, eps};
  return dispatch_rowop<OP_RMS>(a, dtype, (cudaStream_t)stream);
}

extern "C" int ak_layernorm(const void* x, const void* w, const void* b, void* y, int64_t rows,
                            int64_t cols, int64_t ldx, int64_t ldy, float eps, int dtype,
                            void* stream) {
  int rc = check_rows(x, y, rows, cols, ldx, ldy, dtype);
  if (rc) return rc;
  if (rows == 0 || cols == 0) return AK_OK;
  AK_REQUIRE(w && b, AK_ERR_ARG, "layernorm: null weight/bias");
  RowArgs a{x, w, b, y, rows, cols, ldx, ldy, eps};
  return dispatch_rowop<OP_LN>(a, dtype, (cudaStream_t)stream);
}

extern "C" int ak_softmax(const void* x, void* y, int64_t rows, int64_t cols, int64_t ldx,
                          int64_t ldy, int dtype, void* stream) {
  int rc = check_rows(x, y, rows, cols, ldx, ldy, dtype);
  if (rc) return rc;
  if (rows == 0 || cols == 0) return AK_OK;
  RowArgs a{x, nullptr, nullptr, y, rows, cols, ldx, ldy, 0.f};
  return dispatch_rowop<OP_SOFTMAX>(a, dtype, (cudaStream_t)stream);
}
