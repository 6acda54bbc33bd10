// Row-wise normalisation kernels: RMSNorm, LayerNorm and softmax over the
// last dimension of a [rows, cols] view.
//
// Math follows the reference oracle:
//   rmsnorm   y = (x / sqrt(mean(x^2) + eps)) * w          reference.py:26-29
//   layernorm y = (x - mean) * rsqrt(var + eps) * w + b    reference.py:20-23 (F.layer_norm)
//   softmax   y = exp(x - max) / sum(exp(x - max))         reference.py:15-17
// all accumulated in fp32 with fixed-order (deterministic) reductions.
//
// RMSNorm comes in two roundings.  OP_RMS_REF is reference.py's operator sequence in the
// input dtype: each of x*x, mean, + eps, sqrt, x / rms and * w is computed in fp32 and
// rounded to the input dtype, as ATen's 16-bit elementwise ops do (the sum inside the mean
// accumulates in fp32).  So it gives reference.py's results -- including its fp16 overflow
// of x*x for |x| > 256, which zeroes the row -- up to the order of the fp32 sum.  OP_RMS is
// the fp32 form x * (1 / sqrt(mean(x^2) + eps)) * w with one rounding at the end (the model
// path, where that overflow would be a defect).  For LayerNorm and softmax the reference
// rounds once (ATen computes them in fp32), and so do these kernels; their per-element
// divisions are one reciprocal per row times a multiply (at most one extra fp32 rounding, far
// below every output tolerance), which keeps the ALU work under the HBM time.
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

enum RowOp { OP_RMS = 0, OP_LN = 1, OP_SOFTMAX = 2, OP_RMS_REF = 3 };

// Round an fp32 value to the storage dtype and back (identity for fp32).
template <int DT>
AK_D float rnd(float v) {
  return Elem<DT>::to_f(Elem<DT>::from_f(v));
}

// a / b correctly rounded in fp32, from inv = 1 / b (rounded): q0 = a * inv carries at most
// ~1.5 ulp of error, and one step on the exact remainder a - q0 * b (an fma) brings it to the
// correctly rounded quotient -- the fp32 division ATen performs -- for the finite, normal
// operands a normalisation sees, at 3 FMA-pipe operations instead of a full IEEE division.
// With b = inf (an overflowed rms) or a = +-inf the remainder is NaN and q0 (a * 0 = 0, or
// inf / NaN) is already the IEEE quotient.
AK_D float div_rn(float a, float b, float inv) {
  const float q0 = a * inv;
  const float r = fmaf(-q0, b, a);
  return r == r ? fmaf(r, inv, q0) : q0;
}

// Packed pairs of a 16-bit dtype.  A product of two 16-bit values is exact in fp32, so the
// packed multiply, which rounds once, gives exactly ATen's float(a) * float(b) rounded to the
// dtype: reference.py's x ** 2 and (x / rms) * w without unpacking.
template <int DT> struct Pair16;
template <> struct Pair16<AK_F16> {
  using T2 = __half2;
  static AK_D T2 pack(float a, float b) { return __floats2half2_rn(a, b); }
  static AK_D float2 unpack(T2 v) { return __half22float2(v); }
};
template <> struct Pair16<AK_BF16> {
  using T2 = __nv_bfloat162;
  static AK_D T2 pack(float a, float b) { return __floats2bfloat162_rn(a, b); }
  static AK_D float2 unpack(T2 v) { return __bfloat1622float2(v); }
};

// rms of reference.py:26-29 from the fp32 sum of the rounded squares: mean = sum * (1 / n)
// (ATen's mean multiplies by the fp32 reciprocal of the count), then + eps and sqrt, each
// rounded to the dtype.
template <int DT>
AK_D float rms_ref(float sumsq, int64_t n, float eps) {
  const float mean = rnd<DT>(sumsq * __frcp_rn((float)n));
  return rnd<DT>(__fsqrt_rn(rnd<DT>(mean + eps)));
}

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
  } else if (OP == OP_RMS_REF) {
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      if constexpr (DT == AK_F32) {
        float f[VEC];
        elems(i, f);
#pragma unroll
        for (int j = 0; j < VEC; ++j) acc = fmaf(f[j], f[j], acc);
      } else {
        using P = Pair16<DT>;
        const typename P::T2* x2 = reinterpret_cast<const typename P::T2*>(&raw[i]);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float2 sq = P::unpack(__hmul2(x2[k], x2[k]));  // x*x rounded to the dtype
          acc += sq.x + sq.y;
        }
      }
    }
    acc = rsum(acc);
    s0 = rms_ref<DT>(acc, a.cols, a.eps);  // rms, rounded like reference.py's
    s1 = 1.0f / s0;
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
    } else if (OP == OP_RMS_REF) {
      if constexpr (DT == AK_F32) {
        float wf[VEC];
        load_vec<DT>(w + v * VEC, wf);
#pragma unroll
        for (int j = 0; j < VEC; ++j) o[j] = div_rn(f[j], s0, s1) * wf[j];
      } else {
        // rounded x / rms times w, rounded: one packed multiply per pair, stored as is
        using P = Pair16<DT>;
        const uint4 wraw = __ldg(reinterpret_cast<const uint4*>(w + v * VEC));
        const typename P::T2* w2 = reinterpret_cast<const typename P::T2*>(&wraw);
        uint4 out;
        typename P::T2* y2 = reinterpret_cast<typename P::T2*>(&out);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          y2[k] = __hmul2(P::pack(div_rn(f[2 * k], s0, s1), div_rn(f[2 * k + 1], s0, s1)), w2[k]);
        *reinterpret_cast<uint4*>(yr + v * VEC) = out;
        continue;
      }
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
  } else if (OP == OP_RMS_REF) {
    float acc = 0.f;
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x) {
      float f = E::to_f(xr[c]);
      acc += rnd<DT>(f * f);
    }
    const float rms = rms_ref<DT>(block_sum(acc, red), a.cols, a.eps);
    const float inv = 1.0f / rms;
    for (int64_t c = threadIdx.x; c < a.cols; c += blockDim.x)
      yr[c] = E::from_f(rnd<DT>(div_rn(E::to_f(xr[c]), rms, inv)) * E::to_f(w[c]));
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
  return dispatch_rowop<OP_RMS_REF>(a, dtype, (cudaStream_t)stream);
}

extern "C" int ak_rmsnorm_fp32(const void* x, const void* w, void* y, int64_t rows,
                               int64_t cols, int64_t ldx, int64_t ldy, float eps, int dtype,
                               void* stream) {
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
