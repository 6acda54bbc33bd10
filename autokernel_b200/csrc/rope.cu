// Rotary position embedding on interleaved pairs (reference.py:63-69):
//   y[..., 2i]   = x[2i] * cos[i] - x[2i+1] * sin[i]
//   y[..., 2i+1] = x[2i] * sin[i] + x[2i+1] * cos[i]
// x and y are contiguous [rows, D]; cos and sin are contiguous [cs_rows, D/2]
// and row r of x uses cos/sin row (r / cs_div) % cs_rows.  That covers the
// broadcasts the callers use: bench-style x [B,H,S,D] with cos [S,D/2]
// (cs_div = 1, cs_rows = S) and model-style x [B,S,H,D] with cos [S,1,D/2]
// (cs_div = H).  cos/sin may be the dtype of x or fp32.
//
// Each thread handles 16-byte vectors of x (4 pairs in 16-bit types, 2 in
// fp32) and the matching cos/sin pieces, four vectors in flight at a time, so x
// is read once and y written once with 128-bit accesses; cos/sin (1 MB at
// S=4096) stay in L2.
//
// Rounding: when cos/sin have x's dtype (the kernel_fn / reference.py case) the arithmetic is
// reference.py's operator sequence -- each product x * cos, x * sin rounded to the dtype, then
// the difference / sum rounded -- so the output is bit-identical to reference.py (the products
// of two 16-bit values are exact in fp32, and ATen rounds each one to the dtype).  With fp32
// tables (the model path, models/llama_7b.py:40-48, which rotates in fp32) it is fp32
// arithmetic with a single rounding at the store.
#include "ak_common.cuh"

#include <type_traits>

namespace ak {

struct RopeArgs {
  const void* x;
  const void* cos;
  const void* sin;
  void* y;
  int64_t rows, d, cs_div, cs_rows;
  FastDiv f_vpr, f_div, f_rows;  // 32-bit index path (total vectors < 2^31)
};

template <int CDT, int N>
AK_D void load_cs(const typename Elem<CDT>::T* p, float* out) {
  // N consecutive elements, N * sizeof(T) bytes (8 or 16): aligned by caller.
  if constexpr (sizeof(typename Elem<CDT>::T) * N == 8) {
    uint2 r = __ldg(reinterpret_cast<const uint2*>(p));
    const typename Elem<CDT>::T* e = reinterpret_cast<const typename Elem<CDT>::T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = Elem<CDT>::to_f(e[i]);
  } else {
    uint4 r = __ldg(reinterpret_cast<const uint4*>(p));
    const typename Elem<CDT>::T* e = reinterpret_cast<const typename Elem<CDT>::T*>(&r);
#pragma unroll
    for (int i = 0; i < N; ++i) out[i] = Elem<CDT>::to_f(e[i]);
  }
}

// cos/sin pieces kept as the raw loaded words until the arithmetic (half the registers of
// the widened floats for 16-bit tables), so more vectors stay in flight per SM.
template <int CDT, int N>
struct CsRaw {
  using T = typename Elem<CDT>::T;
  using W = typename std::conditional<sizeof(T) * N == 8, uint2, uint4>::type;
  W w;
  AK_D void load(const T* p) { w = __ldg(reinterpret_cast<const W*>(p)); }
  AK_D float at(int i) const { return Elem<CDT>::to_f(reinterpret_cast<const T*>(&w)[i]); }
};

// One rotated pair.  REF: reference.py's rounding (products rounded to the dtype, no fma
// contraction); otherwise fp32 fmas.
template <int DT, bool REF>
AK_D void rope_pair(float x1, float x2, float c, float s, float& o1, float& o2) {
  if constexpr (REF) {
    float a = __fmul_rn(x1, c), b = __fmul_rn(x2, s), e = __fmul_rn(x1, s), f = __fmul_rn(x2, c);
    rnd2<DT>(a, b);
    rnd2<DT>(e, f);
    o1 = __fsub_rn(a, b);
    o2 = __fadd_rn(e, f);
  } else {
    o1 = fmaf(x1, c, -x2 * s);
    o2 = fmaf(x1, s, x2 * c);
  }
}

template <int DT, int CDT>
__global__ void __launch_bounds__(256) rope_vec_kernel(RopeArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  using CT = typename Elem<CDT>::T;
  constexpr int VEC = E::kVec;
  constexpr int P = VEC / 2;  // pairs per vector
  constexpr int U = 4;        // vectors in flight per thread
  const int64_t vpr = a.d / VEC;  // vectors per row
  const int64_t total = a.rows * vpr;
  const int64_t half = a.d / 2;
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  for (int64_t g0 = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g0 < total; g0 += U * stride) {
    uint4 xr[U];
    float c[U][P], s[U][P];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = g0 + u * stride;
      if (g < total) xr[u] = __ldcs(reinterpret_cast<const uint4*>(a.x) + g);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = g0 + u * stride;
      if (g < total) {
        const int64_t row = g / vpr;
        const int64_t v = g - row * vpr;
        const int64_t coff = ((row / a.cs_div) % a.cs_rows) * half + v * P;
        load_cs<CDT, P>(reinterpret_cast<const CT*>(a.cos) + coff, c[u]);
        load_cs<CDT, P>(reinterpret_cast<const CT*>(a.sin) + coff, s[u]);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t g = g0 + u * stride;
      if (g >= total) continue;
      const T* e = reinterpret_cast<const T*>(&xr[u]);
      float o[VEC];
#pragma unroll
      for (int q = 0; q < P; ++q) {
        const float x1 = E::to_f(e[2 * q]), x2 = E::to_f(e[2 * q + 1]);
        rope_pair<DT, CDT == DT>(x1, x2, c[u][q], s[u][q], o[2 * q], o[2 * q + 1]);
      }
      store_vec<DT>(reinterpret_cast<T*>(a.y) + g * VEC, o);
    }
  }
}

// Same as rope_vec_kernel with 32-bit indices and multiply-high divisions:
// the 64-bit divisions above cost more issue slots than the memory traffic
// leaves.  Used when rows * D / VEC < 2^31.
template <int DT, int CDT>
__global__ void __launch_bounds__(256) rope_vec32_kernel(RopeArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  using CT = typename Elem<CDT>::T;
  constexpr int VEC = E::kVec;
  constexpr int P = VEC / 2;
  constexpr int U = 4;
  const uint32_t total = (uint32_t)(a.rows * (a.d / VEC));
  const uint32_t half = (uint32_t)(a.d / 2);
  const uint32_t stride = gridDim.x * blockDim.x;
  for (uint32_t g0 = blockIdx.x * blockDim.x + threadIdx.x; g0 < total; g0 += U * stride) {
    uint4 xr[U];
    CsRaw<CDT, P> c[U], s[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t g = g0 + u * stride;
      if (g < total) xr[u] = __ldcs(reinterpret_cast<const uint4*>(a.x) + g);
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t g = g0 + u * stride;
      if (g < total) {
        const uint32_t row = a.f_vpr.div(g);
        const uint32_t v = g - row * a.f_vpr.d;
        const uint32_t coff = a.f_rows.mod(a.f_div.div(row)) * half + v * P;
        c[u].load(reinterpret_cast<const CT*>(a.cos) + coff);
        s[u].load(reinterpret_cast<const CT*>(a.sin) + coff);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const uint32_t g = g0 + u * stride;
      if (g >= total) continue;
      const T* e = reinterpret_cast<const T*>(&xr[u]);
      float o[VEC];
#pragma unroll
      for (int q = 0; q < P; ++q) {
        const float x1 = E::to_f(e[2 * q]), x2 = E::to_f(e[2 * q + 1]);
        rope_pair<DT, CDT == DT>(x1, x2, c[u].at(q), s[u].at(q), o[2 * q], o[2 * q + 1]);
      }
      store_vec<DT>(reinterpret_cast<T*>(a.y) + (size_t)g * VEC, o);
    }
  }
}

// Scalar fallback: one thread per pair, any head_dim / alignment.
template <int DT, int CDT>
__global__ void __launch_bounds__(256) rope_scalar_kernel(RopeArgs a) {
  using E = Elem<DT>;
  using T = typename E::T;
  using CE = Elem<CDT>;
  using CT = typename CE::T;
  const int64_t half = a.d / 2;
  const int64_t total = a.rows * half;
  const T* x = reinterpret_cast<const T*>(a.x);
  T* y = reinterpret_cast<T*>(a.y);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < total;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = g / half;
    const int64_t p = g - row * half;
    const int64_t crow = (row / a.cs_div) % a.cs_rows;
    const float c = CE::to_f(reinterpret_cast<const CT*>(a.cos)[crow * half + p]);
    const float s = CE::to_f(reinterpret_cast<const CT*>(a.sin)[crow * half + p]);
    const float x1 = E::to_f(x[row * a.d + 2 * p]), x2 = E::to_f(x[row * a.d + 2 * p + 1]);
    float o1, o2;
    rope_pair<DT, CDT == DT>(x1, x2, c, s, o1, o2);
    y[row * a.d + 2 * p] = E::from_f(o1);
    y[row * a.d + 2 * p + 1] = E::from_f(o2);
  }
}

template <int DT, int CDT>
static int run_rope(const RopeArgs& a, cudaStream_t st) {
  constexpr int VEC = Elem<DT>::kVec;
  const int sms = device_info().sm_count;
  const bool vec = (a.d % VEC == 0) && aligned16(a.x) && aligned16(a.y) &&
                   ((reinterpret_cast<uintptr_t>(a.cos) | reinterpret_cast<uintptr_t>(a.sin)) % 16 == 0);
  const int64_t units = vec ? a.rows * (a.d / VEC) : a.rows * (a.d / 2);
  int64_t blocks = (units + 255) / 256;
  const int64_t cap = (int64_t)sms * 16;  // grid-stride beyond 16 CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  const bool small = units < (1LL << 31) && a.rows < (1LL << 31) && a.cs_div < (1LL << 31) &&
                     a.cs_rows < (1LL << 31);
  if (vec && small) {
    RopeArgs b = a;
    b.f_vpr = FastDiv((uint32_t)(a.d / VEC));
    b.f_div = FastDiv((uint32_t)a.cs_div);
    b.f_rows = FastDiv((uint32_t)a.cs_rows);
    rope_vec32_kernel<DT, CDT><<<(unsigned)blocks, 256, 0, st>>>(b);
  } else if (vec) rope_vec_kernel<DT, CDT><<<(unsigned)blocks, 256, 0, st>>>(a);
  else rope_scalar_kernel<DT, CDT><<<(unsigned)blocks, 256, 0, st>>>(a);
  return launch_status("rotary_embedding");
}

}  // namespace ak

using namespace ak;

extern "C" int ak_rotary_embedding(const void* x, const void* cos, const void* sin, void* y,
                                   int64_t rows, int64_t head_dim, int64_t cs_div,
                                   int64_t cs_rows, int dtype, int cs_dtype, void* stream) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(cs_dtype == dtype || cs_dtype == AK_F32, AK_ERR_DTYPE,
             "cos/sin dtype must equal x dtype or be fp32");
  AK_REQUIRE(head_dim % 2 == 0 && head_dim > 0, AK_ERR_SHAPE, "head_dim must be even, got %lld",
             (long long)head_dim);
  AK_REQUIRE(rows >= 0 && cs_div >= 1 && cs_rows >= 1, AK_ERR_SHAPE, "bad rope broadcast");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(x && y && cos && sin, AK_ERR_ARG, "null tensor pointer");
  RopeArgs a{x, cos, sin, y, rows, head_dim, cs_div, cs_rows, FastDiv(), FastDiv(), FastDiv()};
  cudaStream_t st = (cudaStream_t)stream;
  if (cs_dtype == AK_F32) {
    switch (dtype) {
      case AK_F32: return run_rope<AK_F32, AK_F32>(a, st);
      case AK_F16: return run_rope<AK_F16, AK_F32>(a, st);
      case AK_BF16: return run_rope<AK_BF16, AK_F32>(a, st);
    }
  }
  switch (dtype) {
    case AK_F16: return run_rope<AK_F16, AK_F16>(a, st);
    case AK_BF16: return run_rope<AK_BF16, AK_BF16>(a, st);
  }
  return AK_ERR_DTYPE;
}
