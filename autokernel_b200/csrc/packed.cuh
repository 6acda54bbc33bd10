// Packed 16-byte-vector helpers shared by the softmax / cross-entropy kernels.
#pragma once
#include "ak_common.cuh"

namespace ak {

// Packed helpers on one 16-byte vector.  16-bit types take the max on bf16x2 /
// half2 pairs (exact: the max of stored values is one of them) and widen to
// fp32 with bit operations; the exponent is exp2((x - max) * log2e), one
// FADD, one FMUL and one MUFU ex2 per element (x - max is exact near the max,
// so inputs of any magnitude are safe).  Keeps the inner loops near 5
// instructions per element so the CTA stays memory-bound.
template <int DT> struct Packed;
template <> struct Packed<AK_BF16> {
  static AK_D void max4(const uint4& r, __nv_bfloat162& m) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&r);
    m = __hmax2(m, __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3])));
  }
  static AK_D float init_m(__nv_bfloat162 m) { return fmaxf(__low2float(m), __high2float(m)); }
  static AK_D __nv_bfloat162 neg_inf() { return __bfloat162bfloat162(__ushort_as_bfloat16(0xff80)); }
  static AK_D void widen(const uint4& r, float* f) {
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      f[2 * i] = __uint_as_float(w[i] << 16);
      f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  static AK_D uint4 narrow(const float* f) {
    uint4 r;
    uint32_t* w = reinterpret_cast<uint32_t*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      __nv_bfloat162 h = __floats2bfloat162_rn(f[2 * i], f[2 * i + 1]);
      w[i] = *reinterpret_cast<uint32_t*>(&h);
    }
    return r;
  }
};
template <> struct Packed<AK_F16> {
  static AK_D void max4(const uint4& r, __half2& m) {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
    m = __hmax2(m, __hmax2(__hmax2(h[0], h[1]), __hmax2(h[2], h[3])));
  }
  static AK_D float init_m(__half2 m) { return fmaxf(__low2float(m), __high2float(m)); }
  static AK_D __half2 neg_inf() { return __half2half2(__ushort_as_half(0xfc00)); }
  static AK_D void widen(const uint4& r, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 v = __half22float2(h[i]);
      f[2 * i] = v.x;
      f[2 * i + 1] = v.y;
    }
  }
  static AK_D uint4 narrow(const float* f) {
    uint4 r;
    __half2* h = reinterpret_cast<__half2*>(&r);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(f[2 * i], f[2 * i + 1]);
    return r;
  }
};
template <> struct Packed<AK_F32> {
  static AK_D void max4(const uint4& r, float& m) {
    m = fmaxf(fmaxf(m, fmaxf(__uint_as_float(r.x), __uint_as_float(r.y))),
              fmaxf(__uint_as_float(r.z), __uint_as_float(r.w)));
  }
  static AK_D float init_m(float m) { return m; }
  static AK_D float neg_inf() { return -INFINITY; }
  static AK_D void widen(const uint4& r, float* f) {
    f[0] = __uint_as_float(r.x); f[1] = __uint_as_float(r.y);
    f[2] = __uint_as_float(r.z); f[3] = __uint_as_float(r.w);
  }
  static AK_D uint4 narrow(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]), __float_as_uint(f[2]),
                      __float_as_uint(f[3]));
  }
};

constexpr float kLog2e = 1.4426950408889634f;

}  // namespace ak
