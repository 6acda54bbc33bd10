// Softmax building blocks of the tcgen05 attention kernels: P = exp2(x) for 32 keys of
// one query row, packed as 16-bit pairs, with part of the exponentials on the FMA pipe.
#pragma once
#include "sm100.cuh"

namespace ak {
namespace attn_sm {

using sm100::ex2_approx;

// exp2 on the FMA pipe for two values: x = j + f with j = rint(x), f in [-1/2, 1/2];
// 2^f from a degree-3 polynomial (fitted here to minimise the relative error on that
// interval, max 7.5e-5), and 2^j added to the exponent field.  Inputs below -125 are
// clamped (the result, < 2^-124, is far below the row sum, which is >= 2^-8).
AK_D float2 ex2_poly2(float2 x) {
  constexpr float kMagic = 12582912.f;  // 1.5 * 2^23: adding it rounds to an integer
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 t = __fadd2_rn(x, make_float2(kMagic, kMagic));
  const float2 j = __fadd2_rn(t, make_float2(-kMagic, -kMagic));
  const float2 f = __ffma2_rn(j, make_float2(-1.f, -1.f), x);
  float2 p = __ffma2_rn(f, make_float2(0.05517164f, 0.05517164f),
                        make_float2(0.24261114f, 0.24261114f));
  p = __ffma2_rn(p, f, make_float2(0.69326097f, 0.69326097f));
  p = __ffma2_rn(p, f, make_float2(0.99992806f, 0.99992806f));
  // unsigned arithmetic: the shift discards t's high bits on purpose (modulo 2^32)
  return make_float2(__uint_as_float(__float_as_uint(p.x) + (__float_as_uint(t.x) << 23)),
                     __uint_as_float(__float_as_uint(p.y) + (__float_as_uint(t.y) << 23)));
}

template <int DT>
AK_D uint32_t pack2(float a, float b) {
  if constexpr (DT == AK_BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

// P for one 32-key chunk (16 packed pairs) into pk; EMU of the 16 pairs use the FMA-pipe
// exponential.  Returns the chunk's sum of the unrounded exponentials.
template <int DT, int EMU>
AK_D float2 p_chunk(const uint32_t* r, float2 sl, float2 nm, uint32_t* pk) {
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const float2 s = make_float2(__uint_as_float(r[2 * i]), __uint_as_float(r[2 * i + 1]));
    const float2 xx = __ffma2_rn(s, sl, nm);
    float2 e;
    if (i >= 16 - EMU) {
      e = ex2_poly2(xx);
    } else {
      e.x = ex2_approx(xx.x);
      e.y = ex2_approx(xx.y);
    }
    if (i & 1)
      acc1 = __fadd2_rn(acc1, e);
    else
      acc0 = __fadd2_rn(acc0, e);
    pk[i] = pack2<DT>(e.x, e.y);
  }
  return __fadd2_rn(acc0, acc1);
}

}  // namespace attn_sm
}  // namespace ak
