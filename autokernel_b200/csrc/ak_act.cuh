// Gate activations of the fused MLP (reference.py:49-54), computed in fp32 as ATen computes
// them for 16-bit tensors:
//   AK_ACT_SILU  silu(g) = g / (1 + exp(-g))
//   AK_ACT_GELU  exact gelu(g) = 0.5 g (1 + erf(g / sqrt(2)))
//   AK_ACT_RELU2 relu(g)^2
#pragma once
#include "ak_common.cuh"

namespace ak {

AK_D float apply_act(int act, float g) {
  if (act == AK_ACT_GELU) return 0.5f * g * (1.f + erff(g * 0.70710678118654752f));
  if (act == AK_ACT_RELU2) {
    const float r = fmaxf(g, 0.f);
    return r * r;
  }
  return g / (1.f + expf(-g));
}

// One element of the SwiGLU hidden act(g) * u with reference.py's rounding (reference.py:45-55
// in a 16-bit dtype): the gate and up projections are stored in the dtype, the activation is
// computed from the stored gate and stored, and the product is rounded at the final store.
// For fp32 every rounding is the identity.
template <int DT>
AK_D float swiglu_ref(int act, float g, float u) {
  float gr = g, ur = u;
  rnd2<DT>(gr, ur);
  float a = apply_act(act, gr), unused = 0.f;
  rnd2<DT>(a, unused);
  return a * ur;
}

}  // namespace ak
