// Gate activations of the fused MLP (reference.py:49-54):
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
  return g / (1.f + __expf(-g));
}

}  // namespace ak
