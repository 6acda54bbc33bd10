// Shape / layout of one attention call, shared by the C ABI and the kernels.
#pragma once
#include "ak_common.cuh"

namespace ak {

struct AttnShape {
  const void* Q;
  const void* K;
  const void* V;
  void* O;
  int64_t B, H, Hkv;  // batch, query heads, key/value heads (H % Hkv == 0)
  int Sq, Sk, D;
  int64_t qs[3], ks[3], vs[3], os[3];  // strides in elements: batch, head, sequence
  int causal;
  float scale;
  int dtype;
};

bool tc_attention_ok(const AttnShape& a);
int tc_attention(const AttnShape& a, cudaStream_t s);

}  // namespace ak
