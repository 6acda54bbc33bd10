// Tensor-core causal flash attention for sm_100a (placeholder: the tcgen05
// kernel is not built yet, so every call takes the SIMT kernel).
#include "ak_common.cuh"

namespace ak {
bool tc_attention_ok(int, const void*, const void*, const void*, const void*, int) { return false; }
int tc_attention(int, const void*, const void*, const void*, void*, int64_t, int, int, int, int,
                 float, cudaStream_t) {
  set_error("tensor-core attention not built");
  return AK_ERR_UNSUPPORTED;
}
}  // namespace ak
