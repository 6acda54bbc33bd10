// Shared device/host helpers for the autokernel_b200 CUDA library (sm_100a).
//
// Every kernel in this library reads/writes fp32, fp16 or bf16 tensors and
// accumulates in fp32 (fp64 for cross-CTA partial sums).  This header holds
// the dtype plumbing, 128-bit vector access, the warp/CTA reductions, the
// thread-local error string behind ak_last_error() and the device status word
// that bounded spin-waits write instead of trapping.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <mutex>
#include <string>

#include "../../include/ak_b200.h"

#define AK_HD __host__ __device__ __forceinline__
#define AK_D __device__ __forceinline__

namespace ak {

// ---------------------------------------------------------------- errors
void set_error(const char* fmt, ...);
int launch_status(const char* what);  // checks cudaGetLastError after a launch

#define AK_REQUIRE(cond, code, ...)            \
  do {                                          \
    if (!(cond)) {                              \
      ::ak::set_error(__VA_ARGS__);             \
      return (code);                            \
    }                                           \
  } while (0)

// Device status word.  Bounded waits set a non-zero code here and return
// instead of trapping, so the context stays usable; ak_device_status() reads
// and clears it.
extern __device__ int g_status;  // defined in abi.cu

AK_D void report_status(int code) { atomicCAS(&g_status, 0, code); }

// ---------------------------------------------------------------- dtypes
template <int DT> struct Elem;
template <> struct Elem<AK_F32> {
  using T = float;
  static constexpr int kVec = 4;  // elements per 16-byte vector
  static AK_D float to_f(T v) { return v; }
  static AK_D T from_f(float v) { return v; }
};
template <> struct Elem<AK_F16> {
  using T = __half;
  static constexpr int kVec = 8;
  static AK_D float to_f(T v) { return __half2float(v); }
  static AK_D T from_f(float v) { return __float2half_rn(v); }
};
template <> struct Elem<AK_BF16> {
  using T = __nv_bfloat16;
  static constexpr int kVec = 8;
  static AK_D float to_f(T v) { return __bfloat162float(v); }
  static AK_D T from_f(float v) { return __float2bfloat16_rn(v); }
};

// Round two fp32 values to the storage dtype and back with one packed conversion.
template <int DT>
AK_D void rnd2(float& a, float& b) {
  if constexpr (DT == AK_F16) {
    const float2 r = __half22float2(__floats2half2_rn(a, b));
    a = r.x;
    b = r.y;
  } else if constexpr (DT == AK_BF16) {
    const float2 r = __bfloat1622float2(__floats2bfloat162_rn(a, b));
    a = r.x;
    b = r.y;
  }
}

inline int dtype_size(int dt) { return dt == AK_F32 ? 4 : 2; }
inline bool dtype_ok(int dt) { return dt == AK_F32 || dt == AK_F16 || dt == AK_BF16; }

// Load/store a 16-byte vector of kVec elements as fp32.
template <int DT>
AK_D void load_vec(const typename Elem<DT>::T* p, float* out) {
  uint4 raw = __ldg(reinterpret_cast<const uint4*>(p));
  const typename Elem<DT>::T* e = reinterpret_cast<const typename Elem<DT>::T*>(&raw);
#pragma unroll
  for (int i = 0; i < Elem<DT>::kVec; ++i) out[i] = Elem<DT>::to_f(e[i]);
}
// Streaming load (evict-first): for data read exactly once.
template <int DT>
AK_D void load_vec_stream(const typename Elem<DT>::T* p, float* out) {
  uint4 raw = __ldcs(reinterpret_cast<const uint4*>(p));
  const typename Elem<DT>::T* e = reinterpret_cast<const typename Elem<DT>::T*>(&raw);
#pragma unroll
  for (int i = 0; i < Elem<DT>::kVec; ++i) out[i] = Elem<DT>::to_f(e[i]);
}
template <int DT>
AK_D void store_vec(typename Elem<DT>::T* p, const float* in) {
  uint4 raw;
  typename Elem<DT>::T* e = reinterpret_cast<typename Elem<DT>::T*>(&raw);
#pragma unroll
  for (int i = 0; i < Elem<DT>::kVec; ++i) e[i] = Elem<DT>::from_f(in[i]);
  __stcs(reinterpret_cast<uint4*>(p), raw);
}

// ---------------------------------------------------------------- reductions
AK_D float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
AK_D float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
AK_D double warp_sum_d(double v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Sum over all threads of the CTA in a fixed order (deterministic).  `red`
// must hold 32 floats; the result is broadcast to every thread.
AK_D float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  __syncthreads();  // protect `red` from a previous use
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : 0.f;
  return warp_sum(t);
}
AK_D float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}
AK_D double block_sum_d(double v, double* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum_d(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  double t = lane < nw ? red[lane] : 0.0;
  return warp_sum_d(t);
}

// Online-softmax merge of (max, sum-of-exp) pairs.
AK_D void lse_merge(float& m, float& s, float m2, float s2) {
  float mn = fmaxf(m, m2);
  if (mn == -INFINITY) { m = mn; s = 0.f; return; }
  s = s * __expf(m - mn) + s2 * __expf(m2 - mn);
  m = mn;
}

AK_HD bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Division of 32-bit unsigned n by a run-time constant d with a multiply-high
// (Granlund & Montgomery, "Division by invariant integers using
// multiplication", 1994): q = (umulhi(n, m) + n) >> l with l = ceil(log2 d) and
// m = floor(2^32 (2^l - d) / d) + 1.  Exact for n < 2^31 (the sum never
// overflows 32 bits).  Built on the host, used in index arithmetic.
struct FastDiv {
  uint32_t d, m, l;
  FastDiv() : d(1), m(0), l(0) {}
  explicit FastDiv(uint32_t div) : d(div) {
    l = 0;
    while ((1ull << l) < div) ++l;
    m = (uint32_t)(((1ull << 32) * ((1ull << l) - div)) / div + 1);
  }
  AK_D uint32_t div(uint32_t n) const { return (__umulhi(n, m) + n) >> l; }
  AK_D uint32_t mod(uint32_t n) const { return n - div(n) * d; }
};

struct DeviceInfo {
  int sm_count;
  int max_smem_optin;
  int l2_bytes;
  int cc_major, cc_minor;
};
const DeviceInfo& device_info();  // cached per device, thread safe

constexpr int kMaxDevices = 64;
int current_device();  // the calling thread's current device, clamped to [0, kMaxDevices)

// Opt `Kernel` into `bytes` of dynamic shared memory.  The attribute belongs to the
// current device's context, so it is set once per (kernel, device) and the result kept
// per device: a process that launches on cuda:0 and then cuda:1 sets it on both.
template <auto Kernel>
cudaError_t smem_optin(int bytes) {
  static std::once_flag once[kMaxDevices];
  static cudaError_t err[kMaxDevices];
  const int dev = current_device();
  std::call_once(once[dev], [dev, bytes] {
    err[dev] = cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  });
  return err[dev];
}

}  // namespace ak
