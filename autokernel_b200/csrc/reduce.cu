// Sum reductions (reference.py:72-74, x.sum(dim)) and the cross-entropy loss
// (reference.py:58-60, F.cross_entropy with mean reduction).
//
// Full reductions (one scalar out of n elements, the 2^30-element config) run
// as two launches so that no zero-initialised state is needed:
//   1. reduce_partial_kernel: a grid of sm_count*4 CTAs, each summing a
//      contiguous chunk with 128-bit streaming loads and fp32 per-thread
//      accumulators, writes one fp64 partial per CTA into the caller's
//      workspace;
//   2. reduce_final_kernel: one CTA adds those partials in a fixed order and
//      writes the fp64 total (and, if asked, the value cast to the output
//      dtype).
// Both orders are fixed by the launch shape, so results are bitwise
// reproducible run to run.  The fp64 total is what a multi-GPU caller
// all-reduces.
//
// Cross-entropy: one pass per row keeps a running (max, sum exp) pair per
// thread, merges them across the CTA and subtracts the target logit, giving a
// per-row loss; the finalize kernel adds the per-row losses in fixed order in
// fp64 and divides by the number of rows whose target is not ignore_index.
#include "ak_common.cuh"
#include "rowring.cuh"
#include "packed.cuh"
#include "sm100.cuh"

#include <mutex>

namespace ak {

// ------------------------------------------------------------------ full sum
template <int DT>
__global__ void __launch_bounds__(512) reduce_partial_kernel(const void* xv, int64_t n,
                                                             double* partials) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VEC = E::kVec;
  __shared__ double redd[32];
  const T* x = reinterpret_cast<const T*>(xv);
  // contiguous chunk per CTA, in whole vectors
  const int64_t nvec = n / VEC;
  const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = (int64_t)blockIdx.x * per;
  const int64_t v1 = min(nvec, v0 + per);
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  int64_t v = v0 + threadIdx.x;
  // four independent 16-byte loads in flight per thread
  for (; v + 3 * (int64_t)blockDim.x < v1; v += 4 * (int64_t)blockDim.x) {
    uint4 r[4];
#pragma unroll
    for (int u = 0; u < 4; ++u)
      r[u] = __ldcs(reinterpret_cast<const uint4*>(x) + v + u * (int64_t)blockDim.x);
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const T* e = reinterpret_cast<const T*>(&r[u]);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc[u] += E::to_f(e[j]);
    }
  }
  for (; v < v1; v += blockDim.x) {
    float f[VEC];
    load_vec_stream<DT>(x + v * VEC, f);
#pragma unroll
    for (int j = 0; j < VEC; ++j) acc[0] += f[j];
  }
  double t = (double)acc[0] + (double)acc[1] + (double)acc[2] + (double)acc[3];
  // scalar tail (n not a multiple of VEC) goes to the last CTA
  if (blockIdx.x == gridDim.x - 1)
    for (int64_t i = nvec * VEC + threadIdx.x; i < n; i += blockDim.x) t += (double)E::to_f(x[i]);
  t = block_sum_d(t, redd);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

// Unaligned input: scalar loads, same partial layout.
template <int DT>
__global__ void __launch_bounds__(512) reduce_partial_scalar_kernel(const void* xv, int64_t n,
                                                                    double* partials) {
  using E = Elem<DT>;
  using T = typename E::T;
  __shared__ double redd[32];
  const T* x = reinterpret_cast<const T*>(xv);
  const int64_t per = (n + gridDim.x - 1) / gridDim.x;
  const int64_t i0 = (int64_t)blockIdx.x * per, i1 = min(n, i0 + per);
  float acc = 0.f;
  for (int64_t i = i0 + threadIdx.x; i < i1; i += blockDim.x) acc += E::to_f(x[i]);
  double t = block_sum_d((double)acc, redd);
  if (threadIdx.x == 0) partials[blockIdx.x] = t;
}

template <int ODT>
__global__ void __launch_bounds__(1024) reduce_final_kernel(const double* partials, int np,
                                                            double* total, void* out) {
  __shared__ double redd[32];
  double t = 0.0;
  for (int i = threadIdx.x; i < np; i += blockDim.x) t += partials[i];
  t = block_sum_d(t, redd);
  if (threadIdx.x == 0) {
    if (total) *total = t;
    if (out) *reinterpret_cast<typename Elem<ODT>::T*>(out) = Elem<ODT>::from_f((float)t);
  }
}

static int partial_blocks() { return device_info().sm_count * 4; }

// ------------------------------------------------------------------ row sums
// x viewed as [outer, n, inner]; out[o, i] = sum_r x[o, r, i].
template <int DT, int ODT>
__global__ void __launch_bounds__(256) reduce_rows_kernel(const void* xv, void* outv,
                                                          int64_t rows, int64_t n) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VEC = E::kVec;
  // one warp per row
  const int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = reinterpret_cast<const T*>(xv) + row * n;
  float acc = 0.f;
  const bool vec = (n % VEC == 0) && aligned16(xv);
  if (vec) {
    const int64_t nv = n / VEC;
    for (int64_t v = lane; v < nv; v += 32) {
      float f[VEC];
      load_vec_stream<DT>(xr + v * VEC, f);
#pragma unroll
      for (int j = 0; j < VEC; ++j) acc += f[j];
    }
  } else {
    for (int64_t c = lane; c < n; c += 32) acc += E::to_f(xr[c]);
  }
  acc = warp_sum(acc);
  if (lane == 0) reinterpret_cast<typename Elem<ODT>::T*>(outv)[row] = Elem<ODT>::from_f(acc);
}

template <int DT, int ODT>
__global__ void __launch_bounds__(256) reduce_mid_kernel(const void* xv, void* outv, int64_t outer,
                                                         int64_t n, int64_t inner) {
  using E = Elem<DT>;
  using T = typename E::T;
  const T* x = reinterpret_cast<const T*>(xv);
  for (int64_t g = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; g < outer * inner;
       g += (int64_t)gridDim.x * blockDim.x) {
    const int64_t o = g / inner, i = g - o * inner;
    const T* p = x + o * n * inner + i;
    float acc = 0.f;
    for (int64_t r = 0; r < n; ++r) acc += E::to_f(p[r * inner]);
    reinterpret_cast<typename Elem<ODT>::T*>(outv)[g] = Elem<ODT>::from_f(acc);
  }
}

// ------------------------------------------------------------------ cross entropy
template <int DT>
__global__ void __launch_bounds__(512) xent_row_kernel(const void* logits, const int64_t* targets,
                                                       int64_t rows, int64_t vocab, int64_t ld,
                                                       int64_t ignore_index, float* row_loss,
                                                       float* row_max, float* row_tgt,
                                                       int* bad_target) {
  using E = Elem<DT>;
  using T = typename E::T;
  constexpr int VEC = E::kVec;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = reinterpret_cast<const T*>(logits) + row * ld;
  float m = -INFINITY, s = 0.f;
  auto push = [&](float f) {
    if (f > m) {
      s = (m == -INFINITY) ? 0.f : s * __expf(m - f);
      m = f;
    }
    s += __expf(f - m);
  };
  const bool vec = (vocab % VEC == 0) && (ld % VEC == 0) && aligned16(logits);
  if (vec) {
    const int64_t nv = vocab / VEC;
    for (int64_t v = threadIdx.x; v < nv; v += blockDim.x) {
      float f[VEC];
      load_vec_stream<DT>(xr + v * VEC, f);
      float vm = f[0];
#pragma unroll
      for (int j = 1; j < VEC; ++j) vm = fmaxf(vm, f[j]);
      if (vm > m) {
        s = (m == -INFINITY) ? 0.f : s * __expf(m - vm);
        m = vm;
      }
#pragma unroll
      for (int j = 0; j < VEC; ++j) s += __expf(f[j] - m);
    }
  } else {
    for (int64_t c = threadIdx.x; c < vocab; c += blockDim.x) push(E::to_f(xr[c]));
  }
  const float gm = block_max(m, red);
  const float gs = block_sum(m == -INFINITY ? 0.f : s * __expf(m - gm), red);
  if (threadIdx.x == 0) {
    const int64_t t = targets[row];
    float loss = 0.f, tl = 0.f;
    if (t == ignore_index) {
      loss = 0.f;
      tl = NAN;
    } else if (t < 0 || t >= vocab) {
      loss = NAN;
      tl = NAN;
      if (bad_target) atomicExch(bad_target, 1);
    } else {
      tl = E::to_f(xr[t]);
      loss = (gm + logf(gs)) - tl;  // logsumexp - target logit
    }
    row_loss[row] = loss;
    if (row_max) row_max[row] = gm;
    if (row_tgt) row_tgt[row] = tl;
  }
}

// Streaming cross entropy for rows whose start and length are 16-byte
// multiples: 256 threads per row, four 16-byte loads in flight per thread, a
// packed max over each group of four vectors, then one running-max update and
// exp2((x - m) log2e) per element.  One HBM read per logit.
template <int DT>
__global__ void __launch_bounds__(256) xent_stream_kernel(const void* logits,
                                                          const int64_t* targets, int64_t vocab,
                                                          int64_t ld, int64_t ignore_index,
                                                          float* row_loss, float* row_max,
                                                          float* row_tgt, int* bad_target) {
  using E = Elem<DT>;
  using T = typename E::T;
  using PK = Packed<DT>;
  constexpr int VEC = E::kVec;
  constexpr int U = 4;
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xrow = reinterpret_cast<const T*>(logits) + row * ld;
  const uint4* xr = reinterpret_cast<const uint4*>(xrow);
  const int nvi = (int)(vocab / VEC);
  const int bd = blockDim.x;
  int64_t tg = 0;
  if (threadIdx.x == 0) tg = targets[row];
  float m = -INFINITY, s = 0.f;
  for (int v0 = threadIdx.x; v0 < nvi; v0 += U * bd) {
    uint4 r[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v0 + u * bd < nvi) r[u] = __ldcs(xr + v0 + u * bd);
    auto pm = PK::neg_inf();
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (v0 + u * bd < nvi) PK::max4(r[u], pm);
    const float cm = PK::init_m(pm);
    if (cm > m) {
      s = (m == -INFINITY) ? 0.f : s * sm100::ex2_approx((m - cm) * kLog2e);
      m = cm;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      if (v0 + u * bd < nvi) {
        float f[VEC];
        PK::widen(r[u], f);
#pragma unroll
        for (int j = 0; j < VEC; ++j) s += sm100::ex2_approx((f[j] - m) * kLog2e);
      }
    }
  }
  const float gm = block_max(m, red);
  const float gs =
      block_sum(m == -INFINITY ? 0.f : s * sm100::ex2_approx((m - gm) * kLog2e), red);
  if (threadIdx.x == 0) {
    float loss, tl;
    if (tg == ignore_index) {
      loss = 0.f;
      tl = NAN;
    } else if (tg < 0 || tg >= vocab) {
      loss = NAN;
      tl = NAN;
      if (bad_target) atomicExch(bad_target, 1);
    } else {
      tl = E::to_f(xrow[tg]);
      loss = (gm + logf(gs)) - tl;
    }
    row_loss[row] = loss;
    if (row_max) row_max[row] = gm;
    if (row_tgt) row_tgt[row] = tl;
  }
}

template <int ODT>
__global__ void __launch_bounds__(1024) xent_final_kernel(const float* row_loss,
                                                          const int64_t* targets, int64_t rows,
                                                          int64_t ignore_index, double* sum_count,
                                                          void* out) {
  __shared__ double redd[32];
  double s = 0.0, c = 0.0;
  for (int64_t i = threadIdx.x; i < rows; i += blockDim.x) {
    if (targets[i] != ignore_index) {
      s += (double)row_loss[i];
      c += 1.0;
    }
  }
  s = block_sum_d(s, redd);
  c = block_sum_d(c, redd);
  if (threadIdx.x == 0) {
    if (sum_count) {
      sum_count[0] = s;
      sum_count[1] = c;
    }
    if (out) *reinterpret_cast<typename Elem<ODT>::T*>(out) = Elem<ODT>::from_f((float)(s / c));
  }
}

template <int ODT>
__global__ void mean_from_sum_count_kernel(const double* sc, void* out) {
  *reinterpret_cast<typename Elem<ODT>::T*>(out) = Elem<ODT>::from_f((float)(sc[0] / sc[1]));
}
template <int ODT>
__global__ void scalar_from_sum_kernel(const double* s, void* out) {
  *reinterpret_cast<typename Elem<ODT>::T*>(out) = Elem<ODT>::from_f((float)s[0]);
}

#define AK_DISPATCH_DT(dt, F, ...)                                  \
  switch (dt) {                                                     \
    case AK_F32: F<AK_F32> __VA_ARGS__; break;                      \
    case AK_F16: F<AK_F16> __VA_ARGS__; break;                      \
    case AK_BF16: F<AK_BF16> __VA_ARGS__; break;                    \
    default: set_error("unsupported dtype %d", dt); return AK_ERR_DTYPE; \
  }

}  // namespace ak

using namespace ak;

extern "C" size_t ak_reduce_workspace_size(void) {
  return (size_t)partial_blocks() * sizeof(double);
}

extern "C" int ak_reduce_sum_full(const void* x, int64_t n, int dtype, double* total, void* out,
                                  int out_dtype, void* workspace, size_t ws_bytes, void* stream) {
  AK_REQUIRE(dtype_ok(dtype) && dtype_ok(out_dtype), AK_ERR_DTYPE, "unsupported dtype");
  AK_REQUIRE(n >= 0, AK_ERR_SHAPE, "negative n");
  const int nb = partial_blocks();
  AK_REQUIRE(workspace && ws_bytes >= (size_t)nb * sizeof(double), AK_ERR_ARG,
             "reduce workspace too small: need %zu bytes", (size_t)nb * sizeof(double));
  AK_REQUIRE(n == 0 || x, AK_ERR_ARG, "null input");
  cudaStream_t st = (cudaStream_t)stream;
  double* partials = reinterpret_cast<double*>(workspace);
  const bool vec = aligned16(x);
  if (vec) {
    AK_DISPATCH_DT(dtype, reduce_partial_kernel, <<<nb, 512, 0, st>>>(x, n, partials))
  } else {
    AK_DISPATCH_DT(dtype, reduce_partial_scalar_kernel, <<<nb, 512, 0, st>>>(x, n, partials))
  }
  AK_DISPATCH_DT(out_dtype, reduce_final_kernel, <<<1, 1024, 0, st>>>(partials, nb, total, out))
  return launch_status("reduce_sum_full");
}

extern "C" int ak_reduce_sum(const void* x, void* out, int64_t outer, int64_t n, int64_t inner,
                             int dtype, int out_dtype, void* stream) {
  AK_REQUIRE(dtype_ok(dtype) && dtype_ok(out_dtype), AK_ERR_DTYPE, "unsupported dtype");
  AK_REQUIRE(outer >= 0 && n >= 0 && inner >= 0, AK_ERR_SHAPE, "negative shape");
  if (outer * inner == 0) return AK_OK;
  AK_REQUIRE(x && out, AK_ERR_ARG, "null tensor pointer");
  cudaStream_t st = (cudaStream_t)stream;
#define AK_RR(D, O)                                                                       \
  if (inner == 1) {                                                                       \
    const int64_t blocks = (outer + 7) / 8;                                               \
    AK_REQUIRE(blocks <= 0x7fffffffLL, AK_ERR_SHAPE, "too many rows");                    \
    reduce_rows_kernel<D, O><<<(unsigned)blocks, 256, 0, st>>>(x, out, outer, n);         \
  } else {                                                                                \
    int64_t blocks = (outer * inner + 255) / 256;                                         \
    if (blocks > device_info().sm_count * 32) blocks = device_info().sm_count * 32;       \
    reduce_mid_kernel<D, O><<<(unsigned)blocks, 256, 0, st>>>(x, out, outer, n, inner);   \
  }
  if (dtype == AK_F32 && out_dtype == AK_F32) { AK_RR(AK_F32, AK_F32) }
  else if (dtype == AK_F16 && out_dtype == AK_F16) { AK_RR(AK_F16, AK_F16) }
  else if (dtype == AK_BF16 && out_dtype == AK_BF16) { AK_RR(AK_BF16, AK_BF16) }
  else if (dtype == AK_F16 && out_dtype == AK_F32) { AK_RR(AK_F16, AK_F32) }
  else if (dtype == AK_BF16 && out_dtype == AK_F32) { AK_RR(AK_BF16, AK_F32) }
  else { set_error("unsupported dtype pair"); return AK_ERR_DTYPE; }
#undef AK_RR
  return launch_status("reduce_sum");
}

extern "C" int ak_scalar_from_sum(const double* total, void* out, int out_dtype, void* stream) {
  AK_REQUIRE(dtype_ok(out_dtype), AK_ERR_DTYPE, "unsupported dtype");
  cudaStream_t st = (cudaStream_t)stream;
  AK_DISPATCH_DT(out_dtype, scalar_from_sum_kernel, <<<1, 1, 0, st>>>(total, out))
  return launch_status("scalar_from_sum");
}

extern "C" int ak_cross_entropy_rows(const void* logits, const int64_t* targets, int64_t rows,
                                     int64_t vocab, int64_t ld, int dtype, int64_t ignore_index,
                                     float* row_loss, float* row_max, float* row_target_logit,
                                     int* bad_target, void* stream) {
  AK_REQUIRE(dtype_ok(dtype), AK_ERR_DTYPE, "unsupported dtype %d", dtype);
  AK_REQUIRE(rows >= 0 && vocab > 0 && ld >= vocab, AK_ERR_SHAPE, "bad logits shape");
  AK_REQUIRE(rows <= 0x7fffffffLL, AK_ERR_SHAPE, "too many rows");
  if (rows == 0) return AK_OK;
  AK_REQUIRE(logits && targets && row_loss, AK_ERR_ARG, "null tensor pointer");
  cudaStream_t st = (cudaStream_t)stream;
  if (vocab % 8 == 0 && ld % 8 == 0 && aligned16(logits)) {
    AK_DISPATCH_DT(dtype, xent_stream_kernel,
                   <<<(unsigned)rows, 256, 0, st>>>(logits, targets, vocab, ld, ignore_index,
                                                    row_loss, row_max, row_target_logit,
                                                    bad_target))
    return launch_status("cross_entropy_rows");
  }
  const int threads = vocab >= 16384 ? 512 : vocab >= 2048 ? 256 : 128;
  AK_DISPATCH_DT(dtype, xent_row_kernel,
                 <<<(unsigned)rows, threads, 0, st>>>(logits, targets, rows, vocab, ld,
                                                      ignore_index, row_loss, row_max,
                                                      row_target_logit, bad_target))
  return launch_status("cross_entropy_rows");
}

extern "C" int ak_cross_entropy_finalize(const float* row_loss, const int64_t* targets,
                                         int64_t rows, int64_t ignore_index, double* sum_count,
                                         void* out, int out_dtype, void* stream) {
  AK_REQUIRE(dtype_ok(out_dtype), AK_ERR_DTYPE, "unsupported dtype");
  AK_REQUIRE(rows >= 0, AK_ERR_SHAPE, "negative rows");
  cudaStream_t st = (cudaStream_t)stream;
  AK_DISPATCH_DT(out_dtype, xent_final_kernel,
                 <<<1, 1024, 0, st>>>(row_loss, targets, rows, ignore_index, sum_count, out))
  return launch_status("cross_entropy_finalize");
}

extern "C" int ak_mean_from_sum_count(const double* sum_count, void* out, int out_dtype,
                                      void* stream) {
  AK_REQUIRE(dtype_ok(out_dtype), AK_ERR_DTYPE, "unsupported dtype");
  cudaStream_t st = (cudaStream_t)stream;
  AK_DISPATCH_DT(out_dtype, mean_from_sum_count_kernel, <<<1, 1, 0, st>>>(sum_count, out))
  return launch_status("mean_from_sum_count");
}

// ------------------------------------------------------------------ no-allocation variant
// Some callers cannot call cudaMalloc at all: code that runs inside another framework's
// memory pool or allocator callback, plugin hosts that forbid device allocation after
// start-up, or real-time paths where an allocation (and its implicit synchronisation) is not
// allowed.  They still need the full sum, whose first kernel writes one fp64 partial per CTA
// into scratch memory.  ak_reduce_sum_full_noalloc keeps that scratch in this file-scope
// device array instead of asking the caller for a workspace.
//
// The array is module memory: every GPU that loads the library holds it (16 KiB) until the
// process exits.  Its host-side name is only a stand-in, so its device address is looked up
// once per device with cudaGetSymbolAddress (with that device current) on the first call on
// that device; make that first call before any stream capture.  All calls on a device share
// the array and it keeps the last call's partials; every partial slot the final kernel reads
// is rewritten by the partial kernel of the same call, so nothing needs clearing.  Calls that
// overlap on the GPU (different streams, no ordering between them) race on the array.
namespace ak {
constexpr int kNoAllocMaxPartials = 2048;  // scratch capacity: fp64 partials (16 KiB)
static __device__ __align__(256) double g_noalloc_partials[kNoAllocMaxPartials];

static double* noalloc_scratch(int* err) {
  static std::mutex mu;
  static double* ptr[64] = {};
  static bool done[64] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) {
    *err = 1;
    set_error("ak_reduce_sum_full_noalloc: no usable current device (%s)",
              cudaGetErrorString(e));
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!done[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_partials);
    if (e != cudaSuccess || p == nullptr) {
      *err = 1;
      set_error("ak_reduce_sum_full_noalloc: cudaGetSymbolAddress failed: %s",
                cudaGetErrorString(e));
      return nullptr;
    }
    ptr[dev] = static_cast<double*>(p);
    done[dev] = true;
  }
  return ptr[dev];
}
}  // namespace ak

extern "C" int ak_reduce_sum_full_noalloc(const void* x, int64_t n, int dtype, double* total,
                                          void* out, int out_dtype, void* stream) {
  AK_REQUIRE(dtype_ok(dtype) && dtype_ok(out_dtype), AK_ERR_DTYPE, "unsupported dtype");
  AK_REQUIRE(n >= 0, AK_ERR_SHAPE, "negative n");
  AK_REQUIRE(n == 0 || x, AK_ERR_ARG, "null input");
  const int nb = partial_blocks();
  AK_REQUIRE(nb <= kNoAllocMaxPartials, AK_ERR_SHAPE,
             "ak_reduce_sum_full_noalloc: this device needs %d partial slots but the built-in "
             "scratch holds at most %d; use ak_reduce_sum_full with a workspace",
             nb, kNoAllocMaxPartials);
  int err = 0;
  double* partials = noalloc_scratch(&err);
  if (err) return AK_ERR_LAUNCH;
  cudaStream_t st = (cudaStream_t)stream;
  if (aligned16(x)) {
    AK_DISPATCH_DT(dtype, reduce_partial_kernel, <<<nb, 512, 0, st>>>(x, n, partials))
  } else {
    AK_DISPATCH_DT(dtype, reduce_partial_scalar_kernel, <<<nb, 512, 0, st>>>(x, n, partials))
  }
  AK_DISPATCH_DT(out_dtype, reduce_final_kernel, <<<1, 1024, 0, st>>>(partials, nb, total, out))
  return launch_status("reduce_sum_full_noalloc");
}
