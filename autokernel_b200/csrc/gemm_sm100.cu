// Tensor-core GEMM for sm_100a: C[M,N] = A[M,K] @ B, bf16/fp16 in, fp32
// accumulate in TMEM, input dtype out.  Serves matmul (reference.py:10-12),
// and both halves of the fused MLP (reference.py:45-55):
//   MODE_MN   B is [K, N] row-major (torch.matmul(A, B)); UMMA B is MN-major
//   MODE_K    B is [N, K] row-major (x @ W^T, the down projection)
//   MODE_DUAL two K-major weights Wg, Wu [H, K]: the epilogue writes
//             act(x @ Wg^T) * (x @ Wu^T), the SwiGLU hidden, in one pass.
//   MODE_XENT B is [N, K] (an LM head [vocab, dim]): nothing is stored; the epilogue
//             rounds each logit to the dtype and reduces every row of its 256-column vocab
//             tile to (max, sum of exp(logit - max)), and copies out the target's logit
//             when the target falls in the tile (cross entropy without the logits tensor).
//
// Structure: persistent CTAs (one per SM, 192 threads), warp-specialised:
//   warp 0      TMA producer: 4-stage ring of {A 128x64, B 256x64} tiles,
//               128-byte swizzle, completion on per-stage mbarriers
//   warp 1      TMEM allocator + single-thread tcgen05.mma issuer
//               (M=128, N=256, K=16 per instruction), commits free each
//               stage and publish a finished accumulator
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 32 columns, convert, store
// The accumulator is double-buffered in TMEM (2 x 256 of the 512 columns)
// so the epilogue of tile i overlaps the main loop of tile i+1.  Tiles are
// visited in GROUP_M-row bands so that concurrently running CTAs share A and
// B panels in L2.  No split-K and no atomics: results are deterministic.
// Every mbarrier wait is bounded (see sm100.cuh).
#include "sm100.cuh"
#include "ak_act.cuh"
#include "gemm.cuh"

#include <cudaTypedefs.h>
#include <cstdlib>
#include <mutex>

namespace ak {

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

bool make_tmap(CUtensorMap* map, int dtype, int rank, const void* base, const uint64_t* dims,
               const uint64_t* strides_bytes, const uint32_t* box) {
  auto fn = encode_fn();
  if (!fn) {
    set_error("cuTensorMapEncodeTiled unavailable from the driver");
    return false;
  }
  cuuint64_t gd[5], gs[4];
  cuuint32_t bx[5], es[5];
  for (int i = 0; i < rank; ++i) {
    gd[i] = dims[i];
    bx[i] = box[i];
    es[i] = 1;
  }
  for (int i = 0; i + 1 < rank; ++i) gs[i] = strides_bytes[i];
  CUresult r = fn(map, dtype == AK_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                        : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  (cuuint32_t)rank, const_cast<void*>(base), gd, gs, bx, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed (CUresult %d)", (int)r);
    return false;
  }
  return true;
}

namespace gemm {

using namespace sm100;

constexpr int BM = 128, BN = 256, BK = 64, STAGES = 4, THREADS = 192, GROUP_M = 8;
constexpr int A_BYTES = BM * BK * 2;  // 16 KB
constexpr int B_BYTES = BN * BK * 2;  // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024;
constexpr int TMEM_COLS = 512;

enum { MODE_K = 0, MODE_MN = 1, MODE_DUAL = 2, MODE_XENT = 3 };

struct Params {
  int M, N, K;  // N = output columns (hidden columns in MODE_DUAL)
  void* C;
  int64_t ldc;
  int tiles_m, tiles_n, num_tiles;
  int act;
  int vec_store;  // C rows (and R rows) are 16-byte aligned
  uint32_t idesc;
  const void* R;  // optional residual added in the epilogue (may alias C)
  int64_t ldr;
  // optional rotary embedding of output columns [0, rope_cols): interleaved pairs within
  // head_dim-wide groups, position = row % rope_T, fp32 tables [rope_T, rope_hd / 2]
  const float* rope_cos;
  const float* rope_sin;
  int rope_T, rope_hd, rope_cols;
  // MODE_XENT: targets [M] (int64), partials [tiles_n][M] of (max, sum exp), target logits [M]
  const int64_t* xt_targets;
  float2* xt_part;
  float* xt_tgt;
  // RMSNorm folded into the GEMM (models/llama_7b.py:22-30 in front of a projection):
  // rs_in [rs_tiles][M] holds per-row sums of squares of A's rows, and each output row is
  // scaled by 1 / sqrt(sum / K + eps) before rounding (the norm weight is folded into B).
  // ss_out [tiles_n][M] receives per-row sums of squares of the stored outputs, one per
  // 256-column tile, for the RMSNorm that follows.
  const float* rs_in;
  int rs_tiles;
  float rs_inv_k, rs_eps;
  float* ss_out;
};

// 1 / rms of row `row` from its partial sums of squares
AK_D float row_scale(const Params& p, int row) {
  if (!p.rs_in || row >= p.M) return 1.f;
  float ss = 0.f;
  for (int t = 0; t < p.rs_tiles; ++t) ss += __ldg(p.rs_in + (int64_t)t * p.M + row);
  return rsqrtf(ss * p.rs_inv_k + p.rs_eps);
}

// max of 32 floats with the 3-input max (depth 4)
AK_D float max32f(const float* v) {
  float a[11];
#pragma unroll
  for (int t = 0; t < 10; ++t) a[t] = fmax3(v[3 * t], v[3 * t + 1], v[3 * t + 2]);
  a[10] = fmaxf(v[30], v[31]);
  const float w0 = fmax3(a[0], a[1], a[2]), w1 = fmax3(a[3], a[4], a[5]);
  const float w2 = fmax3(a[6], a[7], a[8]), w3 = fmaxf(a[9], a[10]);
  return fmaxf(fmax3(w0, w1, w2), w3);
}

// Cross-entropy epilogue of one row of a 256-column vocab tile (MODE_XENT).  The logits are
// rounded to the dtype first -- the values an unfused LM head would store -- so the row max
// and the target logit are bitwise those of the unfused path (reference.py:58-60 over
// models/llama_7b.py's logits).
template <int DT>
AK_D void xent_row_tile(const Params& p, uint32_t tbase, int row, int tn) {
  constexpr float kL2e = 1.4426950408889634f;
  const int64_t tg = row < p.M ? __ldg(p.xt_targets + row) : -1;
  const int col0 = tn * BN;
  const int64_t rel = tg - col0;
  float m = -INFINITY, s = 0.f, tl = 0.f;
#pragma unroll 1
  for (int c = 0; c < BN; c += 32) {
    uint32_t r[32];
    tmem_ld32(tbase + c, r);
    tmem_wait_ld();
    tmem_regs_ready(r);
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; j += 2) {
      v[j] = __uint_as_float(r[j]);
      v[j + 1] = __uint_as_float(r[j + 1]);
      rnd2<DT>(v[j], v[j + 1]);
    }
    if (col0 + c + 32 > p.N) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (col0 + c + j >= p.N) v[j] = -INFINITY;
    }
    const float cm = max32f(v);
    if (cm > m) {
      s = (m == -INFINITY) ? 0.f : s * ex2_approx((m - cm) * kL2e);
      m = cm;
    }
    if (m != -INFINITY) {
      float s0 = 0.f, s1 = 0.f;
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        s0 += ex2_approx((v[j] - m) * kL2e);
        s1 += ex2_approx((v[j + 1] - m) * kL2e);
      }
      s += s0 + s1;
    }
    const int64_t rc = rel - c;
    if (rc >= 0 && rc < 32) {
#pragma unroll
      for (int j = 0; j < 32; ++j)
        if (j == rc) tl = v[j];
    }
  }
  if (row < p.M) {
    p.xt_part[(int64_t)tn * p.M + row] = make_float2(m, s);
    if (rel >= 0 && rel < BN && col0 + rel < p.N) p.xt_tgt[row] = tl;
  }
}

AK_D void tile_coords(int t, const Params& p, int& tm, int& tn) {
  const int group = GROUP_M * p.tiles_n;
  const int g = t / group;
  const int first = g * GROUP_M;
  const int gsz = min(p.tiles_m - first, GROUP_M);
  const int r = t - g * group;
  tm = first + r % gsz;
  tn = r / gsz;
}

// Rotate the (even, odd) column pairs of 32 consecutive outputs of one row
// (reference.py:63-69 applied to the projection output, before rounding).
AK_D void rope_row32(const Params& p, int row, int col, float* v) {
  if (!p.rope_cos || col >= p.rope_cols || row >= p.M) return;
  const int t = row % p.rope_T;
  const int half = p.rope_hd >> 1;
  if ((p.rope_hd & 31) == 0 && col + 32 <= p.rope_cols && (half & 3) == 0 &&
      ((reinterpret_cast<uintptr_t>(p.rope_cos) | reinterpret_cast<uintptr_t>(p.rope_sin)) & 15) == 0) {
    // a 32-column chunk lies inside one head: its 16 pairs use 16 consecutive table entries,
    // read as float4s (the table rows are 16-byte aligned when head_dim / 2 is a multiple of 4)
    const int i0 = (col % p.rope_hd) >> 1;
    const float4* cs = reinterpret_cast<const float4*>(p.rope_cos + (int64_t)t * half + i0);
    const float4* sn = reinterpret_cast<const float4*>(p.rope_sin + (int64_t)t * half + i0);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 c4 = __ldg(cs + q), s4 = __ldg(sn + q);
      const float co[4] = {c4.x, c4.y, c4.z, c4.w}, si[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int jj = q * 4 + e;
        const float x1 = v[2 * jj], x2 = v[2 * jj + 1];
        v[2 * jj] = fmaf(x1, co[e], -x2 * si[e]);
        v[2 * jj + 1] = fmaf(x1, si[e], x2 * co[e]);
      }
    }
    return;
  }
  const float* cs = p.rope_cos + (int64_t)t * half;
  const float* sn = p.rope_sin + (int64_t)t * half;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int c = col + 2 * j;
    if (c >= p.rope_cols) break;
    const int i = (c % p.rope_hd) >> 1;
    const float co = __ldg(cs + i), si = __ldg(sn + i);
    const float x1 = v[2 * j], x2 = v[2 * j + 1];
    v[2 * j] = fmaf(x1, co, -x2 * si);
    v[2 * j + 1] = fmaf(x1, si, x2 * co);
  }
}

template <int DT>
AK_D float store_row32(const Params& p, int row, int col, const float* v) {
  using E = Elem<DT>;
  using T = typename E::T;
  float ss = 0.f;
  if (row >= p.M) return ss;
  T* c = reinterpret_cast<T*>(p.C) + (int64_t)row * p.ldc + col;
  const T* rr = p.R ? reinterpret_cast<const T*>(p.R) + (int64_t)row * p.ldr + col : nullptr;
  if (p.vec_store && col + 32 <= p.N) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      float add[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      if (rr) {
        const uint4 rv = reinterpret_cast<const uint4*>(rr)[q];
        const T* re = reinterpret_cast<const T*>(&rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) add[j] = E::to_f(re[j]);
      }
      uint4 raw;
      T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        e[j] = E::from_f(v[q * 8 + j] + add[j]);
        const float st = E::to_f(e[j]);
        ss = fmaf(st, st, ss);
      }
      reinterpret_cast<uint4*>(c)[q] = raw;
    }
  } else {
    for (int j = 0; j < 32 && col + j < p.N; ++j) {
      const T e = E::from_f(v[j] + (rr ? E::to_f(rr[j]) : 0.f));
      c[j] = e;
      ss = fmaf(E::to_f(e), E::to_f(e), ss);
    }
  }
  return ss;
}

template <int DT, int MODE>
__global__ void __launch_bounds__(THREADS, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                const __grid_constant__ CUtensorMap tb2, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ uint64_t full[STAGES], empty[STAGES], acc_full[2], acc_empty[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&ta);
    tma_prefetch_desc(&tb);
    if (MODE == MODE_DUAL) tma_prefetch_desc(&tb2);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;
  const int nk = (p.K + BK - 1) / BK;

  if (warp == 0) {
    if (lane == 0) {  // ---------------- TMA producer
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x) {
        int tm, tn;
        tile_coords(t, p, tm, tn);
        const int m0 = tm * BM;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&empty[s], ph ^ 1, abort_p)) {
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * STAGE_BYTES;
          uint8_t* sb = sa + A_BYTES;
          mbar_expect_tx(&full[s], STAGE_BYTES);
          const int k0 = kb * BK;
          tma_load_2d(sa, &ta, &full[s], k0, m0);
          if (MODE == MODE_K || MODE == MODE_XENT) {
            tma_load_2d(sb, &tb, &full[s], k0, tn * BN);
          } else if (MODE == MODE_DUAL) {
            tma_load_2d(sb, &tb, &full[s], k0, tn * (BN / 2));
            tma_load_2d(sb + B_BYTES / 2, &tb2, &full[s], k0, tn * (BN / 2));
          } else {
#pragma unroll
            for (int c = 0; c < BN / 64; ++c)
              tma_load_2d(sb + c * (64 * BK * 2), &tb, &full[s], tn * BN + c * 64, k0);
          }
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ---------------- MMA issuer
      int s = 0;
      uint32_t ph = 0;
      bool ok = true;
      int it = 0;
      for (int t = blockIdx.x; ok && t < p.num_tiles; t += gridDim.x, ++it) {
        const int b = it & 1;
        const uint32_t aph = (it >> 1) & 1;
        if (!mbar_wait(&acc_empty[b], aph ^ 1, abort_p)) break;
        tc_fence_after();
        const uint32_t d = tmem + b * BN;
        for (int kb = 0; kb < nk; ++kb) {
          if (!mbar_wait(&full[s], ph, abort_p)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * STAGE_BYTES);
          const uint32_t sb = sa + A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = desc_kmajor(sa + k * 32);
            const uint64_t bd = (MODE == MODE_MN) ? desc_mnmajor(sb + k * 16 * 128, 64 * BK * 2)
                                                  : desc_kmajor(sb + k * 32);
            umma_ss(d, ad, bd, p.idesc, (kb | k) != 0);
          }
          umma_commit(&empty[s]);
          if (++s == STAGES) {
            s = 0;
            ph ^= 1;
          }
        }
        if (ok) umma_commit(&acc_full[b]);
      }
    }
  } else {  // ---------------- epilogue warps 2..5
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    int it = 0;
    for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, ++it) {
      const int b = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      // one lane waits, the warp follows: tcgen05.ld below is warp-collective
      int ok = 0;
      if (lane == 0) ok = mbar_wait(&acc_full[b], aph, abort_p) ? 1 : 0;
      ok = __shfl_sync(0xffffffffu, ok, 0);
      if (!ok) break;
      tc_fence_after();
      int tm, tn;
      tile_coords(t, p, tm, tn);
      const int row = tm * BM + q * 32 + lane;
      const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + b * BN;
      const float rsc = row_scale(p, row);
      if (MODE == MODE_XENT) {
        xent_row_tile<DT>(p, tbase, row, tn);
      } else if (MODE != MODE_DUAL) {
        float ss = 0.f;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_wait_ld();
          tmem_regs_ready(r);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]) * rsc;
          rope_row32(p, row, tn * BN + c, v);
          ss += store_row32<DT>(p, row, tn * BN + c, v);
        }
        if (p.ss_out && row < p.M) p.ss_out[(int64_t)tn * p.M + row] = ss;
      } else {
#pragma unroll 1
        for (int c = 0; c < BN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + BN / 2 + c, u);
          tmem_wait_ld();
          tmem_regs_ready(g);
          tmem_regs_ready(u);
          float v[32];
#pragma unroll
          for (int j = 0; j < 32; ++j)
            v[j] = swiglu_ref<DT>(p.act, __uint_as_float(g[j]) * rsc, __uint_as_float(u[j]) * rsc);
          store_row32<DT>(p, row, tn * (BN / 2) + c, v);
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, TMEM_COLS);
  }
}

template <int DT, int MODE>
static int launch(const void* A, const void* B, const void* B2, void* C, int M, int N, int K,
                  int64_t lda, int64_t ldb, int64_t ldc, int act, const void* R, int64_t ldr,
                  const RopeEpilogue& rope, cudaStream_t st, const XentEpilogue* xent = nullptr,
                  const RmsEpilogue* rms = nullptr) {
  CUtensorMap ta, tb, tb2;
  {
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)M}, str[1] = {(uint64_t)lda * 2};
    uint32_t box[2] = {BK, BM};
    if (!make_tmap(&ta, DT, 2, A, dims, str, box)) return AK_ERR_LAUNCH;
  }
  if (MODE == MODE_MN) {
    uint64_t dims[2] = {(uint64_t)N, (uint64_t)K}, str[1] = {(uint64_t)ldb * 2};
    uint32_t box[2] = {64, BK};
    if (!make_tmap(&tb, DT, 2, B, dims, str, box)) return AK_ERR_LAUNCH;
    tb2 = tb;
  } else {
    const uint32_t rows = MODE == MODE_DUAL ? BN / 2 : BN;
    uint64_t dims[2] = {(uint64_t)K, (uint64_t)N}, str[1] = {(uint64_t)ldb * 2};
    uint32_t box[2] = {BK, rows};
    if (!make_tmap(&tb, DT, 2, B, dims, str, box)) return AK_ERR_LAUNCH;
    if (MODE == MODE_DUAL) {
      if (!make_tmap(&tb2, DT, 2, B2, dims, str, box)) return AK_ERR_LAUNCH;
    } else {
      tb2 = tb;
    }
  }
  Params p;
  p.M = M;
  p.N = N;
  p.K = K;
  p.C = C;
  p.ldc = ldc;
  p.tiles_m = (M + BM - 1) / BM;
  const int bn_out = MODE == MODE_DUAL ? BN / 2 : BN;
  p.tiles_n = (N + bn_out - 1) / bn_out;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.act = act;
  p.vec_store = (ldc % 8 == 0) && aligned16(C) && (!R || ((ldr % 8 == 0) && aligned16(R)));
  p.R = R;
  p.ldr = ldr;
  p.rope_cos = rope.cos;
  p.rope_sin = rope.sin;
  p.rope_T = rope.T;
  p.rope_hd = rope.head_dim;
  p.rope_cols = rope.cols;
  p.xt_targets = xent ? xent->targets : nullptr;
  p.xt_part = xent ? reinterpret_cast<float2*>(xent->part) : nullptr;
  p.xt_tgt = xent ? xent->tgt : nullptr;
  p.rs_in = rms ? rms->rs_in : nullptr;
  p.rs_tiles = rms ? rms->rs_tiles : 0;
  p.rs_inv_k = 1.f / (float)K;
  p.rs_eps = rms ? rms->eps : 0.f;
  p.ss_out = rms ? rms->ss_out : nullptr;
  p.idesc = sm100::idesc_f16(DT == AK_BF16 ? 1 : 0, BM, BN, false, MODE == MODE_MN);

  const cudaError_t attr_err = smem_optin<gemm_kernel<DT, MODE>>(SMEM_BYTES);
  AK_REQUIRE(attr_err == cudaSuccess, AK_ERR_LAUNCH, "gemm: smem attribute: %s",
             cudaGetErrorString(attr_err));
  int grid = device_info().sm_count;
  if (grid > p.num_tiles) grid = p.num_tiles;
  gemm_kernel<DT, MODE><<<grid, THREADS, SMEM_BYTES, st>>>(ta, tb, tb2, p);
  return launch_status("tc_gemm");
}

}  // namespace gemm

// Tensor-core eligibility: 16-bit types, TMA-describable operands (16-byte
// aligned bases, row strides that are 16-byte multiples).
bool tc_gemm_ok(int dtype, const void* A, const void* B, const void* B2, int64_t K, int64_t lda,
                int64_t ldb, bool b_mn) {
  if (dtype != AK_F16 && dtype != AK_BF16) return false;
  if (!aligned16(A) || !aligned16(B) || (B2 && !aligned16(B2))) return false;
  if (lda % 8 || ldb % 8 || K % 8) return false;
  (void)b_mn;
  return device_info().cc_major == 10;
}

int tc_gemm(int dtype, int mode, const void* A, const void* B, const void* B2, void* C, int M,
            int N, int K, int64_t lda, int64_t ldb, int64_t ldc, int act, const void* R,
            int64_t ldr, const RopeEpilogue& rope, cudaStream_t st) {
  using namespace gemm;
#define AK_TCG(D)                                                                               \
  if (mode == MODE_K) return launch<D, MODE_K>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, rope, st);   \
  if (mode == MODE_MN) return launch<D, MODE_MN>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, rope, st); \
  return launch<D, MODE_DUAL>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, rope, st);
  if (dtype == AK_BF16) { AK_TCG(AK_BF16) }
  AK_TCG(AK_F16)
#undef AK_TCG
}

int tc_gemm_rms(int dtype, bool dual, const void* A, const void* B, const void* B2, void* C,
                int M, int N, int K, int64_t lda, int64_t ldb, int64_t ldc, int act,
                const void* R, int64_t ldr, const RmsEpilogue& rms, const RopeEpilogue& none,
                cudaStream_t st) {
  using namespace gemm;
  if (dtype == AK_BF16) {
    if (dual)
      return launch<AK_BF16, MODE_DUAL>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, none,
                                        st, nullptr, &rms);
    return launch<AK_BF16, MODE_K>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, none, st,
                                   nullptr, &rms);
  }
  if (dual)
    return launch<AK_F16, MODE_DUAL>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, none, st,
                                     nullptr, &rms);
  return launch<AK_F16, MODE_K>(A, B, B2, C, M, N, K, lda, ldb, ldc, act, R, ldr, none, st,
                                nullptr, &rms);
}

int tc_gemm_xent(int dtype, const void* x, const void* w, int M, int N, int K, int64_t ldx,
                 int64_t ldw, const XentEpilogue& xe, cudaStream_t st) {
  using namespace gemm;
  if (dtype == AK_BF16)
    return launch<AK_BF16, MODE_XENT>(x, w, nullptr, nullptr, M, N, K, ldx, ldw, 0, 0, nullptr,
                                      0, RopeEpilogue(), st, &xe);
  return launch<AK_F16, MODE_XENT>(x, w, nullptr, nullptr, M, N, K, ldx, ldw, 0, 0, nullptr, 0,
                                   RopeEpilogue(), st, &xe);
}

}  // namespace ak

