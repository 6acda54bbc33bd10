// Tensor-core flash attention over a CTA pair (tcgen05 cta_group::2), head_dim 128
// (reference.py:32-42):  O = softmax(Q K^T * scale [+ causal mask]) V.
//
// Layout.  Two CTAs on neighbouring SMs share one M = 256 MMA.  The pair owns 256 query
// rows of one (batch, head): CTA r holds rows [q0 + 128 r, +128) as its A operand and
// accumulator rows, but only HALF of every key/value block as B: 64 keys x 128 for
// S = Q K^T, and 128 keys x 64 head columns for O += P V.  So each SM stages half of the
// K/V traffic in shared memory and reads 96 B/clk (not 128) for Q K^T.
//
// Pipeline.  TMEM per CTA: O (128 fp32 columns) and THREE score buffers S0..S2 (128
// columns each).  The MMA issuer keeps Q K^T up to two key blocks ahead of the softmax,
// so the softmax of block j does not wait for its scores and the tensor core always has
// the next block's Q K^T or the previous block's P V to run.  P overwrites the first 64
// columns of its own score buffer as packed 16-bit pairs (read by the A-from-TMEM MMA).
//
// 384 threads:
//   warps 0..7   softmax / epilogue; warp w serves TMEM lane quarter w % 4 (32 rows) and
//                key half w / 4 (64 of the block's 128 keys).  The two warps of a row
//                quarter exchange their partial row max through shared memory on a
//                64-thread named barrier, and publish their half of P on their own
//                barrier so the first half of P V starts before the second is ready.
//   warp 8       TMA producer (both CTAs): Q once, a STAGES-deep ring of K/V halves
//   warp 9       TMEM allocator (pair, 512 columns) + MMA issuer (CTA 0 only)
// In blocks without masked keys a fixed share of the exponentials runs on the FMA pipe
// (attn_softmax.cuh) to relieve the MUFU unit.
//
// Online softmax with a lazily moved reference max: O and l are rescaled only when a
// block raises the row max by more than 8 (log2 units).  The rescale of O in TMEM waits
// for the previous block's P V to finish (the release of its K/V stage).
//
// Every wait is bounded; on timeout a CTA records AK_STATUS_TIMEOUT, unwinds, meets its
// peer at the closing cluster barrier and frees its TMEM.  No load uses cluster multicast.
#include "sm100.cuh"

#include <mutex>

#include "attn.cuh"
#include "attn_softmax.cuh"

namespace ak {
namespace attn_pair {

using namespace sm100;
using namespace attn_sm;

constexpr int D = 128, BQ = 128, BKV = 128, THREADS = 384, STAGES = 5, NS = 3;
constexpr int CHUNK = 128 * 64 * 2;   // 128 rows x 64 16-bit elements (one TMA box)
constexpr int Q_TILE = 2 * CHUNK;     // 128 rows x 128
constexpr int K_HALF = 64 * 128 * 2;  // 64 keys x 128 (two 64-row chunks of 8 KB)
constexpr int V_HALF = 128 * 64 * 2;  // 128 keys x 64 head columns
constexpr int KV_STAGE = K_HALF + V_HALF;
constexpr int Q_OFF = 0;
constexpr int KV_OFF = Q_TILE;
constexpr int SMEM = KV_OFF + STAGES * KV_STAGE + 1024;
constexpr int T_O = 0, T_S = 128;  // TMEM columns: O, then the NS score buffers

struct Params {
  void* O;
  int64_t o_sb, o_sh, o_ss;
  int Sq, Sk, H, rep, causal;
  float scale_log2;
  uint32_t idesc_qk, idesc_pv;
  int n_qblk;  // 256-row query blocks per head
};

template <int DT, int EMU>
__global__ void __launch_bounds__(THREADS, 1)
    attn_pair_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                     const __grid_constant__ CUtensorMap tv, Params p) {
  using E = Elem<DT>;
  using T = typename E::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ uint64_t q_full, kv_full[STAGES], kv_empty[STAGES], s_full[NS], p_half[NS][2], o_done;
  __shared__ float red_max[2][2][128];  // [block parity][key half][row]
  __shared__ float red_sum[2][128];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int bh = (int)blockIdx.y;
  const int b = bh / p.H, h = bh % p.H, hk = h / p.rep;
  const int qblk = p.n_qblk - 1 - (int)(blockIdx.x >> 1);  // heavy (late) blocks first
  const int q0 = qblk * 2 * BQ;
  int n_kv = (p.Sk + BKV - 1) / BKV;
  if (p.causal) n_kv = min(n_kv, min(q0 + 2 * BQ - 1, p.Sq - 1) / BKV + 1);

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    for (int i = 0; i < STAGES; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    // P barriers per score buffer: warps run up to NS - 1 blocks apart, and a count-based
    // barrier shared by consecutive blocks could complete on a mix of their arrivals
    for (int i = 0; i < NS; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_half[i][0], 8);  // 4 softmax warps of a key half, in each CTA of the pair
      mbar_init(&p_half[i][1], 8);
    }
    mbar_init(&o_done, 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 8 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 9) {
    tmem_alloc_pair(&tmem_slot, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  cluster_sync();  // both CTAs' barriers exist before anyone signals a peer
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;

  if (warp == 8) {
    if (lane == 0) {  // ------------------------------------------ TMA producer
      if (leader) mbar_expect_tx(&q_full, 2 * Q_TILE);
      for (int c = 0; c < 2; ++c)
        tma_load_4d_pair(smem + Q_OFF + c * CHUNK, &tq, &q_full, c * 64, q0 + BQ * (int)rank, h,
                         b);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j % STAGES;
        if (!mbar_wait(&kv_empty[st], ((j / STAGES) & 1) ^ 1, abort_p)) break;
        uint8_t* sk = smem + KV_OFF + st * KV_STAGE;
        if (leader) mbar_expect_tx(&kv_full[st], 2 * KV_STAGE);
        for (int c = 0; c < 2; ++c)
          tma_load_4d_pair(sk + c * (K_HALF / 2), &tk, &kv_full[st], c * 64,
                           j * BKV + 64 * (int)rank, hk, b);
        tma_load_4d_pair(sk + K_HALF, &tv, &kv_full[st], 64 * (int)rank, j * BKV, hk, b);
      }
    }
  } else if (warp == 9) {
    if (lane == 0 && leader) {  // --------------------------------- MMA issuer
      const uint32_t sq = smem_u32(smem + Q_OFF);
      const uint32_t skv = smem_u32(smem + KV_OFF);
      auto qk = [&](int blk) {  // S[blk % NS] = Q K_blk^T   (M 256, N 128, K 128)
        const uint32_t d = tmem + T_S + (blk % NS) * 128;
        const uint32_t sk = skv + (blk % STAGES) * KV_STAGE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk)
          umma_ss_pair(d, desc_kmajor(sq + (kk >> 2) * CHUNK + (kk & 3) * 32),
                       desc_kmajor(sk + (kk >> 2) * (K_HALF / 2) + (kk & 3) * 32), p.idesc_qk,
                       kk > 0);
      };
      auto pv = [&](int blk, int half) {  // O += P_blk V_blk over keys [64 half, +64)
        const uint32_t a = tmem + T_S + (blk % NS) * 128;
        const uint32_t sv = skv + (blk % STAGES) * KV_STAGE + K_HALF;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int kk = half * 4 + k;
          umma_ts_pair(tmem + T_O, a + kk * 8, desc_mnmajor(sv + kk * 16 * 128, V_HALF),
                       p.idesc_pv, (blk > 0 || kk > 0) ? 1 : 0);
        }
      };
      auto kv_ready = [&](int blk) {
        return mbar_wait(&kv_full[blk % STAGES], (blk / STAGES) & 1, abort_p);
      };
      bool ok = mbar_wait(&q_full, 0, abort_p);
      const int ahead = min(NS, n_kv);
      for (int i = 0; ok && i < ahead; ++i) {
        if (!kv_ready(i)) {
          ok = false;
          break;
        }
        tc_fence_after();
        qk(i);
        umma_commit_pair_both(&s_full[i % NS]);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (!mbar_wait(&p_half[j % NS][0], (j / NS) & 1, abort_p)) {
          ok = false;
          break;
        }
        tc_fence_after();
        pv(j, 0);
        if (!mbar_wait(&p_half[j % NS][1], (j / NS) & 1, abort_p)) {
          ok = false;
          break;
        }
        tc_fence_after();
        pv(j, 1);
        umma_commit_pair_both(&kv_empty[j % STAGES]);  // K/V stage free; O holds P_j V_j
        const int nb = j + NS;
        if (nb < n_kv) {
          if (!kv_ready(nb)) {
            ok = false;
            break;
          }
          tc_fence_after();
          qk(nb);  // into the buffer P_j just left (P_j V_j precedes it in the MMA order)
          umma_commit_pair_both(&s_full[nb % NS]);
        }
      }
      if (ok) umma_commit_pair_both(&o_done);
    }
  } else if (warp < 8) {  // ------------------------------- softmax / epilogue
    const int quarter = warp & 3, kh = warp >> 2;  // row quarter, key half
    const int row_in_tile = quarter * 32 + lane;
    const int qrow = q0 + BQ * (int)rank + row_in_tile;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const float2 sl = make_float2(p.scale_log2, p.scale_log2);
    float m_ref = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      int w = 0;
      if (lane == 0) w = mbar_wait(&s_full[j % NS], (j / NS) & 1, abort_p) ? 1 : 0;
      if (!__shfl_sync(0xffffffffu, w, 0)) {
        ok = false;
        break;
      }
      tc_fence_after();
      const uint32_t t_s = tmem + lane_base + T_S + (j % NS) * 128;
      // keys [k0, k0 + kmax) of this warp's 64 are visible to the row
      const int k0 = j * BKV + kh * 64;
      int kmax = p.Sk - k0;
      if (p.causal) kmax = min(kmax, qrow - k0 + 1);
      uint32_t r[64];
      tmem_ld32(t_s + kh * 64, r);
      tmem_ld32(t_s + kh * 64 + 32, r + 32);
      tmem_wait_ld();
      tmem_regs_ready(r);
      tmem_regs_ready(r + 32);
      const bool full = __all_sync(0xffffffffu, kmax >= 64);
      if (!full) {
#pragma unroll
        for (int i = 0; i < 64; ++i)
          if (i >= kmax) r[i] = __float_as_uint(-INFINITY);
      }
      float a8[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) a8[k] = fmaxf(__uint_as_float(r[k]), __uint_as_float(r[k + 8]));
#pragma unroll
      for (int base = 16; base < 64; base += 16)
#pragma unroll
        for (int k = 0; k < 8; ++k)
          a8[k] = fmax3(a8[k], __uint_as_float(r[base + k]), __uint_as_float(r[base + 8 + k]));
      const float pmax =
          fmax3(fmax3(a8[0], a8[1], a8[2]), fmax3(a8[3], a8[4], a8[5]), fmaxf(a8[6], a8[7]));
      red_max[j & 1][kh][row_in_tile] = pmax;
      // the partner's P store below overwrites S columns this warp has just read
      tc_fence_before();
      named_bar_sync(1 + quarter, 64);
      tc_fence_after();
      const float bmax = fmaxf(pmax, red_max[j & 1][kh ^ 1][row_in_tile]) * p.scale_log2;
      // lazy rescale (the same decision in both warps of the row quarter)
      float alpha = 1.f;
      if (bmax > m_ref + 8.f) {
        if (j > 0 && m_ref != -INFINITY) alpha = ex2_approx(m_ref - bmax);
        m_ref = bmax;
      }
      l *= alpha;
      if (__any_sync(0xffffffffu, alpha != 1.f)) {
        // O must hold P_{j-1} V_{j-1} before it is rescaled: wait for that block's stage
        // release, committed after its P V.  (Phase j-1 of that barrier cannot be
        // overtaken: the next release of the stage needs this block's P.)
        int w2 = 0;
        if (lane == 0)
          w2 = mbar_wait(&kv_empty[(j - 1) % STAGES], ((j - 1) / STAGES) & 1, abort_p) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, w2, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t t_o = tmem + lane_base + T_O + kh * 64;
#pragma unroll 1
        for (int c = 0; c < 2; ++c) {
          uint32_t o[32];
          tmem_ld32(t_o + c * 32, o);
          tmem_wait_ld();
          tmem_regs_ready(o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
          tmem_st32(t_o + c * 32, o);
        }
        tmem_wait_st();
        // every P V accumulates into all of O: neither key half may publish P_j (and let
        // the MMA start) before both halves of O are rescaled
        tc_fence_before();
        named_bar_sync(1 + quarter, 64);
      }
      const float mr = m_ref == -INFINITY ? 0.f : m_ref;  // fully masked row: all P = 0
      const float2 nm = make_float2(-mr, -mr);
      float2 bsum = make_float2(0.f, 0.f);
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        uint32_t pk[16];
        const float2 s = full ? p_chunk<DT, EMU>(r + c * 32, sl, nm, pk)
                              : p_chunk<DT, 0>(r + c * 32, sl, nm, pk);
        bsum = __fadd2_rn(bsum, s);
        tmem_st16(t_s + kh * 32 + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(map_to_rank(&p_half[j % NS][kh], 0));
      l += bsum.x + bsum.y;
    }
    // epilogue: l over both key halves, then O / l for this warp's 64 head columns
    red_sum[kh][row_in_tile] = l;
    named_bar_sync(1 + quarter, 64);
    l += red_sum[kh ^ 1][row_in_tile];
    int w = 0;
    if (ok && lane == 0) w = mbar_wait(&o_done, 0, abort_p) ? 1 : 0;
    w = __shfl_sync(0xffffffffu, w, 0);
    if (w) {
      tc_fence_after();
      const float inv = l > 0.f ? 1.f / l : 0.f;
      T* orow = reinterpret_cast<T*>(p.O) + b * p.o_sb + h * p.o_sh + (int64_t)qrow * p.o_ss +
                kh * 64;
      const uint32_t t_o = tmem + lane_base + T_O + kh * 64;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        uint32_t r[32];
        tmem_ld32(t_o + c * 32, r);
        tmem_wait_ld();
        tmem_regs_ready(r);
        if (qrow < p.Sq) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            uint4 raw;
            T* e = reinterpret_cast<T*>(&raw);
#pragma unroll
            for (int i = 0; i < 8; ++i) e[i] = E::from_f(__uint_as_float(r[q * 8 + i]) * inv);
            reinterpret_cast<uint4*>(orow + c * 32)[q] = raw;
          }
        }
      }
    }
  }
  tc_fence_before();
  cluster_sync();  // neither CTA frees TMEM or exits while its peer may still signal it
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

static bool make_map(CUtensorMap* m, int dtype, const void* base, int64_t B, int64_t H, int S,
                     const int64_t* st, uint32_t rows) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  uint32_t box[4] = {64, rows, 1, 1};
  return make_tmap(m, dtype, 4, base, dims, strides, box);
}

template <int DT, int EMU>
static int launch_t(const AttnShape& a, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  if (!make_map(&tq, DT, a.Q, a.B, a.H, a.Sq, a.qs, 128) ||
      !make_map(&tk, DT, a.K, a.B, a.Hkv, a.Sk, a.ks, 64) ||
      !make_map(&tv, DT, a.V, a.B, a.Hkv, a.Sk, a.vs, 128))
    return AK_ERR_LAUNCH;
  Params p;
  p.O = a.O;
  p.o_sb = a.os[0];
  p.o_sh = a.os[1];
  p.o_ss = a.os[2];
  p.Sq = a.Sq;
  p.Sk = a.Sk;
  p.H = (int)a.H;
  p.rep = (int)(a.H / a.Hkv);
  p.causal = a.causal;
  p.scale_log2 = a.scale * 1.4426950408889634f;
  const int fmt = DT == AK_BF16 ? 1 : 0;
  p.idesc_qk = idesc_f16(fmt, 256, BKV, false, false);
  p.idesc_pv = idesc_f16(fmt, 256, D, false, true);
  p.n_qblk = (a.Sq + 2 * BQ - 1) / (2 * BQ);
  static std::once_flag once;
  static cudaError_t attr = cudaSuccess;
  std::call_once(once, [] {
    attr = cudaFuncSetAttribute(attn_pair_kernel<DT, EMU>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM);
  });
  AK_REQUIRE(attr == cudaSuccess, AK_ERR_LAUNCH, "attention pair smem attribute: %s",
             cudaGetErrorString(attr));
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)(2 * p.n_qblk), (unsigned)(a.B * a.H), 1);
  cfg.blockDim = dim3(THREADS, 1, 1);
  cfg.dynamicSmemBytes = SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attrs[1];
  attrs[0].id = cudaLaunchAttributeClusterDimension;
  attrs[0].val.clusterDim.x = 2;
  attrs[0].val.clusterDim.y = 1;
  attrs[0].val.clusterDim.z = 1;
  cfg.attrs = attrs;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, attn_pair_kernel<DT, EMU>, tq, tk, tv, p);
  AK_REQUIRE(e == cudaSuccess, AK_ERR_LAUNCH, "attention pair launch: %s",
             cudaGetErrorString(e));
  return launch_status("tc_attention_pair");
}

// Share of the exponentials on the FMA pipe in mask-free blocks: 4 of every 16 pairs.
// Measured (8x32x4096x128 bf16): 0 / 4 / 6 / 8 of 16 -> 741 / 758 / 728 / 703 TFLOP/s causal.
constexpr int kEmuPairs = 4;

template <int DT>
static int launch(const AttnShape& a, cudaStream_t st) {
  return launch_t<DT, kEmuPairs>(a, st);
}

}  // namespace attn_pair

int tc_attention_pair(const AttnShape& a, cudaStream_t s) {
  if (a.dtype == AK_BF16) return attn_pair::launch<AK_BF16>(a, s);
  return attn_pair::launch<AK_F16>(a, s);
}

}  // namespace ak
