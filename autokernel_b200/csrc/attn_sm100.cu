// Tensor-core flash attention for sm_100a (reference.py:32-42):
//   O = softmax(Q K^T * scale [+ causal mask]) V,  Q/O [BH, Sq, D], K/V [BH, Sk, D],
// bf16/fp16 in, fp32 softmax statistics and accumulators, D in {64, 128}.
//
// Q/K/V/O may be strided views [batch, heads, seq, D] (e.g. the [B, T, H, D]
// projection outputs of a transformer read in place); K/V may have fewer heads
// (grouped-query attention: query head h reads key/value head h / (H / Hkv)).
// Persistent: one CTA per SM walks a static list of work items.  An item is two 128-row
// query tiles (A, B) of one (batch, head); the CTA walks that item's key/value sequence in
// 128-key blocks.  320 threads, warp-specialised:
//   warp 0      TMA producer: each item's Q tiles, then a 2-stage ring of {K, V} blocks
//               (4-D tensor maps [B, H, S, D], so tails zero-fill inside a head)
//   warp 1      TMEM allocator (512 columns) + single-thread MMA issuer
//   warps 2..5  softmax / epilogue of tile A, one thread per query row
//   warps 6..9  softmax / epilogue of tile B
// TMEM per tile: S = Q K^T (128 fp32 columns) and O (D columns).  The softmax
// threads read their row of S, write P = exp2(S*scale*log2e - m) as packed 16-bit
// pairs over the first 64 columns of S, and the MMA computes O += P V with P read
// from TMEM (tcgen05.mma A-from-TMEM form) and V from shared memory (MN-major).
// While tile A is in its softmax the tensor core works on tile B and vice versa.
//
// Online softmax with a lazily updated reference max: P is computed against the
// row's current reference m; only when a new block raises the row max by more
// than 8 (log2 units, so P stays <= 256) are O and l rescaled by exp2(m_old - m_new)
// in TMEM.  The final O / l is exact up to rounding whatever m is.  Causal
// blocks above the diagonal are skipped; the diagonal block and key tails are
// masked to -inf before the exponent.
//
// Every mbarrier wait is bounded (sm100.cuh): on timeout the CTA unwinds, frees
// its TMEM and records AK_STATUS_TIMEOUT in the device status word.
#include "sm100.cuh"

#include <cstdlib>
#include <mutex>

#include "attn.cuh"

namespace ak {
namespace attn {

using namespace sm100;

constexpr int BQ = 128, BKV = 128, THREADS = 320;
constexpr int CHUNK_BYTES = 128 * 64 * 2;  // one TMA box: 128 rows x 64 16-bit elements

template <int D>
struct Cfg {
  static constexpr int NC = D / 64;                         // 64-wide chunks per row
  static constexpr int TILE_BYTES = NC * CHUNK_BYTES;       // 128 rows x D
  static constexpr int Q_OFF = 0;                           // 2 query tiles
  static constexpr int K_OFF = 2 * TILE_BYTES;              // 2 stages of K
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;      // 2 stages of V
  static constexpr int SMEM = V_OFF + 2 * TILE_BYTES + 1024;
  static constexpr int TMEM_TILE = 256;                     // S (128) + O (<= 128)
};

struct Params {
  void* O;
  int64_t o_sb, o_sh, o_ss;  // output strides (elements): batch, head, sequence
  int Sq, Sk, H, rep;        // rep = query heads per key/value head
  int causal;
  float scale_log2;  // sm_scale * log2(e)
  float ovf;         // |raw score| at which reference.py's 16-bit scores overflow (inf: none)
  uint32_t idesc_qk, idesc_pv;
  int n_qblk;        // query blocks of 256 rows
  int n_items;       // n_qblk * batch * heads
};

// One work item = two 128-row query tiles (one query block) of one (batch, head).
struct Item {
  int b, h, hk, q0, n_kv, n_kv0;  // n_kv0: key blocks of the first tile (causal: may be fewer)
};

AK_D Item item_of(const Params& p, int it) {
  // head-major, heavy (late, causal) query blocks first within each head: consecutive items
  // share a head's K/V blocks in L2
  Item t;
  const int bh = it / p.n_qblk;
  t.b = bh / p.H;
  t.h = bh % p.H;
  t.hk = t.h / p.rep;
  const int qblk = p.n_qblk - 1 - (it - bh * p.n_qblk);
  t.q0 = qblk * 2 * BQ;
  // key blocks the item needs: all of them, or up to the diagonal of its last row; the first
  // tile stops one block earlier when the second tile's diagonal block lies above all its rows
  t.n_kv = (p.Sk + BKV - 1) / BKV;
  t.n_kv0 = t.n_kv;
  if (p.causal) {
    t.n_kv = min(t.n_kv, (min(t.q0 + 2 * BQ, p.Sq) - 1) / BKV + 1);
    t.n_kv0 = min(t.n_kv, (min(t.q0 + BQ, p.Sq) - 1) / BKV + 1);
  }
  return t;
}

// Item of this CTA's k-th round, or -1: CTAs walk the item list in rounds of gridDim.x items,
// forwards in even rounds and backwards in odd ones, which balances the causal work (heavy and
// light query blocks alternate) to within ~1% without any global counter.
AK_D int item_index(const Params& p, int k) {
  const int G = (int)gridDim.x, c = (int)blockIdx.x;
  const int it = k * G + ((k & 1) ? G - 1 - c : c);
  return it < p.n_items ? it : -1;
}

// Persistent: one CTA per SM walks its items; TMEM, barriers and the K/V ring stay live across
// items, and the phases of every barrier follow running counters (items, key blocks per tile,
// ring slots).  The next item's Q is loaded as soon as the current item's last Q K^T is done
// (q_empty), and an item's first P V waits until the previous item's epilogue has read O
// (o_free), so one item's tail overlaps the next one's start.
template <int DT, int D>
__global__ void __launch_bounds__(THREADS, 1)
    attn_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                const __grid_constant__ CUtensorMap tv, Params p) {
  using C = Cfg<D>;
  using E = Elem<DT>;
  using T = typename E::T;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~(uintptr_t)1023);
  __shared__ uint64_t q_full, q_empty, k_full[2], v_full[2], kv_empty[2], s_full[2], p_full[2],
      o_done[2], o_free[2];
  __shared__ uint32_t tmem_slot;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(&q_full, 1);
    mbar_init(&q_empty, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_done[i], 1);
      mbar_init(&o_free[i], 4);
    }
    abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    tma_prefetch_desc(&tq);
    tma_prefetch_desc(&tk);
    tma_prefetch_desc(&tv);
  }
  if (warp == 1) {
    tmem_alloc(&tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_slot;
  volatile int* abort_p = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {  // ------------------------------------------ TMA producer
      bool ok = true;
      int g = 0;  // K/V ring slots used so far
      for (int k = 0; ok; ++k) {
        const int it = item_index(p, k);
        if (it < 0) break;
        const Item t = item_of(p, it);
        // Q of this item once the previous item's last Q K^T has read the old one
        if (k > 0 && !mbar_wait(&q_empty, (k - 1) & 1, abort_p)) break;
        mbar_expect_tx(&q_full, 2 * C::TILE_BYTES);
        for (int x = 0; x < 2; ++x)
          for (int c = 0; c < C::NC; ++c)
            tma_load_4d(smem + C::Q_OFF + x * C::TILE_BYTES + c * CHUNK_BYTES, &tq, &q_full,
                        c * 64, t.q0 + x * BQ, t.h, t.b);
        for (int j = 0; j < t.n_kv; ++j, ++g) {
          const int st = g & 1;
          if (!mbar_wait(&kv_empty[st], ((g >> 1) & 1) ^ 1, abort_p)) { ok = false; break; }
          mbar_expect_tx(&k_full[st], C::TILE_BYTES);
          for (int c = 0; c < C::NC; ++c)
            tma_load_4d(smem + C::K_OFF + st * C::TILE_BYTES + c * CHUNK_BYTES, &tk, &k_full[st],
                        c * 64, j * BKV, t.hk, t.b);
          mbar_expect_tx(&v_full[st], C::TILE_BYTES);
          for (int c = 0; c < C::NC; ++c)
            tma_load_4d(smem + C::V_OFF + st * C::TILE_BYTES + c * CHUNK_BYTES, &tv, &v_full[st],
                        c * 64, j * BKV, t.hk, t.b);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {  // ------------------------------------------ MMA issuer
      const uint32_t sq = smem_u32(smem + C::Q_OFF);
      const uint32_t sk = smem_u32(smem + C::K_OFF);
      const uint32_t sv = smem_u32(smem + C::V_OFF);
      auto qk = [&](int x, int st) {  // S_x = Q_x K_st^T
        const uint32_t d = tmem + x * C::TMEM_TILE;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * CHUNK_BYTES + (kk & 3) * 32;
          umma_ss(d, desc_kmajor(sq + x * C::TILE_BYTES + off),
                  desc_kmajor(sk + st * C::TILE_BYTES + off), p.idesc_qk, kk > 0);
        }
      };
      auto pv = [&](int x, int st, bool acc) {  // O_x += P_x V_st
        const uint32_t d = tmem + x * C::TMEM_TILE + 128;
        const uint32_t a = tmem + x * C::TMEM_TILE;
#pragma unroll
        for (int kk = 0; kk < BKV / 16; ++kk)
          umma_ts(d, a + kk * 8, desc_mnmajor(sv + st * C::TILE_BYTES + kk * 16 * 128, CHUNK_BYTES),
                  p.idesc_pv, (acc || kk > 0) ? 1 : 0);
      };
      bool ok = true;
      int g = 0;               // K/V ring slots consumed so far
      int cnt[2] = {0, 0};     // key blocks processed so far by each tile (S / P phases)
      for (int k = 0; ok; ++k) {
        const int it = item_index(p, k);
        if (it < 0) break;
        const Item t = item_of(p, it);
        if (!mbar_wait(&q_full, k & 1, abort_p) || !mbar_wait(&k_full[g & 1], (g >> 1) & 1, abort_p)) break;
        tc_fence_after();
        // S of both tiles for block 0 (the previous item's P V, issued earlier, has read S)
        qk(0, g & 1);
        umma_commit(&s_full[0]);
        qk(1, g & 1);
        umma_commit(&s_full[1]);
        if (t.n_kv == 1) umma_commit(&q_empty);  // that was the item's last read of Q
        for (int j = 0; ok && j < t.n_kv; ++j, ++g) {
          const int st = g & 1;
          bool v_ready = false, k_ready = false;  // waited for V_j / K_{j+1} in this block
          for (int x = 0; x < 2 && ok; ++x) {
            const int nx = x == 0 ? t.n_kv0 : t.n_kv;  // key blocks of tile x
            if (j >= nx) continue;
            if (!mbar_wait(&p_full[x], cnt[x] & 1, abort_p)) { ok = false; break; }
            // the item's first P V overwrites O: the previous item's epilogue must have read it
            if (j == 0 && k > 0 && !mbar_wait(&o_free[x], (k - 1) & 1, abort_p)) { ok = false; break; }
            if (!v_ready && !mbar_wait(&v_full[st], (g >> 1) & 1, abort_p)) { ok = false; break; }
            v_ready = true;
            tc_fence_after();
            pv(x, st, j > 0);
            ++cnt[x];
            if (x == 1) umma_commit(&kv_empty[st]);  // tile 1 takes every block
            if (j == nx - 1) {
              umma_commit(&o_done[x]);
            } else {
              const int ng = g + 1;
              if (!k_ready && !mbar_wait(&k_full[ng & 1], (ng >> 1) & 1, abort_p)) { ok = false; break; }
              k_ready = true;
              tc_fence_after();
              qk(x, ng & 1);
              umma_commit(&s_full[x]);
              if (x == 1 && j + 1 == t.n_kv - 1) umma_commit(&q_empty);  // last read of Q
            }
          }
        }
      }
    }
  } else {  // ------------------------------------------------ softmax / epilogue
    const int x = (warp - 2) >> 2;       // query tile 0 (warps 2..5) or 1 (warps 6..9)
    const int quarter = warp & 3;        // TMEM lanes this warp may access
    const int row_in_tile = quarter * 32 + lane;
    const uint32_t lane_base = (uint32_t)(quarter * 32) << 16;
    const uint32_t t_s = tmem + x * C::TMEM_TILE + lane_base;
    const uint32_t t_o = t_s + 128;
    bool ok = true;
    int cnt = 0;  // key blocks this tile has processed so far (S / P phases)
    for (int k = 0; ok; ++k) {
      const int it = item_index(p, k);
      if (it < 0) break;
      int qrow, nx;  // this thread's query row, the tile's key blocks
      {
        const Item t = item_of(p, it);
        qrow = t.q0 + x * BQ + row_in_tile;
        nx = x == 0 ? t.n_kv0 : t.n_kv;
      }
      float m_ref = -INFINITY, l = 0.f;
      float rmax_raw = -INFINITY;  // the row's largest visible raw score
      for (int j = 0; j < nx; ++j, ++cnt) {
        // every lane polls the barrier itself: a lane-0 wait plus a broadcast put a divergent
        // branch and a shuffle on each block's critical path (+9% measured)
        const bool w = mbar_wait(&s_full[x], cnt & 1, abort_p);
        if (!__all_sync(0xffffffffu, w)) { ok = false; break; }
        tc_fence_after();
        const int k0 = j * BKV;
        // keys < kmax are visible to this row
        int kmax = p.Sk - k0;
        if (p.causal) kmax = min(kmax, qrow - k0 + 1);
        // The row's 128 scores come out of TMEM once (four loads, one wait) and stay in
        // registers for both the max and the exponentials.
        uint32_t r[128];
  #pragma unroll
        for (int c = 0; c < 4; ++c) tmem_ld32(t_s + c * 32, r + c * 32);
        tmem_wait_ld();
  #pragma unroll
        for (int c = 0; c < 4; ++c) tmem_regs_ready(r + c * 32);
        // no per-element masks when every row of the warp sees the whole block
        const bool full = __all_sync(0xffffffffu, kmax >= BKV);
        if (!full) {
  #pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i >= kmax) r[i] = __float_as_uint(-INFINITY);
        }
        // four independent chains of 3-input max (one dependent 128-long chain costs its
        // latency 128 times)
        float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
  #pragma unroll
        for (int i = 0; i < 128; i += 8)
  #pragma unroll
          for (int q = 0; q < 4; ++q)
            mx[q] = fmax3(mx[q], __uint_as_float(r[i + 2 * q]), __uint_as_float(r[i + 2 * q + 1]));
        float bmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
        rmax_raw = fmaxf(rmax_raw, bmax);
        bmax *= p.scale_log2;
        // lazy rescale: move the reference max only when it grows by more than 8.  The
        // decision is per row (lane); the TMEM rescale of O is warp-collective, so the whole
        // warp runs it whenever any lane needs it, with alpha = 1 for the others.
        float alpha = 1.f;
        if (bmax > m_ref + 8.f) {
          if (j > 0 && m_ref != -INFINITY) alpha = ex2_approx(m_ref - bmax);
          m_ref = bmax;
        }
        l *= alpha;
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
  #pragma unroll 1
          for (int c = 0; c < D / 8; ++c) {
            uint32_t o[8];
            tmem_ld8(t_o + c * 8, o);
            tmem_wait_ld();
            tmem_regs_ready8(o);
  #pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * alpha);
            tmem_st8(t_o + c * 8, o);
          }
          tmem_wait_st();
        }
        // P = exp2(s * scale_log2 - m_ref) (masked scores are -inf -> 0), packed in pairs
        // over S columns [0, 64)
        const float mr = m_ref == -INFINITY ? 0.f : m_ref;  // fully masked row: all P = 0
        float2 sum2[2] = {{0.f, 0.f}, {0.f, 0.f}};  // packed partial sums of P
  #pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint32_t pk[8];
  #pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float2 e = ffma2_bcast(__uint_as_float(r[c * 16 + 2 * i]),
                                         __uint_as_float(r[c * 16 + 2 * i + 1]), p.scale_log2, -mr);
            const float a = ex2_approx(e.x), b = ex2_approx(e.y);
            fadd2_acc(sum2[i & 1], a, b);
            if constexpr (DT == AK_BF16) {
              __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
              pk[i] = *reinterpret_cast<uint32_t*>(&h);
            } else {
              __half2 h = __floats2half2_rn(a, b);
              pk[i] = *reinterpret_cast<uint32_t*>(&h);
            }
          }
          tmem_st8(t_s + c * 8, pk);
        }
        l += (sum2[0].x + sum2[1].x) + (sum2[0].y + sum2[1].y);
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[x]);
      }
      // epilogue: O / l -> global
      int w = 0;
      if (ok && lane == 0) w = mbar_wait(&o_done[x], k & 1, abort_p) ? 1 : 0;
      w = __shfl_sync(0xffffffffu, w, 0);
      if (!w) {
        ok = false;
        break;
      }
      tc_fence_after();
      // reference.py forms the scores in the input dtype: in fp16 a visible score beyond
      // +-65504 (or one that leaves no finite key) turns the row's softmax into NaN there
      const bool nan_row = rmax_raw >= p.ovf || rmax_raw <= -p.ovf;
      const float inv = nan_row ? __int_as_float(0x7fffffff) : (l > 0.f ? 1.f / l : 0.f);
      const int bh = it / p.n_qblk;
      T* orow = reinterpret_cast<T*>(p.O) + (bh / p.H) * p.o_sb + (bh % p.H) * p.o_sh +
                (int64_t)qrow * p.o_ss;
#pragma unroll 1
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        tmem_ld32(t_o + c * 32, r);
        tmem_wait_ld();
        tmem_regs_ready(r);
        if (c == D / 32 - 1) {  // O has been read: the next item's first P V may overwrite it
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&o_free[x]);
        }
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
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace attn

namespace attn {

// 4-D map over [batch, heads, seq, D] with arbitrary (16-byte multiple) strides,
// innermost D contiguous; boxes of 128 rows x 64 elements.
static bool make_tmap_4d(CUtensorMap* m, int dtype, const void* base, int64_t B, int64_t H,
                         int S, int D, const int64_t* st) {
  uint64_t dims[4] = {(uint64_t)D, (uint64_t)S, (uint64_t)H, (uint64_t)B};
  uint64_t strides[3] = {(uint64_t)st[2] * 2, (uint64_t)st[1] * 2, (uint64_t)st[0] * 2};
  uint32_t box[4] = {64, 128, 1, 1};
  return make_tmap(m, dtype, 4, base, dims, strides, box);
}

template <int DT, int D>
static int launch(const AttnShape& a, cudaStream_t st) {
  CUtensorMap tq, tk, tv;
  if (!make_tmap_4d(&tq, DT, a.Q, a.B, a.H, a.Sq, D, a.qs) ||
      !make_tmap_4d(&tk, DT, a.K, a.B, a.Hkv, a.Sk, D, a.ks) ||
      !make_tmap_4d(&tv, DT, a.V, a.B, a.Hkv, a.Sk, D, a.vs))
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
  // fp16 scores round to inf from 65520 on, before and after the scale (reference.py:36)
  p.ovf = DT == AK_F16 ? 65520.f * fminf(1.f, 1.f / a.scale) : INFINITY;
  const int fmt = DT == AK_BF16 ? 1 : 0;
  p.idesc_qk = idesc_f16(fmt, BQ, BKV, false, false);
  p.idesc_pv = idesc_f16(fmt, BQ, D, false, true);
  p.n_qblk = (a.Sq + 2 * BQ - 1) / (2 * BQ);
  p.n_items = (int)(p.n_qblk * a.B * a.H);
  const cudaError_t attr = smem_optin<attn_kernel<DT, D>>(Cfg<D>::SMEM);
  AK_REQUIRE(attr == cudaSuccess, AK_ERR_LAUNCH, "attention smem attribute: %s",
             cudaGetErrorString(attr));
  const int grid = min(p.n_items, device_info().sm_count);
  attn_kernel<DT, D><<<grid, THREADS, Cfg<D>::SMEM, st>>>(tq, tk, tv, p);
  return launch_status("tc_attention");
}

}  // namespace attn

static bool strides_ok(const int64_t* st) {
  return st[0] % 8 == 0 && st[1] % 8 == 0 && st[2] % 8 == 0 && st[0] > 0 && st[1] > 0 &&
         st[2] > 0;
}

bool tc_attention_ok(const AttnShape& a) {
  if (a.dtype != AK_F16 && a.dtype != AK_BF16) return false;
  if (a.D != 64 && a.D != 128) return false;
  if (!aligned16(a.Q) || !aligned16(a.K) || !aligned16(a.V) || !aligned16(a.O)) return false;
  if (!strides_ok(a.qs) || !strides_ok(a.ks) || !strides_ok(a.vs) || !strides_ok(a.os))
    return false;
  if (a.Hkv <= 0 || a.H % a.Hkv) return false;
  return device_info().cc_major == 10;
}

int tc_attention(const AttnShape& a, cudaStream_t s) {
  AK_REQUIRE(a.B * a.H <= 0x7fffffffLL, AK_ERR_SHAPE, "batch*heads too large");
  AK_REQUIRE(a.B * a.H <= 65535, AK_ERR_SHAPE, "batch*heads %lld exceeds 65535",
             (long long)(a.B * a.H));
  if (a.dtype == AK_BF16) {
    if (a.D == 128) return attn::launch<AK_BF16, 128>(a, s);
    return attn::launch<AK_BF16, 64>(a, s);
  }
  if (a.D == 128) return attn::launch<AK_F16, 128>(a, s);
  return attn::launch<AK_F16, 64>(a, s);
}

}  // namespace ak

