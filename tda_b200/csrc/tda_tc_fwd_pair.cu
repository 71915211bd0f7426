// Tensor-core forward on CTA pairs (tcgen05 cta_group::2), head_dim 128:
// the same math and transform as tda_tc_fwd.cu's one-CTA-per-tile kernel
// (triton_threshold_attention.py:19-115, :489-519), with two neighbouring
// query tiles of one (batch, head) on the two CTAs of a cluster.
//
// Why pairs: one thread of the even CTA issues every product for both tiles
// as M = 256 products.  Each CTA then holds only half of every key tile (64
// keys of K for S = Q K^T, 64 of the 128 head-dim columns of V for O += P V),
// so a 16 KB ring slot carries what a 32 KB slot carried before and the ring
// runs twice as many key steps ahead -- the one-tile kernel's differential
// form, with three 32 KB tiles per key step and room for four, runs with
// under one step of lead.  The issuing thread's fixed cost per step (waits,
// commits: 50-200 cycles each) is also spread over twice the work.
//
// Measured on B200 (TDA_B200_FWD_PAIR=1 selects this kernel; it is not the
// default): 13-22% slower than the one-tile kernel (differential
// (8,32,8192,128) 1186 against 1358 TFLOP/s for the main kernel, rect
// (4,32,4096,128) 946 against 1124).  Traces of one cluster: a key step in
// the loop takes about as long as in the one-tile kernel (~1.23 us; the
// transform and the hand-off of S, not the ring, bound it), while a CTA
// spends ~7.4 us outside its loop against ~4-5 us (cluster synchronisation,
// the peer's first copies only after it, two CTAs' start-up on one path).
// Results are bit-identical to the one-tile kernel's.
//
// Per CTA (rank 0 = even, "leader"; rank 1 = odd, "peer"):
//   warp 0      TMA producer: its own query tile(s) once, its half of every
//               K / V tile into the ring, the key-table entries (all 128
//               keys: its S rows span the whole key tile) into a local ring.
//               The halves complete on the leader's ring barriers, whose
//               expected byte count (both halves) the leader's producer sets.
//   warp 1      leader: PV (and QK1) issuer; peer: forwards "query tile
//               landed" to the leader.
//   warps 2-9   transform of the CTA's own 128 rows (as in the one-tile
//               kernel).  P-ready (with the warp's nonzero-slab mask) and
//               S2-released reach the leader's barriers: the leader's warps
//               arrive locally, the peer's warps send asynchronous stores that
//               complete transaction bytes there (an arrive with release at
//               cluster scope would stall the warp for the round trip).
//   warp 10     leader: QK (rect) / QK2 (differential) issuer.
// Products finish into barriers of both CTAs (one commit per CTA).  Causal
// skipping runs per pair: both CTAs step through the key tiles up to the odd
// tile's diagonal, and the even tile masks the extra tile to zero.
//
// Every wait is bounded (WaitCtl).  Both CTAs meet at a cluster barrier
// before the TMEM is freed, so no product of the pair still reads the other
// CTA's shared memory or TMEM when a CTA leaves.
#include <cuda_bf16.h>

#include <cstdio>
#include <cstdlib>

#include "tda_internal.h"
#include "tda_ptx.cuh"
#include "tda_transform.cuh"

namespace tda {
namespace {

using namespace tc;

constexpr int kPairRkRing = 4;
constexpr int kPairHeadGroup = 2;      // (batch, head) slices interleaved in launch order
constexpr int kPairSmemBudget = 232448;
constexpr int kPairMaxSlots = 12;

constexpr int ST_PP_SLOT = 0x801, ST_PP_RK = 0x802;
constexpr int ST_PM_Q = 0x901, ST_PM_SLOT = 0x902, ST_PM_P = 0x903, ST_PM_S2 = 0x904;
constexpr int ST_PT_Q = 0xA01, ST_PT_RK = 0xA02, ST_PT_S = 0xA03, ST_PT_O = 0xA04;

template <bool DIFF>
struct PairCfg {
  static constexpr int D = 128;
  static constexpr int kTWG = 2;                 // transform warpgroups
  static constexpr int kTW = 8;                  // transform warps 2 .. 9
  static constexpr int kQk2W = 10;               // QK issuer (rect) / QK2 issuer (differential)
  static constexpr int kThreads = 32 * 11;
  static constexpr int kBoxBytes = kTile * 128;  // 128 rows x 64 bf16: Q boxes, V halves, output staging
  static constexpr int kKBoxBytes = 64 * 128;    // 64 key rows x 64 bf16: the two boxes of a K half
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr int kHalfBytes = kTileBytes / 2;  // one CTA's half of a K or V tile
  static constexpr int kNQ = DIFF ? 2 : 1;
  static constexpr int kRkPerTile = (DIFF ? 2 : 1) * (kTile + 8);
  static constexpr int kRkFloats = kPairRkRing * kRkPerTile;
  static constexpr int kBarBytes = 1024;
  static constexpr int kQssBytes = kNQ * kTWG * kTile * 4;
  static constexpr int kFixed = kNQ * kTileBytes + kRkFloats * 4 + kBarBytes + kQssBytes + 1024;
  static constexpr int kSlotsRaw = (kPairSmemBudget - kFixed) / kHalfBytes;
  static constexpr int kSlots = kSlotsRaw > kPairMaxSlots ? kPairMaxSlots : kSlotsRaw;
  static_assert(kSlots >= 6, "not enough shared memory for the K/V ring");
  static_assert(kSlots * kHalfBytes >= kTile * D * 4, "the ring stages the fp32 output tile");
  static constexpr int kOffRing = kNQ * kTileBytes;
  static constexpr int kOffRk = kOffRing + kSlots * kHalfBytes;
  static constexpr int kOffBar = kOffRk + kRkFloats * 4;
  static constexpr int kOffQss = kOffBar + kBarBytes;
  static constexpr int kSmemBytes = kOffQss + kQssBytes + 1024;
  // TMEM columns (512 per CTA): rect S slots {0,128,256}, O at 384;
  // differential S1 slots {0,256}, S2 at 128, O at 384.
  static constexpr int kSSlots = DIFF ? 2 : 3;
  static constexpr int kColS2 = 128;
  static constexpr int kColO = 384;
  static __device__ __forceinline__ uint32_t col_s(int slot) {
    return DIFF ? (slot ? 256u : 0u) : static_cast<uint32_t>(slot * 128);
  }
};

struct PairBars {
  uint64_t q_full;   // this CTA's query tile(s) landed
  uint64_t q_pair;   // leader: the peer's query tile(s) landed (forwarded by the peer)
  uint64_t o_full;   // every product of the pair has completed
  uint64_t drain;    // leader, warp 1's own products (abort)
  uint64_t drain2;   // leader, warp 10's own products (abort)
  uint64_t s_full[3];
  uint64_t p_full[3];   // leader: 8 local arrivals + 8 peer mask words (4 B each) of the slot
  uint64_t pv_done[3];  // leader, rect: the PV reading the slot's P has run
  uint64_t s2_free[2];  // leader, differential: 8 local arrivals + 8 peer tokens: every warp holds S2
  uint64_t rk_full[kPairRkRing];
  uint64_t rk_empty[kPairRkRing];
  uint64_t slot_full[kPairMaxSlots];   // leader: both halves of a ring entry landed
  uint64_t slot_empty[kPairMaxSlots];  // both CTAs: the products reading the entry have run
  uint32_t tmem_base;
  int abort_flag;
  // leader: per S slot, CTA and transform warp, (j + 1) << 8 | mask of the
  // 16-key slabs of key tile j in which that warp's rows hold a nonzero P
  // (every warp writes its word for every tile)
  alignas(16) uint32_t tile_mask[3][2][8];
  uint32_t s2_token[2][8];  // leader: targets of the peer warps' S2-released stores
};
static_assert(sizeof(PairBars) <= 1024, "barrier block too large");

// Ring order (differential): K1_0, K2_0, K1_1, then per key tile j: K2_{j+1},
// V_j, K1_{j+2}; (rect): K_0, K_1, K_2, then per j: V_j, K_{j+3}.
__device__ __forceinline__ int pr_k1(int m) { return m == 0 ? 0 : (m == 1 ? 2 : 3 * m - 1); }
__device__ __forceinline__ int pr_k2(int m) { return m == 0 ? 1 : 3 * m; }
__device__ __forceinline__ int pr_v(int j, int n_kt) { return j <= n_kt - 2 ? 4 + 3 * j : 3 * n_kt - 1; }
__device__ __forceinline__ int pr_v_rect(int j, int n_kt) {
  const int ahead = n_kt > 3 ? n_kt - 3 : 0;
  return (n_kt < 3 ? n_kt : 3) + j + (j < ahead ? j : ahead);
}

__device__ __forceinline__ uint32_t leader_addr(const void* p) { return mapa_shared(smem_u32(p), 0); }

// ------------------------------------------------------------------ producer
// Copies that only this CTA waits on, issued by the thread that initialised
// the barriers before the cluster is synchronised: the query tile(s) and
// key-table entry 0.
template <bool DIFF, bool NORM>
__device__ void pair_first_loads(const TcFwdParams& p, uint8_t* smem, PairBars* bars, int bh, int qt) {
  using C = PairCfg<DIFF>;
  const int h_idx = bh % p.heads, b_idx = bh / p.heads;
  if (!(p.inject & 1)) {
    mbar_arrive_expect_tx(&bars->q_full, C::kNQ * C::kTileBytes);
#pragma unroll
    for (int b = 0; b < 2; ++b) {
      tma_load_4d(smem + b * C::kBoxBytes, &p.tm_q1, &bars->q_full, b * 64, qt * kTile, h_idx, b_idx);
      if constexpr (DIFF)
        tma_load_4d(smem + C::kTileBytes + b * C::kBoxBytes, &p.tm_q2, &bars->q_full, b * 64, qt * kTile, h_idx,
                    b_idx);
    }
  }
  if constexpr (NORM) {
    float* dst = reinterpret_cast<float*>(smem + C::kOffRk);
    constexpr int kNB = DIFF ? 2 : 1;
    mbar_arrive_expect_tx(&bars->rk_full[0], C::kRkPerTile * 4);
    const size_t off = static_cast<size_t>(bh) * p.S_pad;
    const size_t moff = static_cast<size_t>(p.BH) * p.S_pad + static_cast<size_t>(bh) * (p.S_pad / 16);
    bulk_load(dst, p.rk1 + off, kTile * 4, &bars->rk_full[0]);
    if constexpr (DIFF) bulk_load(dst + kTile, p.rk2 + off, kTile * 4, &bars->rk_full[0]);
    bulk_load(dst + kNB * kTile, p.rk1 + moff, 32, &bars->rk_full[0]);
    if constexpr (DIFF) bulk_load(dst + kNB * kTile + 8, p.rk2 + moff, 32, &bars->rk_full[0]);
  }
}

// This CTA's halves of the K / V tiles (and the key-table entries from tile 1
// on), in the order the leader's issuers consume them.  A K half is keys
// [64 rank, 64 rank + 64) of the tile (two 8 KB boxes), a V half head-dim
// columns [64 rank, 64 rank + 64) of all 128 keys (one 16 KB box).
template <bool DIFF, bool NORM>
__device__ void pair_producer(const TcFwdParams& p, uint8_t* smem, PairBars* bars, const WaitCtl& ctl, int bh,
                              int n_kt, uint32_t rank) {
  using C = PairCfg<DIFF>;
  uint8_t* ring = smem + C::kOffRing;
  float* rk_s = reinterpret_cast<float*>(smem + C::kOffRk);
  const int h_idx = bh % p.heads, b_idx = bh / p.heads;
  const bool leader = rank == 0;
  int ridx = 0;
  int rk_n = NORM ? 1 : 0;
  bool ok = true;
  // kind: 0 = K1 (K), 1 = K2, 2 = V
  auto load_half = [&](int kind, int j) {
    if (!ok) return;
    const int slot = ridx % C::kSlots;
    const uint32_t par = ((ridx / C::kSlots) & 1) ^ 1;
    if (!mbar_wait(&bars->slot_empty[slot], par, ctl, ST_PP_SLOT)) {
      ok = false;
      return;
    }
    // the leader's barrier expects both halves; the peer's bytes may land
    // before this arrival, which only delays the phase until it
    if (leader) mbar_arrive_expect_tx(&bars->slot_full[slot], 2 * C::kHalfBytes);
    const uint32_t fb = leader_addr(&bars->slot_full[slot]);
    uint8_t* dst = ring + slot * C::kHalfBytes;
    if (kind == 2) {
      tma_load_4d_pair(dst, &p.tm_v, fb, static_cast<int>(rank) * 64, j * kTile, h_idx, b_idx);
    } else {
      const CUtensorMap* map = kind == 0 ? &p.tm_k1h : &p.tm_k2h;
#pragma unroll
      for (int b = 0; b < 2; ++b)
        tma_load_4d_pair(dst + b * C::kKBoxBytes, map, fb, b * 64, j * kTile + static_cast<int>(rank) * 64, h_idx,
                         b_idx);
    }
    ++ridx;
  };
  auto load_rk = [&](int j) {
    if constexpr (NORM) {
      if (!ok) return;
      const int e = j % kPairRkRing;
      const uint32_t par = ((j / kPairRkRing) & 1) ^ 1;
      if (!mbar_wait(&bars->rk_empty[e], par, ctl, ST_PP_RK)) {
        ok = false;
        return;
      }
      mbar_arrive_expect_tx(&bars->rk_full[e], C::kRkPerTile * 4);
      float* dst = rk_s + e * C::kRkPerTile;
      constexpr int kNB = DIFF ? 2 : 1;
      const size_t off = static_cast<size_t>(bh) * p.S_pad + static_cast<size_t>(j) * kTile;
      const size_t moff = static_cast<size_t>(p.BH) * p.S_pad + static_cast<size_t>(bh) * (p.S_pad / 16) +
                          static_cast<size_t>(j) * (kTile / 16);
      bulk_load(dst, p.rk1 + off, kTile * 4, &bars->rk_full[e]);
      if constexpr (DIFF) bulk_load(dst + kTile, p.rk2 + off, kTile * 4, &bars->rk_full[e]);
      bulk_load(dst + kNB * kTile, p.rk1 + moff, 32, &bars->rk_full[e]);
      if constexpr (DIFF) bulk_load(dst + kNB * kTile + 8, p.rk2 + moff, 32, &bars->rk_full[e]);
      ++rk_n;
    }
  };

  if constexpr (!DIFF) {
    for (int j = 0; j < 3 && j < n_kt; ++j) {
      if (j > 0) load_rk(j);
      load_half(0, j);
    }
    for (int j = 0; j < n_kt && ok; ++j) {
      load_half(2, j);
      if (j + 3 < n_kt) {
        load_rk(j + 3);
        load_half(0, j + 3);
      }
    }
  } else {
    load_half(0, 0);
    load_half(1, 0);
    if (n_kt > 1) {
      load_rk(1);
      load_half(0, 1);
    }
    for (int j = 0; j < n_kt && ok; ++j) {
      if (j + 1 < n_kt) load_half(1, j + 1);
      load_half(2, j);
      if (j + 2 < n_kt) {
        load_rk(j + 2);
        load_half(0, j + 2);
      }
    }
  }

  if (!ok) {
    // Abort: wait for the copies this CTA can see complete.  The leader's
    // ring barriers count both halves; the peer's halves complete there, so
    // the peer lets a fixed time pass instead (a 16 KB copy lands within
    // microseconds) before it goes on to the cluster barrier.
    if (!(p.inject & 1)) drain_wait(&bars->q_full, 0, ctl);
    if (leader) {
      const int first = ridx > C::kSlots ? ridx - C::kSlots : 0;
      for (int i = first; i < ridx; ++i) drain_wait(&bars->slot_full[i % C::kSlots], (i / C::kSlots) & 1, ctl);
    } else {
      const uint64_t t0 = global_timer_ns();
      while (global_timer_ns() - t0 < 200000ull) {
      }
    }
    const int rfirst = rk_n > kPairRkRing ? rk_n - kPairRkRing : 0;
    for (int i = rfirst; i < rk_n; ++i) drain_wait(&bars->rk_full[i % kPairRkRing], (i / kPairRkRing) & 1, ctl);
  }
}

// ------------------------------------------------------------------ issuers
// One thread of the leader.  Products are M = 256 (both CTAs' rows): S = Q K^T
// with N = 128 keys (64 from each CTA's ring half), O += P V with N = 128
// head-dim columns (64 from each CTA) and P from each CTA's TMEM.
template <bool DIFF, bool F16>
struct PairIssuer {
  using C = PairCfg<DIFF>;
  static constexpr uint32_t kIdQK = idesc_f16(256, 128, !F16, false);
  static constexpr uint32_t kIdPV = idesc_f16(256, C::D, !F16, true);
  PairBars* bars;
  const WaitCtl& ctl;
  uint32_t tmem;
  uint32_t ring_base;
  bool ok;
  bool o_started;
  unsigned slabs = 0;  // 16-key slabs multiplied by pv_at, per CTA of the pair (diagnostics)

  __device__ PairIssuer(uint8_t* smem, PairBars* b, const WaitCtl& c, uint32_t t)
      : bars(b), ctl(c), tmem(t), ring_base(smem_u32(smem + C::kOffRing)), ok(true), o_started(false) {}

  // arrive on the barrier at the same place in both CTAs once this thread's
  // products so far have completed
  __device__ void commit_both(uint64_t* bar) {
    if (!ok) return;
    const uint32_t a = smem_u32(bar);
    tc_commit_pair(a);
    tc_commit_pair(mapa_shared(a, 1));
  }
  __device__ void commit_own(uint64_t* bar) {
    if (ok) tc_commit_pair(smem_u32(bar));
  }
  __device__ int acquire(int idx) {
    const int slot = idx % C::kSlots;
    if (!ok) return slot;
    ok = mbar_wait(&bars->slot_full[slot], (idx / C::kSlots) & 1, ctl, ST_PM_SLOT);
    tc_fence_after();
    return slot;
  }
  __device__ void wait(uint64_t* bar, uint32_t parity, int code) {
    if (!ok) return;
    ok = mbar_wait(bar, parity, ctl, code);
    tc_fence_after();
  }
  // a barrier that the other CTA's threads arrive on
  __device__ void wait_cl(uint64_t* bar, uint32_t parity, int code) {
    if (!ok) return;
    ok = mbar_wait_cluster(bar, parity, ctl, code);
    tc_fence_after();
  }
  __device__ void qk(int idx, uint32_t dcol, uint32_t q_base) { qk_at(acquire(idx), dcol, q_base); }
  __device__ void qk_at(int slot, uint32_t dcol, uint32_t q_base) {
    if (!ok) return;
    const uint32_t k_base = ring_base + slot * C::kHalfBytes;
#pragma unroll
    for (int kk = 0; kk < C::D / 16; ++kk) {
      const uint32_t ka = (kk & 3) * 32;
      mma_ss_pair(tmem + dcol, smem_desc_sw128(q_base + (kk >> 2) * C::kBoxBytes + ka, 16, 1024),
                  smem_desc_sw128(k_base + (kk >> 2) * C::kKBoxBytes + ka, 16, 1024), kIdQK, kk > 0 ? 1u : 0u);
    }
    commit_both(&bars->slot_empty[slot]);
  }
  // O += P V over the 16-key slabs in `mask`; P hi / lo of chunk c at
  // pcol + 32 c + [0, 16) / [16, 32).  The first PV always issues a slab (it
  // initialises O).
  __device__ void pv_at(int slot, uint32_t pcol, uint32_t mask) {
    if (!ok) return;
    if (!o_started) mask |= 1u;
    if (mask == 0u) {  // no product reads the entry: release it (asynchronously) in both CTAs
      commit_both(&bars->slot_empty[slot]);
      return;
    }
    const uint32_t v_base = ring_base + slot * C::kHalfBytes;
    slabs += __popc(mask);
#pragma unroll
    for (int m = 0; m < kTile / 16; ++m) {
      if (!(mask & (1u << m))) continue;
      const uint64_t bdesc = smem_desc_sw128(v_base + m * 2048, C::kBoxBytes, 1024);
      const uint32_t a_hi = tmem + pcol + 32 * (m >> 1) + 8 * (m & 1);
      mma_ts_pair(tmem + C::kColO, a_hi, bdesc, kIdPV, o_started ? 1u : 0u);
      mma_ts_pair(tmem + C::kColO, a_hi + 16, bdesc, kIdPV, 1u);
      o_started = true;
    }
    commit_both(&bars->slot_empty[slot]);
  }
  // OR of both CTAs' warps' slab masks of key tile j
  __device__ uint32_t slab_mask(int j) const {
    const uint4* w = reinterpret_cast<const uint4*>(&bars->tile_mask[j % C::kSSlots][0][0]);
    const uint32_t tag = static_cast<uint32_t>(j + 1);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 x = w[i];
      m |= ((x.x >> 8) == tag ? x.x : 0u) | ((x.y >> 8) == tag ? x.y : 0u) | ((x.z >> 8) == tag ? x.z : 0u) |
           ((x.w >> 8) == tag ? x.w : 0u);
    }
    return m & 0xFFu;
  }
  __device__ void drain(uint64_t* bar) {
    tc_commit_pair(smem_u32(bar));
    drain_wait(bar, 0, ctl);
  }
};

// Leader warp 1: every PV (and, differential, QK1_{j+2} into P_j's slot right
// after PV_j: one thread's products run in order on the tensor pipe, so no
// wait for PV_j is needed); V_j's entry is acquired before the wait for P_j.
// (Issuing QK1 from the QK2 thread instead, after PV_j has completed, measured
// 12% slower: the wait for PV_j's completion delays S1 of tile j + 2.)
template <bool DIFF, bool F16>
__device__ void run_pair_mma(uint8_t* smem, PairBars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt,
                             unsigned long long* stats) {
  using C = PairCfg<DIFF>;
  PairIssuer<DIFF, F16> m(smem, bars, ctl, tmem);
  const uint32_t q1_base = smem_u32(smem);
  if constexpr (DIFF) {
    m.wait(&bars->q_full, 0, ST_PM_Q);
    m.wait_cl(&bars->q_pair, 0, ST_PM_Q);
    for (int t = 0; t < 2 && t < n_kt; ++t) {
      m.qk(pr_k1(t), C::col_s(t), q1_base);
      m.commit_both(&bars->s_full[t]);
    }
  }
  for (int j = 0; j < n_kt && m.ok; ++j) {
    const int slot = j % C::kSSlots;
    const int vslot = m.acquire(DIFF ? pr_v(j, n_kt) : pr_v_rect(j, n_kt));
    m.wait(&bars->p_full[slot], (j / C::kSSlots) & 1, ST_PM_P);
    m.pv_at(vslot, C::col_s(slot), m.slab_mask(j));
    if constexpr (DIFF) {
      if (j + 2 < n_kt) {
        m.qk(pr_k1(j + 2), C::col_s(slot), q1_base);
        m.commit_both(&bars->s_full[slot]);
      }
    } else {
      m.commit_own(&bars->pv_done[slot]);
    }
  }
  if (m.ok)
    m.commit_both(&bars->o_full);
  else
    m.drain(&bars->drain);
  if (stats) {  // a slab of the pair serves both CTAs' query tiles
    atomicAdd(stats, 2ull * m.slabs);
    atomicAdd(stats + 1, 2ull * n_kt * (kTile / 16));
  }
}

// Leader warp 10, rect: QK_{j+3} into P_j's slot once PV_j has run.
template <bool F16>
__device__ void run_pair_mma_qk(uint8_t* smem, PairBars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = PairCfg<false>;
  PairIssuer<false, F16> m(smem, bars, ctl, tmem);
  const uint32_t q1_base = smem_u32(smem);
  m.wait(&bars->q_full, 0, ST_PM_Q);
  m.wait_cl(&bars->q_pair, 0, ST_PM_Q);
  for (int t = 0; t < C::kSSlots && t < n_kt; ++t) {
    m.qk(t, C::col_s(t), q1_base);
    m.commit_both(&bars->s_full[t]);
  }
  for (int j = 0; j + C::kSSlots < n_kt && m.ok; ++j) {
    const int slot = j % C::kSSlots;
    const int kslot = m.acquire(pr_v_rect(j, n_kt) + 1);
    m.wait(&bars->pv_done[slot], (j / C::kSSlots) & 1, ST_PM_P);
    m.qk_at(kslot, C::col_s(slot), q1_base);
    m.commit_both(&bars->s_full[slot]);
  }
  if (!m.ok) m.drain(&bars->drain2);
}

// Leader warp 10, differential: S2 = Q2 K2^T into its single slot, free once
// every transform warp of both CTAs holds S2 of the previous tile.
template <bool F16>
__device__ void run_pair_mma_qk2(uint8_t* smem, PairBars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = PairCfg<true>;
  PairIssuer<true, F16> m(smem, bars, ctl, tmem);
  const uint32_t q2_base = smem_u32(smem) + C::kTileBytes;
  m.wait(&bars->q_full, 0, ST_PM_Q);
  m.wait_cl(&bars->q_pair, 0, ST_PM_Q);
  m.qk(pr_k2(0), C::kColS2, q2_base);
  m.commit_both(&bars->s_full[0]);
  for (int j = 0; j + 1 < n_kt && m.ok; ++j) {
    m.wait(&bars->s2_free[j & 1], (j >> 1) & 1, ST_PM_S2);
    m.qk(pr_k2(j + 1), C::kColS2, q2_base);
    m.commit_both(&bars->s_full[(j + 1) & 1]);
  }
  if (!m.ok) m.drain(&bars->drain2);
}

// ------------------------------------------------------------------ transform
// As the one-tile kernel's transform warps: warp w owns TMEM lane quarter
// w % 4 and, as warpgroup g = (w - 2) / 4, key chunks [2g, 2g + 2) of every
// tile and output columns [64g, 64g + 64).
template <bool DIFF, bool NORM, bool POS, int PM, bool F16>
__device__ void run_pair_transform(const TcFwdParams& p, uint8_t* smem, PairBars* bars, const WaitCtl& ctl,
                                   uint32_t tmem, int bh, int qt, int n_kt, int warp, int lane, uint32_t rank) {
  using C = PairCfg<DIFF>;
  constexpr bool kFold = PM != POW_GENERAL;
  constexpr int kChunks = 4 / C::kTWG;
  constexpr int kQChunks = 8 / C::kTWG;
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int q0 = qt * kTile;
  const int grow = q0 + row;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float* rk_s = reinterpret_cast<const float*>(smem + C::kOffRk);

  // tau(i) = beta * sqrt(2 * log(i + 1) / D) (triton_threshold_attention.py:62-63)
  const float tau = p.beta * sqrtf((2.0f * logf(static_cast<float>(grow + 1))) / static_cast<float>(C::D));
  float lam = p.lam, lam_root = p.lam_root;
  if (DIFF && p.lam_dev.ptr) {
    lam = lambda_of(p.lam_dev, bh, p.lam);
    lam_root = lambda_root<PM>(lam);
  }
  const float lam2 = (DIFF && kFold) ? lam_root : 1.0f;
  RowCoef c{tau, 1.0f, tau, lam2, lam};
  bool ok = true;
  if constexpr (NORM) {
    ok = mbar_wait_warp(&bars->q_full, 0, ctl, ST_PT_Q);
    // ||q_i||: the two warpgroups each sum half of every row's 16-B chunks
    // (the swizzle permutes chunks within a row only)
    float* qss = reinterpret_cast<float*>(smem + C::kOffQss);
    if (ok) {
#pragma unroll 1
      for (int t = 0; t < C::kNQ; ++t) {
        float ss = 0.0f;
#pragma unroll 1
        for (int bx = 0; bx < 2; ++bx) {
          const uint8_t* rb = smem + t * C::kTileBytes + bx * C::kBoxBytes + row * 128;
#pragma unroll
          for (int k = 0; k < kQChunks; ++k) {
            const int cc = kQChunks * wg + k;
            const uint4 u = *reinterpret_cast<const uint4*>(rb + ((cc ^ (row & 7)) << 4));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float2 x = F16 ? unpack_f16x2(w[h]) : unpack_bf16x2(w[h]);
              ss = fmaf(x.x, x.x, ss);
              ss = fmaf(x.y, x.y, ss);
            }
          }
        }
        qss[(t * C::kTWG + wg) * kTile + row] = ss;
      }
    }
    ok = named_barrier_and(1, 32 * C::kTW, ok);
    if (ok) {
      float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
      for (int g = 0; g < C::kTWG; ++g) {
        s1 += qss[g * kTile + row];
        if constexpr (DIFF) s2 += qss[(C::kTWG + g) * kTile + row];
      }
      const float m1 = fmaxf(sqrtf(s1), 1e-12f);
      c.rq1 = 1.0f / m1;
      c.tq1 = tau * m1;
      if constexpr (DIFF) {
        const float m2 = fmaxf(sqrtf(s2), 1e-12f);
        c.rq2 = lam2 / m2;
        c.tq2 = tau * m2;
      }
    }
  }

  const int tw = warp - 2;
  // A transform warp's per-tile signal to a leader barrier that counts the
  // leader's 8 warps as arrivals and the peer's 8 warps as 4-byte stores:
  // the leader's warp 0 also announces those 32 bytes.
  auto signal_leader = [&](uint64_t* bar, uint32_t* peer_word, uint32_t value) {
    if (rank == 0) {
      if (tw == 0)
        mbar_arrive_expect_tx(bar, 4 * C::kTW);
      else
        mbar_arrive(bar);
    } else {
      st_async_u32(leader_addr(peer_word), value, leader_addr(bar));
    }
  };
  for (int j = 0; j < n_kt && ok; ++j) {
    const int re = j % kPairRkRing;
    if constexpr (NORM) {
      ok = mbar_wait_warp(&bars->rk_full[re], (j / kPairRkRing) & 1, ctl, ST_PT_RK);
      if (!ok) break;
    }
    const int slot = j % C::kSSlots;
    ok = mbar_wait_warp(&bars->s_full[slot], (j / C::kSSlots) & 1, ctl, ST_PT_S);
    if (!ok) break;
    tc_fence_after();
    const uint32_t nz = transform_tile<PM, DIFF, NORM, POS, DIFF, false, F16, kChunks>(
        tmem + lane_off, C::col_s(slot), C::kColS2, wg, rk_s + re * C::kRkPerTile, grow - j * kTile, j >= qt, c,
        p.relu_power, c.lam, p.p_scale, [&] {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) signal_leader(&bars->s2_free[j & 1], &bars->s2_token[j & 1][tw], 1u);
        });
    // this warp's slab mask goes to the leader with its P-ready signal
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, nz) << (2 * kChunks * wg);
    const uint32_t word = (static_cast<uint32_t>(j + 1) << 8) | wmask;
    if (rank == 0 && lane == 0) bars->tile_mask[slot][0][tw] = word;
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      signal_leader(&bars->p_full[slot], &bars->tile_mask[slot][1][tw], word);
      if constexpr (NORM) mbar_arrive(&bars->rk_empty[re]);
    }
  }

  // epilogue: O -> bf16 (or f32) rows staged in the ring (idle once every
  // product of the pair has completed), then TMA stores of this CTA's rows
  if (ok) ok = mbar_wait_warp(&bars->o_full, 0, ctl, ST_PT_O);
  uint8_t* stage = smem + C::kOffRing;
  if (ok) {
    tc_fence_after();
    constexpr int kCols = C::D / C::kTWG;
    uint8_t* srow = stage + row * 128;
    const uint32_t sw = static_cast<uint32_t>(row & 7);
#pragma unroll
    for (int c0 = 0; c0 < kCols; c0 += 32) {
      const int col = wg * kCols + c0;
      uint32_t o[32];
      tmem_ld32(tmem + lane_off + C::kColO + col, o);
      tmem_wait_ld();
      if constexpr (F16) {
#pragma unroll
        for (int t = 0; t < 32; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * p.o_unscale);
      }
      if (p.out_f32) {
#pragma unroll
        for (int t = 0; t < 8; ++t) {
          const int cc = col + 4 * t;
          *reinterpret_cast<uint4*>(srow + (cc >> 5) * C::kBoxBytes + ((((cc & 31) >> 2) ^ sw) << 4)) =
              make_uint4(o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
        }
      } else {
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const int cc = col + 8 * t;
          uint32_t w[4];
#pragma unroll
          for (int h = 0; h < 4; ++h)
            w[h] = F16 ? pack_f16x2(__uint_as_float(o[8 * t + 2 * h]), __uint_as_float(o[8 * t + 2 * h + 1]))
                       : pack_bf16x2(__uint_as_float(o[8 * t + 2 * h]), __uint_as_float(o[8 * t + 2 * h + 1]));
          *reinterpret_cast<uint4*>(srow + (cc >> 6) * C::kBoxBytes + ((((cc & 63) >> 3) ^ sw) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    fence_proxy_async_smem();
  }
  ok = named_barrier_and(2, 32 * C::kTW, ok);
  // the odd CTA of a pair past the last query tile has no rows to write
  if (ok && warp == 2 && lane == 0 && q0 < p.S) {
    const int n_boxes = p.out_f32 ? C::D / 32 : C::D / 64;
    const int box_cols = p.out_f32 ? 32 : 64;
    for (int b = 0; b < n_boxes; ++b) tma_store_3d(&p.tm_out, stage + b * C::kBoxBytes, b * box_cols, q0, bh);
    bulk_commit_group();
    bulk_wait_group_read0();
  }
}

template <bool DIFF, bool NORM, bool POS, int PM, bool F16>
__global__ void __cluster_dims__(2, 1, 1) __maxnreg__(168)
    tda_tc_fwd_pair_kernel(const __grid_constant__ TcFwdParams p) {
  using C = PairCfg<DIFF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PairBars* bars = reinterpret_cast<PairBars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();

  // Launch order: clusters take pairs of query tiles, in groups of
  // kPairHeadGroup (batch, head) slices, longest pairs first with the
  // group's heads interleaved (as the one-tile kernel orders its tiles).
  const int n_pairs = (p.n_qtiles + 1) >> 1;
  const int cid = static_cast<int>(blockIdx.x >> 1);
  const int per_group = kPairHeadGroup * n_pairs;
  const int g0 = (cid / per_group) * kPairHeadGroup;
  const int gsz = min(kPairHeadGroup, p.BH - g0);
  const int r = cid % per_group;
  const int bh = g0 + r % gsz;
  const int pair = n_pairs - 1 - r / gsz;
  const int qt = 2 * pair + static_cast<int>(rank);
  const int n_kt = p.causal_skip ? min(2 * pair + 2, p.n_qtiles) : p.n_qtiles;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->q_pair, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->drain2, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->s_full[i], DIFF ? 2 : 1);
      mbar_init(&bars->p_full[i], C::kTW);
      mbar_init(&bars->pv_done[i], 1);
      for (int c = 0; c < 2; ++c)
        for (int w = 0; w < 8; ++w) bars->tile_mask[i][c][w] = 0;
    }
    for (int i = 0; i < 2; ++i) mbar_init(&bars->s2_free[i], C::kTW);
    for (int i = 0; i < kPairRkRing; ++i) {
      mbar_init(&bars->rk_full[i], 1);
      mbar_init(&bars->rk_empty[i], C::kTW);
    }
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    pair_first_loads<DIFF, NORM>(p, smem, bars, bh, qt);
    tma_prefetch_desc(&p.tm_v);
    tma_prefetch_desc(&p.tm_k1h);
    if constexpr (DIFF) tma_prefetch_desc(&p.tm_k2h);
  }
  if (warp == 1) {
    tmem_alloc_pair(&bars->tmem_base, 512);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  // both CTAs' barriers are initialised before any copy, arrival or commit
  // crosses to the other CTA
  cluster_sync();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const WaitCtl ctl = make_wait_ctl(&bars->abort_flag, p.status, p.timeout_ns);

  if (warp == 0) {
    if (lane == 0) pair_producer<DIFF, NORM>(p, smem, bars, ctl, bh, n_kt, rank);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      if (rank == 0) {
        run_pair_mma<DIFF, F16>(smem, bars, ctl, tmem, n_kt, p.stats);
      } else if (!(p.inject & 1)) {
        // the leader's products read this CTA's query tile(s) too
        if (mbar_wait(&bars->q_full, 0, ctl, ST_PM_Q)) mbar_arrive_cluster(leader_addr(&bars->q_pair));
      }
    }
    __syncwarp();
  } else if (warp < C::kQk2W) {
    run_pair_transform<DIFF, NORM, POS, PM, F16>(p, smem, bars, ctl, tmem, bh, qt, n_kt, warp, lane, rank);
  } else {
    if (lane == 0 && rank == 0) {
      if constexpr (DIFF)
        run_pair_mma_qk2<F16>(smem, bars, ctl, tmem, n_kt);
      else
        run_pair_mma_qk<F16>(smem, bars, ctl, tmem, n_kt);
    }
    __syncwarp();
  }

  tc_fence_before();
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, 512);
  }
}

template <bool DIFF, bool NORM, bool POS, int PM, bool F16>
cudaError_t launch_pair(const TcFwdParams& p, cudaStream_t stream) {
  using C = PairCfg<DIFF>;
  auto kern = tda_tc_fwd_pair_kernel<DIFF, NORM, POS, PM, F16>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const unsigned n_pairs = static_cast<unsigned>((p.n_qtiles + 1) / 2);
  const unsigned grid = 2u * static_cast<unsigned>(p.BH) * n_pairs;
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

template <bool DIFF, bool NORM, bool POS, bool F16>
cudaError_t pair_pow(const TcFwdParams& p, int pm, cudaStream_t s) {
  switch (pm) {
    case POW_1: return launch_pair<DIFF, NORM, POS, POW_1, F16>(p, s);
    case POW_2: return launch_pair<DIFF, NORM, POS, POW_2, F16>(p, s);
    case POW_3: return launch_pair<DIFF, NORM, POS, POW_3, F16>(p, s);
    default: return launch_pair<DIFF, NORM, POS, POW_GENERAL, F16>(p, s);
  }
}

template <bool DIFF>
cudaError_t pair_norm(const TcFwdParams& p, bool norm, int pm, bool fp16, cudaStream_t s) {
  if (fp16) {
    if (!norm) return cudaErrorInvalidValue;
    return p.causal_skip ? pair_pow<DIFF, true, true, true>(p, pm, s) : pair_pow<DIFF, true, false, true>(p, pm, s);
  }
  if (norm) return p.causal_skip ? pair_pow<DIFF, true, true, false>(p, pm, s) : pair_pow<DIFF, true, false, false>(p, pm, s);
  return p.causal_skip ? pair_pow<DIFF, false, true, false>(p, pm, s) : pair_pow<DIFF, false, false, false>(p, pm, s);
}

}  // namespace

cudaError_t launch_tc_fwd_pair(const TcFwdParams& p, bool differential, bool normalize, int pow_mode, bool fp16,
                               cudaStream_t stream) {
  return differential ? pair_norm<true>(p, normalize, pow_mode, fp16, stream)
                      : pair_norm<false>(p, normalize, pow_mode, fp16, stream);
}

}  // namespace tda
