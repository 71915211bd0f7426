// Tensor-core (tcgen05 + TMEM + TMA) forward of threshold rectified attention
// and its differential form, bf16 storage, fp32 accumulation.
//
// Math (triton_threshold_attention.py:19-115 and :489-519):
//   s_ij  = q_i . k_j                       (raw bf16 operands, f32 accumulate)
//   s_ij  = 0 for j > i                     (causal mask to zero, :79-80)
//   z_ij  = s_ij * rk_j * rq_i - tau_i      (normalize: rq, rk = 1/max(||.||,1e-12))
//         = s_ij - tau_i                    (no normalize)
//   P_ij  = relu(z_ij)^p                    (:85-101)
//   diff: P_ij = P1_ij - lambda * P2_ij     (:512-517, one PV on the combined P)
//   out_i = sum_j P_ij v_j
//
// One CTA computes one 128-row query tile of one (batch, head):
//   warp 0      TMA producer: Q tile(s) once, then a ring of K/V tiles in the
//               exact order the MMA warp consumes them, plus the per-key
//               inverse norms into a small ring.
//   warp 1      MMA issuer (one thread): S = Q K^T (S1 = Q1 K1^T) into TMEM
//               (SS form), and O += P V with P read from TMEM (TS form).
//   warps 2-9   two transform warpgroups; each thread owns one query row
//               (its TMEM lane), warpgroup g handles key columns [64g, 64g+64)
//               of every tile: S -> threshold -> ReLU^p (-> combine) ->
//               bf16 hi + bf16 lo split of P written back over S in TMEM.
//               They also run the epilogue (O from TMEM -> global).
//   warp 10     differential form only: second MMA issuer for S2 = Q2 K2^T.
//               An issuing thread blocks while the tensor pipe's queue is
//               full, so one issuer for everything would see the S2 slot
//               freed only after its PV and QK1 products went in, and the
//               pipe would idle in between.
//
// P precision: P is stored as bf16 hi + bf16 lo (P = hi + lo to ~16 bits) and
// multiplied into O by two MMAs; a single bf16 P misses the 1e-3 accuracy gate.
//
// Every mbarrier wait is bounded (WaitCtl): on timeout the CTA records a code
// in the status word, drains its in-flight copies / MMAs, frees TMEM and exits.
#include <cuda_bf16.h>

#include <atomic>
#include <cstdio>
#include <cstdlib>

#include "tda_internal.h"
#include "tda_ptx.cuh"
#include "tda_transform.cuh"

namespace tda {
namespace {

using namespace tc;

// Persistent kernel: two transform warpgroups (warps 2 .. 9), each thread two
// 32-key chunks of every key tile; warp 10 issues the QK products (rect) or
// the QK2 products (differential), warp 1 the PV (and QK1) products.
constexpr int kTransformWG = 2;
constexpr int kTransformWarps = 4 * kTransformWG;
constexpr int kQk2Warp = 2 + kTransformWarps;
template <bool DIFF>
constexpr int threads_for() { return 32 * (3 + kTransformWarps); }
constexpr int kRkRing = 4;
constexpr int kHeadGroup = 2;  // (batch, head) slices interleaved in launch order
// Transform code layout (instruction-cache footprint versus register moves),
// chosen per form by measurement: the differential transform is twice the
// code and runs from one rolled chunk loop (the kernel was instruction-fetch
// bound with both chunks unrolled); the rectified one stays unrolled.
template <bool DIFF>
constexpr bool kRollChunks = DIFF;
template <bool DIFF>
constexpr bool kRollHalves = false;
constexpr int kSmemBudget = 232448;  // 227 KB opt-in dynamic shared memory

// status codes (role << 8 | site)
constexpr int ST_PROD_SLOT = 0x101, ST_PROD_RK = 0x102;
constexpr int ST_MMA_Q = 0x201, ST_MMA_SLOT = 0x202, ST_MMA_P = 0x203, ST_MMA_S2 = 0x204;
constexpr int ST_TR_Q = 0x301, ST_TR_RK = 0x302, ST_TR_S = 0x303, ST_TR_O = 0x304;

// One-CTA-per-tile kernel: two transform warpgroups (warps 2 .. 9), each
// thread two 32-key chunks of every key tile.  The MMAs come from two
// single-thread issuers so that one issuer's waits and commits (each some
// 100-200 cycles of latency on a single thread) overlap the other's MMAs:
// warp 1 issues every PV (and QK1 for the differential form), warp 10 the QK
// products (rect) or QK2 (differential).  Two transform warpgroups, two
// 32-key chunks per thread.  Four (one chunk per thread, 608 threads, 96
// registers; kTWG = 4 is supported and bit-identical) measured, A/B on one
// box: rect +3.5% at (4,32,2048,128), +1.8% at (4,32,4096,128), equal at
// (8,32,8192,128), but -3.6% with dense P (beta = 0) there; differential -8%.
template <int D, bool DIFF>
struct Cfg {
  static constexpr int kTWG = 2;                 // transform warpgroups
  static constexpr int kSumWG = 2;               // warpgroups summing the query norms
  static constexpr int kTW = 4 * kTWG;           // transform warps 2 .. 1 + kTW
  static constexpr int kQk2W = 2 + kTW;          // QK issuer (rect) / QK2 issuer (differential)
  static constexpr int kThreads = 32 * (3 + kTW);
  static constexpr int kMaxRegs = kTWG == 2 ? 168 : 96;  // per-thread register cap of the launch
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = kTile * 128;  // 128 rows x 64 bf16 (128 B)
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr int kNQ = DIFF ? 2 : 1;
  static constexpr int kRkPerTile = (DIFF ? 2 : 1) * (kTile + 8);  // rk then per-16-key maxima
  static constexpr int kRkFloats = kRkRing * kRkPerTile;
  static constexpr int kBarBytes = 1024;
  static constexpr int kQssBytes = kNQ * kSumWG * kTile * 4;  // partial sums of ||q||^2
  static constexpr int kFixed = kNQ * kTileBytes + kRkFloats * 4 + kBarBytes + kQssBytes + 1024;
  static constexpr int kSlotsRaw = (kSmemBudget - kFixed) / kTileBytes;
  static constexpr int kSlots = kSlotsRaw > 8 ? 8 : kSlotsRaw;
  static_assert(kSlots >= 3, "not enough shared memory for the K/V ring");
  static constexpr int kOffRing = kNQ * kTileBytes;
  static constexpr int kOffRk = kOffRing + kSlots * kTileBytes;
  static constexpr int kOffBar = kOffRk + kRkFloats * 4;
  static constexpr int kOffQss = kOffBar + kBarBytes;
  static constexpr int kSmemBytes = kOffQss + kQssBytes + 1024;
  // TMEM columns (512 allocated): rect S slots {0,128,256}, O at 384;
  // diff S1 slots {0,256}, S2 slot 128, O at 384.
  static constexpr int kSSlots = DIFF ? 2 : 3;
  static constexpr int kColS2 = 128;
  static constexpr int kColO = 384;
  static __device__ __forceinline__ uint32_t col_s(int slot) {
    return DIFF ? (slot ? 256u : 0u) : static_cast<uint32_t>(slot * 128);
  }
};

struct Bars {
  uint64_t q_full;
  uint64_t o_full;
  uint64_t drain;       // warp 1's own MMAs (abort)
  uint64_t drain2;      // the QK (rect) / QK2 (differential) issuer's own MMAs
  uint64_t s_full[3];   // per S slot; differential: one arrival per QK issuer
  uint64_t p_full[3];
  uint64_t pv_done[3];  // rect, per S slot: the PV reading P from it has run
  uint64_t s2_free[2];  // differential: every transform warp has read S2 of the tile
  uint64_t rk_full[kRkRing];
  uint64_t rk_empty[kRkRing];
  uint64_t slot_full[8];
  uint64_t slot_empty[8];
  uint32_t tmem_base;
  int abort_flag;
  // per S slot: (j + 1) << 8 | mask of 16-key slabs of key tile j with a
  // nonzero P; stale words carry an older tag and read as mask 0
  uint32_t tile_mask[3];
};
static_assert(sizeof(Bars) <= 1024, "barrier block too large");

// ------------------------------------------------------------------ producer
// The first copies of a CTA: the query tile(s), key tile 0 (K1_0 and K2_0
// for the differential form) into ring slots 0 (and 1), and key-table entry
// 0.  Issued by the thread that initialised the barriers, before the CTA-wide
// barrier, so their latency overlaps the TMEM allocation and the start-up of
// the other warps; every barrier they use is fresh, so nothing waits.
template <int D, bool DIFF, bool NORM>
__device__ void issue_first_loads(const TcFwdParams& p, uint8_t* smem, Bars* bars, int bh, int qt) {
  using C = Cfg<D, DIFF>;
  const int h_idx = bh % p.heads, b_idx = bh / p.heads;  // tensor-map coordinates of this (batch, head)
  if (!(p.inject & 1)) {
    mbar_arrive_expect_tx(&bars->q_full, C::kNQ * C::kTileBytes);
#pragma unroll
    for (int b = 0; b < C::kBoxes; ++b) {
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
  constexpr int kFirst = DIFF ? 2 : 1;
#pragma unroll
  for (int t = 0; t < kFirst; ++t) {
    const CUtensorMap* map = t == 0 ? &p.tm_k1 : &p.tm_k2;
    mbar_arrive_expect_tx(&bars->slot_full[t], C::kTileBytes);
    uint8_t* dst = smem + C::kOffRing + t * C::kTileBytes;
#pragma unroll
    for (int b = 0; b < C::kBoxes; ++b)
      tma_load_4d(dst + b * C::kBoxBytes, map, &bars->slot_full[t], b * 64, 0, h_idx, b_idx);
  }
}

// Every later copy, in consumption order, after issue_first_loads.
template <int D, bool DIFF, bool NORM>
__device__ void run_producer(const TcFwdParams& p, uint8_t* smem, Bars* bars, const WaitCtl& ctl, int bh, int qt,
                             int n_kt) {
  using C = Cfg<D, DIFF>;
  uint8_t* ring = smem + C::kOffRing;
  float* rk_s = reinterpret_cast<float*>(smem + C::kOffRk);
  const int h_idx = bh % p.heads, b_idx = bh / p.heads;  // tensor-map coordinates of this (batch, head)
  const bool q_issued = !(p.inject & 1);

  int ridx = DIFF ? 2 : 1;    // tiles issued into the ring (key tile 0 by issue_first_loads)
  int rk_n = NORM ? 1 : 0;    // rk ring entries issued
  bool ok = true;
  auto load_tile = [&](const CUtensorMap* map, int j) {
    if (!ok) return;
    const int slot = ridx % C::kSlots;
    const uint32_t par = ((ridx / C::kSlots) & 1) ^ 1;
    if (!mbar_wait(&bars->slot_empty[slot], par, ctl, ST_PROD_SLOT)) {
      ok = false;
      return;
    }
    mbar_arrive_expect_tx(&bars->slot_full[slot], C::kTileBytes);
    uint8_t* dst = ring + slot * C::kTileBytes;
#pragma unroll
    for (int b = 0; b < C::kBoxes; ++b)
      tma_load_4d(dst + b * C::kBoxBytes, map, &bars->slot_full[slot], b * 64, j * kTile, h_idx, b_idx);
    ++ridx;
  };
  auto load_rk = [&](int j) {
    if constexpr (NORM) {
      if (!ok) return;
      const int e = j % kRkRing;
      const uint32_t par = ((j / kRkRing) & 1) ^ 1;
      if (!mbar_wait(&bars->rk_empty[e], par, ctl, ST_PROD_RK)) {
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
    // consumption order: K0, K1, K2, then per j: V_j, K_{j+3}
    for (int j = 1; j < 3 && j < n_kt; ++j) {
      load_rk(j);
      load_tile(&p.tm_k1, j);
    }
    for (int j = 0; j < n_kt && ok; ++j) {
      load_tile(&p.tm_v, j);
      if (j + 3 < n_kt) {
        load_rk(j + 3);
        load_tile(&p.tm_k1, j + 3);
      }
    }
  } else {
    // consumption order: K1_0, K2_0, K1_1, then per j: K2_{j+1}, V_j, K1_{j+2}
    if (n_kt > 1) {
      load_rk(1);
      load_tile(&p.tm_k1, 1);
    }
    for (int j = 0; j < n_kt && ok; ++j) {
      if (j + 1 < n_kt) load_tile(&p.tm_k2, j + 1);
      load_tile(&p.tm_v, j);
      if (j + 2 < n_kt) {
        load_rk(j + 2);
        load_tile(&p.tm_k1, j + 2);
      }
    }
  }

  if (!ok) {
    // Abort: wait for the copies this thread issued and that may still be in
    // flight (the newest load of each ring slot / rk entry, and Q).
    if (q_issued) drain_wait(&bars->q_full, 0, ctl);
    const int first = ridx > C::kSlots ? ridx - C::kSlots : 0;
    for (int i = first; i < ridx; ++i) drain_wait(&bars->slot_full[i % C::kSlots], (i / C::kSlots) & 1, ctl);
    const int rfirst = rk_n > kRkRing ? rk_n - kRkRing : 0;
    for (int i = rfirst; i < rk_n; ++i) drain_wait(&bars->rk_full[i % kRkRing], (i / kRkRing) & 1, ctl);
  }
}

// ------------------------------------------------------------------ MMA issuers
// Position of a tile in the producer's ring order (differential form):
//   K1_0, K2_0, K1_1, then per key tile j: K2_{j+1}, V_j, K1_{j+2}
// (entries past the last tile are not loaded).
__device__ __forceinline__ int ring_k1(int m) { return m == 0 ? 0 : (m == 1 ? 2 : 3 * m - 1); }
__device__ __forceinline__ int ring_k2(int m) { return m == 0 ? 1 : 3 * m; }
__device__ __forceinline__ int ring_v(int j, int n_kt) { return j <= n_kt - 2 ? 4 + 3 * j : 3 * n_kt - 1; }

// C: shared-memory layout (ring, box and tile sizes, TMEM columns); B: the
// barrier block (slot_full / slot_empty / tile_mask) of the kernel using it.
template <int D, bool DIFF, class C = Cfg<D, DIFF>, class B = Bars, bool F16 = false>
struct MmaIssuer {
  // kind::f16 instruction descriptors: bf16 or fp16 operands, f32 accumulation
  static constexpr uint32_t kIdQK = idesc_f16(128, 128, !F16, false);
  static constexpr uint32_t kIdPV = idesc_f16(128, D, !F16, true);
  B* bars;
  const WaitCtl& ctl;
  uint32_t tmem;
  uint32_t ring_base;
  bool ok;
  bool o_started;
  unsigned slabs = 0;  // 16-key slabs multiplied by pv (diagnostics)

  __device__ MmaIssuer(uint8_t* smem, B* b, const WaitCtl& c, uint32_t t)
      : bars(b), ctl(c), tmem(t), ring_base(smem_u32(smem + C::kOffRing)), ok(true), o_started(false) {}

  // wait for ring entry `idx` to land; returns its slot
  __device__ int acquire(int idx) {
    const int slot = idx % C::kSlots;
    if (!ok) return slot;
    ok = mbar_wait(&bars->slot_full[slot], (idx / C::kSlots) & 1, ctl, ST_MMA_SLOT);
    tc_fence_after();
    return slot;
  }
  // S[dcol] = Q K^T over D in UMMA_K = 16 steps (32 B inside a 128-B swizzled row)
  __device__ void qk(int idx, uint32_t dcol, uint32_t q_base) { qk_at(acquire(idx), dcol, q_base); }
  // the same with K already in ring slot `slot` (acquired)
  __device__ void qk_at(int slot, uint32_t dcol, uint32_t q_base) {
    if (!ok) return;
    const uint32_t k_base = ring_base + slot * C::kTileBytes;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * C::kBoxBytes + (kk & 3) * 32;
      mma_ss(tmem + dcol, smem_desc_sw128(q_base + off, 16, 1024), smem_desc_sw128(k_base + off, 16, 1024),
             kIdQK, kk > 0 ? 1u : 0u);
    }
    tc_commit(&bars->slot_empty[slot]);
  }
  // O += P V, P (hi, lo) in TMEM columns [pcol, pcol+128): for key chunk c of
  // 32 keys, hi at pcol + 32c + [0,16), lo at pcol + 32c + [16,32).  Only the
  // 16-key slabs set in `mask` are multiplied (the others hold P = 0); the
  // first PV of the CTA initialises O (accumulate = 0) and therefore always
  // issues at least its first slab.
  __device__ void pv(int idx, uint32_t pcol, uint32_t mask) { pv_at(acquire(idx), pcol, mask); }
  // the same with V already in ring slot `slot` (acquired)
  __device__ void pv_at(int slot, uint32_t pcol, uint32_t mask) {
    if (!ok) return;
    if (!o_started) mask |= 1u;
    if (mask == 0u) {
      mbar_arrive(&bars->slot_empty[slot]);
      return;
    }
    const uint32_t v_base = ring_base + slot * C::kTileBytes;
    slabs += __popc(mask);
#pragma unroll
    for (int m = 0; m < kTile / 16; ++m) {
      if (!(mask & (1u << m))) continue;
      const uint64_t bdesc = smem_desc_sw128(v_base + m * 2048, C::kBoxBytes, 1024);
      const uint32_t a_hi = tmem + pcol + 32 * (m >> 1) + 8 * (m & 1);
      mma_ts(tmem + C::kColO, a_hi, bdesc, kIdPV, o_started ? 1u : 0u);
      mma_ts(tmem + C::kColO, a_hi + 16, bdesc, kIdPV, 1u);
      o_started = true;
    }
    tc_commit(&bars->slot_empty[slot]);
  }
  __device__ uint32_t slab_mask(int j) const {
    const uint32_t w = *reinterpret_cast<volatile uint32_t*>(&bars->tile_mask[j % C::kSSlots]);
    return (w >> 8) == static_cast<uint32_t>(j + 1) ? (w & 0xFFu) : 0u;
  }
  __device__ void wait(uint64_t* bar, uint32_t parity, int code) {
    if (!ok) return;
    ok = mbar_wait(bar, parity, ctl, code);
    tc_fence_after();
  }
  __device__ void commit(uint64_t* bar) {
    if (ok) tc_commit(bar);
  }
  // Abort: let every MMA this thread issued finish before TMEM is freed.
  __device__ void drain(uint64_t* bar) {
    tc_commit(bar);
    drain_wait(bar, 0, ctl);
  }
};

// Ring position of V_j in the rectified form's load order K0, K1, K2, then per
// key tile j: V_j, K_{j+3} (K_{j+3} only while j + 3 < n_kt).
__device__ __forceinline__ int ring_v_rect(int j, int n_kt) {
  const int ahead = n_kt > 3 ? n_kt - 3 : 0;
  return (n_kt < 3 ? n_kt : 3) + j + (j < ahead ? j : ahead);
}

// PV issuer (warp 1): every O += P V, with V_j's ring slot acquired before
// the wait for P_j (V_j is loaded well ahead, and the data does not depend
// on P, so this takes the acquire off the path from P_j to PV_j).
//   rect: after PV_j it commits pv_done of P_j's S slot (arrives once PV_j
//     has run), which hands the slot to the QK issuer (warp 10).
//   differential: the same thread also issues QK1_{j+2} into P_j's slot right
//     after PV_j (the tensor pipe runs one thread's MMAs in order, so no wait
//     for PV_j is needed).  Its K1 tile is acquired only after PV_j: with four
//     32 KB ring slots for three tiles per key step the K1 load is often
//     still in flight, and waiting for it first would hold PV_j back.
template <int D, bool DIFF, bool F16>
__device__ void run_mma(uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt,
                        unsigned long long* stats) {
  using C = Cfg<D, DIFF>;
  MmaIssuer<D, DIFF, C, Bars, F16> m(smem, bars, ctl, tmem);
  const uint32_t q1_base = smem_u32(smem);
  if constexpr (DIFF) {
    m.wait(&bars->q_full, 0, ST_MMA_Q);
    for (int t = 0; t < 2 && t < n_kt; ++t) {
      m.qk(ring_k1(t), C::col_s(t), q1_base);
      m.commit(&bars->s_full[t]);
    }
  }
  for (int j = 0; j < n_kt && m.ok; ++j) {
    const int slot = j % C::kSSlots;
    const int vslot = m.acquire(DIFF ? ring_v(j, n_kt) : ring_v_rect(j, n_kt));
    m.wait(&bars->p_full[slot], (j / C::kSSlots) & 1, ST_MMA_P);
    m.pv_at(vslot, C::col_s(slot), m.slab_mask(j));
    if constexpr (DIFF) {
      if (j + 2 < n_kt) {
        m.qk(ring_k1(j + 2), C::col_s(slot), q1_base);
        m.commit(&bars->s_full[slot]);
      }
    } else {
      m.commit(&bars->pv_done[slot]);
    }
  }
  if (m.ok)
    tc_commit(&bars->o_full);
  else
    m.drain(&bars->drain);
  if (stats) {
    atomicAdd(stats, static_cast<unsigned long long>(m.slabs));
    atomicAdd(stats + 1, static_cast<unsigned long long>(n_kt) * (kTile / 16));
  }
}

// QK issuer of the rectified form (warp 10).  The first three products go
// into free S slots; QK_{j+3} waits until PV_j, which reads P_j from the same
// slot, has run (pv_done), its K slot acquired before that wait.
template <int D, bool F16>
__device__ void run_mma_qk(uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = Cfg<D, false>;
  MmaIssuer<D, false, C, Bars, F16> m(smem, bars, ctl, tmem);
  const uint32_t q1_base = smem_u32(smem);
  m.wait(&bars->q_full, 0, ST_MMA_Q);
  for (int t = 0; t < C::kSSlots && t < n_kt; ++t) {
    m.qk(t, C::col_s(t), q1_base);
    m.commit(&bars->s_full[t]);
  }
  for (int j = 0; j + C::kSSlots < n_kt && m.ok; ++j) {
    const int slot = j % C::kSSlots;
    const int kslot = m.acquire(ring_v_rect(j, n_kt) + 1);
    m.wait(&bars->pv_done[slot], (j / C::kSSlots) & 1, ST_MMA_P);
    m.qk_at(kslot, C::col_s(slot), q1_base);
    m.commit(&bars->s_full[slot]);
  }
  if (!m.ok) m.drain(&bars->drain2);
}

// Second issuer of the differential form (warp 10): S2 = Q2 K2^T into its
// single TMEM slot.  The slot is free once every transform warp holds S2_j in
// registers (s2_free), which happens long before P_j is ready; a separate
// thread issues these products so that the main issuer, blocked while the
// tensor pipe accepts its PV and QK1 products, does not delay them.
template <int D, bool F16>
__device__ void run_mma_qk2(uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = Cfg<D, true>;
  MmaIssuer<D, true, C, Bars, F16> m(smem, bars, ctl, tmem);
  const uint32_t q2_base = smem_u32(smem) + C::kTileBytes;
  m.wait(&bars->q_full, 0, ST_MMA_Q);
  m.qk(ring_k2(0), C::kColS2, q2_base);
  m.commit(&bars->s_full[0]);
  for (int j = 0; j + 1 < n_kt && m.ok; ++j) {
    m.wait(&bars->s2_free[j & 1], (j >> 1) & 1, ST_MMA_S2);
    m.qk(ring_k2(j + 1), C::kColS2, q2_base);
    m.commit(&bars->s_full[(j + 1) & 1]);
  }
  if (!m.ok) m.drain(&bars->drain2);
}

// Transform warps: warp w (2 <= w < 2 + C::kTW) owns TMEM lane quarter w % 4
// (query rows) and, as warpgroup g = (w - 2) / 4, the key chunks
// [g kChunks, (g+1) kChunks) of every key tile (32 keys each) and the output
// columns [g D/kTWG, (g+1) D/kTWG).
template <int D, bool DIFF, bool NORM, bool POS, int PM, bool F16>
__device__ void run_transform(const TcFwdParams& p, uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem,
                              int bh, int qt, int n_kt, int warp, int lane) {
  using C = Cfg<D, DIFF>;
  constexpr bool kFold = PM != POW_GENERAL;
  constexpr int kChunks = 4 / C::kTWG;  // 32-key chunks per thread per tile
  constexpr int kQChunks = 8 / C::kSumWG;  // 16-B chunks of each 128-B query row a summing warpgroup sums
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int q0 = qt * kTile;
  const int grow = q0 + row;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float* rk_s = reinterpret_cast<const float*>(smem + C::kOffRk);

  // tau(i) = beta * sqrt(2 * log(i + 1) / D) in fp32 (triton_threshold_attention.py:62-63)
  const float tau = p.beta * sqrtf((2.0f * logf(static_cast<float>(grow + 1))) / static_cast<float>(D));
  float lam = p.lam, lam_root = p.lam_root;
  if (DIFF && p.lam_dev.ptr) {  // lambda of this (batch, head) from the device
    lam = lambda_of(p.lam_dev, bh, p.lam);
    lam_root = lambda_root<PM>(lam);
  }
  const float lam2 = (DIFF && kFold) ? lam_root : 1.0f;
  RowCoef c{tau, 1.0f, tau, lam2, lam};
  bool ok = true;
  if constexpr (NORM) {
    ok = mbar_wait_warp(&bars->q_full, 0, ctl, ST_TR_Q);
    // ||q_i|| from the swizzled tile(s): row r's 16-B chunks are permuted
    // within the row only, so summing chunks needs no unswizzle.  Warpgroups
    // 0 and 1 (which own the same rows) each sum half of every row's chunks
    // and exchange the partial sums through shared memory -- with four
    // warpgroups too, so that the norms (and every result) are bit-identical
    // to the two-warpgroup kernels.  A rolled loop keeps this once-per-CTA
    // code small in the instruction cache.
    float* qss = reinterpret_cast<float*>(smem + C::kOffQss);  // [kNQ][kSumWG][kTile]
    if (ok && wg < C::kSumWG) {
#pragma unroll 1
      for (int t = 0; t < C::kNQ; ++t) {
        float ss = 0.0f;
#pragma unroll 1
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          const uint8_t* rb = smem + t * C::kTileBytes + bx * C::kBoxBytes + row * 128;
#pragma unroll
          for (int k = 0; k < kQChunks; ++k) {
            // logical chunk cc sits at (cc ^ (row & 7)): for one cc the 8 rows of
            // each group of 8 lanes hit 8 different 16-B bank groups
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
        qss[(t * C::kSumWG + wg) * kTile + row] = ss;
      }
    }
    // every transform thread arrives, also one whose wait gave up
    ok = named_barrier_and(1, 32 * C::kTW, ok);
    if (ok) {
      float s1 = 0.0f, s2 = 0.0f;
#pragma unroll
      for (int g = 0; g < C::kSumWG; ++g) {
        s1 += qss[g * kTile + row];
        if constexpr (DIFF) s2 += qss[(C::kSumWG + g) * kTile + row];
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

  for (int j = 0; j < n_kt && ok; ++j) {
    const int re = j % kRkRing;
    if constexpr (NORM) {
      ok = mbar_wait_warp(&bars->rk_full[re], (j / kRkRing) & 1, ctl, ST_TR_RK);
      if (!ok) break;
    }
    const int slot = j % C::kSSlots;
    const uint32_t sphase = (j / C::kSSlots) & 1;
    ok = mbar_wait_warp(&bars->s_full[slot], sphase, ctl, ST_TR_S);
    if (!ok) break;
    tc_fence_after();
    const uint32_t s1col = C::col_s(slot);
    const uint32_t nz = transform_tile<PM, DIFF, NORM, POS, kRollChunks<DIFF>, kRollHalves<DIFF>, F16, kChunks>(
        tmem + lane_off, s1col, C::kColS2, wg, rk_s + re * C::kRkPerTile, grow - j * kTile, j >= qt, c,
        p.relu_power, c.lam, p.p_scale, [&] {
          // S2 is in registers: hand its TMEM slot back so QK2 of the next
          // tile runs on the tensor cores while this tile is transformed
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->s2_free[j & 1]);
        });
    // publish which 16-key slabs of this tile hold a nonzero P (this
    // warpgroup owns slabs [2 kChunks wg, 2 kChunks (wg + 1))); slabs nobody
    // marks are skipped by the PV.  The p_full arrive below orders the store
    // before the MMA warp reads the word.
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, nz) << (2 * kChunks * wg);
    if (wmask != 0u && lane == 0) {
      uint32_t* word = &bars->tile_mask[slot];
      const uint32_t tag = static_cast<uint32_t>(j + 1) << 8;
      uint32_t old = *reinterpret_cast<volatile uint32_t*>(word), assumed;
      do {
        assumed = old;
        const uint32_t base = (assumed & ~0xFFu) == tag ? assumed : tag;
        old = atomicCAS(word, assumed, base | wmask);
      } while (old != assumed);
    }
    // every lane's TMEM stores are complete (wait::st) and ordered before the
    // warp sync; one arrival per warp then publishes the whole warp's P
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&bars->p_full[slot]);
      if constexpr (NORM) mbar_arrive(&bars->rk_empty[re]);
    }
  }

  // epilogue: O (f32 in TMEM) -> bf16 (or f32) rows staged in the K/V ring,
  // idle once every product has completed, in the 128-B swizzled layout of
  // the output tensor map; then one TMA store per 128-byte column box.  The
  // stores are coalesced (one thread per row would write 32 rows per warp
  // instruction) and TMA clips rows past S.  Every transform thread reaches
  // the barrier, also one whose wait gave up.
  if (ok) ok = mbar_wait_warp(&bars->o_full, 0, ctl, ST_TR_O);
  uint8_t* stage = smem + C::kOffRing;
  if (ok) {
    tc_fence_after();
    constexpr int kCols = D / C::kTWG;                 // output columns of this warpgroup
    constexpr int kPiece = kCols < 32 ? kCols : 32;    // columns per TMEM load
    static_assert(kCols % kPiece == 0 && kPiece % 16 == 0, "epilogue reads 16- or 32-column pieces");
    uint8_t* srow = stage + row * 128;
    const uint32_t sw = static_cast<uint32_t>(row & 7);
#pragma unroll
    for (int c0 = 0; c0 < kCols; c0 += kPiece) {
      const int col = wg * kCols + c0;
      uint32_t o[kPiece];
      if constexpr (kPiece == 32)
        tmem_ld32(tmem + lane_off + C::kColO + col, o);
      else
        tmem_ld16(tmem + lane_off + C::kColO + col, o);
      tmem_wait_ld();
      if constexpr (F16) {
#pragma unroll
        for (int t = 0; t < kPiece; ++t) o[t] = __float_as_uint(__uint_as_float(o[t]) * p.o_unscale);
      }
      if (p.out_f32) {
#pragma unroll
        for (int t = 0; t < kPiece / 4; ++t) {
          const int c = col + 4 * t;  // box c / 32, 16-B chunk (c % 32) / 4
          *reinterpret_cast<uint4*>(srow + (c >> 5) * C::kBoxBytes + ((((c & 31) >> 2) ^ sw) << 4)) =
              make_uint4(o[4 * t], o[4 * t + 1], o[4 * t + 2], o[4 * t + 3]);
        }
      } else {
#pragma unroll
        for (int t = 0; t < kPiece / 8; ++t) {
          const int c = col + 8 * t;  // box c / 64, 16-B chunk (c % 64) / 8
          uint32_t w[4];
#pragma unroll
          for (int h = 0; h < 4; ++h)
            w[h] = F16 ? pack_f16x2(__uint_as_float(o[8 * t + 2 * h]), __uint_as_float(o[8 * t + 2 * h + 1]))
                       : pack_bf16x2(__uint_as_float(o[8 * t + 2 * h]), __uint_as_float(o[8 * t + 2 * h + 1]));
          *reinterpret_cast<uint4*>(srow + (c >> 6) * C::kBoxBytes + ((((c & 63) >> 3) ^ sw) << 4)) =
              make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
    fence_proxy_async_smem();
  }
  ok = named_barrier_and(2, 32 * C::kTW, ok);
  if (ok && warp == 2 && lane == 0) {
    const int n_boxes = p.out_f32 ? D / 32 : D / 64;
    const int box_cols = p.out_f32 ? 32 : 64;
    for (int b = 0; b < n_boxes; ++b) tma_store_3d(&p.tm_out, stage + b * C::kBoxBytes, b * box_cols, q0, bh);
    bulk_commit_group();
    bulk_wait_group_read0();  // the shared-memory source stays valid until read
  }
}

template <int D, bool DIFF, bool NORM, bool POS, int PM, bool F16>
__global__ void __maxnreg__((Cfg<D, DIFF>::kMaxRegs)) tda_tc_fwd_kernel(const __grid_constant__ TcFwdParams p) {
  using C = Cfg<D, DIFF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Launch order: groups of kHeadGroup (batch, head) slices, and inside a
  // group the query tiles longest first with the group's heads interleaved.
  // The CTAs in flight at any time then cover only a few slices, so each K/V
  // tile is read from HBM about once and served from L2 to every query tile
  // of its head, and the causal work per CTA falls monotonically towards the
  // end of each group (longest-processing-time-first: short tiles fill the
  // SMs that free up while the long tiles of the group finish).
  const int per_group = kHeadGroup * p.n_qtiles;
  const int g0 = static_cast<int>(blockIdx.x / per_group) * kHeadGroup;
  const int gsz = min(kHeadGroup, p.BH - g0);
  const int r = static_cast<int>(blockIdx.x % per_group);
  const int bh = g0 + r % gsz;
  const int qt = p.n_qtiles - 1 - r / gsz;
  const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->drain2, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->s_full[i], DIFF ? 2 : 1);
      mbar_init(&bars->p_full[i], C::kTW);
      mbar_init(&bars->pv_done[i], 1);
      bars->tile_mask[i] = 0;
    }
    for (int i = 0; i < 2; ++i) mbar_init(&bars->s2_free[i], C::kTW);
    for (int i = 0; i < kRkRing; ++i) {
      mbar_init(&bars->rk_full[i], 1);
      mbar_init(&bars->rk_empty[i], C::kTW);
    }
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    issue_first_loads<D, DIFF, NORM>(p, smem, bars, bh, qt);
    tma_prefetch_desc(&p.tm_v);
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const WaitCtl ctl = make_wait_ctl(&bars->abort_flag, p.status, p.timeout_ns);

  if (warp == 0) {
    if (lane == 0) run_producer<D, DIFF, NORM>(p, smem, bars, ctl, bh, qt, n_kt);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) run_mma<D, DIFF, F16>(smem, bars, ctl, tmem, n_kt, p.stats);
    __syncwarp();
  } else if (warp < C::kQk2W) {
    run_transform<D, DIFF, NORM, POS, PM, F16>(p, smem, bars, ctl, tmem, bh, qt, n_kt, warp, lane);
  } else if (warp == C::kQk2W) {
    if (lane == 0) {
      if constexpr (DIFF)
        run_mma_qk2<D, F16>(smem, bars, ctl, tmem, n_kt);
      else
        run_mma_qk<D, F16>(smem, bars, ctl, tmem, n_kt);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================ persistent
// One CTA per SM; each CTA takes work items -- one 128-row query tile of one
// (batch, head) -- from a global counter, in the same grouped longest-first
// order as the one-tile-per-CTA launch, so the items in flight still cover a
// few (batch, head) slices and late items are the short ones.  Every ring,
// S slot and barrier phase continues across items (global tile and ring
// counters), so the K/V ring does not drain between items and one item's
// start-up overlaps the previous one's last products:
//   rect: two query buffers; the next item's Q is loaded after the current
//         item's last K/V load, and a finished item's query buffer stages its
//         output for the TMA store.
//   diff: one Q1/Q2 buffer, reloaded as soon as the current item's last QK
//         products have completed; the output is written directly.
template <int D, bool DIFF>
struct PCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = kTile * 128;
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr int kNQ = DIFF ? 2 : 1;
  static constexpr int kQBufs = DIFF ? 1 : 2;
  static constexpr int kQBytes = kNQ * kTileBytes;  // one item's query tile(s)
  static constexpr int kRkPerTile = (DIFF ? 2 : 1) * (kTile + 8);
  static constexpr int kRkFloats = kRkRing * kRkPerTile;
  static constexpr int kBarBytes = 1024;
  // norm partial sums, one set per item parity: a set is rewritten two items
  // later, after a barrier that follows every read of it
  static constexpr int kQssFloats = kNQ * kTransformWG * kTile;
  static constexpr int kQssBytes = 2 * kQssFloats * 4;
  static constexpr int kFixed = kQBufs * kQBytes + kRkFloats * 4 + kBarBytes + kQssBytes + 1024;
  static constexpr int kSlotsRaw = (kSmemBudget - kFixed) / kTileBytes;
  static constexpr int kSlots = kSlotsRaw > 8 ? 8 : kSlotsRaw;
  static_assert(kSlots >= 3, "not enough shared memory for the K/V ring");
  static constexpr int kOffRing = kQBufs * kQBytes;
  static constexpr int kOffRk = kOffRing + kSlots * kTileBytes;
  static constexpr int kOffBar = kOffRk + kRkFloats * 4;
  static constexpr int kOffQss = kOffBar + kBarBytes;
  static constexpr int kSmemBytes = kOffQss + kQssBytes + 1024;
  static constexpr int kSSlots = DIFF ? 2 : 3;
  static constexpr int kColS2 = 128;
  static constexpr int kColO = 384;
  static __device__ __forceinline__ uint32_t col_s(int slot) {
    return DIFF ? (slot ? 256u : 0u) : static_cast<uint32_t>(slot * 128);
  }
  // ring entries per key tile: K and V (rect); K1, K2, V (diff)
  static constexpr int kLoadsPerTile = DIFF ? 3 : 2;
};

struct PBars {
  uint64_t q_full[2];
  uint64_t q_empty[2];   // rect: last QK committed + output stored; diff: both issuers' last QK + norms read
  uint64_t o_full;
  uint64_t o_empty;      // every transform warp holds O in registers
  uint64_t drain;
  uint64_t drain2;
  uint64_t s_full[3];
  uint64_t p_full[3];
  uint64_t pv_done[3];   // rect, per S slot: the PV reading P from it has run
  uint64_t s2_free[2];
  uint64_t rk_full[kRkRing];
  uint64_t rk_empty[kRkRing];
  uint64_t slot_full[8];
  uint64_t slot_empty[8];
  uint64_t item_full[2];
  uint64_t item_empty[2];
  int item[2];           // work item index, -1 = no more work
  uint32_t tmem_base;
  int abort_flag;
  uint32_t tile_mask[3]; // tag = global tile index + 1
};
static_assert(sizeof(PBars) <= 1024, "barrier block too large");

constexpr int ST_PROD_Q = 0x103, ST_PROD_ITEM = 0x104, ST_MMA_ITEM = 0x205, ST_MMA_O = 0x206, ST_TR_ITEM = 0x305;

__device__ __forceinline__ void decode_item(const TcFwdParams& p, int idx, int& bh, int& qt) {
  const int per_group = kHeadGroup * p.n_qtiles;
  const int g0 = (idx / per_group) * kHeadGroup;
  const int gsz = min(kHeadGroup, p.BH - g0);
  const int r = idx % per_group;
  bh = g0 + r % gsz;
  qt = p.n_qtiles - 1 - r / gsz;
}

template <int D, bool DIFF, bool NORM>
__device__ void p_producer(const TcFwdParams& p, uint8_t* smem, PBars* bars, const WaitCtl& ctl, int n_items) {
  using C = PCfg<D, DIFF>;
  uint8_t* ring = smem + C::kOffRing;
  float* rk_s = reinterpret_cast<float*>(smem + C::kOffRk);
  int ridx = 0;  // ring entries issued (all items)
  int rk_n = 0;  // key-table ring entries issued (= key tiles of all items)
  int q_n = 0;   // query loads issued
  bool ok = true;
  int h_idx = 0, b_idx = 0, bh = 0;
  auto load_tile = [&](const CUtensorMap* map, int j) {
    if (!ok) return;
    const int slot = ridx % C::kSlots;
    if (!mbar_wait(&bars->slot_empty[slot], ((ridx / C::kSlots) & 1) ^ 1, ctl, ST_PROD_SLOT)) {
      ok = false;
      return;
    }
    mbar_arrive_expect_tx(&bars->slot_full[slot], C::kTileBytes);
    uint8_t* dst = ring + slot * C::kTileBytes;
#pragma unroll
    for (int b = 0; b < C::kBoxes; ++b)
      tma_load_4d(dst + b * C::kBoxBytes, map, &bars->slot_full[slot], b * 64, j * kTile, h_idx, b_idx);
    ++ridx;
  };
  auto load_rk = [&](int j) {
    if constexpr (NORM) {
      if (!ok) return;
      const int e = rk_n % kRkRing;
      if (!mbar_wait(&bars->rk_empty[e], ((rk_n / kRkRing) & 1) ^ 1, ctl, ST_PROD_RK)) {
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
    }
    ++rk_n;
  };
  // publish item `it` (index or -1) to the consumers
  auto publish = [&](int it, int idx) {
    if (!ok) return;
    const int e = it & 1;
    if (!mbar_wait(&bars->item_empty[e], ((it >> 1) & 1) ^ 1, ctl, ST_PROD_ITEM)) {
      ok = false;
      return;
    }
    bars->item[e] = idx;
    mbar_arrive(&bars->item_full[e]);
  };
  // query tile(s) of item `it` into its buffer, once the buffer's previous
  // item has released it
  auto load_q = [&](int it, int qbh, int qt) {
    if (!ok) return;
    const int b = DIFF ? 0 : (it & 1);
    const int use = DIFF ? it : (it >> 1);
    if (use > 0 && !mbar_wait(&bars->q_empty[b], (use - 1) & 1, ctl, ST_PROD_Q)) {
      ok = false;
      return;
    }
    if (p.inject & 1) return;
    const int qh = qbh % p.heads, qb = qbh / p.heads;
    uint8_t* dst = smem + b * C::kQBytes;
    mbar_arrive_expect_tx(&bars->q_full[b], C::kQBytes);
#pragma unroll
    for (int x = 0; x < C::kBoxes; ++x) {
      tma_load_4d(dst + x * C::kBoxBytes, &p.tm_q1, &bars->q_full[b], x * 64, qt * kTile, qh, qb);
      if constexpr (DIFF)
        tma_load_4d(dst + C::kTileBytes + x * C::kBoxBytes, &p.tm_q2, &bars->q_full[b], x * 64, qt * kTile, qh, qb);
    }
    ++q_n;
  };
  auto fetch = [&]() {
    const int idx = static_cast<int>(atomicAdd(p.item_ctr, 1u));
    return idx < n_items ? idx : -1;
  };

  int it = 0;
  int cur = fetch();
  publish(0, cur);
  if (cur >= 0) {
    int qt0;
    decode_item(p, cur, bh, qt0);
    load_q(0, bh, qt0);
  }
  while (cur >= 0 && ok) {
    int qt;
    decode_item(p, cur, bh, qt);
    h_idx = bh % p.heads;
    b_idx = bh / p.heads;
    const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;
    if constexpr (!DIFF) {
      // consumption order: K0, K1, K2, then per j: V_j, K_{j+3}
      for (int j = 0; j < 3 && j < n_kt; ++j) {
        load_rk(j);
        load_tile(&p.tm_k1, j);
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        load_tile(&p.tm_v, j);
        if (j + 3 < n_kt) {
          load_rk(j + 3);
          load_tile(&p.tm_k1, j + 3);
        }
      }
    } else {
      // consumption order: K1_0, K2_0, K1_1, then per j: K2_{j+1}, V_j, K1_{j+2}
      load_rk(0);
      load_tile(&p.tm_k1, 0);
      load_tile(&p.tm_k2, 0);
      if (n_kt > 1) {
        load_rk(1);
        load_tile(&p.tm_k1, 1);
      }
      for (int j = 0; j < n_kt && ok; ++j) {
        if (j + 1 < n_kt) load_tile(&p.tm_k2, j + 1);
        load_tile(&p.tm_v, j);
        if (j + 2 < n_kt) {
          load_rk(j + 2);
          load_tile(&p.tm_k1, j + 2);
        }
      }
    }
    const int nxt = fetch();
    publish(it + 1, nxt);
    if (nxt >= 0) {
      int nbh, nqt;
      decode_item(p, nxt, nbh, nqt);
      load_q(it + 1, nbh, nqt);
    }
    cur = nxt;
    ++it;
  }
  if (!ok) {
    // abort: wait for the copies still in flight (newest per ring slot, rk
    // entry and query buffer)
    const int first = ridx > C::kSlots ? ridx - C::kSlots : 0;
    for (int i = first; i < ridx; ++i) drain_wait(&bars->slot_full[i % C::kSlots], (i / C::kSlots) & 1, ctl);
    if constexpr (NORM) {
      const int rfirst = rk_n > kRkRing ? rk_n - kRkRing : 0;
      for (int i = rfirst; i < rk_n; ++i) drain_wait(&bars->rk_full[i % kRkRing], (i / kRkRing) & 1, ctl);
    }
    const int qfirst = q_n > C::kQBufs ? q_n - C::kQBufs : 0;
    for (int i = qfirst; i < q_n; ++i) {
      const int b = DIFF ? 0 : (i & 1);
      const int use = DIFF ? i : (i >> 1);
      drain_wait(&bars->q_full[b], use & 1, ctl);
    }
  }
}

// consumer side of the item ring: every consumer thread / warp reads entry
// `it` and releases it (one arrival per consumer)
__device__ __forceinline__ int take_item(PBars* bars, int it, const WaitCtl& ctl, int code, bool& ok, bool warp_wide,
                                         int lane) {
  const int e = it & 1;
  bool got = warp_wide ? mbar_wait_warp(&bars->item_full[e], (it >> 1) & 1, ctl, code)
                       : mbar_wait(&bars->item_full[e], (it >> 1) & 1, ctl, code);
  int idx = -1;
  if (got) idx = *reinterpret_cast<volatile int*>(&bars->item[e]);
  if (warp_wide) __syncwarp();
  if (got && lane == 0) mbar_arrive(&bars->item_empty[e]);
  ok = ok && got;
  return got ? idx : -1;
}

// PV issuer (warp 1), every item in turn: V_j's ring entry is acquired
// before the wait for P_j.  rect: after PV_j it commits pv_done of P_j's S
// slot, which hands the slot to the QK issuer (warp 10).  differential: it
// also issues QK1_{j+2} into P_j's slot right after PV_j.
template <int D, bool DIFF>
__device__ void p_mma(const TcFwdParams& p, uint8_t* smem, PBars* bars, const WaitCtl& ctl, uint32_t tmem) {
  using C = PCfg<D, DIFF>;
  MmaIssuer<D, DIFF, C, PBars> m(smem, bars, ctl, tmem);
  int g = 0;     // global key-tile counter (S slots, tile tags)
  int base = 0;  // ring position of the item's first entry
  bool ok = true;
  for (int it = 0;; ++it) {
    const int idx = take_item(bars, it, ctl, ST_MMA_ITEM, ok, false, 0);
    if (idx < 0 || !ok || !m.ok) break;
    int bh, qt;
    decode_item(p, idx, bh, qt);
    const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;
    m.o_started = false;
    if constexpr (!DIFF) {
      for (int j = 0; j < n_kt && m.ok; ++j) {
        const int G = g + j, slot = G % C::kSSlots;
        const int vslot = m.acquire(base + ring_v_rect(j, n_kt));
        m.wait(&bars->p_full[slot], (G / C::kSSlots) & 1, ST_MMA_P);
        if (j == 0 && it > 0) m.wait(&bars->o_empty, (it - 1) & 1, ST_MMA_O);
        m.pv_at(vslot, C::col_s(slot), m.slab_mask(G));
        m.commit(&bars->pv_done[slot]);
      }
    } else {
      m.wait(&bars->q_full[0], it & 1, ST_MMA_Q);
      const uint32_t q1_base = smem_u32(smem);
      m.qk(base + ring_k1(0), C::col_s(g & 1), q1_base);
      m.commit(&bars->s_full[g & 1]);
      if (n_kt == 1) m.commit(&bars->q_empty[0]);
      if (n_kt > 1) {
        m.qk(base + ring_k1(1), C::col_s((g + 1) & 1), q1_base);
        m.commit(&bars->s_full[(g + 1) & 1]);
        if (n_kt == 2) m.commit(&bars->q_empty[0]);
      }
      for (int j = 0; j < n_kt && m.ok; ++j) {
        const int G = g + j, slot = G & 1;
        const int vslot = m.acquire(base + ring_v(j, n_kt));
        m.wait(&bars->p_full[slot], (G >> 1) & 1, ST_MMA_P);
        if (j == 0 && it > 0) m.wait(&bars->o_empty, (it - 1) & 1, ST_MMA_O);
        m.pv_at(vslot, C::col_s(slot), m.slab_mask(G));
        if (j + 2 < n_kt) {
          m.qk(base + ring_k1(j + 2), C::col_s(slot), q1_base);
          m.commit(&bars->s_full[slot]);
          if (j + 2 == n_kt - 1) m.commit(&bars->q_empty[0]);
        }
      }
    }
    m.commit(&bars->o_full);
    g += n_kt;
    base += C::kLoadsPerTile * n_kt;
  }
  if (!m.ok || !ok) m.drain(&bars->drain);
  if (p.stats) {
    atomicAdd(p.stats, static_cast<unsigned long long>(m.slabs));
    atomicAdd(p.stats + 1, static_cast<unsigned long long>(g) * (kTile / 16));
  }
}

// QK issuer of the rectified form (warp 10): S_G = Q K_G^T into slot G % 3
// once PV_{G-3}, which read P from that slot, has run (the slots continue
// across items); the K entry is acquired before that wait.  The item's last
// QK releases its query buffer (q_empty).
template <int D>
__device__ void p_mma_qk(const TcFwdParams& p, uint8_t* smem, PBars* bars, const WaitCtl& ctl, uint32_t tmem) {
  using C = PCfg<D, false>;
  MmaIssuer<D, false, C, PBars> m(smem, bars, ctl, tmem);
  int g = 0, base = 0;
  bool ok = true;
  for (int it = 0;; ++it) {
    const int idx = take_item(bars, it, ctl, ST_MMA_ITEM, ok, false, 0);
    if (idx < 0 || !ok || !m.ok) break;
    int bh, qt;
    decode_item(p, idx, bh, qt);
    const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;
    const int b = it & 1;
    m.wait(&bars->q_full[b], (it >> 1) & 1, ST_MMA_Q);
    const uint32_t q1_base = smem_u32(smem + b * C::kQBytes);
    for (int t = 0; t < n_kt && m.ok; ++t) {
      const int G = g + t, slot = G % C::kSSlots;
      // ring order per item: K_0, K_1, K_2, then per j: V_j, K_{j+3}
      const int kslot = m.acquire(base + (t < C::kSSlots ? t : ring_v_rect(t - C::kSSlots, n_kt) + 1));
      if (G >= C::kSSlots) m.wait(&bars->pv_done[slot], ((G - C::kSSlots) / C::kSSlots) & 1, ST_MMA_P);
      m.qk_at(kslot, C::col_s(slot), q1_base);
      m.commit(&bars->s_full[slot]);
      if (t == n_kt - 1) m.commit(&bars->q_empty[b]);
    }
    g += n_kt;
    base += C::kLoadsPerTile * n_kt;
  }
  if (!m.ok || !ok) m.drain(&bars->drain2);
}

template <int D>
__device__ void p_mma_qk2(const TcFwdParams& p, uint8_t* smem, PBars* bars, const WaitCtl& ctl, uint32_t tmem) {
  using C = PCfg<D, true>;
  MmaIssuer<D, true, C, PBars> m(smem, bars, ctl, tmem);
  const uint32_t q2_base = smem_u32(smem) + C::kTileBytes;
  int g = 0, base = 0;
  bool ok = true;
  for (int it = 0;; ++it) {
    const int idx = take_item(bars, it, ctl, ST_MMA_ITEM, ok, false, 0);
    if (idx < 0 || !ok || !m.ok) break;
    int bh, qt;
    decode_item(p, idx, bh, qt);
    const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;
    m.wait(&bars->q_full[0], it & 1, ST_MMA_Q);
    for (int j = 0; j < n_kt && m.ok; ++j) {
      const int G = g + j;
      // S2 is single-buffered: tile G - 1 must have been read out of it
      if (G > 0) m.wait(&bars->s2_free[(G - 1) & 1], ((G - 1) >> 1) & 1, ST_MMA_S2);
      m.qk(base + ring_k2(j), C::kColS2, q2_base);
      m.commit(&bars->s_full[G & 1]);
    }
    m.commit(&bars->q_empty[0]);  // the item's last QK2
    g += n_kt;
    base += C::kLoadsPerTile * n_kt;
  }
  if (!m.ok || !ok) m.drain(&bars->drain2);
}

// Query norms of one item into c (and tau for its rows); every transform
// thread reaches the barrier.  Returns the AND over the transform threads of
// (ok and the item is real).
template <int D, bool DIFF, bool NORM, int PM>
__device__ bool p_prologue(const TcFwdParams& p, uint8_t* smem, PBars* bars, const WaitCtl& ctl, int it, int idx,
                           int row, int wg, bool ok, RowCoef& c, int& bh, int& qt) {
  using C = PCfg<D, DIFF>;
  constexpr bool kFold = PM != POW_GENERAL;
  bh = 0;
  qt = 0;
  if (idx >= 0) decode_item(p, idx, bh, qt);
  const int grow = qt * kTile + row;
  const float tau = p.beta * sqrtf((2.0f * logf(static_cast<float>(grow + 1))) / static_cast<float>(D));
  float lam = p.lam, lam_root = p.lam_root;
  if (DIFF && p.lam_dev.ptr && idx >= 0) {  // lambda of this item's (batch, head) from the device
    lam = lambda_of(p.lam_dev, bh, p.lam);
    lam_root = lambda_root<PM>(lam);
  }
  const float lam2 = (DIFF && kFold) ? lam_root : 1.0f;
  c = RowCoef{tau, 1.0f, tau, lam2, lam};
  bool live = ok && idx >= 0;
  if constexpr (NORM) {
    const int b = DIFF ? 0 : (it & 1);
    const int use = DIFF ? it : (it >> 1);
    if (live) live = mbar_wait_warp(&bars->q_full[b], use & 1, ctl, ST_TR_Q);
    float* qss = reinterpret_cast<float*>(smem + C::kOffQss) + (it & 1) * C::kQssFloats;
    if (live) {
#pragma unroll 1
      for (int t = 0; t < C::kNQ; ++t) {
        float ss = 0.0f;
#pragma unroll 1
        for (int bx = 0; bx < C::kBoxes; ++bx) {
          const uint8_t* rb = smem + b * C::kQBytes + t * C::kTileBytes + bx * C::kBoxBytes + row * 128;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            // logical chunk cc sits at (cc ^ (row & 7)): conflict-free across 8 rows
            const int cc = 4 * wg + k;
            const uint4 u = *reinterpret_cast<const uint4*>(rb + ((cc ^ (row & 7)) << 4));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float lo = __uint_as_float(w[h] << 16), hi = __uint_as_float(w[h] & 0xFFFF0000u);
              ss = fmaf(lo, lo, ss);
              ss = fmaf(hi, hi, ss);
            }
          }
        }
        qss[(t * kTransformWG + wg) * kTile + row] = ss;
      }
    }
    live = named_barrier_and(1, 32 * kTransformWarps, live);
    if (live) {
      const float m1 = fmaxf(sqrtf(qss[row] + qss[kTile + row]), 1e-12f);
      c.rq1 = 1.0f / m1;
      c.tq1 = tau * m1;
      if constexpr (DIFF) {
        const float m2 = fmaxf(sqrtf(qss[2 * kTile + row] + qss[3 * kTile + row]), 1e-12f);
        c.rq2 = lam2 / m2;
        c.tq2 = tau * m2;
      }
    }
  } else {
    live = named_barrier_and(1, 32 * kTransformWarps, live);
  }
  if constexpr (DIFF) {
    // the query buffer may be reloaded once both issuers' last QK products of
    // this item are done and the norms have been read (this arrival)
    if (live && threadIdx.x == 64) mbar_arrive(&bars->q_empty[0]);
  }
  return live;
}

// Transform warps of the persistent kernel.  Per item: key tile 0, then the
// previous item's epilogue (its O is complete by then, and the current
// item's first PV waits only for O to be read out), then the remaining key
// tiles, then the next item's query norms.  Both named barriers (norms: 1,
// epilogue: 2) are reached by every transform warp in the same order, and
// whether to go on is decided from their AND-reductions, so a wait that gave
// up in one warp cannot leave the others at a barrier.
template <int D, bool DIFF, bool NORM, bool POS, int PM>
__device__ void p_transform(const TcFwdParams& p, uint8_t* smem, PBars* bars, const WaitCtl& ctl, uint32_t tmem,
                            int warp, int lane) {
  using C = PCfg<D, DIFF>;
  constexpr int kChunks = 4 / kTransformWG;
  static_assert(kChunks == 2, "transform_tile handles two chunks");
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float* rk_s = reinterpret_cast<const float*>(smem + C::kOffRk);

  // key tile j (global index G) of the item whose query tile is qt
  auto tile = [&](int j, int G, int qt, const RowCoef& c) -> bool {
    const int re = G % kRkRing;
    if constexpr (NORM) {
      if (!mbar_wait_warp(&bars->rk_full[re], (G / kRkRing) & 1, ctl, ST_TR_RK)) return false;
    }
    const int slot = G % C::kSSlots;
    if (!mbar_wait_warp(&bars->s_full[slot], (G / C::kSSlots) & 1, ctl, ST_TR_S)) return false;
    tc_fence_after();
    const uint32_t nz = transform_tile<PM, DIFF, NORM, POS, kRollChunks<DIFF>, kRollHalves<DIFF>, false, kChunks>(
        tmem + lane_off, C::col_s(slot), C::kColS2, wg, rk_s + re * C::kRkPerTile, qt * kTile + row - j * kTile,
        j >= qt, c, p.relu_power, c.lam, 1.0f, [&] {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->s2_free[G & 1]);
        });
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, nz) << (2 * kChunks * wg);
    if (wmask != 0u && lane == 0) {
      uint32_t* word = &bars->tile_mask[slot];
      const uint32_t tag = static_cast<uint32_t>(G + 1) << 8;
      uint32_t old = *reinterpret_cast<volatile uint32_t*>(word), assumed;
      do {
        assumed = old;
        const uint32_t base = (assumed & ~0xFFu) == tag ? assumed : tag;
        old = atomicCAS(word, assumed, base | wmask);
      } while (old != assumed);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&bars->p_full[slot]);
      if constexpr (NORM) mbar_arrive(&bars->rk_empty[re]);
    }
    return true;
  };

  // epilogue of item e_it, 32 columns at a time: O -> registers -> output
  // (rect bf16: staged in the item's query buffer, free once its last QK and
  // its norms are done, then TMA-stored); O is handed back (o_empty) once the
  // last chunk is in registers.  Returns the AND over the transform warps.
  auto epilogue = [&](int e_it, int e_bh, int e_qt, bool in_ok) -> bool {
    const bool eok = in_ok && mbar_wait_warp(&bars->o_full, e_it & 1, ctl, ST_TR_O);
    constexpr int kCols = D / kTransformWG;
    const int egrow = e_qt * kTile + row;
    const bool staged = !DIFF && !p.out_f32;
    uint8_t* stage = smem + (e_it & 1) * C::kQBytes;
    if (eok) {
      tc_fence_after();
      const size_t row_off = (static_cast<size_t>(e_bh) * p.S + (egrow < p.S ? egrow : 0)) * D;
#pragma unroll 1
      for (int c0 = 0; c0 < kCols; c0 += 32) {
        const int col = wg * kCols + c0;
        uint32_t o[32];
        tmem_ld32(tmem + lane_off + C::kColO + col, o);
        tmem_wait_ld();
        if (c0 + 32 == kCols) {
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&bars->o_empty);
        }
        if (staged) {
          uint8_t* srow = stage + row * 128;
          const uint32_t sw = static_cast<uint32_t>(row & 7);
#pragma unroll
          for (int t = 0; t < 4; ++t) {
            const int cc = col + 8 * t;  // box cc / 64, 16-B chunk (cc % 64) / 8
            uint32_t w[4];
#pragma unroll
            for (int h = 0; h < 4; ++h)
              w[h] = pack_bf16x2(__uint_as_float(o[8 * t + 2 * h]), __uint_as_float(o[8 * t + 2 * h + 1]));
            *reinterpret_cast<uint4*>(srow + (cc >> 6) * C::kBoxBytes + ((((cc & 63) >> 3) ^ sw) << 4)) =
                make_uint4(w[0], w[1], w[2], w[3]);
          }
        } else if (egrow < p.S) {
          if (p.out_f32) {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row_off + col);
#pragma unroll
            for (int t = 0; t < 8; ++t)
              dst[t] = make_float4(__uint_as_float(o[4 * t]), __uint_as_float(o[4 * t + 1]),
                                   __uint_as_float(o[4 * t + 2]), __uint_as_float(o[4 * t + 3]));
          } else {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(p.out) + row_off + col);
#pragma unroll
            for (int t = 0; t < 4; ++t) {
              uint32_t w[4];
#pragma unroll
              for (int h = 0; h < 4; ++h)
                w[h] = pack_bf16x2(__uint_as_float(o[8 * t + 2 * h]), __uint_as_float(o[8 * t + 2 * h + 1]));
              dst[t] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          }
        }
      }
      if (staged) fence_proxy_async_smem();
    }
    const bool sok = named_barrier_and(2, 32 * kTransformWarps, eok);
    if (!DIFF && warp == 2 && lane == 0) {
      if (staged && sok) {
        for (int x = 0; x < C::kBoxes; ++x)
          tma_store_3d(&p.tm_out, stage + x * C::kBoxBytes, x * 64, e_qt * kTile, e_bh);
        bulk_commit_group();
        bulk_wait_group_read0();
      }
      mbar_arrive(&bars->q_empty[e_it & 1]);  // the query buffer may be reloaded
    }
    return sok;
  };

  bool ok = true;
  int g = 0, it = 0;
  const int idx0 = take_item(bars, 0, ctl, ST_TR_ITEM, ok, true, lane);
  RowCoef c;
  int bh, qt;
  bool live = p_prologue<D, DIFF, NORM, PM>(p, smem, bars, ctl, 0, idx0, row, wg, ok, c, bh, qt);
  ok = live;
  bool pending = false;  // the previous item's epilogue is still to be done
  int p_it = 0, p_bh = 0, p_qt = 0;
  while (live) {
    const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;
    // one call site of the (large) tile body; iteration 0 is run by every
    // warp, so the deferred epilogue after it is reached by all of them
    for (int j = 0; j < n_kt; ++j) {
      if (ok) ok = tile(j, g + j, qt, c);
      if (j == 0 && pending) {
        ok = epilogue(p_it, p_bh, p_qt, ok);  // uniform from here
        pending = false;
      }
      if (!ok) break;
    }
    const int nidx = take_item(bars, it + 1, ctl, ST_TR_ITEM, ok, true, lane);
    RowCoef cn;
    int nbh, nqt;
    live = p_prologue<D, DIFF, NORM, PM>(p, smem, bars, ctl, it + 1, nidx, row, wg, ok, cn, nbh, nqt);
    pending = true;
    p_it = it;
    p_bh = bh;
    p_qt = qt;
    g += n_kt;
    ++it;
    c = cn;
    bh = nbh;
    qt = nqt;
    ok = live;
  }
  if (pending) epilogue(p_it, p_bh, p_qt, true);
}

template <int D, bool DIFF, bool NORM, bool POS, int PM>
__global__ void __maxnreg__(168) tda_tc_fwd_persistent_kernel(const __grid_constant__ TcFwdParams p) {
  using C = PCfg<D, DIFF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  PBars* bars = reinterpret_cast<PBars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int n_items = p.BH * p.n_qtiles;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->q_full[i], 1);
      mbar_init(&bars->q_empty[i], DIFF ? 3 : 2);
      mbar_init(&bars->item_full[i], 1);
      mbar_init(&bars->item_empty[i], 2 + kTransformWarps);
      mbar_init(&bars->s2_free[i], kTransformWarps);
      bars->item[i] = -1;
    }
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->o_empty, kTransformWarps);
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->drain2, 1);
    for (int i = 0; i < 3; ++i) {
      mbar_init(&bars->s_full[i], DIFF ? 2 : 1);
      mbar_init(&bars->p_full[i], kTransformWarps);
      mbar_init(&bars->pv_done[i], 1);
      bars->tile_mask[i] = 0;
    }
    for (int i = 0; i < kRkRing; ++i) {
      mbar_init(&bars->rk_full[i], 1);
      mbar_init(&bars->rk_empty[i], kTransformWarps);
    }
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&p.tm_q1);
    tma_prefetch_desc(&p.tm_k1);
    tma_prefetch_desc(&p.tm_v);
    if constexpr (DIFF) {
      tma_prefetch_desc(&p.tm_q2);
      tma_prefetch_desc(&p.tm_k2);
    }
  }
  if (warp == 1) {
    tmem_alloc(&bars->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bars->tmem_base;
  const WaitCtl ctl = make_wait_ctl(&bars->abort_flag, p.status, p.timeout_ns);
  if (warp == 0) {
    if (lane == 0) p_producer<D, DIFF, NORM>(p, smem, bars, ctl, n_items);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) p_mma<D, DIFF>(p, smem, bars, ctl, tmem);
    __syncwarp();
  } else if (warp < kQk2Warp) {
    p_transform<D, DIFF, NORM, POS, PM>(p, smem, bars, ctl, tmem, warp, lane);
  } else {
    if (lane == 0) {
      if constexpr (DIFF)
        p_mma_qk2<D>(p, smem, bars, ctl, tmem);
      else
        p_mma_qk<D>(p, smem, bars, ctl, tmem);
    }
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool DIFF, bool NORM, bool POS, int PM>
cudaError_t launch_persistent(const TcFwdParams& p, cudaStream_t stream) {
  using C = PCfg<D, DIFF>;
  auto kern = tda_tc_fwd_persistent_kernel<D, DIFF, NORM, POS, PM>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  const long long n_items = static_cast<long long>(p.BH) * p.n_qtiles;
  const unsigned grid = static_cast<unsigned>(n_items < sms ? n_items : sms);
  kern<<<grid, threads_for<DIFF>(), C::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

template <int D, bool DIFF, bool NORM, bool POS, int PM, bool F16>
cudaError_t launch_one(const TcFwdParams& p, cudaStream_t stream) {
  if constexpr (!F16) {
    if (p.item_ctr) return launch_persistent<D, DIFF, NORM, POS, PM>(p, stream);
  }
  using C = Cfg<D, DIFF>;
  auto kern = tda_tc_fwd_kernel<D, DIFF, NORM, POS, PM, F16>;
  static bool attr_done = false;  // per instantiation; attribute is per-function, idempotent
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const unsigned grid = static_cast<unsigned>(p.BH) * static_cast<unsigned>(p.n_qtiles);
  constexpr int kThreads = C::kThreads;
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e == cudaErrorLaunchOutOfResources) {
    cudaFuncAttributes fa;
    if (cudaFuncGetAttributes(&fa, kern) == cudaSuccess) {
      char msg[256];
      snprintf(msg, sizeof(msg),
               "tensor-core kernel does not fit: %d threads requested, %d allowed (%d registers/thread, %zu B "
               "local, %zu B dynamic shared)",
               kThreads, fa.maxThreadsPerBlock, fa.numRegs, static_cast<size_t>(fa.localSizeBytes),
               static_cast<size_t>(C::kSmemBytes));
      set_last_error(msg);
    }
  }
  return e;
}

template <int D, bool DIFF, bool NORM, bool POS, bool F16 = false>
cudaError_t dispatch_pow(const TcFwdParams& p, int pm, cudaStream_t s) {
  switch (pm) {
    case POW_1: return launch_one<D, DIFF, NORM, POS, POW_1, F16>(p, s);
    case POW_2: return launch_one<D, DIFF, NORM, POS, POW_2, F16>(p, s);
    case POW_3: return launch_one<D, DIFF, NORM, POS, POW_3, F16>(p, s);
    default: return launch_one<D, DIFF, NORM, POS, POW_GENERAL, F16>(p, s);
  }
}

// beta >= 0 (tau >= 0): zero halves are recognised from the raw scores, and
// with normalize the ReLU is a saturating multiply
template <int D, bool DIFF>
cudaError_t dispatch_norm(const TcFwdParams& p, bool norm, int pm, bool fp16, cudaStream_t s) {
  if (fp16) {
    // fp16 operands: normalized scores only (P bounded, see the launcher)
    if (!norm) return cudaErrorInvalidValue;
    return p.causal_skip ? dispatch_pow<D, DIFF, true, true, true>(p, pm, s)
                         : dispatch_pow<D, DIFF, true, false, true>(p, pm, s);
  }
  if (norm)
    return p.causal_skip ? dispatch_pow<D, DIFF, true, true>(p, pm, s) : dispatch_pow<D, DIFF, true, false>(p, pm, s);
  return p.causal_skip ? dispatch_pow<D, DIFF, false, true>(p, pm, s) : dispatch_pow<D, DIFF, false, false>(p, pm, s);
}

template <int D>
cudaError_t dispatch_diff(const TcFwdParams& p, bool diff, bool norm, int pm, bool fp16, cudaStream_t s) {
  return diff ? dispatch_norm<D, true>(p, norm, pm, fp16, s) : dispatch_norm<D, false>(p, norm, pm, fp16, s);
}

}  // namespace

// Work-item counters of the persistent kernel: one per launch in flight, taken
// round-robin and zeroed in the launch's stream right before it.  Limit: at
// most 1024 persistent launches of one process may be in flight at once
// (across all streams and CUDA graphs; a graph that captured a launch keeps
// its counter word for good).  The 1025th concurrent launch would share a
// word with a running one, which would then skip work items.
__device__ unsigned g_item_ctr[1024];

// Kernel choice.  The one-CTA-per-tile kernel is the default: it measured
// 0.531 ms at rect bf16 (4,32,4096,128) against 0.528 ms for the persistent
// kernel (both with split PV / QK issuers), and ahead everywhere else
// (rect (4,32,2048,128) +2%, S = 8192 +3% rect / +13% differential).
// TDA_B200_FWD_PERSISTENT=1 selects the persistent kernel (=0 or unset: not).
static bool use_persistent_forward(bool /*differential*/, int /*head_dim*/, int /*n_qtiles*/) {
  static const bool forced = [] {
    const char* v = std::getenv("TDA_B200_FWD_PERSISTENT");
    return v && v[0] == '1';
  }();
  return forced;
}

// Device address of g_item_ctr on the current device, looked up once per
// device (the host-side symbol is only a stand-in for it).
static cudaError_t item_counters_on_current_device(unsigned** out) {
  constexpr int kMaxDevices = 64;
  static std::atomic<unsigned*> addr[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  unsigned* a = addr[dev].load(std::memory_order_acquire);
  if (!a) {
    e = cudaGetSymbolAddress(reinterpret_cast<void**>(&a), g_item_ctr);
    if (e != cudaSuccess) return e;
    addr[dev].store(a, std::memory_order_release);
  }
  *out = a;
  return cudaSuccess;
}

static cudaError_t prepare_item_counter(TcFwdParams& p, cudaStream_t stream) {
  static std::atomic<unsigned> next{0};
  unsigned* base = nullptr;
  cudaError_t e = item_counters_on_current_device(&base);
  if (e != cudaSuccess) return e;
  p.item_ctr = base + (next.fetch_add(1u) % 1024u);
  return cudaMemsetAsync(p.item_ctr, 0, sizeof(unsigned), stream);
}

// CTA-pair kernel (tda_tc_fwd_pair.cu) at head_dim 128: TDA_B200_FWD_PAIR=1
// selects it, =0 or unset the one-CTA-per-tile kernel.
static bool use_pair_forward(int head_dim) {
  static const bool on = [] {
    const char* v = std::getenv("TDA_B200_FWD_PAIR");
    return v && v[0] == '1';
  }();
  return on && head_dim == 128;
}

bool tc_fwd_uses_pair(int head_dim) {
  return use_pair_forward(head_dim) && !use_persistent_forward(false, head_dim, 0);
}

cudaError_t launch_tc_fwd(const TcFwdParams& p_in, int head_dim, bool differential, bool normalize, int pow_mode,
                          bool fp16, cudaStream_t stream) {
  TcFwdParams p = p_in;
  p.item_ctr = nullptr;
  if (tc_fwd_uses_pair(head_dim)) return launch_tc_fwd_pair(p, differential, normalize, pow_mode, fp16, stream);
  if (!fp16 && use_persistent_forward(differential, head_dim, p.n_qtiles)) {
    cudaError_t e = prepare_item_counter(p, stream);
    if (e != cudaSuccess) return e;
  }
  if (head_dim == 128) return dispatch_diff<128>(p, differential, normalize, pow_mode, fp16, stream);
  if (head_dim == 64) return dispatch_diff<64>(p, differential, normalize, pow_mode, fp16, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tda
