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
//   warp 1      MMA issuer (one thread): S = Q K^T into TMEM (SS form), and
//               O += P V with P read from TMEM (TS form).
//   warps 2-9   two transform warpgroups; each thread owns one query row
//               (its TMEM lane), warpgroup g handles key columns [64g, 64g+64)
//               of every tile: S -> threshold -> ReLU^p (-> combine) ->
//               bf16 hi + bf16 lo split of P written back over S in TMEM.
//               They also run the epilogue (O from TMEM -> global).
//
// P precision: P is stored as bf16 hi + bf16 lo (P = hi + lo to ~16 bits) and
// multiplied into O by two MMAs; a single bf16 P misses the 1e-3 accuracy gate.
//
// Every mbarrier wait is bounded (WaitCtl): on timeout the CTA records a code
// in the status word, drains its in-flight copies / MMAs, frees TMEM and exits.
#include <cuda_bf16.h>

#include "tda_internal.h"
#include "tda_ptx.cuh"

namespace tda {
namespace {

constexpr int kThreads = 320;
constexpr int kRkRing = 4;
constexpr int kSmemBudget = 232448;  // 227 KB opt-in dynamic shared memory

// status codes (role << 8 | site)
constexpr int ST_PROD_SLOT = 0x101, ST_PROD_RK = 0x102;
constexpr int ST_MMA_Q = 0x201, ST_MMA_SLOT = 0x202, ST_MMA_P = 0x203;
constexpr int ST_TR_Q = 0x301, ST_TR_RK = 0x302, ST_TR_S = 0x303, ST_TR_O = 0x304;
constexpr int ST_DRAIN = 0x401;

template <int D, bool DIFF>
struct Cfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = kTile * 128;  // 128 rows x 64 bf16 (128 B)
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr int kNQ = DIFF ? 2 : 1;
  static constexpr int kRkPerTile = (DIFF ? 2 : 1) * kTile;
  static constexpr int kRkFloats = kRkRing * kRkPerTile;
  static constexpr int kBarBytes = 1024;
  static constexpr int kFixed = kNQ * kTileBytes + kRkFloats * 4 + kBarBytes + 1024;
  static constexpr int kSlotsRaw = (kSmemBudget - kFixed) / kTileBytes;
  static constexpr int kSlots = kSlotsRaw > 8 ? 8 : kSlotsRaw;
  static_assert(kSlots >= 3, "not enough shared memory for the K/V ring");
  static constexpr int kOffRing = kNQ * kTileBytes;
  static constexpr int kOffRk = kOffRing + kSlots * kTileBytes;
  static constexpr int kOffBar = kOffRk + kRkFloats * 4;
  static constexpr int kSmemBytes = kOffBar + kBarBytes + 1024;
  // TMEM columns (512 allocated): rect S slots {0,128}, O at 256;
  // diff S1 slots {0,256}, S2 slot 128, O at 384.
  static constexpr int kColS2 = 128;
  static constexpr int kColO = DIFF ? 384 : 256;
  static constexpr uint32_t kIdescQK = idesc_f16(128, 128, true, false);
  static constexpr uint32_t kIdescPV = idesc_f16(128, D, true, true);
};

struct Bars {
  uint64_t q_full;
  uint64_t o_full;
  uint64_t drain;
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t rk_full[kRkRing];
  uint64_t rk_empty[kRkRing];
  uint64_t slot_full[8];
  uint64_t slot_empty[8];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Bars) <= 1024, "barrier block too large");

template <int PM>
__device__ __forceinline__ float relu_pow(float z, float p) {
  const float x = fmaxf(z, 0.0f);
  if constexpr (PM == POW_1) {
    return x;
  } else if constexpr (PM == POW_2) {
    return x * x;
  } else if constexpr (PM == POW_3) {
    return x * x * x;
  } else {
    // exp(p * log(x + 1e-10)) for x > 0 (triton_threshold_attention.py:97-101)
    return x > 0.0f ? fast_ex2(p * fast_lg2(x + 1e-10f)) : 0.0f;
  }
}

// Drain-time wait: ignores the abort flag, bounded by its own timeout.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity, const WaitCtl& ctl) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(a, parity)) {
    if (global_timer_ns() - t0 > ctl.timeout_ns) {
      atomicCAS(ctl.status, 0, ST_DRAIN);
      return;
    }
  }
}

// ------------------------------------------------------------------ producer
template <int D, bool DIFF, bool NORM>
__device__ void run_producer(const TcFwdParams& p, uint8_t* smem, Bars* bars, const WaitCtl& ctl, int bh, int qt,
                             int n_kt) {
  using C = Cfg<D, DIFF>;
  uint8_t* ring = smem + C::kOffRing;
  float* rk_s = reinterpret_cast<float*>(smem + C::kOffRk);
  const int q0 = qt * kTile;
  bool q_issued = false;
  if (!(p.inject & 1)) {
    mbar_arrive_expect_tx(&bars->q_full, C::kNQ * C::kTileBytes);
#pragma unroll
    for (int b = 0; b < C::kBoxes; ++b) {
      tma_load_3d(smem + b * C::kBoxBytes, &p.tm_q1, &bars->q_full, b * 64, q0, bh);
      if constexpr (DIFF)
        tma_load_3d(smem + C::kTileBytes + b * C::kBoxBytes, &p.tm_q2, &bars->q_full, b * 64, q0, bh);
    }
    q_issued = true;
  }

  int ridx = 0;    // tiles issued into the ring
  int rk_n = 0;    // rk ring entries issued
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
    for (int b = 0; b < C::kBoxes; ++b) tma_load_3d(dst + b * C::kBoxBytes, map, &bars->slot_full[slot], b * 64, j * kTile, bh);
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
      const size_t off = static_cast<size_t>(bh) * p.S_pad + static_cast<size_t>(j) * kTile;
      bulk_load(dst, p.rk1 + off, kTile * 4, &bars->rk_full[e]);
      if constexpr (DIFF) bulk_load(dst + kTile, p.rk2 + off, kTile * 4, &bars->rk_full[e]);
      ++rk_n;
    }
  };

  if constexpr (!DIFF) {
    // consumption order: K0, K1, then per j: V_j, K_{j+2}
    load_rk(0);
    load_tile(&p.tm_k1, 0);
    if (n_kt > 1) {
      load_rk(1);
      load_tile(&p.tm_k1, 1);
    }
    for (int j = 0; j < n_kt && ok; ++j) {
      load_tile(&p.tm_v, j);
      if (j + 2 < n_kt) {
        load_rk(j + 2);
        load_tile(&p.tm_k1, j + 2);
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

// ------------------------------------------------------------------ MMA issuer
template <int D, bool DIFF>
__device__ void run_mma(uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = Cfg<D, DIFF>;
  const uint32_t q1_base = smem_u32(smem);
  const uint32_t q2_base = q1_base + C::kTileBytes;
  const uint32_t ring_base = smem_u32(smem + C::kOffRing);
  bool ok = mbar_wait(&bars->q_full, 0, ctl, ST_MMA_Q);
  tc_fence_after();
  int ridx = 0;

  auto acquire = [&](int& slot) {
    slot = ridx % C::kSlots;
    const uint32_t par = (ridx / C::kSlots) & 1;
    ++ridx;
    if (!ok) return;
    ok = mbar_wait(&bars->slot_full[slot], par, ctl, ST_MMA_SLOT);
    tc_fence_after();
  };
  // S[dcol] = Q K^T over D in UMMA_K = 16 steps (32 B inside a 128-B swizzled row).
  auto qk = [&](uint32_t dcol, uint32_t q_base) {
    int slot;
    acquire(slot);
    if (!ok) return;
    const uint32_t k_base = ring_base + slot * C::kTileBytes;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * C::kBoxBytes + (kk & 3) * 32;
      mma_ss(tmem + dcol, smem_desc_sw128(q_base + off, 16, 1024), smem_desc_sw128(k_base + off, 16, 1024),
             C::kIdescQK, kk > 0 ? 1u : 0u);
    }
    tc_commit(&bars->slot_empty[slot]);
  };
  // O += P V, P (hi, lo) in TMEM columns [pcol, pcol+128): for key chunk c of
  // 32 keys, hi at pcol + 32c + [0,16), lo at pcol + 32c + [16,32).
  auto pv = [&](uint32_t pcol, bool accumulate) {
    int slot;
    acquire(slot);
    if (!ok) return;
    const uint32_t v_base = ring_base + slot * C::kTileBytes;
#pragma unroll
    for (int m = 0; m < kTile / 16; ++m) {
      const uint64_t bdesc = smem_desc_sw128(v_base + m * 2048, C::kBoxBytes, 1024);
      const uint32_t a_hi = tmem + pcol + 32 * (m >> 1) + 8 * (m & 1);
      mma_ts(tmem + C::kColO, a_hi, bdesc, C::kIdescPV, (accumulate || m > 0) ? 1u : 0u);
      mma_ts(tmem + C::kColO, a_hi + 16, bdesc, C::kIdescPV, 1u);
    }
    tc_commit(&bars->slot_empty[slot]);
  };
  auto wait_p = [&](int j) {
    if (!ok) return;
    ok = mbar_wait(&bars->p_full[j & 1], (j >> 1) & 1, ctl, ST_MMA_P);
    tc_fence_after();
  };

  if constexpr (!DIFF) {
    qk(0, q1_base);
    if (ok) tc_commit(&bars->s_full[0]);
    if (n_kt > 1) {
      qk(128, q1_base);
      if (ok) tc_commit(&bars->s_full[1]);
    }
    for (int j = 0; j < n_kt && ok; ++j) {
      const uint32_t col = (j & 1) * 128;
      wait_p(j);
      pv(col, j > 0);
      if (j + 2 < n_kt) {
        qk(col, q1_base);
        if (ok) tc_commit(&bars->s_full[j & 1]);
      }
    }
  } else {
    qk(0, q1_base);
    qk(C::kColS2, q2_base);
    if (ok) tc_commit(&bars->s_full[0]);
    if (n_kt > 1) qk(256, q1_base);
    for (int j = 0; j < n_kt && ok; ++j) {
      const uint32_t col = (j & 1) ? 256 : 0;
      wait_p(j);
      if (j + 1 < n_kt) {
        qk(C::kColS2, q2_base);
        if (ok) tc_commit(&bars->s_full[(j + 1) & 1]);
      }
      pv(col, j > 0);
      if (j + 2 < n_kt) qk(col, q1_base);
    }
  }
  if (ok) {
    tc_commit(&bars->o_full);
  } else {
    // Abort: let every MMA already issued finish before TMEM is freed.
    tc_commit(&bars->drain);
    drain_wait(&bars->drain, 0, ctl);
  }
}

// ------------------------------------------------------------------ transform
template <int PM, bool DIFF, bool NORM, bool MASK>
__device__ __forceinline__ void transform_chunk(uint32_t s1_addr, uint32_t s2_addr, const float* rk1,
                                                const float* rk2, int limit, float tq1, float rq1, float tq2,
                                                float rq2, float tau, float relu_power, float lam) {
  uint32_t a[32];
  uint32_t b[32];
  tmem_ld32(s1_addr, a);
  if constexpr (DIFF) tmem_ld32(s2_addr, b);
  tmem_wait_ld();
  float P[32];
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    float4 r1 = make_float4(1.f, 1.f, 1.f, 1.f), r2 = r1;
    if constexpr (NORM) {
      r1 = *reinterpret_cast<const float4*>(rk1 + 4 * e4);
      if constexpr (DIFF) r2 = *reinterpret_cast<const float4*>(rk2 + 4 * e4);
    }
    const float rr1[4] = {r1.x, r1.y, r1.z, r1.w};
    const float rr2[4] = {r2.x, r2.y, r2.z, r2.w};
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const int e = 4 * e4 + t;
      float s1 = __uint_as_float(a[e]);
      if constexpr (MASK) s1 = (e <= limit) ? s1 : 0.0f;
      const float z1 = NORM ? fmaf(s1, rr1[t], -tq1) * rq1 : s1 - tau;
      float pe = relu_pow<PM>(z1, relu_power);
      if constexpr (DIFF) {
        float s2 = __uint_as_float(b[e]);
        if constexpr (MASK) s2 = (e <= limit) ? s2 : 0.0f;
        const float z2 = NORM ? fmaf(s2, rr2[t], -tq2) * rq2 : s2 - tau;
        pe = fmaf(-lam, relu_pow<PM>(z2, relu_power), pe);
      }
      P[e] = pe;
    }
  }
  uint32_t hi[16], lo[16];
#pragma unroll
  for (int e2 = 0; e2 < 16; ++e2) {
    const float x0 = P[2 * e2], x1 = P[2 * e2 + 1];
    const uint32_t h = pack_bf16x2(x0, x1);
    hi[e2] = h;
    lo[e2] = pack_bf16x2(x0 - __uint_as_float(h << 16), x1 - __uint_as_float(h & 0xFFFF0000u));
  }
  tmem_st16(s1_addr, hi);
  tmem_st16(s1_addr + 16, lo);
}

template <int D, bool DIFF, bool NORM, int PM>
__device__ void run_transform(const TcFwdParams& p, uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem,
                              int bh, int qt, int n_kt, int warp, int lane) {
  using C = Cfg<D, DIFF>;
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int q0 = qt * kTile;
  const int grow = q0 + row;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float* rk_s = reinterpret_cast<const float*>(smem + C::kOffRk);

  // tau(i) = beta * sqrt(2 * log(i + 1) / D) in fp32 (triton_threshold_attention.py:62-63)
  const float tau = p.beta * sqrtf((2.0f * logf(static_cast<float>(grow + 1))) / static_cast<float>(D));
  float tq1 = tau, rq1 = 1.0f, tq2 = tau, rq2 = 1.0f;
  bool ok = true;
  if constexpr (NORM) {
    ok = mbar_wait_warp(&bars->q_full, 0, ctl, ST_TR_Q);
    if (ok) {
      // ||q_i|| from the swizzled tile: row r's 16-B chunks are permuted
      // within the row only, so summing all chunks needs no unswizzle; the
      // chunk visit order is rotated by (r & 7) to avoid bank conflicts.
      float ss[2] = {0.f, 0.f};
#pragma unroll
      for (int t = 0; t < C::kNQ; ++t) {
        const uint8_t* qb = smem + t * C::kTileBytes + row * 128;
#pragma unroll
        for (int b = 0; b < C::kBoxes; ++b) {
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const uint4 u = *reinterpret_cast<const uint4*>(qb + b * C::kBoxBytes + ((c ^ (row & 7)) << 4));
            const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const float lo = __uint_as_float(w[h] << 16), hi = __uint_as_float(w[h] & 0xFFFF0000u);
              ss[t] = fmaf(lo, lo, ss[t]);
              ss[t] = fmaf(hi, hi, ss[t]);
            }
          }
        }
      }
      const float m1 = fmaxf(sqrtf(ss[0]), 1e-12f);
      rq1 = 1.0f / m1;
      tq1 = tau * m1;
      if constexpr (DIFF) {
        const float m2 = fmaxf(sqrtf(ss[1]), 1e-12f);
        rq2 = 1.0f / m2;
        tq2 = tau * m2;
      }
    }
  }

  for (int j = 0; j < n_kt && ok; ++j) {
    const int re = j % kRkRing;
    if constexpr (NORM) {
      ok = mbar_wait_warp(&bars->rk_full[re], (j / kRkRing) & 1, ctl, ST_TR_RK);
      if (!ok) break;
    }
    ok = mbar_wait_warp(&bars->s_full[j & 1], (j >> 1) & 1, ctl, ST_TR_S);
    if (!ok) break;
    tc_fence_after();
    const uint32_t s1col = DIFF ? ((j & 1) ? 256u : 0u) : static_cast<uint32_t>((j & 1) * 128);
    const bool need_mask = j >= qt;
#pragma unroll
    for (int cc = 0; cc < 2; ++cc) {
      const int c = wg * 2 + cc;
      const uint32_t s1 = tmem + lane_off + s1col + 32 * c;
      const uint32_t s2 = tmem + lane_off + C::kColS2 + 32 * c;
      const float* r1 = rk_s + re * C::kRkPerTile + 32 * c;
      const float* r2 = r1 + kTile;
      const int limit = grow - (j * kTile + 32 * c);
      if (need_mask)
        transform_chunk<PM, DIFF, NORM, true>(s1, s2, r1, r2, limit, tq1, rq1, tq2, rq2, tau, p.relu_power, p.lam);
      else
        transform_chunk<PM, DIFF, NORM, false>(s1, s2, r1, r2, limit, tq1, rq1, tq2, rq2, tau, p.relu_power, p.lam);
    }
    tmem_wait_st();
    tc_fence_before();
    mbar_arrive(&bars->p_full[j & 1]);
    if constexpr (NORM) mbar_arrive(&bars->rk_empty[re]);
  }

  // epilogue: O (f32 in TMEM) -> global
  if (ok) ok = mbar_wait_warp(&bars->o_full, 0, ctl, ST_TR_O);
  if (!ok) return;
  tc_fence_after();
  const bool row_ok = grow < p.S;
  const size_t row_off = (static_cast<size_t>(bh) * p.S + (row_ok ? grow : 0)) * D;
#pragma unroll
  for (int cc = 0; cc < D / 64; ++cc) {
    const int col = wg * (D / 2) + 32 * cc;
    uint32_t o[32];
    tmem_ld32(tmem + lane_off + C::kColO + col, o);
    tmem_wait_ld();
    if (row_ok) {
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
}

template <int D, bool DIFF, bool NORM, int PM>
__global__ void __launch_bounds__(kThreads, 1) tda_tc_fwd_kernel(const __grid_constant__ TcFwdParams p) {
  using C = Cfg<D, DIFF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Longest-first order: the first wave holds the query tiles with the most
  // causal key tiles.
  const int bh = blockIdx.x % p.BH;
  const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x / p.BH);
  const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], 256);
    }
    for (int i = 0; i < kRkRing; ++i) {
      mbar_init(&bars->rk_full[i], 1);
      mbar_init(&bars->rk_empty[i], 256);
    }
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
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
  const WaitCtl ctl{&bars->abort_flag, p.status, p.timeout_ns};

  if (warp == 0) {
    if (lane == 0) run_producer<D, DIFF, NORM>(p, smem, bars, ctl, bh, qt, n_kt);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) run_mma<D, DIFF>(smem, bars, ctl, tmem, n_kt);
    __syncwarp();
  } else {
    run_transform<D, DIFF, NORM, PM>(p, smem, bars, ctl, tmem, bh, qt, n_kt, warp, lane);
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D, bool DIFF, bool NORM, int PM>
cudaError_t launch_one(const TcFwdParams& p, cudaStream_t stream) {
  using C = Cfg<D, DIFF>;
  auto kern = tda_tc_fwd_kernel<D, DIFF, NORM, PM>;
  static bool attr_done = false;  // per instantiation; attribute is per-function, idempotent
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const unsigned grid = static_cast<unsigned>(p.BH) * static_cast<unsigned>(p.n_qtiles);
  kern<<<grid, kThreads, C::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

template <int D, bool DIFF, bool NORM>
cudaError_t dispatch_pow(const TcFwdParams& p, int pm, cudaStream_t s) {
  switch (pm) {
    case POW_1: return launch_one<D, DIFF, NORM, POW_1>(p, s);
    case POW_2: return launch_one<D, DIFF, NORM, POW_2>(p, s);
    case POW_3: return launch_one<D, DIFF, NORM, POW_3>(p, s);
    default: return launch_one<D, DIFF, NORM, POW_GENERAL>(p, s);
  }
}

template <int D, bool DIFF>
cudaError_t dispatch_norm(const TcFwdParams& p, bool norm, int pm, cudaStream_t s) {
  return norm ? dispatch_pow<D, DIFF, true>(p, pm, s) : dispatch_pow<D, DIFF, false>(p, pm, s);
}

template <int D>
cudaError_t dispatch_diff(const TcFwdParams& p, bool diff, bool norm, int pm, cudaStream_t s) {
  return diff ? dispatch_norm<D, true>(p, norm, pm, s) : dispatch_norm<D, false>(p, norm, pm, s);
}

}  // namespace

cudaError_t launch_tc_fwd(const TcFwdParams& p, int head_dim, bool differential, bool normalize, int pow_mode,
                          cudaStream_t stream) {
  if (head_dim == 128) return dispatch_diff<128>(p, differential, normalize, pow_mode, stream);
  if (head_dim == 64) return dispatch_diff<64>(p, differential, normalize, pow_mode, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tda
