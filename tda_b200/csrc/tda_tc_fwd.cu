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

#include <cstdio>

#include "tda_internal.h"
#include "tda_ptx.cuh"

namespace tda {
namespace {

constexpr int kTransformWG = 2;                    // transform warpgroups
constexpr int kTransformWarps = 4 * kTransformWG;  // warps 2 .. 17
constexpr int kThreads = 32 * (2 + kTransformWarps);
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
  uint64_t s2_free[2];  // differential: every transform warp has read S2 of the tile
  uint64_t rk_full[kRkRing];
  uint64_t rk_empty[kRkRing];
  uint64_t slot_full[8];
  uint64_t slot_empty[8];
  uint32_t tmem_base;
  int abort_flag;
  // per key tile (by parity): (j + 1) << 8 | mask of 16-key slabs with a
  // nonzero P; stale words carry an older tag and read as mask 0
  uint32_t tile_mask[2];
};
static_assert(sizeof(Bars) <= 1024, "barrier block too large");

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
  // 32 keys, hi at pcol + 32c + [0,16), lo at pcol + 32c + [16,32).  Only the
  // 16-key slabs set in `mask` are multiplied (the others hold P = 0); the
  // first PV of the CTA initialises O (accumulate = 0) and therefore always
  // issues at least its first slab.
  bool o_started = false;
  auto pv = [&](uint32_t pcol, uint32_t mask) {
    int slot;
    acquire(slot);
    if (!ok) return;
    if (!o_started) mask |= 1u;
    if (mask == 0u) {
      mbar_arrive(&bars->slot_empty[slot]);
      return;
    }
    const uint32_t v_base = ring_base + slot * C::kTileBytes;
#pragma unroll
    for (int m = 0; m < kTile / 16; ++m) {
      if (!(mask & (1u << m))) continue;
      const uint64_t bdesc = smem_desc_sw128(v_base + m * 2048, C::kBoxBytes, 1024);
      const uint32_t a_hi = tmem + pcol + 32 * (m >> 1) + 8 * (m & 1);
      mma_ts(tmem + C::kColO, a_hi, bdesc, C::kIdescPV, o_started ? 1u : 0u);
      mma_ts(tmem + C::kColO, a_hi + 16, bdesc, C::kIdescPV, 1u);
      o_started = true;
    }
    tc_commit(&bars->slot_empty[slot]);
  };
  auto slab_mask = [&](int j) -> uint32_t {
    const uint32_t w = *reinterpret_cast<volatile uint32_t*>(&bars->tile_mask[j & 1]);
    return (w >> 8) == static_cast<uint32_t>(j + 1) ? (w & 0xFFu) : 0u;
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
      pv(col, slab_mask(j));
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
      if (j + 1 < n_kt) {
        // S2 has one TMEM slot: it is free once every transform warp holds
        // S2_j in registers, long before P_j is ready
        ok = mbar_wait(&bars->s2_free[j & 1], (j >> 1) & 1, ctl, ST_MMA_P);
        tc_fence_after();
        qk(C::kColS2, q2_base);
        if (ok) tc_commit(&bars->s_full[(j + 1) & 1]);
      }
      wait_p(j);
      pv(col, slab_mask(j));
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
// Per-row coefficients: z = (s * rk_j - tq) * rq for each branch.  With
// normalize, tq = tau * m and rq = 1 / m, m = max(||q_i||, 1e-12), so z is the
// normalized score minus tau.  For p in {1, 2, 3} the differential weight is
// folded into the second branch, rq2 *= lambda^(1/p), because
// relu(c z)^p = c^p relu(z)^p for c >= 0; the general power keeps an explicit
// lambda multiply.
struct RowCoef {
  float tq1, rq1, tq2, rq2;
};

__device__ __forceinline__ float2 f2u(uint32_t x, uint32_t y) {
  return make_float2(__uint_as_float(x), __uint_as_float(y));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float2 relu2(float2 z) { return make_float2(fmaxf(z.x, 0.0f), fmaxf(z.y, 0.0f)); }

template <int PM>
__device__ __forceinline__ float2 relu_pow2(float2 z, float p) {
  const float2 u = relu2(z);
  if constexpr (PM == POW_1) {
    return u;
  } else if constexpr (PM == POW_2) {
    return __fmul2_rn(u, u);
  } else if constexpr (PM == POW_3) {
    return __fmul2_rn(__fmul2_rn(u, u), u);
  } else {
    // exp(p * log(x + 1e-10)) for x > 0 (triton_threshold_attention.py:97-101)
    return make_float2(u.x > 0.0f ? fast_ex2(p * fast_lg2(u.x + 1e-10f)) : 0.0f,
                       u.y > 0.0f ? fast_ex2(p * fast_lg2(u.y + 1e-10f)) : 0.0f);
  }
}

// One 32-key chunk of one row, from registers (a = S1, b = S2 as loaded from
// TMEM) to P written over S1 in TMEM as bf16 hi (columns [0,16)) and lo
// ([16,32)).  First pass computes y = s * rk - tq for every entry and its max;
// P is nonzero only where y > 0, so when no lane of the warp has a positive y
// the chunk is written as zeros without the power / combine / split work
// (exact, and the common case for the sparse threshold maps TDA produces).
// Returns this lane's 2-bit mask of 16-key halves holding a nonzero P.
template <int PM, bool DIFF, bool NORM, bool MASK>
__device__ __forceinline__ uint32_t transform_chunk(uint32_t (&a)[32], uint32_t (&b)[32], uint32_t s1_addr,
                                                    const float* rk1, const float* rk2, int limit, const RowCoef& c,
                                                    float relu_power, float lam) {
  constexpr bool kFold = PM != POW_GENERAL;
  float mx[2] = {-3.0e38f, -3.0e38f};  // max y over keys [0,16) and [16,32)
#pragma unroll
  for (int e4 = 0; e4 < 8; ++e4) {
    float4 r1 = make_float4(1.f, 1.f, 1.f, 1.f), r2 = r1;
    if constexpr (NORM) {
      r1 = *reinterpret_cast<const float4*>(rk1 + 4 * e4);
      if constexpr (DIFF) r2 = *reinterpret_cast<const float4*>(rk2 + 4 * e4);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int i = 4 * e4 + 2 * h;
      uint32_t x0 = a[i], x1 = a[i + 1];
      if constexpr (MASK) {
        x0 = (i <= limit) ? x0 : 0u;
        x1 = (i + 1 <= limit) ? x1 : 0u;
      }
      const float2 rr = h ? make_float2(r1.z, r1.w) : make_float2(r1.x, r1.y);
      const float2 y = NORM ? __ffma2_rn(f2u(x0, x1), rr, make_float2(-c.tq1, -c.tq1))
                            : __fadd2_rn(f2u(x0, x1), make_float2(-c.tq1, -c.tq1));
      a[i] = __float_as_uint(y.x);
      a[i + 1] = __float_as_uint(y.y);
      mx[e4 >> 2] = max3f(mx[e4 >> 2], y.x, y.y);
      if constexpr (DIFF) {
        uint32_t w0 = b[i], w1 = b[i + 1];
        if constexpr (MASK) {
          w0 = (i <= limit) ? w0 : 0u;
          w1 = (i + 1 <= limit) ? w1 : 0u;
        }
        const float2 rs = h ? make_float2(r2.z, r2.w) : make_float2(r2.x, r2.y);
        const float2 y2 = NORM ? __ffma2_rn(f2u(w0, w1), rs, make_float2(-c.tq2, -c.tq2))
                               : __fadd2_rn(f2u(w0, w1), make_float2(-c.tq2, -c.tq2));
        b[i] = __float_as_uint(y2.x);
        b[i + 1] = __float_as_uint(y2.y);
        mx[e4 >> 2] = max3f(mx[e4 >> 2], y2.x, y2.y);
      }
    }
  }
  const uint32_t nz = (mx[0] > 0.0f ? 1u : 0u) | (mx[1] > 0.0f ? 2u : 0u);
  if (__any_sync(0xffffffffu, nz != 0u)) {
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      uint32_t hi[8], lo[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int e2 = 8 * half + q;
        const float2 y1 = f2u(a[2 * e2], a[2 * e2 + 1]);
        const float2 z1 = NORM ? __fmul2_rn(y1, make_float2(c.rq1, c.rq1)) : y1;
        float2 P;
        if constexpr (DIFF) {
          const float2 y2 = f2u(b[2 * e2], b[2 * e2 + 1]);
          const float2 z2 = (NORM || kFold) ? __fmul2_rn(y2, make_float2(c.rq2, c.rq2)) : y2;
          if constexpr (PM == POW_2) {
            const float2 u1 = relu2(z1), u2 = relu2(z2);
            P = __ffma2_rn(u1, u1, __fmul2_rn(u2, make_float2(-u2.x, -u2.y)));
          } else if constexpr (kFold) {
            const float2 p2 = relu_pow2<PM>(z2, relu_power);
            P = __fadd2_rn(relu_pow2<PM>(z1, relu_power), make_float2(-p2.x, -p2.y));
          } else {
            P = __ffma2_rn(make_float2(-lam, -lam), relu_pow2<PM>(z2, relu_power),
                           relu_pow2<PM>(z1, relu_power));
          }
        } else {
          P = relu_pow2<PM>(z1, relu_power);
        }
        // hi = P truncated to bf16 (exact in fp32), lo = bf16(P - hi): hi + lo
        // carries ~16 significant bits of P.
        const uint32_t p0 = __float_as_uint(P.x), p1 = __float_as_uint(P.y);
        hi[q] = __byte_perm(p0, p1, 0x7632);
        const float2 l = __fadd2_rn(P, make_float2(-__uint_as_float(p0 & 0xFFFF0000u),
                                                   -__uint_as_float(p1 & 0xFFFF0000u)));
        lo[q] = pack_bf16x2(l.x, l.y);
      }
      tmem_st8(s1_addr + 8 * half, hi);
      tmem_st8(s1_addr + 16 + 8 * half, lo);
    }
  } else {
    const uint32_t zero[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
    tmem_st8(s1_addr, zero);
    tmem_st8(s1_addr + 8, zero);
    tmem_st8(s1_addr + 16, zero);
    tmem_st8(s1_addr + 24, zero);
  }
  return nz;
}

// Transform warps: warp w (2 <= w < 2 + kTransformWarps) owns TMEM lane
// quarter w % 4 (query rows) and, as warpgroup g = (w - 2) / 4, the key
// chunks [g kChunks, (g+1) kChunks) of every key tile (32 keys each) and the
// output columns [g D/kTransformWG, (g+1) D/kTransformWG).
template <int D, bool DIFF, bool NORM, int PM>
__device__ void run_transform(const TcFwdParams& p, uint8_t* smem, Bars* bars, const WaitCtl& ctl, uint32_t tmem,
                              int bh, int qt, int n_kt, int warp, int lane) {
  using C = Cfg<D, DIFF>;
  constexpr bool kFold = PM != POW_GENERAL;
  constexpr int kChunks = 4 / kTransformWG;  // 32-key chunks per thread per tile
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int q0 = qt * kTile;
  const int grow = q0 + row;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float* rk_s = reinterpret_cast<const float*>(smem + C::kOffRk);

  // tau(i) = beta * sqrt(2 * log(i + 1) / D) in fp32 (triton_threshold_attention.py:62-63)
  const float tau = p.beta * sqrtf((2.0f * logf(static_cast<float>(grow + 1))) / static_cast<float>(D));
  const float lam2 = (DIFF && kFold) ? p.lam_root : 1.0f;
  RowCoef c{tau, 1.0f, tau, lam2};
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
        for (int bx = 0; bx < C::kBoxes; ++bx) {
#pragma unroll
          for (int cc = 0; cc < 8; ++cc) {
            const uint4 u = *reinterpret_cast<const uint4*>(qb + bx * C::kBoxBytes + ((cc ^ (row & 7)) << 4));
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
      c.rq1 = 1.0f / m1;
      c.tq1 = tau * m1;
      if constexpr (DIFF) {
        const float m2 = fmaxf(sqrtf(ss[1]), 1e-12f);
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
    ok = mbar_wait_warp(&bars->s_full[j & 1], (j >> 1) & 1, ctl, ST_TR_S);
    if (!ok) break;
    tc_fence_after();
    const uint32_t s1col = DIFF ? ((j & 1) ? 256u : 0u) : static_cast<uint32_t>((j & 1) * 128);
    // all of this thread's S (and S2) columns in one round of TMEM loads
    uint32_t a[kChunks][32];
    uint32_t b[kChunks][32];
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      const int ch = wg * kChunks + cc;
      tmem_ld32(tmem + lane_off + s1col + 32 * ch, a[cc]);
      if constexpr (DIFF) tmem_ld32(tmem + lane_off + C::kColS2 + 32 * ch, b[cc]);
    }
    tmem_wait_ld();
    if constexpr (DIFF) {
      // S2 is in registers: hand its TMEM slot back so QK2 of the next tile
      // runs on the tensor cores while this tile is transformed
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&bars->s2_free[j & 1]);
    }
    uint32_t nz = 0;  // bit (2 cc + h): 16-key half h of chunk cc has a nonzero P
#pragma unroll
    for (int cc = 0; cc < kChunks; ++cc) {
      const int ch = wg * kChunks + cc;
      const uint32_t s1 = tmem + lane_off + s1col + 32 * ch;
      const float* r1 = rk_s + re * C::kRkPerTile + 32 * ch;
      const float* r2 = r1 + kTile;
      const int limit = grow - (j * kTile + 32 * ch);
      if (j >= qt)  // tile overlaps the causal diagonal
        nz |= transform_chunk<PM, DIFF, NORM, true>(a[cc], b[cc], s1, r1, r2, limit, c, p.relu_power, p.lam)
              << (2 * cc);
      else
        nz |= transform_chunk<PM, DIFF, NORM, false>(a[cc], b[cc], s1, r1, r2, limit, c, p.relu_power, p.lam)
              << (2 * cc);
    }
    // publish which 16-key slabs of this tile hold a nonzero P (this
    // warpgroup owns slabs [2 kChunks wg, 2 kChunks (wg + 1))); slabs nobody
    // marks are skipped by the PV.  The p_full arrive below orders the store
    // before the MMA warp reads the word.
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, nz) << (2 * kChunks * wg);
    if (wmask != 0u && lane == 0) {
      uint32_t* word = &bars->tile_mask[j & 1];
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
      mbar_arrive(&bars->p_full[j & 1]);
      if constexpr (NORM) mbar_arrive(&bars->rk_empty[re]);
    }
  }

  // epilogue: O (f32 in TMEM) -> global, D / kTransformWG columns per warpgroup
  if (ok) ok = mbar_wait_warp(&bars->o_full, 0, ctl, ST_TR_O);
  if (!ok) return;
  tc_fence_after();
  constexpr int kCols = D / kTransformWG;
  static_assert(kCols % 32 == 0, "epilogue reads 32-column chunks");
  const bool row_ok = grow < p.S;
  const size_t row_off = (static_cast<size_t>(bh) * p.S + (row_ok ? grow : 0)) * D;
#pragma unroll
  for (int c0 = 0; c0 < kCols; c0 += 32) {
    const int col = wg * kCols + c0;
    uint32_t o[32];
    tmem_ld32(tmem + lane_off + C::kColO + col, o);
    tmem_wait_ld();
    if (!row_ok) continue;
    if (p.out_f32) {
      float4* dst = reinterpret_cast<float4*>(static_cast<float*>(p.out) + row_off + col);
#pragma unroll
      for (int t = 0; t < 8; ++t)
        dst[t] = make_float4(__uint_as_float(o[4 * t]), __uint_as_float(o[4 * t + 1]), __uint_as_float(o[4 * t + 2]),
                             __uint_as_float(o[4 * t + 3]));
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

template <int D, bool DIFF, bool NORM, int PM>
__global__ void __maxnreg__(168) tda_tc_fwd_kernel(const __grid_constant__ TcFwdParams p) {
  using C = Cfg<D, DIFF>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Head-major order, longest query tile first within a head: the CTAs in
  // flight at any time cover only a few (batch, head) slices, so each K/V tile
  // is read from HBM about once and then served from L2 to every query tile
  // of that head.
  const int bh = static_cast<int>(blockIdx.x / p.n_qtiles);
  const int qt = p.n_qtiles - 1 - static_cast<int>(blockIdx.x % p.n_qtiles);
  const int n_kt = p.causal_skip ? qt + 1 : p.n_qtiles;

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], kTransformWarps);
      mbar_init(&bars->s2_free[i], kTransformWarps);
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
    bars->tile_mask[0] = 0;
    bars->tile_mask[1] = 0;
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
