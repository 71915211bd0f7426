// Tensor-core (tcgen05 + TMEM + TMA) backward of one threshold rectified
// attention branch, bf16 operands, fp32 accumulation, head_dim 64 / 128.
//
// Gradients as the reference's backward kernels form them
// (triton_threshold_attention.py:118-224 for dQ, :227-324 for dK / dV), on
// F.normalize'd q, k when NORM (chain rule through F.normalize in the
// epilogues, as torch autograd applies it around the reference op, :505-512):
//   s_ij  = q_i . k_j (raw bf16 operands), 0 for j > i
//   z_ij  = s_ij rk_j rq_i - tau_i = (s_ij rk_j - tq_i) rq_i   (NORM; else s_ij - tau_i)
//   P_ij  = relu(z_ij)^p,  G_ij = d relu(z)^p / dz (z_ij)
//   dP_ij = g_i . v_j,  g = scale * dout
//   dA_ij = dP_ij G_ij           (not masked: with beta < 0 masked entries count, as in the reference)
//   dqh_i = sum_j dA_ij kh_j = sum_j (dA_ij rk_j) k_j
//   dkh_j = sum_i dA_ij qh_i = sum_i (dA_ij rq_i) q_i
//   dv_j  = sum_i P_ij g_i
// P and dA enter the tensor cores as bf16 hi + bf16 lo (~16 bits), two MMAs.
//
// dq kernel (one CTA = 128 query rows of one (batch, head)), the pipeline of
// the forward's differential kernel with the roles mapped
//   Q1 -> Q, Q2 -> dout, K1 -> K, K2 -> V, V -> K (dQ += dA K, K MN-major):
//   warp 0 TMA producer, warp 1 issues S = Q K^T and dQ += dA K, warp 10
//   issues dP = dout V^T into its single slot (released as soon as the
//   transform holds it in registers), warps 2-9 form dA over S in TMEM and
//   run the epilogue.  TMEM: S slots {0, 256}, dP at 128, dQ at 384.
// dkv kernel (one CTA = 128 keys of one (batch, head)), rows = keys: per
//   query tile S^T = K Q^T and dP^T = V dout^T, the transform writes P^T over
//   S^T and dA^T over dP^T, then dV += P^T dout and dK += dA^T Q.  TMEM:
//   S^T 0, dP^T 128, dV 256, dK 256 + D -- all 512 columns, so one query tile
//   is in flight at a time (one MMA issuer).
// Every mbarrier wait is bounded (WaitCtl), as in the forward.
#include <cuda_bf16.h>

#include <cstdio>

#include "tda_internal.h"
#include "tda_ptx.cuh"
#include "tda_transform.cuh"

namespace tda {
namespace {

using namespace tc;

constexpr int kTrWarps = 8;      // transform warps 2..9
constexpr int kQk2Warp = 10;     // dq kernel: dP issuer
constexpr int kRing4 = 4;
constexpr int kHeadGroup = 4;
constexpr int kSmemBudget = 232448;

constexpr int ST_BQ_PROD = 0x601, ST_BQ_MMA = 0x602, ST_BQ_TR = 0x603;
constexpr int ST_BK_PROD = 0x701, ST_BK_MMA = 0x702, ST_BK_TR = 0x703;

// d relu(z)^p / dz for a pair, as at triton_threshold_attention.py:195-206
template <int PM>
__device__ __forceinline__ float2 pgrad2(float2 z, float p) {
  const float2 x = relu2(z);
  if constexpr (PM == POW_1) {
    return make_float2(z.x > 0.f ? 1.f : 0.f, z.y > 0.f ? 1.f : 0.f);
  } else if constexpr (PM == POW_2) {
    return __fmul2_rn(make_float2(2.f, 2.f), x);
  } else if constexpr (PM == POW_3) {
    return __fmul2_rn(make_float2(3.f, 3.f), __fmul2_rn(x, x));
  } else {
    return make_float2(x.x > 0.f ? p * fast_ex2((p - 1.f) * fast_lg2(x.x + 1e-10f)) : 0.f,
                       x.y > 0.f ? p * fast_ex2((p - 1.f) * fast_lg2(x.y + 1e-10f)) : 0.f);
  }
}

// bf16 hi (truncated) + bf16 lo of a pair
__device__ __forceinline__ void split_hi_lo(float2 v, uint32_t& hi, uint32_t& lo) {
  const uint32_t p0 = __float_as_uint(v.x), p1 = __float_as_uint(v.y);
  hi = __byte_perm(p0, p1, 0x7632);
  const float2 l = sub2(v, f2u(p0 & 0xFFFF0000u, p1 & 0xFFFF0000u));
  lo = pack_bf16x2(l.x, l.y);
}

// 32 bf16 elements [col0, col0 + 32) of row r of a 128-row tile stored as
// D/64 swizzled 16 KB boxes (128-B rows, 16-B chunks XOR (r & 7)).
__device__ __forceinline__ void load_row32(const uint8_t* tile, int r, int col0, float (&x)[32]) {
  const uint8_t* base = tile + (col0 >> 6) * (kTile * 128) + r * 128;
  const int c0 = (col0 & 63) >> 3;
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const uint4 u = *reinterpret_cast<const uint4*>(base + (((c0 + k) ^ (r & 7)) << 4));
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      x[8 * k + 2 * h] = __uint_as_float(w[h] << 16);
      x[8 * k + 2 * h + 1] = __uint_as_float(w[h] & 0xFFFF0000u);
    }
  }
}

template <int D>
struct BCfg {
  static constexpr int kBoxes = D / 64;
  static constexpr int kBoxBytes = kTile * 128;
  static constexpr int kTileBytes = kTile * D * 2;
  static constexpr uint32_t kIdescQK = idesc_f16(128, 128, true, false);
  static constexpr uint32_t kIdescPV = idesc_f16(128, D, true, true);
};

// ================================================================== dq kernel
template <int D>
struct DqCfg : BCfg<D> {
  using B = BCfg<D>;
  static constexpr int kRkFloats = kRing4 * kTile;
  static constexpr int kBarBytes = 1024;
  static constexpr int kFixed = 2 * B::kTileBytes + kRkFloats * 4 + kBarBytes + 1024;
  static constexpr int kSlotsRaw = (kSmemBudget - kFixed) / B::kTileBytes;
  static constexpr int kSlots = kSlotsRaw > 8 ? 8 : kSlotsRaw;
  static_assert(kSlots >= 3, "not enough shared memory for the K/V ring");
  static_assert(kSlots * B::kTileBytes >= kTile * D * 4, "the ring must hold the fp32 dQ tile");
  static constexpr int kOffRing = 2 * B::kTileBytes;
  static constexpr int kOffRk = kOffRing + kSlots * B::kTileBytes;
  static constexpr int kOffBar = kOffRk + kRkFloats * 4;
  static constexpr int kSmemBytes = kOffBar + kBarBytes + 1024;
  static constexpr int kColS2 = 128;
  static constexpr int kColO = 384;
  static __device__ __forceinline__ uint32_t col_s(int slot) { return slot ? 256u : 0u; }
};

struct DqBars {
  uint64_t q_full, o_full, drain, drain2;
  uint64_t s_full[2], p_full[2], s2_free[2];
  uint64_t rk_full[kRing4], rk_empty[kRing4];
  uint64_t slot_full[8], slot_empty[8];
  uint32_t tmem_base;
  int abort_flag;
  uint32_t tile_mask[2];
};
static_assert(sizeof(DqBars) <= 1024, "barrier block too large");

// ring order per item: K_0, V_0, K_1, then per key tile j: V_{j+1}, K_j (dQ), K_{j+2}
__device__ __forceinline__ int ring_k(int m) { return m == 0 ? 0 : (m == 1 ? 2 : 3 * m - 1); }
__device__ __forceinline__ int ring_vv(int m) { return m == 0 ? 1 : 3 * m; }
__device__ __forceinline__ int ring_kq(int j, int n_kt) { return j <= n_kt - 2 ? 4 + 3 * j : 3 * n_kt - 1; }

__device__ __forceinline__ void item_of(const TcBwdParams& p, int& bh, int& t) {
  // groups of kHeadGroup heads; inside a group longest-first tiles, heads interleaved
  const int per_group = kHeadGroup * p.n_tiles;
  const int g0 = static_cast<int>(blockIdx.x / per_group) * kHeadGroup;
  const int gsz = min(kHeadGroup, p.BH - g0);
  const int r = static_cast<int>(blockIdx.x % per_group);
  bh = g0 + r % gsz;
  t = r / gsz;  // 0 = longest
}

template <int D, bool NORM>
__device__ void dq_producer(const TcBwdParams& p, uint8_t* smem, DqBars* bars, const WaitCtl& ctl, int bh, int qt,
                            int n_kt) {
  using C = DqCfg<D>;
  uint8_t* ring = smem + C::kOffRing;
  float* rk_s = reinterpret_cast<float*>(smem + C::kOffRk);
  mbar_arrive_expect_tx(&bars->q_full, 2 * C::kTileBytes);
#pragma unroll
  for (int b = 0; b < C::kBoxes; ++b) {
    tma_load_3d(smem + b * C::kBoxBytes, &p.tm_q, &bars->q_full, b * 64, qt * kTile, bh);
    tma_load_3d(smem + C::kTileBytes + b * C::kBoxBytes, &p.tm_do, &bars->q_full, b * 64, qt * kTile, bh);
  }
  int ridx = 0, rk_n = 0;
  bool ok = true;
  auto load_tile = [&](const CUtensorMap* map, int j) {
    if (!ok) return;
    const int slot = ridx % C::kSlots;
    if (!mbar_wait(&bars->slot_empty[slot], ((ridx / C::kSlots) & 1) ^ 1, ctl, ST_BQ_PROD)) {
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
      const int e = j % kRing4;
      if (!mbar_wait(&bars->rk_empty[e], ((j / kRing4) & 1) ^ 1, ctl, ST_BQ_PROD)) {
        ok = false;
        return;
      }
      mbar_arrive_expect_tx(&bars->rk_full[e], kTile * 4);
      bulk_load(rk_s + e * kTile, p.rk + static_cast<size_t>(bh) * p.S_pad + static_cast<size_t>(j) * kTile,
                kTile * 4, &bars->rk_full[e]);
      ++rk_n;
    }
  };
  load_rk(0);
  load_tile(&p.tm_k, 0);
  load_tile(&p.tm_v, 0);
  if (n_kt > 1) {
    load_rk(1);
    load_tile(&p.tm_k, 1);
  }
  for (int j = 0; j < n_kt && ok; ++j) {
    if (j + 1 < n_kt) load_tile(&p.tm_v, j + 1);
    load_tile(&p.tm_k, j);
    if (j + 2 < n_kt) {
      load_rk(j + 2);
      load_tile(&p.tm_k, j + 2);
    }
  }
  if (!ok) {
    drain_wait(&bars->q_full, 0, ctl);
    const int first = ridx > C::kSlots ? ridx - C::kSlots : 0;
    for (int i = first; i < ridx; ++i) drain_wait(&bars->slot_full[i % C::kSlots], (i / C::kSlots) & 1, ctl);
    const int rfirst = rk_n > kRing4 ? rk_n - kRing4 : 0;
    for (int i = rfirst; i < rk_n; ++i) drain_wait(&bars->rk_full[i % kRing4], (i / kRing4) & 1, ctl);
  }
}

template <int D, int NSLOT, typename Bars>
struct Mma {
  using B = BCfg<D>;
  Bars* bars;
  const WaitCtl& ctl;
  uint32_t tmem, ring_base;
  int code;
  bool ok = true;
  __device__ Mma(Bars* b, const WaitCtl& c, uint32_t t, uint32_t rb, int cd)
      : bars(b), ctl(c), tmem(t), ring_base(rb), code(cd) {}
  __device__ int acquire(int idx) {
    const int slot = idx % NSLOT;
    if (!ok) return slot;
    ok = mbar_wait(&bars->slot_full[slot], (idx / NSLOT) & 1, ctl, code);
    tc_fence_after();
    return slot;
  }
  __device__ uint32_t slot_addr(int slot) const { return ring_base + slot * B::kTileBytes; }
  // D[dcol] = A B^T over D, A and B K-major 128-row tiles
  __device__ void qk(uint32_t dcol, uint32_t a_base, uint32_t b_base) {
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      const uint32_t off = (kk >> 2) * B::kBoxBytes + (kk & 3) * 32;
      mma_ss(tmem + dcol, smem_desc_sw128(a_base + off, 16, 1024), smem_desc_sw128(b_base + off, 16, 1024),
             B::kIdescQK, kk > 0 ? 1u : 0u);
    }
  }
  // D[ocol] += A[pcol] (hi, lo in TMEM, forward P layout) X, X an MN-major
  // 128-row tile; only 16-row slabs in `mask`; `started` false -> overwrite
  __device__ void pv(uint32_t ocol, uint32_t pcol, uint32_t x_base, uint32_t mask, bool& started) {
    if (!started) mask |= 1u;
#pragma unroll
    for (int m = 0; m < kTile / 16; ++m) {
      if (!(mask & (1u << m))) continue;
      const uint64_t bdesc = smem_desc_sw128(x_base + m * 2048, B::kBoxBytes, 1024);
      const uint32_t a_hi = tmem + pcol + 32 * (m >> 1) + 8 * (m & 1);
      mma_ts(tmem + ocol, a_hi, bdesc, B::kIdescPV, started ? 1u : 0u);
      mma_ts(tmem + ocol, a_hi + 16, bdesc, B::kIdescPV, 1u);
      started = true;
    }
  }
  __device__ void wait(uint64_t* bar, uint32_t parity) {
    if (!ok) return;
    ok = mbar_wait(bar, parity, ctl, code);
    tc_fence_after();
  }
  __device__ void drain(uint64_t* bar) {
    tc_commit(bar);
    drain_wait(bar, 0, ctl);
  }
};

template <int D>
__device__ void dq_mma(uint8_t* smem, DqBars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = DqCfg<D>;
  Mma<D, C::kSlots, DqBars> m(bars, ctl, tmem, smem_u32(smem + C::kOffRing), ST_BQ_MMA);
  const uint32_t q_base = smem_u32(smem);
  m.wait(&bars->q_full, 0);
  bool started = false;
  auto qk1 = [&](int idx, uint32_t col, int slot_bar) {
    const int s = m.acquire(idx);
    if (!m.ok) return;
    m.qk(col, q_base, m.slot_addr(s));
    tc_commit(&bars->slot_empty[s]);
    tc_commit(&bars->s_full[slot_bar]);
  };
  qk1(ring_k(0), C::col_s(0), 0);
  if (n_kt > 1) qk1(ring_k(1), C::col_s(1), 1);
  for (int j = 0; j < n_kt && m.ok; ++j) {
    const int slot = j & 1;
    m.wait(&bars->p_full[slot], (j >> 1) & 1);
    const int s = m.acquire(ring_kq(j, n_kt));
    if (!m.ok) break;
    const uint32_t w = *reinterpret_cast<volatile uint32_t*>(&bars->tile_mask[slot]);
    const uint32_t mask = (w >> 8) == static_cast<uint32_t>(j + 1) ? (w & 0xFFu) : 0u;
    if (mask != 0u || !started) {
      m.pv(C::kColO, C::col_s(slot), m.slot_addr(s), mask, started);
      tc_commit(&bars->slot_empty[s]);
    } else {
      mbar_arrive(&bars->slot_empty[s]);
    }
    if (j + 2 < n_kt) qk1(ring_k(j + 2), C::col_s(slot), slot);
  }
  if (m.ok)
    tc_commit(&bars->o_full);
  else
    m.drain(&bars->drain);
}

template <int D>
__device__ void dq_mma_dp(uint8_t* smem, DqBars* bars, const WaitCtl& ctl, uint32_t tmem, int n_kt) {
  using C = DqCfg<D>;
  Mma<D, C::kSlots, DqBars> m(bars, ctl, tmem, smem_u32(smem + C::kOffRing), ST_BQ_MMA);
  const uint32_t do_base = smem_u32(smem) + C::kTileBytes;
  m.wait(&bars->q_full, 0);
  for (int j = 0; j < n_kt && m.ok; ++j) {
    if (j > 0) m.wait(&bars->s2_free[(j - 1) & 1], ((j - 1) >> 1) & 1);
    const int s = m.acquire(ring_vv(j));
    if (!m.ok) break;
    m.qk(C::kColS2, do_base, m.slot_addr(s));
    tc_commit(&bars->slot_empty[s]);
    tc_commit(&bars->s_full[j & 1]);
  }
  if (!m.ok) m.drain(&bars->drain2);
}

// One 32-key chunk of one query row: a = S (raw), b = dP; writes dA (hi, lo)
// over S.  Returns the 2-bit mask of 16-key halves with a nonzero dA.
template <int PM, bool NORM>
__device__ __forceinline__ uint32_t dq_chunk(uint32_t (&a)[32], const uint32_t (&b)[32], uint32_t s_addr,
                                             const float* rk, int limit, bool diag, float tq, float rq, float scale,
                                             float p) {
  if (diag) {
#pragma unroll
    for (int i = 0; i < 32; ++i) a[i] = (i <= limit) ? a[i] : 0u;
  }
  uint32_t nz = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = -3.0e38f;
#pragma unroll
    for (int q4 = 0; q4 < 4; ++q4) {
      float4 r = make_float4(1.f, 1.f, 1.f, 1.f);
      if constexpr (NORM) r = *reinterpret_cast<const float4*>(rk + 16 * h + 4 * q4);
#pragma unroll
      for (int t = 0; t < 2; ++t) {
        const int i = 16 * h + 4 * q4 + 2 * t;
        const float2 rr = t ? make_float2(r.z, r.w) : make_float2(r.x, r.y);
        const float2 y = NORM ? __ffma2_rn(f2u(a[i], a[i + 1]), rr, make_float2(-tq, -tq))
                              : __fadd2_rn(f2u(a[i], a[i + 1]), make_float2(-tq, -tq));
        a[i] = __float_as_uint(y.x);
        a[i + 1] = __float_as_uint(y.y);
        mx = max3f(mx, y.x, y.y);
      }
    }
    const bool lnz = mx > 0.0f;
    const bool any = __any_sync(0xffffffffu, lnz);
    nz |= lnz ? (1u << h) : 0u;
    uint32_t hi[8], lo[8];
    if (any) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = 16 * h + 2 * q;
        float2 z = f2u(a[i], a[i + 1]);
        if constexpr (NORM) z = __fmul2_rn(z, make_float2(rq, rq));
        float2 g = __fmul2_rn(pgrad2<PM>(z, p), __fmul2_rn(f2u(b[i], b[i + 1]), make_float2(scale, scale)));
        if constexpr (NORM) g = __fmul2_rn(g, *reinterpret_cast<const float2*>(rk + i));
        split_hi_lo(g, hi[q], lo[q]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) hi[q] = lo[q] = 0u;
    }
    tmem_st8(s_addr + 8 * h, hi);
    tmem_st8(s_addr + 16 + 8 * h, lo);
  }
  return nz;
}

template <int D, bool NORM, int PM>
__device__ void dq_transform(const TcBwdParams& p, uint8_t* smem, DqBars* bars, const WaitCtl& ctl, uint32_t tmem,
                             int bh, int qt, int n_kt, int warp, int lane) {
  using C = DqCfg<D>;
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;
  const int grow = qt * kTile + row;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float* rk_s = reinterpret_cast<const float*>(smem + C::kOffRk);
  const float2 qc = p.qc[static_cast<size_t>(bh) * p.S_pad + grow];
  const float rq = qc.x, tq = qc.y;
  bool ok = true;
  for (int j = 0; j < n_kt && ok; ++j) {
    const int re = j % kRing4;
    if constexpr (NORM) {
      ok = mbar_wait_warp(&bars->rk_full[re], (j / kRing4) & 1, ctl, ST_BQ_TR);
      if (!ok) break;
    }
    ok = mbar_wait_warp(&bars->s_full[j & 1], (j >> 1) & 1, ctl, ST_BQ_TR);
    if (!ok) break;
    tc_fence_after();
    const uint32_t scol = C::col_s(j & 1);
    const int ch0 = 2 * wg;
    uint32_t a[32], b[32], b1[32];
    tmem_ld32(tmem + lane_off + scol + 32 * ch0, a);
    tmem_ld32(tmem + lane_off + C::kColS2 + 32 * ch0, b);
    tmem_ld32(tmem + lane_off + C::kColS2 + 32 * (ch0 + 1), b1);
    tmem_wait_ld();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&bars->s2_free[j & 1]);  // dP slot free for the next tile
    const int limit0 = grow - j * kTile;
    const bool diag = j >= qt;
    uint32_t nz = 0;
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      const int ch = ch0 + cc;
      if (cc == 1) {
        tmem_ld32(tmem + lane_off + scol + 32 * ch, a);
#pragma unroll
        for (int i = 0; i < 32; ++i) b[i] = b1[i];
        tmem_wait_ld();
      }
      nz |= dq_chunk<PM, NORM>(a, b, tmem + lane_off + scol + 32 * ch, rk_s + re * kTile + 32 * ch,
                               limit0 - 32 * ch, diag, tq, rq, p.scale, p.relu_power)
            << (2 * cc);
    }
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, nz) << (4 * wg);
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
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) {
      mbar_arrive(&bars->p_full[j & 1]);
      if constexpr (NORM) mbar_arrive(&bars->rk_empty[re]);
    }
  }
  // epilogue: dq = rq (dqh - (dqh . qh) qh) with qh = q rq (NORM), else dqh.
  // fp32 rows are staged in the idle K/V ring (128-B swizzled 32-column
  // boxes) and written by TMA stores: coalesced, rows past S clipped.  Every
  // transform thread reaches the barrier, also one whose wait gave up.
  if (ok) ok = mbar_wait_warp(&bars->o_full, 0, ctl, ST_BQ_TR);
  uint8_t* stage = smem + C::kOffRing;
  if (ok) {
    tc_fence_after();
    float dot = 0.f;
    if constexpr (NORM) {
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        float x[32];
        tmem_ld32(tmem + lane_off + C::kColO + c0, o);
        load_row32(smem, row, c0, x);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) dot = fmaf(__uint_as_float(o[t]), x[t], dot);
      }
      dot *= rq;  // dqh . qh
    }
    const bool big = rq < 1e12f;
    uint8_t* srow = stage + row * 128;
    const uint32_t sw = static_cast<uint32_t>(row & 7);
#pragma unroll 1
    for (int c0 = wg * (D / 2); c0 < (wg + 1) * (D / 2); c0 += 32) {
      uint32_t o[32];
      float x[32];
      tmem_ld32(tmem + lane_off + C::kColO + c0, o);
      if constexpr (NORM) load_row32(smem, row, c0, x);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < 32; t += 4) {
        float v[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          float g = __uint_as_float(o[t + e]);
          if constexpr (NORM) g = rq * (big ? g - dot * x[t + e] * rq : g);
          v[e] = g;
        }
        const int c = c0 + t;  // box c / 32, 16-B chunk (c % 32) / 4
        *reinterpret_cast<float4*>(srow + (c >> 5) * C::kBoxBytes + ((((c & 31) >> 2) ^ sw) << 4)) =
            make_float4(v[0], v[1], v[2], v[3]);
      }
    }
    fence_proxy_async_smem();
  }
  ok = named_barrier_and(2, 32 * kTrWarps, ok);
  if (ok && warp == 2 && lane == 0) {
    for (int b = 0; b < D / 32; ++b) tma_store_3d(&p.tm_dq, stage + b * C::kBoxBytes, b * 32, qt * kTile, bh);
    bulk_commit_group();
    bulk_wait_group_read0();  // the shared-memory source stays valid until read
  }
}

template <int D, bool NORM, bool POS, int PM>
__global__ void __maxnreg__(168) tda_tc_bwd_dq_kernel(const __grid_constant__ TcBwdParams p) {
  using C = DqCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DqBars* bars = reinterpret_cast<DqBars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int bh, t;
  item_of(p, bh, t);
  const int qt = p.n_tiles - 1 - t;
  const int n_kt = POS ? qt + 1 : p.n_tiles;
  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->drain2, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->s_full[i], 2);
      mbar_init(&bars->p_full[i], kTrWarps);
      mbar_init(&bars->s2_free[i], kTrWarps);
      bars->tile_mask[i] = 0;
    }
    for (int i = 0; i < kRing4; ++i) {
      mbar_init(&bars->rk_full[i], 1);
      mbar_init(&bars->rk_empty[i], kTrWarps);
    }
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    bars->abort_flag = 0;
    fence_mbar_init();
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
    if (lane == 0) dq_producer<D, NORM>(p, smem, bars, ctl, bh, qt, n_kt);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) dq_mma<D>(smem, bars, ctl, tmem, n_kt);
    __syncwarp();
  } else if (warp < kQk2Warp) {
    dq_transform<D, NORM, PM>(p, smem, bars, ctl, tmem, bh, qt, n_kt, warp, lane);
  } else {
    if (lane == 0) dq_mma_dp<D>(smem, bars, ctl, tmem, n_kt);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================== dkv kernel
template <int D>
struct DkvCfg : BCfg<D> {
  using B = BCfg<D>;
  static constexpr int kQcFloats = kRing4 * kTile * 2;
  static constexpr int kBarBytes = 1024;
  static constexpr int kFixed = 2 * B::kTileBytes + kQcFloats * 4 + kBarBytes + 1024;
  static constexpr int kSlotsRaw = (kSmemBudget - kFixed) / B::kTileBytes;
  static constexpr int kSlots = kSlotsRaw > 8 ? 8 : kSlotsRaw;
  static_assert(kSlots >= 2, "not enough shared memory for the Q/dout ring");
  static_assert(kSlots * B::kTileBytes >= 2 * kTile * D * 4, "the ring must hold the fp32 dK and dV tiles");
  static constexpr int kOffRing = 2 * B::kTileBytes;
  static constexpr int kOffQc = kOffRing + kSlots * B::kTileBytes;
  static constexpr int kOffBar = kOffQc + kQcFloats * 4;
  static constexpr int kSmemBytes = kOffBar + kBarBytes + 1024;
  static constexpr int kColP = 0, kColA = 128, kColDV = 256, kColDK = 256 + D;
};

struct DkvBars {
  uint64_t kv_full, o_full, drain, s_full, p_full;
  uint64_t qc_full[kRing4], qc_empty[kRing4];
  uint64_t slot_full[8], slot_empty[8];
  uint32_t tmem_base;
  int abort_flag;
  uint32_t tile_mask;
};
static_assert(sizeof(DkvBars) <= 1024, "barrier block too large");

template <int D>
__device__ void dkv_producer(const TcBwdParams& p, uint8_t* smem, DkvBars* bars, const WaitCtl& ctl, int bh, int kt,
                             int i0, int n_steps) {
  using C = DkvCfg<D>;
  uint8_t* ring = smem + C::kOffRing;
  float2* qc_s = reinterpret_cast<float2*>(smem + C::kOffQc);
  mbar_arrive_expect_tx(&bars->kv_full, 2 * C::kTileBytes);
#pragma unroll
  for (int b = 0; b < C::kBoxes; ++b) {
    tma_load_3d(smem + b * C::kBoxBytes, &p.tm_k, &bars->kv_full, b * 64, kt * kTile, bh);
    tma_load_3d(smem + C::kTileBytes + b * C::kBoxBytes, &p.tm_v, &bars->kv_full, b * 64, kt * kTile, bh);
  }
  int ridx = 0, qn = 0;
  bool ok = true;
  auto load_tile = [&](const CUtensorMap* map, int i) {
    if (!ok) return;
    const int slot = ridx % C::kSlots;
    if (!mbar_wait(&bars->slot_empty[slot], ((ridx / C::kSlots) & 1) ^ 1, ctl, ST_BK_PROD)) {
      ok = false;
      return;
    }
    mbar_arrive_expect_tx(&bars->slot_full[slot], C::kTileBytes);
    uint8_t* dst = ring + slot * C::kTileBytes;
#pragma unroll
    for (int b = 0; b < C::kBoxes; ++b) tma_load_3d(dst + b * C::kBoxBytes, map, &bars->slot_full[slot], b * 64, i * kTile, bh);
    ++ridx;
  };
  for (int t = 0; t < n_steps && ok; ++t) {
    const int i = i0 + t;
    const int e = t % kRing4;
    if (!mbar_wait(&bars->qc_empty[e], ((t / kRing4) & 1) ^ 1, ctl, ST_BK_PROD)) {
      ok = false;
      break;
    }
    mbar_arrive_expect_tx(&bars->qc_full[e], kTile * 8);
    bulk_load(qc_s + e * kTile, p.qc + static_cast<size_t>(bh) * p.S_pad + static_cast<size_t>(i) * kTile,
              kTile * 8, &bars->qc_full[e]);
    ++qn;
    load_tile(&p.tm_q, i);
    load_tile(&p.tm_do, i);
  }
  if (!ok) {
    drain_wait(&bars->kv_full, 0, ctl);
    const int first = ridx > C::kSlots ? ridx - C::kSlots : 0;
    for (int k = first; k < ridx; ++k) drain_wait(&bars->slot_full[k % C::kSlots], (k / C::kSlots) & 1, ctl);
    const int qfirst = qn > kRing4 ? qn - kRing4 : 0;
    for (int k = qfirst; k < qn; ++k) drain_wait(&bars->qc_full[k % kRing4], (k / kRing4) & 1, ctl);
  }
}

template <int D>
__device__ void dkv_mma(uint8_t* smem, DkvBars* bars, const WaitCtl& ctl, uint32_t tmem, int n_steps) {
  using C = DkvCfg<D>;
  Mma<D, C::kSlots, DkvBars> m(bars, ctl, tmem, smem_u32(smem + C::kOffRing), ST_BK_MMA);
  const uint32_t k_base = smem_u32(smem), v_base = k_base + C::kTileBytes;
  m.wait(&bars->kv_full, 0);
  bool dv_started = false, dk_started = false;
  for (int t = 0; t < n_steps && m.ok; ++t) {
    const int sq = m.acquire(2 * t);
    const int sd = m.acquire(2 * t + 1);
    if (!m.ok) break;
    m.qk(C::kColP, k_base, m.slot_addr(sq));   // S^T = K Q^T
    m.qk(C::kColA, v_base, m.slot_addr(sd));   // dP^T = V dout^T
    tc_commit(&bars->s_full);
    m.wait(&bars->p_full, t & 1);
    if (!m.ok) break;
    const uint32_t w = *reinterpret_cast<volatile uint32_t*>(&bars->tile_mask);
    const uint32_t mask = (w >> 8) == static_cast<uint32_t>(t + 1) ? (w & 0xFFu) : 0u;
    if (mask != 0u || !dv_started) m.pv(C::kColDV, C::kColP, m.slot_addr(sd), mask, dv_started);  // dV += P^T dout
    if (mask != 0u || !dk_started) m.pv(C::kColDK, C::kColA, m.slot_addr(sq), mask, dk_started);  // dK += dA^T Q
    tc_commit(&bars->slot_empty[sq]);
    tc_commit(&bars->slot_empty[sd]);
  }
  if (m.ok)
    tc_commit(&bars->o_full);
  else
    m.drain(&bars->drain);
}

// One 32-query chunk of one key row: a = S^T, b = dP^T; writes P^T (hi, lo)
// over S^T and dA^T (hi, lo, times rq_i) over dP^T.  qc: this chunk's 32
// query coefficients {rq, tq}; query columns c < mlim are masked (key after
// query).  Returns the 2-bit mask of 16-query halves with nonzero output.
template <int PM, bool NORM>
__device__ __forceinline__ uint32_t dkv_chunk(uint32_t (&a)[32], const uint32_t (&b)[32], uint32_t p_addr,
                                              uint32_t a_addr, const float2* qc, int mlim, float rk, float scale,
                                              float p) {
  if (mlim > 0) {
#pragma unroll
    for (int i = 0; i < 32; ++i) a[i] = (i < mlim) ? 0u : a[i];
  }
  uint32_t nz = 0;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    float mx = -3.0e38f;
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const int i = 16 * h + 2 * q;
      const float4 c2 = *reinterpret_cast<const float4*>(qc + i);  // {rq_i, tq_i, rq_i+1, tq_i+1}
      const float2 s = f2u(a[i], a[i + 1]);
      const float2 y = NORM ? __ffma2_rn(s, make_float2(rk, rk), make_float2(-c2.y, -c2.w))
                            : __fadd2_rn(s, make_float2(-c2.y, -c2.w));
      a[i] = __float_as_uint(y.x);
      a[i + 1] = __float_as_uint(y.y);
      mx = max3f(mx, y.x, y.y);
    }
    const bool lnz = mx > 0.0f;
    const bool any = __any_sync(0xffffffffu, lnz);
    nz |= lnz ? (1u << h) : 0u;
    uint32_t phi[8], plo[8], ahi[8], alo[8];
    if (any) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int i = 16 * h + 2 * q;
        const float4 c2 = *reinterpret_cast<const float4*>(qc + i);
        float2 z = f2u(a[i], a[i + 1]);
        if constexpr (NORM) z = __fmul2_rn(z, make_float2(c2.x, c2.z));
        const float2 u = relu2(z);
        const float2 P = __fmul2_rn(pow2v<PM>(u, p), make_float2(scale, scale));
        float2 g = __fmul2_rn(pgrad2<PM>(z, p), __fmul2_rn(f2u(b[i], b[i + 1]), make_float2(scale, scale)));
        if constexpr (NORM) g = __fmul2_rn(g, make_float2(c2.x, c2.z));
        split_hi_lo(P, phi[q], plo[q]);
        split_hi_lo(g, ahi[q], alo[q]);
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) phi[q] = plo[q] = ahi[q] = alo[q] = 0u;
    }
    tmem_st8(p_addr + 8 * h, phi);
    tmem_st8(p_addr + 16 + 8 * h, plo);
    tmem_st8(a_addr + 8 * h, ahi);
    tmem_st8(a_addr + 16 + 8 * h, alo);
  }
  return nz;
}

template <int D, bool NORM, int PM>
__device__ void dkv_transform(const TcBwdParams& p, uint8_t* smem, DkvBars* bars, const WaitCtl& ctl,
                              uint32_t tmem, int bh, int kt, int i0, int n_steps, int warp, int lane) {
  using C = DkvCfg<D>;
  const int wg = (warp - 2) >> 2;
  const int quarter = warp & 3;
  const int row = quarter * 32 + lane;  // key within the tile
  const int gkey = kt * kTile + row;
  const uint32_t lane_off = static_cast<uint32_t>(quarter * 32) << 16;
  const float2* qc_s = reinterpret_cast<const float2*>(smem + C::kOffQc);
  float rk = 1.0f;
  if constexpr (NORM) rk = p.rk[static_cast<size_t>(bh) * p.S_pad + gkey];
  bool ok = mbar_wait_warp(&bars->kv_full, 0, ctl, ST_BK_TR);
  for (int t = 0; t < n_steps && ok; ++t) {
    const int i = i0 + t;
    const int e = t % kRing4;
    ok = mbar_wait_warp(&bars->qc_full[e], (t / kRing4) & 1, ctl, ST_BK_TR);
    if (!ok) break;
    ok = mbar_wait_warp(&bars->s_full, t & 1, ctl, ST_BK_TR);
    if (!ok) break;
    tc_fence_after();
    uint32_t nz = 0;
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      const int ch = 2 * wg + cc;
      uint32_t a[32], b[32];
      tmem_ld32(tmem + lane_off + C::kColP + 32 * ch, a);
      tmem_ld32(tmem + lane_off + C::kColA + 32 * ch, b);
      tmem_wait_ld();
      // query column c of this chunk is masked when its query precedes the key
      const int mlim = gkey - (i * kTile + 32 * ch);
      nz |= dkv_chunk<PM, NORM>(a, b, tmem + lane_off + C::kColP + 32 * ch, tmem + lane_off + C::kColA + 32 * ch,
                                qc_s + e * kTile + 32 * ch, mlim, rk, p.scale, p.relu_power)
            << (2 * cc);
    }
    const uint32_t wmask = __reduce_or_sync(0xffffffffu, nz) << (4 * wg);
    if (wmask != 0u && lane == 0) {
      uint32_t* word = &bars->tile_mask;
      const uint32_t tag = static_cast<uint32_t>(t + 1) << 8;
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
      mbar_arrive(&bars->p_full);
      mbar_arrive(&bars->qc_empty[e]);
    }
  }
  // epilogue: dV and dkh -> dk = rk (dkh - (dkh . kh) kh) (NORM), fp32 rows
  // staged in the idle Q/dout ring (dK boxes, then dV boxes) and written by
  // TMA; with accumulate_dv the dV tile is added into global memory by a TMA
  // reduce-add.  Every transform thread reaches the barrier.
  if (ok) ok = mbar_wait_warp(&bars->o_full, 0, ctl, ST_BK_TR);
  uint8_t* stage_k = smem + C::kOffRing;
  uint8_t* stage_v = stage_k + (D / 32) * C::kBoxBytes;
  if (ok) {
    tc_fence_after();
    float dot = 0.f;
    if constexpr (NORM) {
#pragma unroll 1
      for (int c0 = 0; c0 < D; c0 += 32) {
        uint32_t o[32];
        float x[32];
        tmem_ld32(tmem + lane_off + C::kColDK + c0, o);
        load_row32(smem, row, c0, x);
        tmem_wait_ld();
#pragma unroll
        for (int t = 0; t < 32; ++t) dot = fmaf(__uint_as_float(o[t]), x[t], dot);
      }
      dot *= rk;  // dkh . kh
    }
    const bool big = rk < 1e12f;
    const uint32_t sw = static_cast<uint32_t>(row & 7);
#pragma unroll 1
    for (int c0 = wg * (D / 2); c0 < (wg + 1) * (D / 2); c0 += 32) {
      uint32_t ok_[32], ov[32];
      float x[32];
      tmem_ld32(tmem + lane_off + C::kColDK + c0, ok_);
      tmem_ld32(tmem + lane_off + C::kColDV + c0, ov);
      if constexpr (NORM) load_row32(smem, row, c0, x);
      tmem_wait_ld();
#pragma unroll
      for (int t = 0; t < 32; t += 4) {
        float kv[4];
#pragma unroll
        for (int e2 = 0; e2 < 4; ++e2) {
          float g = __uint_as_float(ok_[t + e2]);
          if constexpr (NORM) g = rk * (big ? g - dot * x[t + e2] * rk : g);
          kv[e2] = g;
        }
        const int c = c0 + t;  // box c / 32, 16-B chunk (c % 32) / 4
        const uint32_t off = row * 128 + (c >> 5) * C::kBoxBytes + ((((c & 31) >> 2) ^ sw) << 4);
        *reinterpret_cast<float4*>(stage_k + off) = make_float4(kv[0], kv[1], kv[2], kv[3]);
        *reinterpret_cast<uint4*>(stage_v + off) = make_uint4(ov[t], ov[t + 1], ov[t + 2], ov[t + 3]);
      }
    }
    fence_proxy_async_smem();
  }
  ok = named_barrier_and(2, 32 * kTrWarps, ok);
  if (ok && warp == 2 && lane == 0) {
    for (int b = 0; b < D / 32; ++b) {
      tma_store_3d(&p.tm_dk, stage_k + b * C::kBoxBytes, b * 32, kt * kTile, bh);
      if (p.accumulate_dv)
        tma_reduce_add_3d(&p.tm_dv, stage_v + b * C::kBoxBytes, b * 32, kt * kTile, bh);
      else
        tma_store_3d(&p.tm_dv, stage_v + b * C::kBoxBytes, b * 32, kt * kTile, bh);
    }
    bulk_commit_group();
    bulk_wait_group_read0();  // the shared-memory sources stay valid until read
  }
}

template <int D, bool NORM, bool POS, int PM>
__global__ void __maxnreg__(168) tda_tc_bwd_dkv_kernel(const __grid_constant__ TcBwdParams p) {
  using C = DkvCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DkvBars* bars = reinterpret_cast<DkvBars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int bh, t;
  item_of(p, bh, t);
  const int kt = t;  // key tiles near the start see the most query tiles
  const int i0 = POS ? kt : 0;
  const int n_steps = p.n_tiles - i0;
  if (threadIdx.x == 0) {
    mbar_init(&bars->kv_full, 1);
    mbar_init(&bars->o_full, 1);
    mbar_init(&bars->drain, 1);
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->p_full, kTrWarps);
    for (int i = 0; i < kRing4; ++i) {
      mbar_init(&bars->qc_full[i], 1);
      mbar_init(&bars->qc_empty[i], kTrWarps);
    }
    for (int i = 0; i < C::kSlots; ++i) {
      mbar_init(&bars->slot_full[i], 1);
      mbar_init(&bars->slot_empty[i], 1);
    }
    bars->tile_mask = 0;
    bars->abort_flag = 0;
    fence_mbar_init();
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
    if (lane == 0) dkv_producer<D>(p, smem, bars, ctl, bh, kt, i0, n_steps);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) dkv_mma<D>(smem, bars, ctl, tmem, n_steps);
    __syncwarp();
  } else {
    dkv_transform<D, NORM, PM>(p, smem, bars, ctl, tmem, bh, kt, i0, n_steps, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

// ================================================================== query table
template <int D>
__global__ void __launch_bounds__(256) query_table_kernel(const __nv_bfloat16* __restrict__ x, float2* __restrict__ qc,
                                                          int BH, int S, int S_pad, float beta, int normalize) {
  constexpr int kLanesPerRow = D * 2 / 16;
  constexpr int kRowsPerIter = 32 / kLanesPerRow;
  const int lane = threadIdx.x & 31;
  const int sub = lane / kLanesPerRow, sl = lane % kLanesPerRow;
  const long long rows = static_cast<long long>(BH) * S_pad;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long r0 = ((static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5) * kRowsPerIter;
       r0 < rows; r0 += n_warps * kRowsPerIter) {
    const long long r = r0 + sub;
    const int bh = static_cast<int>(r / S_pad), i = static_cast<int>(r % S_pad);
    float ss = 0.f;
    if (r < rows && i < S) {
      const uint4 u = reinterpret_cast<const uint4*>(x + (static_cast<size_t>(bh) * S + i) * D)[sl];
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float lo = __uint_as_float(w[h] << 16), hi = __uint_as_float(w[h] & 0xFFFF0000u);
        ss = fmaf(lo, lo, ss);
        ss = fmaf(hi, hi, ss);
      }
    }
#pragma unroll
    for (int off = kLanesPerRow / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (r < rows && sl == 0) {
      float2 c;
      if (i >= S) {
        c = make_float2(0.0f, 3.0e38f);
      } else {
        // tau(i) = beta * sqrt(2 * log(i + 1) / D) (triton_threshold_attention.py:62-63)
        const float tau = beta * sqrtf((2.0f * logf(static_cast<float>(i + 1))) / static_cast<float>(D));
        if (normalize) {
          const float m = fmaxf(sqrtf(ss), 1e-12f);
          c = make_float2(1.0f / m, tau * m);
        } else {
          c = make_float2(1.0f, tau);
        }
      }
      qc[r] = c;
    }
  }
}

template <int D, bool NORM, bool POS, int PM>
cudaError_t launch_bwd_one(const TcBwdParams& p, cudaStream_t stream) {
  auto kq = tda_tc_bwd_dq_kernel<D, NORM, POS, PM>;
  auto kkv = tda_tc_bwd_dkv_kernel<D, NORM, POS, PM>;
  static bool attr_done = false;
  if (!attr_done) {
    cudaError_t e = cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, DqCfg<D>::kSmemBytes);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, DkvCfg<D>::kSmemBytes);
    if (e != cudaSuccess) return e;
    attr_done = true;
  }
  const unsigned grid = static_cast<unsigned>(p.BH) * static_cast<unsigned>(p.n_tiles);
  kq<<<grid, 32 * 11, DqCfg<D>::kSmemBytes, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kkv<<<grid, 32 * 10, DkvCfg<D>::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

template <int D, bool NORM, bool POS>
cudaError_t bwd_pow(const TcBwdParams& p, int pm, cudaStream_t s) {
  switch (pm) {
    case POW_1: return launch_bwd_one<D, NORM, POS, POW_1>(p, s);
    case POW_2: return launch_bwd_one<D, NORM, POS, POW_2>(p, s);
    case POW_3: return launch_bwd_one<D, NORM, POS, POW_3>(p, s);
    default: return launch_bwd_one<D, NORM, POS, POW_GENERAL>(p, s);
  }
}

template <int D>
cudaError_t bwd_dispatch(const TcBwdParams& p, bool norm, int pm, cudaStream_t s) {
  if (norm) return p.causal_skip ? bwd_pow<D, true, true>(p, pm, s) : bwd_pow<D, true, false>(p, pm, s);
  return p.causal_skip ? bwd_pow<D, false, true>(p, pm, s) : bwd_pow<D, false, false>(p, pm, s);
}

template <int D>
cudaError_t launch_qt(const void* q, float2* qc, int BH, int S, int S_pad, float beta, int normalize,
                      cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int kRowsPerWarp = 32 / (D * 2 / 16);
  const long long rows = static_cast<long long>(BH) * S_pad;
  long long blocks = (rows / kRowsPerWarp + 7) / 8;
  const long long cap = static_cast<long long>(sms) * 16;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  query_table_kernel<D><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(q), qc,
                                                                            BH, S, S_pad, beta, normalize);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_query_table(const void* q, float2* qc, int BH, int S, int S_pad, int D, float beta, int normalize,
                               cudaStream_t stream) {
  if (D == 64) return launch_qt<64>(q, qc, BH, S, S_pad, beta, normalize, stream);
  if (D == 128) return launch_qt<128>(q, qc, BH, S, S_pad, beta, normalize, stream);
  return cudaErrorInvalidValue;
}

cudaError_t launch_tc_bwd(const TcBwdParams& p, int head_dim, bool normalize, int pow_mode, cudaStream_t stream) {
  if (head_dim == 64) return bwd_dispatch<64>(p, normalize, pow_mode, stream);
  if (head_dim == 128) return bwd_dispatch<128>(p, normalize, pow_mode, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tda
