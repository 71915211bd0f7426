// Device code of the tensor-core forward kernel's transform warps: the
// per-chunk score transform and the drain-time wait.
#pragma once

#include <cuda_bf16.h>

#include "tda_internal.h"
#include "tda_ptx.cuh"

namespace tda {
namespace tc {

// status codes (role << 8 | site)
constexpr int ST_DRAIN = 0x401;

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

// ------------------------------------------------------------------ transform
// Per-row coefficients: z = (s * rk_j - tq) * rq for each branch.  With
// normalize, tq = tau * m and rq = 1 / m, m = max(||q_i||, 1e-12), so z is the
// normalized score minus tau.  For p in {1, 2, 3} the differential weight is
// folded into the second branch, rq2 *= lambda^(1/p), because
// relu(c z)^p = c^p relu(z)^p for c >= 0; the general power keeps an explicit
// lambda multiply.
struct RowCoef {
  float tq1, rq1, tq2, rq2;
  float lam;  // clamped lambda of this (batch, head) (the general power's explicit weight)
};

// lambda^(1/p) for the folded powers (lambda itself for the general one, which
// weights the second branch explicitly).
template <int PM>
__device__ __forceinline__ float lambda_root(float lam) {
  if constexpr (PM == POW_2) return sqrtf(lam);
  if constexpr (PM == POW_3) return cbrtf(lam);
  return lam;
}

__device__ __forceinline__ float2 f2u(uint32_t x, uint32_t y) {
  return make_float2(__uint_as_float(x), __uint_as_float(y));
}

__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float2 relu2(float2 z) { return make_float2(fmaxf(z.x, 0.0f), fmaxf(z.y, 0.0f)); }

__device__ __forceinline__ float2 sub2(float2 a, float2 b) {
  unsigned long long r;
  asm("sub.rn.f32x2 %0, %1, %2;"
      : "=l"(r)
      : "l"((static_cast<unsigned long long>(__float_as_uint(a.y)) << 32) | __float_as_uint(a.x)),
        "l"((static_cast<unsigned long long>(__float_as_uint(b.y)) << 32) | __float_as_uint(b.x)));
  return make_float2(__uint_as_float(static_cast<uint32_t>(r)), __uint_as_float(static_cast<uint32_t>(r >> 32)));
}

__device__ __forceinline__ float mul_sat(float a, float b) {
  float r;
  asm("mul.rn.sat.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

// relu(y * r).  SAT: the caller guarantees y * r <= 1 (normalized scores with
// beta >= 0: cos - tau <= 1), so the saturating multiply's clamp to [0, 1]
// is exactly the ReLU and costs nothing extra.
template <bool SAT>
__device__ __forceinline__ float2 scaled_relu(float2 y, float r) {
  if constexpr (SAT) {
    return make_float2(mul_sat(y.x, r), mul_sat(y.y, r));
  } else {
    return relu2(__fmul2_rn(y, make_float2(r, r)));
  }
}

// u^p for u >= 0 (u already ReLU'd).
template <int PM>
__device__ __forceinline__ float2 pow2v(float2 u, float p) {
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
// ([16,32)).  P is nonzero only where y = s * rk - tq > 0, so each 16-key half
// in which no lane of the warp can have a positive y is written as zeros
// without the power / combine / split work (exact; the common case for the
// sparse threshold maps TDA produces).
//   diag: the tile holds the causal diagonal; scores of keys past the row
//     (index > limit) are replaced by 0 first, as the reference masks them
//     (triton_threshold_attention.py:79-80).
//   POS (beta >= 0, tq >= 0): first from the raw scores alone,
//     max_j s_j * max_j rk_j <= tq implies s_j rk_j <= tq for every j of the
//     half (rkm = per-16-key max of rk; without normalize max_j s_j <= tau is
//     already exact); a half this bound cannot clear gets y formed and tested
//     exactly before any further work.  Masked zeros give y = -tq <= 0.
//   otherwise (beta < 0): y is formed for every entry.
// ROLL: the halves run through one rolled loop (the second half is shifted
// into the first half's registers), which keeps the code small in the
// instruction cache at the cost of the register moves.  rk1/rk2: this chunk's 32 inverse key norms; rkm1/rkm2:
// the maxima of its two halves.  Returns this lane's 2-bit mask of halves
// holding a nonzero P.
// F16: the operands are fp16 (q, k, v), so P is written as fp16 hi + lo of
// P * pscale (a power of two that keeps P in fp16's normal range; the
// epilogue divides it out exactly).
template <int PM, bool DIFF, bool NORM, bool POS, bool ROLL, bool F16 = false>
__device__ __forceinline__ uint32_t transform_chunk(uint32_t (&a)[32], uint32_t (&b)[32], uint32_t s1_addr,
                                                    const float* rk1, const float* rk2, const float* rkm1,
                                                    const float* rkm2, int limit, bool diag, const RowCoef& c,
                                                    float relu_power, float lam, float pscale = 1.0f) {
  constexpr bool kFold = PM != POW_GENERAL;
  constexpr bool SAT = NORM && POS;  // normalized scores minus tau <= 1
  if (diag) {
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      a[i] = (i <= limit) ? a[i] : 0u;
      if constexpr (DIFF) b[i] = (i <= limit) ? b[i] : 0u;
    }
  }
  uint32_t lane_nz = 0;  // bit h: this lane may have a positive y in half h
  if constexpr (POS) {
    float m1[2][2] = {{-3.0e38f, -3.0e38f}, {-3.0e38f, -3.0e38f}};
    float m2[2][2] = {{-3.0e38f, -3.0e38f}, {-3.0e38f, -3.0e38f}};
#pragma unroll
    for (int i = 0; i < 32; i += 4) {
      const int h = i >> 4, k = (i >> 2) & 1;
      m1[h][k] = max3f(m1[h][k], __uint_as_float(a[i]), __uint_as_float(a[i + 1]));
      m1[h][k] = max3f(m1[h][k], __uint_as_float(a[i + 2]), __uint_as_float(a[i + 3]));
      if constexpr (DIFF) {
        m2[h][k] = max3f(m2[h][k], __uint_as_float(b[i]), __uint_as_float(b[i + 1]));
        m2[h][k] = max3f(m2[h][k], __uint_as_float(b[i + 2]), __uint_as_float(b[i + 3]));
      }
    }
    float2 g1 = make_float2(1.f, 1.f), g2 = g1;
    if constexpr (NORM) {
      g1 = *reinterpret_cast<const float2*>(rkm1);
      if constexpr (DIFF) g2 = *reinterpret_cast<const float2*>(rkm2);
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float gm1 = h ? g1.y : g1.x, gm2 = h ? g2.y : g2.x;
      const float ms1 = fmaxf(m1[h][0], m1[h][1]);
      bool nzh = (NORM ? ms1 * gm1 : ms1) > c.tq1;
      if constexpr (DIFF) {
        const float ms2 = fmaxf(m2[h][0], m2[h][1]);
        nzh = nzh || ((NORM ? ms2 * gm2 : ms2) > c.tq2);
      }
      lane_nz |= nzh ? (1u << h) : 0u;
    }
  } else {
    // two independent max chains per 16-key half
    float mx[2][2] = {{-3.0e38f, -3.0e38f}, {-3.0e38f, -3.0e38f}};
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
        const float2 rr = h ? make_float2(r1.z, r1.w) : make_float2(r1.x, r1.y);
        const float2 y = NORM ? __ffma2_rn(f2u(a[i], a[i + 1]), rr, make_float2(-c.tq1, -c.tq1))
                              : __fadd2_rn(f2u(a[i], a[i + 1]), make_float2(-c.tq1, -c.tq1));
        a[i] = __float_as_uint(y.x);
        a[i + 1] = __float_as_uint(y.y);
        mx[e4 >> 2][h] = max3f(mx[e4 >> 2][h], y.x, y.y);
        if constexpr (DIFF) {
          const float2 rs = h ? make_float2(r2.z, r2.w) : make_float2(r2.x, r2.y);
          const float2 y2 = NORM ? __ffma2_rn(f2u(b[i], b[i + 1]), rs, make_float2(-c.tq2, -c.tq2))
                                 : __fadd2_rn(f2u(b[i], b[i + 1]), make_float2(-c.tq2, -c.tq2));
          b[i] = __float_as_uint(y2.x);
          b[i + 1] = __float_as_uint(y2.y);
          mx[e4 >> 2][h] = max3f(mx[e4 >> 2][h], y2.x, y2.y);
        }
      }
    }
    lane_nz |= fmaxf(mx[0][0], mx[0][1]) > 0.0f ? 1u : 0u;
    lane_nz |= fmaxf(mx[1][0], mx[1][1]) > 0.0f ? 2u : 0u;
  }

  uint32_t nz = 0;
  constexpr int kUnroll = ROLL ? 1 : 2;
#pragma unroll kUnroll
  for (int half = 0; half < 2; ++half) {
    // this half's 16 scores sit in a[o..o+15] (b[o..o+15])
    const int o = ROLL ? 0 : 16 * half;
    bool lnz = (lane_nz >> half) & 1u;
    bool any = __any_sync(0xffffffffu, lnz);
    if constexpr (POS) {
      if (any) {
        // the bound could not clear this half: form y exactly and test again
        float mx[2] = {-3.0e38f, -3.0e38f};
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          float4 r1 = make_float4(1.f, 1.f, 1.f, 1.f), r2 = r1;
          if constexpr (NORM) {
            r1 = *reinterpret_cast<const float4*>(rk1 + 16 * half + 4 * q4);
            if constexpr (DIFF) r2 = *reinterpret_cast<const float4*>(rk2 + 16 * half + 4 * q4);
          }
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            const int i = o + 4 * q4 + 2 * t;
            const float2 rr = t ? make_float2(r1.z, r1.w) : make_float2(r1.x, r1.y);
            const float2 y = NORM ? __ffma2_rn(f2u(a[i], a[i + 1]), rr, make_float2(-c.tq1, -c.tq1))
                                  : __fadd2_rn(f2u(a[i], a[i + 1]), make_float2(-c.tq1, -c.tq1));
            a[i] = __float_as_uint(y.x);
            a[i + 1] = __float_as_uint(y.y);
            mx[t] = max3f(mx[t], y.x, y.y);
            if constexpr (DIFF) {
              const float2 rs = t ? make_float2(r2.z, r2.w) : make_float2(r2.x, r2.y);
              const float2 y2 = NORM ? __ffma2_rn(f2u(b[i], b[i + 1]), rs, make_float2(-c.tq2, -c.tq2))
                                     : __fadd2_rn(f2u(b[i], b[i + 1]), make_float2(-c.tq2, -c.tq2));
              b[i] = __float_as_uint(y2.x);
              b[i + 1] = __float_as_uint(y2.y);
              mx[t] = max3f(mx[t], y2.x, y2.y);
            }
          }
        }
        lnz = fmaxf(mx[0], mx[1]) > 0.0f;
        any = __any_sync(0xffffffffu, lnz);
      }
    }
    nz |= lnz ? (1u << half) : 0u;
    uint32_t hi[8], lo[8];
    if (any) {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float2 y1 = f2u(a[o + 2 * q], a[o + 2 * q + 1]);
        const float2 u1 = NORM ? scaled_relu<SAT>(y1, c.rq1) : relu2(y1);
        float2 P;
        if constexpr (DIFF) {
          const float2 y2 = f2u(b[o + 2 * q], b[o + 2 * q + 1]);
          const float2 u2 = (NORM || kFold) ? scaled_relu<SAT>(y2, c.rq2) : relu2(y2);
          if constexpr (kFold) {
            P = sub2(pow2v<PM>(u1, relu_power), pow2v<PM>(u2, relu_power));
          } else {
            P = __ffma2_rn(make_float2(-lam, -lam), pow2v<PM>(u2, relu_power), pow2v<PM>(u1, relu_power));
          }
        } else {
          P = pow2v<PM>(u1, relu_power);
        }
        if constexpr (F16) {
          // hi = fp16(P * pscale), lo = fp16(P * pscale - hi): ~22 bits
          const float2 t = __fmul2_rn(P, make_float2(pscale, pscale));
          hi[q] = pack_f16x2(t.x, t.y);
          const float2 l = sub2(t, unpack_f16x2(hi[q]));
          lo[q] = pack_f16x2(l.x, l.y);
        } else {
          // hi = P truncated to bf16 (exact in fp32), lo = bf16(P - hi): hi + lo
          // carries ~16 significant bits of P.
          const uint32_t p0 = __float_as_uint(P.x), p1 = __float_as_uint(P.y);
          hi[q] = __byte_perm(p0, p1, 0x7632);
          const float2 l = sub2(P, f2u(p0 & 0xFFFF0000u, p1 & 0xFFFF0000u));
          lo[q] = pack_bf16x2(l.x, l.y);
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        hi[q] = 0u;
        lo[q] = 0u;
      }
    }
    tmem_st8(s1_addr + 8 * half, hi);
    tmem_st8(s1_addr + 16 + 8 * half, lo);
    if (ROLL && half == 0) {
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        a[i] = a[16 + i];
        if constexpr (DIFF) b[i] = b[16 + i];
      }
    }
  }
  return nz;
}

// The 32-key chunks a transform thread owns in one key tile: NCH = 2 (two
// transform warpgroups; warpgroup `wg` owns chunks 2 wg, 2 wg + 1) or NCH = 1
// (four warpgroups; chunk wg).  TMEM columns: S1 at s1col, S2 at s2col (differential).
// rk_tile: the tile's entry of the key-table ring: rk1[128] (rk2[128]) then
// the per-16-key maxima rkmax1[8] (rkmax2[8]).
// With the differential form, all of S2 is loaded first and `release_s2()` is
// called as soon as it sits in registers, so the next tile's QK2 can reuse the
// S2 columns while this tile is transformed; S1 of the second chunk is loaded
// after the first chunk is done (keeps register use down).  The rectified
// form loads both of its S chunks at once.  ROLL_C: the chunks run through one
// rolled loop (the second chunk's registers are moved into the first's);
// ROLL_H: likewise for the two halves of a chunk.
// Returns bit (2 cc + h): 16-key half h of chunk cc holds a nonzero P.
template <int PM, bool DIFF, bool NORM, bool POS, bool ROLL_C, bool ROLL_H, bool F16, int NCH, typename ReleaseS2>
__device__ __forceinline__ uint32_t transform_tile(uint32_t tmem_row, uint32_t s1col, uint32_t s2col, int wg,
                                                   const float* rk_tile, int limit0, bool diag, const RowCoef& c,
                                                   float relu_power, float lam, float pscale,
                                                   ReleaseS2&& release_s2) {
  static_assert(NCH == 1 || NCH == 2, "one or two 32-key chunks per thread");
  constexpr int kMaxOff = DIFF ? 256 : 128;  // rkmax after rk1 (and rk2)
  const int ch0 = NCH * wg;
  uint32_t nz = 0;
  if constexpr (NCH == 1) {
    // one 32-key chunk per thread (four transform warpgroups): its S1 (and
    // S2) columns in one load; S2's TMEM slot is handed back as soon as it
    // sits in registers
    uint32_t a[32], b[32];
    tmem_ld32(tmem_row + s1col + 32 * ch0, a);
    if constexpr (DIFF) tmem_ld32(tmem_row + s2col + 32 * ch0, b);
    tmem_wait_ld();
    if constexpr (DIFF) release_s2();
    const float* r1 = rk_tile + 32 * ch0;
    const float* m1 = rk_tile + kMaxOff + 2 * ch0;
    return transform_chunk<PM, DIFF, NORM, POS, ROLL_H, F16>(a, b, tmem_row + s1col + 32 * ch0, r1, r1 + 128, m1,
                                                             m1 + 8, limit0 - 32 * ch0, diag, c, relu_power, lam,
                                                             pscale);
  }
  uint32_t a[32], b[32], b1[32];
  if constexpr (DIFF) {
    tmem_ld32(tmem_row + s1col + 32 * ch0, a);
    tmem_ld32(tmem_row + s2col + 32 * ch0, b);
    tmem_ld32(tmem_row + s2col + 32 * (ch0 + 1), b1);
    tmem_wait_ld();
    release_s2();
  } else {
    tmem_ld32(tmem_row + s1col + 32 * ch0, a);
    tmem_ld32(tmem_row + s1col + 32 * (ch0 + 1), b1);
    tmem_wait_ld();
  }
  auto chunk = [&](uint32_t(&x)[32], uint32_t(&y)[32], int cc) {
    const int ch = ch0 + cc;
    const float* r1 = rk_tile + 32 * ch;
    const float* m1 = rk_tile + kMaxOff + 2 * ch;
    nz |= transform_chunk<PM, DIFF, NORM, POS, ROLL_H, F16>(x, y, tmem_row + s1col + 32 * ch, r1, r1 + 128, m1,
                                                            m1 + 8, limit0 - 32 * ch, diag, c, relu_power, lam,
                                                            pscale)
          << (2 * cc);
  };
  if constexpr (ROLL_C) {
#pragma unroll 1
    for (int cc = 0; cc < 2; ++cc) {
      if (cc == 1) {
        if constexpr (DIFF) {
          tmem_ld32(tmem_row + s1col + 32 * (ch0 + 1), a);
#pragma unroll
          for (int i = 0; i < 32; ++i) b[i] = b1[i];
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) a[i] = b1[i];
        }
      }
      chunk(a, b, cc);
    }
  } else {
    chunk(a, b, 0);
    if constexpr (DIFF) {
      tmem_ld32(tmem_row + s1col + 32 * (ch0 + 1), a);
      tmem_wait_ld();
      chunk(a, b1, 1);
    } else {
      chunk(b1, b, 1);
    }
  }
  return nz;
}

}  // namespace tc
}  // namespace tda
