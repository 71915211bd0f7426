// Tensor-core forward for fp32 inputs at head_dim 64 and 128 (tcgen05, kind::tf32).
//
// fp32 results must stay within 1e-5 rel-L2 of an fp64 oracle; one TF32
// product per score (10-bit mantissa) misses that by far.  Each fp32 operand
// x is therefore split into h = x rounded to TF32 and l = x - h (exact in
// fp32) rounded to TF32, and every product is formed from three TF32
// products, h_a*h_b + h_a*l_b + l_a*h_b.  The dropped l_a*l_b term and l's
// rounding are ~2^-23 relative and unbiased (both parts rounded to nearest).
// O += P V uses the same three products, with P split after the threshold /
// ReLU^p transform.
// Semantics as the reference forward (triton_threshold_attention.py:19-115,
// mask-to-zero causal rule, tau(i) = beta*sqrt(2 log(i+1)/D), power branch
// incl. exp(p*log(x+1e-10))) and its differential wrapper (:489-519: both
// branches accumulate into one output, the second weighted by -clamp(lambda)).
//
// Pre-pass (one stream-ordered launch, into the caller's workspace):
//   q, k rows -> h, l copies [BH][S][D], and per row 1/m, tau*m (queries) or
//   1/m (keys), m = max(||x||, 1e-12) when normalized, m = 1 otherwise;
//   v -> transposed h, l copies [BH][D][S_pad] (zero past S), so that V^T is
//   a K-major operand like K.
// Main kernel: one CTA = 128 query rows of one (batch, head); key tiles of 64
// (head_dim 64) or 32 (head_dim 128); layout per head_dim in TfCfg below.  At 64:
//   warp 0  TMA producer: Q h/l once per branch, K h/l and V^T h/l rings of
//           two entries each (K released by QK, V by PV)
//   warp 1  PV issuer (one thread): P V^T (3 x 8 MMAs, P from TMEM) per tile
//   last warp  QK issuer (one thread): S = Q K^T (3 x 8 MMAs of M128 N64 K8)
//           into one of two TMEM S slots, once the PV reading the slot has run
//           (two issuing threads, so that one's waits and commits overlap the
//           other's MMAs)
//   warps 2-5  transform: thread = query row = TMEM lane; S -> P, written back
//           as P_h over S and P_l beside it; adds each tile's P V^T into
//           fp32 registers; epilogue O -> out.
// TMEM (64 columns each): S slot b holds the h*h part of S at 128 b (then
// P_h) and the cross terms at 128 b + 64 (then P_l); the partial O of tile t
// has its h*h part at 256 + 128 (t % 2) and its cross terms 64 further;
// the parts are added in fp32 registers, and the tiles' partial O too.
#include "tda_internal.h"
#include "tda_ptx.cuh"

namespace tda {
namespace {

constexpr int kBM = 128;
constexpr int kBox64 = 64 * 128;  // one TMA box of 64 rows of 32 fp32 (128 B), 8 KB

__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4)                                 // D f32
         | (2u << 7) | (2u << 10)                  // A, B tf32, both K-major
         | (static_cast<uint32_t>(N >> 3) << 17)   // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);  // M / 16
}

// Per head_dim layout.  D = 64: 64-key tiles, one transform warpgroup, two V^T
// entries and two partial-O slots.  D = 128: Q high / low alone take 128 KB of
// shared memory, so 32-key tiles, one V^T entry, one partial-O slot, and two
// transform warpgroups (each half of every key tile and half of O).
template <int D>
struct TfCfg {
  static constexpr int kBN = D == 64 ? 64 : 32;         // keys per tile
  static constexpr int kWG = D == 64 ? 1 : 2;           // transform warpgroups
  static constexpr int kVSlots = D == 64 ? 2 : 1;
  static constexpr int kOSlots = D == 64 ? 2 : 1;
  static constexpr int kQkWarp = 2 + 4 * kWG;           // the QK issuer, after the transform warps
  static constexpr int kThreads = 64 + 128 * kWG + 32;
  static constexpr int kCB = D / 32;                    // 128-byte column boxes of a D-wide row
  static constexpr int kQBytes = kCB * 2 * kBox64;      // 128 rows: two 64-row boxes per column box
  static constexpr int kKBytes = kCB * kBN * 128;       // one K tile (high or low part)
  static constexpr int kVBytes = (kBN / 32) * D * 128;  // one V^T tile (high or low part)
  static constexpr int kOffQh = 0, kOffQl = kQBytes;
  static constexpr int kOffK = 2 * kQBytes;             // 2 entries x (K_h, K_l)
  static constexpr int kOffV = kOffK + 2 * 2 * kKBytes; // kVSlots entries x (Vt_h, Vt_l)
  static constexpr int kOffBar = kOffV + kVSlots * 2 * kVBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;  // + barriers + alignment slack
  static constexpr uint32_t kColO = 4 * kBN;            // partial O slots after the two S slots
  static constexpr int kCW = kBN / kWG >= 32 ? 32 : 16;   // transform chunk (keys)
  static constexpr int kNCh = kBN / kWG / kCW;          // chunks per warpgroup per tile
  static constexpr int kOCols = D / kWG;                // output columns per warpgroup
  static constexpr uint32_t kIdescQK = idesc_tf32(128, kBN);
  static constexpr uint32_t kIdescPV = idesc_tf32(128, D);
  static_assert(kSmemBytes <= 232448, "shared memory");
  static_assert(kColO + kOSlots * 2 * D <= 512, "TMEM columns");
};

constexpr int ST_TF_PROD = 0x601, ST_TF_MMA = 0x602, ST_TF_TR = 0x603, ST_TF_DRAIN = 0x604;

struct Tf32Bars {
  uint64_t q_full, q_empty, drain, drain2;
  uint64_t pv_done[2];            // per S slot: the PV reading P from it has run
  uint64_t o_full[2], o_free[2];  // per-tile partial O: written by PV, read by the transform
  uint64_t k_full[2], k_empty[2], v_full[2], v_empty[2];
  uint64_t s_full[2], p_full[2];
  uint32_t tmem_base;
  int abort_flag;
};
static_assert(sizeof(Tf32Bars) <= 256, "barrier block too large");

// S slot e: h*h part of S at 2 kBN e (then P_h), cross terms kBN further (then P_l)
template <int BN>
__device__ __forceinline__ uint32_t col_s(int e) { return 2u * BN * static_cast<uint32_t>(e); }

__device__ __forceinline__ void mma_ss_tf32(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void mma_ts_tf32(uint32_t d, uint32_t a_tmem, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}\n" ::"r"(d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc)
      : "memory");
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
      "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
      "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
      "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}

// Waits with a time limit; used only while tearing down after an abort.
__device__ void tf_drain_wait(uint64_t* bar, uint32_t parity, const WaitCtl& ctl) {
  const uint32_t a = smem_u32(bar);
  const uint64_t t0 = global_timer_ns();
  while (!mbar_try_wait(a, parity)) {
    if (global_timer_ns() - t0 > ctl.timeout_ns) {
      atomicCAS(ctl.status, 0, ST_TF_DRAIN);
      return;
    }
  }
}

// Round to the nearest TF32 value (10 explicit mantissa bits), returned as an
// fp32 whose 13 low mantissa bits are zero, so that the tensor core reads it
// exactly.  Rounding (not truncation) leaves the split errors unbiased.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// x = h + l exactly up to l's own rounding: h = tf32(x), l = tf32(x - h)
// (x - h is exact in fp32; |l| <= 2^-11 |x|, its rounding error <= 2^-23 |x|).
__device__ __forceinline__ void tf32_split(float x, float& h, float& l) {
  h = tf32_rna(x);
  l = tf32_rna(x - h);
}

template <int PM>
__device__ __forceinline__ float relu_pow(float z, float p) {
  const float x = fmaxf(z, 0.0f);
  if constexpr (PM == POW_1) return x;
  if constexpr (PM == POW_2) return x * x;
  if constexpr (PM == POW_3) return x * x * x;
  return x > 0.0f ? expf(p * logf(x + 1e-10f)) : 0.0f;
}

// ------------------------------------------------------------------ pre-pass
// One launch for every split: blockIdx.y = job (2 br: rows of q of branch br,
// 2 br + 1: rows of k, 2 n_br: V^T), blockIdx.x = a 32-row slab of the padded
// (BH * S_pad) rows (S_pad is a multiple of 64, so a slab lies in one head).
struct Tf32SplitArgs {
  const float* q[2];
  const float* k[2];
  const float* v;
  Tf32Workspace w;
  int S;
  int S_pad;
  int n_br;
  int normalize;
  float beta;
};

template <int D>
__global__ void __launch_bounds__(256) tf32_split_kernel(const __grid_constant__ Tf32SplitArgs a) {
  __shared__ float t[32][D + 1];
  const int job = blockIdx.y;
  const int64_t row0 = static_cast<int64_t>(blockIdx.x) * 32;
  const int64_t bh = row0 / a.S_pad;
  const int i0 = static_cast<int>(row0 % a.S_pad);
  if (job < 2 * a.n_br) {
    // rows: D / 8 threads per row, 8 floats (two 16-byte loads) each
    constexpr int kTpr = D / 8, kRpp = 256 / kTpr;
    const int br = job >> 1;
    const bool is_q = (job & 1) == 0;
    float* r1 = is_q ? a.w.rq[br] : a.w.rk[br];
    for (int r0 = 0; r0 < 32; r0 += kRpp) {
      const int r = r0 + static_cast<int>(threadIdx.x) / kTpr, part = threadIdx.x % kTpr;
      const int i = i0 + r;
      const int64_t row = row0 + r;
      const bool valid = i < a.S;  // padded rows get zero coefficients; every lane takes part in the shuffles
      const size_t off = (static_cast<size_t>(bh) * a.S + (valid ? i : 0)) * D + 8 * part;
      float4 v0 = make_float4(0.f, 0.f, 0.f, 0.f), v1 = v0;
      if (valid) {
        const float* x = (is_q ? a.q[br] : a.k[br]) + off;
        v0 = *reinterpret_cast<const float4*>(x);
        v1 = *reinterpret_cast<const float4*>(x + 4);
      }
      const float xv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
      float h[8], l[8], ss = 0.0f;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        tf32_split(xv[c], h[c], l[c]);
        ss = fmaf(xv[c], xv[c], ss);
      }
      if (valid) {
        float* hi = (is_q ? a.w.qh[br] : a.w.kh[br]) + off;
        float* lo = (is_q ? a.w.ql[br] : a.w.kl[br]) + off;
        *reinterpret_cast<float4*>(hi) = make_float4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<float4*>(hi + 4) = make_float4(h[4], h[5], h[6], h[7]);
        *reinterpret_cast<float4*>(lo) = make_float4(l[0], l[1], l[2], l[3]);
        *reinterpret_cast<float4*>(lo + 4) = make_float4(l[4], l[5], l[6], l[7]);
      }
#pragma unroll
      for (int o = 1; o < kTpr; o <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      if (part == 0) {
        const float m = a.normalize ? fmaxf(sqrtf(ss), 1e-12f) : 1.0f;
        r1[row] = valid ? 1.0f / m : 0.0f;
        if (is_q) {
          const float tau = a.beta * sqrtf((2.0f * logf(static_cast<float>(i + 1))) / static_cast<float>(D));
          a.w.tq[br][row] = valid ? tau * m : 0.0f;
        }
      }
    }
    return;
  }
  // V^T: the slab's 32 keys x D dims through shared memory, written as D
  // rows of 32 keys (zero for keys >= S)
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  for (int r = ty; r < 32; r += 8)
    for (int c = tx; c < D; c += 32) {
      const int key = i0 + r;
      t[r][c] = key < a.S ? a.v[(static_cast<size_t>(bh) * a.S + key) * D + c] : 0.0f;
    }
  __syncthreads();
  for (int d = ty; d < D; d += 8) {
    float h, l;
    tf32_split(t[tx][d], h, l);
    const size_t o = (static_cast<size_t>(bh) * D + d) * a.S_pad + i0 + tx;
    a.w.vth[o] = h;
    a.w.vtl[o] = l;
  }
}

// ------------------------------------------------------------------ roles
// Producer (warp 0, one thread).  Loads run one K tile ahead of the V^T tiles
// (K(t+1) before V(t)), so that with a single V^T entry (D = 128) the K tile
// for the next QK never waits behind the previous PV.
template <int D>
__device__ void tf_producer(const Tf32FwdParams& p, uint8_t* smem, Tf32Bars* b, const WaitCtl& ctl, int bh, int m0,
                            int n_kt) {
  using C = TfCfg<D>;
  const int T = p.n_br * n_kt;
  int q_n = 0, k_n = 0, v_n = 0;
  bool ok = true;
  auto load_q = [&](int br) {
    mbar_arrive_expect_tx(&b->q_full, 2 * C::kQBytes);
    for (int cb = 0; cb < C::kCB; ++cb)
      for (int h = 0; h < 2; ++h) {
        const int off = cb * 2 * kBox64 + h * kBox64;
        tma_load_3d(smem + C::kOffQh + off, &p.tm_qh[br], &b->q_full, 32 * cb, m0 + 64 * h, bh);
        tma_load_3d(smem + C::kOffQl + off, &p.tm_ql[br], &b->q_full, 32 * cb, m0 + 64 * h, bh);
      }
    ++q_n;
  };
  auto load_k = [&](int t) {  // false when a wait gave up
    const int br = t / n_kt, j = t % n_kt, e = t & 1, u = t >> 1;
    if (j == 0 && br > 0) {
      if (!mbar_wait(&b->q_empty, (br - 1) & 1, ctl, ST_TF_PROD)) return false;
      load_q(br);
    }
    if (u > 0 && !mbar_wait(&b->k_empty[e], (u - 1) & 1, ctl, ST_TF_PROD)) return false;
    uint8_t* kd = smem + C::kOffK + e * 2 * C::kKBytes;
    mbar_arrive_expect_tx(&b->k_full[e], 2 * C::kKBytes);
    for (int cb = 0; cb < C::kCB; ++cb) {
      tma_load_3d(kd + cb * C::kBN * 128, &p.tm_kh[br], &b->k_full[e], 32 * cb, C::kBN * j, bh);
      tma_load_3d(kd + C::kKBytes + cb * C::kBN * 128, &p.tm_kl[br], &b->k_full[e], 32 * cb, C::kBN * j, bh);
    }
    ++k_n;
    return true;
  };
  auto load_v = [&](int t) {
    const int j = t % n_kt, e = t % C::kVSlots, u = t / C::kVSlots;
    if (u > 0 && !mbar_wait(&b->v_empty[e], (u - 1) & 1, ctl, ST_TF_PROD)) return false;
    uint8_t* vd = smem + C::kOffV + e * 2 * C::kVBytes;
    mbar_arrive_expect_tx(&b->v_full[e], 2 * C::kVBytes);
    for (int kb = 0; kb < C::kBN / 32; ++kb) {
      tma_load_3d(vd + kb * D * 128, &p.tm_vh, &b->v_full[e], C::kBN * j + 32 * kb, 0, bh);
      tma_load_3d(vd + C::kVBytes + kb * D * 128, &p.tm_vl, &b->v_full[e], C::kBN * j + 32 * kb, 0, bh);
    }
    ++v_n;
    return true;
  };
  if (!(p.inject & 1)) load_q(0);  // test hook: with bit 0 set the first Q tile never arrives
  ok = load_k(0);
  for (int t = 0; t < T && ok; ++t) {
    if (t + 1 < T && !(ok = load_k(t + 1))) break;
    ok = load_v(t);
  }
  if (!ok) {  // let the copies already issued land before the CTA exits
    if (q_n > 0) tf_drain_wait(&b->q_full, (q_n - 1) & 1, ctl);
    for (int i = k_n > 2 ? k_n - 2 : 0; i < k_n; ++i) tf_drain_wait(&b->k_full[i & 1], (i >> 1) & 1, ctl);
    for (int i = v_n > C::kVSlots ? v_n - C::kVSlots : 0; i < v_n; ++i)
      tf_drain_wait(&b->v_full[i % C::kVSlots], (i / C::kVSlots) & 1, ctl);
  }
}

// QK issuer (last warp): S = Q K^T into S slot t % 2.  QK_{t+2} waits until
// PV_t, which reads P_t from the same slot, has run (pv_done).
template <int D>
__device__ void tf_mma_qk(const Tf32FwdParams& p, uint8_t* smem, Tf32Bars* b, const WaitCtl& ctl, uint32_t tmem,
                          int n_kt) {
  using C = TfCfg<D>;
  const int T = p.n_br * n_kt;
  const uint32_t qh = smem_u32(smem + C::kOffQh), ql = smem_u32(smem + C::kOffQl);
  bool ok = mbar_wait(&b->q_full, 0, ctl, ST_TF_MMA);
  tc_fence_after();
  auto qk = [&](int t) {
    const int br = t / n_kt, j = t % n_kt, e = t & 1, u = t >> 1;
    if (j == 0 && br > 0) {
      if (!(ok = mbar_wait(&b->q_full, br & 1, ctl, ST_TF_MMA))) return;
      tc_fence_after();
    }
    if (!(ok = mbar_wait(&b->k_full[e], u & 1, ctl, ST_TF_MMA))) return;
    if (t >= 2 && !(ok = mbar_wait(&b->pv_done[e], (u - 1) & 1, ctl, ST_TF_MMA))) return;
    tc_fence_after();
    const uint32_t kh = smem_u32(smem + C::kOffK + e * 2 * C::kKBytes), kl = kh + C::kKBytes;
    const uint32_t d = tmem + col_s<C::kBN>(e);
#pragma unroll
    for (int kk = 0; kk < D / 8; ++kk) {
      // k step of 8 fp32 = 32 B inside a 128-B swizzled row; column box kk / 4
      const uint32_t oq = (kk >> 2) * 2 * kBox64 + (kk & 3) * 32;
      const uint32_t okk = (kk >> 2) * C::kBN * 128 + (kk & 3) * 32;
      const uint64_t aqh = smem_desc_sw128(qh + oq, 16, 1024), aql = smem_desc_sw128(ql + oq, 16, 1024);
      const uint64_t bkh = smem_desc_sw128(kh + okk, 16, 1024), bkl = smem_desc_sw128(kl + okk, 16, 1024);
      // h*h products and the two cross terms go to separate accumulators so
      // that the small terms are not added onto the large partial sums
      mma_ss_tf32(d, aqh, bkh, C::kIdescQK, kk > 0 ? 1u : 0u);
      mma_ss_tf32(d + C::kBN, aqh, bkl, C::kIdescQK, kk > 0 ? 1u : 0u);
      mma_ss_tf32(d + C::kBN, aql, bkh, C::kIdescQK, 1u);
    }
    tc_commit(&b->k_empty[e]);
    tc_commit(&b->s_full[e]);
    if (j == n_kt - 1 && br + 1 < p.n_br) tc_commit(&b->q_empty);
  };
  for (int t = 0; t < T && ok; ++t) qk(t);
  if (!ok) {  // let every MMA this thread issued finish before TMEM is freed
    tc_commit(&b->drain2);
    tf_drain_wait(&b->drain2, 0, ctl);
  }
}

// PV issuer (warp 1).  Each tile's P V goes into a fresh partial O that the
// transform threads add into fp32 registers: the tensor core accumulates one
// tile's products instead of the whole key range.  The V^T slot is acquired
// before the wait for P (its load does not depend on P).
template <int D>
__device__ void tf_mma_pv(const Tf32FwdParams& p, uint8_t* smem, Tf32Bars* b, const WaitCtl& ctl, uint32_t tmem,
                          int n_kt) {
  using C = TfCfg<D>;
  const int T = p.n_br * n_kt;
  bool ok = true;
  for (int t = 0; t < T && ok; ++t) {
    const int e = t & 1, u = t >> 1;
    const int ev = t % C::kVSlots, uv = t / C::kVSlots;
    const int eo = t % C::kOSlots, uo = t / C::kOSlots;
    if (!(ok = mbar_wait(&b->v_full[ev], uv & 1, ctl, ST_TF_MMA))) break;
    if (!(ok = mbar_wait(&b->p_full[e], u & 1, ctl, ST_TF_MMA))) break;
    if (uo > 0 && !(ok = mbar_wait(&b->o_free[eo], (uo - 1) & 1, ctl, ST_TF_MMA))) break;
    tc_fence_after();
    const uint32_t vh = smem_u32(smem + C::kOffV + ev * 2 * C::kVBytes), vl = vh + C::kVBytes;
    const uint32_t d = tmem + C::kColO + 2 * D * eo;
#pragma unroll
    for (int kk = 0; kk < C::kBN / 8; ++kk) {
      const uint32_t ov = (kk >> 2) * D * 128 + (kk & 3) * 32;
      const uint64_t bvh = smem_desc_sw128(vh + ov, 16, 1024), bvl = smem_desc_sw128(vl + ov, 16, 1024);
      const uint32_t ah = tmem + col_s<C::kBN>(e) + 8 * kk, al = ah + C::kBN;
      mma_ts_tf32(d, ah, bvh, C::kIdescPV, kk > 0 ? 1u : 0u);
      mma_ts_tf32(d + D, ah, bvl, C::kIdescPV, kk > 0 ? 1u : 0u);
      mma_ts_tf32(d + D, al, bvh, C::kIdescPV, 1u);
    }
    tc_commit(&b->v_empty[ev]);
    tc_commit(&b->o_full[eo]);
    tc_commit(&b->pv_done[e]);
  }
  if (!ok) {  // let every MMA this thread issued finish before TMEM is freed
    tc_commit(&b->drain);
    tf_drain_wait(&b->drain, 0, ctl);
  }
}

template <int CW>
__device__ __forceinline__ void tmem_ld_cw(uint32_t taddr, uint32_t (&r)[CW]) {
  if constexpr (CW == 32) tmem_ld32(taddr, r); else tmem_ld16(taddr, r);
}
template <int CW>
__device__ __forceinline__ void tmem_st_cw(uint32_t taddr, const uint32_t (&r)[CW]) {
  if constexpr (CW == 32) tmem_st32(taddr, r); else tmem_st16(taddr, r);
}

// Transform warps 2 .. 2 + 4 kWG - 1: warp w owns TMEM lane quarter w % 4 (32
// query rows) and, as warpgroup g = (w - 2) / 4, keys [g kBN / kWG, (g+1) kBN
// / kWG) of every tile (in chunks of kCW) and output columns [g kOCols,
// (g+1) kOCols).
template <int D, int PM>
__device__ void tf_transform(const Tf32FwdParams& p, Tf32Bars* b, const WaitCtl& ctl, uint32_t tmem, int bh, int m0,
                             int n_kt, int warp, int lane) {
  using C = TfCfg<D>;
  constexpr int kCW = C::kCW;
  const int quarter = warp & 3;
  const int g = (warp - 2) >> 2;
  const int row = 32 * quarter + lane;
  const int gi = m0 + row;
  const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
  const int T = p.n_br * n_kt;
  const size_t rbase = static_cast<size_t>(bh) * p.S_pad;
  float rq = 0.0f, tq = 0.0f, w = 1.0f;
  float acc[C::kOCols];
#pragma unroll
  for (int c = 0; c < C::kOCols; ++c) acc[c] = 0.0f;
  bool ok = true;
  // add this warpgroup's columns of tile x's partial O into acc, release the slot
  auto harvest = [&](int x) {
    const int eo = x % C::kOSlots, uo = x / C::kOSlots;
    if (!(ok = mbar_wait_warp(&b->o_full[eo], uo & 1, ctl, ST_TF_TR))) return;
    tc_fence_after();
    const uint32_t base = tl + C::kColO + 2 * D * eo + C::kOCols * g;
#pragma unroll
    for (int c2 = 0; c2 < C::kOCols / 32; ++c2) {
      uint32_t ob[32], os[32];
      tmem_ld32(base + 32 * c2, ob);
      tmem_ld32(base + D + 32 * c2, os);
      tmem_wait_ld();
#pragma unroll
      for (int c = 0; c < 32; ++c) acc[32 * c2 + c] += __uint_as_float(ob[c]) + __uint_as_float(os[c]);
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&b->o_free[eo]);
  };
  for (int t = 0; t < T; ++t) {
    const int br = t / n_kt, j = t % n_kt, e = t & 1, u = t >> 1;
    if (j == 0) {
      w = br ? -lambda_of(p.lam_dev, bh, p.lam) : 1.0f;
      rq = gi < p.S ? p.rq[br][rbase + gi] : 0.0f;  // rows past S: z = 0, P = 0
      tq = gi < p.S ? p.tq[br][rbase + gi] : 0.0f;
    }
    if (!(ok = mbar_wait_warp(&b->s_full[e], u & 1, ctl, ST_TF_TR))) break;
    tc_fence_after();
    // rolled: one copy of the chunk body keeps the loop inside the SM's
    // instruction cache (unrolled, instruction fetch was the main stall)
#pragma unroll 1
    for (int ch = 0; ch < C::kNCh; ++ch) {
      const int kr = g * (C::kBN / C::kWG) + ch * kCW;  // first key of the chunk within the tile
      const int key0 = C::kBN * j + kr;
      float4 rk4[kCW / 4];  // key coefficients of this chunk, loaded before the TMEM wait
      const float* rk = p.rk[br] + rbase + key0;
#pragma unroll
      for (int c4 = 0; c4 < kCW / 4; ++c4) rk4[c4] = *reinterpret_cast<const float4*>(rk + 4 * c4);
      const bool diag = key0 + kCW - 1 > m0;  // some key of the chunk lies past some row
      uint32_t s[kCW], sl[kCW];
      tmem_ld_cw<kCW>(tl + col_s<C::kBN>(e) + kr, s);
      tmem_ld_cw<kCW>(tl + col_s<C::kBN>(e) + C::kBN + kr, sl);
      tmem_wait_ld();
      uint32_t hi[kCW], lo[kCW];
#pragma unroll
      for (int c4 = 0; c4 < kCW / 4; ++c4) {
        const float rr[4] = {rk4[c4].x, rk4[c4].y, rk4[c4].z, rk4[c4].w};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const int c = 4 * c4 + q;
          float sv = __uint_as_float(s[c]) + __uint_as_float(sl[c]);
          if (diag && key0 + c > gi) sv = 0.0f;  // causal mask to zero
          const float pv = w * relu_pow<PM>(fmaf(sv, rr[q], -tq) * rq, p.relu_power);
          float h, l;
          tf32_split(pv, h, l);
          hi[c] = __float_as_uint(h);
          lo[c] = __float_as_uint(l);
        }
      }
      tmem_st_cw<kCW>(tl + col_s<C::kBN>(e) + kr, hi);
      tmem_st_cw<kCW>(tl + col_s<C::kBN>(e) + C::kBN + kr, lo);
    }
    tmem_wait_st();
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(&b->p_full[e]);
    if (t > 0) {
      harvest(t - 1);
      if (!ok) break;
    }
  }
  if (ok) harvest(T - 1);
  if (!ok || gi >= p.S) return;
  float* dst = p.out + (static_cast<size_t>(bh) * p.S + gi) * D + C::kOCols * g;
#pragma unroll
  for (int c4 = 0; c4 < C::kOCols / 4; ++c4)
    *reinterpret_cast<float4*>(dst + 4 * c4) = make_float4(acc[4 * c4], acc[4 * c4 + 1], acc[4 * c4 + 2], acc[4 * c4 + 3]);
}

template <int D, int PM>
__global__ void __launch_bounds__(TfCfg<D>::kThreads, 1) tda_tf32_fwd_kernel(const __grid_constant__ Tf32FwdParams p) {
  using C = TfCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Tf32Bars* b = reinterpret_cast<Tf32Bars*>(smem + C::kOffBar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // longest query tiles (most key tiles) first
  const int qt = p.n_qt - 1 - static_cast<int>(blockIdx.x / p.BH);
  const int bh = static_cast<int>(blockIdx.x % p.BH);
  const int m0 = kBM * qt;
  const int n_kt = p.causal_skip ? min(kBM * (qt + 1) / C::kBN, p.n_kt_all) : p.n_kt_all;

  if (threadIdx.x == 0) {
    mbar_init(&b->q_full, 1);
    mbar_init(&b->q_empty, 1);
    mbar_init(&b->drain, 1);
    mbar_init(&b->drain2, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&b->pv_done[i], 1);
      mbar_init(&b->k_full[i], 1);
      mbar_init(&b->k_empty[i], 1);
      mbar_init(&b->v_full[i], 1);
      mbar_init(&b->v_empty[i], 1);
      mbar_init(&b->s_full[i], 1);
      mbar_init(&b->p_full[i], 4 * C::kWG);
      mbar_init(&b->o_full[i], 1);
      mbar_init(&b->o_free[i], 4 * C::kWG);
    }
    b->abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&b->tmem_base, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = b->tmem_base;
  const WaitCtl ctl = make_wait_ctl(&b->abort_flag, p.status, p.timeout_ns);
  if (warp == 0) {
    if (lane == 0) tf_producer<D>(p, smem, b, ctl, bh, m0, n_kt);
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) tf_mma_pv<D>(p, smem, b, ctl, tmem, n_kt);
    __syncwarp();
  } else if (warp == C::kQkWarp) {
    if (lane == 0) tf_mma_qk<D>(p, smem, b, ctl, tmem, n_kt);
    __syncwarp();
  } else {
    tf_transform<D, PM>(p, b, ctl, tmem, bh, m0, n_kt, warp, lane);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

template <int D>
cudaError_t launch_fwd_d(const Tf32FwdParams& p, int pow_mode, cudaStream_t stream) {
  using C = TfCfg<D>;
  void (*kern)(Tf32FwdParams);
  switch (pow_mode) {
    case POW_1: kern = tda_tf32_fwd_kernel<D, POW_1>; break;
    case POW_2: kern = tda_tf32_fwd_kernel<D, POW_2>; break;
    case POW_3: kern = tda_tf32_fwd_kernel<D, POW_3>; break;
    default: kern = tda_tf32_fwd_kernel<D, POW_GENERAL>; break;
  }
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (e != cudaSuccess) return e;
  const unsigned grid = static_cast<unsigned>(p.BH) * static_cast<unsigned>(p.n_qt);
  kern<<<grid, C::kThreads, C::kSmemBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

int tf32_key_tile(int head_dim) { return head_dim == 64 ? TfCfg<64>::kBN : TfCfg<128>::kBN; }

cudaError_t launch_tf32_split(const float* const q[2], const float* const k[2], const float* v,
                              const Tf32Workspace& ws, int n_br, int BH, int S, int D, float beta, int normalize,
                              cudaStream_t stream) {
  Tf32SplitArgs a;
  for (int br = 0; br < 2; ++br) {
    a.q[br] = q[br];
    a.k[br] = k[br];
  }
  a.v = v;
  a.w = ws;
  a.S = S;
  a.S_pad = static_cast<int>(tf32_padded_seq(S));
  a.n_br = n_br;
  a.normalize = normalize;
  a.beta = beta;
  const dim3 grid(static_cast<unsigned>(static_cast<int64_t>(BH) * a.S_pad / 32), static_cast<unsigned>(2 * n_br + 1));
  if (D == 64) tf32_split_kernel<64><<<grid, 256, 0, stream>>>(a);
  else if (D == 128) tf32_split_kernel<128><<<grid, 256, 0, stream>>>(a);
  else return cudaErrorInvalidValue;
  return cudaGetLastError();
}

cudaError_t launch_tf32_fwd(const Tf32FwdParams& p, int head_dim, int pow_mode, cudaStream_t stream) {
  if (head_dim == 64) return launch_fwd_d<64>(p, pow_mode, stream);
  if (head_dim == 128) return launch_fwd_d<128>(p, pow_mode, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tda
