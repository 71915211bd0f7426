// CUDA-core fp32 backward of threshold rectified attention (one branch).
//
// Gradients as the reference's backward kernels form them
// (triton_threshold_attention.py:118-224 for dQ, :227-324 for dK / dV), on
// F.normalize'd q, k when `normalize` (the chain rule through F.normalize is
// applied in the epilogue, as torch autograd applies it around the reference
// op, :505-512):
//   s_ij  = qh_i . kh_j, set to 0 for j > i         (qh, kh: normalized or raw)
//   z_ij  = s_ij - tau_i,  P_ij = relu(z_ij)^p
//   dP_ij = g_i . v_j,  g = dout_scale * dout
//   dA_ij = dP_ij * d relu(z)^p / dz (z_ij)
//   dqh_i = sum_j dA_ij kh_j,  dkh_j = sum_i dA_ij qh_i,  dv_j = sum_i P_ij g_i
// dA is not masked: with beta < 0 the masked entries (z = -tau > 0) add to dQ
// and dK exactly as in the reference; with beta >= 0 they have zero gradient
// and key / query tiles beyond the diagonal are skipped.
//
// Two kernels on a BT x BT tile grid (BT = 64; 32 at head_dim 256, where four
// fp32 64-row tiles would not fit in shared memory), 256 threads as 16 x 16,
// exact fp32 FFMA (inputs bf16 or fp32, widened in shared memory):
//   dq kernel   one CTA per (batch, head, BT query rows), loop over key tiles
//   dkv kernel  one CTA per (batch, head, BT keys), loop over query tiles
// Thread (ty, tx) owns tile rows {ty + 16 i} x columns {tx + 16 c} (i, c <
// BT / 16) of the score-like BT x BT products and rows {ty + 16 i} x head-dim
// columns {64 g + 4 tx + t} (D >= 64) or {CPT tx + t} (D < 64) of the
// accumulators.
#include <cuda_bf16.h>

#include "tda_internal.h"

namespace tda {
namespace {

constexpr int kThreads = 256;

template <int D>
struct BwdCfg {
  static constexpr int BT = D >= 256 ? 32 : 64;    // tile rows (queries or keys)
  static constexpr int RPT = BT / 16;              // tile rows (and product columns) per thread
  static constexpr int LDP = BT + 16;              // row stride of the BT x BT shared products
  static constexpr int LD = D + 4;                 // row stride of the D-wide tiles
  static constexpr int CPT = D / 16;               // accumulator columns per thread
  static constexpr int kTileFloats = BT * LD;
  // 4 D-wide tiles, 2 products, per-row scalars (norm factor, tau) x 2
  static constexpr int kFloats = 4 * kTileFloats + 2 * BT * LDP + 4 * BT;
  static constexpr int kBytes = kFloats * 4;
  static_assert(kBytes <= 227 * 1024, "backward tiles exceed shared memory");
};

__device__ __forceinline__ float relu_pow_ref(float z, float p) {
  const float x = fmaxf(z, 0.0f);
  if (p == 2.0f) return x * x;
  if (p == 1.0f) return x;
  return x > 0.0f ? expf(p * logf(x + 1e-10f)) : 0.0f;
}

// d relu(z)^p / dz as at triton_threshold_attention.py:195-206
__device__ __forceinline__ float relu_pow_grad_ref(float z, float p) {
  const float x = fmaxf(z, 0.0f);
  if (p == 2.0f) return 2.0f * x;
  if (p == 1.0f) return z > 0.0f ? 1.0f : 0.0f;
  return x > 0.0f ? p * expf((p - 1.0f) * logf(x + 1e-10f)) : 0.0f;
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* src);
template <>
__device__ __forceinline__ float4 load4<float>(const float* src) {
  return *reinterpret_cast<const float4*>(src);
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* src) {
  const uint2 u = *reinterpret_cast<const uint2*>(src);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}

// rows [r0, r0 + BT) of a (BH, S, D) array -> shared [BT][ld] fp32 times
// `scale`, zero past S.
template <int D, typename T>
__device__ __forceinline__ void load_rows(float* dst, int ld, const T* src, int bh, int r0, int S, float scale) {
  constexpr int V4 = D / 4;
  for (int idx = threadIdx.x; idx < BwdCfg<D>::BT * V4; idx += kThreads) {
    const int r = idx / V4, c4 = idx % V4;
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < S) {
      val = load4<T>(src + (static_cast<size_t>(bh) * S + r0 + r) * D + 4 * c4);
      val.x *= scale;
      val.y *= scale;
      val.z *= scale;
      val.w *= scale;
    }
    *reinterpret_cast<float4*>(dst + r * ld + 4 * c4) = val;
  }
}

// Row inverse norms of a loaded tile (1 / max(||x||, 1e-12)), then the tile is
// scaled in place to unit rows.  Rows past S are zero and stay zero.
template <int D>
__device__ __forceinline__ void normalize_rows(float* tile, float* rinv) {
  using C = BwdCfg<D>;
  {
    // kParts adjacent lanes per row (4 for 64 rows, 8 for 32), D / kParts dims each
    constexpr int kParts = kThreads / C::BT;
    const int row = threadIdx.x / kParts, part = threadIdx.x % kParts;
    float ss = 0.f;
#pragma unroll
    for (int d = part * (D / kParts); d < (part + 1) * (D / kParts); d += 4) {
      const float4 x = *reinterpret_cast<const float4*>(tile + row * C::LD + d);
      ss = fmaf(x.x, x.x, ss);
      ss = fmaf(x.y, x.y, ss);
      ss = fmaf(x.z, x.z, ss);
      ss = fmaf(x.w, x.w, ss);
    }
#pragma unroll
    for (int off = 1; off < kParts; off <<= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (part == 0) rinv[row] = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
  }
  __syncthreads();
  for (int idx = threadIdx.x; idx < C::BT * D; idx += kThreads) {
    const int r = idx / D, d = idx % D;
    tile[r * C::LD + d] *= rinv[r];
  }
}

// a[i][c] = A[ty+16i] . B[tx+16c] and b[i][c] = A2[ty+16i] . B2[tx+16c] over D
template <int D>
__device__ __forceinline__ void two_score_tiles(float (&a)[BwdCfg<D>::RPT][BwdCfg<D>::RPT],
                                                float (&b)[BwdCfg<D>::RPT][BwdCfg<D>::RPT], const float* A,
                                                const float* B, const float* A2, const float* B2, int ty, int tx) {
  using C = BwdCfg<D>;
  constexpr int R = C::RPT;
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int c = 0; c < R; ++c) {
      a[i][c] = 0.f;
      b[i][c] = 0.f;
    }
#pragma unroll 2
  for (int d = 0; d < D; d += 4) {
    float4 xa[R], xb[R], ya[R], yb[R];
#pragma unroll
    for (int i = 0; i < R; ++i) {
      xa[i] = *reinterpret_cast<const float4*>(A + (ty + 16 * i) * C::LD + d);
      ya[i] = *reinterpret_cast<const float4*>(A2 + (ty + 16 * i) * C::LD + d);
    }
#pragma unroll
    for (int c = 0; c < R; ++c) {
      xb[c] = *reinterpret_cast<const float4*>(B + (tx + 16 * c) * C::LD + d);
      yb[c] = *reinterpret_cast<const float4*>(B2 + (tx + 16 * c) * C::LD + d);
    }
#pragma unroll
    for (int i = 0; i < R; ++i)
#pragma unroll
      for (int c = 0; c < R; ++c) {
        a[i][c] = fmaf(xa[i].x, xb[c].x, a[i][c]);
        a[i][c] = fmaf(xa[i].y, xb[c].y, a[i][c]);
        a[i][c] = fmaf(xa[i].z, xb[c].z, a[i][c]);
        a[i][c] = fmaf(xa[i].w, xb[c].w, a[i][c]);
        b[i][c] = fmaf(ya[i].x, yb[c].x, b[i][c]);
        b[i][c] = fmaf(ya[i].y, yb[c].y, b[i][c]);
        b[i][c] = fmaf(ya[i].z, yb[c].z, b[i][c]);
        b[i][c] = fmaf(ya[i].w, yb[c].w, b[i][c]);
      }
  }
}

// acc[i][col] += sum_j M[ty+16i][j] * X[j][col] (M: BT x BT at stride LDP, X: BT x D at stride LD)
template <int D>
__device__ __forceinline__ void mac_rows(float (&acc)[BwdCfg<D>::RPT][BwdCfg<D>::CPT], const float* M,
                                         const float* X, int ty, int tx) {
  using C = BwdCfg<D>;
  constexpr int R = C::RPT;
#pragma unroll 2
  for (int j = 0; j < C::BT; j += 4) {
    float4 m4[R];  // four j per 16-byte load of each row of M
#pragma unroll
    for (int i = 0; i < R; ++i) m4[i] = *reinterpret_cast<const float4*>(M + (ty + 16 * i) * C::LDP + j);
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      float m[R];
#pragma unroll
      for (int i = 0; i < R; ++i) m[i] = jj == 0 ? m4[i].x : (jj == 1 ? m4[i].y : (jj == 2 ? m4[i].z : m4[i].w));
      if constexpr (D >= 64) {
#pragma unroll
        for (int g = 0; g < D / 64; ++g) {
          const float4 x = *reinterpret_cast<const float4*>(X + (j + jj) * C::LD + 64 * g + 4 * tx);
#pragma unroll
          for (int i = 0; i < R; ++i) {
            acc[i][4 * g + 0] = fmaf(m[i], x.x, acc[i][4 * g + 0]);
            acc[i][4 * g + 1] = fmaf(m[i], x.y, acc[i][4 * g + 1]);
            acc[i][4 * g + 2] = fmaf(m[i], x.z, acc[i][4 * g + 2]);
            acc[i][4 * g + 3] = fmaf(m[i], x.w, acc[i][4 * g + 3]);
          }
        }
      } else {
#pragma unroll
        for (int t = 0; t < C::CPT; ++t) {
          const float x = X[(j + jj) * C::LD + C::CPT * tx + t];
#pragma unroll
          for (int i = 0; i < R; ++i) acc[i][t] = fmaf(m[i], x, acc[i][t]);
        }
      }
    }
  }
}

template <int D>
__device__ __forceinline__ int acc_col(int tx, int t) {
  return D >= 64 ? 64 * (t / 4) + 4 * tx + (t % 4) : BwdCfg<D>::CPT * tx + t;
}

// Epilogue of one accumulator row: with normalize, the chain rule through
// F.normalize, dx = r (dxh - (dxh . xh) xh) (xh = unit row, r = 1/max(||x||,eps);
// for ||x|| < eps this is dxh / eps, as xh = x / eps there), then the store.
// The 16 threads sharing a row (one half warp) reduce the dot product.
template <int D>
__device__ __forceinline__ void store_grad_row(float* dst, float (&acc)[BwdCfg<D>::CPT], const float* xh_row,
                                               float rinv, bool normalize, bool accumulate, bool valid, int tx) {
  using C = BwdCfg<D>;
  if (normalize) {
    float dot = 0.f;
#pragma unroll
    for (int t = 0; t < C::CPT; ++t) dot = fmaf(acc[t], xh_row[acc_col<D>(tx, t)], dot);
#pragma unroll
    for (int off = 1; off < 16; off <<= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
    const bool big = rinv < 1e12f;  // ||x|| > eps
#pragma unroll
    for (int t = 0; t < C::CPT; ++t) {
      const float gx = big ? (acc[t] - dot * xh_row[acc_col<D>(tx, t)]) : acc[t];
      acc[t] = gx * rinv;
    }
  }
  if (!valid) return;
#pragma unroll
  for (int t = 0; t < C::CPT; ++t) {
    const int col = acc_col<D>(tx, t);
    dst[col] = accumulate ? dst[col] + acc[t] : acc[t];
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) tda_bwd_dq_kernel(const BwdParams p) {
  using C = BwdCfg<D>;
  constexpr int BT = C::BT, R = C::RPT, LDP = C::LDP;
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* Qs = sm;                       // [BT][LD] unit (or raw) query rows
  float* Gs = Qs + C::kTileFloats;      // [BT][LD] scaled dout rows
  float* Ks = Gs + C::kTileFloats;      // [BT][LD]
  float* Vs = Ks + C::kTileFloats;      // [BT][LD]
  float* As = Vs + C::kTileFloats;      // [BT][LDP] dA
  float* rq = As + 2 * BT * LDP;        // [BT]
  float* tau = rq + BT;                 // [BT]
  float* rk = tau + BT;                 // [BT]

  const int n_t = (p.S + BT - 1) / BT;
  const int bh = blockIdx.x % p.BH;
  const int mt = n_t - 1 - static_cast<int>(blockIdx.x / p.BH);
  const int m0 = mt * BT;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int n_kt = p.beta >= 0.0f ? mt + 1 : n_t;
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* v = static_cast<const T*>(p.v);
  const T* g = static_cast<const T*>(p.dout);

  if (threadIdx.x < BT) {
    tau[threadIdx.x] = p.beta * sqrtf((2.0f * logf(static_cast<float>(m0 + threadIdx.x + 1))) / static_cast<float>(D));
    rq[threadIdx.x] = 1.0f;
  }
  load_rows<D, T>(Qs, C::LD, q, bh, m0, p.S, 1.0f);
  load_rows<D, T>(Gs, C::LD, g, bh, m0, p.S, p.dout_scale);
  __syncthreads();
  if (p.normalize) normalize_rows<D>(Qs, rq);

  float acc[R][C::CPT];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int t = 0; t < C::CPT; ++t) acc[i][t] = 0.f;

  for (int kt = 0; kt < n_kt; ++kt) {
    const int n0 = kt * BT;
    __syncthreads();  // previous tile's K and dA consumed
    load_rows<D, T>(Ks, C::LD, k, bh, n0, p.S, 1.0f);
    load_rows<D, T>(Vs, C::LD, v, bh, n0, p.S, 1.0f);
    __syncthreads();
    if (p.normalize) {
      normalize_rows<D>(Ks, rk);
      __syncthreads();
    }
    float s[R][R], dp[R][R];
    two_score_tiles<D>(s, dp, Qs, Ks, Gs, Vs, ty, tx);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int r = ty + 16 * i;
#pragma unroll
      for (int c = 0; c < R; ++c) {
        const int cj = tx + 16 * c;
        const float sv = (n0 + cj <= m0 + r) ? s[i][c] : 0.0f;  // causal mask to zero
        As[r * LDP + cj] = dp[i][c] * relu_pow_grad_ref(sv - tau[r], p.relu_power);
      }
    }
    __syncthreads();
    mac_rows<D>(acc, As, Ks, ty, tx);
  }

#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int r = ty + 16 * i;
    const bool valid = m0 + r < p.S;
    float* dst = p.dq + (static_cast<size_t>(bh) * p.S + (valid ? m0 + r : 0)) * D;
    store_grad_row<D>(dst, acc[i], Qs + r * C::LD, rq[r], p.normalize != 0, false, valid, tx);
  }
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads) tda_bwd_dkv_kernel(const BwdParams p) {
  using C = BwdCfg<D>;
  constexpr int BT = C::BT, R = C::RPT, LDP = C::LDP;
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* Ks = sm;                       // [BT][LD] unit (or raw) key rows
  float* Vs = Ks + C::kTileFloats;      // [BT][LD]
  float* Qs = Vs + C::kTileFloats;      // [BT][LD]
  float* Gs = Qs + C::kTileFloats;      // [BT][LD] scaled dout rows
  float* Pt = Gs + C::kTileFloats;      // [BT keys][LDP] P^T
  float* At = Pt + BT * LDP;            // [BT keys][LDP] dA^T
  float* rk = At + BT * LDP;            // [BT]
  float* tau = rk + BT;                 // [BT]
  float* rq = tau + BT;                 // [BT]

  const int n_t = (p.S + BT - 1) / BT;
  const int bh = blockIdx.x % p.BH;
  const int nt = static_cast<int>(blockIdx.x / p.BH);  // key tiles near the start see the most queries
  const int n0 = nt * BT;
  const int ty = threadIdx.x >> 4, tx = threadIdx.x & 15;
  const int mt_first = p.beta >= 0.0f ? nt : 0;
  const T* q = static_cast<const T*>(p.q);
  const T* k = static_cast<const T*>(p.k);
  const T* v = static_cast<const T*>(p.v);
  const T* g = static_cast<const T*>(p.dout);

  if (threadIdx.x < BT) rk[threadIdx.x] = 1.0f;
  load_rows<D, T>(Ks, C::LD, k, bh, n0, p.S, 1.0f);
  load_rows<D, T>(Vs, C::LD, v, bh, n0, p.S, 1.0f);
  __syncthreads();
  if (p.normalize) normalize_rows<D>(Ks, rk);

  float dk[R][C::CPT], dv[R][C::CPT];
#pragma unroll
  for (int i = 0; i < R; ++i)
#pragma unroll
    for (int t = 0; t < C::CPT; ++t) {
      dk[i][t] = 0.f;
      dv[i][t] = 0.f;
    }

  for (int mt = mt_first; mt < n_t; ++mt) {
    const int m0 = mt * BT;
    __syncthreads();  // previous tile's Q, dout, P^T, dA^T consumed
    load_rows<D, T>(Qs, C::LD, q, bh, m0, p.S, 1.0f);
    load_rows<D, T>(Gs, C::LD, g, bh, m0, p.S, p.dout_scale);
    if (threadIdx.x < BT)
      tau[threadIdx.x] =
          p.beta * sqrtf((2.0f * logf(static_cast<float>(m0 + threadIdx.x + 1))) / static_cast<float>(D));
    __syncthreads();
    if (p.normalize) {
      normalize_rows<D>(Qs, rq);
      __syncthreads();
    }
    // rows = keys (ty + 16 i), columns = queries (tx + 16 c)
    float s[R][R], dp[R][R];
    two_score_tiles<D>(s, dp, Ks, Qs, Vs, Gs, ty, tx);
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const int rj = ty + 16 * i;
#pragma unroll
      for (int c = 0; c < R; ++c) {
        const int ci = tx + 16 * c;
        const bool in_seq = m0 + ci < p.S;
        const float sv = (n0 + rj <= m0 + ci) ? s[i][c] : 0.0f;  // causal mask to zero
        const float z = sv - tau[ci];
        // queries past S carry zero dout rows; their P must not reach dV
        Pt[rj * LDP + ci] = in_seq ? relu_pow_ref(z, p.relu_power) : 0.0f;
        At[rj * LDP + ci] = dp[i][c] * relu_pow_grad_ref(z, p.relu_power);
      }
    }
    __syncthreads();
    mac_rows<D>(dv, Pt, Gs, ty, tx);
    mac_rows<D>(dk, At, Qs, ty, tx);
  }

#pragma unroll
  for (int i = 0; i < R; ++i) {
    const int r = ty + 16 * i;
    const bool valid = n0 + r < p.S;
    const size_t off = (static_cast<size_t>(bh) * p.S + (valid ? n0 + r : 0)) * D;
    store_grad_row<D>(p.dk + off, dk[i], Ks + r * C::LD, rk[r], p.normalize != 0, false, valid, tx);
    store_grad_row<D>(p.dv + off, dv[i], nullptr, 1.0f, false, p.accumulate_dv != 0, valid, tx);
  }
}

template <int D, typename T>
cudaError_t launch_bwd_d(const BwdParams& p, cudaStream_t stream) {
  using C = BwdCfg<D>;
  auto kq = tda_bwd_dq_kernel<D, T>;
  auto kkv = tda_bwd_dkv_kernel<D, T>;
  cudaError_t e = cudaFuncSetAttribute(kq, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
  if (e != cudaSuccess) return e;
  const int n_t = (p.S + C::BT - 1) / C::BT;
  const unsigned grid = static_cast<unsigned>(p.BH) * static_cast<unsigned>(n_t);
  kq<<<grid, kThreads, C::kBytes, stream>>>(p);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  kkv<<<grid, kThreads, C::kBytes, stream>>>(p);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_bwd_t(const BwdParams& p, int head_dim, cudaStream_t stream) {
  switch (head_dim) {
    case 16: return launch_bwd_d<16, T>(p, stream);
    case 32: return launch_bwd_d<32, T>(p, stream);
    case 64: return launch_bwd_d<64, T>(p, stream);
    case 128: return launch_bwd_d<128, T>(p, stream);
    case 256: return launch_bwd_d<256, T>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t launch_rect_bwd(const BwdParams& p, int head_dim, bool in_bf16, cudaStream_t stream) {
  return in_bf16 ? launch_bwd_t<__nv_bfloat16>(p, head_dim, stream) : launch_bwd_t<float>(p, head_dim, stream);
}

}  // namespace tda
