// CUDA-core fp32 forward of threshold rectified / differential attention.
//
// The fp32 path must meet rel-L2 <= 1e-5 against an fp64 oracle, which rules
// out single-pass TF32 tensor-core math, so this kernel does exact fp32 FFMA
// (it is the path for fp32 inputs and any head_dim outside {64, 128}).
// Semantics follow triton_threshold_attention.py:19-115 (mask-to-zero causal,
// threshold, power branch incl. exp(p*log(x+1e-10))) and :489-519 (normalize,
// clamp(lambda), out1 - lambda*out2, here accumulated into one output).
//
// One CTA = 64 query rows x one (batch, head); 256 threads as a 16 x 16 grid.
// Thread (ty, tx) owns score rows {ty + 16 i} and key columns {tx + 16 c}
// (i, c < 4), and output rows {ty + 16 i} x columns {64 g + 4 tx + t}.
#include "tda_internal.h"

namespace tda {
namespace {

constexpr int BM = 64;
constexpr int BN = 64;
constexpr int kSimtThreads = 256;
constexpr int LDP = BN + 16;  // P row stride (floats), bank-conflict free for both phases

template <int D>
struct SimtCfg {
  static constexpr int LD = D + 4;  // Q/K row stride (floats)
  static constexpr int kFloats = 2 * BM * LD + BN * D + BM * LDP + BN + 3 * BM;
  static constexpr int kBytes = kFloats * 4;
  static constexpr int kColGroups = D >= 64 ? D / 64 : 1;  // float4 groups per thread along D
  static constexpr int kColsPerThread = D / 16;
};

__device__ __forceinline__ float relu_pow_ref(float z, float p) {
  const float x = fmaxf(z, 0.0f);
  if (p == 2.0f) return x * x;
  if (p == 1.0f) return x;
  return x > 0.0f ? expf(p * logf(x + 1e-10f)) : 0.0f;
}

// rows [r0, r0 + 64) of a (BH, S, D) fp32 array -> shared [64][ld], zero past S.
template <int D>
__device__ __forceinline__ void load_rows(float* dst, int ld, const float* src, int bh, int r0, int S) {
  constexpr int V4 = D / 4;
  for (int idx = threadIdx.x; idx < 64 * V4; idx += kSimtThreads) {
    const int r = idx / V4, c4 = idx % V4;
    float4 val = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < S)
      val = *reinterpret_cast<const float4*>(src + (static_cast<size_t>(bh) * S + r0 + r) * D + 4 * c4);
    *reinterpret_cast<float4*>(dst + r * ld + 4 * c4) = val;
  }
}

template <int D>
__global__ void __launch_bounds__(kSimtThreads) tda_simt_fwd_kernel(const SimtFwdParams p) {
  using C = SimtCfg<D>;
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* Qs = sm;                  // [BM][LD]
  float* Ks = Qs + BM * C::LD;     // [BN][LD]
  float* Vs = Ks + BN * C::LD;     // [BN][D]
  float* Ps = Vs + BN * D;         // [BM][LDP]
  float* rk = Ps + BM * LDP;       // [BN]
  float* rq = rk + BN;             // [BM]
  float* tq = rq + BM;             // [BM]
  float* tau = tq + BM;            // [BM]

  const int n_mt = (p.S + BM - 1) / BM;
  const int bh = blockIdx.x % p.BH;
  const int mt = n_mt - 1 - static_cast<int>(blockIdx.x / p.BH);
  const int m0 = mt * BM;
  const int tid = threadIdx.x;
  const int ty = tid >> 4, tx = tid & 15;
  const int n_kt = p.beta >= 0.0f ? mt + 1 : n_mt;

  if (tid < BM) {
    const int gi = m0 + tid;
    tau[tid] = p.beta * sqrtf((2.0f * logf(static_cast<float>(gi + 1))) / static_cast<float>(D));
  }

  float o[4][C::kColsPerThread];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int c = 0; c < C::kColsPerThread; ++c) o[i][c] = 0.f;

  const int n_branch = p.differential ? 2 : 1;
  for (int br = 0; br < n_branch; ++br) {
    const float* q = br ? p.q2 : p.q1;
    const float* k = br ? p.k2 : p.k1;
    const float w = br ? -p.lam : 1.0f;
    __syncthreads();
    load_rows<D>(Qs, C::LD, q, bh, m0, p.S);
    __syncthreads();
    if (tid < BM) {
      float m = 1.0f, t = tau[tid];
      if (p.normalize) {
        float ss = 0.f;
        for (int d = 0; d < D; ++d) ss = fmaf(Qs[tid * C::LD + d], Qs[tid * C::LD + d], ss);
        m = fmaxf(sqrtf(ss), 1e-12f);
        t = t * m;
      }
      rq[tid] = 1.0f / m;
      tq[tid] = t;
    }
    for (int kt = 0; kt < n_kt; ++kt) {
      const int n0 = kt * BN;
      __syncthreads();  // previous tile's P and V fully consumed
      load_rows<D>(Ks, C::LD, k, bh, n0, p.S);
      load_rows<D>(Vs, D, p.v, bh, n0, p.S);
      __syncthreads();
      if (tid < BN) {
        float r = 1.0f;
        if (p.normalize) {
          float ss = 0.f;
          for (int d = 0; d < D; ++d) ss = fmaf(Ks[tid * C::LD + d], Ks[tid * C::LD + d], ss);
          r = 1.0f / fmaxf(sqrtf(ss), 1e-12f);
        }
        rk[tid] = r;
      }
      // S = Q K^T for this thread's 4 x 4 entries
      float s[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int c = 0; c < 4; ++c) s[i][c] = 0.f;
#pragma unroll 2
      for (int d = 0; d < D; d += 4) {
        float4 qa[4], kb[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) qa[i] = *reinterpret_cast<const float4*>(Qs + (ty + 16 * i) * C::LD + d);
#pragma unroll
        for (int c = 0; c < 4; ++c) kb[c] = *reinterpret_cast<const float4*>(Ks + (tx + 16 * c) * C::LD + d);
#pragma unroll
        for (int i = 0; i < 4; ++i)
#pragma unroll
          for (int c = 0; c < 4; ++c) {
            s[i][c] = fmaf(qa[i].x, kb[c].x, s[i][c]);
            s[i][c] = fmaf(qa[i].y, kb[c].y, s[i][c]);
            s[i][c] = fmaf(qa[i].z, kb[c].z, s[i][c]);
            s[i][c] = fmaf(qa[i].w, kb[c].w, s[i][c]);
          }
      }
      __syncthreads();  // rk visible
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = ty + 16 * i;
        const int gi = m0 + r;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int cidx = tx + 16 * c;
          const int gj = n0 + cidx;
          float sv = (gj <= gi) ? s[i][c] : 0.0f;  // causal mask to zero
          const float z = p.normalize ? fmaf(sv, rk[cidx], -tq[r]) * rq[r] : sv - tau[r];
          Ps[r * LDP + cidx] = w * relu_pow_ref(z, p.relu_power);
        }
      }
      __syncthreads();
      // O += P V
#pragma unroll 4
      for (int j = 0; j < BN; ++j) {
        float pr[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) pr[i] = Ps[(ty + 16 * i) * LDP + j];
        if constexpr (D >= 64) {
#pragma unroll
          for (int g = 0; g < C::kColGroups; ++g) {
            const float4 vv = *reinterpret_cast<const float4*>(Vs + j * D + 64 * g + 4 * tx);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
              o[i][4 * g + 0] = fmaf(pr[i], vv.x, o[i][4 * g + 0]);
              o[i][4 * g + 1] = fmaf(pr[i], vv.y, o[i][4 * g + 1]);
              o[i][4 * g + 2] = fmaf(pr[i], vv.z, o[i][4 * g + 2]);
              o[i][4 * g + 3] = fmaf(pr[i], vv.w, o[i][4 * g + 3]);
            }
          }
        } else {
#pragma unroll
          for (int cc = 0; cc < C::kColsPerThread; ++cc) {
            const float vv = Vs[j * D + tx * C::kColsPerThread + cc];
#pragma unroll
            for (int i = 0; i < 4; ++i) o[i][cc] = fmaf(pr[i], vv, o[i][cc]);
          }
        }
      }
    }
  }

#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int gi = m0 + ty + 16 * i;
    if (gi >= p.S) continue;
    float* dst = p.out + (static_cast<size_t>(bh) * p.S + gi) * D;
    if constexpr (D >= 64) {
#pragma unroll
      for (int g = 0; g < C::kColGroups; ++g)
        *reinterpret_cast<float4*>(dst + 64 * g + 4 * tx) =
            make_float4(o[i][4 * g + 0], o[i][4 * g + 1], o[i][4 * g + 2], o[i][4 * g + 3]);
    } else {
#pragma unroll
      for (int cc = 0; cc < C::kColsPerThread; ++cc) dst[tx * C::kColsPerThread + cc] = o[i][cc];
    }
  }
}

template <int D>
cudaError_t launch_d(const SimtFwdParams& p, cudaStream_t stream) {
  using C = SimtCfg<D>;
  auto kern = tda_simt_fwd_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kBytes);
  if (e != cudaSuccess) return e;
  const int n_mt = (p.S + BM - 1) / BM;
  const unsigned grid = static_cast<unsigned>(p.BH) * static_cast<unsigned>(n_mt);
  kern<<<grid, kSimtThreads, C::kBytes, stream>>>(p);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_simt_fwd(const SimtFwdParams& p, int head_dim, cudaStream_t stream) {
  switch (head_dim) {
    case 16: return launch_d<16>(p, stream);
    case 32: return launch_d<32>(p, stream);
    case 64: return launch_d<64>(p, stream);
    case 128: return launch_d<128>(p, stream);
    case 256: return launch_d<256>(p, stream);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tda
