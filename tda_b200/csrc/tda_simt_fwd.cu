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
// K/V tiles are fetched with cp.async into two stages (one where the stages
// would not fit in shared memory, head_dim 256), so the next tile's loads
// overlap this tile's arithmetic; 1/||k_j|| is summed by four threads per key;
// the P.V loop reads P four keys at a time (one 16-byte load per row).
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
  static constexpr int kStageFloats = BN * LD + BN * D;  // one K tile + one V tile
  static constexpr int kFixedFloats = BM * LD + BM * LDP + BN + 3 * BM;
  static constexpr int kStages = (kFixedFloats + 2 * kStageFloats) * 4 <= 232448 ? 2 : 1;
  static constexpr int kFloats = kFixedFloats + kStages * kStageFloats;
  static constexpr int kBytes = kFloats * 4;
  static constexpr int kColGroups = D >= 64 ? D / 64 : 1;  // float4 groups per thread along D
  static constexpr int kColsPerThread = D / 16;
};

// 16-byte global -> shared copy that bypasses registers; src_bytes = 0 fills
// the destination with zeros (rows past S).
__device__ __forceinline__ void cp_async16(float* dst, const float* src, bool valid) {
  const unsigned d = static_cast<unsigned>(__cvta_generic_to_shared(dst));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(d), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;\n" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;\n" ::"n"(N) : "memory"); }

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

// the same rows, copied asynchronously (completion: cp_async_wait + a barrier)
template <int D>
__device__ __forceinline__ void load_rows_async(float* dst, int ld, const float* src, int bh, int r0, int S) {
  constexpr int V4 = D / 4;
  const float* base = src + static_cast<size_t>(bh) * S * D;
  for (int idx = threadIdx.x; idx < 64 * V4; idx += kSimtThreads) {
    const int r = idx / V4, c4 = idx % V4;
    const bool ok = r0 + r < S;
    cp_async16(dst + r * ld + 4 * c4, base + static_cast<size_t>(ok ? r0 + r : 0) * D + 4 * c4, ok);
  }
}

template <int D>
__global__ void __launch_bounds__(kSimtThreads) tda_simt_fwd_kernel(const SimtFwdParams p) {
  using C = SimtCfg<D>;
  extern __shared__ float4 smem_f4[];
  float* sm = reinterpret_cast<float*>(smem_f4);
  float* Qs = sm;                              // [BM][LD]
  float* stage0 = Qs + BM * C::LD;             // per stage: K [BN][LD], then V [BN][D]
  float* Ps = stage0 + C::kStages * C::kStageFloats;  // [BM][LDP]
  float* rk = Ps + BM * LDP;                    // [BN]
  float* rq = rk + BN;                         // [BM]
  float* tq = rq + BM;                         // [BM]
  float* tau = tq + BM;                        // [BM]

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
    const float w = br ? -lambda_of(p.lam_dev, bh, p.lam) : 1.0f;
    __syncthreads();  // the previous branch's last tile fully consumed
    load_rows<D>(Qs, C::LD, q, bh, m0, p.S);
    load_rows_async<D>(stage0, C::LD, k, bh, 0, p.S);
    load_rows_async<D>(stage0 + BN * C::LD, D, p.v, bh, 0, p.S);
    cp_async_commit();
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
      float* Ks = stage0 + (C::kStages == 2 ? (kt & 1) : 0) * C::kStageFloats;
      float* Vs = Ks + BN * C::LD;
      // Stage reuse: the stage written here was last read before the barrier
      // that ended the previous iteration.
      if constexpr (C::kStages == 2) {
        if (kt + 1 < n_kt) {
          float* nk = stage0 + ((kt + 1) & 1) * C::kStageFloats;
          load_rows_async<D>(nk, C::LD, k, bh, n0 + BN, p.S);
          load_rows_async<D>(nk + BN * C::LD, D, p.v, bh, n0 + BN, p.S);
          cp_async_commit();
          cp_async_wait<1>();
        } else {
          cp_async_wait<0>();
        }
      } else {
        if (kt > 0) {
          load_rows_async<D>(Ks, C::LD, k, bh, n0, p.S);
          load_rows_async<D>(Vs, D, p.v, bh, n0, p.S);
          cp_async_commit();
        }
        cp_async_wait<0>();
      }
      __syncthreads();  // tile kt in shared memory for every thread
      {
        // 1/max(||k_j||, eps): four adjacent lanes per key, D/4 dims each
        const int key = tid >> 2, part = tid & 3;
        float ss = 0.f;
        if (p.normalize) {
#pragma unroll
          for (int d = part * (D / 4); d < (part + 1) * (D / 4); d += 4) {
            const float4 x = *reinterpret_cast<const float4*>(Ks + key * C::LD + d);
            ss = fmaf(x.x, x.x, ss);
            ss = fmaf(x.y, x.y, ss);
            ss = fmaf(x.z, x.z, ss);
            ss = fmaf(x.w, x.w, ss);
          }
          ss += __shfl_xor_sync(0xffffffffu, ss, 1);
          ss += __shfl_xor_sync(0xffffffffu, ss, 2);
        }
        if (part == 0) rk[key] = p.normalize ? 1.0f / fmaxf(sqrtf(ss), 1e-12f) : 1.0f;
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
      // O += P V, four keys per step: one 16-byte P load per row
#pragma unroll 2
      for (int j = 0; j < BN; j += 4) {
        float4 p4[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) p4[i] = *reinterpret_cast<const float4*>(Ps + (ty + 16 * i) * LDP + j);
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          float pr[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            pr[i] = jj == 0 ? p4[i].x : (jj == 1 ? p4[i].y : (jj == 2 ? p4[i].z : p4[i].w));
          if constexpr (D >= 64) {
#pragma unroll
            for (int g = 0; g < C::kColGroups; ++g) {
              const float4 vv = *reinterpret_cast<const float4*>(Vs + (j + jj) * D + 64 * g + 4 * tx);
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
              const float vv = Vs[(j + jj) * D + tx * C::kColsPerThread + cc];
#pragma unroll
              for (int i = 0; i < 4; ++i) o[i][cc] = fmaf(pr[i], vv, o[i][cc]);
            }
          }
        }
      }
      __syncthreads();  // P and this stage consumed before they are overwritten
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
