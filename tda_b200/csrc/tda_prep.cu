// Key-norm pre-pass for the normalized tensor-core path (any (batch, head,
// seq, dim) strides with a contiguous last dimension).  For one key tensor
// it writes a "key table" of BH * S_pad * 17/16 floats:
//   rk[bh * S_pad + j]              = 1 / max(||k[bh][j]||_2, 1e-12)  (F.normalize
//                                     eps, triton_threshold_attention.py:505-509),
//                                     0 for padding rows S <= j < S_pad
//   rkmax[bh * S_pad / 16 + g]      = max of rk over keys [16 g, 16 g + 16)
// (rkmax starts right after rk).  The forward kernels use rkmax to prove a
// 16-key group of scores lies below the threshold from the raw scores alone.
// HBM-bound: reads B*H*S*D*2 bytes per key tensor (bf16 or fp16).  One warp per
// 16 consecutive keys; all of its 16-byte loads issued first, fp32 sums of
// squares, IEEE sqrt and divide.  The differential form's two key tensors go
// through one launch.
#include <cuda_bf16.h>

#include "tda_internal.h"
#include "tda_ptx.cuh"

namespace tda {
namespace {

// Up to two key tensors per launch (the differential form's k1 and k2): each a
// (batch, head, seq, dim) view with element strides (sb, sh, ss) and a
// contiguous last dimension; bh = b * heads + h.
struct KeyViews {
  const void* x[2];
  float* table[2];
  long long sb[2], sh[2], ss[2];
  int n;
};

template <int D, bool F16>
__global__ void __launch_bounds__(256) key_norm_kernel(const KeyViews kv, int BH, int S, int S_pad, int heads) {
  constexpr int kRowBytes = D * 2;
  constexpr int kLanesPerRow = kRowBytes / 16;       // 16 (D = 128) or 8 (D = 64)
  constexpr int kRowsPerIter = 32 / kLanesPerRow;    // 2 or 4
  constexpr int kIters = 16 / kRowsPerIter;
  const int lane = threadIdx.x & 31;
  const int sub = lane / kLanesPerRow;
  const int sl = lane % kLanesPerRow;
  const long long groups = static_cast<long long>(BH) * (S_pad / 16);  // per tensor
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long gt = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; gt < kv.n * groups;
       gt += n_warps) {
    const int t = gt >= groups ? 1 : 0;
    const long long g = gt - t * groups;
    // selects rather than a runtime index into the parameter arrays (which
    // would copy them to local memory)
    float* table = t ? kv.table[1] : kv.table[0];
    float* rkmax = table + static_cast<size_t>(BH) * S_pad;
    const int bh = static_cast<int>(g / (S_pad / 16));
    const int j0 = static_cast<int>(g % (S_pad / 16)) * 16;
    const uint16_t* xb = static_cast<const uint16_t*>(t ? kv.x[1] : kv.x[0]) +
                         static_cast<long long>(bh / heads) * (t ? kv.sb[1] : kv.sb[0]) +
                         static_cast<long long>(bh % heads) * (t ? kv.sh[1] : kv.sh[0]);
    const long long ss_ = t ? kv.ss[1] : kv.ss[0];
    // all of the group's 16-byte loads first (more bytes in flight), then
    // the sums of squares with packed f32x2 FMAs (two accumulators per lane)
    uint4 u[kIters];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int j = j0 + it * kRowsPerIter + sub;
      u[it] = j < S ? reinterpret_cast<const uint4*>(xb + static_cast<long long>(j) * ss_)[sl] : make_uint4(0, 0, 0, 0);
    }
    float mx = 0.0f;
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int j = j0 + it * kRowsPerIter + sub;
      const uint32_t w[4] = {u[it].x, u[it].y, u[it].z, u[it].w};
      float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float2 v = F16 ? unpack_f16x2(w[h]) : unpack_bf16x2(w[h]);
        acc = __ffma2_rn(v, v, acc);
      }
      float ss = acc.x + acc.y;
#pragma unroll
      for (int off = kLanesPerRow / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
      const float r = (j < S) ? 1.0f / fmaxf(sqrtf(ss), 1e-12f) : 0.0f;
      if (sl == 0) table[static_cast<size_t>(bh) * S_pad + j] = r;
      mx = fmaxf(mx, r);
    }
#pragma unroll
    for (int off = kLanesPerRow; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    if (lane == 0) rkmax[g] = mx;
  }
}

template <int D, bool F16>
cudaError_t launch_kn(const KeyViews& kv, int BH, int S, int S_pad, int heads, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long groups = static_cast<long long>(kv.n) * BH * (S_pad / 16);
  long long blocks = (groups + 7) / 8;
  const long long cap = static_cast<long long>(sms) * 16;  // grid-stride beyond 16 CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  key_norm_kernel<D, F16><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(kv, BH, S, S_pad, heads);
  return cudaGetLastError();
}

cudaError_t launch_views(const KeyViews& kv, int dtype, int BH, int heads, int S, int S_pad, int D,
                         cudaStream_t stream) {
  const bool f16 = dtype == 2;
  if (dtype != 1 && dtype != 2) return cudaErrorInvalidValue;
  if (D == 64) return f16 ? launch_kn<64, true>(kv, BH, S, S_pad, heads, stream)
                          : launch_kn<64, false>(kv, BH, S, S_pad, heads, stream);
  if (D == 128) return f16 ? launch_kn<128, true>(kv, BH, S, S_pad, heads, stream)
                           : launch_kn<128, false>(kv, BH, S, S_pad, heads, stream);
  return cudaErrorInvalidValue;
}

}  // namespace

cudaError_t launch_key_norms(const void* x, int dtype, float* rk, int BH, int S, int S_pad, int D,
                             cudaStream_t stream) {
  return launch_key_norms_pair(x, nullptr, dtype, rk, nullptr, BH, S, S_pad, D, stream);
}

cudaError_t launch_key_norms_pair(const void* x1, const void* x2, int dtype, float* rk1, float* rk2, int BH, int S,
                                  int S_pad, int D, cudaStream_t stream) {
  // contiguous (BH, S, D): one "batch" of BH heads
  const long long sh = static_cast<long long>(S) * D;
  KeyViews kv{{x1, x2}, {rk1, rk2}, {sh * BH, sh * BH}, {sh, sh}, {D, D}, x2 ? 2 : 1};
  return launch_views(kv, dtype, BH, BH, S, S_pad, D, stream);
}

cudaError_t launch_key_norms_strided(int n, const void* const x[2], float* const rk[2], int dtype, int BH, int heads,
                                     int S, int S_pad, int D, const int64_t stride_b[2], const int64_t stride_h[2],
                                     const int64_t stride_s[2], cudaStream_t stream) {
  if (n < 1 || n > 2) return cudaErrorInvalidValue;
  KeyViews kv{};
  kv.n = n;
  for (int t = 0; t < n; ++t) {
    kv.x[t] = x[t];
    kv.table[t] = rk[t];
    kv.sb[t] = stride_b[t];
    kv.sh[t] = stride_h[t];
    kv.ss[t] = stride_s[t];
  }
  return launch_views(kv, dtype, BH, heads, S, S_pad, D, stream);
}

}  // namespace tda
