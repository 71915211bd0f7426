// Key-norm pre-pass for the normalized tensor-core path (any (batch, head,
// seq, dim) strides with a contiguous last dimension).  For one key tensor
// it writes a "key table" of BH * S_pad * 17/16 floats:
//   rk[bh * S_pad + j]              = 1 / max(||k[bh][j]||_2, 1e-12)  (F.normalize
//                                     eps, triton_threshold_attention.py:505-509),
//                                     0 for padding rows S <= j < S_pad
//   rkmax[bh * S_pad / 16 + g]      = max of rk over keys [16 g, 16 g + 16)
// (rkmax starts right after rk).  The forward kernels use rkmax to prove a
// 16-key group of scores lies below the threshold from the raw scores alone.
// HBM-bound: reads B*H*S*D*2 bytes.  One warp per 16 consecutive keys; all of
// its 16-byte loads issued first, fp32 sums of squares, IEEE sqrt and divide.
#include <cuda_bf16.h>

#include "tda_internal.h"

namespace tda {
namespace {

// x is a (batch, head, seq, dim) view with element strides (sb, sh, ss) and a
// contiguous last dimension; bh = b * heads + h.
template <int D>
__global__ void __launch_bounds__(256) key_norm_kernel(const __nv_bfloat16* __restrict__ x, float* __restrict__ table,
                                                       int BH, int S, int S_pad, int heads, long long sb,
                                                       long long sh, long long ss_) {
  constexpr int kRowBytes = D * 2;
  constexpr int kLanesPerRow = kRowBytes / 16;       // 16 (D = 128) or 8 (D = 64)
  constexpr int kRowsPerIter = 32 / kLanesPerRow;    // 2 or 4
  constexpr int kIters = 16 / kRowsPerIter;
  const int lane = threadIdx.x & 31;
  const int sub = lane / kLanesPerRow;
  const int sl = lane % kLanesPerRow;
  const long long groups = static_cast<long long>(BH) * (S_pad / 16);
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  float* rkmax = table + static_cast<size_t>(BH) * S_pad;
  for (long long g = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5; g < groups; g += n_warps) {
    const int bh = static_cast<int>(g / (S_pad / 16));
    const int j0 = static_cast<int>(g % (S_pad / 16)) * 16;
    const __nv_bfloat16* xb = x + static_cast<long long>(bh / heads) * sb + static_cast<long long>(bh % heads) * sh;
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
        const float2 v = make_float2(__uint_as_float(w[h] << 16), __uint_as_float(w[h] & 0xFFFF0000u));
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

template <int D>
cudaError_t launch_kn(const void* x, float* table, int BH, int S, int S_pad, int heads, long long sb, long long sh,
                      long long ss, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const long long groups = static_cast<long long>(BH) * (S_pad / 16);
  long long blocks = (groups + 7) / 8;
  const long long cap = static_cast<long long>(sms) * 16;  // grid-stride beyond 16 CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  key_norm_kernel<D><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(static_cast<const __nv_bfloat16*>(x), table,
                                                                         BH, S, S_pad, heads, sb, sh, ss);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_key_norms(const void* x, int x_is_bf16, float* rk, int BH, int S, int S_pad, int D,
                             cudaStream_t stream) {
  if (x_is_bf16) {
    // contiguous (BH, S, D): one "batch" of BH heads
    const long long sh = static_cast<long long>(S) * D;
    if (D == 64) return launch_kn<64>(x, rk, BH, S, S_pad, BH, sh * BH, sh, D, stream);
    if (D == 128) return launch_kn<128>(x, rk, BH, S, S_pad, BH, sh * BH, sh, D, stream);
  }
  return cudaErrorInvalidValue;
}

cudaError_t launch_key_norms_strided(const void* x, float* rk, int BH, int heads, int S, int S_pad, int D,
                                     int64_t stride_b, int64_t stride_h, int64_t stride_s, cudaStream_t stream) {
  if (D == 64) return launch_kn<64>(x, rk, BH, S, S_pad, heads, stride_b, stride_h, stride_s, stream);
  if (D == 128) return launch_kn<128>(x, rk, BH, S, S_pad, heads, stride_b, stride_h, stride_s, stream);
  return cudaErrorInvalidValue;
}

}  // namespace tda
