// Key-norm pre-pass for the normalized tensor-core path:
//   rk[bh][j] = 1 / max(||k[bh][j]||_2, 1e-12)   (F.normalize eps,
//   triton_threshold_attention.py:505-509), 0 for padding rows S <= j < S_pad.
// HBM-bound: reads B*H*S*D*elt bytes, writes B*H*S_pad*4 bytes.  One warp per
// key row group; 16-byte loads, fp32 sum of squares, IEEE sqrt and divide.
#include <cuda_bf16.h>

#include "tda_internal.h"

namespace tda {
namespace {

template <int D, bool BF16>
__global__ void __launch_bounds__(256) key_norm_kernel(const void* __restrict__ x, float* __restrict__ rk, int BH,
                                                       int S, int S_pad) {
  // bytes per row and lanes per row: one 16-byte vector per lane
  constexpr int kRowBytes = D * (BF16 ? 2 : 4);
  constexpr int kLanesPerRow = kRowBytes / 16 < 32 ? kRowBytes / 16 : 32;
  constexpr int kVecPerLane = kRowBytes / 16 / kLanesPerRow;
  constexpr int kRowsPerWarp = 32 / kLanesPerRow;
  const int lane = threadIdx.x & 31;
  const int sub = lane / kLanesPerRow;
  const int sl = lane % kLanesPerRow;
  const long long total_rows = static_cast<long long>(BH) * S_pad;
  const long long warp_global = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const long long n_warps = (static_cast<long long>(gridDim.x) * blockDim.x) >> 5;
  for (long long base = warp_global * kRowsPerWarp; base < total_rows; base += n_warps * kRowsPerWarp) {
    const long long r = base + sub;
    const int bh = static_cast<int>(r / S_pad);
    const int j = static_cast<int>(r % S_pad);
    float ss = 0.f;
    const bool valid = (r < total_rows) && (j < S);
    if (valid) {
      const uint4* row = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(x) +
                                                        (static_cast<size_t>(bh) * S + j) * kRowBytes);
#pragma unroll
      for (int v = 0; v < kVecPerLane; ++v) {
        const uint4 u = row[sl + v * kLanesPerRow];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
        if constexpr (BF16) {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float lo = __uint_as_float(w[h] << 16), hi = __uint_as_float(w[h] & 0xFFFF0000u);
            ss = fmaf(lo, lo, ss);
            ss = fmaf(hi, hi, ss);
          }
        } else {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float f = __uint_as_float(w[h]);
            ss = fmaf(f, f, ss);
          }
        }
      }
    }
#pragma unroll
    for (int off = kLanesPerRow / 2; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
    if (sl == 0 && r < total_rows) rk[r] = (j < S) ? 1.0f / fmaxf(sqrtf(ss), 1e-12f) : 0.0f;
  }
}

template <int D, bool BF16>
cudaError_t launch_kn(const void* x, float* rk, int BH, int S, int S_pad, cudaStream_t stream) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  constexpr int kRowBytes = D * (BF16 ? 2 : 4);
  constexpr int kLanesPerRow = kRowBytes / 16 < 32 ? kRowBytes / 16 : 32;
  constexpr int kRowsPerWarp = 32 / kLanesPerRow;
  const long long rows = static_cast<long long>(BH) * S_pad;
  const long long warps_needed = (rows + kRowsPerWarp - 1) / kRowsPerWarp;
  long long blocks = (warps_needed + 7) / 8;
  const long long cap = static_cast<long long>(sms) * 16;  // grid-stride beyond 16 CTAs per SM
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  key_norm_kernel<D, BF16><<<static_cast<unsigned>(blocks), 256, 0, stream>>>(x, rk, BH, S, S_pad);
  return cudaGetLastError();
}

}  // namespace

cudaError_t launch_key_norms(const void* x, int x_is_bf16, float* rk, int BH, int S, int S_pad, int D,
                             cudaStream_t stream) {
  if (x_is_bf16) {
    if (D == 64) return launch_kn<64, true>(x, rk, BH, S, S_pad, stream);
    if (D == 128) return launch_kn<128, true>(x, rk, BH, S, S_pad, stream);
  }
  return cudaErrorInvalidValue;
}

}  // namespace tda
