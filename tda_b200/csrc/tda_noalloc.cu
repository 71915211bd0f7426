// tda_diff_fwd_noalloc: the fused differential forward for callers that must
// not allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- for example
// inside a custom allocator or memory-pool callback (allocating there would
// re-enter the allocator), in a pre-sized inference runtime that forbids any
// allocation after start-up, or in a plugin whose host framework owns all
// device memory and hands it only inputs and outputs.  tda_diff_fwd needs a
// caller-provided workspace for the per-key inverse norms; this variant keeps
// that scratch in a fixed-size array compiled into the library instead.
//
// The first call on each device looks up the array's device address (the
// set-up step); make that first call before capturing the stream into a CUDA
// graph.  The array below is reserved on every GPU that loads the library, for
// the life of the process (8.5 MiB).  It holds the inverse key norms of k1 and k2
// (it is passed to tda_diff_fwd as its workspace), so it limits
// batch_heads * round_up(seq_len, 128) to kNoAllocMaxRows.
//
// All calls share the one array and it keeps whatever the last call wrote.
// Nothing in it has to start at zero: each call's norm pass rewrites every
// entry that call's main kernel reads (padding included) before the main
// kernel runs on the same stream.  Two calls whose GPU work overlaps (on
// different streams, or from different host threads without ordering) race on
// the array and can corrupt each other's results; order them on one stream.
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "../../include/tda_b200.h"
#include "tda_internal.h"

namespace {

constexpr long long kNoAllocMaxRows = 1ll << 20;  // per key tensor: batch_heads * padded seq_len
constexpr long long kTableFloats = kNoAllocMaxRows / 16 * 17;  // key table of one key tensor

// Key tables (inverse norms and their per-16-key maxima) of k1 (first half)
// and k2 (second half).
static __device__ __align__(256) float g_noalloc_scratch[2 * kTableFloats];

constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_addr[kMaxDevices] = {nullptr};

// Device address of g_noalloc_scratch on the current device.  The symbol's
// host-side name is only a stand-in, not a device address, so it must be
// looked up once per device with that device current.
int scratch_on_current_device(float** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return TDA_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return TDA_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char msg[200];
      snprintf(msg, sizeof(msg), "tda_diff_fwd_noalloc: cudaGetSymbolAddress failed on device %d: %s", dev,
               cudaGetErrorString(e));
      tda::set_last_error(msg);
      return TDA_ERR_CUDA;
    }
    g_scratch_addr[dev] = static_cast<float*>(p);
  }
  *out = g_scratch_addr[dev];
  return TDA_OK;
}

}  // namespace

extern "C" int tda_diff_fwd_noalloc(const void* q1, const void* q2, const void* k1, const void* k2, const void* v,
                                    void* out, int dtype, int out_dtype, int64_t batch_heads, int64_t seq_len,
                                    int64_t head_dim, float beta, float lambda_param, float relu_power,
                                    int normalize, int* status, void* stream) {
  const size_t need = dtype == TDA_F32 ? 0 : tda_workspace_size(1, dtype, batch_heads, seq_len, head_dim, normalize);
  if (need == 0) {
    // This configuration uses no scratch at all (fp32 inputs on the CUDA-core
    // kernel, or no normalize).
    return tda_diff_fwd(q1, q2, k1, k2, v, out, dtype, out_dtype, batch_heads, seq_len, head_dim, beta,
                        lambda_param, relu_power, normalize, nullptr, 0, status, stream);
  }
  const long long rows = static_cast<long long>(batch_heads) * tda::padded_seq(seq_len);
  if (rows > kNoAllocMaxRows) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "tda_diff_fwd_noalloc: batch_heads * padded seq_len = %lld exceeds the static scratch limit of "
             "%lld rows (8.5 MiB); use tda_diff_fwd with a caller workspace",
             rows, kNoAllocMaxRows);
    tda::set_last_error(msg);
    return TDA_ERR_INVALID;
  }
  float* scratch = nullptr;
  int rc = scratch_on_current_device(&scratch);
  if (rc != TDA_OK) return rc;
  // The array serves as tda_diff_fwd's workspace: it holds that call's two
  // key tables (bf16 or fp16 keys) for any size within the limit above.
  return tda_diff_fwd(q1, q2, k1, k2, v, out, dtype, out_dtype, batch_heads, seq_len, head_dim, beta, lambda_param,
                      relu_power, normalize, scratch, sizeof(g_noalloc_scratch), status, stream);
}
