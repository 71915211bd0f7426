// Internal (non-exported) launch interfaces shared by the kernel translation
// units and the C-ABI layer.
#pragma once

#include <cstddef>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

namespace tda {

// Power-of-ReLU specialisations (triton_threshold_attention.py:89-101).
enum PowMode : int { POW_1 = 0, POW_2 = 1, POW_3 = 2, POW_GENERAL = 3 };

inline int pow_mode_of(float p) {
  if (p == 1.0f) return POW_1;
  if (p == 2.0f) return POW_2;
  if (p == 3.0f) return POW_3;
  return POW_GENERAL;
}

// lambda of the differential form read on the device per (batch, head): the
// weight of the second branch is clamp(ptr[b * sb + h * sh], 0, 1) with
// b = bh / heads, h = bh % heads (sb / sh = 0 broadcast that dimension).
// ptr == nullptr: every (batch, head) uses the host scalar instead.
struct LamSpec {
  const float* ptr;
  long long sb;
  long long sh;
  int heads;
};

#ifdef __CUDACC__
__device__ __forceinline__ float lambda_of(const LamSpec& l, int bh, float scalar) {
  if (l.ptr == nullptr) return scalar;
  const float x = __ldg(l.ptr + (bh / l.heads) * l.sb + (bh % l.heads) * l.sh);
  return fminf(fmaxf(x, 0.0f), 1.0f);
}
#endif

// Query/key tile edge of the tensor-core kernels (one UMMA M / one key block).
constexpr int kTile = 128;

inline int64_t padded_seq(int64_t S) { return (S + kTile - 1) / kTile * kTile; }

// Tensor-core (tcgen05) forward, bf16 storage.  q/k/v tensor maps view the
// (batch*heads, S, D) arrays as 3-D {D, S, BH} with a {64, 128, 1} box and
// 128-byte swizzle.
// The forward kernel's tensor maps are 4-D {D, S, heads, batches}: a
// (batch, head) index bh is loaded at (bh % heads, bh / heads), so strided
// (batch, head, seq, dim) views (e.g. a (B, S, H, D) tensor transposed) need
// no copy; a contiguous (BH, S, D) array is heads = BH, batches = 1.
struct TcFwdParams {
  CUtensorMap tm_q1;
  CUtensorMap tm_q2;  // differential only
  CUtensorMap tm_k1;
  CUtensorMap tm_k2;  // differential only
  CUtensorMap tm_v;
  CUtensorMap tm_out;  // out, contiguous (BH, S, D) as 3-D {D, S, BH}: box {128 B of elements, 128, 1}, 128-B swizzle
  CUtensorMap tm_k1h;  // head_dim 128: k1 with 64-row boxes (a CTA's half of a key tile, CTA-pair kernel)
  CUtensorMap tm_k2h;  // same for k2 (differential only)
  const float* rk1;   // key table of k1 (normalize only): rk [BH][S_pad] then rkmax [BH][S_pad/16]
  const float* rk2;   // same for k2 (differential + normalize)
  void* out;          // [BH][S][D], bf16 or f32 (out_f32)
  int* status;        // device status word; nonzero after a bounded wait gave up
  int S;
  int S_pad;
  int BH;
  int heads;          // heads per batch in the tensor maps
  int n_qtiles;
  int out_f32;
  int causal_skip;    // 1 when beta >= 0: key tiles past the diagonal contribute 0
  float beta;
  float relu_power;
  float lam;          // clamped lambda (differential)
  float lam_root;     // lambda^(1/p) for p in {1, 2, 3} (folded into the second branch)
  LamSpec lam_dev;    // per-(batch, head) lambda on the device (ptr null: lam / lam_root)
  float tau_scale;    // 2 / D
  float p_scale;      // fp16 inputs: P is multiplied by this power of two before its fp16 split
  float o_unscale;    // fp16 inputs: 1 / p_scale, applied to O in the epilogue
  unsigned long long timeout_ns;
  int inject;         // test hook: bit 0 = producer never loads Q (forces a timeout)
  unsigned* item_ctr;  // persistent kernel: zeroed work-item counter (null: one CTA per query tile)
  // diagnostics (null: off): [0] += 16-key PV slabs multiplied, [1] += slabs a
  // dense PV would multiply, per query tile (one atomic add each per CTA)
  unsigned long long* stats;
};

// fp16 = true: q, k, v (and the output, unless fp32) are fp16 -- kind::f16 with
// fp16 operands, P split into fp16 hi + lo; only with normalize (P bounded).
cudaError_t launch_tc_fwd(const TcFwdParams& p, int head_dim, bool differential, bool normalize, int pow_mode,
                          bool fp16, cudaStream_t stream);
// Whether launch_tc_fwd runs the CTA-pair kernel at this head dim (then the
// caller sets tm_k1h / tm_k2h).
bool tc_fwd_uses_pair(int head_dim);
// The same forward at head_dim 128 on CTA pairs (tm_k1h / tm_k2h set).
cudaError_t launch_tc_fwd_pair(const TcFwdParams& p, bool differential, bool normalize, int pow_mode, bool fp16,
                               cudaStream_t stream);


// CUDA-core fp32 forward (exact fp32 FFMA), any power-of-two D in [16, 256].
struct SimtFwdParams {
  const float* q1;
  const float* k1;
  const float* q2;  // differential only
  const float* k2;  // differential only
  const float* v;
  float* out;
  int S;
  int BH;
  float beta;
  float relu_power;
  float lam;
  LamSpec lam_dev;  // per-(batch, head) lambda on the device (ptr null: lam)
  int normalize;
  int differential;
};

cudaError_t launch_simt_fwd(const SimtFwdParams& p, int head_dim, cudaStream_t stream);

// Tensor-core fp32 forward at head_dim 64 / 128 (tcgen05 kind::tf32, three
// TF32 products per fp32 product).  Sequence padded to whole 64-key tiles.
inline int64_t tf32_padded_seq(int64_t S) { return (S + 63) / 64 * 64; }

// Caller workspace of the fp32 tensor-core path, per branch: TF32 high / low
// copies of q and k ([BH][S][D]), the query coefficients 1/m and tau*m and
// the key coefficients 1/m ([BH][S_pad]); shared: V^T high / low copies
// ([BH][D][S_pad]).  Each array starts on a 256-byte boundary.  With base =
// nullptr only `bytes` is computed.
struct Tf32Workspace {
  float* qh[2];
  float* ql[2];
  float* kh[2];
  float* kl[2];
  float* rq[2];
  float* tq[2];
  float* rk[2];
  float* vth;
  float* vtl;
  size_t bytes;
};

inline Tf32Workspace tf32_carve(void* base, int64_t BH, int64_t S, int64_t D, int n_br) {
  Tf32Workspace w{};
  char* b = static_cast<char*>(base);
  size_t off = 0;
  auto take = [&](size_t floats) -> float* {
    float* p = b ? reinterpret_cast<float*>(b + off) : nullptr;
    off += (floats * sizeof(float) + 255) / 256 * 256;
    return p;
  };
  const size_t x = static_cast<size_t>(BH) * S * D, r = static_cast<size_t>(BH) * tf32_padded_seq(S);
  for (int br = 0; br < n_br; ++br) {
    w.qh[br] = take(x);
    w.ql[br] = take(x);
    w.kh[br] = take(x);
    w.kl[br] = take(x);
    w.rq[br] = take(r);
    w.tq[br] = take(r);
    w.rk[br] = take(r);
  }
  w.vth = take(r * D);
  w.vtl = take(r * D);
  w.bytes = off;
  return w;
}

// Tensor maps, all fp32 with 128-byte swizzle and 32-element (128 B) boxes:
// q high / low copies as 3-D {D, S, BH} with 64-row boxes, k copies with
// key-tile-row boxes (tf32_key_tile), V^T copies as {S_pad, D, BH} with D-row
// boxes.
struct Tf32FwdParams {
  CUtensorMap tm_qh[2];
  CUtensorMap tm_ql[2];
  CUtensorMap tm_kh[2];
  CUtensorMap tm_kl[2];
  CUtensorMap tm_vh;
  CUtensorMap tm_vl;
  const float* rq[2];
  const float* tq[2];
  const float* rk[2];
  float* out;  // [BH][S][D] fp32
  int* status;
  int S;
  int S_pad;
  int BH;
  int n_qt;       // 128-row query tiles
  int n_kt_all;   // key tiles (S_pad / tf32_key_tile)
  int causal_skip;
  int n_br;       // 1 rectified, 2 differential
  float relu_power;
  float lam;      // clamped lambda (second branch weight -lam)
  LamSpec lam_dev;  // per-(batch, head) lambda on the device (ptr null: lam)
  unsigned long long timeout_ns;
  int inject;     // test hook: bit 0 = producer never loads Q (forces a timeout)
};

int tf32_key_tile(int head_dim);  // keys per tile: 64 at head_dim 64, 32 at 128
cudaError_t launch_tf32_split(const float* const q[2], const float* const k[2], const float* v,
                              const Tf32Workspace& ws, int n_br, int BH, int S, int D, float beta, int normalize,
                              cudaStream_t stream);
cudaError_t launch_tf32_fwd(const Tf32FwdParams& p, int head_dim, int pow_mode, cudaStream_t stream);

// CUDA-core fp32 backward of one rectified branch (dq, dk through F.normalize
// when normalize; dv written or accumulated).  Inputs bf16 or fp32.
struct BwdParams {
  const void* q;
  const void* k;
  const void* v;
  const void* dout;
  float* dq;
  float* dk;
  float* dv;
  int S;
  int BH;
  float beta;
  float relu_power;
  float dout_scale;
  int normalize;
  int accumulate_dv;
};

cudaError_t launch_rect_bwd(const BwdParams& p, int head_dim, bool in_bf16, cudaStream_t stream);

// Tensor-core backward of one rectified branch (bf16 inputs, head_dim 64/128).
// Tables (workspace): the key table of k (as for the forward) and a query
// table qc[bh][i] = {rq_i, tq_i} (rq = 1/max(||q_i||,1e-12) or 1, tq = tau_i *
// ||q_i|| or tau_i; rows past S: {0, +huge}).
struct TcBwdParams {
  CUtensorMap tm_q;
  CUtensorMap tm_k;
  CUtensorMap tm_v;
  CUtensorMap tm_do;
  CUtensorMap tm_dq;  // fp32 gradients, contiguous (BH, S, D) as 3-D {D, S, BH}: box {32, 128, 1}, 128-B swizzle
  CUtensorMap tm_dk;
  CUtensorMap tm_dv;
  const float* rk;   // key table of k
  const float2* qc;  // query table
  float* dq;
  float* dk;
  float* dv;
  int* status;
  int S;
  int S_pad;
  int BH;
  int n_tiles;
  int causal_skip;  // beta >= 0
  int accumulate_dv;
  float beta;
  float relu_power;
  float scale;      // dout_scale
  unsigned long long timeout_ns;
};

// (S_pad per bh) query table floats: 2 per row
inline size_t query_table_floats(int64_t BH, int64_t S) { return static_cast<size_t>(BH) * padded_seq(S) * 2; }
cudaError_t launch_query_table(const void* q, float2* qc, int BH, int S, int S_pad, int D, float beta, int normalize,
                               cudaStream_t stream);
cudaError_t launch_tc_bwd(const TcBwdParams& p, int head_dim, bool normalize, int pow_mode, cudaStream_t stream);

// Key table of x: rk[bh][j] = 1 / max(||x[bh][j]||_2, 1e-12) for j < S, 0 for
// S <= j < S_pad, followed by rkmax[bh][g] = max of rk over keys [16 g, 16 g + 16).
inline size_t key_table_floats(int64_t BH, int64_t S) { return static_cast<size_t>(BH) * padded_seq(S) / 16 * 17; }
// dtype: 1 = bf16, 2 = fp16 (the TDA_BF16 / TDA_F16 codes).
cudaError_t launch_key_norms(const void* x, int dtype, float* rk, int BH, int S, int S_pad, int D,
                             cudaStream_t stream);
// Both key tensors of the differential form in one launch (x2 = nullptr: x1 only).
cudaError_t launch_key_norms_pair(const void* x1, const void* x2, int dtype, float* rk1, float* rk2, int BH, int S,
                                  int S_pad, int D, cudaStream_t stream);
// Same for n (1 or 2) strided (batch, head, seq, dim) views (strides in
// elements, last dimension contiguous); bh = b * heads + h.
cudaError_t launch_key_norms_strided(int n, const void* const x[2], float* const rk[2], int dtype, int BH, int heads,
                                     int S, int S_pad, int D, const int64_t stride_b[2], const int64_t stride_h[2],
                                     const int64_t stride_s[2], cudaStream_t stream);

// Sets the thread-local message returned by tda_last_error().
void set_last_error(const char* msg);

}  // namespace tda
