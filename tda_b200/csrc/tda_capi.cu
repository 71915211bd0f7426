// extern "C" entry points declared in include/tda_b200.h: argument checks,
// TMA descriptor construction and stream-ordered launches.  No allocation, no
// host synchronisation.
#include <cudaTypedefs.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cmath>
#include <cstring>
#include <mutex>
#include <string>

#include "../../include/tda_b200.h"
#include "tda_internal.h"

namespace {

thread_local std::string g_last_error;
std::atomic<int> g_inject{0};
std::atomic<unsigned long long> g_timeout_ns{1000000000ull};
std::atomic<unsigned long long*> g_stats{nullptr};

int fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int cuda_fail(cudaError_t e, const char* what) {
  return fail(TDA_ERR_CUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// (BH, S, D) bf16 array viewed as 3-D {D, S, BH}; box {64, 128, 1}; 128-B swizzle.
int make_map(CUtensorMap* m, const void* base, int64_t BH, int64_t S, int64_t D) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * 2), static_cast<cuuint64_t>(S * D * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(tda::kTile), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return TDA_OK;
}

// A contiguous (BH, S, D) bf16 or f32 output array (forward output, fp32
// gradients) as 3-D {D, S, BH}; box {128 bytes of elements, 128 rows, 1},
// 128-B swizzle (the layout the epilogues stage each 128-row tile in before
// its TMA store).
int make_out_map(CUtensorMap* m, void* out, bool f32, int64_t BH, int64_t S, int64_t D, bool f16 = false) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  const int64_t es = f32 ? 4 : 2;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(BH)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(D * es), static_cast<cuuint64_t>(S * D * es)};
  cuuint32_t box[3] = {static_cast<cuuint32_t>(128 / es), static_cast<cuuint32_t>(tda::kTile), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m,
                   f32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                       : (f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16),
                   3, out, dims, strides,
                   box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                   CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return TDA_OK;
}

// A (batch, head, seq, dim) bf16 view: element strides of the first three
// dimensions, the last one contiguous.
struct View {
  const void* p;
  int64_t sb, sh, ss;
};

View contiguous_view(const void* p, int64_t BH, int64_t S, int64_t D) { return View{p, BH * S * D, S * D, D}; }

// View viewed as 4-D {D, S, heads, batches}; box {64, box_rows, 1, 1}; 128-B
// swizzle; 2-byte elements, bf16 or fp16.
int make_map4(CUtensorMap* m, const View& x, int64_t batches, int64_t heads, int64_t S, int64_t D,
              bool f16 = false, int box_rows = tda::kTile) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(D), static_cast<cuuint64_t>(S), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(batches)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(x.ss * 2), static_cast<cuuint64_t>(x.sh * 2),
                           static_cast<cuuint64_t>(x.sb * 2)};
  cuuint32_t box[4] = {64, static_cast<cuuint32_t>(box_rows), 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(m, f16 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4,
                   const_cast<void*>(x.p), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return TDA_OK;
}

// A contiguous fp32 array viewed as 3-D {d0, d1, d2}; box {32, box_rows, 1} (128 B x box_rows); 128-B swizzle.
int make_map_f32(CUtensorMap* m, const void* base, int64_t d0, int64_t d1, int64_t d2, int box_rows) {
  auto enc = tensor_map_encoder();
  if (!enc) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(d0 * 4), static_cast<cuuint64_t>(d0 * d1 * 4)};
  cuuint32_t box[3] = {32, static_cast<cuuint32_t>(box_rows), 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(TDA_ERR_CUDA, "cuTensorMapEncodeTiled failed (CUresult %d)", static_cast<int>(r));
  return TDA_OK;
}

int check_common(int64_t BH, int64_t S, int64_t D, int* status) {
  if (BH < 1 || S < 1) return fail(TDA_ERR_INVALID, "batch_heads and seq_len must be >= 1 (got %lld, %lld)",
                                   static_cast<long long>(BH), static_cast<long long>(S));
  if (D < 16 || D > 256 || (D & (D - 1)) != 0)
    return fail(TDA_ERR_INVALID, "head_dim must be a power of two in [16, 256] (got %lld)", static_cast<long long>(D));
  if (S > (1ll << 30)) return fail(TDA_ERR_INVALID, "seq_len too large (%lld)", static_cast<long long>(S));
  const int64_t tiles = BH * ((S + 63) / 64);
  if (tiles > 0x7fffffffll) return fail(TDA_ERR_INVALID, "batch_heads * seq_len tiles exceed the grid limit");
  if (!status) return fail(TDA_ERR_INVALID, "status must point to a device int32");
  return TDA_OK;
}

bool tc_supported(int dtype, int64_t D) { return (dtype == TDA_BF16 || dtype == TDA_F16) && (D == 64 || D == 128); }

// fp16 operands: P = relu(z)^p is split into fp16 hi + lo after a power-of-two
// scale, so it needs a bound.  With normalize, z = cos - tau <= 1 + max(0, -tau_max),
// tau_max = |beta| sqrt(2 ln S / D), and |P| <= z_max^p (the differential form's
// P1 - lambda P2 too).  Returns the scale 2^e (e <= 14) that keeps |P| * scale
// <= 16384, or 0 when fp16 cannot carry this configuration (no normalize,
// p <= 0, or a bound above 16384).
float fp16_p_scale(int normalize, float beta, float p, int64_t S, int64_t D) {
  if (!normalize || !(p > 0.0f)) return 0.0f;
  const double tau_max = beta < 0.0f ? -static_cast<double>(beta) * std::sqrt(2.0 * std::log(static_cast<double>(S)) /
                                                                            static_cast<double>(D))
                                     : 0.0;
  const double pmax = std::pow(1.0 + tau_max, static_cast<double>(p));
  if (!(pmax <= 16384.0)) return 0.0f;
  int e = static_cast<int>(std::floor(std::log2(16384.0 / pmax)));
  if (e > 14) e = 14;
  return std::ldexp(1.0f, e);
}

// No device lambda: every (batch, head) uses the host scalar.
constexpr tda::LamSpec kNoLam{nullptr, 0, 0, 1};

int run_tc(const View& q1, const View& q2, const View& k1, const View& k2, const View& v, void* out, int out_dtype,
           int64_t BH, int64_t heads, int64_t S, int64_t D, float beta, float lam, float p, int normalize,
           const float* rk1, const float* rk2, int* status, void* stream, bool differential,
           const tda::LamSpec& lam_dev = kNoLam, int in_dtype = TDA_BF16) {
  if (int e = check_common(BH, S, D, status)) return e;
  if (heads < 1 || BH % heads != 0) return fail(TDA_ERR_INVALID, "heads must divide batch * heads");
  if (!(D == 64 || D == 128)) return fail(TDA_ERR_UNSUPPORTED, "tensor-core path needs head_dim 64 or 128");
  const bool f16 = in_dtype == TDA_F16;
  if (out_dtype != in_dtype && out_dtype != TDA_F32)
    return fail(TDA_ERR_INVALID, "out_dtype must be the input dtype or TDA_F32");
  float p_scale = 1.0f;
  if (f16 && (p_scale = fp16_p_scale(normalize, beta, p, S, D)) == 0.0f)
    return fail(TDA_ERR_UNSUPPORTED,
                "fp16 inputs run on the tensor cores only with normalize and a bounded ReLU power "
                "(normalize = %d, beta = %g, relu_power = %g); widen them to fp32",
                normalize, static_cast<double>(beta), static_cast<double>(p));
  const View* ins[5] = {&q1, &k1, &v, differential ? &q2 : &q1, differential ? &k2 : &k1};
  for (const View* x : ins) {
    if (!x->p || !aligned16(x->p)) return fail(TDA_ERR_INVALID, "inputs must be non-NULL and 16-byte aligned");
    if (x->sb <= 0 || x->sh <= 0 || x->ss <= 0 || (x->sb | x->sh | x->ss) % 8 != 0)
      return fail(TDA_ERR_INVALID, "input strides must be positive multiples of 8 elements (16 bytes)");
  }
  if (!out || !aligned16(out)) return fail(TDA_ERR_INVALID, "out must be non-NULL and 16-byte aligned");
  if (normalize && (!rk1 || (differential && !rk2) || !aligned16(rk1) || (differential && !aligned16(rk2))))
    return fail(TDA_ERR_INVALID, "normalize needs 16-byte aligned key inverse norms");
  if (!(p == p)) return fail(TDA_ERR_INVALID, "relu_power is NaN");

  tda::TcFwdParams prm;
  std::memset(&prm, 0, sizeof(prm));
  int e;
  const int64_t batches = BH / heads;
  if ((e = make_map4(&prm.tm_q1, q1, batches, heads, S, D, f16))) return e;
  if ((e = make_map4(&prm.tm_k1, k1, batches, heads, S, D, f16))) return e;
  if ((e = make_map4(&prm.tm_v, v, batches, heads, S, D, f16))) return e;
  if (differential) {
    if ((e = make_map4(&prm.tm_q2, q2, batches, heads, S, D, f16))) return e;
    if ((e = make_map4(&prm.tm_k2, k2, batches, heads, S, D, f16))) return e;
  }
  if (tda::tc_fwd_uses_pair(static_cast<int>(D))) {  // the CTA-pair kernel loads half key tiles (64 rows)
    if ((e = make_map4(&prm.tm_k1h, k1, batches, heads, S, D, f16, tda::kTile / 2))) return e;
    if (differential && (e = make_map4(&prm.tm_k2h, k2, batches, heads, S, D, f16, tda::kTile / 2))) return e;
  }
  if ((e = make_out_map(&prm.tm_out, out, out_dtype == TDA_F32, BH, S, D, f16))) return e;
  prm.rk1 = rk1;
  prm.rk2 = rk2;
  prm.out = out;
  prm.status = status;
  prm.S = static_cast<int>(S);
  prm.S_pad = static_cast<int>(tda::padded_seq(S));
  prm.BH = static_cast<int>(BH);
  prm.heads = static_cast<int>(heads);
  prm.n_qtiles = static_cast<int>((S + tda::kTile - 1) / tda::kTile);
  prm.out_f32 = out_dtype == TDA_F32;
  prm.causal_skip = beta >= 0.0f ? 1 : 0;
  prm.beta = beta;
  prm.relu_power = p;
  prm.lam = lam;
  prm.lam_root = p == 2.0f ? std::sqrt(lam) : (p == 3.0f ? std::cbrt(lam) : lam);
  prm.lam_dev = lam_dev;
  prm.tau_scale = 2.0f / static_cast<float>(D);
  prm.p_scale = p_scale;
  prm.o_unscale = 1.0f / p_scale;
  prm.timeout_ns = g_timeout_ns.load();
  prm.inject = g_inject.load();
  prm.stats = g_stats.load();
  cudaError_t ce = tda::launch_tc_fwd(prm, static_cast<int>(D), differential, normalize != 0, tda::pow_mode_of(p),
                                      f16, static_cast<cudaStream_t>(stream));
  if (ce == cudaErrorLaunchOutOfResources && !g_last_error.empty() &&
      g_last_error.rfind("tensor-core kernel does not fit", 0) == 0)
    return TDA_ERR_CUDA;
  if (ce != cudaSuccess) return cuda_fail(ce, "tensor-core forward launch");
  return TDA_OK;
}

int run_simt(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out, int64_t BH,
             int64_t S, int64_t D, float beta, float lam, float p, int normalize, int* status, void* stream,
             bool differential, const tda::LamSpec& lam_dev = kNoLam) {
  if (int e = check_common(BH, S, D, status)) return e;
  const void* ins[5] = {q1, k1, v, differential ? q2 : q1, differential ? k2 : k1};
  for (const void* x : ins)
    if (!x || !aligned16(x)) return fail(TDA_ERR_INVALID, "inputs must be non-NULL and 16-byte aligned");
  if (!out || !aligned16(out)) return fail(TDA_ERR_INVALID, "out must be non-NULL and 16-byte aligned");
  tda::SimtFwdParams prm;
  prm.q1 = static_cast<const float*>(q1);
  prm.k1 = static_cast<const float*>(k1);
  prm.q2 = static_cast<const float*>(differential ? q2 : q1);
  prm.k2 = static_cast<const float*>(differential ? k2 : k1);
  prm.v = static_cast<const float*>(v);
  prm.out = static_cast<float*>(out);
  prm.S = static_cast<int>(S);
  prm.BH = static_cast<int>(BH);
  prm.beta = beta;
  prm.relu_power = p;
  prm.lam = lam;
  prm.lam_dev = lam_dev;
  prm.normalize = normalize != 0;
  prm.differential = differential;
  cudaError_t ce = tda::launch_simt_fwd(prm, static_cast<int>(D), static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) return cuda_fail(ce, "fp32 forward launch");
  return TDA_OK;
}

// fp32 inputs at head_dim 64 / 128 on the tensor cores (three TF32 products
// per fp32 product): TF32 split pre-pass into the workspace, then the forward.
bool tf32_supported(int64_t D) { return D == 64 || D == 128; }

size_t tf32_bytes(int64_t BH, int64_t S, int64_t D, bool differential) {
  return tda::tf32_carve(nullptr, BH, S, D, differential ? 2 : 1).bytes;
}

int run_tf32(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out, int64_t BH,
             int64_t S, int64_t D, float beta, float lam, float p, int normalize, void* workspace, int* status,
             void* stream, bool differential, const tda::LamSpec& lam_dev = kNoLam) {
  if (int e = check_common(BH, S, D, status)) return e;
  const void* ins[5] = {q1, k1, v, differential ? q2 : q1, differential ? k2 : k1};
  for (const void* x : ins)
    if (!x || !aligned16(x)) return fail(TDA_ERR_INVALID, "inputs must be non-NULL and 16-byte aligned");
  if (!out || !aligned16(out)) return fail(TDA_ERR_INVALID, "out must be non-NULL and 16-byte aligned");
  if (!workspace || !aligned16(workspace)) return fail(TDA_ERR_WORKSPACE, "workspace must be 16-byte aligned");
  const int n_br = differential ? 2 : 1;
  const tda::Tf32Workspace w = tda::tf32_carve(workspace, BH, S, D, n_br);
  const float* qs[2] = {static_cast<const float*>(q1), static_cast<const float*>(differential ? q2 : q1)};
  const float* ks[2] = {static_cast<const float*>(k1), static_cast<const float*>(differential ? k2 : k1)};
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t ce = tda::launch_tf32_split(qs, ks, static_cast<const float*>(v), w, n_br, static_cast<int>(BH),
                                          static_cast<int>(S), static_cast<int>(D), beta, normalize, st);
  if (ce != cudaSuccess) return cuda_fail(ce, "fp32 split pre-pass launch");
  const int64_t S_pad = tda::tf32_padded_seq(S);
  const int kt = tda::tf32_key_tile(static_cast<int>(D));
  tda::Tf32FwdParams prm;
  memset(&prm, 0, sizeof(prm));
  for (int br = 0; br < 2; ++br) {
    const int b = br < n_br ? br : 0;
    int e;
    if ((e = make_map_f32(&prm.tm_qh[br], w.qh[b], D, S, BH, 64))) return e;
    if ((e = make_map_f32(&prm.tm_ql[br], w.ql[b], D, S, BH, 64))) return e;
    if ((e = make_map_f32(&prm.tm_kh[br], w.kh[b], D, S, BH, kt))) return e;
    if ((e = make_map_f32(&prm.tm_kl[br], w.kl[b], D, S, BH, kt))) return e;
    prm.rq[br] = w.rq[b];
    prm.tq[br] = w.tq[b];
    prm.rk[br] = w.rk[b];
  }
  if (int e = make_map_f32(&prm.tm_vh, w.vth, S_pad, D, BH, static_cast<int>(D))) return e;
  if (int e = make_map_f32(&prm.tm_vl, w.vtl, S_pad, D, BH, static_cast<int>(D))) return e;
  prm.out = static_cast<float*>(out);
  prm.status = status;
  prm.S = static_cast<int>(S);
  prm.S_pad = static_cast<int>(S_pad);
  prm.BH = static_cast<int>(BH);
  prm.n_qt = static_cast<int>((S + 127) / 128);
  prm.n_kt_all = static_cast<int>(S_pad / kt);
  prm.causal_skip = beta >= 0.0f;
  prm.n_br = n_br;
  prm.relu_power = p;
  prm.lam = lam;
  prm.lam_dev = lam_dev;
  prm.timeout_ns = g_timeout_ns.load();
  prm.inject = g_inject.load();
  ce = tda::launch_tf32_fwd(prm, static_cast<int>(D), tda::pow_mode_of(p), st);
  if (ce != cudaSuccess) return cuda_fail(ce, "fp32 tensor-core forward launch");
  return TDA_OK;
}

float clamp01(float x) { return x < 0.0f ? 0.0f : (x > 1.0f ? 1.0f : x); }

size_t rk_bytes(int64_t BH, int64_t S) { return tda::key_table_floats(BH, S) * sizeof(float); }

}  // namespace

void tda::set_last_error(const char* msg) { g_last_error = msg ? msg : ""; }

extern "C" {

int tda_version(void) { return 101; }

const char* tda_last_error(void) { return g_last_error.c_str(); }

int tda_debug_stats(void* counters) {
  g_stats.store(static_cast<unsigned long long*>(counters));
  return TDA_OK;
}

int tda_debug_set(int inject, uint64_t wait_timeout_ns) {
  g_inject.store(inject);
  g_timeout_ns.store(wait_timeout_ns ? wait_timeout_ns : 1000000000ull);
  return TDA_OK;
}

size_t tda_workspace_size(int differential, int dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim,
                          int normalize) {
  if (dtype == TDA_F32 && tf32_supported(head_dim) && batch_heads >= 1 && seq_len >= 1)
    return tf32_bytes(batch_heads, seq_len, head_dim, differential != 0);
  if (!normalize || !tc_supported(dtype, head_dim) || batch_heads < 1 || seq_len < 1) return 0;
  const size_t one = (rk_bytes(batch_heads, seq_len) + 255) / 256 * 256;
  return differential ? 2 * one : one;
}

int tda_key_inv_norms_pair(const void* k1, const void* k2, int dtype, int64_t batch_heads, int64_t seq_len,
                           int64_t head_dim, float* rk1, float* rk2, void* stream) {
  if (batch_heads < 1 || seq_len < 1) return fail(TDA_ERR_INVALID, "batch_heads and seq_len must be >= 1");
  if (batch_heads * tda::padded_seq(seq_len) > 0x7fffffffll) return fail(TDA_ERR_INVALID, "key table too large");
  if (!tc_supported(dtype, head_dim))
    return fail(TDA_ERR_UNSUPPORTED, "key norms need bf16 or fp16 with head_dim 64 or 128");
  if (!k1 || !rk1 || !aligned16(k1) || !aligned16(rk1) || (k2 && (!rk2 || !aligned16(k2) || !aligned16(rk2))))
    return fail(TDA_ERR_INVALID, "k / rk must be 16-byte aligned");
  cudaError_t ce = tda::launch_key_norms_pair(k1, k2, dtype, rk1, k2 ? rk2 : nullptr, static_cast<int>(batch_heads),
                                              static_cast<int>(seq_len), static_cast<int>(tda::padded_seq(seq_len)),
                                              static_cast<int>(head_dim), static_cast<cudaStream_t>(stream));
  if (ce != cudaSuccess) return cuda_fail(ce, "key norm launch");
  return TDA_OK;
}

int tda_key_inv_norms(const void* k, int dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float* rk,
                      void* stream) {
  return tda_key_inv_norms_pair(k, nullptr, dtype, batch_heads, seq_len, head_dim, rk, nullptr, stream);
}

int tda_rect_fwd_tc(const void* q, const void* k, const void* v, void* out, int out_dtype, int64_t batch_heads,
                    int64_t seq_len, int64_t head_dim, float beta, float relu_power, int normalize,
                    const float* rk, int* status, void* stream) {
  auto cv = [&](const void* x) { return contiguous_view(x, batch_heads, seq_len, head_dim); };
  return run_tc(cv(q), cv(nullptr), cv(k), cv(nullptr), cv(v), out, out_dtype, batch_heads, batch_heads, seq_len,
                head_dim, beta, 0.0f, relu_power, normalize, rk, nullptr, status, stream, false);
}

int tda_diff_fwd_tc(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out,
                    int out_dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta,
                    float lambda_param, float relu_power, int normalize, const float* rk1, const float* rk2,
                    int* status, void* stream) {
  auto cv = [&](const void* x) { return contiguous_view(x, batch_heads, seq_len, head_dim); };
  return run_tc(cv(q1), cv(q2), cv(k1), cv(k2), cv(v), out, out_dtype, batch_heads, batch_heads, seq_len, head_dim,
                beta, clamp01(lambda_param), relu_power, normalize, rk1, rk2, status, stream, true);
}

namespace {
// Contiguous bf16 / fp16 differential form on the tensor cores: the key tables
// of k1 and k2 in one launch, then the fused kernel.
int diff_tc_path(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out, int dtype,
                 int out_dtype, int64_t BH, int64_t S, int64_t D, float beta, float lam, float p, int normalize,
                 void* workspace, size_t workspace_bytes, int* status, void* stream, const tda::LamSpec& lam_dev) {
  if (dtype != TDA_BF16 && dtype != TDA_F16) return fail(TDA_ERR_INVALID, "dtype must be TDA_F32, TDA_BF16 or TDA_F16");
  if (!tc_supported(dtype, D))
    return fail(TDA_ERR_UNSUPPORTED, "bf16 / fp16 path supports head_dim 64 or 128 (got %lld)", static_cast<long long>(D));
  if (dtype == TDA_F16 && fp16_p_scale(normalize, beta, p, S, D) == 0.0f)
    return fail(TDA_ERR_UNSUPPORTED, "fp16 inputs run on the tensor cores only with normalize and a bounded ReLU "
                                     "power; widen them to fp32");
  float* rk1 = nullptr;
  float* rk2 = nullptr;
  if (normalize) {
    const size_t need = tda_workspace_size(1, dtype, BH, S, D, normalize);
    if (!workspace || workspace_bytes < need) return fail(TDA_ERR_WORKSPACE, "workspace of %zu bytes required", need);
    rk1 = static_cast<float*>(workspace);
    rk2 = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + need / 2);
    if (int e = tda_key_inv_norms_pair(k1, k2, dtype, BH, S, D, rk1, rk2, stream)) return e;
  }
  auto cv = [&](const void* x) { return contiguous_view(x, BH, S, D); };
  return run_tc(cv(q1), cv(q2), cv(k1), cv(k2), cv(v), out, out_dtype, BH, BH, S, D, beta, lam, p, normalize, rk1,
                rk2, status, stream, true, lam_dev, dtype);
}

// Strided entry points: key tables of the strided keys, then the fused kernel.
int run_strided(const View* views, int n, void* out, int out_dtype, int64_t batch, int64_t heads, int64_t S,
                int64_t D, float beta, float lam, float p, int normalize, void* workspace, size_t workspace_bytes,
                int* status, void* stream, const tda::LamSpec& lam_dev = kNoLam) {
  const bool diff = n == 5;
  if (batch < 1 || heads < 1) return fail(TDA_ERR_INVALID, "batch and heads must be >= 1");
  if (!(D == 64 || D == 128))
    return fail(TDA_ERR_UNSUPPORTED, "strided inputs run on the tensor-core path: head_dim 64 or 128 (got %lld)",
                static_cast<long long>(D));
  const int64_t BH = batch * heads;
  if (int e = check_common(BH, S, D, status)) return e;
  for (int i = 0; i < n; ++i)
    if (views[i].sb <= 0 || views[i].sh <= 0 || views[i].ss <= 0 || (views[i].sb | views[i].sh | views[i].ss) % 8)
      return fail(TDA_ERR_INVALID, "input strides must be positive multiples of 8 elements (16 bytes)");
  // views: rect q, k, v; differential q1, q2, k1, k2, v
  const View& q1 = views[0];
  const View& q2 = diff ? views[1] : views[0];
  const View& k1 = diff ? views[2] : views[1];
  const View& k2 = diff ? views[3] : views[1];
  const View& v = diff ? views[4] : views[2];
  float* rk1 = nullptr;
  float* rk2 = nullptr;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (normalize) {
    const size_t need = tda_workspace_size(diff ? 1 : 0, TDA_BF16, BH, S, D, normalize);
    if (!workspace || workspace_bytes < need) return fail(TDA_ERR_WORKSPACE, "workspace of %zu bytes required", need);
    if (!aligned16(k1.p) || !aligned16(k2.p)) return fail(TDA_ERR_INVALID, "inputs must be 16-byte aligned");
    rk1 = static_cast<float*>(workspace);
    rk2 = diff ? reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + need / 2) : nullptr;
    const int S_pad = static_cast<int>(tda::padded_seq(S));
    const void* kx[2] = {k1.p, k2.p};
    float* const kt[2] = {rk1, rk2};
    const int64_t sb[2] = {k1.sb, k2.sb}, sh[2] = {k1.sh, k2.sh}, ss[2] = {k1.ss, k2.ss};
    cudaError_t ce = tda::launch_key_norms_strided(diff ? 2 : 1, kx, kt, TDA_BF16, static_cast<int>(BH),
                                                   static_cast<int>(heads), static_cast<int>(S), S_pad,
                                                   static_cast<int>(D), sb, sh, ss, st);
    if (ce != cudaSuccess) return cuda_fail(ce, "key table launch");
  }
  return run_tc(q1, q2, k1, k2, v, out, out_dtype, BH, heads, S, D, beta, lam, p, normalize, rk1, rk2, status, stream,
                diff, lam_dev);
}
}  // namespace

int tda_rect_fwd_strided(const void* q, const void* k, const void* v, const int64_t* strides, void* out,
                         int out_dtype, int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, float beta,
                         float relu_power, int normalize, void* workspace, size_t workspace_bytes, int* status,
                         void* stream) {
  if (!strides) return fail(TDA_ERR_INVALID, "strides must point to 9 int64 values");
  const View views[3] = {{q, strides[0], strides[1], strides[2]},
                         {k, strides[3], strides[4], strides[5]},
                         {v, strides[6], strides[7], strides[8]}};
  return run_strided(views, 3, out, out_dtype, batch, heads, seq_len, head_dim, beta, 0.0f, relu_power, normalize,
                     workspace, workspace_bytes, status, stream);
}

int tda_diff_fwd_strided(const void* q1, const void* q2, const void* k1, const void* k2, const void* v,
                         const int64_t* strides, void* out, int out_dtype, int64_t batch, int64_t heads,
                         int64_t seq_len, int64_t head_dim, float beta, float lambda_param, float relu_power,
                         int normalize, void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (!strides) return fail(TDA_ERR_INVALID, "strides must point to 15 int64 values");
  const View views[5] = {{q1, strides[0], strides[1], strides[2]},
                         {q2, strides[3], strides[4], strides[5]},
                         {k1, strides[6], strides[7], strides[8]},
                         {k2, strides[9], strides[10], strides[11]},
                         {v, strides[12], strides[13], strides[14]}};
  return run_strided(views, 5, out, out_dtype, batch, heads, seq_len, head_dim, beta, clamp01(lambda_param),
                     relu_power, normalize, workspace, workspace_bytes, status, stream);
}

int tda_rect_fwd(const void* q, const void* k, const void* v, void* out, int dtype, int out_dtype,
                 int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta, float relu_power,
                 int normalize, void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (dtype == TDA_F32) {
    if (out_dtype != TDA_F32) return fail(TDA_ERR_INVALID, "fp32 inputs produce fp32 output");
    if (tf32_supported(head_dim) && workspace && batch_heads >= 1 && seq_len >= 1 &&
        workspace_bytes >= tf32_bytes(batch_heads, seq_len, head_dim, false))
      return run_tf32(q, nullptr, k, nullptr, v, out, batch_heads, seq_len, head_dim, beta, 0.0f, relu_power,
                      normalize, workspace, status, stream, false);
    return run_simt(q, nullptr, k, nullptr, v, out, batch_heads, seq_len, head_dim, beta, 0.0f, relu_power,
                    normalize, status, stream, false);
  }
  if (dtype != TDA_BF16 && dtype != TDA_F16) return fail(TDA_ERR_INVALID, "dtype must be TDA_F32, TDA_BF16 or TDA_F16");
  if (!tc_supported(dtype, head_dim))
    return fail(TDA_ERR_UNSUPPORTED, "bf16 / fp16 path supports head_dim 64 or 128 (got %lld)",
                static_cast<long long>(head_dim));
  if (dtype == TDA_F16 && fp16_p_scale(normalize, beta, relu_power, seq_len, head_dim) == 0.0f)
    return fail(TDA_ERR_UNSUPPORTED, "fp16 inputs run on the tensor cores only with normalize and a bounded ReLU "
                                     "power; widen them to fp32");
  float* rk = nullptr;
  if (normalize) {
    const size_t need = tda_workspace_size(0, dtype, batch_heads, seq_len, head_dim, normalize);
    if (!workspace || workspace_bytes < need)
      return fail(TDA_ERR_WORKSPACE, "workspace of %zu bytes required", need);
    rk = static_cast<float*>(workspace);
    if (int e = tda_key_inv_norms(k, dtype, batch_heads, seq_len, head_dim, rk, stream)) return e;
  }
  auto cv = [&](const void* x) { return contiguous_view(x, batch_heads, seq_len, head_dim); };
  return run_tc(cv(q), cv(nullptr), cv(k), cv(nullptr), cv(v), out, out_dtype, batch_heads, batch_heads, seq_len,
                head_dim, beta, 0.0f, relu_power, normalize, rk, nullptr, status, stream, false, kNoLam, dtype);
}

int tda_diff_fwd(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out,
                 int dtype, int out_dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta,
                 float lambda_param, float relu_power, int normalize, void* workspace, size_t workspace_bytes,
                 int* status, void* stream) {
  if (dtype == TDA_F32) {
    if (out_dtype != TDA_F32) return fail(TDA_ERR_INVALID, "fp32 inputs produce fp32 output");
    if (tf32_supported(head_dim) && workspace && batch_heads >= 1 && seq_len >= 1 &&
        workspace_bytes >= tf32_bytes(batch_heads, seq_len, head_dim, true))
      return run_tf32(q1, q2, k1, k2, v, out, batch_heads, seq_len, head_dim, beta, clamp01(lambda_param),
                      relu_power, normalize, workspace, status, stream, true);
    return run_simt(q1, q2, k1, k2, v, out, batch_heads, seq_len, head_dim, beta, clamp01(lambda_param),
                    relu_power, normalize, status, stream, true);
  }
  return diff_tc_path(q1, q2, k1, k2, v, out, dtype, out_dtype, batch_heads, seq_len, head_dim, beta,
                      clamp01(lambda_param), relu_power, normalize, workspace, workspace_bytes, status, stream, kNoLam);
}

size_t tda_bwd_workspace_size(int dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, int normalize) {
  if (dtype != TDA_BF16 || (head_dim != 64 && head_dim != 128) || batch_heads < 1 || seq_len < 1) return 0;
  const size_t keys = normalize ? (tda::key_table_floats(batch_heads, seq_len) * 4 + 255) / 256 * 256 : 0;
  return keys + (tda::query_table_floats(batch_heads, seq_len) * 4 + 255) / 256 * 256;
}

int tda_rect_bwd(const void* q, const void* k, const void* v, const void* dout, int dtype, float* dq, float* dk,
                 float* dv, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta, float relu_power,
                 int normalize, float dout_scale, int accumulate_dv, void* workspace, size_t workspace_bytes,
                 int* status, void* stream) {
  if (batch_heads < 1 || seq_len < 1)
    return fail(TDA_ERR_INVALID, "batch_heads and seq_len must be >= 1 (got %lld, %lld)",
                static_cast<long long>(batch_heads), static_cast<long long>(seq_len));
  if (dtype != TDA_F32 && dtype != TDA_BF16) return fail(TDA_ERR_INVALID, "dtype must be TDA_F32 or TDA_BF16");
  if (head_dim != 16 && head_dim != 32 && head_dim != 64 && head_dim != 128 && head_dim != 256)
    return fail(TDA_ERR_UNSUPPORTED, "backward supports head_dim 16, 32, 64, 128 or 256 (got %lld)",
                static_cast<long long>(head_dim));
  if (seq_len > (1ll << 30)) return fail(TDA_ERR_INVALID, "seq_len too large (%lld)", static_cast<long long>(seq_len));
  if (batch_heads * ((seq_len + 63) / 64) > 0x7fffffffll)
    return fail(TDA_ERR_INVALID, "batch_heads * seq_len tiles exceed the grid limit");
  const void* ptrs[7] = {q, k, v, dout, dq, dk, dv};
  for (const void* ptr : ptrs)
    if (!ptr || !aligned16(ptr)) return fail(TDA_ERR_INVALID, "q, k, v, dout, dq, dk, dv must be 16-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (dtype == TDA_BF16 && (head_dim == 64 || head_dim == 128)) {
    // tensor-core path: key table (normalize) and query table in the workspace
    if (!status) return fail(TDA_ERR_INVALID, "status must point to a device int32");
    const size_t need = tda_bwd_workspace_size(dtype, batch_heads, seq_len, head_dim, normalize);
    if (!workspace || workspace_bytes < need)
      return fail(TDA_ERR_WORKSPACE, "workspace of %zu bytes required", need);
    const int BH = static_cast<int>(batch_heads), S = static_cast<int>(seq_len), D = static_cast<int>(head_dim);
    const int S_pad = static_cast<int>(tda::padded_seq(seq_len));
    const size_t key_bytes = normalize ? (tda::key_table_floats(batch_heads, seq_len) * 4 + 255) / 256 * 256 : 0;
    float* rk = normalize ? static_cast<float*>(workspace) : nullptr;
    float2* qc = reinterpret_cast<float2*>(static_cast<uint8_t*>(workspace) + key_bytes);
    tda::TcBwdParams prm{};
    int e;
    if ((e = make_map(&prm.tm_q, q, batch_heads, seq_len, head_dim))) return e;
    if ((e = make_map(&prm.tm_k, k, batch_heads, seq_len, head_dim))) return e;
    if ((e = make_map(&prm.tm_v, v, batch_heads, seq_len, head_dim))) return e;
    if ((e = make_map(&prm.tm_do, dout, batch_heads, seq_len, head_dim))) return e;
    if ((e = make_out_map(&prm.tm_dq, dq, true, batch_heads, seq_len, head_dim))) return e;
    if ((e = make_out_map(&prm.tm_dk, dk, true, batch_heads, seq_len, head_dim))) return e;
    if ((e = make_out_map(&prm.tm_dv, dv, true, batch_heads, seq_len, head_dim))) return e;
    cudaError_t ce;
    if (normalize && (ce = tda::launch_key_norms(k, 1, rk, BH, S, S_pad, D, st)) != cudaSuccess)
      return cuda_fail(ce, "key table launch");
    if ((ce = tda::launch_query_table(q, qc, BH, S, S_pad, D, beta, normalize, st)) != cudaSuccess)
      return cuda_fail(ce, "query table launch");
    prm.rk = rk;
    prm.qc = qc;
    prm.dq = dq;
    prm.dk = dk;
    prm.dv = dv;
    prm.status = status;
    prm.S = S;
    prm.S_pad = S_pad;
    prm.BH = BH;
    prm.n_tiles = S_pad / tda::kTile;
    prm.causal_skip = beta >= 0.0f ? 1 : 0;
    prm.accumulate_dv = accumulate_dv ? 1 : 0;
    prm.beta = beta;
    prm.relu_power = relu_power;
    prm.scale = dout_scale;
    prm.timeout_ns = g_timeout_ns.load();
    ce = tda::launch_tc_bwd(prm, D, normalize != 0, tda::pow_mode_of(relu_power), st);
    if (ce != cudaSuccess) return cuda_fail(ce, "tensor-core backward launch");
    return TDA_OK;
  }
  tda::BwdParams prm{};
  prm.q = q;
  prm.k = k;
  prm.v = v;
  prm.dout = dout;
  prm.dq = dq;
  prm.dk = dk;
  prm.dv = dv;
  prm.S = static_cast<int>(seq_len);
  prm.BH = static_cast<int>(batch_heads);
  prm.beta = beta;
  prm.relu_power = relu_power;
  prm.dout_scale = dout_scale;
  prm.normalize = normalize ? 1 : 0;
  prm.accumulate_dv = accumulate_dv ? 1 : 0;
  cudaError_t ce = tda::launch_rect_bwd(prm, static_cast<int>(head_dim), dtype == TDA_BF16, st);
  if (ce != cudaSuccess) return cuda_fail(ce, "backward kernel launch");
  return TDA_OK;
}

int tda_diff_fwd_lambda(const void* q1, const void* q2, const void* k1, const void* k2, const void* v,
                        const int64_t* strides, void* out, int dtype, int out_dtype, int64_t batch, int64_t heads,
                        int64_t seq_len, int64_t head_dim, float beta, const float* lambda_param,
                        int64_t lambda_stride_batch, int64_t lambda_stride_head, float relu_power, int normalize,
                        void* workspace, size_t workspace_bytes, int* status, void* stream) {
  if (batch < 1 || heads < 1) return fail(TDA_ERR_INVALID, "batch and heads must be >= 1");
  if (!lambda_param || (reinterpret_cast<uintptr_t>(lambda_param) & 3u))
    return fail(TDA_ERR_INVALID, "lambda must be a non-NULL, 4-byte aligned device pointer to fp32 values");
  if (lambda_stride_batch < 0 || lambda_stride_head < 0)
    return fail(TDA_ERR_INVALID, "lambda strides must be >= 0");
  if (heads > 0x7fffffffll) return fail(TDA_ERR_INVALID, "heads too large");
  const tda::LamSpec lam{lambda_param, static_cast<long long>(lambda_stride_batch),
                         static_cast<long long>(lambda_stride_head), static_cast<int>(heads)};
  const int64_t BH = batch * heads;
  if (strides) {
    if (dtype != TDA_BF16) return fail(TDA_ERR_UNSUPPORTED, "strided inputs must be bf16");
    const View views[5] = {{q1, strides[0], strides[1], strides[2]},
                           {q2, strides[3], strides[4], strides[5]},
                           {k1, strides[6], strides[7], strides[8]},
                           {k2, strides[9], strides[10], strides[11]},
                           {v, strides[12], strides[13], strides[14]}};
    return run_strided(views, 5, out, out_dtype, batch, heads, seq_len, head_dim, beta, 0.0f, relu_power, normalize,
                       workspace, workspace_bytes, status, stream, lam);
  }
  if (dtype == TDA_F32) {
    if (out_dtype != TDA_F32) return fail(TDA_ERR_INVALID, "fp32 inputs produce fp32 output");
    if (tf32_supported(head_dim) && workspace && workspace_bytes >= tf32_bytes(BH, seq_len, head_dim, true))
      return run_tf32(q1, q2, k1, k2, v, out, BH, seq_len, head_dim, beta, 0.0f, relu_power, normalize, workspace,
                      status, stream, true, lam);
    return run_simt(q1, q2, k1, k2, v, out, BH, seq_len, head_dim, beta, 0.0f, relu_power, normalize, status, stream,
                    true, lam);
  }
  return diff_tc_path(q1, q2, k1, k2, v, out, dtype, out_dtype, BH, seq_len, head_dim, beta, 0.0f, relu_power,
                      normalize, workspace, workspace_bytes, status, stream, lam);
}

}  // extern "C"
