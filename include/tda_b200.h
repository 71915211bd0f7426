/*
 * tda_b200 -- C ABI of the B200-native Threshold (Differential) Attention
 * forward pass.
 *
 * These entry points are the drop-in boundary for the two public functions of
 * the reference implementation (snap-research/TDA, triton_threshold_attention.py):
 *
 *   threshold_rela_triton(q, k, v, beta, relu_power)            :472-486
 *   differential_threshold_rela_triton(q1, q2, k1, k2, v, beta,
 *                                      lambda_param, relu_power,
 *                                      normalize)                :489-519
 *
 * and of the launcher/kernel pair under them
 * (ThresholdRelaFunction.forward :335-403, _threshold_rela_fwd_kernel :19-115).
 *
 * Conventions (all entry points):
 *   - q, k, v, out are DEVICE pointers to contiguous (batch*heads, seq_len,
 *     head_dim) row-major arrays, i.e. (B, H, S, D) tensors flattened over
 *     (B, H).  All inputs share one shape (the reference asserts this, :348).
 *   - dtype is TDA_F32, TDA_BF16 or TDA_F16 for the inputs; out_dtype is the
 *     element type written to out (equal to dtype, or TDA_F32 to receive the
 *     fp32 accumulator of a bf16 / fp16 computation).
 *   - Causal, with the reference's mask-to-zero semantics (:79-80):
 *     out_i = sum_j relu(s_ij - tau_i)^p v_j, s_ij = q_i.k_j for j <= i and 0
 *     for j > i, tau_i = beta * sqrt(2 * log(i + 1) / head_dim).
 *   - stream is a cudaStream_t (NULL = legacy default stream).  Calls are
 *     asynchronous and stream-ordered; no host synchronisation happens.
 *   - status points to one device int32 that the kernels set to a nonzero
 *     code when a bounded internal wait gives up (the output is then
 *     invalid).  It is never cleared by the library.  A kernel reacts only to
 *     a change of the word during its own run, so a code left by an earlier
 *     call does not stop later calls.
 *   - Persistent kernel: at head_dim 128 with seq_len <= 4096 the rectified
 *     form runs a one-CTA-per-SM kernel that takes query tiles from a work
 *     counter in the library (1024 words, used round-robin).  At most 1024
 *     such launches of one process may be in flight at the same time, across
 *     all streams and CUDA graphs (a graph that captured a launch keeps its
 *     word); a 1025th concurrent launch would share a word with a running one.
 *   - workspace is device scratch of at least tda_workspace_size() bytes
 *     (may be NULL when that size is 0).  It is only used during the call.
 *   - Return value: TDA_OK, or a negative TDA_ERR_* code with a message from
 *     tda_last_error() (thread-local).
 *
 * Supported: dtype TDA_BF16 with head_dim 64 or 128 runs on the tcgen05
 * tensor cores; dtype TDA_F16 with head_dim 64 or 128 does too (fp16 operands)
 * when normalize != 0 and relu_power > 0 with P = relu(z)^p bounded by 16384
 * (always for beta >= 0; for beta < 0, (1 + |beta| sqrt(2 ln S / D))^p),
 * else it returns TDA_ERR_UNSUPPORTED; dtype TDA_F32 with head_dim 64 or 128, given the workspace
 * that tda_workspace_size reports, runs on the tcgen05 tensor cores too
 * (three TF32 products per fp32 product, fp32 accuracy); dtype TDA_F32 with
 * head_dim in {16, 32, 64, 128, 256} and no workspace runs the exact-fp32
 * CUDA-core kernel.  Other combinations return TDA_ERR_UNSUPPORTED (the
 * Python layer widens them to fp32 first).
 */
#ifndef TDA_B200_H_
#define TDA_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TDA_F32 0
#define TDA_BF16 1
#define TDA_F16 2

#define TDA_OK 0
#define TDA_ERR_INVALID (-1)     /* bad argument: shape, dtype, NULL or misaligned pointer */
#define TDA_ERR_UNSUPPORTED (-2) /* valid but not implemented for this dtype / head_dim */
#define TDA_ERR_CUDA (-3)        /* a CUDA runtime / driver call failed */
#define TDA_ERR_WORKSPACE (-4)   /* workspace missing or too small */

/* ABI version of this header (major * 100 + minor). */
int tda_version(void);

/* Thread-local description of the last error returned on this thread. */
const char* tda_last_error(void);

/* Device workspace bytes needed by tda_rect_fwd (differential = 0) or
 * tda_diff_fwd (differential = 1) for these sizes.  Replaces the fp32 upcast
 * copies the reference allocates per call (triton_threshold_attention.py:356-363):
 * for bf16 only per-key inverse norms (normalize) are kept; for fp32 at
 * head_dim 64 or 128 it holds the TF32 high / low copies of q, k and v^T and
 * per-row coefficients of the tensor-core path (about 2.5x the input bytes);
 * other fp32 head dims need none. */
size_t tda_workspace_size(int differential, int dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim,
                          int normalize);

/* Threshold rectified attention forward.
 * Replaces threshold_rela_triton (triton_threshold_attention.py:472-486) ->
 * ThresholdRelaFunction.forward (:335-403) -> _threshold_rela_fwd_kernel (:19-115).
 * normalize != 0 computes the reference applied to F.normalize(q), F.normalize(k)
 * (as each branch of :505-512 does); the reference's own entry point has no
 * such argument, normalize = 0 is its behaviour. */
int tda_rect_fwd(const void* q, const void* k, const void* v, void* out, int dtype, int out_dtype,
                 int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta, float relu_power,
                 int normalize, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Threshold differential attention forward, fused into one pass over the keys:
 * out = rect(q1, k1, v) - clamp(lambda, 0, 1) * rect(q2, k2, v).
 * Replaces differential_threshold_rela_triton (triton_threshold_attention.py:489-519),
 * which runs F.normalize x4 (:505-509), the forward kernel twice (:512-513) and
 * the clamp/combine (:516-517). */
int tda_diff_fwd(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out,
                 int dtype, int out_dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta,
                 float lambda_param, float relu_power, int normalize, void* workspace, size_t workspace_bytes,
                 int* status, void* stream);

/* tda_diff_fwd with lambda as a device tensor instead of a host scalar:
 * out[b][h] = rect(q1, k1, v)[b][h] - clamp(lambda[b * lambda_stride_batch +
 * h * lambda_stride_head], 0, 1) * rect(q2, k2, v)[b][h], computed in the same
 * single fused pass.  Replaces the reference's combine with a tensor lambda
 * that broadcasts over (batch, head) -- a scalar, a per-head or a
 * per-(batch, head) weight (triton_threshold_attention.py:516-517) -- without
 * a second kernel pass and without reading lambda on the host (no host
 * synchronisation).  lambda points to fp32 values on the device; a stride of 0
 * broadcasts that dimension (both 0: one scalar).  Inputs are (batch, heads,
 * seq_len, head_dim): contiguous when strides is NULL (any dtype / head_dim
 * tda_diff_fwd accepts, same workspace), or bf16 strided views at head_dim 64 /
 * 128 as for tda_diff_fwd_strided (15 element strides).  out is a contiguous
 * (batch * heads, seq_len, head_dim) array. */
int tda_diff_fwd_lambda(const void* q1, const void* q2, const void* k1, const void* k2, const void* v,
                        const int64_t* strides, void* out, int dtype, int out_dtype, int64_t batch, int64_t heads,
                        int64_t seq_len, int64_t head_dim, float beta, const float* lambda_param,
                        int64_t lambda_stride_batch, int64_t lambda_stride_head, float relu_power, int normalize,
                        void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Device workspace bytes needed by tda_rect_bwd for these sizes (0 on the
 * CUDA-core path): the key table of k (normalize) and a per-query table of
 * 1/||q_i|| and tau_i * ||q_i||. */
size_t tda_bwd_workspace_size(int dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, int normalize);

/* Backward of one threshold rectified attention branch, given the upstream
 * gradient dout of its output (same shape and dtype as q):
 *   dq, dk, dv = gradients w.r.t. q, k, v of rect(q, k, v) for the gradient
 *   dout_scale * dout, in fp32 (batch_heads, seq_len, head_dim) arrays.
 * Replaces ThresholdRelaFunction.backward (triton_threshold_attention.py:405-469)
 * and its kernels _threshold_rela_bwd_kernel_dq (:118-224) and
 * _threshold_rela_bwd_kernel_dkv (:227-324), including their handling of
 * masked entries: dQ / dK are not masked, so with beta < 0 keys after a query
 * row contribute as they do in the reference.  normalize != 0: q, k are
 * F.normalize'd inside and dq, dk are chained back through F.normalize (torch
 * autograd's part of :505-512).  accumulate_dv != 0 adds into dv (the
 * differential form calls this once per branch: dout_scale = 1, then
 * -clamp(lambda, 0, 1) with accumulate_dv = 1).
 * bf16 inputs with head_dim 64 / 128 run on the tensor cores (tcgen05, bf16
 * operands, P and dA as bf16 hi + lo, fp32 accumulation) and need the
 * workspace (tda_bwd_workspace_size) and a device status word; fp32 inputs and
 * head_dim 16 / 32 / 256 run exact fp32 on CUDA cores (workspace and status
 * unused).
 * dq, dk, dv must not alias the inputs. */
int tda_rect_bwd(const void* q, const void* k, const void* v, const void* dout, int dtype, float* dq, float* dk,
                 float* dv, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta, float relu_power,
                 int normalize, float dout_scale, int accumulate_dv, void* workspace, size_t workspace_bytes,
                 int* status, void* stream);

/* tda_rect_fwd / tda_diff_fwd for bf16 inputs given as strided
 * (batch, heads, seq_len, head_dim) views with a contiguous last dimension,
 * e.g. a (batch, seq_len, heads, head_dim) projection transposed to
 * (batch, heads, seq_len, head_dim): the tensor maps and the key-norm pass
 * read them in place (no copy).  strides: element strides (batch, head, seq)
 * of each input in argument order (3 per input), positive multiples of 8;
 * out is a contiguous (batch * heads, seq_len, head_dim) array.  head_dim 64 or
 * 128.  Workspace as tda_workspace_size(differential, TDA_BF16, batch * heads,
 * seq_len, head_dim, normalize).  Replaces the same reference entry points as
 * tda_rect_fwd / tda_diff_fwd; the reference indexes such views with the
 * (batch * heads) stride only (triton_threshold_attention.py:49-51), which is
 * wrong for them. */
int tda_rect_fwd_strided(const void* q, const void* k, const void* v, const int64_t* strides, void* out,
                         int out_dtype, int64_t batch, int64_t heads, int64_t seq_len, int64_t head_dim, float beta,
                         float relu_power, int normalize, void* workspace, size_t workspace_bytes, int* status,
                         void* stream);
int tda_diff_fwd_strided(const void* q1, const void* q2, const void* k1, const void* k2, const void* v,
                         const int64_t* strides, void* out, int out_dtype, int64_t batch, int64_t heads,
                         int64_t seq_len, int64_t head_dim, float beta, float lambda_param, float relu_power,
                         int normalize, void* workspace, size_t workspace_bytes, int* status, void* stream);

/* Stage 1 of the normalized tensor-core path, exposed so callers can time or
 * reuse it.  Writes the key table of k into rk (batch_heads * pad * 17 / 16
 * floats, pad = seq_len rounded up to 128): rk[bh * pad + j] =
 * 1 / max(||k[bh][j]||, 1e-12) for j < seq_len and 0 up to pad, followed by
 * rk[batch_heads * pad + bh * pad / 16 + g] = the maximum of those inverse norms
 * over keys [16 g, 16 g + 16).
 * This is the key half of F.normalize (triton_threshold_attention.py:507,509). */
int tda_key_inv_norms(const void* k, int dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float* rk,
                      void* stream);

/* Stage 1 for the two key tensors of the differential form (k1, k2) in one
 * launch: the key tables of k1 into rk1 and of k2 into rk2, laid out as for
 * tda_key_inv_norms (k2 = NULL: k1 only).  dtype TDA_BF16 or TDA_F16.  Key
 * halves of F.normalize(k1), F.normalize(k2) (triton_threshold_attention.py:507,509). */
int tda_key_inv_norms_pair(const void* k1, const void* k2, int dtype, int64_t batch_heads, int64_t seq_len,
                           int64_t head_dim, float* rk1, float* rk2, void* stream);

/* Stage 2 of tda_rect_fwd on the tensor-core path (dtype TDA_BF16), given the
 * key inverse norms from tda_key_inv_norms (ignored, may be NULL, when
 * normalize = 0).  Same semantics as tda_rect_fwd
 * (triton_threshold_attention.py:19-115, :335-403). */
int tda_rect_fwd_tc(const void* q, const void* k, const void* v, void* out, int out_dtype, int64_t batch_heads,
                    int64_t seq_len, int64_t head_dim, float beta, float relu_power, int normalize,
                    const float* rk, int* status, void* stream);

/* Stage 2 of tda_diff_fwd on the tensor-core path (dtype TDA_BF16), given the
 * inverse norms of k1 (rk1) and k2 (rk2).  Same semantics as tda_diff_fwd
 * (triton_threshold_attention.py:489-519). */
int tda_diff_fwd_tc(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out,
                    int out_dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim, float beta,
                    float lambda_param, float relu_power, int normalize, const float* rk1, const float* rk2,
                    int* status, void* stream);

/* Same computation and arguments as tda_diff_fwd, minus the workspace: for
 * callers that cannot allocate device memory -- e.g. code running inside an
 * allocator or memory-pool callback (allocating there would re-enter the
 * allocator), runtimes that forbid allocation after start-up, or plugins whose
 * host owns all device memory and passes only inputs and outputs.  No
 * counterpart in the reference (which allocates fp32 copies on every call).
 * The scratch (inverse key norms) lives in a fixed 8.5 MiB array inside the
 * library, reserved on every GPU that loads it: requires
 * batch_heads * round_up(seq_len, 128) <= 1048576, else TDA_ERR_INVALID.
 * fp32 inputs run the exact-fp32 CUDA-core kernel here (the tensor-core fp32
 * path of tda_diff_fwd needs a caller workspace), and calls with
 * normalize = 0 need no scratch at all.
 * Makes no cudaMalloc / cudaFree call.  The first call on a device looks up
 * the array's address (do it before any stream capture).  All calls share the
 * array: calls whose GPU work overlaps race and must be ordered on one stream. */
int tda_diff_fwd_noalloc(const void* q1, const void* q2, const void* k1, const void* k2, const void* v, void* out,
                         int dtype, int out_dtype, int64_t batch_heads, int64_t seq_len, int64_t head_dim,
                         float beta, float lambda_param, float relu_power, int normalize, int* status,
                         void* stream);

/* Test hook (no counterpart in the reference): inject = 1 makes the next
 * tensor-core launches skip their Q load so every internal wait times out
 * after wait_timeout_ns; inject = 0 restores normal operation.  A
 * wait_timeout_ns of 0 keeps the default (1 s).  Process-wide setting. */
int tda_debug_set(int inject, uint64_t wait_timeout_ns);

/* Diagnostic (no counterpart in the reference): with `counters` pointing at
 * two zeroed uint64 on the device, every later bf16 / fp16 tensor-core forward
 * launch adds [0] the number of 16-key P.V slabs it multiplied and [1] the
 * number a dense P.V would have multiplied (causally skipped key tiles count
 * in neither).  NULL turns it off (the default).  Process-wide setting. */
int tda_debug_stats(void* counters);

#ifdef __cplusplus
}
#endif

#endif /* TDA_B200_H_ */
