/*
 * mx_matmul.h -- C ABI of the B200-native dense-matmul path for moonxi-net.
 *
 * This library replaces the reference's Linear/MLP matmul path behind its own
 * C stub layer.  Reference paths below are relative to the moonxi-net project
 * root.  Every entry point takes plain pointers and sizes, returns an int32
 * status (0 = success, see MX_* codes) and never aborts the process.
 *
 * Pointers are raw device pointers owned by the caller (the reference's bump
 * pool hands out 256-byte aligned blocks, moonxi-net-gpu/cuda/cuda_kernels.cu
 * :922-1004; any 4-byte aligned pointer is accepted).  All launches are
 * asynchronous on the context's stream (the legacy default stream unless set),
 * exactly like the reference's cuBLAS call.
 *
 * `handle`: the reference passes an opaque handle (its cuBLAS handle created
 * by gpu_init, moonxi-net-gpu/cuda/gpu_context.mbt:23-27, and fetched per call
 * with get_context, :34-39).  A handle created by
 * mx_context_create() selects that context; any other value (NULL, or a
 * cuBLAS handle the caller still passes) selects the default context of the
 * current device.  Unknown handles are never dereferenced.
 */
#ifndef MX_MATMUL_H
#define MX_MATMUL_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MX_OK 0
#define MX_ERR_INVALID 1     /* bad argument (negative size, null pointer, ...) */
#define MX_ERR_UNSUPPORTED 2 /* shape/stride this build cannot run            */
#define MX_ERR_CUDA 3        /* a CUDA runtime call failed                      */
#define MX_ERR_TIMEOUT 4     /* a bounded in-kernel wait gave up                */
#define MX_ERR_NOMEM 5       /* workspace allocation failed                     */
#define MX_ERR_NO_DEVICE 6   /* no usable CUDA device                           */
#define MX_ERR_COMM 7        /* a collective failed / the communicator is in error */

/* Precision modes for the contraction. */
#define MX_PREC_DEFAULT 0 /* the context's mode (env MX_MATMUL_PRECISION, else AUTO) */
#define MX_PREC_AUTO 1    /* fp32-class: 3xTF32 tensor cores for large shapes, FP32 SIMT otherwise */
#define MX_PREC_FP32 2    /* exact-fp32 SIMT (FFMA) kernel                     */
#define MX_PREC_3XTF32 3  /* tcgen05 3xTF32 split, fp32-class accuracy         */
#define MX_PREC_TF32 4    /* tcgen05 plain TF32 (opt-in, ~1e-3 relative)       */
#define MX_PREC_NPARRAY 5 /* bit-exact to the NpArray CPU path: fp32 multiply then add in
                           * k order, no split-K (SIMT, half the FP32 rate).  On a
                           * context it also puts the training-step ops in NpArray order. */

/* ---------------------------------------------------------------------- */
/* Reference-compatible entry points                                       */
/* ---------------------------------------------------------------------- */

/* Replaces `cuda_matmul` (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499).
 * Row-major C[M,N] = alpha * op(A) op(B) + beta * C.
 * transpose_a = 0: A stored [M,K]; 1: A stored [K,M] and used transposed.
 * transpose_b = 0: B stored [K,N]; 1: B stored [N,K] and used transposed.
 * beta == 0 never reads C.  Uses the context's precision mode. */
int cuda_matmul(void* handle, float* a, float* b, float* c, int M, int K, int N,
                int transpose_a, int transpose_b, float alpha, float beta);

/* Replaces `moonbit_cuda_matmul` (moonxi-net-gpu/cuda/cuda_stub.c:948-969),
 * the stub bound by `extern "c" fn moonbit_cuda_matmul`
 * (moonxi-net-gpu/cuda/ffi.mbt:526-539).  Same signature and semantics. */
int32_t moonbit_cuda_matmul(void* handle, void* a, void* b, void* c, int32_t M, int32_t K,
                            int32_t N, int32_t transpose_a, int32_t transpose_b, float alpha,
                            float beta);

/* ---------------------------------------------------------------------- */
/* New entry points on the same path                                        */
/* ---------------------------------------------------------------------- */

/* moonbit_cuda_matmul with an explicit stream (NULL = context stream) and
 * precision (MX_PREC_*).  Extends moonxi-net-gpu/cuda/cuda_stub.c:948-969. */
int32_t moonbit_cuda_matmul_ex(void* handle, void* a, void* b, void* c, int32_t M, int32_t K,
                               int32_t N, int32_t transpose_a, int32_t transpose_b, float alpha,
                               float beta, void* stream, int32_t precision);

/* Fused Linear forward: y[M,N] = act(alpha * x[M,K] op(w) + bias[N]), act =
 * ReLU when relu != 0.  transpose_w = 0: w stored [K,N] (Linear::forward,
 * moonxi-net/model/layers.mbt:59-64); 1: w stored [N,K] (MLP::forward,
 * moonxi-net/model/mlp.mbt:16-23).  bias may be NULL.  Replaces the
 * reference's matmul + add + relu sequence (tensor/trait_impl.mbt:209-250,
 * cuda_kernels.cu:132-139 elementwise_add, :795-810 cuDNN ReLU) and its dead
 * gpu_linear (moonxi-net-gpu/tensor/linear.mbt:5-37).  The bias is a true
 * row broadcast, added after the matmul is rounded (NpArray order). */
int32_t moonbit_cuda_linear_fwd(void* handle, void* x, void* w, void* bias, void* y, int32_t M,
                                int32_t K, int32_t N, int32_t transpose_w, int32_t relu,
                                float alpha);

/* moonbit_cuda_linear_fwd with explicit stream and precision. */
int32_t moonbit_cuda_linear_fwd_ex(void* handle, void* x, void* w, void* bias, void* y,
                                   int32_t M, int32_t K, int32_t N, int32_t transpose_w,
                                   int32_t relu, float alpha, void* stream, int32_t precision);

/* The reference's fused forward in its own rounding order:
 * y = act(bias + sum_k x[m,k] op(w)[k,n]), the sum started from the bias and
 * accumulated as fp32 multiply then add in k order -- fused_linear_relu /
 * fused_linear (moonxi-net/nparray/fused_ops.mbt:12-78; weights [out, in],
 * i.e. transpose_w = 1, there), bit-identical to that CPU code.  pre (may be
 * NULL) receives the pre-ReLU values, the second result of
 * fused_linear_relu.  The ordinary forward (moonbit_cuda_linear_fwd) adds
 * the bias after the rounded matmul (matmul -> add -> relu). */
int32_t mx_linear_fwd_bias_first(void* handle, const float* x, const float* w, const float* bias,
                                 float* y, float* pre, int32_t M, int32_t K, int32_t N,
                                 int32_t transpose_w, int32_t relu, void* stream);

/* General form behind all of the above: C[M,N] = act(alpha op(A) op(B) +
 * beta C + bias[N]) for any transpose flags, explicit leading dimensions
 * (lda/ldb/ldc in elements; 0 = the packed default of cuda_matmul), bias may
 * be NULL.  Used by the backward GEMMs and by tests of every layout. */
int32_t mx_gemm_ex(void* handle, const float* a, const float* b, float* c, const float* bias,
                   int32_t M, int32_t K, int32_t N, int32_t transpose_a, int32_t transpose_b,
                   int64_t lda, int64_t ldb, int64_t ldc, float alpha, float beta, int32_t relu,
                   void* stream, int32_t precision);

/* ---- Split-form (3xTF32) operands, produced once by the kernels that write
 * them instead of by a prepass inside every matmul.  A split copy of x is
 * hi = tf32_rna(x), lo = tf32_rna(x - hi), stored as fp32 bit patterns. */

/* hi/lo split of a row-major [rows, cols] matrix (leading dimension ld) into
 * hi/lo with leading dimension ld_out (lo may be NULL: TF32 only).  New; the
 * reference has no split operands. */
int32_t mx_split_tf32(void* handle, const float* src, int32_t rows, int32_t cols, int64_t ld,
                      float* hi, float* lo, int64_t ld_out, void* stream);

/* The tcgen05 GEMM on split operands: C[M,N] = act(alpha A B + beta C +
 * bias), optionally zeroed where mask[row*ldm+col] <= 0 (the ReLU backward of
 * the layer below, grad/image.mbt:45-61), written to c and/or as a split copy
 * to c_hi/c_lo (leading dimension ldc).  a_kmajor = 1: A(m,k) at
 * a[m*lda + k]; 0: at a[k*lda + m] (B likewise with n).  passes = 3: 3xTF32
 * (a_lo/b_lo used), 1: TF32.  Base pointers and leading dimensions must be
 * 16-byte multiples (TMA); M, N, K >= 1.  flags bit 0 (A) / bit 1 (B): the
 * MN-major copies stay readable for 32 floats past their last row, which lets
 * the kernel fetch whole 32-wide chunks when M (N) is not a multiple of 32.
 * Used by the Linear/MLP step for X W, dY W^T and X^T dY (grad/blas.mbt:35,37)
 * without any transpose. */
int32_t mx_gemm_split_ex(void* handle, const float* a_hi, const float* a_lo, int64_t lda,
                         int32_t a_kmajor, const float* b_hi, const float* b_lo, int64_t ldb,
                         int32_t b_kmajor, float* c, float* c_hi, float* c_lo, int64_t ldc,
                         int32_t M, int32_t K, int32_t N, float alpha, float beta,
                         const float* bias, int32_t relu, const float* mask, int64_t ldm,
                         int32_t passes, int32_t flags, void* stream);

/* mx_gemm_split_ex that also writes colsum[N] = the sums over the M rows of
 * the stored output (after bias, ReLU and mask).  When the output is a
 * layer's dY -- the dX GEMM of the layer above, masked by this layer's ReLU --
 * these are the layer's bias gradient: reduce_sum_to on the tape
 * (moonxi-net/grad/grad.mbt:163-174, moonxi-net-gpu/tensor/
 * trait_impl.mbt:85-133), which the reference runs as a separate kernel
 * (cuda_kernels.cu:1383-1406), fused into the GEMM's epilogue.  Deterministic
 * (fixed summation order).  scratch: mx_gemm_colsum_scratch_bytes(M, N)
 * bytes of device memory owned by the caller, 256-byte aligned, not shared
 * with a call that overlaps this one. */
int32_t mx_gemm_split_colsum_ex(void* handle, const float* a_hi, const float* a_lo, int64_t lda,
                                int32_t a_kmajor, const float* b_hi, const float* b_lo,
                                int64_t ldb, int32_t b_kmajor, float* c, float* c_hi, float* c_lo,
                                int64_t ldc, int32_t M, int32_t K, int32_t N, float alpha,
                                float beta, const float* bias, int32_t relu, const float* mask,
                                int64_t ldm, int32_t passes, int32_t flags, float* colsum,
                                void* scratch, uint64_t scratch_bytes, void* stream);
uint64_t mx_gemm_colsum_scratch_bytes(int32_t M, int32_t N);

/* One GEMM of mx_gemm_split_pair: the arguments of mx_gemm_split_colsum_ex
 * (passes = 3) as a plain struct; colsum = NULL: no column sums. */
typedef struct mx_split_gemm {
  const float* a_hi;
  const float* a_lo;
  int64_t lda;
  int32_t a_kmajor;
  const float* b_hi;
  const float* b_lo;
  int64_t ldb;
  int32_t b_kmajor;
  float* c;
  float* c_hi;
  float* c_lo;
  int64_t ldc;
  int32_t M, K, N;
  float alpha, beta;
  const float* bias;
  int32_t relu;
  const float* mask;
  int64_t ldm;
  int32_t flags;
  float* colsum;
  void* colsum_scratch;
  uint64_t colsum_scratch_bytes;
} mx_split_gemm;

/* Two independent 3xTF32 GEMMs on split operands in one persistent launch:
 * a Linear layer's backward, dX = dY W^T and dW = X^T dY (grad/blas.mbt:
 * 35,37), which both read dY and neither reads the other's output.  The
 * tiles of the GEMM with more k-blocks per tile come first, then the
 * other's, round robin over the CTAs, so the second GEMM's tiles run their
 * main loops while the first's epilogues drain: one launch, one prologue and
 * one unhidden epilogue instead of two.  Every tile is computed whole (no
 * split of K), so each output equals that of mx_gemm_split_colsum_ex
 * whenever that call also runs whole tiles.  Layout pairs other than (A
 * K-major, B either) with (A and B MN-major) run as two launches.  The two
 * GEMMs' outputs, column-sum scratch and counters must not overlap. */
int32_t mx_gemm_split_pair(void* handle, const mx_split_gemm* g0, const mx_split_gemm* g1,
                           void* stream);

/* The work split the tcgen05 GEMM of this context picks for an M x N x K
 * shape (passes 3 or 1): out[0] = mode (0 whole tiles, 1 stream-K, 2 tail
 * split), out[1] = first split tile, out[2] = remainder tiles, out[3] =
 * k-blocks of a remainder tile's primary CTA, out[4] = pieces per tail (tail
 * split with at least as many idle CTAs as tiles), out[5] = tails per helper
 * CTA (fewer idle CTAs than tiles).  For tests and tuning. */
int32_t mx_tc_split_plan(void* handle, int32_t M, int32_t N, int32_t K, int32_t passes,
                         int32_t* out);

/* Allocation-free 3xTF32 GEMM.  No counterpart in the reference: it exists
 * for callers that must not allocate device memory inside a library call --
 * for example a host runtime that reserved its whole device-memory budget up
 * front and hands out slices itself (as the reference GPU backend does with
 * its single bump pool), or a process running under a fixed memory budget.
 * Same math and arguments as mx_gemm_ex with transpose flags, packed leading
 * dimensions (cuda_matmul's) and MX_PREC_3XTF32, on the current device and
 * the given stream (NULL = legacy default stream).  It calls no cudaMalloc or
 * cudaFree and no allocating library routine: its scratch (the hi/lo split
 * copies of A and B) is a 64 MiB array compiled into this library, which
 * every GPU that loads the library holds until the process exits.
 *   - Limit: the split copies need 2 * (M*Kp + N*Kp) * 4 bytes (Kp = K
 *     rounded up to a multiple of 4, each copy padded to 256 bytes), at most
 *     64 MiB; larger problems are rejected with MX_ERR_UNSUPPORTED before
 *     anything is launched.
 *   - The first call on a device looks up the device address of that array
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *   - When the 64 MiB is committed: with CUDA's default lazy module loading,
 *     when this library's tensor-core module first loads on a device -- the
 *     first tensor-core GEMM of any entry point, or the first call of this
 *     one -- and at library load under CUDA_MODULE_LOADING=EAGER.  A caller
 *     that reserves the rest of the device's memory for its own pool should
 *     make one call (any size) before reserving it.  If the device has no room
 *     left at that point the call returns MX_ERR_NOMEM (or MX_ERR_CUDA).
 *   - Every call, on every stream, shares the one array, which keeps the last
 *     call's contents: calls that overlap on the GPU race and corrupt each
 *     other's results.  Serialise them (one stream, or events).
 *   - dev_status: optional device pointer to two int32 words; a bounded
 *     in-kernel wait that gives up writes MX_ERR_TIMEOUT and the call site
 *     there (NULL: into a status word inside the library, read and cleared by
 *     mx_noalloc_status). */
int32_t mx_gemm_3xtf32_noalloc(const float* a, const float* b, float* c, const float* bias,
                               int32_t M, int32_t K, int32_t N, int32_t transpose_a,
                               int32_t transpose_b, float alpha, float beta, int32_t relu,
                               int32_t* dev_status, void* stream);

/* Status word of mx_gemm_3xtf32_noalloc calls made with dev_status == NULL on
 * the current device: synchronises the device, returns the recorded status
 * (MX_ERR_TIMEOUT if a bounded in-kernel wait gave up, else MX_OK), writes
 * the call site to `where` (may be NULL) and clears the word.  Allocates
 * nothing.  No counterpart in the reference. */
int32_t mx_noalloc_status(int32_t* where);

/* cudaSetDevice for the calling host thread (the reference hard-codes
 * device 0 at every call site: get_context(0), moonxi-net-gpu/tensor/
 * trait_impl.mbt:232,265,277,287,311). */
int32_t moonbit_cuda_set_device(int32_t device);

/* ---------------------------------------------------------------------- */
/* Contexts (the `handle`)                                                   */
/* ---------------------------------------------------------------------- */

/* Creates a context on `device` (allocates its status word).  NULL on error.
 * Replaces the role of gpu_init's handle (gpu_context.mbt:23-27).  Every entry
 * point that takes a context handle makes the context's device current for
 * the call and restores the caller's current device before it returns. */
void* mx_context_create(int32_t device);
void mx_context_destroy(void* handle);
int32_t mx_context_set_stream(void* handle, void* stream);
int32_t mx_context_set_precision(void* handle, int32_t precision);
/* SMs this context's tensor-core GEMMs prefer to occupy (0 = all).  A
 * data-parallel step sets it below the SM count so that collectives
 * launched on another stream find free SMs while a GEMM runs; a launch still
 * takes every SM (up to the limit below) when that finishes it more than 3 %
 * sooner. */
int32_t mx_context_set_sm_budget(void* handle, int32_t sms);
/* Hard cap on the SMs of this context's tensor-core GEMMs (0 = none): for a
 * step whose collectives must overlap every GEMM (the weight all-gathers of
 * a sharded update run beside the forward GEMMs that need them). */
int32_t mx_context_set_sm_limit(void* handle, int32_t sms);
/* Bound (nanoseconds) on every in-kernel wait; default 2 s. */
int32_t mx_context_set_timeout_ns(void* handle, uint64_t ns);
/* Pre-sizes the context workspace (split operands, split-K partials) so that
 * later calls allocate nothing; required before CUDA-graph capture. */
int32_t mx_context_reserve_workspace(void* handle, uint64_t bytes);
/* Workspace bytes a matmul of this shape and precision would need. */
uint64_t mx_matmul_workspace_bytes(void* handle, int32_t M, int32_t K, int32_t N,
                                   int32_t transpose_a, int32_t transpose_b, int32_t precision);
/* Synchronises the context's device, returns the device status word
 * (MX_ERR_TIMEOUT if a bounded wait gave up since the last query) and clears
 * it.  `where` (may be NULL) receives the in-kernel call site code. */
int32_t mx_context_status(void* handle, int32_t* where);
/* Precision the dispatcher would pick for this call (MX_PREC_FP32,
 * MX_PREC_3XTF32 or MX_PREC_TF32). */
int32_t mx_matmul_resolve_precision(void* handle, int32_t M, int32_t K, int32_t N,
                                    int32_t precision);
const char* mx_status_string(int32_t status);
/* Number of kernels this library has launched in this process (all devices);
 * lets callers count the native launches inside a timed region. */
uint64_t mx_kernel_launch_count(void);

/* ---------------------------------------------------------------------- */
/* The rest of one Linear/MLP training step (adjacent ops on the tape)      */
/* ---------------------------------------------------------------------- */

/* grad_in[i] = saved[i] > 0 ? grad_out[i] : 0 over n elements.  `saved` may
 * be the ReLU input or its output (x > 0 <=> relu(x) > 0).  Replaces
 * cudnn_relu_backward (cuda_kernels.cu:812-831), NpArray semantics
 * moonxi-net/nparray/image_impl.mbt:146-159. */
int32_t mx_relu_backward(void* handle, const float* grad_out, const float* saved,
                         float* grad_in, int64_t n, void* stream);

/* out[j] = sum_i in[i * output_numel + j] for i < lead_stride (bias
 * gradient).  Same arguments as cuda_reduce_sum_leading
 * (cuda_kernels.cu:1383-1406); deterministic fixed-order tree sum. */
int32_t mx_reduce_sum_leading(void* handle, const float* in, float* out, int32_t output_numel,
                              int32_t lead_stride, void* stream);

/* Softmax cross-entropy with integer labels (stored as floats), forward and
 * backward in one pass: loss[0] = sum_rows(-log_softmax[label]) / denom and
 * grad[b,j] = (softmax[b,j] - onehot) / denom.  denom is the local batch on
 * one device or the global batch under data parallelism.  grad may be NULL.
 * Replaces cuda_softmax_ce_forward_labels / _backward_labels
 * (cuda_kernels.cu:1283-1374); NpArray semantics
 * moonxi-net/nparray/image_impl.mbt:83-114,202-238. */
int32_t mx_softmax_ce_labels(void* handle, const float* logits, const float* labels,
                             float* grad, float* loss, int32_t batch, int32_t num_classes,
                             int32_t denom, void* stream);

/* Momentum SGD with global-norm auto clipping over one flat parameter
 * buffer (all parameters concatenated in [w1, b1, w2, b2, ...] order):
 *   norm = ||grads||, c = norm > max_norm ? max_norm / norm : 1,
 *   v = momentum*v + g*c + weight_decay*p,  p = p - lr*v.
 * Runs without a host round trip; norm_out (device, may be NULL) receives the
 * norm.  Replaces mt_norm_sq + mt_sgd_momentum_autoclip (cuda_kernels.cu
 * :1884-2029, driven by moonxi-net-gpu/tensor/optimizer.mbt:106-178). */
int32_t mx_sgd_momentum_autoclip(void* handle, float* params, const float* grads, float* vels,
                                 int64_t n, float lr, float momentum, float weight_decay,
                                 float max_grad_norm, float* norm_out, void* stream);

/* mx_softmax_ce_labels that also writes the split copy g_hi/g_lo of the
 * gradient (same layout) for the split-form backward GEMMs. */
int32_t mx_softmax_ce_labels_split(void* handle, const float* logits, const float* labels,
                                   float* grad, float* g_hi, float* g_lo, float* loss,
                                   int32_t batch, int32_t num_classes, int32_t denom,
                                   void* stream);

/* mx_softmax_ce_labels_split that also writes colsum[num_classes] = the
 * column sums of the gradient: the output layer's bias gradient
 * (reduce_sum_to, grad/grad.mbt:163-174; cuda_kernels.cu:1383-1406 in the
 * reference), fused into the loss kernel, deterministic.  scratch:
 * mx_softmax_ce_colsum_scratch_bytes(batch, num_classes) bytes of caller
 * device memory, 256-byte aligned (0 bytes: num_classes above 4096, not
 * fused; the call then returns MX_ERR_UNSUPPORTED). */
int32_t mx_softmax_ce_labels_split_colsum(void* handle, const float* logits, const float* labels,
                                          float* grad, float* g_hi, float* g_lo, float* loss,
                                          int32_t batch, int32_t num_classes, int32_t denom,
                                          float* colsum, void* scratch, uint64_t scratch_bytes,
                                          void* stream);
uint64_t mx_softmax_ce_colsum_scratch_bytes(int32_t batch, int32_t num_classes);

/* mx_sgd_momentum_autoclip that also writes the split copy p_hi/p_lo of the
 * updated parameters (same flat layout) for the next step's GEMMs. */
int32_t mx_sgd_momentum_autoclip_split(void* handle, float* params, const float* grads,
                                       float* vels, int64_t n, float lr, float momentum,
                                       float weight_decay, float max_grad_norm, float* norm_out,
                                       float* p_hi, float* p_lo, void* stream);

/* The two halves of mx_sgd_momentum_autoclip, for a data-parallel update
 * sharded over ranks (each rank owns some ranges of the flat buffers).  The
 * reference replicates the whole update on its one device (cuda_kernels.cu
 * :1884-2029); these let each of G ranks update 1/G of the parameters:
 *   mx_sum_squares: out[0] = (accumulate ? out[0] : 0) + sum x[i]^2, a fixed
 *     reduction tree (deterministic); a rank sums its gradient ranges, then
 *     the ranks all-reduce the partial sums into the squared global norm;
 *   mx_sgd_momentum_clip: the update of mx_sgd_momentum_autoclip on one
 *     range, with norm = sqrt(*norm_sq) read on the device. */
int32_t mx_sum_squares(void* handle, const float* x, int64_t n, float* out, int32_t accumulate,
                       void* stream);
int32_t mx_sgd_momentum_clip(void* handle, float* params, const float* grads, float* vels,
                             int64_t n, float lr, float momentum, float weight_decay,
                             float max_grad_norm, const float* norm_sq, void* stream);

/* ---------------------------------------------------------------------- */
/* Data-parallel collectives (NCCL over NVLink / NVSwitch)                  */
/* ---------------------------------------------------------------------- */
/* The reference has no collectives: its only host loop, run_gpu
 * (moonxi-net-gpu/train/run.mbt:14-57), trains on one device and reaches
 * native code only through MOONBIT_FFI_EXPORT stubs
 * (moonxi-net-gpu/cuda/cuda_stub.c).  These stubs give such a host the
 * data-parallel step: one process per GPU, a communicator per process, the
 * weight-gradient all-reduce (or reduce-scatter + all-gather for a sharded
 * update) on a stream of the caller's choice.  NCCL is loaded at run time;
 * without it every call returns MX_ERR_UNSUPPORTED.  Handles are never
 * dereferenced when unknown (MX_ERR_INVALID). */
#define MX_NCCL_UNIQUE_ID_BYTES 128

/* NCCL version (e.g. 22809), or -1 when NCCL cannot be loaded. */
int32_t moonbit_nccl_version(void);
/* Fills id[128] with a fresh NCCL unique id: rank 0 makes it and hands the
 * bytes to every other rank by any side channel. */
int32_t moonbit_nccl_get_unique_id(uint8_t* id);
/* Communicator of `rank` in `world` ranks on `device` from the shared id
 * (every rank calls it; it returns once all have).  NULL on failure, with
 * the reason in moonbit_nccl_last_status().  Like the reference's
 * moonbit_cublas_create (cuda_stub.c:240-242), the handle is a plain void*. */
void* moonbit_nccl_init(const uint8_t* id, int32_t rank, int32_t world, int32_t device);
/* moonbit_nccl_init with a cap on the CTAs (SMs) each of the communicator's
 * collectives may take (max_ctas = 0: NCCL's default).  A data-parallel step
 * whose GEMMs leave S SMs free passes S, so that a collective overlapping a
 * GEMM runs all of its channels at once instead of waiting for the GEMM to
 * release SMs (NCCL's ncclCommInitRankConfig: maxCTAs, and cgaClusterSize 1
 * so that no launch needs several free SMs of one GPC at once). */
void* moonbit_nccl_init_ex(const uint8_t* id, int32_t rank, int32_t world, int32_t device,
                           int32_t max_ctas);
/* moonbit_nccl_init with a file as the side channel, for hosts that have no
 * other: rank 0 writes a fresh id to `path` (written to a temporary name and
 * renamed, so readers never see part of it), the other ranks wait up to
 * timeout_ms for it (then NULL with MX_ERR_TIMEOUT).  Delete the file after
 * every rank has initialised. */
void* moonbit_nccl_init_file(const char* path, int32_t rank, int32_t world, int32_t device,
                             int32_t timeout_ms);
/* Status of the calling thread's last moonbit_nccl_init / _init_file. */
int32_t moonbit_nccl_last_status(void);
int32_t moonbit_nccl_comm_info(void* comm, int32_t* rank, int32_t* world, int32_t* device);
/* Sum of `count` floats over all ranks, enqueued on `stream` (NULL = legacy
 * default stream); send == recv is the in-place form. */
int32_t moonbit_nccl_allreduce_sum_f32(void* comm, const float* send, float* recv, int64_t count,
                                       void* stream);
/* recv[recv_count] = this rank's piece of the sum of send[world *
 * recv_count]; in place when recv == send + rank * recv_count. */
int32_t moonbit_nccl_reduce_scatter_sum_f32(void* comm, const float* send, float* recv,
                                            int64_t recv_count, void* stream);
/* recv[world * send_count] = every rank's send[send_count] in rank order; in
 * place when send == recv + rank * send_count. */
int32_t moonbit_nccl_all_gather_f32(void* comm, const float* send, float* recv,
                                    int64_t send_count, void* stream);
/* recv[count] = root's send[count] (send is read on the root only). */
int32_t moonbit_nccl_broadcast_f32(void* comm, const float* send, float* recv, int64_t count,
                                   int32_t root, void* stream);
/* Brackets several collectives into one launch (ncclGroupStart/End). */
int32_t moonbit_nccl_group_start(void);
int32_t moonbit_nccl_group_end(void);
/* MX_OK while the communicator is healthy, MX_ERR_COMM once NCCL has
 * recorded an asynchronous error (e.g. a peer that went away). */
int32_t moonbit_nccl_get_async_error(void* comm);
/* Host-side watchdog: waits until `stream` has drained, polling the
 * communicator's asynchronous error.  On an error (MX_ERR_COMM) or after
 * timeout_ms (MX_ERR_TIMEOUT) it aborts the communicator -- its kernels stop
 * waiting for peers -- and the handle becomes invalid.  The reference aborts
 * the whole process on any failure instead (gpu_tensor.mbt:12-16). */
int32_t moonbit_nccl_wait(void* comm, void* stream, int32_t timeout_ms);
/* Aborts the communicator (ncclCommAbort); the handle becomes invalid. */
int32_t moonbit_nccl_abort(void* comm);
/* Finalises and destroys the communicator; every rank calls it. */
int32_t moonbit_nccl_destroy(void* comm);

#ifdef __cplusplus
}
#endif

#endif /* MX_MATMUL_H */
