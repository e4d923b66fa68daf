// mx_internal.h -- host-side declarations shared by the kernel files and the
// C-ABI layer (abi.cu).  Nothing here is exported.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <atomic>
#include <cstddef>
#include <cstdint>

namespace mx {

// Per-device execution context.  The reference passes an opaque handle to
// every matmul (a cuBLAS handle created by gpu_init,
// moonxi-net-gpu/cuda/gpu_context.mbt:23-27);
// this library's handle is a Context, or NULL for the per-device default.
struct Context {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;  // stream used by calls that take none
  int precision = 0;              // MX_PREC_* default for calls that take none
  int* status = nullptr;          // device words: [0] status code, [1] call site
  int* sched = nullptr;           // device word: dynamic tile counter (status + 2)
  void* workspace = nullptr;      // scratch for split operands / split-K partials
  size_t ws_bytes = 0;
  void* small_scratch = nullptr;  // reduction partials (loss, gradient norm)
  size_t small_bytes = 0;
  uint64_t timeout_ns = 2000000000ull;  // bound on every in-kernel wait
  int sync_check = 0;             // synchronise and check status after each call
  // Arrival counters of split-K launches that leave them zero (the skinny
  // kernel): zeroed once when the context is made, so those launches need
  // no memset.  Calls that overlap on the GPU must not share a context.
  static constexpr int kCounters = 65536;
  int* counters = nullptr;
  // SMs the tensor-core GEMMs prefer to occupy (0: all).  A data-parallel
  // step leaves the rest free so that NCCL kernels overlapping a GEMM find
  // SMs (a persistent GEMM CTA and an NCCL CTA do not fit on one SM
  // together); a launch still takes every SM when that finishes it more than
  // 3 % sooner (tc_launch_sms).
  int sm_budget = 0;
  // Hard cap on those SMs (0: none).
  int sm_limit = 0;
  int tc_all() const { return sm_limit > 0 && sm_limit < num_sms ? sm_limit : num_sms; }
  int tc_sms() const { return sm_budget > 0 && sm_budget < tc_all() ? sm_budget : tc_all(); }
};

// One GEMM as the reference defines it (cuda_kernels.cu:1444-1499), with the
// fused epilogue added: C = act(alpha * op(A) op(B) + beta * C + bias[col]).
// Leading dimensions are in elements; ta/tb select the stored layout.
struct GemmArgs {
  const float* a = nullptr;
  const float* b = nullptr;
  float* c = nullptr;
  int M = 0, K = 0, N = 0;
  int ta = 0, tb = 0;
  int64_t lda = 0, ldb = 0, ldc = 0;
  float alpha = 1.0f, beta = 0.0f;
  const float* bias = nullptr;
  int relu = 0;
  // NpArray order: fp32 multiply then add, k ascending, no split-K.  Only the
  // SIMT kernel honours it; results are bit-identical to the CPU path.
  int strict = 0;
  // With strict: every sum starts from bias[col] (the bias-first order of
  // nparray/fused_ops.mbt:12-78) instead of adding the bias after it.
  int bias_first = 0;
  // Optional pre-ReLU output (leading dimension ldc), SIMT kernels only.
  float* pre = nullptr;
};

// Grows ctx->workspace to at least `bytes` (stream-ordered free of the old
// block is not needed: growth synchronises the device first).
int ensure_workspace(Context* ctx, size_t bytes);
int ensure_small_scratch(Context* ctx, size_t bytes);

// Exact-fp32 SIMT GEMM (FFMA), TMA-fed when strides allow, cp.async-fed
// otherwise.  Uses ctx workspace for split-K partials.
int simt_gemm(Context* ctx, const GemmArgs& g, cudaStream_t s);
// Launch step of simt_gemm with the split-K scratch given explicitly
// (`scratch` may be NULL when the plan needs none).  Never allocates.
int simt_gemm_launch(Context* ctx, const GemmArgs& g, cudaStream_t s, float* scratch,
                     size_t scratch_bytes);
// Bytes of split-K scratch simt_gemm would use for this shape on this device.
size_t simt_gemm_scratch_bytes(const Context* ctx, const GemmArgs& g);

// Exact-fp32 GEMM for skinny shapes (min(M, N) <= 64, gemm_skinny.cu): streams
// the big operand once.  simt_gemm dispatches to it whenever it applies.
bool skinny_applies(const GemmArgs& g);
size_t skinny_scratch_bytes(const Context* ctx, const GemmArgs& g);
int skinny_gemm(Context* ctx, const GemmArgs& g, cudaStream_t s, void* scratch,
                size_t scratch_bytes);

// tcgen05 tensor-core GEMM.  passes = 3: 3xTF32 split (fp32-class);
// passes = 1: plain TF32.  Uses ctx workspace for the split operands.
int tc_gemm(Context* ctx, const GemmArgs& g, int passes, cudaStream_t s);

size_t tc_gemm_workspace_bytes(const GemmArgs& g, int passes);

// tcgen05 GEMM on operands already in split form.
struct TcLaunch {
  int num_sms;
  int* status;
  uint64_t timeout_ns;
  // scratch for stream-K partial tiles and counters (tc_streamk_bytes); when
  // too small the GEMM runs data-parallel over whole tiles
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // device int for dynamic whole-tile scheduling (zeroed per launch on the
  // launch stream), or null for a static tile order
  int* sched = nullptr;
  // all SMs of the device; num_sms is then the preferred budget (0: num_sms)
  int all_sms = 0;
};
// Scratch of the partial tiles a launch of this shape splits (stream-K or
// tail split; 0: whole tiles only).
size_t tc_streamk_bytes(int M, int N, int K, int num_sms, int passes);
// SMs a single tcgen05 GEMM launch of this shape uses: `budget`, or `all`
// when all SMs finish it more than 3 % sooner (cost model in gemm_tc.cu).
int tc_launch_sms(int M, int N, int K, int budget, int all, int passes);
// Scratch of the partial tiles for a launch on context c.
inline size_t tc_split_scratch(const Context* c, int M, int N, int K, int passes) {
  return tc_streamk_bytes(M, N, K, tc_launch_sms(M, N, K, c->tc_sms(), c->tc_all(), passes),
                          passes);
}
// One operand in hi/lo split form (lo may be null for passes = 1).
// kmajor: element (r, k) at hi[r * ld + k]; else at hi[k * ld + r].
struct SplitOperand {
  const float* hi;
  const float* lo;
  int64_t ld;
  bool kmajor;
  // MN-major only: memory stays readable for at least 32 floats past the
  // last row of every copy, so whole 32-row chunks may be read (the rows
  // past the operand feed only output rows/columns that are not stored).
  bool padded = false;
};
// Epilogue: v = alpha*acc (+ beta*c) (+ bias[col]), ReLU if relu, zeroed
// where mask[row*ldm+col] <= 0 if mask; written to c (if non-null) and as
// hi/lo split to c_hi/c_lo (if non-null), all with leading dimension ldc.
struct TcEpilogue {
  float* c = nullptr;
  int64_t ldc = 0;
  float alpha = 1.0f, beta = 0.0f;
  const float* bias = nullptr;
  int relu = 0;
  const float* mask = nullptr;
  int64_t ldm = 0;
  float* c_hi = nullptr;
  float* c_lo = nullptr;
  // optional column sums of the stored output over its M rows (the bias
  // gradient when the output is a layer's dY); scratch of
  // tc_colsum_scratch_bytes(M, N) bytes, 256-byte aligned
  float* colsum = nullptr;
  void* colsum_scratch = nullptr;
  size_t colsum_scratch_bytes = 0;
};
size_t tc_colsum_scratch_bytes(int M, int N);
int tc_gemm_split(const TcLaunch& L, const SplitOperand& A, const SplitOperand& B,
                  const TcEpilogue& E, int M, int N, int K, int passes, cudaStream_t s);
// One GEMM of a paired launch (3xTF32 split operands).
struct TcPairGemm {
  SplitOperand A, B;
  TcEpilogue E;
  int M = 0, N = 0, K = 0;
};
// Two independent 3xTF32 GEMMs in one persistent launch (whole tiles, the
// GEMM with more k-blocks per tile first); layout pairs other than those of
// a Linear layer's backward (dX with a K-major A, dW with both operands
// MN-major) run as two launches.
int tc_gemm_pair(const TcLaunch& L, const TcPairGemm& g0, const TcPairGemm& g1, cudaStream_t s);
// The split plan tc_gemm_split picks for a shape: out[0..5] = mode (0 whole
// tiles, 1 stream-K, 2 tail split), first split tile, remainder tiles r,
// primary k-blocks kp, pieces per tail s, tails per helper j.
void tc_split_plan(int M, int N, int K, int num_sms, int passes, int32_t* out);
// hi/lo split of a row-major [rows][cols] matrix (leading dimension ld) into
// hi/lo with leading dimension ld_out.
int split_tf32(Context* ctx, const float* src, int64_t ld, int rows, int cols, float* hi,
               float* lo, int64_t ld_out, cudaStream_t s);

// Adjacent ops of the training step (mlp_ops.cu).
int relu_backward(Context* ctx, const float* g, const float* x, float* out, int64_t n,
                  cudaStream_t s);
int reduce_sum_leading(Context* ctx, const float* in, float* out, int cols, int rows,
                       cudaStream_t s);
// g_hi/g_lo, p_hi/p_lo (optional): also write the 3xTF32 hi/lo split of the
// gradient / of the updated parameters (the fast path's operands).
int softmax_ce_labels(Context* ctx, const float* logits, const float* labels, float* grad,
                      float* loss, int batch, int C, int denom, cudaStream_t s,
                      float* g_hi = nullptr, float* g_lo = nullptr);
// softmax_ce_labels that also writes colsum[C] = column sums of the gradient
// (the output layer's bias gradient), fused; scratch of
// softmax_ce_colsum_scratch_bytes(batch, C) bytes (0: C too large to fuse).
size_t softmax_ce_colsum_scratch_bytes(int batch, int C);
int softmax_ce_labels_colsum(Context* ctx, const float* logits, const float* labels, float* grad,
                             float* loss, int batch, int C, int denom, cudaStream_t s,
                             float* g_hi, float* g_lo, float* colsum, void* scratch,
                             size_t scratch_bytes);
int sgd_momentum_autoclip(Context* ctx, float* p, const float* g, float* v, int64_t n, float lr,
                          float momentum, float wd, float max_norm, float* norm_out,
                          cudaStream_t s, float* p_hi = nullptr, float* p_lo = nullptr);
// Data-parallel sharded update: out[0] (+)= sum of x^2 over one range, and
// the momentum-SGD update of one range clipped by sqrt(*norm_sq).
int sum_squares(Context* ctx, const float* x, int64_t n, float* out, int accumulate,
                cudaStream_t s);
int sgd_momentum_clip(Context* ctx, float* p, const float* g, float* v, int64_t n, float lr,
                      float momentum, float wd, float max_norm, const float* norm_sq,
                      cudaStream_t s);

// cuTensorMapEncodeTiled through the runtime's driver entry point.
bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle);

// 3-D variant (dims and box innermost first; strides of dims 1 and 2).
bool make_tmap_3d(CUtensorMap* map, const void* base, const uint64_t dims[3],
                  const uint64_t strides_bytes[2], const uint32_t box[3],
                  CUtensorMapSwizzle swizzle);

int cuda_status(cudaError_t e);

// Counts kernel launches (diagnostic, exported as mx_kernel_launch_count).
void note_launches(int n);

// Raises a kernel's dynamic shared-memory limit once per device.  One static
// instance per kernel; safe from several host threads (a race only repeats
// the idempotent attribute call).  Devices beyond the table are configured on
// every launch.
struct SmemOptIn {
  static constexpr int kMaxDevices = 64;
  std::atomic<bool> done[kMaxDevices] = {};
  template <typename Kernel>
  cudaError_t ensure(Kernel kern, int bytes) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < kMaxDevices && done[dev].load(std::memory_order_acquire))
      return cudaSuccess;
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e == cudaSuccess && dev >= 0 && dev < kMaxDevices)
      done[dev].store(true, std::memory_order_release);
    return e;
  }
};

}  // namespace mx
