// abi.cu -- the C-ABI layer (include/mx_matmul.h): contexts, argument
// checking, precision dispatch and the exported entry points.
//
// The exported matmul keeps the reference's name, signature and semantics
// (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499 cuda_matmul and
// moonxi-net-gpu/cuda/cuda_stub.c:948-969 moonbit_cuda_matmul): row-major,
// transpose flags select the stored layout, C = alpha op(A) op(B) + beta C,
// asynchronous on the stream, 0 on success.  Unlike the reference, invalid
// arguments and in-kernel timeouts are reported as status codes instead of
// being left to cuBLAS.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <atomic>
#include <mutex>
#include <unordered_set>

#include "../../include/mx_matmul.h"
#include "mx_internal.h"
#include "mx_ptx.cuh"

#define MX_EXPORT extern "C" __attribute__((visibility("default")))

namespace mx {

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return kOk;
  if (e == cudaErrorMemoryAllocation) return kErrNoMem;
  if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) return kErrNoDevice;
  return kErrCuda;
}

static std::atomic<unsigned long long> g_launches{0};
void note_launches(int n) { g_launches.fetch_add(static_cast<unsigned long long>(n)); }

namespace {

std::mutex g_mu;
std::unordered_set<Context*> g_contexts;  // contexts handed out by mx_context_create
Context* g_default[64] = {};              // per-device default contexts

int env_precision() {
  const char* e = std::getenv("MX_MATMUL_PRECISION");
  if (!e) return MX_PREC_AUTO;
  if (!strcmp(e, "fp32")) return MX_PREC_FP32;
  if (!strcmp(e, "3xtf32")) return MX_PREC_3XTF32;
  if (!strcmp(e, "tf32")) return MX_PREC_TF32;
  if (!strcmp(e, "nparray")) return MX_PREC_NPARRAY;
  return MX_PREC_AUTO;
}

int init_context(Context* c, int device) {
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return kErrNoDevice;
  if (device < 0 || device >= count) return kErrInvalid;
  int prev = 0;
  cudaGetDevice(&prev);
  if (prev != device) cudaSetDevice(device);
  c->device = device;
  cudaDeviceGetAttribute(&c->num_sms, cudaDevAttrMultiProcessorCount, device);
  c->precision = env_precision();
  c->sync_check = std::getenv("MX_SYNC_CHECK") ? std::atoi(std::getenv("MX_SYNC_CHECK")) : 0;
  // words: [0] status, [1] call site, [2] dynamic tile counter of the GEMMs
  cudaError_t e = cudaMalloc(&c->status, 4 * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->status, 0, 4 * sizeof(int));
  c->sched = c->status + 2;
  if (e == cudaSuccess) e = cudaMalloc(&c->counters, Context::kCounters * sizeof(int));
  if (e == cudaSuccess) e = cudaMemset(c->counters, 0, Context::kCounters * sizeof(int));
  if (prev != device) cudaSetDevice(prev);
  return cuda_status(e);
}

// The context for `handle`: a registered context, else the current device's
// default context (created on first use).  Never dereferences unknown handles.
// A registered context on another device is made current; *prev receives the
// device to restore afterwards (-1 when nothing was switched).
Context* resolve(void* handle, int* prev) {
  *prev = -1;
  std::lock_guard<std::mutex> lk(g_mu);
  Context* c = static_cast<Context*>(handle);
  if (c && g_contexts.count(c)) {
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != c->device) {
      if (cudaSetDevice(c->device) != cudaSuccess) return nullptr;
      *prev = cur;
    }
    return c;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  if (!g_default[dev]) {
    Context* d = new Context();
    if (init_context(d, dev) != kOk) {
      delete d;
      return nullptr;
    }
    g_default[dev] = d;
  }
  return g_default[dev];
}

// An entry point's context for the duration of the call: the context's
// device is current inside the call, and the caller's current device is
// restored on return (a host thread that drives several devices keeps its
// own device selection).
struct Scoped {
  Context* c = nullptr;
  int prev = -1;
  explicit Scoped(void* handle) { c = resolve(handle, &prev); }
  ~Scoped() {
    if (prev >= 0) cudaSetDevice(prev);
  }
  Scoped(const Scoped&) = delete;
  Scoped& operator=(const Scoped&) = delete;
};

cudaStream_t pick_stream(Context* c, void* stream) {
  return stream ? static_cast<cudaStream_t>(stream) : c->stream;
}

int resolve_precision(Context* c, int M, int K, int N, int precision) {
  int p = precision == MX_PREC_DEFAULT ? c->precision : precision;
  if (p == MX_PREC_DEFAULT) p = MX_PREC_AUTO;
  if (p == MX_PREC_AUTO) {
    // Tensor cores pay off once the problem fills the machine; small or
    // skinny products stay on the exact SIMT kernel.
    const double flops = 2.0 * M * static_cast<double>(N) * K;
    p = (M >= 128 && N >= 128 && K >= 64 && flops >= 1.0e9) ? MX_PREC_3XTF32 : MX_PREC_FP32;
  }
  return p;
}

int finish(Context* c, int rc, cudaStream_t s) {
  if (rc != kOk || !c->sync_check) return rc;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return cuda_status(e);
  int st[2] = {0, 0};
  cudaMemcpy(st, c->status, sizeof(st), cudaMemcpyDeviceToHost);
  if (st[0] != 0) {
    cudaMemset(c->status, 0, sizeof(st));
    return st[0];
  }
  return kOk;
}

int run_gemm(Context* c, const GemmArgs& g, int precision, cudaStream_t s) {
  if (g.M < 0 || g.N < 0 || g.K < 0) return kErrInvalid;
  if (g.M == 0 || g.N == 0) return kOk;
  if (!g.c || ((!g.a || !g.b) && g.K > 0)) return kErrInvalid;
  const int p = resolve_precision(c, g.M, g.K, g.N, precision);
  int rc;
  if (p == MX_PREC_3XTF32) rc = tc_gemm(c, g, 3, s);
  else if (p == MX_PREC_TF32) rc = tc_gemm(c, g, 1, s);
  else if (p == MX_PREC_FP32) rc = simt_gemm(c, g, s);
  else if (p == MX_PREC_NPARRAY) {
    GemmArgs gs = g;
    gs.strict = 1;
    rc = simt_gemm(c, gs, s);
  } else rc = kErrInvalid;
  return finish(c, rc, s);
}

GemmArgs ref_args(float* a, float* b, float* c, int M, int K, int N, int ta, int tb, float alpha,
                  float beta) {
  GemmArgs g;
  g.a = a; g.b = b; g.c = c;
  g.M = M; g.K = K; g.N = N;
  g.ta = ta ? 1 : 0; g.tb = tb ? 1 : 0;
  // Leading dimensions exactly as the reference derives them
  // (cuda_kernels.cu:1482-1483): lda = ta ? M : K, ldb = tb ? K : N, ldc = N.
  g.lda = ta ? M : K;
  g.ldb = tb ? K : N;
  g.ldc = N;
  g.alpha = alpha; g.beta = beta;
  return g;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

bool make_tmap_2d(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer,
                  uint64_t row_stride_bytes, uint32_t box_inner, uint32_t box_outer,
                  CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  // Host-side checks of every TMA rule the hardware would otherwise trap on.
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if (row_stride_bytes % 16 != 0 || (box_inner * 4) % 16 != 0) return false;
  if (box_inner > 256 || box_outer > 256 || inner == 0 || outer == 0) return false;
  if (swizzle >= CU_TENSOR_MAP_SWIZZLE_128B && box_inner * 4 > 128) return false;
  if (swizzle == CU_TENSOR_MAP_SWIZZLE_64B && box_inner * 4 > 64) return false;
  if (inner >= (1ull << 32) || outer >= (1ull << 32)) return false;
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(base), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

bool make_tmap_3d(CUtensorMap* map, const void* base, const uint64_t dims[3],
                  const uint64_t strides_bytes[2], const uint32_t box[3],
                  CUtensorMapSwizzle swizzle) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  if ((reinterpret_cast<uintptr_t>(base) & 15u) != 0) return false;
  if (strides_bytes[0] % 16 != 0 || strides_bytes[1] % 16 != 0 || (box[0] * 4) % 16 != 0)
    return false;
  for (int i = 0; i < 3; ++i)
    if (box[i] == 0 || box[i] > 256 || dims[i] == 0 || dims[i] >= (1ull << 32)) return false;
  if (swizzle >= CU_TENSOR_MAP_SWIZZLE_128B && box[0] * 4 > 128) return false;
  cuuint64_t d[3] = {dims[0], dims[1], dims[2]};
  cuuint64_t st[2] = {strides_bytes[0], strides_bytes[1]};
  cuuint32_t b[3] = {box[0], box[1], box[2]};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<void*>(base), d, st, b,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int ensure_workspace(Context* c, size_t bytes) {
  if (bytes <= c->ws_bytes) return kOk;
  // Growth is rare (first call of a new largest shape); the old block may
  // still be read by queued kernels, so drain the device before freeing it.
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e);
  if (c->workspace) cudaFree(c->workspace);
  c->workspace = nullptr;
  c->ws_bytes = 0;
  const size_t want = bytes + bytes / 8;
  e = cudaMalloc(&c->workspace, want);
  if (e != cudaSuccess) {
    c->workspace = nullptr;
    return kErrNoMem;
  }
  c->ws_bytes = want;
  return kOk;
}

int ensure_small_scratch(Context* c, size_t bytes) {
  if (bytes <= c->small_bytes) return kOk;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e);
  if (c->small_scratch) cudaFree(c->small_scratch);
  c->small_scratch = nullptr;
  c->small_bytes = 0;
  const size_t want = bytes < 65536 ? 65536 : bytes;
  e = cudaMalloc(&c->small_scratch, want);
  if (e != cudaSuccess) {
    c->small_scratch = nullptr;
    return kErrNoMem;
  }
  c->small_bytes = want;
  return kOk;
}

}  // namespace mx

using namespace mx;

// ------------------------------------------------------------------ matmul
MX_EXPORT int cuda_matmul(void* handle, float* a, float* b, float* c, int M, int K, int N,
                          int transpose_a, int transpose_b, float alpha, float beta) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  return run_gemm(ctx, ref_args(a, b, c, M, K, N, transpose_a, transpose_b, alpha, beta),
                  MX_PREC_DEFAULT, ctx->stream);
}

MX_EXPORT int32_t moonbit_cuda_matmul(void* handle, void* a, void* b, void* c, int32_t M,
                                      int32_t K, int32_t N, int32_t transpose_a,
                                      int32_t transpose_b, float alpha, float beta) {
  return cuda_matmul(handle, static_cast<float*>(a), static_cast<float*>(b),
                     static_cast<float*>(c), M, K, N, transpose_a, transpose_b, alpha, beta);
}

MX_EXPORT int32_t moonbit_cuda_matmul_ex(void* handle, void* a, void* b, void* c, int32_t M,
                                         int32_t K, int32_t N, int32_t transpose_a,
                                         int32_t transpose_b, float alpha, float beta,
                                         void* stream, int32_t precision) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  return run_gemm(ctx,
                  ref_args(static_cast<float*>(a), static_cast<float*>(b), static_cast<float*>(c),
                           M, K, N, transpose_a, transpose_b, alpha, beta),
                  precision, pick_stream(ctx, stream));
}

MX_EXPORT int32_t moonbit_cuda_linear_fwd_ex(void* handle, void* x, void* w, void* bias, void* y,
                                             int32_t M, int32_t K, int32_t N,
                                             int32_t transpose_w, int32_t relu, float alpha,
                                             void* stream, int32_t precision) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  GemmArgs g = ref_args(static_cast<float*>(x), static_cast<float*>(w), static_cast<float*>(y), M,
                        K, N, 0, transpose_w, alpha, 0.0f);
  g.bias = static_cast<const float*>(bias);
  g.relu = relu ? 1 : 0;
  return run_gemm(ctx, g, precision, pick_stream(ctx, stream));
}

MX_EXPORT int32_t moonbit_cuda_linear_fwd(void* handle, void* x, void* w, void* bias, void* y,
                                          int32_t M, int32_t K, int32_t N, int32_t transpose_w,
                                          int32_t relu, float alpha) {
  return moonbit_cuda_linear_fwd_ex(handle, x, w, bias, y, M, K, N, transpose_w, relu, alpha,
                                    nullptr, MX_PREC_DEFAULT);
}

MX_EXPORT int32_t mx_linear_fwd_bias_first(void* handle, const float* x, const float* w,
                                           const float* bias, float* y, float* pre, int32_t M,
                                           int32_t K, int32_t N, int32_t transpose_w,
                                           int32_t relu, void* stream) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  if (!bias || !y) return MX_ERR_INVALID;
  GemmArgs g = ref_args(const_cast<float*>(x), const_cast<float*>(w), y, M, K, N, 0, transpose_w,
                        1.0f, 0.0f);
  g.bias = bias;
  g.relu = relu ? 1 : 0;
  g.strict = 1;
  g.bias_first = 1;
  g.pre = pre;
  if (g.M < 0 || g.N < 0 || g.K < 0) return MX_ERR_INVALID;
  if (g.M == 0 || g.N == 0) return MX_OK;
  if (g.K > 0 && (!x || !w)) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(ctx, stream);
  return finish(ctx, simt_gemm(ctx, g, s), s);
}

MX_EXPORT int32_t mx_gemm_ex(void* handle, const float* a, const float* b, float* c,
                             const float* bias, int32_t M, int32_t K, int32_t N,
                             int32_t transpose_a, int32_t transpose_b, int64_t lda, int64_t ldb,
                             int64_t ldc, float alpha, float beta, int32_t relu, void* stream,
                             int32_t precision) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  GemmArgs g = ref_args(const_cast<float*>(a), const_cast<float*>(b), c, M, K, N, transpose_a,
                        transpose_b, alpha, beta);
  if (lda < 0 || ldb < 0 || ldc < 0) return MX_ERR_INVALID;
  if (lda) g.lda = lda;
  if (ldb) g.ldb = ldb;
  if (ldc) g.ldc = ldc;
  // A leading dimension smaller than the row it spans is an argument error.
  if (g.lda < (g.ta ? M : K) || g.ldb < (g.tb ? K : N) || g.ldc < N) return MX_ERR_INVALID;
  g.bias = bias;
  g.relu = relu ? 1 : 0;
  return run_gemm(ctx, g, precision, pick_stream(ctx, stream));
}

MX_EXPORT int32_t mx_split_tf32(void* handle, const float* src, int32_t rows, int32_t cols,
                                int64_t ld, float* hi, float* lo, int64_t ld_out, void* stream) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  if (rows < 0 || cols < 0 || ld < cols || ld_out < cols) return MX_ERR_INVALID;
  if (rows > 0 && cols > 0 && (!src || !hi)) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(ctx, stream);
  return finish(ctx, split_tf32(ctx, src, ld, rows, cols, hi, lo, ld_out, s), s);
}

namespace {
int gemm_split(void* handle, const float* a_hi, const float* a_lo, int64_t lda, int32_t a_kmajor,
               const float* b_hi, const float* b_lo, int64_t ldb, int32_t b_kmajor, float* c,
               float* c_hi, float* c_lo, int64_t ldc, int32_t M, int32_t K, int32_t N,
               float alpha, float beta, const float* bias, int32_t relu, const float* mask,
               int64_t ldm, int32_t passes, int32_t flags, float* colsum, void* scratch,
               uint64_t scratch_bytes, void* stream) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  if (M < 0 || N < 0 || K < 1) return MX_ERR_INVALID;
  if (lda < (a_kmajor ? K : M) || ldb < (b_kmajor ? K : N) || ldc < N) return MX_ERR_INVALID;
  if (mask && ldm < N) return MX_ERR_INVALID;
  if (!c_hi && c_lo) return MX_ERR_INVALID;
  TcLaunch L{ctx->tc_sms(), ctx->status, ctx->timeout_ns};
  L.all_sms = ctx->tc_all();
  L.sched = ctx->sched;
  const size_t sk = tc_split_scratch(ctx, M, N, K, passes);
  if (sk > 0 && ensure_workspace(ctx, sk) == kOk) {
    L.ws = ctx->workspace;
    L.ws_bytes = ctx->ws_bytes;
  }
  SplitOperand A{a_hi, a_lo, lda, a_kmajor != 0, (flags & 1) != 0};
  SplitOperand B{b_hi, b_lo, ldb, b_kmajor != 0, (flags & 2) != 0};
  TcEpilogue E;
  E.c = c; E.ldc = ldc; E.alpha = alpha; E.beta = beta; E.bias = bias; E.relu = relu ? 1 : 0;
  E.mask = mask; E.ldm = ldm; E.c_hi = c_hi; E.c_lo = c_lo;
  E.colsum = colsum; E.colsum_scratch = scratch; E.colsum_scratch_bytes = scratch_bytes;
  cudaStream_t s = pick_stream(ctx, stream);
  return finish(ctx, tc_gemm_split(L, A, B, E, M, N, K, passes, s), s);
}
}  // namespace

MX_EXPORT int32_t mx_gemm_split_ex(void* handle, const float* a_hi, const float* a_lo,
                                   int64_t lda, int32_t a_kmajor, const float* b_hi,
                                   const float* b_lo, int64_t ldb, int32_t b_kmajor, float* c,
                                   float* c_hi, float* c_lo, int64_t ldc, int32_t M, int32_t K,
                                   int32_t N, float alpha, float beta, const float* bias,
                                   int32_t relu, const float* mask, int64_t ldm, int32_t passes,
                                   int32_t flags, void* stream) {
  return gemm_split(handle, a_hi, a_lo, lda, a_kmajor, b_hi, b_lo, ldb, b_kmajor, c, c_hi, c_lo,
                    ldc, M, K, N, alpha, beta, bias, relu, mask, ldm, passes, flags, nullptr,
                    nullptr, 0, stream);
}

MX_EXPORT int32_t mx_gemm_split_colsum_ex(void* handle, const float* a_hi, const float* a_lo,
                                          int64_t lda, int32_t a_kmajor, const float* b_hi,
                                          const float* b_lo, int64_t ldb, int32_t b_kmajor,
                                          float* c, float* c_hi, float* c_lo, int64_t ldc,
                                          int32_t M, int32_t K, int32_t N, float alpha,
                                          float beta, const float* bias, int32_t relu,
                                          const float* mask, int64_t ldm, int32_t passes,
                                          int32_t flags, float* colsum, void* scratch,
                                          uint64_t scratch_bytes, void* stream) {
  if (!colsum) return MX_ERR_INVALID;
  return gemm_split(handle, a_hi, a_lo, lda, a_kmajor, b_hi, b_lo, ldb, b_kmajor, c, c_hi, c_lo,
                    ldc, M, K, N, alpha, beta, bias, relu, mask, ldm, passes, flags, colsum,
                    scratch, scratch_bytes, stream);
}

MX_EXPORT uint64_t mx_gemm_colsum_scratch_bytes(int32_t M, int32_t N) {
  return tc_colsum_scratch_bytes(M, N);
}

namespace {
// Argument checks of one GEMM of a pair (those of gemm_split) and its
// conversion; kOk or MX_ERR_INVALID.
int pair_gemm(const mx_split_gemm* g, TcPairGemm& out) {
  if (!g) return MX_ERR_INVALID;
  if (g->M < 0 || g->N < 0 || g->K < 1) return MX_ERR_INVALID;
  if (g->lda < (g->a_kmajor ? g->K : g->M) || g->ldb < (g->b_kmajor ? g->K : g->N) ||
      g->ldc < g->N)
    return MX_ERR_INVALID;
  if (g->mask && g->ldm < g->N) return MX_ERR_INVALID;
  if (!g->c_hi && g->c_lo) return MX_ERR_INVALID;
  if (g->M > 0 && g->N > 0 && (!g->a_hi || !g->a_lo || !g->b_hi || !g->b_lo))
    return MX_ERR_INVALID;
  out.A = SplitOperand{g->a_hi, g->a_lo, g->lda, g->a_kmajor != 0, (g->flags & 1) != 0};
  out.B = SplitOperand{g->b_hi, g->b_lo, g->ldb, g->b_kmajor != 0, (g->flags & 2) != 0};
  TcEpilogue& E = out.E;
  E.c = g->c; E.ldc = g->ldc; E.alpha = g->alpha; E.beta = g->beta; E.bias = g->bias;
  E.relu = g->relu ? 1 : 0; E.mask = g->mask; E.ldm = g->ldm; E.c_hi = g->c_hi; E.c_lo = g->c_lo;
  E.colsum = g->colsum; E.colsum_scratch = g->colsum_scratch;
  E.colsum_scratch_bytes = g->colsum_scratch_bytes;
  out.M = g->M; out.N = g->N; out.K = g->K;
  return kOk;
}
}  // namespace

MX_EXPORT int32_t mx_gemm_split_pair(void* handle, const mx_split_gemm* g0,
                                     const mx_split_gemm* g1, void* stream) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  TcPairGemm a, b;
  int rc = pair_gemm(g0, a);
  if (rc == kOk) rc = pair_gemm(g1, b);
  if (rc != kOk) return rc;
  TcLaunch L{ctx->tc_sms(), ctx->status, ctx->timeout_ns};
  L.all_sms = ctx->tc_all();
  // a layout pair without a paired kernel runs as two launches, which may
  // split K and then need the stream-K scratch
  const size_t sk = std::max(tc_split_scratch(ctx, a.M, a.N, a.K, 3),
                             tc_split_scratch(ctx, b.M, b.N, b.K, 3));
  if (sk > 0 && ensure_workspace(ctx, sk) == kOk) {
    L.ws = ctx->workspace;
    L.ws_bytes = ctx->ws_bytes;
  }
  cudaStream_t s = pick_stream(ctx, stream);
  return finish(ctx, tc_gemm_pair(L, a, b, s), s);
}

MX_EXPORT int32_t mx_tc_split_plan(void* handle, int32_t M, int32_t N, int32_t K, int32_t passes,
                                   int32_t* out) {
  Scoped scope(handle);
  Context* ctx = scope.c;
  if (!ctx) return MX_ERR_NO_DEVICE;
  if (!out || M < 1 || N < 1 || K < 1 || (passes != 1 && passes != 3)) return MX_ERR_INVALID;
  tc_split_plan(M, N, K, tc_launch_sms(M, N, K, ctx->tc_sms(), ctx->tc_all(), passes),
                passes, out);
  return MX_OK;
}

MX_EXPORT int32_t moonbit_cuda_set_device(int32_t device) {
  return cuda_status(cudaSetDevice(device));
}

// ---------------------------------------------------------------- contexts
MX_EXPORT void* mx_context_create(int32_t device) {
  Context* c = new Context();
  if (init_context(c, device) != kOk) {
    delete c;
    return nullptr;
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_contexts.insert(c);
  return c;
}

MX_EXPORT void mx_context_destroy(void* handle) {
  Context* c = static_cast<Context*>(handle);
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!c || !g_contexts.count(c)) return;
    g_contexts.erase(c);
  }
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(c->device);
  cudaDeviceSynchronize();
  if (c->workspace) cudaFree(c->workspace);
  if (c->small_scratch) cudaFree(c->small_scratch);
  if (c->status) cudaFree(c->status);
  if (c->counters) cudaFree(c->counters);
  cudaSetDevice(prev);
  delete c;
}

MX_EXPORT int32_t mx_context_set_stream(void* handle, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  c->stream = static_cast<cudaStream_t>(stream);
  return MX_OK;
}

MX_EXPORT int32_t mx_context_set_precision(void* handle, int32_t precision) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (precision < MX_PREC_DEFAULT || precision > MX_PREC_NPARRAY) return MX_ERR_INVALID;
  c->precision = precision == MX_PREC_DEFAULT ? env_precision() : precision;
  return MX_OK;
}

MX_EXPORT int32_t mx_context_set_timeout_ns(void* handle, uint64_t ns) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (ns == 0) return MX_ERR_INVALID;
  c->timeout_ns = ns;
  return MX_OK;
}

MX_EXPORT int32_t mx_context_set_sm_budget(void* handle, int32_t sms) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (sms < 0) return MX_ERR_INVALID;
  c->sm_budget = sms;
  return MX_OK;
}

MX_EXPORT int32_t mx_context_set_sm_limit(void* handle, int32_t sms) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (sms < 0) return MX_ERR_INVALID;
  c->sm_limit = sms;
  return MX_OK;
}

MX_EXPORT int32_t mx_context_reserve_workspace(void* handle, uint64_t bytes) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  int rc = ensure_workspace(c, bytes);
  if (rc == kOk) rc = ensure_small_scratch(c, 1 << 20);
  return rc;
}

MX_EXPORT uint64_t mx_matmul_workspace_bytes(void* handle, int32_t M, int32_t K, int32_t N,
                                             int32_t transpose_a, int32_t transpose_b,
                                             int32_t precision) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c || M <= 0 || N <= 0 || K < 0) return 0;
  GemmArgs g = ref_args(nullptr, nullptr, nullptr, M, K, N, transpose_a, transpose_b, 1.0f, 0.0f);
  const int p = resolve_precision(c, M, K, N, precision);
  if (p == MX_PREC_3XTF32)
    return tc_gemm_workspace_bytes(g, 3) + tc_split_scratch(c, M, N, K, 3);
  if (p == MX_PREC_TF32)
    return tc_gemm_workspace_bytes(g, 1) + tc_split_scratch(c, M, N, K, 1);
  if (p == MX_PREC_NPARRAY) return 0;  // no split-K in NpArray order
  return simt_gemm_scratch_bytes(c, g);
}

MX_EXPORT int32_t mx_context_status(void* handle, int32_t* where) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e);
  int st[2] = {0, 0};
  e = cudaMemcpy(st, c->status, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e);
  if (where) *where = st[1];
  if (st[0] != 0) cudaMemset(c->status, 0, sizeof(st));
  return st[0];
}

MX_EXPORT int32_t mx_matmul_resolve_precision(void* handle, int32_t M, int32_t K, int32_t N,
                                              int32_t precision) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  return resolve_precision(c, M, K, N, precision);
}

MX_EXPORT const char* mx_status_string(int32_t status) {
  switch (status) {
    case MX_OK: return "ok";
    case MX_ERR_INVALID: return "invalid argument";
    case MX_ERR_UNSUPPORTED: return "unsupported shape or stride";
    case MX_ERR_CUDA: return "CUDA runtime error";
    case MX_ERR_TIMEOUT: return "bounded in-kernel wait timed out";
    case MX_ERR_NOMEM: return "workspace allocation failed";
    case MX_ERR_NO_DEVICE: return "no usable CUDA device";
    case MX_ERR_COMM: return "collective communication failed";
    default: return "unknown status";
  }
}

MX_EXPORT uint64_t mx_kernel_launch_count(void) { return g_launches.load(); }

// ------------------------------------------------------- training-step ops
MX_EXPORT int32_t mx_relu_backward(void* handle, const float* grad_out, const float* saved,
                                   float* grad_in, int64_t n, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (n < 0 || (n > 0 && (!grad_out || !saved || !grad_in))) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c, relu_backward(c, grad_out, saved, grad_in, n, s), s);
}

MX_EXPORT int32_t mx_reduce_sum_leading(void* handle, const float* in, float* out,
                                        int32_t output_numel, int32_t lead_stride, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (output_numel < 0 || lead_stride < 0 || (output_numel > 0 && (!in || !out)))
    return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c, reduce_sum_leading(c, in, out, output_numel, lead_stride, s), s);
}

MX_EXPORT int32_t mx_softmax_ce_labels(void* handle, const float* logits, const float* labels,
                                       float* grad, float* loss, int32_t batch,
                                       int32_t num_classes, int32_t denom, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (!logits || !labels || batch <= 0 || num_classes <= 0 || denom <= 0) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c, softmax_ce_labels(c, logits, labels, grad, loss, batch, num_classes, denom, s),
                s);
}

MX_EXPORT int32_t mx_softmax_ce_labels_split(void* handle, const float* logits,
                                             const float* labels, float* grad, float* g_hi,
                                             float* g_lo, float* loss, int32_t batch,
                                             int32_t num_classes, int32_t denom, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (!logits || !labels || !grad || !g_hi || !g_lo || batch <= 0 || num_classes <= 0 ||
      denom <= 0)
    return MX_ERR_INVALID;
  if (c->precision == MX_PREC_NPARRAY) return MX_ERR_UNSUPPORTED;  // split form is the fast path
  cudaStream_t s = pick_stream(c, stream);
  return finish(c, softmax_ce_labels(c, logits, labels, grad, loss, batch, num_classes, denom, s,
                                     g_hi, g_lo),
                s);
}

MX_EXPORT int32_t mx_softmax_ce_labels_split_colsum(void* handle, const float* logits,
                                                    const float* labels, float* grad,
                                                    float* g_hi, float* g_lo, float* loss,
                                                    int32_t batch, int32_t num_classes,
                                                    int32_t denom, float* colsum, void* scratch,
                                                    uint64_t scratch_bytes, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (!logits || !labels || !grad || !g_hi || !g_lo || !colsum || batch <= 0 ||
      num_classes <= 0 || denom <= 0)
    return MX_ERR_INVALID;
  if (c->precision == MX_PREC_NPARRAY) return MX_ERR_UNSUPPORTED;  // split form is the fast path
  cudaStream_t s = pick_stream(c, stream);
  return finish(c,
                softmax_ce_labels_colsum(c, logits, labels, grad, loss, batch, num_classes, denom,
                                         s, g_hi, g_lo, colsum, scratch, scratch_bytes),
                s);
}

MX_EXPORT uint64_t mx_softmax_ce_colsum_scratch_bytes(int32_t batch, int32_t num_classes) {
  return softmax_ce_colsum_scratch_bytes(batch, num_classes);
}

MX_EXPORT int32_t mx_sgd_momentum_autoclip_split(void* handle, float* params, const float* grads,
                                                 float* vels, int64_t n, float lr,
                                                 float momentum, float weight_decay,
                                                 float max_grad_norm, float* norm_out,
                                                 float* p_hi, float* p_lo, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (n < 0 || (n > 0 && (!params || !grads || !vels || !p_hi || !p_lo))) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c,
                sgd_momentum_autoclip(c, params, grads, vels, n, lr, momentum, weight_decay,
                                      max_grad_norm, norm_out, s, p_hi, p_lo),
                s);
}

MX_EXPORT int32_t mx_sum_squares(void* handle, const float* x, int64_t n, float* out,
                                 int32_t accumulate, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (n < 0 || !out || (n > 0 && !x)) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c, sum_squares(c, x, n, out, accumulate, s), s);
}

MX_EXPORT int32_t mx_sgd_momentum_clip(void* handle, float* params, const float* grads,
                                       float* vels, int64_t n, float lr, float momentum,
                                       float weight_decay, float max_grad_norm,
                                       const float* norm_sq, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (n < 0 || !norm_sq || (n > 0 && (!params || !grads || !vels))) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c,
                sgd_momentum_clip(c, params, grads, vels, n, lr, momentum, weight_decay,
                                  max_grad_norm, norm_sq, s),
                s);
}

MX_EXPORT int32_t mx_sgd_momentum_autoclip(void* handle, float* params, const float* grads,
                                           float* vels, int64_t n, float lr, float momentum,
                                           float weight_decay, float max_grad_norm,
                                           float* norm_out, void* stream) {
  Scoped scope(handle);
  Context* c = scope.c;
  if (!c) return MX_ERR_NO_DEVICE;
  if (n < 0 || (n > 0 && (!params || !grads || !vels))) return MX_ERR_INVALID;
  cudaStream_t s = pick_stream(c, stream);
  return finish(c,
                sgd_momentum_autoclip(c, params, grads, vels, n, lr, momentum, weight_decay,
                                      max_grad_norm, norm_out, s),
                s);
}
