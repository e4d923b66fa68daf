// gemm_simt.cu -- exact-fp32 SIMT GEMM for sm_100a (FFMA on the CUDA cores).
//
// Replaces the true-FP32 cublasGemmEx call of the reference's cuda_matmul
// (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499, CUBLAS_COMPUTE_32F).
//
// Tile: 128 x 128 outputs per CTA, k-blocks of 32, 256 threads, 8 x 8 outputs
// per thread, 4-stage shared-memory pipeline.
//
// Operand tiles are kept in the layout their global storage gives, so no
// transpose is ever materialised:
//   * K-contiguous operand (A with ta=0, B with tb=1): [128 rows][32 k],
//     128-byte rows, 16-byte chunks XOR-swizzled by (row & 7) -- exactly the
//     TMA SWIZZLE_128B pattern.  A thread owns rows {t + 16 i}.
//   * MN-contiguous operand (A with ta=1, B with tb=0): [32 k][128 mn],
//     unswizzled 512-byte rows.  A thread owns {4t..4t+3, 64+4t..64+4t+3}.
// Both layouts give conflict-free 16-byte shared loads for every warp.
//
// Feeding: TMA (cp.async.bulk.tensor, mbarrier completion, no multicast)
// when base pointers and row strides are 16-byte aligned; otherwise 4-byte
// cp.async with zero fill (any stride, any edge).  Out-of-range rows/columns
// and the K tail read as zeros either way, so edges need no special path.
//
// Split-K (for grids smaller than the SM count) writes fp32 partials to a
// scratch buffer; a second kernel sums them in split order (deterministic)
// and applies the epilogue.  Epilogue: v = alpha*acc (+ beta*C) (+ bias[col])
// then ReLU -- the NpArray order matmul -> add -> relu.
#include <algorithm>
#include <cstdio>

#include "mx_internal.h"
#include "mx_ptx.cuh"

namespace mx {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 32, kStages = 4, kThreads = 256;
constexpr int kTileFloats = kBM * kBK;                   // 4096 floats = 16 KB
constexpr int kStageBytes = 2 * kTileFloats * 4;         // A + B = 32 KB
constexpr int kSmemBytes = kStages * kStageBytes + 1024 + 256;

struct SimtParams {
  const float* a;
  const float* b;
  float* c;
  float* partial;  // split-K scratch [splits][M][N] (splits > 1 only)
  const float* bias;
  int* status;
  int64_t lda, ldb, ldc;
  int M, N, K;
  int kb_per_split, splits;
  float alpha, beta;
  int relu;
  uint64_t timeout_ns;
};

// Offset (floats) of element (row, k) inside a K-contiguous swizzled tile.
__device__ __forceinline__ int kc_off(int row, int k) {
  return row * 32 + ((((k >> 2) ^ (row & 7))) << 2) + (k & 3);
}

// Element (i, k) of the operand's logical [rows x K] view.
__device__ __forceinline__ const float* op_ptr(const float* base, int64_t ld, bool kcontig,
                                               int64_t row, int64_t k) {
  return kcontig ? base + row * ld + k : base + k * ld + row;
}

// cp.async loader for one operand tile (any alignment).  `rows_total` is M or N.
template <bool KC>
__device__ __forceinline__ void load_tile_async(float* s, const float* g, int64_t ld,
                                                int row0, int k0, int rows_total, int K,
                                                int tid) {
#pragma unroll
  for (int e = 0; e < kTileFloats / kThreads; ++e) {
    const int idx = e * kThreads + tid;
    int r, k, so;
    if (KC) {  // consecutive threads walk k (contiguous in global memory)
      r = idx >> 5;
      k = idx & 31;
      so = kc_off(r, k);
    } else {   // consecutive threads walk rows (contiguous in global memory)
      k = idx >> 7;
      r = idx & 127;
      so = k * 128 + r;
    }
    const int gr = row0 + r, gk = k0 + k;
    const bool in = gr < rows_total && gk < K;
    const float* src = in ? op_ptr(g, ld, KC, gr, gk) : g;
    cp_async_4(s + so, src, in ? 4u : 0u);
  }
}

// Index of the thread's i-th row (or column) inside the 128-wide tile.
template <bool KC>
__device__ __forceinline__ int own_index(int t, int i) {
  return KC ? t + 16 * i : ((i < 4) ? t * 4 + i : 64 + t * 4 + (i - 4));
}

// STRICT: every output is the NpArray sum -- fp32 product rounded, then
// added, k ascending (nparray/trait_impl.mbt:236-241) -- so the result is
// bit-identical to the CPU path (half the FFMA rate).  Otherwise fused
// multiply-add, k ascending.
template <bool AK, bool BKC, bool STRICT>
__device__ __forceinline__ void compute_stage(const float* __restrict__ sA,
                                              const float* __restrict__ sB, int ty, int tx,
                                              float (&acc)[8][8]) {
#pragma unroll 2
  for (int kq = 0; kq < kBK / 4; ++kq) {
    float a[8][4], b[8][4];
    if (AK) {
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int r = ty + 16 * i;
        const float4 v = *reinterpret_cast<const float4*>(sA + r * 32 + ((kq ^ (r & 7)) << 2));
        a[i][0] = v.x; a[i][1] = v.y; a[i][2] = v.z; a[i][3] = v.w;
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float* row = sA + (kq * 4 + kk) * 128;
        const float4 v0 = *reinterpret_cast<const float4*>(row + ty * 4);
        const float4 v1 = *reinterpret_cast<const float4*>(row + 64 + ty * 4);
        a[0][kk] = v0.x; a[1][kk] = v0.y; a[2][kk] = v0.z; a[3][kk] = v0.w;
        a[4][kk] = v1.x; a[5][kk] = v1.y; a[6][kk] = v1.z; a[7][kk] = v1.w;
      }
    }
    if (BKC) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = tx + 16 * j;
        const float4 v = *reinterpret_cast<const float4*>(sB + r * 32 + ((kq ^ (r & 7)) << 2));
        b[j][0] = v.x; b[j][1] = v.y; b[j][2] = v.z; b[j][3] = v.w;
      }
    } else {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const float* row = sB + (kq * 4 + kk) * 128;
        const float4 v0 = *reinterpret_cast<const float4*>(row + tx * 4);
        const float4 v1 = *reinterpret_cast<const float4*>(row + 64 + tx * 4);
        b[0][kk] = v0.x; b[1][kk] = v0.y; b[2][kk] = v0.z; b[3][kk] = v0.w;
        b[4][kk] = v1.x; b[5][kk] = v1.y; b[6][kk] = v1.z; b[7][kk] = v1.w;
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk)
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (STRICT) acc[i][j] = __fadd_rn(acc[i][j], __fmul_rn(a[i][kk], b[j][kk]));
          else        acc[i][j] = fmaf(a[i][kk], b[j][kk], acc[i][j]);
        }
  }
}

template <bool AK, bool BKC, bool TMA, bool STRICT>
__global__ void __launch_bounds__(kThreads, 1)
    simt_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const SimtParams p) {
  extern __shared__ uint8_t smem_raw[];
  float* smem = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * 2 * kTileFloats);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + kStages);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ty = (warp >> 1) * 4 + (lane >> 3);  // 0..15
  const int tx = (warp & 1) * 8 + (lane & 7);    // 0..15
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * kBN;
  const int z = blockIdx.z;

  const int num_kb = (p.K + kBK - 1) / kBK;
  const int kb_begin = z * p.kb_per_split;
  const int kb_end = min(num_kb, kb_begin + p.kb_per_split);
  const int nkb = max(0, kb_end - kb_begin);

  float acc[8][8];
#pragma unroll
  for (int i = 0; i < 8; ++i)
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[i][j] = 0.0f;

  bool aborted = false;
  if (TMA) {
    if (tid == 0) {
      for (int s = 0; s < kStages; ++s) bar_init(&full[s], 1);
      *abort_flag = 0;
      fence_barrier_init();
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
    }
    __syncthreads();
    auto issue = [&](int it) {
      const int s = it % kStages;
      float* sA = smem + s * 2 * kTileFloats;
      float* sB = sA + kTileFloats;
      const int k0 = (kb_begin + it) * kBK;
      bar_arrive_expect_tx(&full[s], kStageBytes);
      if (AK) tma_load_2d(sA, &tmA, &full[s], k0, m0);
      else    tma_load_2d(sA, &tmA, &full[s], m0, k0);
      if (BKC) tma_load_2d(sB, &tmB, &full[s], k0, n0);
      else     tma_load_2d(sB, &tmB, &full[s], n0, k0);
    };
    if (tid == 0)
      for (int it = 0; it < min(kStages, nkb); ++it) issue(it);
    int it = 0;
    for (; it < nkb; ++it) {
      const int s = it % kStages;
      const bool ok = wait_bar(&full[s], (it / kStages) & 1, abort_flag, p.status,
                               p.timeout_ns, 101);
      if (ok) compute_stage<AK, BKC, STRICT>(smem + s * 2 * kTileFloats,
                                     smem + s * 2 * kTileFloats + kTileFloats, ty, tx, acc);
      if (__syncthreads_or(!ok)) { aborted = true; break; }
      if (tid == 0 && it + kStages < nkb) issue(it + kStages);
    }
    if (aborted && tid == 0) {
      // Let every load this CTA issued land before the CTA exits (bounded).
      for (int j = it; j < min(nkb, it + kStages); ++j) {
        const int s = j % kStages;
        uint64_t t0 = globaltimer_ns();
        while (!bar_try_wait(&full[s], (j / kStages) & 1) &&
               globaltimer_ns() - t0 < p.timeout_ns) {
        }
      }
    }
  } else {
    // Classic multistage cp.async pipeline (always terminates).
#pragma unroll 1
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < nkb) {
        float* sA = smem + s * 2 * kTileFloats;
        const int k0 = (kb_begin + s) * kBK;
        load_tile_async<AK>(sA, p.a, p.lda, m0, k0, p.M, p.K, tid);
        load_tile_async<BKC>(sA + kTileFloats, p.b, p.ldb, n0, k0, p.N, p.K, tid);
      }
      cp_async_commit();
    }
#pragma unroll 1
    for (int it = 0; it < nkb; ++it) {
      cp_async_wait<kStages - 2>();
      __syncthreads();
      const int nx = it + kStages - 1;
      if (nx < nkb) {
        float* sA = smem + (nx % kStages) * 2 * kTileFloats;
        const int k0 = (kb_begin + nx) * kBK;
        load_tile_async<AK>(sA, p.a, p.lda, m0, k0, p.M, p.K, tid);
        load_tile_async<BKC>(sA + kTileFloats, p.b, p.ldb, n0, k0, p.N, p.K, tid);
      }
      cp_async_commit();
      const int s = it % kStages;
      compute_stage<AK, BKC, STRICT>(smem + s * 2 * kTileFloats,
                             smem + s * 2 * kTileFloats + kTileFloats, ty, tx, acc);
    }
    cp_async_wait<0>();
  }
  if (aborted) return;

  // ---------------------------------------------------------------- epilogue
  if (p.splits > 1) {
    float* out = p.partial + static_cast<int64_t>(z) * p.M * p.N;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = m0 + own_index<AK>(ty, i);
      if (row >= p.M) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int col = n0 + own_index<BKC>(tx, j);
        if (col < p.N) out[static_cast<int64_t>(row) * p.N + col] = acc[i][j];
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = m0 + own_index<AK>(ty, i);
    if (row >= p.M) continue;
    float* crow = p.c + static_cast<int64_t>(row) * p.ldc;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int col = n0 + own_index<BKC>(tx, j);
      if (col >= p.N) continue;
      float v = p.alpha * acc[i][j];
      if (p.beta != 0.0f) v = v + p.beta * crow[col];
      if (p.bias) v = v + __ldg(p.bias + col);
      if (p.relu) v = v > 0.0f ? v : 0.0f;
      crow[col] = v;
    }
  }
}

// Sums split-K partials in split order and applies the epilogue.
__global__ void splitk_reduce_kernel(const float* __restrict__ partial, float* c, int64_t ldc,
                                     int M, int N, int splits, float alpha, float beta,
                                     const float* __restrict__ bias, int relu) {
  const int64_t total = static_cast<int64_t>(M) * N;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float s = 0.0f;
    for (int zz = 0; zz < splits; ++zz) s += partial[zz * total + idx];
    const int row = static_cast<int>(idx / N), col = static_cast<int>(idx % N);
    float* cp = c + row * ldc + col;
    float v = alpha * s;
    if (beta != 0.0f) v = v + beta * *cp;
    if (bias) v = v + bias[col];
    if (relu) v = v > 0.0f ? v : 0.0f;
    *cp = v;
  }
}

template <bool AK, bool BKC, bool TMA, bool STRICT>
cudaError_t launch_variant(const CUtensorMap& ta, const CUtensorMap& tb, const SimtParams& p,
                           dim3 grid, cudaStream_t s) {
  auto kern = simt_gemm_kernel<AK, BKC, TMA, STRICT>;
  static unsigned configured = 0;  // one bit per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (!(configured & (1u << (dev & 31)))) {
    cudaError_t e =
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    if (e != cudaSuccess) return e;
    configured |= 1u << (dev & 31);
  }
  kern<<<grid, kThreads, kSmemBytes, s>>>(ta, tb, p);
  note_launches(1);
  return cudaGetLastError();
}

template <bool TMA, bool STRICT>
cudaError_t dispatch_layout(bool ak, bool bkc, const CUtensorMap& ta, const CUtensorMap& tb,
                            const SimtParams& p, dim3 grid, cudaStream_t s) {
  if (ak && bkc) return launch_variant<true, true, TMA, STRICT>(ta, tb, p, grid, s);
  if (ak) return launch_variant<true, false, TMA, STRICT>(ta, tb, p, grid, s);
  if (bkc) return launch_variant<false, true, TMA, STRICT>(ta, tb, p, grid, s);
  return launch_variant<false, false, TMA, STRICT>(ta, tb, p, grid, s);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

void plan_splits(const Context* ctx, const GemmArgs& g, int* splits, int* kb_per_split) {
  if (g.strict) {  // one pass over k in order: no split-K
    *splits = 1;
    *kb_per_split = std::max(1, (g.K + kBK - 1) / kBK);
    return;
  }
  const int tiles = ((g.M + kBM - 1) / kBM) * ((g.N + kBN - 1) / kBN);
  const int num_kb = (g.K + kBK - 1) / kBK;
  int sp = 1;
  if (tiles < ctx->num_sms && num_kb >= 8) {
    sp = std::min({ctx->num_sms / std::max(tiles, 1), num_kb / 4, 32});
    sp = std::max(sp, 1);
  }
  int kps = (num_kb + sp - 1) / sp;
  sp = (num_kb + kps - 1) / std::max(kps, 1);  // drop empty splits
  *splits = std::max(sp, 1);
  *kb_per_split = std::max(kps, 1);
}

}  // namespace

size_t simt_gemm_scratch_bytes(const Context* ctx, const GemmArgs& g) {
  int sp, kps;
  plan_splits(ctx, g, &sp, &kps);
  return sp > 1 ? static_cast<size_t>(sp) * g.M * g.N * sizeof(float) : 0;
}

int simt_gemm_launch(Context* ctx, const GemmArgs& g, cudaStream_t s, float* scratch,
                     size_t scratch_bytes) {
  if (g.M == 0 || g.N == 0) return kOk;
  SimtParams p{};
  p.a = g.a; p.b = g.b; p.c = g.c; p.bias = g.bias; p.status = ctx->status;
  p.lda = g.lda; p.ldb = g.ldb; p.ldc = g.ldc;
  p.M = g.M; p.N = g.N; p.K = g.K;
  p.alpha = g.alpha; p.beta = g.beta; p.relu = g.relu;
  p.timeout_ns = ctx->timeout_ns;
  plan_splits(ctx, g, &p.splits, &p.kb_per_split);
  if (g.K == 0) { p.splits = 1; p.kb_per_split = 0; }
  if (p.splits > 1) {
    const size_t need = static_cast<size_t>(p.splits) * g.M * g.N * sizeof(float);
    if (scratch == nullptr || scratch_bytes < need) return kErrNoMem;
    p.partial = scratch;
  }
  const bool ak = (g.ta == 0), bkc = (g.tb != 0);
  // TMA needs 16-byte aligned bases and row strides.
  const bool tma = aligned16(g.a) && aligned16(g.b) && (g.lda % 4 == 0) && (g.ldb % 4 == 0) &&
                   g.K > 0;
  CUtensorMap ta{}, tb{};
  bool use_tma = tma;
  if (use_tma) {
    // A: K-contiguous -> dims {K, M}, box {32, 128}, 128B swizzle;
    //    MN-contiguous (stored [K][M]) -> dims {M, K}, box {128, 32}, no swizzle.
    if (ak)
      use_tma &= make_tmap_2d(&ta, g.a, g.K, g.M, g.lda * 4, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    else
      use_tma &= make_tmap_2d(&ta, g.a, g.M, g.K, g.lda * 4, 128, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (bkc)
      use_tma &= make_tmap_2d(&tb, g.b, g.K, g.N, g.ldb * 4, 32, 128, CU_TENSOR_MAP_SWIZZLE_128B);
    else
      use_tma &= make_tmap_2d(&tb, g.b, g.N, g.K, g.ldb * 4, 128, 32, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  dim3 grid((g.N + kBN - 1) / kBN, (g.M + kBM - 1) / kBM, p.splits);
  if (grid.y > 65535) return kErrUnsupported;
  cudaError_t e;
  if (g.strict) {
    if (use_tma) e = dispatch_layout<true, true>(ak, bkc, ta, tb, p, grid, s);
    else         e = dispatch_layout<false, true>(ak, bkc, ta, tb, p, grid, s);
  } else {
    if (use_tma) e = dispatch_layout<true, false>(ak, bkc, ta, tb, p, grid, s);
    else         e = dispatch_layout<false, false>(ak, bkc, ta, tb, p, grid, s);
  }
  if (e != cudaSuccess) return cuda_status(e);
  if (p.splits > 1) {
    const int64_t total = static_cast<int64_t>(g.M) * g.N;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, ctx->num_sms * 8));
    splitk_reduce_kernel<<<blocks, 256, 0, s>>>(p.partial, g.c, g.ldc, g.M, g.N, p.splits,
                                                g.alpha, g.beta, g.bias, g.relu);
    note_launches(1);
    e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_status(e);
  }
  return kOk;
}

int simt_gemm(Context* ctx, const GemmArgs& g, cudaStream_t s) {
  const size_t need = simt_gemm_scratch_bytes(ctx, g);
  if (need > 0) {
    int rc = ensure_workspace(ctx, need);
    if (rc != kOk) return rc;
  }
  return simt_gemm_launch(ctx, g, s, static_cast<float*>(ctx->workspace), ctx->ws_bytes);
}

}  // namespace mx
