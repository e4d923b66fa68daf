// gemm_simt.cu -- exact-fp32 SIMT GEMM for sm_100a (FFMA on the CUDA cores).
//
// Replaces the true-FP32 cublasGemmEx call of the reference's cuda_matmul
// (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499, CUBLAS_COMPUTE_32F).
//
// Tile: 128 x 128 outputs per CTA, k-blocks of 16, 256 threads, 8 x 8 outputs
// per thread, 4-stage shared-memory pipeline, two CTAs resident per SM
// (<= 128 registers a thread, ~97 KB shared memory a CTA) so one CTA's
// barrier is covered by the other's multiply-adds.
//
// The inner loop reads, for every k, the thread's 8 A values and 8 B values
// as four 16-byte shared loads from MN-major [16 k][128] tiles, then issues
// 32 packed fma.rn.f32x2 (64 multiply-adds).  Operand tiles arrive in the
// layout their global storage gives, so no transpose is ever materialised in
// global memory:
//   * MN-contiguous operand (A with ta=1, B with tb=0): the TMA box {128, 16}
//     lands as [16 k][128 mn] (512-byte rows) and is read in place.
//   * K-contiguous operand (A with ta=0, B with tb=1): the TMA box {16, 128}
//     lands as [128 rows][16 k] with 64-byte rows and the SWIZZLE_64B pattern
//     (16-byte chunk c of row r stored at chunk c ^ ((r >> 1) & 3)); all
//     threads then transpose it once into a double-buffered [16][128] tile:
//     two 16-byte loads and eight 4-byte stores per thread per k-block, both
//     bank-conflict free.
//
// Feeding: TMA (cp.async.bulk.tensor, mbarrier completion, no multicast)
// when base pointers and row strides are 16-byte aligned; otherwise 4-byte
// cp.async with zero fill into the same layouts (any stride, any edge).
// Out-of-range rows/columns and the K tail read as zeros either way, so edges
// need no special path.
//
// Split-K (for grids smaller than the SM count) writes fp32 partials to a
// scratch buffer; a second kernel sums them in split order (deterministic)
// and applies the epilogue.  Epilogue: v = alpha*acc (+ beta*C) (+ bias[col])
// then ReLU -- the NpArray order matmul -> add -> relu; 16-byte stores when
// C's columns allow.
#include <algorithm>
#include <cstdio>

#include "mx_internal.h"
#include "mx_ptx.cuh"

namespace mx {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 16, kStages = 4, kThreads = 256;
constexpr int kTileFloats = kBM * kBK;                   // 2048 floats = 8 KB
constexpr int kStageBytes = 2 * kTileFloats * 4;         // A + B = 16 KB
// Landing stages, two transposed buffers per operand, 1 KB alignment slack
// and the barriers: ~97 KB, so two CTAs fit in an SM's 228 KB.
constexpr int kSmemBytes = kStages * kStageBytes + 4 * kTileFloats * 4 + 1024 + 256;

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
  int vec_c;       // C (and bias) allow 16-byte column groups
  uint64_t timeout_ns;
};

// Offset (floats) of element (row, k) inside a K-contiguous [128][16] tile
// with the TMA SWIZZLE_64B pattern.
__device__ __forceinline__ int kc_off(int row, int k) {
  return row * 16 + ((((k >> 2) ^ ((row >> 1) & 3))) << 2) + (k & 3);
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
      r = idx >> 4;
      k = idx & 15;
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

// Swizzled [128][16] tile -> MN-major [16][128].  Thread t moves row t & 127,
// 16-byte chunks 2*(t >> 7) and 2*(t >> 7) + 1.  Eight consecutive rows hit
// eight distinct bank groups on the load (the swizzle), and 32 consecutive
// rows 32 distinct banks on the stores.
__device__ __forceinline__ void transpose_tile(const float* __restrict__ src,
                                               float* __restrict__ dst, int tid) {
  const int r = tid & 127;
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    const int kq = 2 * (tid >> 7) + h;
    const float4 v =
        *reinterpret_cast<const float4*>(src + r * 16 + ((kq ^ ((r >> 1) & 3)) << 2));
    dst[(4 * kq + 0) * 128 + r] = v.x;
    dst[(4 * kq + 1) * 128 + r] = v.y;
    dst[(4 * kq + 2) * 128 + r] = v.z;
    dst[(4 * kq + 3) * 128 + r] = v.w;
  }
}

// Index of the thread's i-th row (or column) inside the 128-wide tile.
__device__ __forceinline__ int own_index(int t, int i) {
  return (i < 4) ? t * 4 + i : 64 + t * 4 + (i - 4);
}

// Fast path: accumulator pairs (acc[i][2q], acc[i][2q+1]) live in 64-bit
// register pairs and take one fma.rn.f32x2 (sm_100) per two outputs, with
// a[i] duplicated into both halves: per lane the same round-to-nearest fused
// multiply-add, k ascending, in half the issue slots of scalar FFMA, which
// leaves room for the shared loads beside a saturated FP32 pipe.
struct PackedAcc {
  unsigned long long v[8][4];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int q = 0; q < 4; ++q) v[i][q] = 0ull;
  }
  __device__ __forceinline__ float at(int i, int j) const {
    float lo, hi;
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v[i][j >> 1]));
    return (j & 1) ? hi : lo;
  }
  __device__ __forceinline__ void stage(const float* __restrict__ sA,
                                        const float* __restrict__ sB, int ty, int tx) {
#pragma unroll
    for (int k = 0; k < kBK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(sA + k * 128 + ty * 4);
      const float4 a1 = *reinterpret_cast<const float4*>(sA + k * 128 + 64 + ty * 4);
      const ulonglong2 b0 = *reinterpret_cast<const ulonglong2*>(sB + k * 128 + tx * 4);
      const ulonglong2 b1 = *reinterpret_cast<const ulonglong2*>(sB + k * 128 + 64 + tx * 4);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const unsigned long long b[4] = {b0.x, b0.y, b1.x, b1.y};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        unsigned long long ai;
        asm("mov.b64 %0, {%1, %1};" : "=l"(ai) : "f"(a[i]));
#pragma unroll
        for (int q = 0; q < 4; ++q)
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(v[i][q]) : "l"(ai), "l"(b[q]));
      }
    }
  }
};

// STRICT (NpArray) path: every output is the NpArray sum -- fp32 product
// rounded, then added, k ascending (nparray/trait_impl.mbt:236-241) -- so the
// result is bit-identical to the CPU path (half the FFMA rate).
struct StrictAcc {
  float v[8][8];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.0f;
  }
  __device__ __forceinline__ float at(int i, int j) const { return v[i][j]; }
  __device__ __forceinline__ void stage(const float* __restrict__ sA,
                                        const float* __restrict__ sB, int ty, int tx) {
#pragma unroll
    for (int k = 0; k < kBK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(sA + k * 128 + ty * 4);
      const float4 a1 = *reinterpret_cast<const float4*>(sA + k * 128 + 64 + ty * 4);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const float4 b0 = *reinterpret_cast<const float4*>(sB + k * 128 + tx * 4);
      const float4 b1 = *reinterpret_cast<const float4*>(sB + k * 128 + 64 + tx * 4);
      const float b[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) v[i][j] = __fadd_rn(v[i][j], __fmul_rn(a[i], b[j]));
    }
  }
};

template <bool STRICT>
struct AccFor { using type = PackedAcc; };
template <>
struct AccFor<true> { using type = StrictAcc; };

__device__ __forceinline__ float epi(const SimtParams& p, float acc, float cv, float bv) {
  float v = p.alpha * acc;
  if (p.beta != 0.0f) v = v + p.beta * cv;
  if (p.bias) v = v + bv;
  if (p.relu) v = v > 0.0f ? v : 0.0f;
  return v;
}

template <bool AK, bool BKC, bool TMA, bool STRICT>
__global__ void __launch_bounds__(kThreads, 2)
    simt_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const SimtParams p) {
  extern __shared__ uint8_t smem_raw[];
  float* smem = reinterpret_cast<float*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  float* tA = smem + kStages * 2 * kTileFloats;  // [2][16][128] transposed A (AK only)
  float* tB = tA + 2 * kTileFloats;              // [2][16][128] transposed B (BKC only)
  uint64_t* full = reinterpret_cast<uint64_t*>(tB + 2 * kTileFloats);
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

  typename AccFor<STRICT>::type acc;
  acc.zero();

  // Operand tiles of k-block `it` once it has landed (and been transposed).
  auto tile_a = [&](int it) -> const float* {
    return AK ? tA + (it & 1) * kTileFloats : smem + (it % kStages) * 2 * kTileFloats;
  };
  auto tile_b = [&](int it) -> const float* {
    return BKC ? tB + (it & 1) * kTileFloats
               : smem + (it % kStages) * 2 * kTileFloats + kTileFloats;
  };
  auto transpose_stage = [&](int it) {
    const float* st = smem + (it % kStages) * 2 * kTileFloats;
    if (AK) transpose_tile(st, tA + (it & 1) * kTileFloats, tid);
    if (BKC) transpose_tile(st + kTileFloats, tB + (it & 1) * kTileFloats, tid);
  };
  auto compute = [&](int it) { acc.stage(tile_a(it), tile_b(it), ty, tx); };

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
      if (ok && (AK || BKC)) transpose_stage(it);
      // After this barrier every thread has finished k-block it-1 (so its
      // stage and the transposed buffer of it-2 are free) and the transposed
      // tiles of k-block it are complete.
      if (__syncthreads_or(!ok)) { aborted = true; break; }
      if (tid == 0 && it >= 1 && it - 1 + kStages < nkb) issue(it - 1 + kStages);
      compute(it);
    }
    if (aborted && tid == 0) {
      // Let every load this CTA issued land before the CTA exits (bounded).
      const int issued_end = min(nkb, max(it - 1, 0) + kStages);
      for (int j = it; j < issued_end; ++j) {
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
      __syncthreads();  // k-block it visible to all; everyone is done with it-1
      const int nx = it + kStages - 1;
      if (nx < nkb) {
        float* sA = smem + (nx % kStages) * 2 * kTileFloats;
        const int k0 = (kb_begin + nx) * kBK;
        load_tile_async<AK>(sA, p.a, p.lda, m0, k0, p.M, p.K, tid);
        load_tile_async<BKC>(sA + kTileFloats, p.b, p.ldb, n0, k0, p.N, p.K, tid);
      }
      cp_async_commit();
      if (AK || BKC) {
        transpose_stage(it);
        __syncthreads();
      }
      compute(it);
    }
    cp_async_wait<0>();
  }
  if (aborted) return;

  // ---------------------------------------------------------------- epilogue
  if (p.splits > 1) {
    float* out = p.partial + static_cast<int64_t>(z) * p.M * p.N;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = m0 + own_index(ty, i);
      if (row >= p.M) continue;
      float* orow = out + static_cast<int64_t>(row) * p.N;
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int col = n0 + h * 64 + tx * 4;
        if (p.vec_c && col < p.N) {
          *reinterpret_cast<float4*>(orow + col) = make_float4(
              acc.at(i, 4 * h), acc.at(i, 4 * h + 1), acc.at(i, 4 * h + 2), acc.at(i, 4 * h + 3));
        } else {
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (col + j < p.N) orow[col + j] = acc.at(i, 4 * h + j);
        }
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int row = m0 + own_index(ty, i);
    if (row >= p.M) continue;
    float* crow = p.c + static_cast<int64_t>(row) * p.ldc;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int col = n0 + h * 64 + tx * 4;
      if (p.vec_c && col < p.N) {
        float4 cv = make_float4(0.f, 0.f, 0.f, 0.f), bv = cv;
        if (p.beta != 0.0f) cv = *reinterpret_cast<const float4*>(crow + col);
        if (p.bias) bv = __ldg(reinterpret_cast<const float4*>(p.bias + col));
        float4 o;
        o.x = epi(p, acc.at(i, 4 * h + 0), cv.x, bv.x);
        o.y = epi(p, acc.at(i, 4 * h + 1), cv.y, bv.y);
        o.z = epi(p, acc.at(i, 4 * h + 2), cv.z, bv.z);
        o.w = epi(p, acc.at(i, 4 * h + 3), cv.w, bv.w);
        *reinterpret_cast<float4*>(crow + col) = o;
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int cc = col + j;
          if (cc >= p.N) continue;
          const float cv = p.beta != 0.0f ? crow[cc] : 0.0f;
          const float bv = p.bias ? __ldg(p.bias + cc) : 0.0f;
          crow[cc] = epi(p, acc.at(i, 4 * h + j), cv, bv);
        }
      }
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
  const int slots = 2 * ctx->num_sms;  // two CTAs resident per SM
  int sp = 1;
  if (tiles < slots && num_kb >= 16) {
    sp = std::min({slots / std::max(tiles, 1), num_kb / 8, 32});
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
  // 16-byte column groups: N a multiple of 4, C rows and bias 16-byte aligned
  // (split-K partials are dense [M][N] in 256-byte aligned scratch).
  p.vec_c = (g.N % 4 == 0) &&
            (p.splits > 1 || (aligned16(g.c) && g.ldc % 4 == 0 &&
                              (g.bias == nullptr || aligned16(g.bias))));
  const bool ak = (g.ta == 0), bkc = (g.tb != 0);
  // TMA needs 16-byte aligned bases and row strides.
  const bool tma = aligned16(g.a) && aligned16(g.b) && (g.lda % 4 == 0) && (g.ldb % 4 == 0) &&
                   g.K > 0;
  CUtensorMap ta{}, tb{};
  bool use_tma = tma;
  if (use_tma) {
    // K-contiguous (stored [rows][K]) -> dims {K, rows}, box {16, 128}, 64B swizzle;
    // MN-contiguous (stored [K][rows]) -> dims {rows, K}, box {128, 16}, no swizzle.
    if (ak)
      use_tma &= make_tmap_2d(&ta, g.a, g.K, g.M, g.lda * 4, 16, 128, CU_TENSOR_MAP_SWIZZLE_64B);
    else
      use_tma &= make_tmap_2d(&ta, g.a, g.M, g.K, g.lda * 4, 128, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (bkc)
      use_tma &= make_tmap_2d(&tb, g.b, g.K, g.N, g.ldb * 4, 16, 128, CU_TENSOR_MAP_SWIZZLE_64B);
    else
      use_tma &= make_tmap_2d(&tb, g.b, g.N, g.K, g.ldb * 4, 128, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
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
