// gemm_simt.cu -- exact-fp32 SIMT GEMM for sm_100a (FFMA on the CUDA cores).
//
// Replaces the true-FP32 cublasGemmEx call of the reference's cuda_matmul
// (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499, CUBLAS_COMPUTE_32F).
//
// Two kernels.  Grids whose 128 x 256 tiles fill the SMs' waves run the
// warp-specialised simt_ws_kernel (8 x 16 outputs a thread, described at its
// definition).  Everything else runs simt_gemm_kernel:
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

constexpr int kBM = 128, kBK = 16, kThreads = 256;
constexpr int kTileA = kBM * kBK;  // 2048 floats = 8 KB

// Tile shapes, 128 x BN outputs per CTA:
//   BN = 128: simt_gemm_kernel, 8 x 8 outputs a thread, 4 landing stages,
//             ~97 KB of shared memory and <= 128 registers, two CTAs per SM;
//   BN = 256: simt_ws_kernel's tile, 8 x 16 outputs a thread (its epilogue
//             uses kGroups; its pipeline has its own constants).
template <int BN>
struct Shape {
  static constexpr int kTileB = BN * kBK;
  static constexpr int kStageFloats = kTileA + kTileB;
  static constexpr int kStages = BN == 128 ? 4 : 5;
  static constexpr int kCtasPerSm = BN == 128 ? 2 : 1;
  static constexpr int kGroups = BN / 64;  // 16-byte column groups a thread owns
  // landing stages, two transposed buffers per operand, 1 KB alignment slack
  // and the barriers
  static constexpr int kSmemBytes =
      (kStages * kStageFloats + 2 * (kTileA + kTileB)) * 4 + 1024 + 256;
};

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
  // NpArray bias-first order (STRICT only): the sum starts from bias[col]
  // and the epilogue adds no bias; `pre` (may be null) receives the
  // pre-ReLU values.
  int bias_first;
  float* pre;
};

// Offset (floats) of element (row, k) inside a K-contiguous [rows][16] tile
// with the TMA SWIZZLE_64B pattern.
__device__ __forceinline__ int kc_off(int row, int k) {
  return row * 16 + ((((k >> 2) ^ ((row >> 1) & 3))) << 2) + (k & 3);
}

// Element (i, k) of the operand's logical [rows x K] view.
__device__ __forceinline__ const float* op_ptr(const float* base, int64_t ld, bool kcontig,
                                               int64_t row, int64_t k) {
  return kcontig ? base + row * ld + k : base + k * ld + row;
}

// cp.async loader for one operand tile of ROWS rows (any alignment).
// `rows_total` is M or N.
template <bool KC, int ROWS>
__device__ __forceinline__ void load_tile_async(float* s, const float* g, int64_t ld,
                                                int row0, int k0, int rows_total, int K,
                                                int tid) {
#pragma unroll
  for (int e = 0; e < ROWS * kBK / kThreads; ++e) {
    const int idx = e * kThreads + tid;
    int r, k, so;
    if (KC) {  // consecutive threads walk k (contiguous in global memory)
      r = idx >> 4;
      k = idx & 15;
      so = kc_off(r, k);
    } else {   // consecutive threads walk rows (contiguous in global memory)
      k = idx / ROWS;
      r = idx % ROWS;
      so = k * ROWS + r;
    }
    const int gr = row0 + r, gk = k0 + k;
    const bool in = gr < rows_total && gk < K;
    const float* src = in ? op_ptr(g, ld, KC, gr, gk) : g;
    cp_async_4(s + so, src, in ? 4u : 0u);
  }
}

// Swizzled [ROWS][16] tile -> MN-major [16][ROWS] by NT threads.  Work item
// e*NT + t is row (e*NT + t) % ROWS, 16-byte chunk (e*NT + t) / ROWS.  Eight
// consecutive rows hit eight distinct bank groups on the load (the swizzle),
// and 32 consecutive rows 32 distinct banks on the stores.
template <int ROWS, int NT = kThreads>
__device__ __forceinline__ void transpose_tile(const float* __restrict__ src,
                                               float* __restrict__ dst, int tid) {
#pragma unroll(NT == kThreads ? 4 : 1)
  for (int e = 0; e < ROWS * 4 / NT; ++e) {
    const int idx = e * NT + tid;
    const int r = idx % ROWS, kq = idx / ROWS;
    const float4 v =
        *reinterpret_cast<const float4*>(src + r * 16 + ((kq ^ ((r >> 1) & 3)) << 2));
    dst[(4 * kq + 0) * ROWS + r] = v.x;
    dst[(4 * kq + 1) * ROWS + r] = v.y;
    dst[(4 * kq + 2) * ROWS + r] = v.z;
    dst[(4 * kq + 3) * ROWS + r] = v.w;
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
template <int BN>
struct PackedAcc {
  static constexpr int G = BN / 64;  // column groups of 4 (2 pairs each)
  unsigned long long v[8][2 * G];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int q = 0; q < 2 * G; ++q) v[i][q] = 0ull;
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
      unsigned long long b[2 * G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const ulonglong2 bh =
            *reinterpret_cast<const ulonglong2*>(sB + k * BN + h * 64 + tx * 4);
        b[2 * h] = bh.x;
        b[2 * h + 1] = bh.y;
      }
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        unsigned long long ai;
        asm("mov.b64 %0, {%1, %1};" : "=l"(ai) : "f"(a[i]));
#pragma unroll
        for (int q = 0; q < 2 * G; ++q)
          asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(v[i][q]) : "l"(ai), "l"(b[q]));
      }
    }
  }
};

// STRICT (NpArray) path: every output is the NpArray sum -- fp32 product
// rounded, then added, k ascending (nparray/trait_impl.mbt:236-241) -- so the
// result is bit-identical to the CPU path (half the FFMA rate).
template <int BN>
struct StrictAcc {
  static constexpr int G = BN / 64;
  float v[8][4 * G];
  __device__ __forceinline__ void zero() {
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
      for (int j = 0; j < 4 * G; ++j) v[i][j] = 0.0f;
  }
  // Bias-first order (nparray/fused_ops.mbt:12-78): every sum starts from
  // the bias of its column.
  __device__ __forceinline__ void init_bias(const float* bias, int N, int n0, int tx) {
#pragma unroll
    for (int h = 0; h < G; ++h)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int col = n0 + h * 64 + tx * 4 + j;
        const float b = col < N ? __ldg(bias + col) : 0.0f;
#pragma unroll
        for (int i = 0; i < 8; ++i) v[i][4 * h + j] = b;
      }
  }
  __device__ __forceinline__ float at(int i, int j) const { return v[i][j]; }
  __device__ __forceinline__ void stage(const float* __restrict__ sA,
                                        const float* __restrict__ sB, int ty, int tx) {
#pragma unroll
    for (int k = 0; k < kBK; ++k) {
      const float4 a0 = *reinterpret_cast<const float4*>(sA + k * 128 + ty * 4);
      const float4 a1 = *reinterpret_cast<const float4*>(sA + k * 128 + 64 + ty * 4);
      const float a[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      float b[4 * G];
#pragma unroll
      for (int h = 0; h < G; ++h) {
        const float4 bh = *reinterpret_cast<const float4*>(sB + k * BN + h * 64 + tx * 4);
        b[4 * h] = bh.x; b[4 * h + 1] = bh.y; b[4 * h + 2] = bh.z; b[4 * h + 3] = bh.w;
      }
#pragma unroll
      for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 4 * G; ++j) v[i][j] = __fadd_rn(v[i][j], __fmul_rn(a[i], b[j]));
    }
  }
};

template <int BN, bool STRICT>
struct AccFor { using type = PackedAcc<BN>; };
template <int BN>
struct AccFor<BN, true> { using type = StrictAcc<BN>; };

__device__ __forceinline__ float epi_pre(const SimtParams& p, float acc, float cv, float bv) {
  float v = p.alpha * acc;
  if (p.beta != 0.0f) v = v + p.beta * cv;
  if (p.bias && !p.bias_first) v = v + bv;
  return v;
}
__device__ __forceinline__ float epi(const SimtParams& p, float acc, float cv, float bv) {
  const float v = epi_pre(p, acc, cv, bv);
  return p.relu ? (v > 0.0f ? v : 0.0f) : v;
}

// The thread's 8 x (BN/16) outputs: rows own_index(ty, i), columns
// h*64 + tx*4 + j.  Split-K partials (splits > 1) or the epilogue
// v = alpha*acc (+ beta*C) (+ bias) then ReLU, 16-byte stores where allowed.
template <int BN, class Acc>
__device__ __forceinline__ void store_tile(const SimtParams& p, const Acc& acc, int m0, int n0,
                                           int z, int ty, int tx) {
  using S = Shape<BN>;
  if (p.splits > 1) {
    float* out = p.partial + static_cast<int64_t>(z) * p.M * p.N;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int row = m0 + own_index(ty, i);
      if (row >= p.M) continue;
      float* orow = out + static_cast<int64_t>(row) * p.N;
#pragma unroll
      for (int h = 0; h < S::kGroups; ++h) {
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
    for (int h = 0; h < S::kGroups; ++h) {
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
        if (p.pre) {
          float* prow = p.pre + static_cast<int64_t>(row) * p.ldc;
          *reinterpret_cast<float4*>(prow + col) = make_float4(
              epi_pre(p, acc.at(i, 4 * h + 0), cv.x, bv.x), epi_pre(p, acc.at(i, 4 * h + 1), cv.y, bv.y),
              epi_pre(p, acc.at(i, 4 * h + 2), cv.z, bv.z), epi_pre(p, acc.at(i, 4 * h + 3), cv.w, bv.w));
        }
      } else {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int cc = col + j;
          if (cc >= p.N) continue;
          const float cv = p.beta != 0.0f ? crow[cc] : 0.0f;
          const float bv = p.bias ? __ldg(p.bias + cc) : 0.0f;
          if (p.pre)
            p.pre[static_cast<int64_t>(row) * p.ldc + cc] = epi_pre(p, acc.at(i, 4 * h + j), cv, bv);
          crow[cc] = epi(p, acc.at(i, 4 * h + j), cv, bv);
        }
      }
    }
  }
}

template <int BN, bool AK, bool BKC, bool TMA, bool STRICT>
__global__ void __launch_bounds__(kThreads, Shape<BN>::kCtasPerSm)
    simt_gemm_kernel(const __grid_constant__ CUtensorMap tmA,
                     const __grid_constant__ CUtensorMap tmB, const SimtParams p) {
  using S = Shape<BN>;
  constexpr int kStages = S::kStages, kTileB = S::kTileB, kStageFloats = S::kStageFloats;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array by pointer
  // arithmetic, so the compiler still knows every operand access is a
  // shared-memory one (32-bit addresses, ld.shared; an integer round trip
  // through uintptr_t made them generic 64-bit accesses, and the extra
  // registers spilled in the 168-register consumers)
  float* smem = reinterpret_cast<float*>(
      smem_raw +
      ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u));
  float* tA = smem + kStages * kStageFloats;  // [2][16][128] transposed A (AK only)
  float* tB = tA + 2 * kTileA;                // [2][16][BN] transposed B (BKC only)
  uint64_t* full = reinterpret_cast<uint64_t*>(tB + 2 * kTileB);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(full + kStages);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int ty = (warp >> 1) * 4 + (lane >> 3);  // 0..15
  const int tx = (warp & 1) * 8 + (lane & 7);    // 0..15
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * BN;
  const int z = blockIdx.z;

  const int num_kb = (p.K + kBK - 1) / kBK;
  const int kb_begin = z * p.kb_per_split;
  const int kb_end = min(num_kb, kb_begin + p.kb_per_split);
  const int nkb = max(0, kb_end - kb_begin);

  typename AccFor<BN, STRICT>::type acc;
  acc.zero();
  if constexpr (STRICT) {
    if (p.bias_first) acc.init_bias(p.bias, p.N, n0, tx);
  }

  // Operand tiles of k-block `it` once it has landed (and been transposed).
  auto tile_a = [&](int it) -> const float* {
    return AK ? tA + (it & 1) * kTileA : smem + (it % kStages) * kStageFloats;
  };
  auto tile_b = [&](int it) -> const float* {
    return BKC ? tB + (it & 1) * kTileB : smem + (it % kStages) * kStageFloats + kTileA;
  };
  auto transpose_stage = [&](int it) {
    const float* st = smem + (it % kStages) * kStageFloats;
    if (AK) transpose_tile<kBM>(st, tA + (it & 1) * kTileA, tid);
    if (BKC) transpose_tile<BN>(st + kTileA, tB + (it & 1) * kTileB, tid);
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
      float* sA = smem + s * kStageFloats;
      float* sB = sA + kTileA;
      const int k0 = (kb_begin + it) * kBK;
      bar_arrive_expect_tx(&full[s], kStageFloats * 4);
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
        drain_wait(&full[s], (j / kStages) & 1, p.status, 102);
      }
    }
  } else {
    // Classic multistage cp.async pipeline (always terminates).
#pragma unroll 1
    for (int s = 0; s < kStages - 1; ++s) {
      if (s < nkb) {
        float* sA = smem + s * kStageFloats;
        const int k0 = (kb_begin + s) * kBK;
        load_tile_async<AK, kBM>(sA, p.a, p.lda, m0, k0, p.M, p.K, tid);
        load_tile_async<BKC, BN>(sA + kTileA, p.b, p.ldb, n0, k0, p.N, p.K, tid);
      }
      cp_async_commit();
    }
#pragma unroll 1
    for (int it = 0; it < nkb; ++it) {
      cp_async_wait<kStages - 2>();
      __syncthreads();  // k-block it visible to all; everyone is done with it-1
      const int nx = it + kStages - 1;
      if (nx < nkb) {
        float* sA = smem + (nx % kStages) * kStageFloats;
        const int k0 = (kb_begin + nx) * kBK;
        load_tile_async<AK, kBM>(sA, p.a, p.lda, m0, k0, p.M, p.K, tid);
        load_tile_async<BKC, BN>(sA + kTileA, p.b, p.ldb, n0, k0, p.N, p.K, tid);
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
  store_tile<BN>(p, acc, m0, n0, z, ty, tx);
}

// ---------------------------------------------------------------------------
// Warp-specialised form for large grids: 128 x 256 tile, two consumer
// warpgroups (8 warps) with 8 x 16 outputs a thread (0.75 B of shared memory
// per multiply-add instead of 1 B for 8 x 8), and a producer warpgroup: its
// first thread issues the TMA loads, its four warps transpose K-contiguous
// tiles into MN-major compute tiles.  Registers: launched at 168 a thread (12 warps,
// three per scheduler); the producer warpgroup gives back down to 40 and the
// consumers take 232 (setmaxnreg): 3 x 168 = 40 + 2 x 232 per scheduler.
// There is no CTA-wide barrier in the main loop: per stage, `full` (TMA
// landed), `ready` (compute tiles complete) and `empty` (all 8 consumer warps
// done) mbarriers, every wait bounded.  Producer order per k-block `it`: wait
// for it to land, transpose it, signal ready -- then wait until the
// consumers have finished it-1 and refill that landing stage with k-block
// it-1+S, so a transpose is never on the consumers' critical path.
constexpr int kWsStages = 4;
constexpr int kWsThreads = 384;  // warpgroup 0 produces (warp 0), warpgroups 1-2 consume
constexpr int kWsTileB = 256 * kBK;
constexpr int kWsStageFloats = kTileA + kWsTileB;
// landing stages + one compute-tile set per stage + 1 KB alignment + barriers
constexpr int kWsSmemBytes = 2 * kWsStages * kWsStageFloats * 4 + 1024 + 256;

template <bool AK, bool BKC>
__global__ void __launch_bounds__(kWsThreads, 1)
    simt_ws_kernel(const __grid_constant__ CUtensorMap tmA,
                   const __grid_constant__ CUtensorMap tmB, const SimtParams p) {
  constexpr int S = kWsStages, SF = kWsStageFloats;
  extern __shared__ uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array by pointer
  // arithmetic, so the compiler still knows every operand access is a
  // shared-memory one (32-bit addresses, ld.shared; an integer round trip
  // through uintptr_t made them generic 64-bit accesses, and the extra
  // registers spilled in the 168-register consumers)
  float* smem = reinterpret_cast<float*>(
      smem_raw +
      ((1024u - (static_cast<uint32_t>(__cvta_generic_to_shared(smem_raw)) & 1023u)) & 1023u));
  float* land = smem;            // [S][A 128x16 | B 256x16] as the TMA lands them
  float* tbuf = smem + S * SF;   // [S][A 16x128 | B 16x256] MN-major (K-contiguous operands)
  uint64_t* full = reinterpret_cast<uint64_t*>(tbuf + S * SF);
  uint64_t* ready = full + S;
  uint64_t* empty = ready + S;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(empty + S);

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int m0 = blockIdx.y * kBM, n0 = blockIdx.x * 256;
  const int z = blockIdx.z;
  const int num_kb = (p.K + kBK - 1) / kBK;
  const int kb_begin = z * p.kb_per_split;
  const int nkb = max(0, min(num_kb, kb_begin + p.kb_per_split) - kb_begin);

  if (tid == 0) {
    for (int s = 0; s < S; ++s) {
      bar_init(&full[s], 1);
      bar_init(&ready[s], 4);
      bar_init(&empty[s], 8);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  __syncthreads();

  if (warp < 4) {  // -------------------------------------------- producer
    asm volatile("setmaxnreg.dec.sync.aligned.u32 40;\n" ::: "memory");
    auto issue = [&](int j) {
      const int s = j % S;
      float* sA = land + s * SF;
      float* sB = sA + kTileA;
      const int k0 = (kb_begin + j) * kBK;
      bar_arrive_expect_tx(&full[s], SF * 4);
      if (AK) tma_load_2d(sA, &tmA, &full[s], k0, m0);
      else    tma_load_2d(sA, &tmA, &full[s], m0, k0);
      if (BKC) tma_load_2d(sB, &tmB, &full[s], k0, n0);
      else     tma_load_2d(sB, &tmB, &full[s], n0, k0);
    };
    int issued = min(S, nkb), landed = 0;
    if (tid == 0)
      for (int j = 0; j < issued; ++j) issue(j);
    bool ok = true;
    for (int it = 0; it < nkb && ok; ++it) {
      const int s = it % S;
      ok = __all_sync(0xffffffffu,
                      wait_bar(&full[s], (it / S) & 1, abort_flag, p.status, p.timeout_ns, 111));
      if (!ok) break;
      landed = it + 1;
      // (full for k-block it completes only after warp 0 saw the consumers
      // finish it-S, so this stage's compute tiles are free to overwrite)
      if (AK) transpose_tile<kBM, 128>(land + s * SF, tbuf + s * SF, tid);
      if (BKC) transpose_tile<256, 128>(land + s * SF + kTileA, tbuf + s * SF + kTileA, tid);
      __syncwarp();
      if (lane == 0) bar_arrive(&ready[s]);
      const int j = it - 1 + S;  // warp 0: refill the landing stage of k-block it-1
      if (warp == 0 && it >= 1 && j < nkb) {
        const int sj = j % S;
        ok = __all_sync(0xffffffffu, wait_bar(&empty[sj], ((it - 1) / S) & 1, abort_flag,
                                              p.status, p.timeout_ns, 112));
        if (ok && lane == 0) issue(j);
        if (ok) issued = j + 1;
      }
    }
    if (!ok && tid == 0) {
      // let every load this CTA issued land before the CTA exits (bounded)
      for (int j = landed; j < issued; ++j) {
        drain_wait(&full[j % S], (j / S) & 1, p.status, 115);
      }
    }
    return;
  }

  // ------------------------------------------------------------- consumers
  asm volatile("setmaxnreg.inc.sync.aligned.u32 232;\n" ::: "memory");
  const int cw = warp - 4;                      // consumer warp 0..7
  const int ty = (cw >> 1) * 4 + (lane >> 3);   // 0..15
  const int tx = (cw & 1) * 8 + (lane & 7);     // 0..15
  PackedAcc<256> acc;
  acc.zero();
  for (int it = 0; it < nkb; ++it) {
    const int s = it % S;
    bool ok = wait_bar(&ready[s], (it / S) & 1, abort_flag, p.status, p.timeout_ns, 113);
    // tiles read straight from the landing stage: also observe the TMA's own
    // barrier (its phase completed before `ready`; this is the acquire)
    if (ok && (!AK || !BKC))
      ok = wait_bar(&full[s], (it / S) & 1, abort_flag, p.status, p.timeout_ns, 114);
    if (!__all_sync(0xffffffffu, ok)) return;
    const float* sa = AK ? tbuf + s * SF : land + s * SF;
    const float* sb = BKC ? tbuf + s * SF + kTileA : land + s * SF + kTileA;
    acc.stage(sa, sb, ty, tx);
    __syncwarp();
    if (lane == 0) bar_arrive(&empty[s]);
  }
  store_tile<256>(p, acc, m0, n0, z, ty, tx);
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

template <int BN, bool AK, bool BKC, bool TMA, bool STRICT>
cudaError_t launch_variant(const CUtensorMap& ta, const CUtensorMap& tb, const SimtParams& p,
                           dim3 grid, cudaStream_t s) {
  auto kern = simt_gemm_kernel<BN, AK, BKC, TMA, STRICT>;
  constexpr int kSmemBytes = Shape<BN>::kSmemBytes;
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(kern, kSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, kSmemBytes, s>>>(ta, tb, p);
  note_launches(1);
  return cudaGetLastError();
}

template <int BN, bool TMA, bool STRICT>
cudaError_t dispatch_layout(bool ak, bool bkc, const CUtensorMap& ta, const CUtensorMap& tb,
                            const SimtParams& p, dim3 grid, cudaStream_t s) {
  if (ak && bkc) return launch_variant<BN, true, true, TMA, STRICT>(ta, tb, p, grid, s);
  if (ak) return launch_variant<BN, true, false, TMA, STRICT>(ta, tb, p, grid, s);
  if (bkc) return launch_variant<BN, false, true, TMA, STRICT>(ta, tb, p, grid, s);
  return launch_variant<BN, false, false, TMA, STRICT>(ta, tb, p, grid, s);
}

template <int BN>
cudaError_t dispatch_all(bool strict, bool tma, bool ak, bool bkc, const CUtensorMap& ta,
                         const CUtensorMap& tb, const SimtParams& p, dim3 grid,
                         cudaStream_t s) {
  if (strict)
    return tma ? dispatch_layout<BN, true, true>(ak, bkc, ta, tb, p, grid, s)
               : dispatch_layout<BN, false, true>(ak, bkc, ta, tb, p, grid, s);
  return tma ? dispatch_layout<BN, true, false>(ak, bkc, ta, tb, p, grid, s)
             : dispatch_layout<BN, false, false>(ak, bkc, ta, tb, p, grid, s);
}

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

// TMA needs 16-byte aligned bases and row strides.
bool tma_ok(const GemmArgs& g) {
  return aligned16(g.a) && aligned16(g.b) && (g.lda % 4 == 0) && (g.ldb % 4 == 0) && g.K > 0;
}

template <bool AK, bool BKC>
cudaError_t launch_ws_variant(const CUtensorMap& ta, const CUtensorMap& tb, const SimtParams& p,
                              dim3 grid, cudaStream_t s) {
  auto kern = simt_ws_kernel<AK, BKC>;
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(kern, kWsSmemBytes);
  if (e != cudaSuccess) return e;
  kern<<<grid, kWsThreads, kWsSmemBytes, s>>>(ta, tb, p);
  note_launches(1);
  return cudaGetLastError();
}

cudaError_t launch_ws(bool ak, bool bkc, const CUtensorMap& ta, const CUtensorMap& tb,
                      const SimtParams& p, dim3 grid, cudaStream_t s) {
  if (ak && bkc) return launch_ws_variant<true, true>(ta, tb, p, grid, s);
  if (ak) return launch_ws_variant<true, false>(ta, tb, p, grid, s);
  if (bkc) return launch_ws_variant<false, true>(ta, tb, p, grid, s);
  return launch_ws_variant<false, false>(ta, tb, p, grid, s);
}

// Tile width: 256 (the warp-specialised kernel, one CTA per SM) where TMA can
// feed it and its tiles fill the SMs' waves to at least 94 %; 128 (two CTAs
// per SM) otherwise -- measured on B200, the 256-wide kernel leads by ~5 %
// with full waves, while in a part-filled last wave the lone 128-wide CTA on
// an SM runs faster than it did beside a second one, so it loses less.
int tile_width(const Context* ctx, const GemmArgs& g) {
  if (g.strict || !tma_ok(g)) return 128;
  const int64_t wide_tiles =
      static_cast<int64_t>((g.M + kBM - 1) / kBM) * ((g.N + 255) / 256);
  const int64_t waves = (wide_tiles + ctx->num_sms - 1) / ctx->num_sms;
  return wide_tiles >= ctx->num_sms &&
                 static_cast<double>(wide_tiles) / (waves * ctx->num_sms) >= 0.94
             ? 256
             : 128;
}

void plan_splits(const Context* ctx, const GemmArgs& g, int* splits, int* kb_per_split) {
  if (g.strict) {  // one pass over k in order: no split-K
    *splits = 1;
    *kb_per_split = std::max(1, (g.K + kBK - 1) / kBK);
    return;
  }
  const int bn = tile_width(ctx, g);
  const int tiles = ((g.M + kBM - 1) / kBM) * ((g.N + bn - 1) / bn);
  const int num_kb = (g.K + kBK - 1) / kBK;
  const int slots = (bn == 128 ? 2 : 1) * ctx->num_sms;  // resident CTAs
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
  if (skinny_applies(g)) return skinny_scratch_bytes(ctx, g);
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
  p.bias_first = g.strict && g.bias_first && g.bias;
  p.pre = g.pre;
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
  int bn = tile_width(ctx, g);
  const bool tma = tma_ok(g);
  CUtensorMap ta{}, tb{};
  bool use_tma = tma;
  if (use_tma) {
    // K-contiguous (stored [rows][K]) -> dims {K, rows}, box {16, tile rows}, 64B
    // swizzle; MN-contiguous (stored [K][rows]) -> dims {rows, K}, box {tile rows,
    // 16}, no swizzle.  Tile rows: 128 for A, bn for B.
    if (ak)
      use_tma &= make_tmap_2d(&ta, g.a, g.K, g.M, g.lda * 4, 16, 128, CU_TENSOR_MAP_SWIZZLE_64B);
    else
      use_tma &= make_tmap_2d(&ta, g.a, g.M, g.K, g.lda * 4, 128, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
    if (bkc)
      use_tma &= make_tmap_2d(&tb, g.b, g.K, g.N, g.ldb * 4, 16, bn, CU_TENSOR_MAP_SWIZZLE_64B);
    else
      use_tma &= make_tmap_2d(&tb, g.b, g.N, g.K, g.ldb * 4, bn, 16, CU_TENSOR_MAP_SWIZZLE_NONE);
  }
  if (!use_tma) bn = 128;  // a tensor map was refused: cp.async, 128-wide tiles
  dim3 grid((g.N + bn - 1) / bn, (g.M + kBM - 1) / kBM, p.splits);
  if (grid.y > 65535) return kErrUnsupported;
  cudaError_t e = bn == 256 ? launch_ws(ak, bkc, ta, tb, p, grid, s)
                            : dispatch_all<128>(g.strict, use_tma, ak, bkc, ta, tb, p, grid, s);
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
  if (skinny_applies(g)) return skinny_gemm(ctx, g, s, ctx->workspace, ctx->ws_bytes);
  return simt_gemm_launch(ctx, g, s, static_cast<float*>(ctx->workspace), ctx->ws_bytes);
}

}  // namespace mx
