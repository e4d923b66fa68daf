// gemm_skinny.cu -- exact-fp32 GEMM for skinny shapes, min(M, N) <= 64:
// one small dimension, so the product streams the big operand from HBM once
// and does little arithmetic per byte (M = 1: 0.5 FLOP/B).  The reference's
// only matmul benchmark shape, (128,512)x(512,10)
// (moonxi-net-gpu/bench/gpu_bench/kernel_bench_wbtest.mbt:231-236), and the
// small-batch Linear layers are of this kind; cuda_matmul
// (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499) runs them through cuBLAS.
//
// Orientation: the kernel computes C[m][n] for m < Ms <= 64 (the small
// dimension) and any n, with every operand addressed through strides, so
// C = A B with a small N runs as C^T = B^T A^T (strides swapped, the bias
// along rows).  The big operand ("B": K x Ns) is what the kernel streams.
//
// Block: 256 threads, a tile of NT columns, a split of K.  K is consumed in
// 32-deep stages through a cp.async ring, coalesced along whichever
// dimension of the streamed operand is contiguous in memory: 16-byte copies
// when its rows are 16-byte aligned (n-contiguous: stage [k][n], warp w
// multiplies stage rows 4w..4w+3 into MT x CPT register accumulators and the
// eight warps' sums are added in a fixed order in shared memory;
// k-contiguous: stage [n][k], each thread owns one column over the whole
// stage), 4-byte copies with zero fill otherwise (any layout, any
// alignment).  A stages are stored [k][m] and read as broadcast float4s;
// FFMA, exact fp32.  Splits of K meet through [split][Ms][Ns] partials and an
// arrival counter per column tile; the last split to arrive adds the splits
// in order and applies the epilogue (alpha, beta, bias, ReLU).  Deterministic.
#include <algorithm>

#include "mx_internal.h"
#include "mx_ptx.cuh"

namespace mx {
namespace {

constexpr int kSkThreads = 256;
constexpr int kSkKT = 32;       // k per stage
constexpr int kSkMaxM = 64;     // largest small dimension

// How a stage of the streamed operand is copied and laid out:
//   kSkScalar: 4-byte cp.async with zero fill, any layout and alignment;
//              stage [k][n] (rows of NT + 1 floats); warps split k.
//   kSkNVec:   16-byte copies along n (n-contiguous, 16-byte aligned rows);
//              stage [k][n] (rows of NT + 4 floats); warps split k.
//   kSkKVec:   16-byte copies along k (k-contiguous, 16-byte aligned rows);
//              stage [n][k] (rows of 36 floats); every thread owns one
//              column n and runs the whole stage's k for it.
enum { kSkScalar = 0, kSkNVec = 1, kSkKVec = 2 };

struct SkinnyParams {
  const float* a;   // A(m, k) = a[m * sam + k * sak]
  const float* b;   // B(k, n) = b[k * sbk + n * sbn]
  float* c;         // C(m, n) = c[m * scm + n * scn]
  int64_t sam, sak, sbk, sbn, scm, scn;
  int M, N, K;
  float alpha, beta;
  const float* bias;
  int bias_rows;    // 1: bias indexed by m (the transposed orientation)
  int relu;
  int k_per_split;  // multiple of kSkKT
  int splits;
  float* partial;   // [splits][M][N] when splits > 1
  int* cnt;         // [column tiles] arrival counters, zero at launch
};

template <int MT, int CPT, int MODE>
struct SkShape {
  static constexpr int NT = MODE == kSkKVec ? kSkThreads : 32 * CPT;
  static constexpr int kStages = MODE == kSkKVec ? 3 : 4;
  static constexpr int kBRow = MODE == kSkKVec ? kSkKT + 4 : (MODE == kSkNVec ? NT + 4 : NT + 1);
  static constexpr int kBStage = (MODE == kSkKVec ? NT : kSkKT) * kBRow;
  static constexpr int kAStage = kSkKT * MT;
  static constexpr int kStage = kBStage + kAStage;
  static constexpr int kRingFloats = kStages * kStage;
  static constexpr int kRedFloats = MODE == kSkKVec ? 0 : 8 * MT * NT;  // eight warps' sums
  static constexpr int kSmemBytes =
      4 * (kRingFloats > kRedFloats ? kRingFloats : kRedFloats) + 16;
};

__device__ __forceinline__ float epilogue(const SkinnyParams& p, float acc, int m, int n) {
  float v = p.alpha * acc;
  const int64_t off = static_cast<int64_t>(m) * p.scm + static_cast<int64_t>(n) * p.scn;
  if (p.beta != 0.0f) v = v + p.beta * p.c[off];
  if (p.bias) v = v + __ldg(p.bias + (p.bias_rows ? m : n));
  if (p.relu) v = v > 0.0f ? v : 0.0f;
  return v;
}

__device__ __forceinline__ void cp_async_16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}

template <int MT, int CPT, int MODE>
__global__ void __launch_bounds__(kSkThreads) skinny_kernel(const SkinnyParams p) {
  using S = SkShape<MT, CPT, MODE>;
  constexpr int NT = S::NT, ST = S::kStages;
  extern __shared__ __align__(16) float sm[];
  __shared__ int last;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int n0 = blockIdx.x * NT;
  const int split = blockIdx.y;
  const int k_begin = split * p.k_per_split;
  const int k_end = min(p.K, k_begin + p.k_per_split);
  const int nstages = (k_end - k_begin + kSkKT - 1) / kSkKT;
  const bool a_kcontig = p.sak == 1;

  // one stage: B[k0 .. k0+32) x [n0 .. n0+NT) and A[0 .. MT) x [k0 .. k0+32)
  auto issue = [&](int st) {
    float* bs = sm + (st % ST) * S::kStage;
    float* as = bs + S::kBStage;
    const int k0 = k_begin + st * kSkKT;
    if (MODE == kSkScalar) {
      const bool b_ncontig = p.sbn == 1;
#pragma unroll 4
      for (int e = tid; e < kSkKT * NT; e += kSkThreads) {
        const int kk = b_ncontig ? e / NT : e % kSkKT;
        const int nn = b_ncontig ? e % NT : e / kSkKT;
        const int k = k0 + kk, n = n0 + nn;
        const bool in = k < k_end && n < p.N;
        const float* src =
            in ? p.b + static_cast<int64_t>(k) * p.sbk + static_cast<int64_t>(n) * p.sbn : p.b;
        cp_async_4(bs + kk * S::kBRow + nn, src, in ? 4u : 0u);
      }
    } else if (MODE == kSkNVec) {  // quads of n; a row of the stage is NT/4 quads
#pragma unroll 4
      for (int e = tid; e < kSkKT * NT / 4; e += kSkThreads) {
        const int kk = e / (NT / 4), nn = (e % (NT / 4)) * 4;
        const int k = k0 + kk, n = n0 + nn;
        const int cnt = k < k_end ? max(0, min(4, p.N - n)) : 0;
        const float* src = cnt ? p.b + static_cast<int64_t>(k) * p.sbk + n : p.b;
        cp_async_16(bs + kk * S::kBRow + nn, src, 4u * cnt);
      }
    } else {  // quads of k; a row of the stage is one column n (8 quads)
#pragma unroll 4
      for (int e = tid; e < NT * kSkKT / 4; e += kSkThreads) {
        const int nn = e / (kSkKT / 4), kk = (e % (kSkKT / 4)) * 4;
        const int k = k0 + kk, n = n0 + nn;
        const int cnt = n < p.N ? max(0, min(4, k_end - k)) : 0;
        const float* src = cnt ? p.b + static_cast<int64_t>(n) * p.sbn + k : p.b;
        cp_async_16(bs + nn * S::kBRow + kk, src, 4u * cnt);
      }
    }
#pragma unroll 2
    for (int e = tid; e < kSkKT * MT; e += kSkThreads) {
      const int kk = a_kcontig ? e % kSkKT : e / MT;
      const int m = a_kcontig ? e / kSkKT : e % MT;
      const int k = k0 + kk;
      const bool in = k < k_end && m < p.M;
      const float* src =
          in ? p.a + static_cast<int64_t>(m) * p.sam + static_cast<int64_t>(k) * p.sak : p.a;
      cp_async_4(as + kk * MT + m, src, in ? 4u : 0u);
    }
  };

  float acc[MT][CPT];
#pragma unroll
  for (int m = 0; m < MT; ++m)
#pragma unroll
    for (int j = 0; j < CPT; ++j) acc[m][j] = 0.0f;

#pragma unroll 1
  for (int st = 0; st < ST - 1; ++st) {
    if (st < nstages) issue(st);
    cp_async_commit();
  }
#pragma unroll 1
  for (int st = 0; st < nstages; ++st) {
    cp_async_wait<ST - 2>();
    __syncthreads();  // stage st landed for everyone; stage st-1 is free again
    if (st + ST - 1 < nstages) issue(st + ST - 1);
    cp_async_commit();
    const float* bs = sm + (st % ST) * S::kStage;
    const float* as = bs + S::kBStage;
    if (MODE == kSkKVec) {
      // my column's 32 k of this stage, then all MT rows of A against it
      const float4* row = reinterpret_cast<const float4*>(bs + tid * S::kBRow);
#pragma unroll
      for (int q = 0; q < kSkKT / 4; ++q) {
        const float4 b4 = row[q];
        const float bq[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
        for (int t = 0; t < 4; ++t) {
          const float4* a4 = reinterpret_cast<const float4*>(as + (4 * q + t) * MT);
#pragma unroll
          for (int m4 = 0; m4 < MT / 4; ++m4) {
            const float4 av = a4[m4];
            acc[4 * m4 + 0][0] = fmaf(av.x, bq[t], acc[4 * m4 + 0][0]);
            acc[4 * m4 + 1][0] = fmaf(av.y, bq[t], acc[4 * m4 + 1][0]);
            acc[4 * m4 + 2][0] = fmaf(av.z, bq[t], acc[4 * m4 + 2][0]);
            acc[4 * m4 + 3][0] = fmaf(av.w, bq[t], acc[4 * m4 + 3][0]);
          }
        }
      }
    } else {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const int kk = warp * 4 + q;
        float bv[CPT];
#pragma unroll
        for (int j = 0; j < CPT; ++j) bv[j] = bs[kk * S::kBRow + lane + 32 * j];
        const float4* a4 = reinterpret_cast<const float4*>(as + kk * MT);
#pragma unroll
        for (int m4 = 0; m4 < MT / 4; ++m4) {
          const float4 av = a4[m4];
#pragma unroll
          for (int j = 0; j < CPT; ++j) {
            acc[4 * m4 + 0][j] = fmaf(av.x, bv[j], acc[4 * m4 + 0][j]);
            acc[4 * m4 + 1][j] = fmaf(av.y, bv[j], acc[4 * m4 + 1][j]);
            acc[4 * m4 + 2][j] = fmaf(av.z, bv[j], acc[4 * m4 + 2][j]);
            acc[4 * m4 + 3][j] = fmaf(av.w, bv[j], acc[4 * m4 + 3][j]);
          }
        }
      }
    }
  }
  cp_async_wait<0>();
  __syncthreads();  // the ring is free: reuse it for the warps' sums

  const bool direct = p.splits == 1;
  auto emit = [&](int m, int nl, float v) {
    const int n = n0 + nl;
    if (m >= p.M || n >= p.N) return;
    if (direct)
      p.c[static_cast<int64_t>(m) * p.scm + static_cast<int64_t>(n) * p.scn] =
          epilogue(p, v, m, n);
    else
      p.partial[(static_cast<int64_t>(split) * p.M + m) * p.N + n] = v;
  };
  if (MODE == kSkKVec) {
#pragma unroll
    for (int m = 0; m < MT; ++m) emit(m, tid, acc[m][0]);
  } else {
    // red[w][m][nl]: each warp's accumulators, then a fixed-order sum
    float* red = sm;
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int j = 0; j < CPT; ++j) red[(warp * MT + m) * NT + lane + 32 * j] = acc[m][j];
    __syncthreads();
    for (int o = tid; o < MT * NT; o += kSkThreads) {
      const int m = o / NT, nl = o % NT;
      float v = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) v += red[(w * MT + m) * NT + nl];
      emit(m, nl, v);
    }
  }
  if (direct) return;
  // the last split of this column tile to arrive adds the splits in order
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int old = atomicAdd(&p.cnt[blockIdx.x], 1);
    last = old == p.splits - 1;
    if (last) p.cnt[blockIdx.x] = 0;  // ready for the next launch
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  // four outputs at a time, four splits' partials of each loaded before any
  // is added (16 loads in flight a thread); splits added in order
  const int64_t stride = static_cast<int64_t>(p.M) * p.N;
  for (int o0 = tid; o0 < MT * NT; o0 += 4 * kSkThreads) {
    int mm[4], nn[4];
    bool ok[4];
    float sum[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int o = o0 + i * kSkThreads;
      mm[i] = o / NT;
      nn[i] = n0 + o % NT;
      ok[i] = o < MT * NT && mm[i] < p.M && nn[i] < p.N;
      sum[i] = 0.0f;
    }
    for (int sp0 = 0; sp0 < p.splits; sp0 += 4) {
      float v[4][4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int u = 0; u < 4; ++u)
          v[i][u] = (ok[i] && sp0 + u < p.splits)
                        ? __ldcg(p.partial + (sp0 + u) * stride +
                                 static_cast<int64_t>(mm[i]) * p.N + nn[i])
                        : 0.0f;
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int u = 0; u < 4; ++u) sum[i] += v[i][u];
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (ok[i])
        p.c[static_cast<int64_t>(mm[i]) * p.scm + static_cast<int64_t>(nn[i]) * p.scn] =
            epilogue(p, sum[i], mm[i], nn[i]);
  }
}

template <int MT, int CPT, int MODE>
cudaError_t launch_skinny(const SkinnyParams& p, dim3 grid, cudaStream_t s) {
  auto kern = skinny_kernel<MT, CPT, MODE>;
  constexpr int smem = SkShape<MT, CPT, MODE>::kSmemBytes;
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(kern, smem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kSkThreads, smem, s>>>(p);
  note_launches(1);
  return cudaGetLastError();
}

// Accumulator rows of the instance serving a small dimension of `ms`, and
// columns per thread (MT x CPT registers of accumulators, at most 128).
void pick_shape(int ms, int* mt, int* cpt) {
  if (ms <= 4) { *mt = 4; *cpt = 4; }
  else if (ms <= 8) { *mt = 8; *cpt = 4; }
  else if (ms <= 16) { *mt = 16; *cpt = 4; }
  else if (ms <= 24) { *mt = 24; *cpt = 2; }
  else if (ms <= 32) { *mt = 32; *cpt = 2; }
  else if (ms <= 48) { *mt = 48; *cpt = 2; }
  else { *mt = 64; *cpt = 2; }
}

struct SkinnyPlan {
  SkinnyParams p;
  dim3 grid;
  int mt, cpt, mode;
  size_t scratch_bytes;  // partials + counters (0: one split)
};

bool aligned16(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

size_t a256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

SkinnyPlan plan(const Context* ctx, const GemmArgs& g) {
  SkinnyPlan pl{};
  SkinnyParams& p = pl.p;
  // logical strides of the caller's problem
  const int64_t am = g.ta ? 1 : g.lda, ak = g.ta ? g.lda : 1;   // A(m, k)
  const int64_t bk = g.tb ? 1 : g.ldb, bn = g.tb ? g.ldb : 1;   // B(k, n)
  if (g.M <= g.N) {  // small M: stream B
    p.a = g.a; p.sam = am; p.sak = ak;
    p.b = g.b; p.sbk = bk; p.sbn = bn;
    p.scm = g.ldc; p.scn = 1;
    p.M = g.M; p.N = g.N; p.bias_rows = 0;
  } else {           // small N: C^T = B^T A^T, stream A
    p.a = g.b; p.sam = bn; p.sak = bk;
    p.b = g.a; p.sbk = ak; p.sbn = am;
    p.scm = 1; p.scn = g.ldc;
    p.M = g.N; p.N = g.M; p.bias_rows = 1;
  }
  p.c = g.c;
  p.K = g.K;
  p.alpha = g.alpha; p.beta = g.beta; p.bias = g.bias; p.relu = g.relu;
  pick_shape(p.M, &pl.mt, &pl.cpt);
  // 16-byte copies when the streamed operand's rows allow them
  pl.mode = kSkScalar;
  if (aligned16(p.b) && p.sbn == 1 && p.sbk % 4 == 0) pl.mode = kSkNVec;
  else if (aligned16(p.b) && p.sbk == 1 && p.sbn % 4 == 0) pl.mode = kSkKVec;
  const int nt = pl.mode == kSkKVec ? kSkThreads : 32 * pl.cpt;
  const int tiles = (p.N + nt - 1) / nt;
  // enough blocks for three per SM (bytes in flight: one block keeps three
  // 16 KB stages outstanding), each split at least eight stages deep and at
  // most 16 splits: the last split to arrive reads every split's partial
  const int want = 3 * ctx->num_sms;
  const int max_splits = std::max(1, std::min(16, p.K / (8 * kSkKT)));
  int splits = std::max(1, std::min(max_splits, (want + tiles - 1) / tiles));
  int kps = (p.K + splits - 1) / splits;
  kps = (kps + kSkKT - 1) / kSkKT * kSkKT;
  splits = (p.K + kps - 1) / kps;
  p.k_per_split = kps;
  p.splits = splits;
  pl.grid = dim3(tiles, splits, 1);
  pl.scratch_bytes = splits > 1 ? a256(sizeof(float) * static_cast<size_t>(splits) * p.M * p.N) +
                                      a256(sizeof(int) * tiles)
                                : 0;
  return pl;
}

template <int MODE>
cudaError_t dispatch_mt(const SkinnyPlan& pl, cudaStream_t s) {
  // kSkKVec keeps one column a thread: CPT is 1 there
  constexpr bool kv = MODE == kSkKVec;
  switch (pl.mt) {
    case 4: return launch_skinny<4, kv ? 1 : 4, MODE>(pl.p, pl.grid, s);
    case 8: return launch_skinny<8, kv ? 1 : 4, MODE>(pl.p, pl.grid, s);
    case 16: return launch_skinny<16, kv ? 1 : 4, MODE>(pl.p, pl.grid, s);
    case 24: return launch_skinny<24, kv ? 1 : 2, MODE>(pl.p, pl.grid, s);
    case 32: return launch_skinny<32, kv ? 1 : 2, MODE>(pl.p, pl.grid, s);
    case 48: return launch_skinny<48, kv ? 1 : 2, MODE>(pl.p, pl.grid, s);
    default: return launch_skinny<64, kv ? 1 : 2, MODE>(pl.p, pl.grid, s);
  }
}

}  // namespace

bool skinny_applies(const GemmArgs& g) {
  return !g.strict && g.K >= 1 && g.M >= 1 && g.N >= 1 && std::min(g.M, g.N) <= kSkMaxM &&
         g.K < (1 << 30);
}

size_t skinny_scratch_bytes(const Context* ctx, const GemmArgs& g) {
  return plan(ctx, g).scratch_bytes;
}

int skinny_gemm(Context* ctx, const GemmArgs& g, cudaStream_t s, void* scratch,
                size_t scratch_bytes) {
  SkinnyPlan pl = plan(ctx, g);
  if (pl.grid.y > 65535) return kErrUnsupported;
  if (pl.p.splits > 1) {
    if (!scratch || scratch_bytes < pl.scratch_bytes) return kErrNoMem;
    pl.p.partial = static_cast<float*>(scratch);
    if (ctx->counters && pl.grid.x <= static_cast<unsigned>(Context::kCounters)) {
      pl.p.cnt = ctx->counters;  // zero, and left zero by every launch
    } else {
      pl.p.cnt = reinterpret_cast<int*>(
          static_cast<uint8_t*>(scratch) +
          a256(sizeof(float) * static_cast<size_t>(pl.p.splits) * pl.p.M * pl.p.N));
      cudaError_t me = cudaMemsetAsync(pl.p.cnt, 0, sizeof(int) * pl.grid.x, s);
      if (me != cudaSuccess) return cuda_status(me);
    }
  }
  cudaError_t e;
  switch (pl.mode) {
    case kSkNVec: e = dispatch_mt<kSkNVec>(pl, s); break;
    case kSkKVec: e = dispatch_mt<kSkKVec>(pl, s); break;
    default: e = dispatch_mt<kSkScalar>(pl, s); break;
  }
  return e == cudaSuccess ? kOk : cuda_status(e);
}

}  // namespace mx
