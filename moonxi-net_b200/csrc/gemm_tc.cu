// gemm_tc.cu -- tcgen05 / TMEM tensor-core GEMM for sm_100a, fp32-class by
// 3xTF32 splitting (passes = 3) or plain TF32 (passes = 1).
//
// Replaces the cublasGemmEx call of the reference's cuda_matmul
// (moonxi-net-gpu/cuda/cuda_kernels.cu:1464-1499) for large shapes.
//
// Split:  x = hi + lo with hi = rna_tf32(x), lo = rna_tf32(x - hi).  A
// prepass writes hi/lo of each operand in K-major order ([rows][Kp], Kp = K
// rounded up to 4 floats so TMA strides are 16-byte multiples); the prepass
// reads the operand in whatever layout it is stored (ta/tb), so NN/NT/TN all
// reach the tensor cores as K-major tiles.  The product accumulates
//   lo_a*hi_b + hi_a*lo_b + hi_a*hi_b
// per k-step in one fp32 TMEM accumulator (the lo*lo term, below 2^-22
// relative, is dropped).
//
// Main kernel (persistent, one CTA per SM, 192 threads):
//   warp 0     TMA producer: per k-block of 16, loads A_hi, A_lo (128x16) and
//              B_hi, B_lo (256x16) with 64-byte swizzle into a 4-stage ring.
//   warp 1     allocates 512 TMEM columns (two 128x256 fp32 accumulators),
//              one lane issues tcgen05.mma kind::tf32 (M=128, N=256, K=8) and
//              tcgen05.commit to free ring stages / publish accumulators.
//   warps 2-5  epilogue: tcgen05.ld 32 columns at a time, alpha/beta/bias/
//              ReLU, predicated stores.  Two accumulators let the epilogue of
//              tile i overlap the main loop of tile i+1.
// Every mbarrier wait is bounded (mx::wait_bar); a timeout raises a kernel
// abort flag, records kErrTimeout, drains in-flight copies and MMAs, frees
// TMEM and returns.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "mx_internal.h"
#include "mx_ptx.cuh"

namespace mx {
namespace {

constexpr int kBM = 128, kBN = 256, kBK = 16;  // kBK fp32 = 64-byte K-major rows
constexpr int kThreads = 192;
constexpr int kTmemCols = 512;
// K-major tile: [rows][16] fp32, 64-byte rows, 64-byte swizzle; 8-row groups
// 512 B apart.  MN-major tile: 32-wide MN chunks of [16 k][32 mn], 128-byte
// rows; tf32 MN-major operands need the 128-byte swizzle with 32-byte atoms
// (TMA SWIZZLE_128B_ATOM_32B, UMMA layout 128B_BASE32B): 4-row K groups
// 512 B apart, chunks 2048 B apart, an 8-deep MMA slice = 8 rows = 1024 B.
constexpr uint32_t kSboK = 8 * kBK * 4;         // 512 B
constexpr uint32_t kSboMN = 4 * 128;            // 512 B
constexpr uint32_t kK8MN = 8 * 128;             // 1024 B
constexpr uint32_t kChunkMN = kBK * 128;        // 2048 B (BK-deep stages: BK * 128)
constexpr uint32_t kLayoutSw64 = 4, kLayoutSw128Base32 = 1, kLayoutSw128 = 2;

// k-block depth of a stage.  Plain TF32 takes 32 k per stage (K-major rows
// of 128 bytes with the 128-byte swizzle; MN-major chunks of 32 k x 32 mn):
// one pass of MMAs per stage is short, and twice the depth halves the TMA
// copies and barrier round trips per MMA.  3xTF32: 16.
template <int PASSES, bool AK, bool BKM>
__host__ __device__ constexpr int stage_bk() {
  return PASSES == 1 ? 32 : 16;
}

template <int PASSES, int BK = kBK>
struct Cfg {
  static constexpr int kOperandCopies = PASSES == 3 ? 2 : 1;
  static constexpr int kATileB = kBM * BK * 4;  // bytes
  static constexpr int kBTileB = kBN * BK * 4;
  static constexpr int kStageBytes = kOperandCopies * (kATileB + kBTileB);
  static constexpr int kStages = PASSES == 3 ? 4 : (BK == 32 ? 4 : 8);
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 512;
};

struct TcParams {
  float* c;             // may be null when only the split output is wanted
  const float* bias;
  const float* mask;    // ReLU-backward mask: output zeroed where mask <= 0
  float* c_hi;          // optional hi/lo split of the output (same ldc)
  float* c_lo;
  int* status;
  int64_t ldc, ldm;
  int M, N, K;
  int tiles_m, tiles_n, num_tiles;
  float alpha, beta;
  int relu;
  uint64_t timeout_ns;
  bool a_map3d, b_map3d;  // MN-major operand loaded by one 3-D copy per tile
  // Split tiles.  sk = 1 (stream-K): the (tile, k-block) iterations of the
  // tiles from sk_tile0 on are split evenly over the CTAs.  sk = 2 (tail
  // split): after the full data-parallel waves, each of the tail_r remaining
  // tiles keeps a primary CTA for k-blocks [0, tail_kp) and the idle CTAs
  // ("helpers") take the rest -- tail_s pieces of tail_len k-blocks per tile
  // when there are at least as many helpers as tiles, else whole tails of
  // several tiles each (at most tail_j per helper), all helpers walking k in
  // step.  Either way a tile shared by several CTAs is summed, in k order, by
  // whichever finishes last.
  int sk;
  int sk_tile0;           // first tile of the split region
  int tail_r, tail_kp, tail_s, tail_len, tail_j;
  float* sk_partials;     // partial tiles: [slots][128][256] fp32
  int* sk_counters;       // [num_tiles] arrival counters, zero at launch
  int* tile_counter;      // dynamic whole-tile scheduling (zero at launch), or null
  // Column sums of the stored output (the bias gradient of the layer whose
  // dY this GEMM produces): colsum[col] = sum over rows < M of the stored
  // value.  Each tile's sums go to colsum_part[tm][col]; the last tile of an
  // N-tile column to finish (arrival counter colsum_cnt[tn], zero at launch
  // and left zero) adds the M-tiles' rows in order.  Null: off.
  float* colsum;
  float* colsum_part;     // [tiles_m][N]
  int* colsum_cnt;        // [tiles_n]
  // Paired launch (tc_gemm_pair_kernel): the tiles of a second, independent
  // GEMM follow this one's in the tile order -- pair_tiles of them, whole
  // tiles only (sk = 0).  0 for a single GEMM.
  int pair_tiles;
};

// Grouped raster: bands of 16 M-tiles, N-major inside a band, so the CTAs
// running at one time share A and B tiles in L2.
__device__ __forceinline__ void tile_coords(int t, int tiles_m, int tiles_n, int& tm, int& tn) {
  constexpr int G = 16;
  const int band = t / (G * tiles_n);
  const int first_m = band * G;
  const int gm = min(G, tiles_m - first_m);
  const int r = t - band * G * tiles_n;
  tm = first_m + r % gm;
  tn = r / gm;
}

// The sequence of work segments of one CTA: a segment is k-blocks [kb0, kb1)
// of one tile.  Whole tiles below sk_tile0 go data-parallel (tiles
// blockIdx.x, +gridDim.x, ...: every CTA runs the same number of them, in
// lock-step, so concurrent CTAs share k-slices in L2).  In stream-K mode the
// remaining tiles' iterations (tiles x k-blocks) are then split into equal
// contiguous shares, one per CTA, cut at tile boundaries.
// Dynamic whole-tile scheduling (p.tile_counter set): the producer thread
// takes the next tile from a global atomic counter and publishes its id in a
// shared-memory ring that the MMA thread and the epilogue warps read in the
// same order.  A CTA that starts late (its SM busy with another kernel, e.g.
// an NCCL all-reduce running alongside) simply takes fewer tiles, instead of
// leaving its fixed share as a tail.
constexpr int kRing = 4;
struct TileRing {
  uint64_t* full;
  uint64_t* empty;
  int* tile;
};
enum Role { kProducer = 0, kMma = 1, kEpilogue = 2 };

struct SegIter {
  int64_t g, g_end;  // stream-K iteration cursor
  int t;             // static data-parallel tile cursor
  int n;             // dynamic: tiles taken from the ring so far
  int u;             // tail split: segments taken so far
  bool dp_done;
  __device__ __forceinline__ void init(const TcParams& p, int num_kb) {
    t = blockIdx.x;
    n = 0;
    u = 0;
    dp_done = false;
    g = g_end = 0;
    if (p.sk == 1) {
      const int64_t base = static_cast<int64_t>(p.sk_tile0) * num_kb;
      const int64_t W = static_cast<int64_t>(p.num_tiles - p.sk_tile0) * num_kb;
      g = base + W * blockIdx.x / gridDim.x;
      g_end = base + W * (blockIdx.x + 1) / gridDim.x;
    }
  }
  // Next whole tile of the data-parallel phase, -1 when the phase is over
  // (or on abort).
  template <int ROLE>
  __device__ __forceinline__ int next_dp(const TcParams& p, const TileRing& ring,
                                         volatile int* abort_flag) {
    const int dp_end = p.sk ? p.sk_tile0 : p.num_tiles + p.pair_tiles;
    if (!p.tile_counter) {
      if (t >= dp_end) return -1;
      const int r = t;
      t += gridDim.x;
      return r;
    }
    const int slot = n % kRing;
    const uint32_t par = (n / kRing) & 1;
    ++n;
    int r;
    if (ROLE == kProducer) {
      if (!wait_bar(&ring.empty[slot], par ^ 1, abort_flag, p.status, p.timeout_ns, 205))
        return -1;
      r = atomicAdd(p.tile_counter, 1);
      if (r >= dp_end) r = -1;
      ring.tile[slot] = r;
      bar_arrive(&ring.full[slot]);  // release: the id is visible to the waiters
    } else {
      if (!wait_bar(&ring.full[slot], par, abort_flag, p.status, p.timeout_ns, 206)) return -1;
      r = ring.tile[slot];
      if (ROLE == kEpilogue) bar_arrive(&ring.empty[slot]);
    }
    return r;
  }
  // Tail split: this CTA's next segment of the remainder tiles (see TcParams).
  __device__ __forceinline__ bool next_tail(const TcParams& p, int num_kb, int& tile, int& kb0,
                                            int& kb1) {
    const int r = p.tail_r, c = blockIdx.x;
    if (c < r) {  // primary of remainder tile c
      if (u++ > 0) return false;
      tile = p.sk_tile0 + c;
      kb0 = 0;
      kb1 = p.tail_kp;
      return true;
    }
    const int h = c - r, H = gridDim.x - r;
    if (p.tail_s > 0) {  // one piece of one tail
      if (u++ > 0 || h >= r * p.tail_s) return false;
      const int piece = h / r;
      tile = p.sk_tile0 + h % r;
      kb0 = p.tail_kp + piece * p.tail_len;
      kb1 = piece == p.tail_s - 1 ? num_kb : kb0 + p.tail_len;
      return true;
    }
    const int i = h + u * H;  // whole tails of tiles h, h + H, ...
    if (i >= r) return false;
    ++u;
    tile = p.sk_tile0 + i;
    kb0 = p.tail_kp;
    kb1 = num_kb;
    return true;
  }
  template <int ROLE>
  __device__ __forceinline__ bool next(const TcParams& p, int num_kb, int& tile, int& kb0,
                                       int& kb1, const TileRing& ring, volatile int* abort_flag) {
    if (!dp_done) {
      const int r = next_dp<ROLE>(p, ring, abort_flag);
      if (r >= 0) {
        tile = r;
        kb0 = 0;
        kb1 = num_kb;
        return true;
      }
      dp_done = true;
      if (*abort_flag) return false;
    }
    if (p.sk == 2) return next_tail(p, num_kb, tile, kb0, kb1);
    if (g >= g_end) return false;
    tile = static_cast<int>(g / num_kb);
    kb0 = static_cast<int>(g - static_cast<int64_t>(tile) * num_kb);
    const int64_t left = g_end - g;
    kb1 = (kb0 + left < num_kb) ? static_cast<int>(kb0 + left) : num_kb;
    g += kb1 - kb0;
    return true;
  }
};

// Stream-K bookkeeping over the stream-K region (iterations counted from the
// first stream-K tile, W of them): the CTA whose share holds iteration g, and
// the first iteration of a CTA's share.
__device__ __forceinline__ int sk_cta_of(int64_t g, int64_t W, int G) {
  return static_cast<int>(((g + 1) * G + W - 1) / W) - 1;
}
__device__ __forceinline__ int64_t sk_start(int c, int64_t W, int G) { return W * c / G; }

// Partial-tile slots of both split modes (index into p.sk_partials, in
// kBM x kBN tiles).  own_slot: where this CTA parks its part of tile t;
// tile_parts / part_slot: how many parts tile t has and where its j-th part
// in k order lies (the finisher's view).
__device__ __forceinline__ int64_t own_slot(const TcParams& p, int t, int num_kb) {
  if (p.sk == 1) {
    const int64_t W = static_cast<int64_t>(p.num_tiles - p.sk_tile0) * num_kb;
    const int64_t tile_g0 = static_cast<int64_t>(t - p.sk_tile0) * num_kb;
    return static_cast<int64_t>(blockIdx.x) * 2 +
           (sk_start(blockIdx.x, W, gridDim.x) >= tile_g0 ? 0 : 1);
  }
  const int r = p.tail_r, c = blockIdx.x;
  if (c < r) return c;
  const int h = c - r;
  if (p.tail_s > 0) return r + h;
  const int H = gridDim.x - r;
  return r + static_cast<int64_t>(h) * p.tail_j + (t - p.sk_tile0 - h) / H;
}
__device__ __forceinline__ int tile_parts(const TcParams& p, int t, int num_kb, int& c_first) {
  if (p.sk == 1) {
    const int64_t W = static_cast<int64_t>(p.num_tiles - p.sk_tile0) * num_kb;
    const int64_t tile_g0 = static_cast<int64_t>(t - p.sk_tile0) * num_kb;
    c_first = sk_cta_of(tile_g0, W, gridDim.x);
    return sk_cta_of(tile_g0 + num_kb - 1, W, gridDim.x) - c_first + 1;
  }
  c_first = 0;
  return 1 + (p.tail_s > 0 ? p.tail_s : 1);
}
__device__ __forceinline__ int64_t part_slot(const TcParams& p, int t, int num_kb, int c_first,
                                             int j) {
  if (p.sk == 1) {
    const int c = c_first + j;
    const int64_t W = static_cast<int64_t>(p.num_tiles - p.sk_tile0) * num_kb;
    const int64_t tile_g0 = static_cast<int64_t>(t - p.sk_tile0) * num_kb;
    return static_cast<int64_t>(c) * 2 + (sk_start(c, W, gridDim.x) >= tile_g0 ? 0 : 1);
  }
  const int r = p.tail_r, i = t - p.sk_tile0;
  if (j == 0) return i;                                                  // the primary
  if (p.tail_s > 0) return r + static_cast<int64_t>(j - 1) * r + i;      // piece j - 1
  const int H = gridDim.x - r;
  return r + static_cast<int64_t>(i % H) * p.tail_j + i / H;            // the helper's tail
}

// Epilogue of one column of 32 consecutive rows (row0.., col), the lane =
// column layout after the warp's transpose: a warp's loads and stores at one
// row are 32 consecutive floats.  v holds alpha-less accumulator values;
// applies alpha/beta/bias/ReLU/mask, stores c and the hi/lo split, and leaves
// the stored values in v (zero where nothing is stored).
__device__ __forceinline__ void store_rows(const TcParams& p, int row0, int col, float (&v)[32]) {
  const bool colok = col < p.N;
  const float b = (p.bias && colok) ? __ldg(p.bias + col) : 0.0f;
  float m[32];
  if (p.mask) {
#pragma unroll
    for (int i = 0; i < 32; ++i)
      m[i] = (colok && row0 + i < p.M)
                 ? __ldg(p.mask + static_cast<int64_t>(row0 + i) * p.ldm + col) : 0.0f;
  }
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    const int row = row0 + i;
    float x = p.alpha * v[i];
    if (colok && row < p.M) {
      const int64_t off = static_cast<int64_t>(row) * p.ldc + col;
      if (p.beta != 0.0f) x = x + p.beta * p.c[off];
      if (p.bias) x = x + b;
      if (p.relu) x = x > 0.0f ? x : 0.0f;
      if (p.mask && !(m[i] > 0.0f)) x = 0.0f;
      if (p.c) p.c[off] = x;
      if (p.c_hi) {
        const float h = __uint_as_float(f32_to_tf32_rna(x));
        p.c_hi[off] = h;
        if (p.c_lo) p.c_lo[off] = __uint_as_float(f32_to_tf32_rna(x - h));
      }
    } else {
      x = 0.0f;
    }
    v[i] = x;
  }
}

// Epilogue of four consecutive outputs (row, col..col+3): the same math as
// store_rows for a 4-wide group; b4 holds bias[col..col+3] (zero past N),
// loaded once by the caller.
__device__ __forceinline__ float4 store_quad(const TcParams& p, int row, int col, float4 acc,
                                             float4 b4, bool vec_ok, bool mask_vec) {
  const int64_t roff = static_cast<int64_t>(row) * p.ldc;
  const bool full = col + 4 <= p.N;
  float m[4] = {1.0f, 1.0f, 1.0f, 1.0f};
  if (p.mask) {
    const float* mp = p.mask + static_cast<int64_t>(row) * p.ldm + col;
    if (mask_vec && full) {
      const float4 t = __ldg(reinterpret_cast<const float4*>(mp));
      m[0] = t.x; m[1] = t.y; m[2] = t.z; m[3] = t.w;
    } else {
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (col + j < p.N) m[j] = __ldg(mp + j);
    }
  }
  float v[4] = {acc.x, acc.y, acc.z, acc.w};
  const float bb[4] = {b4.x, b4.y, b4.z, b4.w};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float x = p.alpha * v[j];
    if (col + j < p.N) {
      if (p.beta != 0.0f) x = x + p.beta * p.c[roff + col + j];
      if (p.bias) x = x + bb[j];
      if (p.relu) x = x > 0.0f ? x : 0.0f;
      if (p.mask && !(m[j] > 0.0f)) x = 0.0f;
    }
    v[j] = x;
  }
  float hv[4], lv[4];
  if (p.c_hi) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      hv[j] = __uint_as_float(f32_to_tf32_rna(v[j]));
      lv[j] = __uint_as_float(f32_to_tf32_rna(v[j] - hv[j]));
    }
  }
  if (vec_ok && full) {
    if (p.c) *reinterpret_cast<float4*>(p.c + roff + col) = make_float4(v[0], v[1], v[2], v[3]);
    if (p.c_hi) {
      *reinterpret_cast<float4*>(p.c_hi + roff + col) = make_float4(hv[0], hv[1], hv[2], hv[3]);
      if (p.c_lo)
        *reinterpret_cast<float4*>(p.c_lo + roff + col) = make_float4(lv[0], lv[1], lv[2], lv[3]);
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (col + j < p.N) {
        if (p.c) p.c[roff + col + j] = v[j];
        if (p.c_hi) {
          p.c_hi[roff + col + j] = hv[j];
          if (p.c_lo) p.c_lo[roff + col + j] = lv[j];
        }
      }
  }
  return make_float4(v[0], v[1], v[2], v[3]);  // the stored values, for column sums
}

__device__ __forceinline__ void epilogue_bar() {
  asm volatile("bar.sync 1, 128;" ::: "memory");  // the four epilogue warps
}

// One operand tile (rows x 16 k) of one copy (hi or lo) into shared memory.
// MN-major tiles are 32-wide chunks: one 3-D copy (32 mn x 16 k x chunks)
// when the operand's row count is a multiple of 32 (map3d), else one 2-D
// copy per chunk (out-of-range rows then read as zeros).
template <bool KMAJOR, int ROWS, int BK = kBK>
__device__ __forceinline__ void load_operand(uint8_t* dst, const CUtensorMap* map, uint64_t* bar,
                                             int k0, int r0, bool map3d) {
  if (KMAJOR) {
    tma_load_2d(dst, map, bar, k0, r0);
  } else if (map3d) {
    tma_load_3d(dst, map, bar, 0, k0, r0 / 32);
  } else {
#pragma unroll
    for (int c = 0; c < ROWS / 32; ++c) tma_load_2d(dst + c * BK * 128, map, bar, r0 + 32 * c, k0);
  }
}

// Descriptor of the k8-th 8-deep slice of an operand tile (BK-deep stages;
// K-major rows of BK floats: 8-row groups 8*BK*4 bytes apart).
template <bool KMAJOR, int BK = kBK>
__device__ __forceinline__ uint64_t operand_desc(uint32_t saddr, int k8) {
  if (KMAJOR)
    return sdesc_kmajor(saddr + k8 * 32, 8 * BK * 4, BK == 32 ? kLayoutSw128 : kLayoutSw64);
  return sdesc_mnmajor(saddr + k8 * kK8MN, BK * 128, kSboMN, kLayoutSw128Base32);
}

// One stage of operand tiles (A hi/lo, B hi/lo) for k-blocks starting at k0.
template <int PASSES, bool AK, bool BKM, int BK>
__device__ __forceinline__ void load_stage(uint8_t* base, const CUtensorMap* ah,
                                           const CUtensorMap* al, const CUtensorMap* bh,
                                           const CUtensorMap* bl, uint64_t* bar, int k0, int tm,
                                           int tn, bool a3d, bool b3d) {
  using C = Cfg<PASSES, BK>;
  constexpr int kATile = C::kATileB, kBTile = C::kBTileB;
  load_operand<AK, kBM, BK>(base, ah, bar, k0, tm * kBM, a3d);
  if (PASSES == 3) {
    load_operand<AK, kBM, BK>(base + kATile, al, bar, k0, tm * kBM, a3d);
    load_operand<BKM, kBN, BK>(base + 2 * kATile, bh, bar, k0, tn * kBN, b3d);
    load_operand<BKM, kBN, BK>(base + 2 * kATile + kBTile, bl, bar, k0, tn * kBN, b3d);
  } else {
    load_operand<BKM, kBN, BK>(base + kATile, bh, bar, k0, tn * kBN, b3d);
  }
}

// The MMAs of one stage: BK/8 slices, three TF32 MMAs per slice for 3xTF32
// (lo_a.hi_b, hi_a.lo_b, hi_a.hi_b), one for plain TF32.
template <int PASSES, bool AK, bool BKM, int BK>
__device__ __forceinline__ void mma_stage(uint32_t s_base, uint32_t d_tmem, uint32_t idesc,
                                          uint32_t& accumulate) {
  using C = Cfg<PASSES, BK>;
  constexpr int kATile = C::kATileB, kBTile = C::kBTileB;
  const uint32_t s_ah = s_base;
  const uint32_t s_al = s_base + kATile;
  const uint32_t s_bh = s_base + (PASSES == 3 ? 2 * kATile : kATile);
  const uint32_t s_bl = s_base + 2 * kATile + kBTile;
#pragma unroll
  for (int k8 = 0; k8 < BK / 8; ++k8) {
    const uint64_t ah = operand_desc<AK, BK>(s_ah, k8);
    const uint64_t bh = operand_desc<BKM, BK>(s_bh, k8);
    if (PASSES == 3) {
      const uint64_t al = operand_desc<AK, BK>(s_al, k8);
      const uint64_t bl = operand_desc<BKM, BK>(s_bl, k8);
      mma_tf32(d_tmem, al, bh, idesc, accumulate);
      mma_tf32(d_tmem, ah, bl, idesc, 1u);
      mma_tf32(d_tmem, ah, bh, idesc, 1u);
    } else {
      mma_tf32(d_tmem, ah, bh, idesc, accumulate);
    }
    accumulate = 1u;
  }
}

// The kernel body.  PAIR: a second, independent GEMM (p1, tensor maps *1,
// operand layouts AK1/BK1) shares the launch; its tiles follow p's in the
// tile order (whole tiles, static round robin), so a CTA's second tile --
// typically of the other GEMM -- runs its main loop while the first tile's
// epilogue drains, and the two GEMMs pay one launch, one prologue and one
// unhidden epilogue between them.
template <int PASSES, bool AK, bool BKM, bool PAIR, bool AK1, bool BK1>
__device__ __forceinline__ void tc_gemm_body(const CUtensorMap* tmAh, const CUtensorMap* tmAl,
                                             const CUtensorMap* tmBh, const CUtensorMap* tmBl,
                                             const CUtensorMap* tmAh1, const CUtensorMap* tmAl1,
                                             const CUtensorMap* tmBh1, const CUtensorMap* tmBl1,
                                             const TcParams& p, const TcParams& p1) {
  constexpr int BK = stage_bk<PASSES, AK, BKM>();
  static_assert(!PAIR || stage_bk<PASSES, AK1, BK1>() == BK, "paired GEMMs share the stage shape");
  using C = Cfg<PASSES, BK>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + C::kStages * C::kStageBytes);
  uint64_t* empty = full + C::kStages;
  uint64_t* acc_full = empty + C::kStages;   // [2]
  uint64_t* acc_empty = acc_full + 2;        // [2]
  uint64_t* drain = acc_empty + 2;           // [1]
  uint64_t* ring_full = drain + 1;           // [kRing] dynamic tile ids published
  uint64_t* ring_empty = ring_full + kRing;  // [kRing] ... and consumed
  int* ring_tile = reinterpret_cast<int*>(ring_empty + kRing);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring_tile + kRing);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  TileRing ring{ring_full, ring_empty, ring_tile};

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < C::kStages; ++s) {
      bar_init(&full[s], 1);
      bar_init(&empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      bar_init(&acc_full[a], 1);
      bar_init(&acc_empty[a], 128);
    }
    bar_init(drain, 1);
    for (int r = 0; r < kRing; ++r) {
      bar_init(&ring_full[r], 1);
      bar_init(&ring_empty[r], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
    tma_prefetch_desc(tmAh);
    tma_prefetch_desc(tmBh);
    if (PASSES == 3) {
      tma_prefetch_desc(tmAl);
      tma_prefetch_desc(tmBl);
    }
    if (PAIR) {
      tma_prefetch_desc(tmAh1);
      tma_prefetch_desc(tmBh1);
      tma_prefetch_desc(tmAl1);
      tma_prefetch_desc(tmBl1);
    }
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  const int num_kb = (p.K + BK - 1) / BK;
  const int num_kb1 = PAIR ? (p1.K + BK - 1) / BK : num_kb;
  // A segment of the pair's second GEMM: its tile index and k extent.
  auto second = [&](int& t, int& kb1) {
    if (PAIR && t >= p.num_tiles) {
      t -= p.num_tiles;
      kb1 = num_kb1;
      return true;
    }
    return false;
  };

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int armed_parity[C::kStages];
      bool armed[C::kStages];
      for (int s = 0; s < C::kStages; ++s) armed[s] = false;
      bool ok = true;
      SegIter it;
      it.init(p, num_kb);
      int t, kb0, kb1;
      while (ok && it.next<kProducer>(p, num_kb, t, kb0, kb1, ring, abort_flag)) {
        const bool q1 = second(t, kb1);
        const TcParams& q = q1 ? p1 : p;
        int tm, tn;
        tile_coords(t, q.tiles_m, q.tiles_n, tm, tn);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bar(&empty[stage], phase ^ 1, abort_flag, p.status, p.timeout_ns, 201)) {
            ok = false;
            break;
          }
          uint8_t* base = smem + stage * C::kStageBytes;
          bar_arrive_expect_tx(&full[stage], C::kStageBytes);
          armed[stage] = true;
          armed_parity[stage] = phase;
          const int k0 = kb * BK;
          if (PAIR && q1)
            load_stage<PASSES, AK1, BK1, BK>(base, tmAh1, tmAl1, tmBh1, tmBl1, &full[stage], k0,
                                             tm, tn, p1.a_map3d, p1.b_map3d);
          else
            load_stage<PASSES, AK, BKM, BK>(base, tmAh, tmAl, tmBh, tmBl, &full[stage], k0, tm,
                                            tn, p.a_map3d, p.b_map3d);
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Every copy this thread issued must land before the CTA can exit
      // (bounded by the drain limit, not by the caller's wait limit).
      for (int s = 0; s < C::kStages; ++s)
        if (armed[s]) drain_wait(&full[s], armed_parity[s], p.status, 207);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc0 = idesc_tf32(kBM, kBN, !AK, !BKM);
      const uint32_t idesc1 = idesc_tf32(kBM, kBN, !AK1, !BK1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      SegIter it;
      it.init(p, num_kb);
      int t, kb0, kb1;
      while (ok && it.next<kMma>(p, num_kb, t, kb0, kb1, ring, abort_flag)) {
        const bool q1 = second(t, kb1);
        // two accumulators: tile i's epilogue beside tile i+1's main loop
        const int acc = local & 1;
        const uint32_t acc_phase = (local >> 1) & 1;
        ++local;
        if (!wait_bar(&acc_empty[acc], acc_phase ^ 1, abort_flag, p.status, p.timeout_ns, 202)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * kBN;
        uint32_t accumulate = 0;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!wait_bar(&full[stage], phase, abort_flag, p.status, p.timeout_ns, 203)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t s_base = smem_u32(smem + stage * C::kStageBytes);
          if (PAIR && q1)
            mma_stage<PASSES, AK1, BK1, BK>(s_base, d_tmem, idesc1, accumulate);
          else
            mma_stage<PASSES, AK, BKM, BK>(s_base, d_tmem, idesc0, accumulate);
          tc_commit(&empty[stage]);  // frees the stage once these MMAs have read it
          if (++stage == C::kStages) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        tc_commit(&acc_full[acc]);  // accumulator ready for the epilogue
      }
      // Wait for every MMA this thread issued before TMEM is released.
      tc_commit(drain);
      drain_wait(drain, 0, p.status, 208);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    const int lane_grp = warp & 3;                 // TMEM lanes this warp may access
    const int row_in_tile = lane_grp * 32 + lane;
    // 16-byte stores of the output / loads of the mask (per GEMM of a pair)
    auto vec_of = [](const TcParams& q) {
      return (q.ldc % 4 == 0) &&
             ((reinterpret_cast<uintptr_t>(q.c) | reinterpret_cast<uintptr_t>(q.c_hi) |
               reinterpret_cast<uintptr_t>(q.c_lo)) & 15u) == 0;
    };
    auto mask_vec_of = [](const TcParams& q) {
      return (q.ldm % 4 == 0) && ((reinterpret_cast<uintptr_t>(q.mask) & 15u) == 0);
    };
    __shared__ int sk_last;  // broadcast of the arrival test among the epilogue warps
    __shared__ int cs_last;
    __shared__ __align__(16) float cs_warp[4][kBN];  // column sums of parts of the tile's rows
    __shared__ float tr_buf[4][32 * 33];              // per-warp transpose, padded: no conflicts
    // The tile's column sums into colsum_part[tm] (value(c) for the tile's
    // column c), then the arrival test of its N-tile column: the last M-tile
    // to arrive adds every M-tile's row in order (the result does not depend
    // on which tile arrives last).  All four epilogue warps call it.
    auto colsum_commit = [&](const TcParams& q, int tm, int tn, auto value) {
      epilogue_bar();
      const int c_base = tn * kBN;
#pragma unroll
      for (int c = row_in_tile; c < kBN; c += 128) {
        const int col = c_base + c;
        if (col < q.N) q.colsum_part[static_cast<int64_t>(tm) * q.N + col] = value(c);
      }
      __threadfence();
      epilogue_bar();
      if (row_in_tile == 0) {
        const int old = atomicAdd(&q.colsum_cnt[tn], 1);
        cs_last = (old == q.tiles_m - 1) ? 1 : 0;
        if (cs_last) q.colsum_cnt[tn] = 0;  // ready for the next launch
      }
      epilogue_bar();
      if (cs_last) {
        __threadfence();
#pragma unroll
        for (int c = row_in_tile; c < kBN; c += 128) {
          const int col = c_base + c;
          if (col < q.N) {
            const float* src = q.colsum_part + col;
            float s0 = 0.0f, s1 = 0.0f, s2 = 0.0f, s3 = 0.0f;
            int m = 0;
            for (; m + 4 <= q.tiles_m; m += 4) {  // four independent chains
              s0 += __ldcg(src + static_cast<int64_t>(m) * q.N);
              s1 += __ldcg(src + static_cast<int64_t>(m + 1) * q.N);
              s2 += __ldcg(src + static_cast<int64_t>(m + 2) * q.N);
              s3 += __ldcg(src + static_cast<int64_t>(m + 3) * q.N);
            }
            for (; m < q.tiles_m; ++m) s0 += __ldcg(src + static_cast<int64_t>(m) * q.N);
            q.colsum[col] = (s0 + s1) + (s2 + s3);
          }
        }
      }
    };
    int local = 0;
    SegIter it;
    it.init(p, num_kb);
    int t, kb0, kb1;
    while (it.next<kEpilogue>(p, num_kb, t, kb0, kb1, ring, abort_flag)) {
      const int acc = local & 1;
      const uint32_t acc_phase = (local >> 1) & 1;
      ++local;
      if (!wait_bar(&acc_full[acc], acc_phase, abort_flag, p.status, p.timeout_ns, 204)) break;
      tc_fence_after();
      const bool q1 = second(t, kb1);
      const TcParams& q = q1 ? p1 : p;  // the GEMM of this tile
      const bool vec_ok = vec_of(q), mask_vec = mask_vec_of(q);
      int tm, tn;
      tile_coords(t, q.tiles_m, q.tiles_n, tm, tn);
      const bool whole = q1 || (kb0 == 0 && kb1 == num_kb);
      const int rbase = lane_grp * 32;  // this warp's first row in the tile
      float* tw = &tr_buf[lane_grp][0];
#pragma unroll 1
      for (int chunk = 0; chunk < kBN / 32; ++chunk) {
        uint32_t r[32];
        __syncwarp();  // the previous chunk's transpose reads are done
        tmem_ld_32cols(tmem_base + (static_cast<uint32_t>(lane_grp * 32) << 16) + acc * kBN +
                           chunk * 32,
                       r);
        tmem_wait_ld();
        // Transpose the warp's 32 x 32 block (lane = row -> lane = column),
        // so that every global load and store below is one 128-byte line.
#pragma unroll
        for (int j = 0; j < 32; ++j) tw[lane * 33 + j] = __uint_as_float(r[j]);
        __syncwarp();
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = tw[i * 33 + lane];
        if (whole) {
          const int col = tn * kBN + chunk * 32 + lane;
          store_rows(q, tm * kBM + rbase, col, v);
          if (q.colsum) {  // rows past M and columns past N hold zero
            float cs = 0.0f;
#pragma unroll
            for (int i = 0; i < 32; ++i) cs += v[i];
            cs_warp[lane_grp][chunk * 32 + lane] = cs;
          }
        } else {
          // partial tile: this CTA's slot, [row][256 columns]
          float* slot = p.sk_partials + own_slot(p, t, num_kb) * (kBM * kBN) +
                        static_cast<int64_t>(rbase) * kBN + chunk * 32 + lane;
#pragma unroll
          for (int i = 0; i < 32; ++i) slot[static_cast<int64_t>(i) * kBN] = v[i];
        }
      }
      tc_fence_before();
      bar_arrive(&acc_empty[acc]);  // TMEM is free again; partials are in memory
      if (whole && q.colsum)
        colsum_commit(q, tm, tn, [&](int c) {
          return (cs_warp[0][c] + cs_warp[1][c]) + (cs_warp[2][c] + cs_warp[3][c]);
        });
      if (!whole) {
        // Arrival: the last CTA to finish its part of tile t sums all parts
        // (in k order, so the result does not depend on who is last) and runs
        // the epilogue.  Nobody waits for anybody.
        int c_first = 0;
        const int parts = tile_parts(p, t, num_kb, c_first);
        __threadfence();
        epilogue_bar();
        if (row_in_tile == 0) {
          const int old = atomicAdd(&p.sk_counters[t], 1);
          sk_last = (old == parts - 1) ? 1 : 0;
          if (sk_last) p.sk_counters[t] = 0;  // ready for the next launch
        }
        epilogue_bar();
        if (sk_last) {
          __threadfence();
          // Coalesced pass over the tile: each epilogue thread owns one 4-wide
          // column group (q) of every other row, so a warp reads 512
          // contiguous bytes of a partial per load and keeps many in flight.
          const int q = row_in_tile & 63;
          const int64_t tile_off = static_cast<int64_t>(row_in_tile >> 6) * kBN + q * 4;
          const int col = tn * kBN + q * 4;
          float4 b4 = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // bias of my four columns
          if (p.bias && col < p.N) {
            b4.x = __ldg(p.bias + col);
            if (col + 1 < p.N) b4.y = __ldg(p.bias + col + 1);
            if (col + 2 < p.N) b4.z = __ldg(p.bias + col + 2);
            if (col + 3 < p.N) b4.w = __ldg(p.bias + col + 3);
          }
          auto part_src = [&](int j, int i0) {
            return p.sk_partials + part_slot(p, t, num_kb, c_first, j) * (kBM * kBN) + tile_off +
                   static_cast<int64_t>(i0) * 2 * kBN;
          };
          auto add8 = [](float4 (&acc)[8], const float4 (&v)[8]) {
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              acc[u].x += v[u].x;
              acc[u].y += v[u].y;
              acc[u].z += v[u].z;
              acc[u].w += v[u].w;
            }
          };
          float4 cs = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // column sums of my rows
#pragma unroll 1
          for (int i0 = 0; i0 < kBM / 2; i0 += 8) {
            float4 s[8];
#pragma unroll
            for (int u = 0; u < 8; ++u) s[u] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            // k order (same sum on any finisher), two parts' loads in flight
            int j = 0;
            for (; j + 2 <= parts; j += 2) {
              const float* s0 = part_src(j, i0);
              const float* s1 = part_src(j + 1, i0);
              float4 v0[8], v1[8];
#pragma unroll
              for (int u = 0; u < 8; ++u)
                v0[u] = __ldcg(reinterpret_cast<const float4*>(s0 + u * 2 * kBN));
#pragma unroll
              for (int u = 0; u < 8; ++u)
                v1[u] = __ldcg(reinterpret_cast<const float4*>(s1 + u * 2 * kBN));
              add8(s, v0);
              add8(s, v1);
            }
            if (j < parts) {
              const float* s0 = part_src(j, i0);
              float4 v0[8];
#pragma unroll
              for (int u = 0; u < 8; ++u)
                v0[u] = __ldcg(reinterpret_cast<const float4*>(s0 + u * 2 * kBN));
              add8(s, v0);
            }
#pragma unroll
            for (int u = 0; u < 8; ++u) {
              const int r = tm * kBM + (row_in_tile >> 6) + 2 * (i0 + u);
              if (r < p.M && col < p.N) {
                const float4 o = store_quad(p, r, col, s[u], b4, vec_ok, mask_vec);
                cs.x += o.x;
                cs.y += col + 1 < p.N ? o.y : 0.0f;
                cs.z += col + 2 < p.N ? o.z : 0.0f;
                cs.w += col + 3 < p.N ? o.w : 0.0f;
              }
            }
          }
          if (p.colsum) {
            // the two row halves' sums, then the tile's commit
            *reinterpret_cast<float4*>(&cs_warp[row_in_tile >> 6][q * 4]) = cs;
            colsum_commit(p, tm, tn, [&](int c) { return cs_warp[0][c] + cs_warp[1][c]; });
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, kTmemCols);
  }
}

template <int PASSES, bool AK, bool BKM>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmAh, const __grid_constant__ CUtensorMap tmAl,
                   const __grid_constant__ CUtensorMap tmBh, const __grid_constant__ CUtensorMap tmBl,
                   const TcParams p) {
  tc_gemm_body<PASSES, AK, BKM, false, AK, BKM>(&tmAh, &tmAl, &tmBh, &tmBl, &tmAh, &tmAl, &tmBh,
                                                &tmBl, p, p);
}

// Two independent 3xTF32 GEMMs in one launch (tc_gemm_body, PAIR): p's tiles
// first, then p1's.
template <bool AK, bool BKM, bool AK1, bool BK1>
__global__ void __launch_bounds__(kThreads, 1)
    tc_gemm_pair_kernel(const __grid_constant__ CUtensorMap tmAh,
                        const __grid_constant__ CUtensorMap tmAl,
                        const __grid_constant__ CUtensorMap tmBh,
                        const __grid_constant__ CUtensorMap tmBl,
                        const __grid_constant__ CUtensorMap tmAh1,
                        const __grid_constant__ CUtensorMap tmAl1,
                        const __grid_constant__ CUtensorMap tmBh1,
                        const __grid_constant__ CUtensorMap tmBl1, const TcParams p,
                        const TcParams p1) {
  tc_gemm_body<3, AK, BKM, true, AK1, BK1>(&tmAh, &tmAl, &tmBh, &tmBl, &tmAh1, &tmAl1, &tmBh1,
                                           &tmBl1, p, p1);
}

// ----------------------------------------------------------------- prepass
// hi/lo split of an operand viewed as [R rows][K]; writes dst[r * Kp + k].
// K-contiguous source: straight copy order.
__global__ void split_kcontig_kernel(const float* __restrict__ src, int64_t ld, int R, int K,
                                     int64_t Kp, float* __restrict__ hi, float* __restrict__ lo) {
  const int64_t total = static_cast<int64_t>(R) * K;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / K, k = idx - r * K;
    const float x = src[r * ld + k];
    const uint32_t h = f32_to_tf32_rna(x);
    hi[r * Kp + k] = __uint_as_float(h);
    if (lo) lo[r * Kp + k] = __uint_as_float(f32_to_tf32_rna(x - __uint_as_float(h)));
  }
}

// The same with 16-byte accesses, when K, ld and Kp are multiples of 4 and the
// three pointers 16-byte aligned (K4 = K / 4 float4s a row).
__device__ __forceinline__ float tf32_lo(float x, float h) {
  return __uint_as_float(f32_to_tf32_rna(x - h));
}
__global__ void split_kcontig4_kernel(const float4* __restrict__ src, int64_t ld4, int R, int K4,
                                      int64_t Kp4, float4* __restrict__ hi,
                                      float4* __restrict__ lo) {
  const int64_t total = static_cast<int64_t>(R) * K4;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < total;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / K4, k = idx - r * K4;
    const float4 x = __ldg(src + r * ld4 + k);
    float4 h;
    h.x = __uint_as_float(f32_to_tf32_rna(x.x));
    h.y = __uint_as_float(f32_to_tf32_rna(x.y));
    h.z = __uint_as_float(f32_to_tf32_rna(x.z));
    h.w = __uint_as_float(f32_to_tf32_rna(x.w));
    hi[r * Kp4 + k] = h;
    if (lo)
      lo[r * Kp4 + k] =
          make_float4(tf32_lo(x.x, h.x), tf32_lo(x.y, h.y), tf32_lo(x.z, h.z), tf32_lo(x.w, h.w));
  }
}

// MN-contiguous source (element (r, k) at src[k * ld + r]): 32x32 transpose
// through shared memory so both the reads and the writes are coalesced.
__global__ void split_transpose_kernel(const float* __restrict__ src, int64_t ld, int R, int K,
                                       int64_t Kp, float* __restrict__ hi, float* __restrict__ lo) {
  __shared__ float tile[32][33];
  const int r0 = blockIdx.x * 32, k0 = blockIdx.y * 32;
  const int tx = threadIdx.x, ty = threadIdx.y;  // 32 x 8
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int k = k0 + ty + i, r = r0 + tx;
    tile[ty + i][tx] = (k < K && r < R) ? src[static_cast<int64_t>(k) * ld + r] : 0.0f;
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < 32; i += 8) {
    const int r = r0 + ty + i, k = k0 + tx;
    if (r < R && k < K) {
      const float x = tile[tx][ty + i];
      const uint32_t h = f32_to_tf32_rna(x);
      hi[static_cast<int64_t>(r) * Kp + k] = __uint_as_float(h);
      if (lo) lo[static_cast<int64_t>(r) * Kp + k] =
          __uint_as_float(f32_to_tf32_rna(x - __uint_as_float(h)));
    }
  }
}

cudaError_t launch_split(const float* src, int64_t ld, bool kcontig, int R, int K, int64_t Kp,
                         float* hi, float* lo, int num_sms, cudaStream_t s) {
  const bool vec4 = K % 4 == 0 && ld % 4 == 0 && Kp % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(hi) |
                      reinterpret_cast<uintptr_t>(lo)) & 15u) == 0;
  if (kcontig && vec4) {
    const int64_t total = static_cast<int64_t>(R) * (K / 4);
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, num_sms * 16));
    split_kcontig4_kernel<<<blocks, 256, 0, s>>>(
        reinterpret_cast<const float4*>(src), ld / 4, R, K / 4, Kp / 4,
        reinterpret_cast<float4*>(hi), reinterpret_cast<float4*>(lo));
    note_launches(1);
  } else if (kcontig) {
    const int64_t total = static_cast<int64_t>(R) * K;
    const int blocks = static_cast<int>(std::min<int64_t>((total + 255) / 256, num_sms * 16));
    split_kcontig_kernel<<<blocks, 256, 0, s>>>(src, ld, R, K, Kp, hi, lo);
    note_launches(1);
  } else {
    dim3 grid((R + 31) / 32, (K + 31) / 32);
    if (grid.y > 65535) return cudaErrorInvalidValue;
    split_transpose_kernel<<<grid, dim3(32, 8), 0, s>>>(src, ld, R, K, Kp, hi, lo);
    note_launches(1);
  }
  return cudaGetLastError();
}

size_t align256(size_t x) { return (x + 255) & ~static_cast<size_t>(255); }

template <int PASSES, bool AK, bool BKM>
cudaError_t launch_tc(const CUtensorMap& ah, const CUtensorMap& al, const CUtensorMap& bh,
                      const CUtensorMap& bl, const TcParams& p, int grid, cudaStream_t s) {
  auto kern = tc_gemm_kernel<PASSES, AK, BKM>;
  constexpr int kSmem = Cfg<PASSES, stage_bk<PASSES, AK, BKM>()>::kSmem;
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(kern, kSmem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, kSmem, s>>>(ah, al, bh, bl, p);
  note_launches(1);
  return cudaGetLastError();
}

template <int PASSES>
cudaError_t launch_tc_major(bool ak, bool bkm, const CUtensorMap& ah, const CUtensorMap& al,
                            const CUtensorMap& bh, const CUtensorMap& bl, const TcParams& p,
                            int grid, cudaStream_t s) {
  if (ak && bkm) return launch_tc<PASSES, true, true>(ah, al, bh, bl, p, grid, s);
  if (ak) return launch_tc<PASSES, true, false>(ah, al, bh, bl, p, grid, s);
  if (bkm) return launch_tc<PASSES, false, true>(ah, al, bh, bl, p, grid, s);
  return launch_tc<PASSES, false, false>(ah, al, bh, bl, p, grid, s);
}

// Tensor map of one split copy.  K-major: element (r, k) at base[r*ld + k],
// box bk k x rows, 64-byte swizzle (bk = 16) or 128-byte swizzle (bk = 32).
// MN-major: element (r, k) at base[k*ld + r], box 32 mn x bk k, 128-byte
// swizzle of 32-byte atoms.
bool operand_map(CUtensorMap* m, const float* base, bool kmajor, int R, int K, int64_t ld,
                 int rows_tile, bool padded, int bk = kBK) {
  if (kmajor)
    return make_tmap_2d(m, base, K, R, ld * 4, bk, rows_tile,
                        bk == 32 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B);
  if (R % 32 == 0 || padded) {
    // dims (32 mn, K, ceil(R/32) chunks): one copy brings a whole MN-major
    // tile, in the chunk-after-chunk order the MMA descriptors expect; chunks
    // past the last read as zeros.  A partial last chunk (padded operands
    // only) reads the rows past R from memory; they feed only output
    // rows/columns that are never stored.
    const uint64_t dims[3] = {32, static_cast<uint64_t>(K), static_cast<uint64_t>((R + 31) / 32)};
    const uint64_t strides[2] = {static_cast<uint64_t>(ld) * 4, 128};
    const uint32_t box[3] = {32, static_cast<uint32_t>(bk), static_cast<uint32_t>(rows_tile / 32)};
    return make_tmap_3d(m, base, dims, strides, box, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
  }
  return make_tmap_2d(m, base, R, K, ld * 4, 32, bk, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B);
}

}  // namespace

namespace {
// One split copy of an operand, in the layout the operand is stored in (no
// transpose): K-contiguous -> [rows][Kp] (K-major tiles); MN-contiguous ->
// [K][rows4], read as MN-major tiles, with 32 floats of slack so that whole
// 32-wide MN chunks can be fetched.  Kp, rows4: rounded up to 4 (16-byte
// TMA strides).
struct CopyShape {
  bool kmajor;
  int64_t ld;
  size_t bytes;
};
CopyShape copy_shape(bool kcontig, int rows, int K) {
  if (kcontig) {
    const int64_t kp = (static_cast<int64_t>(K) + 3) & ~static_cast<int64_t>(3);
    return {true, kp, align256(static_cast<size_t>(rows) * kp * 4)};
  }
  const int64_t r4 = (static_cast<int64_t>(rows) + 3) & ~static_cast<int64_t>(3);
  return {false, r4, align256((static_cast<size_t>(K) * r4 + 32) * 4)};
}
}  // namespace

// Workspace bytes tc_gemm needs for the split operands of this shape.
size_t tc_gemm_workspace_bytes(const GemmArgs& g, int passes) {
  const size_t copies = passes == 3 ? 2 : 1;
  return copies * (copy_shape(g.ta == 0, g.M, g.K).bytes + copy_shape(g.tb != 0, g.N, g.K).bytes);
}

// K-major split copies of both operands (the carve-up of the allocation-free
// entry point below).
size_t kmajor_split_bytes(const GemmArgs& g, int passes) {
  const size_t kp = (static_cast<size_t>(g.K) + 3) & ~static_cast<size_t>(3);
  const size_t copies = passes == 3 ? 2 : 1;
  return copies * (align256(static_cast<size_t>(g.M) * kp * 4) +
                   align256(static_cast<size_t>(g.N) * kp * 4));
}

// How the tiles of a GEMM are split across the CTAs (see TcParams::sk).
struct SplitPlan {
  int mode = 0;           // 0: whole tiles only, 1: stream-K, 2: tail split
  int tile0 = 0;          // first split tile
  int r = 0, kp = 0, s = 0, len = 0, j = 0;  // tail split
  size_t slots = 0;       // partial tiles of scratch
};

SplitPlan plan_split(int M, int N, int K, int num_sms, int passes) {
  static const bool disabled = [] {
    const char* e = std::getenv("MX_STREAMK");
    return e && e[0] == '0';
  }();
  static const bool tail_enabled = [] {
    const char* e = std::getenv("MX_TAILSPLIT");
    return !(e && e[0] == '0');
  }();
  SplitPlan sp;
  if (disabled || M <= 0 || N <= 0 || K <= 0 || num_sms <= 0) return sp;
  const int bk = passes == 1 ? 32 : kBK;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  const int num_kb = (K + bk - 1) / bk;
  const int waves = (tiles + num_sms - 1) / num_sms;
  const double fill = static_cast<double>(tiles) / (static_cast<double>(waves) * num_sms);
  const int rem = tiles % num_sms;
  // Stream-K when whole tiles leave most SMs idle (e.g. the 32 tiles of a
  // 1000-wide output layer): its CTAs walk k at staggered offsets, which
  // costs L2 reuse, so only there.  Each CTA's share is at least 8 k-blocks.
  if (fill < 0.5) {
    if (static_cast<int64_t>(rem) * num_kb < 8LL * num_sms) return sp;
    sp.mode = 1;
    sp.tile0 = (tiles / num_sms) * num_sms;
    sp.slots = static_cast<size_t>(2) * num_sms;
    return sp;
  }
  // Tail split of a part-filled last wave (e.g. the 128 tiles of a 1024-row
  // layer on 148 SMs, or the 68 left after three waves of 148): the
  // remainder tiles' primaries take k-blocks [0, kp), the idle CTAs the
  // rest, in step with one another.
  if (!tail_enabled || rem == 0 || num_kb < 16) return sp;
  const int r = rem, H = num_sms - r;
  int kp, s = 0, len = 0, j = 0, helper_load;
  if (H >= r) {  // pieces: each tail cut in s pieces, one helper each
    s = std::max(1, std::min(H / r, num_kb / 8));
    kp = num_kb / (s + 1);
    len = (num_kb - kp) / s;
    helper_load = num_kb - kp - (s - 1) * len;
  } else {       // whole tails, j per helper
    j = (r + H - 1) / H;
    kp = static_cast<int>((static_cast<int64_t>(num_kb) * j + j / 2) / (j + 1));
    helper_load = j * (num_kb - kp);
  }
  if (kp < 1 || kp >= num_kb || (s > 0 && len < 1)) return sp;
  // Worth it only if the last wave gets shorter by more than the split
  // costs: every part writes a 128 KB partial tile and the finishing CTA
  // reads them back before its epilogue, some tens of microseconds that no
  // other work hides (measured on B200: a 128-tile GEMM with K = 1000 split
  // over 148 SMs ran 4x slower than whole tiles on 128).  So the last wave
  // must lose at least 64 k-blocks, and a helper's tails must be long enough
  // (32 k-blocks) for its partial-tile stores to hide behind its next tail.
  const int last = std::max(kp, helper_load);
  if (num_kb - last < 64) return sp;
  if (j > 0 && num_kb - kp < 32) return sp;
  sp.mode = 2;
  sp.tile0 = tiles - r;
  sp.r = r;
  sp.kp = kp;
  sp.s = s;
  sp.len = len;
  sp.j = j;
  sp.slots = s > 0 ? static_cast<size_t>(r) + static_cast<size_t>(r) * s
                   : static_cast<size_t>(r) + static_cast<size_t>(H) * j;
  return sp;
}

namespace {
// Cost model of the launch decisions, in k-blocks of one CTA: a launch
// costs its prologue, pipeline fill and last unhidden epilogue (kLaunchKb); a
// split tile costs the partial-tile round trip (kFinishKb).
constexpr int64_t kLaunchKb = 48, kFinishKb = 32;

int64_t tiles_of(int M, int N) {
  return static_cast<int64_t>((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
}

// Busiest CTA of one launch of its own on num_sms SMs, as tc_gemm_split
// schedules it.
int64_t gemm_makespan(int M, int N, int K, int num_sms, int passes) {
  const int bk = passes == 1 ? 32 : kBK;
  const int64_t tiles = tiles_of(M, N), kb = (K + bk - 1) / bk;
  const SplitPlan sp = plan_split(M, N, K, num_sms, passes);
  const int64_t full = tiles / num_sms;
  if (sp.mode == 2) {
    const int64_t helper = sp.s > 0 ? kb - sp.kp - static_cast<int64_t>(sp.s - 1) * sp.len
                                    : static_cast<int64_t>(sp.j) * (kb - sp.kp);
    return full * kb + std::max<int64_t>(sp.kp, helper) + kFinishKb + kLaunchKb;
  }
  if (sp.mode == 1)
    return full * kb + ((tiles - full * num_sms) * kb + num_sms - 1) / num_sms + kFinishKb +
           kLaunchKb;
  return (tiles + num_sms - 1) / num_sms * kb + kLaunchKb;
}

// Busiest CTA of the paired launch: a's tiles, then b's, round robin.
int64_t pair_makespan(const TcPairGemm& a, const TcPairGemm& b, int num_sms) {
  const int64_t ta = tiles_of(a.M, a.N), tb = tiles_of(b.M, b.N);
  const int64_t ka = (a.K + kBK - 1) / kBK, kbb = (b.K + kBK - 1) / kBK;
  const int64_t G = std::min<int64_t>(num_sms, ta + tb);
  int64_t worst = 0;
  for (int64_t c = 0; c < G; ++c) {
    const int64_t na = c < ta ? (ta - c + G - 1) / G : 0;
    // b's tile u sits at index ta + u; CTA c takes those with (ta + u) % G == c
    const int64_t first = ((c - ta) % G + G) % G;
    const int64_t nb = first < tb ? (tb - first + G - 1) / G : 0;
    worst = std::max(worst, na * ka + nb * kbb);
  }
  return worst + kLaunchKb;
}

// The SM budget is a preference: a launch keeps to `budget` SMs (leaving the
// rest to collectives running beside it) unless all SMs would finish it
// more than 3 % sooner.
template <typename Cost>
int pick_sms(int budget, int all, Cost cost) {
  if (all <= budget) return budget;
  return cost(all) * 103 < cost(budget) * 100 ? all : budget;
}
}  // namespace

namespace {
// Tensor maps (A hi, A lo, B hi, B lo) and kernel parameters of one GEMM,
// with its column-sum counters zeroed on stream s.  kOk, or an error code.
int tc_prepare(const TcLaunch& L, const SplitOperand& A, const SplitOperand& B,
               const TcEpilogue& E, int M, int N, int K, int passes, cudaStream_t s,
               CUtensorMap (&maps)[4], TcParams& p) {
  if (K <= 0 || (passes != 1 && passes != 3)) return kErrInvalid;
  if (!A.hi || !B.hi || (passes == 3 && (!A.lo || !B.lo))) return kErrInvalid;
  if (!E.c && !E.c_hi) return kErrInvalid;
  CUtensorMap& tah = maps[0];
  CUtensorMap& tal = maps[1];
  CUtensorMap& tbh = maps[2];
  CUtensorMap& tbl = maps[3];
  // plain TF32 runs 32-deep stages (stage_bk)
  const int bk = passes == 1 ? 32 : kBK;
  bool ok = operand_map(&tah, A.hi, A.kmajor, M, K, A.ld, kBM, A.padded, bk) &&
            operand_map(&tbh, B.hi, B.kmajor, N, K, B.ld, kBN, B.padded, bk);
  if (passes == 3)
    ok = ok && operand_map(&tal, A.lo, A.kmajor, M, K, A.ld, kBM, A.padded) &&
         operand_map(&tbl, B.lo, B.kmajor, N, K, B.ld, kBN, B.padded);
  else {
    tal = tah;
    tbl = tbh;
  }
  if (!ok) return kErrUnsupported;
  p = TcParams{};
  p.c = E.c; p.bias = E.bias; p.mask = E.mask; p.c_hi = E.c_hi; p.c_lo = E.c_lo;
  p.status = L.status; p.ldc = E.ldc; p.ldm = E.ldm;
  p.M = M; p.N = N; p.K = K;
  p.tiles_m = (M + kBM - 1) / kBM;
  p.tiles_n = (N + kBN - 1) / kBN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.alpha = E.alpha; p.beta = E.beta; p.relu = E.relu;
  p.timeout_ns = L.timeout_ns;
  p.a_map3d = !A.kmajor && (M % 32 == 0 || A.padded);
  p.b_map3d = !B.kmajor && (N % 32 == 0 || B.padded);
  if (E.colsum) {
    if (!E.colsum_scratch || E.colsum_scratch_bytes < tc_colsum_scratch_bytes(M, N))
      return kErrInvalid;
    p.colsum = E.colsum;
    p.colsum_part = static_cast<float*>(E.colsum_scratch);
    p.colsum_cnt = reinterpret_cast<int*>(static_cast<uint8_t*>(E.colsum_scratch) +
                                          align256(sizeof(float) * p.tiles_m * N));
    cudaError_t me = cudaMemsetAsync(p.colsum_cnt, 0, sizeof(int) * p.tiles_n, s);
    if (me != cudaSuccess) return cuda_status(me);
  }
  return kOk;
}
}  // namespace

int tc_gemm_split(const TcLaunch& L, const SplitOperand& A, const SplitOperand& B,
                  const TcEpilogue& E, int M, int N, int K, int passes, cudaStream_t s) {
  if (M == 0 || N == 0) return kOk;
  CUtensorMap maps[4] = {};
  TcParams p{};
  const int rc = tc_prepare(L, A, B, E, M, N, K, passes, s, maps, p);
  if (rc != kOk) return rc;
  const CUtensorMap &tah = maps[0], &tal = maps[1], &tbh = maps[2], &tbl = maps[3];
  // Fewest CTAs that still finish the tiles in the same number of waves: a
  // 128- or 512-tile GEMM takes 128 SMs, leaving the rest to a concurrent
  // NCCL all-reduce at no cost to the GEMM (B200 has 148 SMs).
  const int G = L.all_sms > L.num_sms ? tc_launch_sms(M, N, K, L.num_sms, L.all_sms, passes)
                                       : L.num_sms;
  const int waves = (p.num_tiles + G - 1) / G;
  int grid = (p.num_tiles + waves - 1) / waves;
  static const bool dyn_enabled = [] {  // dynamic tile order: opt-in (MX_DYNSCHED=1)
    const char* e = std::getenv("MX_DYNSCHED");
    return e && e[0] == '1';
  }();
  if (L.sched && dyn_enabled) {
    p.tile_counter = L.sched;
    cudaError_t me = cudaMemsetAsync(L.sched, 0, sizeof(int), s);
    if (me != cudaSuccess) return cuda_status(me);
  }
  const SplitPlan sp = plan_split(M, N, K, G, passes);
  const size_t sk_need = tc_streamk_bytes(M, N, K, G, passes);
  if (sp.mode != 0 && L.ws && L.ws_bytes >= sk_need && !p.tile_counter) {
    p.sk = sp.mode;
    p.sk_tile0 = sp.tile0;  // full waves stay data-parallel
    p.tail_r = sp.r;
    p.tail_kp = sp.kp;
    p.tail_s = sp.s;
    p.tail_len = sp.len;
    p.tail_j = sp.j;
    p.sk_partials = static_cast<float*>(L.ws);
    p.sk_counters = reinterpret_cast<int*>(static_cast<uint8_t*>(L.ws) +
                                           sp.slots * kBM * kBN * 4);
    grid = G;
    cudaError_t me = cudaMemsetAsync(p.sk_counters, 0, sizeof(int) * p.num_tiles, s);
    if (me != cudaSuccess) return cuda_status(me);
  }
  cudaError_t e = passes == 3
      ? launch_tc_major<3>(A.kmajor, B.kmajor, tah, tal, tbh, tbl, p, grid, s)
      : launch_tc_major<1>(A.kmajor, B.kmajor, tah, tal, tbh, tbl, p, grid, s);
  return e == cudaSuccess ? kOk : cuda_status(e);
}

namespace {
template <bool AK, bool BKM, bool AK1, bool BK1>
cudaError_t launch_pair(const CUtensorMap (&m0)[4], const CUtensorMap (&m1)[4],
                        const TcParams& p0, const TcParams& p1, int grid, cudaStream_t s) {
  auto kern = tc_gemm_pair_kernel<AK, BKM, AK1, BK1>;
  constexpr int kSmem = Cfg<3, kBK>::kSmem;
  static SmemOptIn opt_in;
  cudaError_t e = opt_in.ensure(kern, kSmem);
  if (e != cudaSuccess) return e;
  kern<<<grid, kThreads, kSmem, s>>>(m0[0], m0[1], m0[2], m0[3], m1[0], m1[1], m1[2], m1[3], p0,
                                     p1);
  note_launches(1);
  return cudaGetLastError();
}

}  // namespace

int tc_gemm_pair(const TcLaunch& L, const TcPairGemm& g0, const TcPairGemm& g1, cudaStream_t s) {
  if (g0.M == 0 || g0.N == 0) return tc_gemm_split(L, g1.A, g1.B, g1.E, g1.M, g1.N, g1.K, 3, s);
  if (g1.M == 0 || g1.N == 0) return tc_gemm_split(L, g0.A, g0.B, g0.E, g0.M, g0.N, g0.K, 3, s);
  // the GEMM with the longer tiles (more k-blocks) first: every CTA starts
  // on one of them and the short tiles fill in behind
  const bool swap = g1.K > g0.K;
  const TcPairGemm& a = swap ? g1 : g0;
  const TcPairGemm& b = swap ? g0 : g1;
  const int la = (a.A.kmajor ? 2 : 0) | (a.B.kmajor ? 1 : 0);
  const int lb = (b.A.kmajor ? 2 : 0) | (b.B.kmajor ? 1 : 0);
  // the layout pairs of a Linear layer's backward (dX: A k-major; dW: both
  // MN-major); others run as two launches
  using Fn = cudaError_t (*)(const CUtensorMap (&)[4], const CUtensorMap (&)[4], const TcParams&,
                             const TcParams&, int, cudaStream_t);
  Fn fn = nullptr;
  if (la == 3 && lb == 0) fn = launch_pair<true, true, false, false>;
  else if (la == 0 && lb == 3) fn = launch_pair<false, false, true, true>;
  else if (la == 2 && lb == 0) fn = launch_pair<true, false, false, false>;
  else if (la == 0 && lb == 2) fn = launch_pair<false, false, true, false>;
  if (!fn) {
    const int rc = tc_gemm_split(L, g0.A, g0.B, g0.E, g0.M, g0.N, g0.K, 3, s);
    return rc != kOk ? rc : tc_gemm_split(L, g1.A, g1.B, g1.E, g1.M, g1.N, g1.K, 3, s);
  }
  // Paired or as two launches, on the budget's SMs or on all of them:
  // whichever the cost model finishes first (MX_PAIR=0: always two launches).
  static const bool pair_off = [] {
    const char* e = std::getenv("MX_PAIR");
    return e && e[0] == '0';
  }();
  auto separate = [&](int G) {
    return gemm_makespan(a.M, a.N, a.K, G, 3) + gemm_makespan(b.M, b.N, b.K, G, 3);
  };
  auto best = [&](int G) { return std::min(pair_makespan(a, b, G), separate(G)); };
  const int G = L.all_sms > L.num_sms ? pick_sms(L.num_sms, L.all_sms, best) : L.num_sms;
  if (pair_off || pair_makespan(a, b, G) > separate(G)) {
    const int rc = tc_gemm_split(L, g0.A, g0.B, g0.E, g0.M, g0.N, g0.K, 3, s);
    return rc != kOk ? rc : tc_gemm_split(L, g1.A, g1.B, g1.E, g1.M, g1.N, g1.K, 3, s);
  }
  CUtensorMap ma[4] = {}, mb[4] = {};
  TcParams pa{}, pb{};
  int rc = tc_prepare(L, a.A, a.B, a.E, a.M, a.N, a.K, 3, s, ma, pa);
  if (rc != kOk) return rc;
  rc = tc_prepare(L, b.A, b.B, b.E, b.M, b.N, b.K, 3, s, mb, pb);
  if (rc != kOk) return rc;
  pa.pair_tiles = pb.num_tiles;
  const int total = pa.num_tiles + pb.num_tiles;
  const int grid = std::min(G, total);
  const cudaError_t e = fn(ma, mb, pa, pb, grid, s);
  return e == cudaSuccess ? kOk : cuda_status(e);
}

size_t tc_colsum_scratch_bytes(int M, int N) {
  if (M <= 0 || N <= 0) return 0;
  const size_t tiles_m = (M + kBM - 1) / kBM, tiles_n = (N + kBN - 1) / kBN;
  return align256(sizeof(float) * tiles_m * N) + align256(sizeof(int) * tiles_n);
}

void tc_split_plan(int M, int N, int K, int num_sms, int passes, int32_t* out) {
  const SplitPlan sp = plan_split(M, N, K, num_sms, passes);
  out[0] = sp.mode;
  out[1] = sp.tile0;
  out[2] = sp.r;
  out[3] = sp.kp;
  out[4] = sp.s;
  out[5] = sp.j;
}

int tc_launch_sms(int M, int N, int K, int budget, int all, int passes) {
  if (M <= 0 || N <= 0 || K <= 0) return budget;
  return pick_sms(budget, all, [&](int G) { return gemm_makespan(M, N, K, G, passes); });
}

size_t tc_streamk_bytes(int M, int N, int K, int num_sms, int passes) {
  const SplitPlan sp = plan_split(M, N, K, num_sms, passes);
  if (sp.mode == 0) return 0;
  const int tiles = ((M + kBM - 1) / kBM) * ((N + kBN - 1) / kBN);
  return sp.slots * kBM * kBN * 4 + align256(sizeof(int) * tiles);
}

int split_tf32(Context* ctx, const float* src, int64_t ld, int rows, int cols, float* hi,
               float* lo, int64_t ld_out, cudaStream_t s) {
  if (rows <= 0 || cols <= 0) return kOk;
  // a row-major [rows][cols] matrix is its own K-contiguous view (R=rows, K=cols)
  return cuda_status(launch_split(src, ld, true, rows, cols, ld_out, hi, lo, ctx->num_sms, s));
}

int tc_gemm(Context* ctx, const GemmArgs& g, int passes, cudaStream_t s) {
  if (g.M == 0 || g.N == 0) return kOk;
  if (g.K == 0) return simt_gemm(ctx, g, s);
  if (passes != 1 && passes != 3) return kErrInvalid;
  // Plain TF32 reads the caller's operands as they are stored when TMA can
  // (16-byte aligned bases, leading dimensions a multiple of 4 floats): the
  // tensor cores take the fp32 bit patterns and use their TF32 part, so no
  // rounded copies are made (cuBLAS's TF32 mode likewise).
  const bool direct = passes == 1 && g.lda % 4 == 0 && g.ldb % 4 == 0 &&
                      ((reinterpret_cast<uintptr_t>(g.a) | reinterpret_cast<uintptr_t>(g.b)) &
                       15u) == 0;
  if (direct) {
    const size_t sk = tc_split_scratch(ctx, g.M, g.N, g.K, 1);
    int rc = sk > 0 ? ensure_workspace(ctx, sk) : kOk;
    if (rc != kOk) return rc;
    TcLaunch L{ctx->tc_sms(), ctx->status, ctx->timeout_ns};
    L.all_sms = ctx->tc_all();
    L.sched = ctx->sched;
    L.ws = ctx->workspace;
    L.ws_bytes = sk > 0 ? ctx->ws_bytes : 0;
    SplitOperand A{g.a, nullptr, g.lda, g.ta == 0, false}, B{g.b, nullptr, g.ldb, g.tb != 0, false};
    TcEpilogue E{};
    E.c = g.c; E.ldc = g.ldc; E.alpha = g.alpha; E.beta = g.beta; E.bias = g.bias;
    E.relu = g.relu;
    return tc_gemm_split(L, A, B, E, g.M, g.N, g.K, 1, s);
  }
  const CopyShape ca = copy_shape(g.ta == 0, g.M, g.K), cb = copy_shape(g.tb != 0, g.N, g.K);
  const size_t split_bytes = tc_gemm_workspace_bytes(g, passes);
  const size_t sk_bytes = tc_split_scratch(ctx, g.M, g.N, g.K, passes);
  int rc = ensure_workspace(ctx, split_bytes + sk_bytes);
  if (rc != kOk) return rc;
  uint8_t* ws = static_cast<uint8_t*>(ctx->workspace);
  float* a_hi = reinterpret_cast<float*>(ws);
  ws += ca.bytes;
  float* b_hi = reinterpret_cast<float*>(ws);
  ws += cb.bytes;
  float* a_lo = nullptr;
  float* b_lo = nullptr;
  if (passes == 3) {
    a_lo = reinterpret_cast<float*>(ws);
    ws += ca.bytes;
    b_lo = reinterpret_cast<float*>(ws);
  }
  // elementwise split in the stored layout: [rows][K] or [K][rows]
  cudaError_t e = ca.kmajor
      ? launch_split(g.a, g.lda, true, g.M, g.K, ca.ld, a_hi, a_lo, ctx->num_sms, s)
      : launch_split(g.a, g.lda, true, g.K, g.M, ca.ld, a_hi, a_lo, ctx->num_sms, s);
  if (e != cudaSuccess) return cuda_status(e);
  e = cb.kmajor ? launch_split(g.b, g.ldb, true, g.N, g.K, cb.ld, b_hi, b_lo, ctx->num_sms, s)
                : launch_split(g.b, g.ldb, true, g.K, g.N, cb.ld, b_hi, b_lo, ctx->num_sms, s);
  if (e != cudaSuccess) return cuda_status(e);
  TcLaunch L{ctx->tc_sms(), ctx->status, ctx->timeout_ns};
  L.all_sms = ctx->tc_all();
  L.sched = ctx->sched;
  L.ws = static_cast<uint8_t*>(ctx->workspace) + split_bytes;  // split_bytes is 256-aligned
  L.ws_bytes = sk_bytes;
  SplitOperand A{a_hi, a_lo, ca.ld, ca.kmajor, !ca.kmajor},
      B{b_hi, b_lo, cb.ld, cb.kmajor, !cb.kmajor};
  TcEpilogue E{};
  E.c = g.c; E.ldc = g.ldc; E.alpha = g.alpha; E.beta = g.beta; E.bias = g.bias; E.relu = g.relu;
  return tc_gemm_split(L, A, B, E, g.M, g.N, g.K, passes, s);
}

}  // namespace mx

// ===========================================================================
// Allocation-free entry point: mx_gemm_3xtf32_noalloc.
//
// Some callers may not allocate device memory at all: a host runtime that
// reserved its whole device-memory budget up front and hands out slices of
// it itself (the reference GPU backend does this with one cudaMalloc'd bump
// pool, moonxi-net-gpu/cuda/cuda_kernels.cu:922-1004), or a process that
// runs under a fixed memory budget where a hidden cudaMalloc inside a library
// call could fail or evict someone else.  The regular entry points grow a
// per-context workspace with cudaMalloc the first time a large shape needs
// it; this one never does.  Its scratch (the hi/lo split copies of A and B)
// lives in a fixed-size array compiled into this library, which every GPU
// that loads the library holds until the process exits.
// ===========================================================================
namespace mx {
namespace {

// Upper bound of the split-operand scratch: 64 MiB, i.e. roughly
// (M + N) * K <= 8 Mi elements (2048^3 fits; the exact check is below).
constexpr size_t kNoAllocScratchBytes = 64ull << 20;

__device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
__device__ __align__(256) int g_noalloc_status[2];

struct NoAllocDevice {
  bool ready = false;
  uint8_t* scratch = nullptr;  // device address of g_noalloc_scratch
  int* status = nullptr;       // device address of g_noalloc_status
  int num_sms = 0;
};
std::mutex g_noalloc_mu;
NoAllocDevice g_noalloc_dev[64];

// Once per device, with that device current: resolve the device addresses of
// the static arrays.  In host code the array names are host-side stand-ins,
// not device addresses, so kernels only ever receive these resolved pointers.
int noalloc_setup(NoAllocDevice** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_status(e);
  if (dev < 0 || dev >= 64) return kErrUnsupported;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  NoAllocDevice& d = g_noalloc_dev[dev];
  if (!d.ready) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) return cuda_status(e);
    d.scratch = static_cast<uint8_t*>(p);
    e = cudaGetSymbolAddress(&p, g_noalloc_status);
    if (e != cudaSuccess) return cuda_status(e);
    d.status = static_cast<int*>(p);
    e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_status(e);
    d.ready = true;
  }
  *out = &d;
  return kOk;
}

}  // namespace
}  // namespace mx

extern "C" __attribute__((visibility("default"))) int32_t mx_gemm_3xtf32_noalloc(
    const float* a, const float* b, float* c, const float* bias, int32_t M, int32_t K,
    int32_t N, int32_t transpose_a, int32_t transpose_b, float alpha, float beta, int32_t relu,
    int32_t* dev_status, void* stream) {
  using namespace mx;
  if (M < 0 || N < 0 || K < 0) return kErrInvalid;
  if (M == 0 || N == 0) return kOk;
  if (!c || ((!a || !b) && K > 0)) return kErrInvalid;
  GemmArgs g;
  g.a = a; g.b = b; g.c = c;
  g.M = M; g.K = K; g.N = N;
  g.ta = transpose_a ? 1 : 0; g.tb = transpose_b ? 1 : 0;
  g.lda = g.ta ? M : K;   // packed leading dimensions, as cuda_matmul
  g.ldb = g.tb ? K : N;
  g.ldc = N;
  g.alpha = alpha; g.beta = beta; g.bias = bias; g.relu = relu ? 1 : 0;
  const size_t need = kmajor_split_bytes(g, 3);
  if (need > kNoAllocScratchBytes) return kErrUnsupported;  // beyond the static scratch
  NoAllocDevice* d = nullptr;
  int rc = noalloc_setup(&d);
  if (rc != kOk) return rc;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* status = dev_status ? reinterpret_cast<int*>(dev_status) : d->status;

  if (K == 0) {  // no product: the SIMT epilogue computes beta*C + bias, no scratch
    Context local;
    local.num_sms = d->num_sms;
    local.status = status;
    return simt_gemm_launch(&local, g, s, nullptr, 0);
  }
  const int64_t Kp = (static_cast<int64_t>(K) + 3) & ~static_cast<int64_t>(3);
  uint8_t* ws = d->scratch;  // K-major copies of both operands (kmajor_split_bytes)
  float* a_hi = reinterpret_cast<float*>(ws);
  ws += align256(static_cast<size_t>(M) * Kp * 4);
  float* b_hi = reinterpret_cast<float*>(ws);
  ws += align256(static_cast<size_t>(N) * Kp * 4);
  float* a_lo = reinterpret_cast<float*>(ws);
  ws += align256(static_cast<size_t>(M) * Kp * 4);
  float* b_lo = reinterpret_cast<float*>(ws);
  // The split kernels overwrite every scratch element the main kernel reads
  // (columns [K, Kp) are outside the tensor maps), so nothing needs clearing.
  cudaError_t e = launch_split(a, g.lda, g.ta == 0, M, K, Kp, a_hi, a_lo, d->num_sms, s);
  if (e != cudaSuccess) return cuda_status(e);
  e = launch_split(b, g.ldb, g.tb != 0, N, K, Kp, b_hi, b_lo, d->num_sms, s);
  if (e != cudaSuccess) return cuda_status(e);
  CUtensorMap tah{}, tal{}, tbh{}, tbl{};
  const bool ok =
      make_tmap_2d(&tah, a_hi, K, M, Kp * 4, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_tmap_2d(&tbh, b_hi, K, N, Kp * 4, kBK, kBN, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_tmap_2d(&tal, a_lo, K, M, Kp * 4, kBK, kBM, CU_TENSOR_MAP_SWIZZLE_64B) &&
      make_tmap_2d(&tbl, b_lo, K, N, Kp * 4, kBK, kBN, CU_TENSOR_MAP_SWIZZLE_64B);
  if (!ok) return kErrUnsupported;
  TcParams p{};
  p.c = c; p.bias = bias; p.status = status; p.ldc = g.ldc;
  p.M = M; p.N = N; p.K = K;
  p.tiles_m = (M + kBM - 1) / kBM;
  p.tiles_n = (N + kBN - 1) / kBN;
  p.num_tiles = p.tiles_m * p.tiles_n;
  p.alpha = alpha; p.beta = beta; p.relu = g.relu;
  p.timeout_ns = 2000000000ull;
  e = launch_tc<3, true, true>(tah, tal, tbh, tbl, p, std::min(p.num_tiles, d->num_sms), s);
  return e == cudaSuccess ? kOk : cuda_status(e);
}

// Reads and clears the library's own status word of the allocation-free
// entry point on the current device (the word its kernels write when the
// caller passes no dev_status).  Synchronises the device first.  No
// allocation: the word is part of the same static data as the scratch.
extern "C" __attribute__((visibility("default"))) int32_t mx_noalloc_status(int32_t* where) {
  using namespace mx;
  NoAllocDevice* d = nullptr;
  int rc = noalloc_setup(&d);
  if (rc != kOk) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_status(e);
  int st[2] = {0, 0};
  e = cudaMemcpy(st, d->status, sizeof(st), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_status(e);
  if (where) *where = st[1];
  if (st[0] != 0) {
    e = cudaMemset(d->status, 0, sizeof(st));
    if (e != cudaSuccess) return cuda_status(e);
  }
  return st[0];
}
