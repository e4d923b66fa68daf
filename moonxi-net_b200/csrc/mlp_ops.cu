// mlp_ops.cu -- the non-GEMM steps of one Linear/MLP training step, written
// so none of them needs a host round trip:
//   relu_backward        (replaces cuDNN ReLU backward, cuda_kernels.cu:812-831)
//   reduce_sum_leading   (bias gradient, replaces cuda_kernels.cu:1383-1406)
//   softmax_ce_labels    (loss + dlogits in one pass, replaces :1283-1374)
//   sgd_momentum_autoclip over one flat parameter buffer (replaces the
//                        pointer-table mt_norm_sq / mt_sgd_momentum_autoclip,
//                        cuda_kernels.cu:1884-2029)
// Reductions use a fixed order (no atomics), so every result is
// run-to-run deterministic.  Arithmetic that NpArray performs as separate
// fp32 multiply and add uses __fmul_rn/__fadd_rn so nvcc cannot fuse it.
#include <algorithm>

#include "../../include/mx_matmul.h"
#include "mx_internal.h"
#include "mx_ptx.cuh"

namespace mx {
namespace {

__global__ void relu_backward_kernel(const float* __restrict__ g, const float* __restrict__ x,
                                     float* __restrict__ out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const int64_t n4 = ((reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(x) |
                       reinterpret_cast<uintptr_t>(out)) & 15u) == 0 ? n / 4 : 0;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += stride) {
    const float4 gv = reinterpret_cast<const float4*>(g)[i];
    const float4 xv = reinterpret_cast<const float4*>(x)[i];
    float4 o;
    o.x = xv.x > 0.0f ? gv.x : 0.0f;
    o.y = xv.y > 0.0f ? gv.y : 0.0f;
    o.z = xv.z > 0.0f ? gv.z : 0.0f;
    o.w = xv.w > 0.0f ? gv.w : 0.0f;
    reinterpret_cast<float4*>(out)[i] = o;
  }
  for (int64_t i = n4 * 4 + blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += stride)
    out[i] = x[i] > 0.0f ? g[i] : 0.0f;
}

// Column sums of in[rows][cols]: block = 32 columns x 8 row lanes; each
// lane sums rows lane, lane+8, ... in order, then the 8 lane sums are added
// in a fixed tree.
__global__ void reduce_leading_kernel(const float* __restrict__ in, float* __restrict__ out,
                                      int cols, int rows) {
  __shared__ float part[8][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;
  const int col = blockIdx.x * 32 + tx;
  float s0 = 0.0f, s1 = 0.0f;
  if (col < cols) {
    int r = ty;
    for (; r + 8 < rows; r += 16) {
      s0 += in[static_cast<int64_t>(r) * cols + col];
      s1 += in[static_cast<int64_t>(r + 8) * cols + col];
    }
    if (r < rows) s0 += in[static_cast<int64_t>(r) * cols + col];
  }
  part[ty][tx] = s0 + s1;
  __syncthreads();
  if (ty == 0 && col < cols) {
    const float a = (part[0][tx] + part[1][tx]) + (part[2][tx] + part[3][tx]);
    const float b = (part[4][tx] + part[5][tx]) + (part[6][tx] + part[7][tx]);
    out[col] = a + b;
  }
}

// Two-pass column sums for wide, 16-byte aligned inputs: pass 1 has block
// (128 columns as float4 x 8 row lanes) per (column block, row split) and
// writes one partial row per split; pass 2 adds the splits in order.  Every
// sum has a fixed order, so the result is deterministic.
__global__ void reduce_leading_part_kernel(const float* __restrict__ in,
                                           float* __restrict__ partial, int cols, int rows,
                                           int rows_per) {
  __shared__ float4 part[8][33];
  const int q = threadIdx.x & 31, lr = threadIdx.x >> 5;
  const int col = blockIdx.x * 128 + q * 4;
  const int r0 = blockIdx.y * rows_per;
  const int r1 = min(rows, r0 + rows_per);
  float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (col < cols) {
    for (int r = r0 + lr; r < r1; r += 8) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(in + static_cast<int64_t>(r) * cols + col));
      s.x += v.x;
      s.y += v.y;
      s.z += v.z;
      s.w += v.w;
    }
  }
  part[lr][q] = s;
  __syncthreads();
  if (lr == 0 && col < cols) {
    float4 t = part[0][q];
#pragma unroll
    for (int k = 1; k < 8; ++k) {
      t.x += part[k][q].x;
      t.y += part[k][q].y;
      t.z += part[k][q].z;
      t.w += part[k][q].w;
    }
    *reinterpret_cast<float4*>(partial + static_cast<int64_t>(blockIdx.y) * cols + col) = t;
  }
}

__global__ void reduce_leading_finish_kernel(const float* __restrict__ partial,
                                             float* __restrict__ out, int cols, int splits) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= cols) return;
  float s = 0.0f;
  for (int k = 0; k < splits; ++k) s += partial[static_cast<int64_t>(k) * cols + col];
  out[col] = s;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// Class index of a label stored as a float.  A label outside [0, C) (or NaN)
// would index past the logits row: it records MX_ERR_INVALID with call site
// `where` in the status word and returns -1 (the row then gets no one-hot
// term and a NaN loss).  The reference reads such a row out of bounds.
__device__ __forceinline__ int checked_label(float lf, int C, int* status, int where) {
  if (lf >= 0.0f && lf < static_cast<float>(C)) return static_cast<int>(lf);
  if (status) {
    atomicCAS(status, kOk, kErrInvalid);
    atomicCAS(status + 1, 0, where);
  }
  return -1;
}

// One warp per row; 8 rows per block.  exp/log are evaluated in double and
// rounded to float, as NpArray does (image_impl.mbt:95-103).  Writes the
// block's partial loss (sum of its rows' -log p[label]) to partial[block].
__global__ void softmax_ce_kernel(const float* __restrict__ logits,
                                  const float* __restrict__ labels, float* __restrict__ grad,
                                  float* __restrict__ g_hi, float* __restrict__ g_lo,
                                  float* __restrict__ partial, int batch, int C, float denom,
                                  int* __restrict__ status) {
  __shared__ float row_loss[8];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + warp;
  float loss = 0.0f;
  if (b < batch) {
    const float* row = logits + static_cast<int64_t>(b) * C;
    const int label = checked_label(labels[b], C, status, 301);
    float mx_ = -INFINITY;
    for (int j = lane; j < C; j += 32) mx_ = fmaxf(mx_, row[j]);
    mx_ = warp_max(mx_);
    float se = 0.0f;
    for (int j = lane; j < C; j += 32)
      se = __fadd_rn(se, static_cast<float>(exp(static_cast<double>(__fsub_rn(row[j], mx_)))));
    se = warp_sum(se);
    const float lse = static_cast<float>(log(static_cast<double>(se)));
    if (lane == 0) {
      // an out-of-range label has no log-probability: the row's loss is NaN
      // (and the status word says why)
      loss = label >= 0 ? -__fsub_rn(__fsub_rn(row[label], mx_), lse) : __int_as_float(0x7fc00000);
    }
    if (grad) {
      float* g = grad + static_cast<int64_t>(b) * C;
      for (int j = lane; j < C; j += 32) {
        const float sm =
            __fdiv_rn(static_cast<float>(exp(static_cast<double>(__fsub_rn(row[j], mx_)))), se);
        const float t = (j == label) ? 1.0f : 0.0f;
        const float gv = __fdiv_rn(__fsub_rn(sm, t), denom);
        g[j] = gv;
        if (g_hi) {  // 3xTF32 split of the gradient for the backward GEMMs
          const int64_t o = static_cast<int64_t>(b) * C + j;
          const float h = __uint_as_float(f32_to_tf32_rna(gv));
          g_hi[o] = h;
          g_lo[o] = __uint_as_float(f32_to_tf32_rna(gv - h));
        }
      }
    }
  }
  if (lane == 0) row_loss[warp] = loss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int w = 0; w < 8; ++w) s = __fadd_rn(s, row_loss[w]);
    partial[blockIdx.x] = s;
  }
}

// softmax_ce_kernel that also produces the column sums of the gradient,
// colsum[j] = sum_b grad[b, j] (the output layer's bias gradient,
// reduce_sum_to of grad/grad.mbt:163-174, which the reference runs as a
// separate kernel, cuda_kernels.cu:1383-1406).  Each block stages its 8
// gradient rows in shared memory ([8][C]) and writes their sum (fixed order)
// to part[block]; the last block of each group of 32 to arrive adds the
// group's rows in order into part2[group]; the last group adds the groups in
// order into colsum.  The result does not depend on arrival order.  Counters
// cnt[groups + 1] are zero at launch and left zero.
constexpr int kCeGroup = 32;

__global__ void softmax_ce_colsum_kernel(const float* __restrict__ logits,
                                         const float* __restrict__ labels,
                                         float* __restrict__ grad, float* __restrict__ g_hi,
                                         float* __restrict__ g_lo, float* __restrict__ partial,
                                         int batch, int C, float denom, int* __restrict__ status,
                                         float* __restrict__ colsum, float* __restrict__ part,
                                         float* __restrict__ part2, int* __restrict__ cnt) {
  extern __shared__ float rows_s[];  // [8][C]
  __shared__ float row_loss[8];
  __shared__ int last;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 8 + warp;
  float* my_row = rows_s + warp * C;
  float loss = 0.0f;
  if (b < batch) {
    const float* row = logits + static_cast<int64_t>(b) * C;
    const int label = checked_label(labels[b], C, status, 303);
    float mx_ = -INFINITY;
    for (int j = lane; j < C; j += 32) mx_ = fmaxf(mx_, row[j]);
    mx_ = warp_max(mx_);
    float se = 0.0f;
    for (int j = lane; j < C; j += 32)
      se = __fadd_rn(se, static_cast<float>(exp(static_cast<double>(__fsub_rn(row[j], mx_)))));
    se = warp_sum(se);
    const float lse = static_cast<float>(log(static_cast<double>(se)));
    if (lane == 0)
      loss = label >= 0 ? -__fsub_rn(__fsub_rn(row[label], mx_), lse) : __int_as_float(0x7fc00000);
    float* g = grad + static_cast<int64_t>(b) * C;
    for (int j = lane; j < C; j += 32) {
      const float sm =
          __fdiv_rn(static_cast<float>(exp(static_cast<double>(__fsub_rn(row[j], mx_)))), se);
      const float gv = __fdiv_rn(__fsub_rn(sm, (j == label) ? 1.0f : 0.0f), denom);
      g[j] = gv;
      my_row[j] = gv;
      if (g_hi) {
        const int64_t o = static_cast<int64_t>(b) * C + j;
        const float h = __uint_as_float(f32_to_tf32_rna(gv));
        g_hi[o] = h;
        g_lo[o] = __uint_as_float(f32_to_tf32_rna(gv - h));
      }
    }
  } else {
    for (int j = lane; j < C; j += 32) my_row[j] = 0.0f;
  }
  if (lane == 0) row_loss[warp] = loss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float s = 0.0f;
    for (int w = 0; w < 8; ++w) s = __fadd_rn(s, row_loss[w]);
    partial[blockIdx.x] = s;
  }
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    float s = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) s += rows_s[w * C + j];
    part[static_cast<int64_t>(blockIdx.x) * C + j] = s;
  }
  // level 1: the group's last block adds the group's partial rows
  const int group = blockIdx.x / kCeGroup;
  const int g0 = group * kCeGroup;
  const int gn = min(kCeGroup, static_cast<int>(gridDim.x) - g0);
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&cnt[group], 1);
    last = old == gn - 1;
    if (last) cnt[group] = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    float s = 0.0f;
    for (int r = g0; r < g0 + gn; ++r) s += __ldcg(part + static_cast<int64_t>(r) * C + j);
    part2[static_cast<int64_t>(group) * C + j] = s;
  }
  // level 2: the last group adds the groups' rows
  const int groups = (gridDim.x + kCeGroup - 1) / kCeGroup;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int old = atomicAdd(&cnt[groups], 1);
    last = old == groups - 1;
    if (last) cnt[groups] = 0;
  }
  __syncthreads();
  if (!last) return;
  __threadfence();
  for (int j = threadIdx.x; j < C; j += blockDim.x) {
    float s = 0.0f;
    for (int r = 0; r < groups; ++r) s += __ldcg(part2 + static_cast<int64_t>(r) * C + j);
    colsum[j] = s;
  }
}

// Sums n partials in a fixed order with one block, then
// mode 0: out[0] = sum / denom;  1: out[0] = sqrt(sum);  2: out[0] += sum.
__global__ void finish_sum_kernel(const float* __restrict__ partial, int n, float denom,
                                  float* __restrict__ out, int mode) {
  __shared__ float sh[256];
  float s = 0.0f;
  for (int i = threadIdx.x; i < n; i += 256) s = __fadd_rn(s, partial[i]);
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) sh[threadIdx.x] = __fadd_rn(sh[threadIdx.x], sh[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    const float v = sh[0];
    out[0] = mode == 1 ? __fsqrt_rn(v) : mode == 2 ? __fadd_rn(out[0], v) : __fdiv_rn(v, denom);
  }
}

// Per-block partial of sum g^2 over a grid-stride range (fixed grid -> fixed order).
__global__ void norm_sq_kernel(const float* __restrict__ g, int64_t n, float* __restrict__ partial) {
  __shared__ float sh[256];
  float s = 0.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride)
    s = __fadd_rn(s, __fmul_rn(g[i], g[i]));
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) sh[threadIdx.x] = __fadd_rn(sh[threadIdx.x], sh[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = sh[0];
}

// v = momentum*v + g*clip + wd*p ; p = p - lr*v  (nparray/trait_impl.mbt:298-308).
__global__ void sgd_update_kernel(float* __restrict__ p, const float* __restrict__ g,
                                  float* __restrict__ v, int64_t n, float lr, float momentum,
                                  float wd, float max_norm, const float* __restrict__ norm,
                                  float* __restrict__ p_hi, float* __restrict__ p_lo,
                                  int norm_is_sq) {
  const float nv = norm_is_sq ? __fsqrt_rn(*norm) : *norm;
  const float clip = nv > max_norm ? __fdiv_rn(max_norm, nv) : 1.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n; i += stride) {
    const float cg = __fmul_rn(g[i], clip);
    const float vn = __fadd_rn(__fadd_rn(__fmul_rn(momentum, v[i]), cg), __fmul_rn(wd, p[i]));
    v[i] = vn;
    const float pn = __fsub_rn(p[i], __fmul_rn(lr, vn));
    p[i] = pn;
    if (p_hi) {  // 3xTF32 split of the updated parameters for the next step
      const float h = __uint_as_float(f32_to_tf32_rna(pn));
      p_hi[i] = h;
      p_lo[i] = __uint_as_float(f32_to_tf32_rna(pn - h));
    }
  }
}

// float4 forms of the two passes above (same per-element arithmetic), for
// 16-byte aligned buffers whose length is a multiple of 4: four times fewer
// memory instructions, so the passes run at HBM speed.
__global__ void norm_sq4_kernel(const float4* __restrict__ g, int64_t n4,
                                float* __restrict__ partial) {
  __shared__ float sh[256];
  float s = 0.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += stride) {
    const float4 v = __ldg(g + i);
    s = __fadd_rn(s, __fmul_rn(v.x, v.x));
    s = __fadd_rn(s, __fmul_rn(v.y, v.y));
    s = __fadd_rn(s, __fmul_rn(v.z, v.z));
    s = __fadd_rn(s, __fmul_rn(v.w, v.w));
  }
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int w = 128; w > 0; w >>= 1) {
    if (threadIdx.x < w) sh[threadIdx.x] = __fadd_rn(sh[threadIdx.x], sh[threadIdx.x + w]);
    __syncthreads();
  }
  if (threadIdx.x == 0) partial[blockIdx.x] = sh[0];
}

__device__ __forceinline__ void sgd_one(float& p, float g, float& v, float lr, float momentum,
                                        float wd, float clip) {
  const float cg = __fmul_rn(g, clip);
  v = __fadd_rn(__fadd_rn(__fmul_rn(momentum, v), cg), __fmul_rn(wd, p));
  p = __fsub_rn(p, __fmul_rn(lr, v));
}

__global__ void sgd_update4_kernel(float4* __restrict__ p, const float4* __restrict__ g,
                                   float4* __restrict__ v, int64_t n4, float lr, float momentum,
                                   float wd, float max_norm, const float* __restrict__ norm,
                                   float4* __restrict__ p_hi, float4* __restrict__ p_lo,
                                   int norm_is_sq) {
  const float nv = norm_is_sq ? __fsqrt_rn(*norm) : *norm;
  const float clip = nv > max_norm ? __fdiv_rn(max_norm, nv) : 1.0f;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n4;
       i += stride) {
    float4 pp = p[i], vv = v[i];
    const float4 gg = __ldg(g + i);
    sgd_one(pp.x, gg.x, vv.x, lr, momentum, wd, clip);
    sgd_one(pp.y, gg.y, vv.y, lr, momentum, wd, clip);
    sgd_one(pp.z, gg.z, vv.z, lr, momentum, wd, clip);
    sgd_one(pp.w, gg.w, vv.w, lr, momentum, wd, clip);
    v[i] = vv;
    p[i] = pp;
    if (p_hi) {
      float4 h, l;
      h.x = __uint_as_float(f32_to_tf32_rna(pp.x));
      h.y = __uint_as_float(f32_to_tf32_rna(pp.y));
      h.z = __uint_as_float(f32_to_tf32_rna(pp.z));
      h.w = __uint_as_float(f32_to_tf32_rna(pp.w));
      l.x = __uint_as_float(f32_to_tf32_rna(pp.x - h.x));
      l.y = __uint_as_float(f32_to_tf32_rna(pp.y - h.y));
      l.z = __uint_as_float(f32_to_tf32_rna(pp.z - h.z));
      l.w = __uint_as_float(f32_to_tf32_rna(pp.w - h.w));
      p_hi[i] = h;
      p_lo[i] = l;
    }
  }
}

// ---- NpArray-order variants (contexts in MX_PREC_NPARRAY mode): the same
// sequential fp32 loops as the CPU path, so results are bit-identical to it.

// reduce_sum_to [rows, cols] -> [cols] (nparray/trait_impl.mbt:128-138):
// one thread per column, rows ascending.
__global__ void reduce_leading_seq_kernel(const float* __restrict__ in, float* __restrict__ out,
                                          int cols, int rows) {
  const int col = blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= cols) return;
  float s = 0.0f;
  for (int r = 0; r < rows; ++r) s = __fadd_rn(s, in[static_cast<int64_t>(r) * cols + col]);
  out[col] = s;
}

// cross_entropy_with_labels + softmax_ce_backward_labels
// (nparray/image_impl.mbt:83-114, 202-238): one thread per row, classes
// ascending; row_loss[b] = -log p[label].
__global__ void softmax_ce_seq_kernel(const float* __restrict__ logits,
                                      const float* __restrict__ labels, float* __restrict__ grad,
                                      float* __restrict__ row_loss, int batch, int C, float denom,
                                      int* __restrict__ status) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= batch) return;
  const float* row = logits + static_cast<int64_t>(b) * C;
  const int label = checked_label(labels[b], C, status, 302);
  float mx_ = row[0];
  for (int j = 1; j < C; ++j)
    if (row[j] > mx_) mx_ = row[j];
  float se = 0.0f;
  for (int j = 0; j < C; ++j)
    se = __fadd_rn(se, static_cast<float>(exp(static_cast<double>(__fsub_rn(row[j], mx_)))));
  const float lse = static_cast<float>(log(static_cast<double>(se)));
  row_loss[b] = label >= 0 ? -__fsub_rn(__fsub_rn(row[label], mx_), lse)
                           : __int_as_float(0x7fc00000);
  if (grad) {
    float* g = grad + static_cast<int64_t>(b) * C;
    for (int j = 0; j < C; ++j) {
      const float sm =
          __fdiv_rn(static_cast<float>(exp(static_cast<double>(__fsub_rn(row[j], mx_)))), se);
      g[j] = __fdiv_rn(__fsub_rn(sm, j == label ? 1.0f : 0.0f), denom);
    }
  }
}

// One thread, elements ascending.  mode 0: out = (sum v) / denom;
// mode 1: out = sqrt(sum v*v) (the optimizer's global norm,
// nparray/trait_impl.mbt:288-295).
__global__ void seq_sum_kernel(const float* __restrict__ v, int64_t n, float denom,
                               float* __restrict__ out, int mode) {
  if (blockIdx.x != 0 || threadIdx.x != 0) return;
  float s = 0.0f;
  if (mode == 0) {
    for (int64_t i = 0; i < n; ++i) s = __fadd_rn(s, v[i]);
    out[0] = __fdiv_rn(s, denom);
  } else {
    for (int64_t i = 0; i < n; ++i) s = __fadd_rn(s, __fmul_rn(v[i], v[i]));
    out[0] = __fsqrt_rn(s);
  }
}

bool nparray_order(const Context* ctx) { return ctx->precision == MX_PREC_NPARRAY; }

int grid_for(int64_t n, int num_sms, int per_sm = 8) {
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, num_sms * per_sm)));
}

}  // namespace

int relu_backward(Context* ctx, const float* g, const float* x, float* out, int64_t n,
                  cudaStream_t s) {
  if (n <= 0) return kOk;
  relu_backward_kernel<<<grid_for((n + 3) / 4, ctx->num_sms), 256, 0, s>>>(g, x, out, n);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

int reduce_sum_leading(Context* ctx, const float* in, float* out, int cols, int rows,
                       cudaStream_t s) {
  if (cols <= 0) return kOk;
  if (nparray_order(ctx)) {
    reduce_leading_seq_kernel<<<(cols + 127) / 128, 128, 0, s>>>(in, out, cols, rows);
    note_launches(1);
    return cuda_status(cudaGetLastError());
  }
  const bool vec = cols % 4 == 0 && (reinterpret_cast<uintptr_t>(in) & 15u) == 0;
  const int col_blocks = (cols + 127) / 128;
  int splits = std::min((4 * ctx->num_sms + col_blocks - 1) / col_blocks, rows / 64);
  if (!vec || splits < 2) {
    reduce_leading_kernel<<<(cols + 31) / 32, 256, 0, s>>>(in, out, cols, rows);
    note_launches(1);
    return cuda_status(cudaGetLastError());
  }
  splits = std::min(splits, 64);
  int rc = ensure_small_scratch(ctx, static_cast<size_t>(splits) * cols * sizeof(float));
  if (rc != kOk) return rc;
  float* partial = static_cast<float*>(ctx->small_scratch);
  const int rows_per = (rows + splits - 1) / splits;
  reduce_leading_part_kernel<<<dim3(col_blocks, splits), 256, 0, s>>>(in, partial, cols, rows,
                                                                       rows_per);
  reduce_leading_finish_kernel<<<(cols + 255) / 256, 256, 0, s>>>(partial, out, cols, splits);
  note_launches(2);
  return cuda_status(cudaGetLastError());
}

int softmax_ce_labels(Context* ctx, const float* logits, const float* labels, float* grad,
                      float* loss, int batch, int C, int denom, cudaStream_t s, float* g_hi,
                      float* g_lo) {
  if (batch <= 0 || C <= 0) return kErrInvalid;
  if (nparray_order(ctx)) {
    int rc = ensure_small_scratch(ctx, static_cast<size_t>(batch) * sizeof(float));
    if (rc != kOk) return rc;
    float* row_loss = static_cast<float*>(ctx->small_scratch);
    softmax_ce_seq_kernel<<<(batch + 127) / 128, 128, 0, s>>>(
        logits, labels, grad, row_loss, batch, C, static_cast<float>(denom), ctx->status);
    note_launches(1);
    if (loss) {
      seq_sum_kernel<<<1, 1, 0, s>>>(row_loss, batch, static_cast<float>(denom), loss, 0);
      note_launches(1);
    }
    return cuda_status(cudaGetLastError());
  }
  const int blocks = (batch + 7) / 8;
  int rc = ensure_small_scratch(ctx, static_cast<size_t>(blocks) * sizeof(float));
  if (rc != kOk) return rc;
  float* partial = static_cast<float*>(ctx->small_scratch);
  softmax_ce_kernel<<<blocks, 256, 0, s>>>(logits, labels, grad, g_hi, g_lo, partial, batch, C,
                                           static_cast<float>(denom), ctx->status);
  note_launches(1);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e);
  if (loss) {
    finish_sum_kernel<<<1, 256, 0, s>>>(partial, blocks, static_cast<float>(denom), loss, 0);
    note_launches(1);
    e = cudaGetLastError();
  }
  return cuda_status(e);
}

// Largest class count the fused column sums stage in shared memory ([8][C]).
constexpr int kCeColsumMaxC = 4096;

size_t softmax_ce_colsum_scratch_bytes(int batch, int C) {
  if (batch <= 0 || C <= 0 || C > kCeColsumMaxC) return 0;
  const size_t blocks = (batch + 7) / 8;
  const size_t groups = (blocks + kCeGroup - 1) / kCeGroup;
  auto a256 = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  return a256(blocks * C * sizeof(float)) + a256(groups * C * sizeof(float)) +
         a256((groups + 1) * sizeof(int));
}

int softmax_ce_labels_colsum(Context* ctx, const float* logits, const float* labels, float* grad,
                             float* loss, int batch, int C, int denom, cudaStream_t s,
                             float* g_hi, float* g_lo, float* colsum, void* scratch,
                             size_t scratch_bytes) {
  if (batch <= 0 || C <= 0 || !grad || !colsum) return kErrInvalid;
  if (C > kCeColsumMaxC) return kErrUnsupported;
  if (!scratch || scratch_bytes < softmax_ce_colsum_scratch_bytes(batch, C)) return kErrInvalid;
  const int blocks = (batch + 7) / 8;
  const int groups = (blocks + kCeGroup - 1) / kCeGroup;
  auto a256 = [](size_t x) { return (x + 255) & ~static_cast<size_t>(255); };
  uint8_t* w = static_cast<uint8_t*>(scratch);
  float* part = reinterpret_cast<float*>(w);
  w += a256(static_cast<size_t>(blocks) * C * sizeof(float));
  float* part2 = reinterpret_cast<float*>(w);
  w += a256(static_cast<size_t>(groups) * C * sizeof(float));
  int* cnt = reinterpret_cast<int*>(w);
  int rc = ensure_small_scratch(ctx, static_cast<size_t>(blocks) * sizeof(float));
  if (rc != kOk) return rc;
  float* partial = static_cast<float*>(ctx->small_scratch);
  cudaError_t e = cudaMemsetAsync(cnt, 0, sizeof(int) * (groups + 1), s);
  if (e != cudaSuccess) return cuda_status(e);
  const int smem = 8 * C * static_cast<int>(sizeof(float));
  static SmemOptIn opt_in;
  e = opt_in.ensure(softmax_ce_colsum_kernel, 8 * kCeColsumMaxC * static_cast<int>(sizeof(float)));
  if (e != cudaSuccess) return cuda_status(e);
  softmax_ce_colsum_kernel<<<blocks, 256, smem, s>>>(logits, labels, grad, g_hi, g_lo, partial,
                                                     batch, C, static_cast<float>(denom),
                                                     ctx->status, colsum, part, part2, cnt);
  note_launches(1);
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_status(e);
  if (loss) {
    finish_sum_kernel<<<1, 256, 0, s>>>(partial, blocks, static_cast<float>(denom), loss, 0);
    note_launches(1);
    e = cudaGetLastError();
  }
  return cuda_status(e);
}

int sgd_momentum_autoclip(Context* ctx, float* p, const float* g, float* v, int64_t n, float lr,
                          float momentum, float wd, float max_norm, float* norm_out,
                          cudaStream_t s, float* p_hi, float* p_lo) {
  if (n <= 0) return kOk;
  const int blocks = grid_for(n, ctx->num_sms, 4);
  int rc = ensure_small_scratch(ctx, static_cast<size_t>(blocks + 1) * sizeof(float));
  if (rc != kOk) return rc;
  float* partial = static_cast<float*>(ctx->small_scratch);
  float* norm = norm_out ? norm_out : partial + blocks;
  const bool vec4 = n % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                      reinterpret_cast<uintptr_t>(v) | reinterpret_cast<uintptr_t>(p_hi) |
                      reinterpret_cast<uintptr_t>(p_lo)) & 15u) == 0;
  if (nparray_order(ctx)) {
    seq_sum_kernel<<<1, 1, 0, s>>>(g, n, 1.0f, norm, 1);
    note_launches(2);  // seq_sum, sgd_update
  } else {
    if (vec4)
      norm_sq4_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(g), n / 4, partial);
    else
      norm_sq_kernel<<<blocks, 256, 0, s>>>(g, n, partial);
    finish_sum_kernel<<<1, 256, 0, s>>>(partial, blocks, 1.0f, norm, 1);
    note_launches(3);  // norm_sq, finish_sum, sgd_update
  }
  if (vec4)
    sgd_update4_kernel<<<grid_for(n / 4, ctx->num_sms), 256, 0, s>>>(
        reinterpret_cast<float4*>(p), reinterpret_cast<const float4*>(g),
        reinterpret_cast<float4*>(v), n / 4, lr, momentum, wd, max_norm, norm,
        reinterpret_cast<float4*>(p_hi), reinterpret_cast<float4*>(p_lo), 0);
  else
    sgd_update_kernel<<<grid_for(n, ctx->num_sms), 256, 0, s>>>(p, g, v, n, lr, momentum, wd,
                                                                max_norm, norm, p_hi, p_lo, 0);
  return cuda_status(cudaGetLastError());
}

// Pieces of the data-parallel sharded update: the squared norm of one
// gradient range (accumulated over a rank's ranges, then all-reduced over the
// ranks by the caller) and the update of one range clipped by that norm.
int sum_squares(Context* ctx, const float* x, int64_t n, float* out, int accumulate,
                cudaStream_t s) {
  if (n <= 0) {
    if (!accumulate) return cuda_status(cudaMemsetAsync(out, 0, sizeof(float), s));
    return kOk;
  }
  const int blocks = grid_for(n, ctx->num_sms, 4);
  int rc = ensure_small_scratch(ctx, static_cast<size_t>(blocks) * sizeof(float));
  if (rc != kOk) return rc;
  float* partial = static_cast<float*>(ctx->small_scratch);
  if (n % 4 == 0 && (reinterpret_cast<uintptr_t>(x) & 15u) == 0)
    norm_sq4_kernel<<<blocks, 256, 0, s>>>(reinterpret_cast<const float4*>(x), n / 4, partial);
  else
    norm_sq_kernel<<<blocks, 256, 0, s>>>(x, n, partial);
  finish_sum_kernel<<<1, 256, 0, s>>>(partial, blocks, 1.0f, out, accumulate ? 2 : 0);
  note_launches(2);
  return cuda_status(cudaGetLastError());
}

int sgd_momentum_clip(Context* ctx, float* p, const float* g, float* v, int64_t n, float lr,
                      float momentum, float wd, float max_norm, const float* norm_sq,
                      cudaStream_t s) {
  if (n <= 0) return kOk;
  const bool vec4 = n % 4 == 0 &&
                    ((reinterpret_cast<uintptr_t>(p) | reinterpret_cast<uintptr_t>(g) |
                      reinterpret_cast<uintptr_t>(v)) & 15u) == 0;
  if (vec4)
    sgd_update4_kernel<<<grid_for(n / 4, ctx->num_sms), 256, 0, s>>>(
        reinterpret_cast<float4*>(p), reinterpret_cast<const float4*>(g),
        reinterpret_cast<float4*>(v), n / 4, lr, momentum, wd, max_norm, norm_sq, nullptr,
        nullptr, 1);
  else
    sgd_update_kernel<<<grid_for(n, ctx->num_sms), 256, 0, s>>>(
        p, g, v, n, lr, momentum, wd, max_norm, norm_sq, nullptr, nullptr, 1);
  note_launches(1);
  return cuda_status(cudaGetLastError());
}

}  // namespace mx
