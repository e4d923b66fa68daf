/*
 * np_oracle.c -- TEST INFRASTRUCTURE ONLY (the CPU oracle).
 *
 * A plain-C restatement of the moonxi-net NpArray CPU backend ops that sit on
 * the Linear/MLP dense-matmul path.  Only tests/, __graft_entry__.smoke() and
 * bench.py's cpu_baseline / `--impl reference` leg may load this library, and
 * only as the checker or the timed CPU baseline.  The product path never calls
 * it.
 *
 * Every function states the reference loop it follows (paths relative to the
 * moonxi-net project root).  Arithmetic is fp32 with the reference's operation
 * order; the file must be compiled WITHOUT -ffast-math and with
 * -ffp-contract=off so that every `sum = sum + a*b` stays a separate multiply
 * and add in the same k order.
 *
 * Multi-threading: the `nthreads` argument splits independent OUTPUT elements
 * across threads (row tiles for matmul, columns for reductions).  Each output
 * element is still produced by exactly the reference's sequential loop, so the
 * results are bit-identical to the single-threaded NpArray code.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define NP_EXPORT __attribute__((visibility("default")))

/* ------------------------------------------------------------------------ */
/* tiny fork/join helper                                                     */
/* ------------------------------------------------------------------------ */
typedef void (*np_range_fn)(void* ctx, int64_t begin, int64_t end);
typedef struct {
  np_range_fn fn;
  void* ctx;
  int64_t begin, end;
} np_job;

static void* np_job_run(void* p) {
  np_job* j = (np_job*)p;
  j->fn(j->ctx, j->begin, j->end);
  return NULL;
}

/* Runs fn over [0, n) split into `nthreads` contiguous chunks of `grain`-sized
 * units.  Chunk boundaries never split a unit, so per-unit work is unchanged. */
static void np_parallel_for(int64_t n, int64_t grain, int nthreads,
                            np_range_fn fn, void* ctx) {
  if (nthreads < 1) nthreads = 1;
  int64_t units = (n + grain - 1) / grain;
  if (nthreads > units) nthreads = (int)(units > 0 ? units : 1);
  if (nthreads == 1) {
    fn(ctx, 0, n);
    return;
  }
  pthread_t th[256];
  np_job jobs[256];
  if (nthreads > 256) nthreads = 256;
  int64_t per = (units + nthreads - 1) / nthreads;
  int started = 0;
  for (int t = 0; t < nthreads; ++t) {
    int64_t b = (int64_t)t * per * grain;
    int64_t e = (int64_t)(t + 1) * per * grain;
    if (b >= n) break;
    if (e > n) e = n;
    jobs[t].fn = fn;
    jobs[t].ctx = ctx;
    jobs[t].begin = b;
    jobs[t].end = e;
    if (pthread_create(&th[t], NULL, np_job_run, &jobs[t]) != 0) {
      fn(ctx, b, e); /* run inline if a thread cannot be started */
      jobs[t].fn = NULL;
    }
    started = t + 1;
  }
  for (int t = 0; t < started; ++t)
    if (jobs[t].fn) pthread_join(th[t], NULL);
}

/* ------------------------------------------------------------------------ */
/* fused_linear_relu / fused_linear  (nparray/fused_ops.mbt:12-52, 54-78)    */
/*   x [n, m], w [p, m] (out x in), bias [p]:                                */
/*   sum = bias[j]; for k in 0..m: sum = sum + x[i*m+k] * w[j*m+k]  (fp32)   */
/*   pre[i*p+j] = sum; out[i*p+j] = relu ? max(sum, 0) : sum                 */
/*   Rows are independent, so they may run on several threads.              */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float* x;
  const float* w;
  const float* bias;
  float* out;
  float* pre;
  int m, p, relu;
} np_fl_ctx;

static void np_fl_rows(void* vctx, int64_t row_begin, int64_t row_end) {
  np_fl_ctx* c = (np_fl_ctx*)vctx;
  for (int64_t i = row_begin; i < row_end; ++i) {
    const float* xrow = c->x + i * (int64_t)c->m;
    for (int64_t j = 0; j < c->p; ++j) {
      const float* wrow = c->w + j * (int64_t)c->m;
      float sum = c->bias[j];
      for (int64_t k = 0; k < c->m; ++k) {
        float prod = xrow[k] * wrow[k];
        sum = sum + prod;
      }
      if (c->pre) c->pre[i * (int64_t)c->p + j] = sum;
      c->out[i * (int64_t)c->p + j] = (c->relu && !(sum > 0.0f)) ? 0.0f : sum;
    }
  }
}

NP_EXPORT void np_fused_linear(const float* x, const float* w, const float* bias, float* out,
                               float* pre, int n, int m, int p, int relu, int nthreads) {
  np_fl_ctx ctx = {x, w, bias, out, pre, m, p, relu};
  np_parallel_for(n, 1, nthreads, np_fl_rows, &ctx);
}

/* ------------------------------------------------------------------------ */
/* NpArray::transpose  (nparray/trait_impl.mbt:252-261)                      */
/*   x [n, m] -> out [m, n], out[i*n + j] = x[j*m + i]                       */
/* ------------------------------------------------------------------------ */
NP_EXPORT void np_transpose(const float* x, float* out, int n, int m) {
  for (int64_t idx = 0; idx < (int64_t)n * m; ++idx) {
    int64_t i = idx / n, j = idx % n;
    out[idx] = x[j * (int64_t)m + i];
  }
}

/* ------------------------------------------------------------------------ */
/* NpArray::matmul  (nparray/trait_impl.mbt:205-249)                         */
/*   a [n, m] . b [m, p] -> c [n, p]                                         */
/*   1. bt = transpose(b) (bt[j*m + k] = b[k*p + j])                         */
/*   2. 32x32 output tiles; each element: sum = 0; for k in 0..m:           */
/*      sum = sum + a[i*m+k] * bt[j*m+k]   (fp32, sequential k)              */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float* a;
  const float* bt;
  float* c;
  int n, m, p;
} np_mm_ctx;

static void np_mm_rows(void* vctx, int64_t row_begin, int64_t row_end) {
  np_mm_ctx* x = (np_mm_ctx*)vctx;
  const int tile = 32;
  const int m = x->m, p = x->p;
  for (int64_t ii = row_begin; ii < row_end; ii += tile) {
    int64_t ii_end = ii + tile < row_end ? ii + tile : row_end;
    for (int64_t jj = 0; jj < p; jj += tile) {
      int64_t jj_end = jj + tile < p ? jj + tile : p;
      for (int64_t i = ii; i < ii_end; ++i) {
        const float* arow = x->a + i * (int64_t)m;
        float* crow = x->c + i * (int64_t)p;
        for (int64_t j = jj; j < jj_end; ++j) {
          const float* btrow = x->bt + j * (int64_t)m;
          float sum = 0.0f;
          for (int64_t k = 0; k < m; ++k) {
            float prod = arow[k] * btrow[k];
            sum = sum + prod;
          }
          crow[j] = sum;
        }
      }
    }
  }
}

NP_EXPORT void np_matmul(const float* a, const float* b, float* c, int n,
                         int m, int p, int nthreads) {
  float* bt = (float*)malloc(sizeof(float) * (size_t)m * (size_t)p + 4);
  for (int64_t k = 0; k < m; ++k)
    for (int64_t j = 0; j < p; ++j) bt[j * (int64_t)m + k] = b[k * (int64_t)p + j];
  np_mm_ctx ctx = {a, bt, c, n, m, p};
  np_parallel_for(n, 32, nthreads, np_mm_rows, &ctx);
  free(bt);
}

/* ------------------------------------------------------------------------ */
/* cuda_matmul semantics (moonxi-net-gpu/cuda/cuda_kernels.cu:1444-1499)     */
/* evaluated with NpArray arithmetic:                                        */
/*   op(A) = ta ? transpose(a stored [K,M]) : a stored [M,K]                 */
/*   op(B) = tb ? transpose(b stored [N,K]) : b stored [K,N]                 */
/*   c[M,N] = alpha * (op(A) . op(B)) + beta * c                             */
/* beta == 0 never reads c (BLAS convention, the reference's callers pass an */
/* uninitialised c with beta 0: tensor/trait_impl.mbt:233-248).              */
/* ------------------------------------------------------------------------ */
NP_EXPORT void np_gemm(const float* a, const float* b, float* c, int M, int K,
                       int N, int ta, int tb, float alpha, float beta,
                       int nthreads) {
  const float* A = a;
  const float* B = b;
  float* at = NULL;
  float* btt = NULL;
  if (ta) {
    at = (float*)malloc(sizeof(float) * (size_t)M * (size_t)K + 4);
    np_transpose(a, at, K, M); /* a is [K, M] -> at is [M, K] */
    A = at;
  }
  if (tb) {
    btt = (float*)malloc(sizeof(float) * (size_t)K * (size_t)N + 4);
    np_transpose(b, btt, N, K); /* b is [N, K] -> btt is [K, N] */
    B = btt;
  }
  float* prod = (float*)malloc(sizeof(float) * (size_t)M * (size_t)N + 4);
  np_matmul(A, B, prod, M, K, N, nthreads);
  int64_t total = (int64_t)M * N;
  if (alpha == 1.0f && beta == 0.0f) {
    memcpy(c, prod, sizeof(float) * (size_t)total);
  } else {
    for (int64_t i = 0; i < total; ++i) {
      float v = alpha * prod[i];
      if (beta != 0.0f) v = v + beta * c[i];
      c[i] = v;
    }
  }
  free(prod);
  free(at);
  free(btt);
}

/* ------------------------------------------------------------------------ */
/* NpArray::add with a row-broadcast bias (nparray/nparray.mbt:32-98)        */
/*   x [rows, cols] + b [cols] -> out; out[i,j] = x[i,j] + b[j] (fp32)       */
/* ------------------------------------------------------------------------ */
NP_EXPORT void np_add_row_bias(const float* x, const float* b, float* out,
                               int rows, int cols) {
  for (int64_t i = 0; i < rows; ++i)
    for (int64_t j = 0; j < cols; ++j)
      out[i * cols + j] = x[i * cols + j] + b[j];
}

/* NpArray::relu (nparray/image_impl.mbt:16-28): x > 0 ? x : 0 */
NP_EXPORT void np_relu(const float* x, float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] > 0.0f ? x[i] : 0.0f;
}

/* NpArray::relu_backward (nparray/image_impl.mbt:146-159):
 * out = input > 0 ? grad_output : 0 */
NP_EXPORT void np_relu_backward(const float* grad_output, const float* input,
                                float* out, int64_t n) {
  for (int64_t i = 0; i < n; ++i) out[i] = input[i] > 0.0f ? grad_output[i] : 0.0f;
}

/* ------------------------------------------------------------------------ */
/* NpArray::reduce_sum_to [rows, cols] -> [cols]                             */
/* (nparray/trait_impl.mbt:118-140, the leading-dimension branch):           */
/*   out[o] = sum over k of x[k*cols + o], fp32, k in increasing order       */
/* ------------------------------------------------------------------------ */
typedef struct {
  const float* x;
  float* out;
  int rows, cols;
} np_rs_ctx;

static void np_rs_cols(void* vctx, int64_t b, int64_t e) {
  np_rs_ctx* c = (np_rs_ctx*)vctx;
  for (int64_t o = b; o < e; ++o) {
    float sum = 0.0f;
    for (int64_t k = 0; k < c->rows; ++k) sum = sum + c->x[k * c->cols + o];
    c->out[o] = sum;
  }
}

NP_EXPORT void np_reduce_sum_leading(const float* x, float* out, int rows,
                                     int cols, int nthreads) {
  np_rs_ctx ctx = {x, out, rows, cols};
  np_parallel_for(cols, 64, nthreads, np_rs_cols, &ctx);
}

/* NpArray::add_into (nparray/trait_impl.mbt:192-197): x[i] = x[i] + y[i] */
NP_EXPORT void np_add_into(float* x, const float* y, int64_t n) {
  for (int64_t i = 0; i < n; ++i) x[i] = x[i] + y[i];
}

/* NpArray::scale (nparray/trait_impl.mbt:89-95): out[i] = x[i] * s */
NP_EXPORT void np_scale(const float* x, float* out, int64_t n, float s) {
  for (int64_t i = 0; i < n; ++i) out[i] = x[i] * s;
}

/* ------------------------------------------------------------------------ */
/* NpArray::cross_entropy_with_labels (nparray/image_impl.mbt:83-114)        */
/*   per row: max; sum_exp += (float)exp((double)(l - max)) in fp32;         */
/*   lse = (float)ln((double)sum_exp); log_prob = l[label] - max - lse;      */
/*   total = total - log_prob (fp32, row order); loss = total / batch        */
/* labels hold class indices as floats (the reference's label tensors).      */
/* `denom` is the divisor (the local batch on one device; callers that shard */
/* a global batch pass the global batch).                                    */
/* ------------------------------------------------------------------------ */
NP_EXPORT float np_ce_labels_forward(const float* logits, const float* labels,
                                     int batch, int num_classes, int denom) {
  float total = 0.0f;
  for (int64_t i = 0; i < batch; ++i) {
    const float* row = logits + i * num_classes;
    int label = (int)labels[i];
    float max_val = row[0];
    for (int j = 1; j < num_classes; ++j)
      if (row[j] > max_val) max_val = row[j];
    float sum_exp = 0.0f;
    for (int j = 0; j < num_classes; ++j)
      sum_exp = sum_exp + (float)exp((double)(row[j] - max_val));
    float lse = (float)log((double)sum_exp);
    float log_prob = row[label] - max_val - lse;
    total = total - log_prob;
  }
  return total / (float)denom;
}

/* NpArray::softmax_ce_backward_labels (nparray/image_impl.mbt:202-238):
 *   out[i,j] = ((float)exp((double)(l - max)) / sum_exp - onehot) / batch   */
NP_EXPORT void np_ce_labels_backward(const float* logits, const float* labels,
                                     float* out, int batch, int num_classes,
                                     int denom) {
  for (int64_t i = 0; i < batch; ++i) {
    const float* row = logits + i * num_classes;
    float* orow = out + i * num_classes;
    int label = (int)labels[i];
    float max_val = row[0];
    for (int j = 1; j < num_classes; ++j)
      if (row[j] > max_val) max_val = row[j];
    float sum_exp = 0.0f;
    for (int j = 0; j < num_classes; ++j)
      sum_exp = sum_exp + (float)exp((double)(row[j] - max_val));
    for (int j = 0; j < num_classes; ++j) {
      float sm = (float)exp((double)(row[j] - max_val)) / sum_exp;
      float target = (j == label) ? 1.0f : 0.0f;
      orow[j] = (sm - target) / (float)denom;
    }
  }
}

/* ------------------------------------------------------------------------ */
/* NpArray::batch_sgd_momentum_autoclip (nparray/trait_impl.mbt:280-311)     */
/*   norm_sq = sum over params (in order) of g*g, fp32 sequential            */
/*   clip = norm > max_norm ? max_norm / norm : 1                            */
/*   v = momentum*v + g*clip + wd*p ; p = p - lr*v                           */
/* Parameters are given as arrays of pointers and element counts.            */
/* Returns the gradient norm.                                                */
/* ------------------------------------------------------------------------ */
NP_EXPORT float np_sgd_momentum_autoclip(float** params, float** grads,
                                         float** vels, const int64_t* sizes,
                                         int count, float lr, float momentum,
                                         float weight_decay,
                                         float max_grad_norm) {
  float norm_sq = 0.0f;
  for (int i = 0; i < count; ++i) {
    const float* g = grads[i];
    for (int64_t j = 0; j < sizes[i]; ++j) norm_sq = norm_sq + g[j] * g[j];
  }
  float norm = sqrtf(norm_sq);
  float clip = norm > max_grad_norm ? max_grad_norm / norm : 1.0f;
  for (int i = 0; i < count; ++i) {
    float* p = params[i];
    const float* g = grads[i];
    float* v = vels[i];
    for (int64_t j = 0; j < sizes[i]; ++j) {
      float clipped = g[j] * clip;
      v[j] = momentum * v[j] + clipped + weight_decay * p[j];
      p[j] = p[j] - lr * v[j];
    }
  }
  return norm;
}
