/*
 * oracle.c — CPU restatement of the Remora reference's CPU path for the
 * data-parallel hot path.  TEST INFRASTRUCTURE ONLY (checker and timed CPU
 * baseline); the product never links it.  See oracle.h for the reference
 * files each function follows.  Compiled with -O2 -fno-fast-math
 * -ffp-contract=off so every f32 multiply and add rounds separately, as the
 * reference's arith.mulf / arith.addf do after convert-linalg-to-loops.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

/* ---------------------------------------------------------------- maps -- */

static float load_as_f32(const void *base, int dtype, int64_t i) {
  switch (dtype) {
  case REMORA_I32: return (float)((const int32_t *)base)[i];
  case REMORA_BOOL: return ((const uint8_t *)base)[i] ? 1.0f : 0.0f;
  default: return ((const float *)base)[i];
  }
}

static int32_t load_as_i32(const void *base, int dtype, int64_t i) {
  switch (dtype) {
  case REMORA_F32: return (int32_t)((const float *)base)[i];
  case REMORA_BOOL: return ((const uint8_t *)base)[i] ? 1 : 0;
  default: return ((const int32_t *)base)[i];
  }
}

/* f32 program, remora/_gpu_map_support.py F32Expr semantics with a true
   select; comparisons give 1.0f / 0.0f. */
static float eval_f32(const RemoraMapProgram *p, const float *inputs) {
  float r[REMORA_MAP_MAX_REGS];
  for (int k = 0; k < p->n_instr; ++k) {
    const RemoraMapInstr *in = &p->code[k];
    float a = r[in->a], b = r[in->b];
    float v = 0.0f;
    switch (in->op) {
    case REMORA_OP_INPUT: v = inputs[in->imm_i]; break;
    case REMORA_OP_CONST: v = in->imm_f; break;
    case REMORA_OP_ADD: v = a + b; break;
    case REMORA_OP_SUB: v = a - b; break;
    case REMORA_OP_MUL: v = a * b; break;
    case REMORA_OP_DIV: v = a / b; break;
    case REMORA_OP_LT: v = a < b ? 1.0f : 0.0f; break;
    case REMORA_OP_LE: v = a <= b ? 1.0f : 0.0f; break;
    case REMORA_OP_GT: v = a > b ? 1.0f : 0.0f; break;
    case REMORA_OP_GE: v = a >= b ? 1.0f : 0.0f; break;
    case REMORA_OP_EQ: v = a == b ? 1.0f : 0.0f; break;
    case REMORA_OP_NE: v = a != b ? 1.0f : 0.0f; break;
    case REMORA_OP_SELECT: v = a != 0.0f ? b : r[in->c]; break;
    case REMORA_OP_AND: v = (a != 0.0f && b != 0.0f) ? 1.0f : 0.0f; break;
    case REMORA_OP_OR: v = (a != 0.0f || b != 0.0f) ? 1.0f : 0.0f; break;
    case REMORA_OP_NEG: v = -a; break;
    case REMORA_OP_EXP: v = expf(a); break;
    case REMORA_OP_LOG: v = logf(a); break;
    case REMORA_OP_SQRT: v = sqrtf(a); break;
    default: v = 0.0f; break;
    }
    r[in->dst] = v;
  }
  return r[p->result];
}

/* i32 / bool programs: two's-complement wrapping arithmetic (llvm add/sub/mul
   on i32), truncating division (llvm.sdiv, remora/operators.py:109).  A zero
   divisor yields 0 and INT_MIN / -1 wraps, here and on the device. */
static int32_t eval_i32(const RemoraMapProgram *p, const int32_t *inputs) {
  int32_t r[REMORA_MAP_MAX_REGS];
  for (int k = 0; k < p->n_instr; ++k) {
    const RemoraMapInstr *in = &p->code[k];
    int32_t a = r[in->a], b = r[in->b];
    int32_t v = 0;
    switch (in->op) {
    case REMORA_OP_INPUT: v = inputs[in->imm_i]; break;
    case REMORA_OP_CONST: v = in->imm_i; break;
    case REMORA_OP_ADD: v = (int32_t)((uint32_t)a + (uint32_t)b); break;
    case REMORA_OP_SUB: v = (int32_t)((uint32_t)a - (uint32_t)b); break;
    case REMORA_OP_MUL: v = (int32_t)((uint32_t)a * (uint32_t)b); break;
    case REMORA_OP_DIV:
      if (b == 0) v = 0;
      else if (b == -1) v = (int32_t)(0u - (uint32_t)a);
      else v = a / b;
      break;
    case REMORA_OP_LT: v = a < b; break;
    case REMORA_OP_LE: v = a <= b; break;
    case REMORA_OP_GT: v = a > b; break;
    case REMORA_OP_GE: v = a >= b; break;
    case REMORA_OP_EQ: v = a == b; break;
    case REMORA_OP_NE: v = a != b; break;
    case REMORA_OP_SELECT: v = a != 0 ? b : r[in->c]; break;
    case REMORA_OP_AND: v = (a != 0 && b != 0); break;
    case REMORA_OP_OR: v = (a != 0 || b != 0); break;
    case REMORA_OP_NEG: v = (int32_t)(0u - (uint32_t)a); break;
    default: v = 0; break;
    }
    r[in->dst] = v;
  }
  return r[p->result];
}

static void store_out(void *out, int dtype, int64_t i, float fv, int32_t iv,
                      int is_float) {
  switch (dtype) {
  case REMORA_F32: ((float *)out)[i] = is_float ? fv : (float)iv; break;
  case REMORA_I32: ((int32_t *)out)[i] = is_float ? (int32_t)fv : iv; break;
  default: ((uint8_t *)out)[i] = is_float ? (fv != 0.0f) : (iv != 0); break;
  }
}

void oracle_map(const RemoraMapProgram *p, int n_in, const void *const *ins,
                const int64_t *in_strides, const int64_t *shape, int rank,
                void *out, int nthreads) {
  int64_t numel = 1;
  for (int d = 0; d < rank; ++d) numel *= shape[d];
  const int is_float = p->compute_dtype == REMORA_F32;
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t i = 0; i < numel; ++i) {
    int64_t idx[REMORA_MAX_RANK];
    int64_t rem = i;
    for (int d = rank - 1; d >= 0; --d) {
      idx[d] = rem % shape[d];
      rem /= shape[d];
    }
    float fin[REMORA_MAP_MAX_INPUTS];
    int32_t iin[REMORA_MAP_MAX_INPUTS];
    for (int k = 0; k < n_in; ++k) {
      int64_t lin = 0;
      for (int d = 0; d < rank; ++d) lin += idx[d] * in_strides[k * rank + d];
      if (is_float) fin[k] = load_as_f32(ins[k], p->in_dtype[k], lin);
      else iin[k] = load_as_i32(ins[k], p->in_dtype[k], lin);
    }
    if (is_float) store_out(out, p->out_dtype, i, eval_f32(p, fin), 0, 1);
    else store_out(out, p->out_dtype, i, 0.0f, eval_i32(p, iin), 0);
  }
}

/* --------------------------------------------------------------- folds -- */

static float fold_elem_f32(const RemoraFoldSpec *s, int n_in,
                           const void *const *ins, int64_t i) {
  if (!s->has_premap) return ((const float *)ins[0])[i];
  float v[REMORA_MAP_MAX_INPUTS];
  for (int k = 0; k < n_in; ++k) v[k] = load_as_f32(ins[k], s->premap.in_dtype[k], i);
  return eval_f32(&s->premap, v);
}

static int32_t fold_elem_i32(const RemoraFoldSpec *s, int n_in,
                             const void *const *ins, int64_t i) {
  if (!s->has_premap) return ((const int32_t *)ins[0])[i];
  int32_t v[REMORA_MAP_MAX_INPUTS];
  for (int k = 0; k < n_in; ++k) v[k] = load_as_i32(ins[k], s->premap.in_dtype[k], i);
  return eval_i32(&s->premap, v);
}

static float epi_f32(const RemoraFoldSpec *s, float acc) {
  return s->epilogue == REMORA_EPI_SQRT ? sqrtf(acc) : acc;
}

void oracle_cell_fold(const RemoraFoldSpec *s, int n_in, const void *const *ins,
                      int64_t rows, int64_t L, void *out, int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    if (s->dtype == REMORA_F32) {
      float acc = s->init_f;
      for (int64_t j = 0; j < L; ++j) {
        float v = fold_elem_f32(s, n_in, ins, r * L + j);
        acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
      }
      ((float *)out)[r] = epi_f32(s, acc);
    } else {
      int64_t acc = s->init_i;
      for (int64_t j = 0; j < L; ++j) {
        int64_t v = fold_elem_i32(s, n_in, ins, r * L + j);
        acc = s->op == REMORA_FOLD_MUL ? (int64_t)((uint64_t)acc * (uint64_t)v)
                                       : (int64_t)((uint64_t)acc + (uint64_t)v);
      }
      ((int32_t *)out)[r] = (int32_t)acc;
    }
  }
}

void oracle_fold_all(const RemoraFoldSpec *s, int n_in, const void *const *ins,
                     int64_t n, void *out) {
  oracle_cell_fold(s, n_in, ins, 1, n, out, 1);
}

void oracle_array_fold(const RemoraFoldSpec *s, const void *in, const void *init,
                       int64_t B, int64_t T, void *out) {
  for (int64_t t = 0; t < T; ++t) {
    if (s->dtype == REMORA_F32) {
      float acc = ((const float *)init)[t];
      for (int64_t b = 0; b < B; ++b) {
        float v = ((const float *)in)[b * T + t];
        acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
      }
      ((float *)out)[t] = acc;
    } else {
      uint32_t acc = (uint32_t)((const int32_t *)init)[t];
      for (int64_t b = 0; b < B; ++b) {
        uint32_t v = (uint32_t)((const int32_t *)in)[b * T + t];
        acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
      }
      ((int32_t *)out)[t] = (int32_t)acc;
    }
  }
}

/* --------------------------------------------------------------- scans -- */

void oracle_scan(const RemoraScanSpec *s, const void *in, int64_t N, int64_t T,
                 void *out) {
  for (int64_t t = 0; t < T; ++t) {
    if (s->dtype == REMORA_F32) {
      const float *x = (const float *)in;
      float *y = (float *)out;
      float acc = s->init_f;
      for (int64_t q = 0; q < N; ++q) {
        int64_t i = s->right ? N - 1 - q : q;
        float v = x[i * T + t];
        if (s->exclusive) {
          y[i * T + t] = acc;
          acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
        } else {
          acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
          y[i * T + t] = acc;
        }
      }
    } else {
      const int32_t *x = (const int32_t *)in;
      int32_t *y = (int32_t *)out;
      uint32_t acc = (uint32_t)s->init_i;
      for (int64_t q = 0; q < N; ++q) {
        int64_t i = s->right ? N - 1 - q : q;
        uint32_t v = (uint32_t)x[i * T + t];
        if (s->exclusive) {
          y[i * T + t] = (int32_t)acc;
          acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
        } else {
          acc = s->op == REMORA_FOLD_MUL ? acc * v : acc + v;
          y[i * T + t] = (int32_t)acc;
        }
      }
    }
  }
}

/* ------------------------------------------------------------- matmul -- */

/* i-k-j order: every C element still receives its products in increasing k,
   each product rounded, then added to the running f32 sum — the same
   rounding sequence as the per-element sequential fold. */
void oracle_matmul(const float *A, const float *B, float *C, int64_t batch,
                   int64_t M, int64_t N, int64_t K, int64_t row0, int64_t row1,
                   int nthreads) {
  for (int64_t b = 0; b < batch; ++b) {
    const float *Ab = A + b * M * K;
    const float *Bb = B + b * K * N;
    float *Cb = C + b * M * N;
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t i = row0; i < row1; ++i) {
      float *c = Cb + i * N;
      for (int64_t j = 0; j < N; ++j) c[j] = 0.0f;
      for (int64_t k = 0; k < K; ++k) {
        const float a = Ab[i * K + k];
        const float *brow = Bb + k * N;
        for (int64_t j = 0; j < N; ++j) {
          float prod = a * brow[j];
          c[j] = c[j] + prod;
        }
      }
    }
  }
}

/* ------------------------------------------------------ im2col / col2im -- */

void oracle_im2col(const float *img, int64_t H, int64_t W, int kh, int kw,
                   int stride, float *cols) {
  int64_t oh = (H - kh) / stride + 1, ow = (W - kw) / stride + 1;
  for (int64_t i = 0; i < oh; ++i)
    for (int64_t j = 0; j < ow; ++j)
      for (int a = 0; a < kh; ++a)
        for (int b = 0; b < kw; ++b)
          cols[(i * ow + j) * (kh * kw) + a * kw + b] =
              img[(i * stride + a) * W + (j * stride + b)];
}

/* The reference overlap-adds into a float64 image (np.zeros default dtype)
   and coerces to f32 once at the end (remora/runtime.py:1290-1305). */
void oracle_col2im(const float *cols, int64_t H, int64_t W, int kh, int kw,
                   int stride, float *img) {
  int64_t oh = (H - kh) / stride + 1, ow = (W - kw) / stride + 1;
  double *acc = (double *)calloc((size_t)(H * W), sizeof(double));
  for (int64_t i = 0; i < oh; ++i)
    for (int64_t j = 0; j < ow; ++j)
      for (int a = 0; a < kh; ++a)
        for (int b = 0; b < kw; ++b)
          acc[(i * stride + a) * W + (j * stride + b)] +=
              (double)cols[(i * ow + j) * (kh * kw) + a * kw + b];
  for (int64_t p = 0; p < H * W; ++p) img[p] = (float)acc[p];
  free(acc);
}

/* ---------------------------------------------------------------- conv -- */

static inline int64_t conv_out(int64_t H, int R, int stride, int pad) {
  return (H + 2 * pad - R) / stride + 1;
}

/* y[n,k,i,j] = (sum_c dot_c) + bias[k], dot_c = fold(+, 0, map(*, patch,
   ravel w[k,c])) in tap order a*S+b: the reference's single-channel conv2d
   (examples/crater_train.py:30-36) summed over input channels in order. */
void oracle_conv2d_fwd(const float *x, const float *w, const float *bias,
                       float *y, int64_t N, int64_t C, int64_t H, int64_t W,
                       int64_t K, int R, int S, int stride, int pad, int64_t n0,
                       int64_t n1, int nthreads) {
  const int64_t OH = conv_out(H, R, stride, pad), OW = conv_out(W, S, stride, pad);
  (void)N;
#pragma omp parallel for collapse(2) num_threads(nthreads) schedule(static)
  for (int64_t n = n0; n < n1; ++n)
    for (int64_t k = 0; k < K; ++k)
      for (int64_t i = 0; i < OH; ++i)
        for (int64_t j = 0; j < OW; ++j) {
          float total = 0.0f;
          for (int64_t c = 0; c < C; ++c) {
            float dot = 0.0f;
            for (int a = 0; a < R; ++a)
              for (int b = 0; b < S; ++b) {
                int64_t h = i * stride + a - pad, q = j * stride + b - pad;
                float xv = (h >= 0 && h < H && q >= 0 && q < W)
                               ? x[((n * C + c) * H + h) * W + q]
                               : 0.0f;
                float prod = xv * w[((k * C + c) * R + a) * S + b];
                dot = dot + prod;
              }
            total = total + dot;
          }
          if (bias) total = total + bias[k];
          y[((n * K + k) * OH + i) * OW + j] = total;
        }
}

/* dx = col2im of (w^T . dy): remora/ad.py:157-171 applied per channel pair,
   accumulated in f64 like the reference's tape. */
void oracle_conv2d_dgrad(const float *dy, const float *w, float *dx, int64_t N,
                         int64_t C, int64_t H, int64_t W, int64_t K, int R,
                         int S, int stride, int pad, int64_t n0, int64_t n1,
                         int nthreads) {
  const int64_t OH = conv_out(H, R, stride, pad), OW = conv_out(W, S, stride, pad);
  (void)N;
#pragma omp parallel for collapse(2) num_threads(nthreads) schedule(static)
  for (int64_t n = n0; n < n1; ++n)
    for (int64_t c = 0; c < C; ++c)
      for (int64_t h = 0; h < H; ++h)
        for (int64_t q = 0; q < W; ++q) {
          double acc = 0.0;
          for (int64_t k = 0; k < K; ++k)
            for (int a = 0; a < R; ++a) {
              int64_t ti = h + pad - a;
              if (ti < 0 || ti % stride) continue;
              int64_t i = ti / stride;
              if (i >= OH) continue;
              for (int b = 0; b < S; ++b) {
                int64_t tj = q + pad - b;
                if (tj < 0 || tj % stride) continue;
                int64_t j = tj / stride;
                if (j >= OW) continue;
                acc += (double)dy[((n * K + k) * OH + i) * OW + j] *
                       (double)w[((k * C + c) * R + a) * S + b];
              }
            }
          dx[((n * C + c) * H + h) * W + q] = (float)acc;
        }
}

void oracle_conv2d_wgrad(const float *x, const float *dy, float *dw, int64_t N,
                         int64_t C, int64_t H, int64_t W, int64_t K, int R,
                         int S, int stride, int pad, int64_t n0, int64_t n1,
                         int nthreads) {
  const int64_t OH = conv_out(H, R, stride, pad), OW = conv_out(W, S, stride, pad);
  (void)N;
#pragma omp parallel for collapse(2) num_threads(nthreads) schedule(static)
  for (int64_t k = 0; k < K; ++k)
    for (int64_t c = 0; c < C; ++c)
      for (int a = 0; a < R; ++a)
        for (int b = 0; b < S; ++b) {
          double acc = 0.0;
          for (int64_t n = n0; n < n1; ++n)
            for (int64_t i = 0; i < OH; ++i) {
              int64_t h = i * stride + a - pad;
              if (h < 0 || h >= H) continue;
              const float *dyr = dy + ((n * K + k) * OH + i) * OW;
              const float *xr = x + ((n * C + c) * H + h) * W;
              for (int64_t j = 0; j < OW; ++j) {
                int64_t q = j * stride + b - pad;
                if (q < 0 || q >= W) continue;
                acc += (double)dyr[j] * (double)xr[q];
              }
            }
          dw[((k * C + c) * R + a) * S + b] = (float)acc;
        }
}

/* ---------------------------------------------------------------- pool -- */

/* 2x2 / stride 2 max; ties keep the first element in window order
   (0,0),(0,1),(1,0),(1,1). */
void oracle_maxpool2x2_fwd(const float *x, float *y, int64_t NC, int64_t H,
                           int64_t W) {
  const int64_t OH = H / 2, OW = W / 2;
  for (int64_t p = 0; p < NC; ++p)
    for (int64_t i = 0; i < OH; ++i)
      for (int64_t j = 0; j < OW; ++j) {
        const float *b = x + (p * H + 2 * i) * W + 2 * j;
        float m = b[0];
        if (b[1] > m) m = b[1];
        if (b[W] > m) m = b[W];
        if (b[W + 1] > m) m = b[W + 1];
        y[(p * OH + i) * OW + j] = m;
      }
}

void oracle_maxpool2x2_bwd(const float *x, const float *dy, float *dx,
                           int64_t NC, int64_t H, int64_t W) {
  const int64_t OH = H / 2, OW = W / 2;
  for (int64_t p = 0; p < NC * H * W; ++p) dx[p] = 0.0f;
  for (int64_t p = 0; p < NC; ++p)
    for (int64_t i = 0; i < OH; ++i)
      for (int64_t j = 0; j < OW; ++j) {
        int64_t base = (p * H + 2 * i) * W + 2 * j;
        int64_t arg = base;
        float m = x[base];
        if (x[base + 1] > m) { m = x[base + 1]; arg = base + 1; }
        if (x[base + W] > m) { m = x[base + W]; arg = base + W; }
        if (x[base + W + 1] > m) { m = x[base + W + 1]; arg = base + W + 1; }
        dx[arg] = dy[(p * OH + i) * OW + j];
      }
}

/* ----------------------------------------------------------------- CNN -- */

enum {
  P_W1 = 0,
  P_B1 = P_W1 + 16 * 9,
  P_W2 = P_B1 + 16,
  P_B2 = P_W2 + 32 * 16 * 9,
  P_W3 = P_B2 + 32,
  P_B3 = P_W3 + 64 * 8192,
  P_W4 = P_B3 + 64,
  P_B4 = P_W4 + 64,
  P_END = P_B4 + 1
};

/* stable BCE of examples/crater_train.py:50-54 */
static float bce_logit(float z, float y) {
  float pos = z > 0.0f ? z : 0.0f;
  float absz = z > 0.0f ? z : 0.0f - z;
  return pos + (-1.0f * (z * y) + logf(1.0f + expf(0.0f - absz)));
}

/* d bce / dz = sigmoid(z) - y, evaluated in the overflow-free branch form */
static float bce_grad(float z, float y) {
  float s;
  if (z > 0.0f) s = 1.0f / (1.0f + expf(-z));
  else { float e = expf(z); s = e / (1.0f + e); }
  return s - y;
}

float oracle_cnn_step(float *params, float *grads, const float *images,
                      const float *labels, int64_t batch, int64_t batch_total,
                      float lr, int apply_sgd, int nthreads) {
  const int64_t B = batch;
  float *a1 = (float *)malloc(sizeof(float) * B * 16 * 64 * 64);
  float *p1 = (float *)malloc(sizeof(float) * B * 16 * 32 * 32);
  float *a2 = (float *)malloc(sizeof(float) * B * 32 * 32 * 32);
  float *p2 = (float *)malloc(sizeof(float) * B * 8192);
  float *h = (float *)malloc(sizeof(float) * B * 64);
  float *z = (float *)malloc(sizeof(float) * B);
  float *dz = (float *)malloc(sizeof(float) * B);
  float *dh = (float *)malloc(sizeof(float) * B * 64);
  float *dp2 = (float *)malloc(sizeof(float) * B * 8192);
  float *da2 = (float *)malloc(sizeof(float) * B * 32 * 32 * 32);
  float *dp1 = (float *)malloc(sizeof(float) * B * 16 * 32 * 32);
  float *da1 = (float *)malloc(sizeof(float) * B * 16 * 64 * 64);
  const float *w1 = params + P_W1, *b1 = params + P_B1;
  const float *w2 = params + P_W2, *b2 = params + P_B2;
  const float *w3 = params + P_W3, *b3 = params + P_B3;
  const float *w4 = params + P_W4, *b4 = params + P_B4;

  /* forward */
  oracle_conv2d_fwd(images, w1, b1, a1, B, 1, 64, 64, 16, 3, 3, 1, 1, 0, B, nthreads);
  for (int64_t i = 0; i < B * 16 * 64 * 64; ++i) a1[i] = a1[i] > 0.0f ? a1[i] : 0.0f;
  oracle_maxpool2x2_fwd(a1, p1, B * 16, 64, 64);
  oracle_conv2d_fwd(p1, w2, b2, a2, B, 16, 32, 32, 32, 3, 3, 1, 1, 0, B, nthreads);
  for (int64_t i = 0; i < B * 32 * 32 * 32; ++i) a2[i] = a2[i] > 0.0f ? a2[i] : 0.0f;
  oracle_maxpool2x2_fwd(a2, p2, B * 32, 32, 32);
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t n = 0; n < B; ++n) {
    for (int o = 0; o < 64; ++o) {
      float acc = 0.0f;
      for (int k = 0; k < 8192; ++k) {
        float prod = w3[(int64_t)o * 8192 + k] * p2[n * 8192 + k];
        acc = acc + prod;
      }
      acc = acc + b3[o];
      h[n * 64 + o] = acc > 0.0f ? acc : 0.0f;
    }
    float acc = 0.0f;
    for (int o = 0; o < 64; ++o) {
      float prod = w4[o] * h[n * 64 + o];
      acc = acc + prod;
    }
    z[n] = acc + b4[0];
  }
  double loss = 0.0;
  const float inv = 1.0f / (float)batch_total;
  for (int64_t n = 0; n < B; ++n) {
    loss += bce_logit(z[n], labels[n]);
    dz[n] = bce_grad(z[n], labels[n]) * inv;
  }

  /* backward */
  memset(grads, 0, sizeof(float) * P_END);
  {
    double gb4 = 0.0;
    for (int64_t n = 0; n < B; ++n) gb4 += dz[n];
    grads[P_B4] = (float)gb4;
    for (int o = 0; o < 64; ++o) {
      double g = 0.0;
      for (int64_t n = 0; n < B; ++n) g += (double)dz[n] * h[n * 64 + o];
      grads[P_W4 + o] = (float)g;
    }
    for (int64_t n = 0; n < B; ++n)
      for (int o = 0; o < 64; ++o)
        dh[n * 64 + o] = h[n * 64 + o] > 0.0f ? dz[n] * w4[o] : 0.0f;
    for (int o = 0; o < 64; ++o) {
      double g = 0.0;
      for (int64_t n = 0; n < B; ++n) g += dh[n * 64 + o];
      grads[P_B3 + o] = (float)g;
    }
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int o = 0; o < 64; ++o)
      for (int k = 0; k < 8192; ++k) {
        double g = 0.0;
        for (int64_t n = 0; n < B; ++n) g += (double)dh[n * 64 + o] * p2[n * 8192 + k];
        grads[P_W3 + (int64_t)o * 8192 + k] = (float)g;
      }
#pragma omp parallel for num_threads(nthreads) schedule(static)
    for (int64_t n = 0; n < B; ++n)
      for (int k = 0; k < 8192; ++k) {
        double g = 0.0;
        for (int o = 0; o < 64; ++o) g += (double)dh[n * 64 + o] * w3[(int64_t)o * 8192 + k];
        dp2[n * 8192 + k] = (float)g;
      }
  }
  oracle_maxpool2x2_bwd(a2, dp2, da2, B * 32, 32, 32);
  for (int64_t i = 0; i < B * 32 * 32 * 32; ++i)
    if (!(a2[i] > 0.0f)) da2[i] = 0.0f;
  for (int k = 0; k < 32; ++k) {
    double g = 0.0;
    for (int64_t n = 0; n < B; ++n)
      for (int p = 0; p < 32 * 32; ++p) g += da2[(n * 32 + k) * 1024 + p];
    grads[P_B2 + k] = (float)g;
  }
  oracle_conv2d_wgrad(p1, da2, grads + P_W2, B, 16, 32, 32, 32, 3, 3, 1, 1, 0, B, nthreads);
  oracle_conv2d_dgrad(da2, w2, dp1, B, 16, 32, 32, 32, 3, 3, 1, 1, 0, B, nthreads);
  oracle_maxpool2x2_bwd(a1, dp1, da1, B * 16, 64, 64);
  for (int64_t i = 0; i < B * 16 * 64 * 64; ++i)
    if (!(a1[i] > 0.0f)) da1[i] = 0.0f;
  for (int k = 0; k < 16; ++k) {
    double g = 0.0;
    for (int64_t n = 0; n < B; ++n)
      for (int p = 0; p < 64 * 64; ++p) g += da1[(n * 16 + k) * 4096 + p];
    grads[P_B1 + k] = (float)g;
  }
  oracle_conv2d_wgrad(images, da1, grads + P_W1, B, 1, 64, 64, 16, 3, 3, 1, 1, 0, B, nthreads);

  if (apply_sgd)
    for (int64_t i = 0; i < P_END; ++i) params[i] = params[i] - lr * grads[i];

  free(a1); free(p1); free(a2); free(p2); free(h); free(z); free(dz);
  free(dh); free(dp2); free(da2); free(dp1); free(da1);
  return (float)(loss / (double)batch_total);
}

/* ------------------------------------------- compiled benchmark loops -- */
/* The two benchmark programs as straight C loops, the form the reference's
   MLIR CPU path compiles them to (one linalg.generic with a sequential f32
   reduction per frame cell, remora/lowering/tensor_ops.py:802-874): used as
   the timed CPU baseline; the generic interpreter above stays the checker. */

void oracle_chained_fold_f32(const float *x, int64_t rows, int64_t L, float *out,
                             int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float *row = x + r * L;
    float acc = 0.0f;
    for (int64_t j = 0; j < L; ++j) {
      float y = row[j] * 2.5f;
      y = y + 1.0f;
      /* select(y > 0.5, y, 0.0) as LLVM lowers arith.select: no branch.
         A 50/50 mask would mispredict half the time; the masked bits give
         y or +0.0 exactly. */
      uint32_t bits;
      memcpy(&bits, &y, sizeof bits);
      bits &= (uint32_t)0 - (uint32_t)(y > 0.5f);
      float v;
      memcpy(&v, &bits, sizeof v);
      acc = acc + v;
    }
    out[r] = acc;
  }
}

void oracle_row_norms_f32(const float *x, int64_t rows, int64_t L, float *out,
                          int nthreads) {
#pragma omp parallel for num_threads(nthreads) schedule(static)
  for (int64_t r = 0; r < rows; ++r) {
    const float *row = x + r * L;
    float acc = 0.0f;
    for (int64_t j = 0; j < L; ++j) {
      float sq = row[j] * row[j];
      acc = acc + sq;
    }
    out[r] = sqrtf(acc);
  }
}

/* ---- sort / grade / filter / replicate (remora/remora_rt.c) ---- */

/* Value order of element i of a row: f32 compares as floats (so -0.0 and
   +0.0 are equal), i32 as signed integers. */
static int rt_less(int dtype, const void *base, int64_t a, int64_t b) {
  if (dtype == REMORA_F32) return ((const float *)base)[a] < ((const float *)base)[b];
  return ((const int32_t *)base)[a] < ((const int32_t *)base)[b];
}

/* Stable bottom-up merge sort of the index array idx[0..n) by the values
   they point at. */
static void rt_stable_order(int dtype, const void *vals, int64_t *idx, int64_t *tmp, int64_t n) {
  for (int64_t w = 1; w < n; w *= 2) {
    for (int64_t lo = 0; lo < n; lo += 2 * w) {
      int64_t mid = lo + w < n ? lo + w : n, hi = lo + 2 * w < n ? lo + 2 * w : n;
      int64_t i = lo, j = mid, k = lo;
      while (i < mid && j < hi) tmp[k++] = rt_less(dtype, vals, idx[j], idx[i]) ? idx[j++] : idx[i++];
      while (i < mid) tmp[k++] = idx[i++];
      while (j < hi) tmp[k++] = idx[j++];
    }
    memcpy(idx, tmp, (size_t)n * sizeof(int64_t));
  }
}

static void rt_sort_or_grade(int dtype, const void *in, void *out, int grade, int64_t rows, int64_t len,
                             int nthreads) {
#pragma omp parallel num_threads(nthreads)
  {
    int64_t *idx = (int64_t *)malloc((size_t)(len > 0 ? len : 1) * sizeof(int64_t));
    int64_t *tmp = (int64_t *)malloc((size_t)(len > 0 ? len : 1) * sizeof(int64_t));
#pragma omp for schedule(dynamic)
    for (int64_t r = 0; r < rows; ++r) {
      const char *row = (const char *)in + r * len * 4;
      for (int64_t i = 0; i < len; ++i) idx[i] = i;
      rt_stable_order(dtype, row, idx, tmp, len);
      for (int64_t i = 0; i < len; ++i) {
        if (grade) ((int32_t *)out)[r * len + i] = (int32_t)idx[i];
        else memcpy((char *)out + (r * len + i) * 4, row + idx[i] * 4, 4);
      }
    }
    free(idx);
    free(tmp);
  }
}

void oracle_sort(int dtype, const void *in, void *out, int64_t rows, int64_t len, int nthreads) {
  rt_sort_or_grade(dtype, in, out, 0, rows, len, nthreads);
}

void oracle_grade(int dtype, const void *in, int32_t *out, int64_t rows, int64_t len, int nthreads) {
  rt_sort_or_grade(dtype, in, out, 1, rows, len, nthreads);
}

static int rt_compare(int op, double x, double lit) {
  switch (op) {
    case REMORA_OP_LT: return x < lit;
    case REMORA_OP_LE: return x <= lit;
    case REMORA_OP_GT: return x > lit;
    case REMORA_OP_GE: return x >= lit;
    case REMORA_OP_EQ: return x == lit;
    default: return x < lit || x > lit; /* ordered not-equal: false for NaN */
  }
}

int64_t oracle_filter(int dtype, const void *src, const void *mask, int mask_dtype,
                      const RemoraFilterPred *pred, int64_t n, void *dst, int64_t cap) {
  int64_t out_n = 0;
  for (int64_t i = 0; i < n; ++i) {
    int keep;
    if (pred) {
      if (dtype == REMORA_F32) keep = rt_compare(pred->op, ((const float *)src)[i], pred->lit_f);
      else keep = rt_compare(pred->op, ((const int32_t *)src)[i], pred->lit_i);
    } else if (mask_dtype == REMORA_BOOL) {
      keep = ((const uint8_t *)mask)[i] != 0;
    } else {
      keep = ((const int32_t *)mask)[i] != 0;
    }
    if (keep) {
      if (out_n < cap) memcpy((char *)dst + out_n * 4, (const char *)src + i * 4, 4);
      ++out_n;
    }
  }
  return out_n;
}

int64_t oracle_replicate(int dtype, const void *src, const int32_t *counts, int64_t n, void *dst, int64_t cap) {
  (void)dtype;
  int64_t out_n = 0;
  for (int64_t i = 0; i < n; ++i)
    for (int32_t r = 0; r < counts[i]; ++r) {
      if (out_n < cap) memcpy((char *)dst + out_n * 4, (const char *)src + i * 4, 4);
      ++out_n;
    }
  return out_n;
}
