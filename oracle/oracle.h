/*
 * oracle.h — CPU restatement of the Remora reference's CPU semantics for the
 * data-parallel hot path.  TEST INFRASTRUCTURE ONLY: the tests, the smoke
 * check and bench.py's cpu_baseline / reference arm call it as the checker
 * and as the timed CPU baseline.  The product (libremora_b200.so and the
 * remora_b200 package) never links, loads or calls it.
 *
 * Loop orders follow the reference's MLIR CPU lowering (linalg.generic with
 * sequential reduction iterators, convert-linalg-to-loops):
 *   maps             remora/lowering/tensor_ops.py:644-734 (+ frame.py:188-211)
 *   cell fold        remora/lowering/tensor_ops.py:802-874
 *   scalar fold      remora/lowering/tensor_ops.py:1135-1204 (i32 -> i64 acc)
 *   array fold       remora/lowering/tensor_ops.py:1223-1296
 *   scans            remora/lowering/tensor_ops.py:2301-2482
 *   im2col/col2im    remora/runtime.py:1274-1305
 *   VJPs             remora/ad.py:85-179
 *   CNN formulas     examples/crater_train.py:46-54,249-253
 *   sort / grade     remora/remora_rt.c:17-121 (interpreter: stable np.sort /
 *                    np.argsort, remora/runtime.py:1171-1177)
 *   filter           remora/remora_rt.c:125-163 (+ the comparison mask of
 *                    remora/lowering/tensor_ops.py:2657-2706)
 *   replicate        remora/remora_rt.c:167-285
 * f32 arithmetic is done as separate IEEE multiplies and adds (the file is
 * compiled with -ffp-contract=off), matching arith.mulf/arith.addf.
 */
#ifndef REMORA_ORACLE_H
#define REMORA_ORACLE_H

#include <stdint.h>
#include "../include/remora_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

int oracle_max_threads(void);

/* Lifted map.  Output is contiguous row-major over shape[0..rank).  Input k
   starts at ins[k] (offset already applied) and is read at
   sum_d idx[d] * in_strides[k*rank + d] (0 strides broadcast). */
void oracle_map(const RemoraMapProgram *p, int n_in, const void *const *ins,
                const int64_t *in_strides, const int64_t *shape, int rank,
                void *out, int nthreads);

/* Cell fold over contiguous rows of length L: out[r] = epi(init op f(x[r,0])
   op f(x[r,1]) ...), sequential. */
void oracle_cell_fold(const RemoraFoldSpec *s, int n_in, const void *const *ins,
                      int64_t rows, int64_t L, void *out, int nthreads);

/* Whole-array fold of n contiguous elements to one value (sequential; i32
   accumulates in i64 and truncates). */
void oracle_fold_all(const RemoraFoldSpec *s, int n_in, const void *const *ins,
                     int64_t n, void *out);

/* Leading-axis fold with array accumulator: out[t] = init[t] op x[0,t] op
   x[1,t] ... for x contiguous [B, T]. */
void oracle_array_fold(const RemoraFoldSpec *s, const void *in, const void *init,
                       int64_t B, int64_t T, void *out);

/* Scan along axis 0 of a contiguous [N, T] array (T = 1 for rank 1). */
void oracle_scan(const RemoraScanSpec *s, const void *in, int64_t N, int64_t T,
                 void *out);

/* C[b, i, j] = fold(+, 0, map(*, A[b, i, :], B[b, :, j])) for rows
   i in [row0, row1); A is [batch, M, K], B is [batch, K, N], all contiguous.
   Sequential in k per element. */
void oracle_matmul(const float *A, const float *B, float *C, int64_t batch,
                   int64_t M, int64_t N, int64_t K, int64_t row0, int64_t row1,
                   int nthreads);

void oracle_im2col(const float *img, int64_t H, int64_t W, int kh, int kw,
                   int stride, float *cols);
void oracle_col2im(const float *cols, int64_t H, int64_t W, int kh, int kw,
                   int stride, float *img);

/* NCHW cross-correlation with zero padding.  Images n in [n0, n1). */
void oracle_conv2d_fwd(const float *x, const float *w, const float *bias,
                       float *y, int64_t N, int64_t C, int64_t H, int64_t W,
                       int64_t K, int R, int S, int stride, int pad, int64_t n0,
                       int64_t n1, int nthreads);
void oracle_conv2d_dgrad(const float *dy, const float *w, float *dx, int64_t N,
                         int64_t C, int64_t H, int64_t W, int64_t K, int R,
                         int S, int stride, int pad, int64_t n0, int64_t n1,
                         int nthreads);
/* dw is summed over images [n0, n1) only. */
void oracle_conv2d_wgrad(const float *x, const float *dy, float *dw, int64_t N,
                         int64_t C, int64_t H, int64_t W, int64_t K, int R,
                         int S, int stride, int pad, int64_t n0, int64_t n1,
                         int nthreads);

void oracle_maxpool2x2_fwd(const float *x, float *y, int64_t NC, int64_t H,
                           int64_t W);
void oracle_maxpool2x2_bwd(const float *x, const float *dy, float *dx,
                           int64_t NC, int64_t H, int64_t W);

/* Crater CNN (conv3x3 1->16 + ReLU, pool, conv3x3 16->32 + ReLU, pool,
   dense 8192->64 + ReLU, dense 64->1, sigmoid-BCE mean over the batch, SGD).
   params is the flat parameter vector in the order
   w1[16,1,3,3] b1[16] w2[32,16,3,3] b2[32] w3[64,8192] b3[64] w4[64] b4[1];
   grads has the same layout.  Returns the mean loss. */
#define ORACLE_CNN_NPARAMS 529217
float oracle_cnn_step(float *params, float *grads, const float *images,
                      const float *labels, int64_t batch, int64_t batch_total,
                      float lr, int apply_sgd, int nthreads);

/* The benchmark programs as compiled loops (timed CPU baseline). */
void oracle_chained_fold_f32(const float *x, int64_t rows, int64_t L, float *out,
                             int nthreads);
void oracle_row_norms_f32(const float *x, int64_t rows, int64_t L, float *out,
                          int nthreads);

/* Ascending sort of `rows` contiguous rows of `len` f32 / i32 values: a
   stable merge sort on the numeric order (-0.0 == +0.0 keep their input
   order, as the interpreter's stable np.sort does; qsort in remora_rt.c
   leaves them in some order). */
void oracle_sort(int dtype, const void *in, void *out, int64_t rows, int64_t len,
                 int nthreads);
/* Stable argsort per row: int32 indices, ties in index order
   (remora_rt.c `_cmp_grade_*` breaks ties by index). */
void oracle_grade(int dtype, const void *in, int32_t *out, int64_t rows,
                  int64_t len, int nthreads);
/* Keeps src[i] where the flag is set (mask != 0 for an i32 or one-byte bool
   mask, or `src[i] op literal` for pred, ordered for f32), in order; writes
   at most cap values and returns how many were kept. */
int64_t oracle_filter(int dtype, const void *src, const void *mask, int mask_dtype,
                      const RemoraFilterPred *pred, int64_t n, void *dst, int64_t cap);
/* src[i] repeated max(counts[i], 0) times, in order; writes at most cap
   values and returns the full length. */
int64_t oracle_replicate(int dtype, const void *src, const int32_t *counts, int64_t n,
                         void *dst, int64_t cap);

#ifdef __cplusplus
}
#endif

#endif
