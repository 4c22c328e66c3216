/*
 * remora_b200_cnn.h — fused kernels of the crater-CNN training step, on top
 * of the hot-path entry points of remora_b200.h (conv2d, gemm, fold, map).
 *
 * The reference trains its crater CNN one example at a time through
 * interpreter callables, one gradient function per parameter
 * (examples/crater_train.py:169-281); its formulas are ReLU as
 * select(v > 0, v, 0), the stable BCE on a logit
 * (examples/crater_train.py:46-54) and SGD p - lr * g (:249-253).  These
 * entry points implement the batched model of the benchmark (64x64 images,
 * conv 1->16 / pool / conv 16->32 / pool / dense 8192->64 / dense 64->1):
 * max-pool, batch-mean BCE and multi-channel convolution have no reference
 * counterpart.
 *
 * Pool codes: one byte per pooled output, the window index (0..3, order
 * (0,0) (0,1) (1,0) (1,1), first maximum wins) of the element that receives
 * the gradient, or 255 when the maximum is not positive (ReLU blocks it).
 */
#ifndef REMORA_B200_CNN_H
#define REMORA_B200_CNN_H

#include "remora_b200.h"

#ifdef __cplusplus
extern "C" {
#endif

/* pooled = maxpool2x2(relu(conv3x3_pad1(x, w) + bias)) for a single input
   channel; x [B,1,H,W], w [K,1,3,3], bias [K], pooled and code [B,K,H/2,W/2]
   (code holds bytes).  The conv sums follow the reference's per-channel dot
   order (remora/runtime.py:1274-1288 with examples/crater_train.py:30-36). */
int remora_b200_conv1_relu_pool(RemoraB200Ctx *ctx, const RemoraMemRef4 *x,
                                const RemoraMemRef4 *w,
                                const RemoraMemRef1 *bias,
                                RemoraMemRef4 *pooled, RemoraMemRef4 *code,
                                remora_stream_t stream);

/* pooled = maxpool2x2(relu(a)) for a [N,C,H,W] (H, W even). */
int remora_b200_relu_pool(RemoraB200Ctx *ctx, const RemoraMemRef4 *a,
                          RemoraMemRef4 *pooled, RemoraMemRef4 *code,
                          remora_stream_t stream);

/* Adjoint of relu_pool: da [N,C,H,W] gets dpooled at each recorded element
   and 0 elsewhere (the select VJP of remora/ad.py:172-179). */
int remora_b200_unpool(RemoraB200Ctx *ctx, const RemoraMemRef4 *dpooled,
                       const RemoraMemRef4 *code, RemoraMemRef4 *da,
                       remora_stream_t stream);

/* z[b] = b + sum_o w[o] h[b,o]; loss[b] = stable BCE(z[b], y[b])
   (examples/crater_train.py:50-54); dz[b] = (sigmoid(z[b]) - y[b]) *
   grad_scale (grad_scale = 1 / global batch for a batch-mean loss). */
int remora_b200_dense_bce(RemoraB200Ctx *ctx, const RemoraMemRef2 *h,
                          const RemoraMemRef1 *w, const RemoraMemRef1 *b,
                          const RemoraMemRef1 *y, RemoraMemRef1 *z,
                          RemoraMemRef1 *loss, RemoraMemRef1 *dz,
                          float grad_scale, remora_stream_t stream);

/* The same with the hidden layer's bias and ReLU fused in front:
   h[b,o] = relu(hpre[b,o] + hb[o]) (the select form of
   examples/crater_train.py:46-48, one rounded add) is written to h and
   feeds the dense 64 -> 1 layer, the BCE and its gradient as above. */
int remora_b200_dense_bias_relu_bce(RemoraB200Ctx *ctx, const RemoraMemRef2 *hpre,
                                    const RemoraMemRef1 *hb, RemoraMemRef2 *h,
                                    const RemoraMemRef1 *w, const RemoraMemRef1 *b,
                                    const RemoraMemRef1 *y, RemoraMemRef1 *z,
                                    RemoraMemRef1 *loss, RemoraMemRef1 *dz,
                                    float grad_scale, remora_stream_t stream);

/* Backward of the dense 64 -> 1 layer on a ReLU'd hidden layer:
   dw[o] = sum_b dz[b] h[b,o], db = sum_b dz[b],
   dh[b,o] = h[b,o] > 0 ? dz[b] * w[o] : 0, and, when dh_colsum is not
   NULL, dh_colsum[o] = sum_b dh[b,o] (the gradient of the hidden layer's
   bias).  Sums in f64, fixed order. */
int remora_b200_dense_relu_bwd(RemoraB200Ctx *ctx, const RemoraMemRef2 *h,
                               const RemoraMemRef1 *w, const RemoraMemRef1 *dz,
                               RemoraMemRef2 *dh, RemoraMemRef1 *dw,
                               RemoraMemRef1 *db, RemoraMemRef1 *dh_colsum,
                               remora_stream_t stream);

/* conv1's weight and bias gradients straight from the pooled gradient and
   the pool codes (the unpooled gradient is never materialised):
   x [B,1,H,W], dpooled/code [B,K,H/2,W/2], dw [K,1,3,3], db [K]. */
int remora_b200_conv1_wgrad_pooled(RemoraB200Ctx *ctx, const RemoraMemRef4 *x,
                                   const RemoraMemRef4 *dpooled,
                                   const RemoraMemRef4 *code, RemoraMemRef4 *dw,
                                   RemoraMemRef1 *db, remora_stream_t stream);

/* Fused second layer: pooled = maxpool2x2(relu(conv3x3_pad1(x, w) + bias))
   on the tensor cores (TF32 or 3xTF32 per spec), x [B,C,H,W] (C = 16,
   W = 32), w [K,C,3,3] (K = 17..32), pooled and code [B,K,H/2,W/2]; the
   full-resolution activation is never written.  Other shapes return
   REMORA_ERR_UNSUPPORTED. */
int remora_b200_conv2d_fwd_relu_pool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                                     const RemoraMemRef4 *x, const RemoraMemRef4 *w,
                                     const RemoraMemRef1 *bias, RemoraMemRef4 *pooled,
                                     RemoraMemRef4 *code, remora_stream_t stream);

/* Input gradient of that layer from the pooled gradient: dx = conv2d_dgrad(
   unpool(dpooled, code), w) with the unpooled gradient formed on the fly
   (dpooled/code [B,K,H/2,W/2], K = 32; w [K,C,3,3], C <= 16; dx [B,C,H,W],
   W = 32). */
int remora_b200_conv2d_dgrad_unpool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                                    const RemoraMemRef4 *dpooled,
                                    const RemoraMemRef4 *code, const RemoraMemRef4 *w,
                                    RemoraMemRef4 *dx, remora_stream_t stream);

/* Weight and bias gradients of that layer from the pooled gradient
   (x [B,16,H,W], W = 32; dpooled/code [B,K,H/2,W/2]; dw [K,16,3,3]; db [K]). */
int remora_b200_conv2d_wgrad_bias_unpool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                                         const RemoraMemRef4 *x,
                                         const RemoraMemRef4 *dpooled,
                                         const RemoraMemRef4 *code, RemoraMemRef4 *dw,
                                         RemoraMemRef1 *db, remora_stream_t stream);

/* Weight gradient plus bias gradient db[k] = sum over n, i, j of dy[n,k,i,j]
   (the fold VJP of remora/ad.py:106-110 for the broadcast bias). */
int remora_b200_conv2d_wgrad_bias(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                                  const RemoraMemRef4 *x,
                                  const RemoraMemRef4 *dy, RemoraMemRef4 *dw,
                                  RemoraMemRef1 *db, remora_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* REMORA_B200_CNN_H */
