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

/* pooled = maxpool2x2(relu(a)) for a [N,C,H,W] (H, W even); ReLU is the
   select form of examples/crater_train.py:46-48, the pooling has no
   reference counterpart. */
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
   bias).  Sums in f64, fixed order.  The dot, fold and select VJPs of
   remora/ad.py (:91-95, :106-110, :172-179) batched over the samples, in
   place of the reference's per-parameter gradient functions
   (examples/crater_train.py:169-198). */
int remora_b200_dense_relu_bwd(RemoraB200Ctx *ctx, const RemoraMemRef2 *h,
                               const RemoraMemRef1 *w, const RemoraMemRef1 *dz,
                               RemoraMemRef2 *dh, RemoraMemRef1 *dw,
                               RemoraMemRef1 *db, RemoraMemRef1 *dh_colsum,
                               remora_stream_t stream);

/* conv1's weight and bias gradients straight from the pooled gradient and
   the pool codes (the unpooled gradient is never materialised):
   x [B,1,H,W], dpooled/code [B,K,H/2,W/2], dw [K,1,3,3], db [K].  The
   select VJP (remora/ad.py:172-179) composed with the conv weight and bias
   VJPs (:91-95, :106-110), in place of the reference's per-parameter
   gradient functions (examples/crater_train.py:169-198). */
int remora_b200_conv1_wgrad_pooled(RemoraB200Ctx *ctx, const RemoraMemRef4 *x,
                                   const RemoraMemRef4 *dpooled,
                                   const RemoraMemRef4 *code, RemoraMemRef4 *dw,
                                   RemoraMemRef1 *db, remora_stream_t stream);

/* Fused second layer: pooled = maxpool2x2(relu(conv3x3_pad1(x, w) + bias))
   on the tensor cores (TF32 or 3xTF32 per spec), x [B,C,H,W] (C = 16,
   W = 32), w [K,C,3,3] (K = 17..32), pooled and code [B,K,H/2,W/2]; the
   full-resolution activation is never written.  Other shapes return
   REMORA_ERR_UNSUPPORTED.  The reference's conv2d (examples/crater_train.py:
   30-36, a dot over each im2col patch) and ReLU (:46-48) for many channels
   at once; the pooling has no reference counterpart. */
int remora_b200_conv2d_fwd_relu_pool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                                     const RemoraMemRef4 *x, const RemoraMemRef4 *w,
                                     const RemoraMemRef1 *bias, RemoraMemRef4 *pooled,
                                     RemoraMemRef4 *code, remora_stream_t stream);

/* Input gradient of that layer from the pooled gradient: dx = conv2d_dgrad(
   unpool(dpooled, code), w) with the unpooled gradient formed on the fly
   (dpooled/code [B,K,H/2,W/2], K = 32; w [K,C,3,3], C <= 16; dx [B,C,H,W],
   W = 32).  The select VJP (remora/ad.py:172-179) composed with the conv
   input VJP (:157-171). */
int remora_b200_conv2d_dgrad_unpool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                                    const RemoraMemRef4 *dpooled,
                                    const RemoraMemRef4 *code, const RemoraMemRef4 *w,
                                    RemoraMemRef4 *dx, remora_stream_t stream);

/* Weight and bias gradients of that layer from the pooled gradient
   (x [B,16,H,W], W = 32; dpooled/code [B,K,H/2,W/2]; dw [K,16,3,3]; db [K]).
   The select VJP (remora/ad.py:172-179) composed with the conv weight and
   bias VJPs (:91-95, :106-110), in place of the reference's per-parameter
   gradient functions (examples/crater_train.py:169-198). */
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

/* ------------------------------------------------------------------------ */
/* One SGD step of the crater CNN in one call                                */
/* ------------------------------------------------------------------------ */
/* Tensor-core precision of the step.  MIXED: 3xTF32 for the second conv
   layer's forward and every dense-layer GEMM, 2xTF32 for that conv layer's
   two gradients (every gradient within 1e-3 of the f32 step).  3XTF32:
   split precision everywhere.  TF32: single-pass TF32 everywhere, outside
   the 1e-3 gradient tolerance (a speed reference). */
enum { REMORA_CNN_MIXED = 0, REMORA_CNN_3XTF32 = 1, REMORA_CNN_TF32 = 2 };

typedef struct {
  int32_t batch;       /* images of this rank's shard                         */
  int32_t batch_total; /* global batch: the loss is the mean over it          */
  float lr;            /* SGD learning rate                                   */
  int32_t precision;   /* REMORA_CNN_*                                        */
} RemoraCnnStepSpec;

/* One SGD step on this rank's shard: forward, backward, the gradient summed
   over the data-parallel ranks, the update p <- p - lr * g; everything is
   enqueued on `stream`.  The reference trains its CNN one example at a time
   through six interpreted gradient functions (examples/crater_train.py:
   169-198, 239-257); this is the batched step of its formulas (stable BCE
   :50-54, ReLU as select :46-48, SGD :249-253).
   params, grads: contiguous f32[529217] device buffers in the layout
   w1[16,1,3,3] b1[16] w2[32,16,3,3] b2[32] w3[64,8192] b3[64] w4[64] b4[1];
   params is updated in place, grads receives the step's gradient (summed
   over the ranks).  images [B,1,64,64], labels [B] (1 crater, 0 none),
   losses [B] (optional, may be NULL): each sample's BCE.
   nccl_comm: an ncclComm_t over the data-parallel ranks, each calling this
   entry point with its own shard (NULL for a single rank); the gradient is
   summed with one ncclAllReduce on `stream`, through the NCCL library the
   process has loaded (the one that made the communicator).  The
   activations live in a device buffer the library keeps per stream (about
   220 KB per image), grown on the first call: make that call before any
   stream capture. */
int remora_b200_cnn_step(RemoraB200Ctx *ctx, const RemoraCnnStepSpec *spec,
                         RemoraMemRef1 *params, RemoraMemRef1 *grads,
                         const RemoraMemRef4 *images, const RemoraMemRef1 *labels,
                         RemoraMemRef1 *losses, void *nccl_comm,
                         remora_stream_t stream);

/* Communicator helpers for callers without NCCL plumbing of their own,
   through the same NCCL as remora_b200_cnn_step: a unique id (128 bytes,
   made by one rank and handed to the others by any host channel), a
   communicator of rank `rank` of `nranks` (the device current on the
   calling thread), and its release.  No counterpart in the reference,
   which trains on one device. */
int remora_b200_nccl_unique_id(void *id_out);
int remora_b200_nccl_comm_init(void **comm_out, int32_t nranks, const void *id,
                               int32_t rank);
int remora_b200_nccl_comm_destroy(void *comm);

#ifdef __cplusplus
}
#endif

#endif /* REMORA_B200_CNN_H */
