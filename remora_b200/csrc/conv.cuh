// conv.cuh — convolution geometry shared by the direct and tensor-core paths.
#pragma once

#include <cudaTypedefs.h>

#include "common.cuh"

namespace remora {

// cuTensorMapEncodeTiled from the driver (gemm.cu), or null.
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

struct ConvGeom {
  int N, C, H, W, K, R, S, OH, OW, stride, pad;
};

// Tensor-core paths: set *handled = false (and do nothing) for shapes they do
// not cover; the caller then runs the direct kernels.
int conv_tc_fwd(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *w, const float *bias,
                float *y, int precision, cudaStream_t stream, bool *handled);
int conv_tc_dgrad(RemoraB200Ctx *ctx, const ConvGeom &g, const float *dy, const float *w, float *dx,
                  int precision, cudaStream_t stream, bool *handled);
int conv_tc_wgrad(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dy, float *dw,
                  int precision, cudaStream_t stream, bool *handled);

// Fused forms for a conv followed by ReLU + 2x2 max-pool (the crater CNN's
// second layer).  Forward: writes the pooled output and one code byte per
// pooled value (the window element, 0..3, that holds the maximum, or 255
// when it is not positive) instead of y.  Input gradient: takes the pooled
// gradient and the codes in place of dy.
int conv_tc_fwd_relu_pool(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *w, const float *bias,
                          float *pooled, uint8_t *codes, int precision, cudaStream_t stream, bool *handled);
int conv_tc_dgrad_unpool(RemoraB200Ctx *ctx, const ConvGeom &g, const float *dpooled, const uint8_t *codes,
                         const float *w, float *dx, int precision, cudaStream_t stream, bool *handled);

// Tensor-core weight gradient (and bias gradient when db is non-null) for
// 3x3 / pad 1 / stride 1, 16 input channels, at most 32 output channels,
// W in {32, 64}, TF32 or 3xTF32.
int conv_tc_wgrad_bias(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dy, float *dw, float *db,
                       int precision, cudaStream_t stream, bool *handled);
// The same from a pooled gradient and its codes (dy = their unpooling).
int conv_tc_wgrad_bias_unpool(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dpooled,
                              const uint8_t *codes, float *dw, float *db, int precision, cudaStream_t stream,
                              bool *handled);

// Register-tiled weight (and bias, when db is non-null) gradient for 3x3 /
// pad 1 / stride 1 with K even, (K/2)*C threads <= 512, W in {32, 64}.
int conv_wgrad3x3(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dy, float *dw, float *db,
                  cudaStream_t stream, bool *handled);

}  // namespace remora
