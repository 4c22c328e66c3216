// conv.cu — NCHW convolution forward and reverse mode.  The implicit-GEMM
// kernels are not in this build yet; the entry points report that.
#include "common.cuh"

using namespace remora;

extern "C" {

int remora_b200_conv2d_fwd(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                           const RemoraMemRef4 *w, const RemoraMemRef1 *bias, RemoraMemRef4 *y,
                           remora_stream_t stream) {
  (void)spec, (void)x, (void)w, (void)bias, (void)y, (void)stream;
  REMORA_TRY(check_ctx(ctx));
  return fail(REMORA_ERR_UNSUPPORTED, "conv2d_fwd: not part of this build yet");
}

int remora_b200_conv2d_dgrad(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *dy,
                             const RemoraMemRef4 *w, RemoraMemRef4 *dx, remora_stream_t stream) {
  (void)spec, (void)dy, (void)w, (void)dx, (void)stream;
  REMORA_TRY(check_ctx(ctx));
  return fail(REMORA_ERR_UNSUPPORTED, "conv2d_dgrad: not part of this build yet");
}

int remora_b200_conv2d_wgrad(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                             const RemoraMemRef4 *dy, RemoraMemRef4 *dw, remora_stream_t stream) {
  (void)spec, (void)x, (void)dy, (void)dw, (void)stream;
  REMORA_TRY(check_ctx(ctx));
  return fail(REMORA_ERR_UNSUPPORTED, "conv2d_wgrad: not part of this build yet");
}

}  // extern "C"
