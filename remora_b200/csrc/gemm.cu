// gemm.cu — dense core (remora_b200_gemm).  The tcgen05 kernel is not in
// this build yet; the entry point reports that instead of computing.
#include "common.cuh"

using namespace remora;

extern "C" int remora_b200_gemm(RemoraB200Ctx *ctx, const RemoraGemmSpec *spec, const void *a_desc,
                                const void *b_desc, void *c_desc, int32_t rank, remora_stream_t stream) {
  (void)spec, (void)a_desc, (void)b_desc, (void)c_desc, (void)rank, (void)stream;
  REMORA_TRY(check_ctx(ctx));
  return fail(REMORA_ERR_UNSUPPORTED, "gemm: the tcgen05 kernel is not part of this build yet");
}
