// wait_check.cu — the failure-detection path of the bounded device waits,
// exercised on its own: one block waits, with the mbarrier wait every
// tcgen05 kernel here uses (tcgen05.cuh), for a phase that completes only
// when the caller asks for it.  A wait that runs out records its code in the
// stream's error word and the kernel returns, so the context stays usable
// and remora_b200_synchronize reports REMORA_ERR_TIMEOUT.  Nothing is in
// flight while it waits (no TMA copy, no MMA, no TMEM), so running out is
// harmless by construction.
#include "common.cuh"
#include "tcgen05.cuh"

namespace remora {
namespace {

constexpr int kWaitCheckCode = 900;

__global__ void __launch_bounds__(32) wait_check_kernel(long long limit, int signal, int *err) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    tc::mbar_init(&bar, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) {
    if (signal) tc::mbar_arrive(&bar);
    tc::mbar_wait_for(&bar, 0, &abort_flag, err, kWaitCheckCode, limit);
  }
}

}  // namespace
}  // namespace remora

using namespace remora;

extern "C" {

int remora_b200_wait_check(RemoraB200Ctx *ctx, int64_t limit_cycles, int32_t signal, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (limit_cycles < 0 || limit_cycles > (1LL << 40))
    return fail(REMORA_ERR_ARG, "wait_check: limit of %lld cycles outside 0 .. 2^40", (long long)limit_cycles);
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, (cudaStream_t)stream, 0, &ws));
  note_launch();
  wait_check_kernel<<<1, 32, 0, (cudaStream_t)stream>>>((long long)limit_cycles, signal ? 1 : 0, ws->err);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

}  // extern "C"
