// context.cu — context, plumbing and error reporting of libremora_b200.so.
// Replaces the reference's CUDARuntime (remora/runtime.py:243-340): device
// selection, allocation, copies, memset and synchronisation.
#include <atomic>
#include <cstdarg>

#include "common.cuh"

namespace remora {

static thread_local std::string g_last_error;
static std::atomic<unsigned long long> g_launches{0};

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

void set_error(const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
}

int fail(int code, const char *fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

int dtype_size(int dtype) {
  switch (dtype) {
  case REMORA_F32: return 4;
  case REMORA_I32: return 4;
  case REMORA_BOOL: return 1;
  default: return 0;
  }
}

int read_desc(const void *desc, int rank, DescView *out, const char *what) {
  if (desc == nullptr) return fail(REMORA_ERR_ARG, "%s: null descriptor", what);
  if (rank < 0 || rank > REMORA_MAX_RANK)
    return fail(REMORA_ERR_RANK, "%s: rank %d outside 0..%d", what, rank,
                REMORA_MAX_RANK);
  const char *p = static_cast<const char *>(desc);
  DescView v;
  std::memcpy(&v.aligned, p + 8, sizeof(void *));
  std::memcpy(&v.offset, p + 16, 8);
  v.rank = rank;
  for (int d = 0; d < rank; ++d) {
    std::memcpy(&v.sizes[d], p + 24 + 8 * d, 8);
    std::memcpy(&v.strides[d], p + 24 + 8 * rank + 8 * d, 8);
    if (v.sizes[d] < 0)
      return fail(REMORA_ERR_ARG, "%s: negative size %lld on axis %d", what,
                  (long long)v.sizes[d], d);
  }
  if (v.aligned == nullptr && v.numel() > 0)
    return fail(REMORA_ERR_ARG, "%s: null aligned pointer", what);
  *out = v;
  return REMORA_OK;
}

int check_ctx(RemoraB200Ctx *ctx) {
  if (ctx == nullptr) return fail(REMORA_ERR_ARG, "null context");
  REMORA_CUDA_TRY(cudaSetDevice(ctx->device));
  return REMORA_OK;
}

int get_workspace(RemoraB200Ctx *ctx, cudaStream_t stream, size_t bytes,
                  Workspace **out) {
  std::lock_guard<std::mutex> lock(ctx->mu);
  Workspace &w = ctx->ws[stream];
  if (w.err == nullptr) {
    REMORA_CUDA_TRY(cudaMalloc(&w.err, 256));
    REMORA_CUDA_TRY(cudaMemsetAsync(w.err, 0, 256, stream));
  }
  if (w.bytes < bytes) {
    if (w.buf) {
      // The old buffer may still be read by work queued on this stream.
      REMORA_CUDA_TRY(cudaStreamSynchronize(stream));
      REMORA_CUDA_TRY(cudaFree(w.buf));
      w.buf = nullptr;
      w.bytes = 0;
    }
    size_t want = bytes < (1u << 20) ? (1u << 20) : bytes;
    REMORA_CUDA_TRY(cudaMalloc(&w.buf, want));
    REMORA_CUDA_TRY(cudaMemsetAsync(w.buf, 0, want, stream));
    w.bytes = want;
  }
  *out = &w;
  return REMORA_OK;
}

int get_activations(RemoraB200Ctx *ctx, cudaStream_t stream, size_t bytes, void **out) {
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  std::lock_guard<std::mutex> lock(ctx->mu);
  if (ws->act_bytes < bytes) {
    if (ws->act) {
      REMORA_CUDA_TRY(cudaStreamSynchronize(stream));
      REMORA_CUDA_TRY(cudaFree(ws->act));
      ws->act = nullptr;
      ws->act_bytes = 0;
    }
    REMORA_CUDA_TRY(cudaMalloc(&ws->act, bytes));
    ws->act_bytes = bytes;
  }
  *out = ws->act;
  return REMORA_OK;
}

}  // namespace remora

using namespace remora;

extern "C" {

const char *remora_b200_version(void) { return "remora_b200 0.1 (sm_100a)"; }

unsigned long long remora_b200_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int remora_b200_last_error(char *buf, size_t n) {
  if (buf == nullptr || n == 0) return REMORA_ERR_ARG;
  std::snprintf(buf, n, "%s", g_last_error.c_str());
  return REMORA_OK;
}

int remora_b200_init(int device, RemoraB200Ctx **ctx) {
  if (ctx == nullptr) return fail(REMORA_ERR_ARG, "init: null ctx out-pointer");
  int count = 0;
  REMORA_CUDA_TRY(cudaGetDeviceCount(&count));
  if (device < 0 || device >= count)
    return fail(REMORA_ERR_ARG, "init: device %d outside 0..%d", device, count - 1);
  cudaDeviceProp prop;
  REMORA_CUDA_TRY(cudaGetDeviceProperties(&prop, device));
  if (prop.major != 10)
    return fail(REMORA_ERR_UNSUPPORTED,
                "init: device %d is sm_%d%d; this library is built for sm_100a",
                device, prop.major, prop.minor);
  REMORA_CUDA_TRY(cudaSetDevice(device));
  RemoraB200Ctx *c = new RemoraB200Ctx();
  c->device = device;
  c->sm_count = prop.multiProcessorCount;
  *ctx = c;
  return REMORA_OK;
}

int remora_b200_shutdown(RemoraB200Ctx *ctx) {
  if (ctx == nullptr) return REMORA_OK;
  cudaSetDevice(ctx->device);
  int status = REMORA_OK;
  for (auto &kv : ctx->ws) {
    cudaStreamSynchronize(kv.first);
    if (kv.second.buf && cudaFree(kv.second.buf) != cudaSuccess) status = REMORA_ERR_CUDA;
    if (kv.second.err && cudaFree(kv.second.err) != cudaSuccess) status = REMORA_ERR_CUDA;
    if (kv.second.act && cudaFree(kv.second.act) != cudaSuccess) status = REMORA_ERR_CUDA;
  }
  ctx->ws.clear();
  delete ctx;
  if (status != REMORA_OK) set_error("shutdown: cudaFree failed");
  return status;
}

int remora_b200_malloc(RemoraB200Ctx *ctx, size_t nbytes, void **dptr) {
  REMORA_TRY(check_ctx(ctx));
  if (dptr == nullptr) return fail(REMORA_ERR_ARG, "malloc: null out-pointer");
  *dptr = nullptr;
  if (nbytes == 0) nbytes = 16;
  REMORA_CUDA_TRY(cudaMalloc(dptr, nbytes));
  return REMORA_OK;
}

int remora_b200_free(RemoraB200Ctx *ctx, void *dptr) {
  REMORA_TRY(check_ctx(ctx));
  if (dptr) REMORA_CUDA_TRY(cudaFree(dptr));
  return REMORA_OK;
}

int remora_b200_memcpy_h2d(RemoraB200Ctx *ctx, void *dst, const void *src,
                           size_t nbytes, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (nbytes == 0) return REMORA_OK;
  REMORA_CUDA_TRY(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyHostToDevice,
                                  (cudaStream_t)stream));
  return REMORA_OK;
}

int remora_b200_memcpy_d2h(RemoraB200Ctx *ctx, void *dst, const void *src,
                           size_t nbytes, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (nbytes == 0) return REMORA_OK;
  REMORA_CUDA_TRY(cudaMemcpyAsync(dst, src, nbytes, cudaMemcpyDeviceToHost,
                                  (cudaStream_t)stream));
  return REMORA_OK;
}

int remora_b200_memset_d32(RemoraB200Ctx *ctx, void *dst, uint32_t value,
                           size_t count, remora_stream_t stream);

int remora_b200_synchronize(RemoraB200Ctx *ctx, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  cudaStream_t s = (cudaStream_t)stream;
  REMORA_CUDA_TRY(cudaStreamSynchronize(s));
  int *err = nullptr;
  {
    std::lock_guard<std::mutex> lock(ctx->mu);
    auto it = ctx->ws.find(s);
    if (it != ctx->ws.end()) err = it->second.err;
  }
  if (err) {
    int host_err = 0;
    REMORA_CUDA_TRY(cudaMemcpy(&host_err, err, sizeof(int), cudaMemcpyDeviceToHost));
    if (host_err != 0) {
      REMORA_CUDA_TRY(cudaMemset(err, 0, sizeof(int)));
      return fail(REMORA_ERR_TIMEOUT,
                  "a bounded device wait ran out (code %d); results of the "
                  "affected call are invalid",
                  host_err);
    }
  }
  return REMORA_OK;
}

int remora_b200_set_persistent_sms(RemoraB200Ctx *ctx, int32_t n) {
  REMORA_TRY(check_ctx(ctx));
  ctx->persistent_sms.store(n > 0 ? n : 0, std::memory_order_relaxed);
  return REMORA_OK;
}

int remora_b200_host_register(void *ptr, size_t nbytes) {
  REMORA_CUDA_TRY(cudaHostRegister(ptr, nbytes, cudaHostRegisterDefault));
  return REMORA_OK;
}

int remora_b200_host_unregister(void *ptr) {
  REMORA_CUDA_TRY(cudaHostUnregister(ptr));
  return REMORA_OK;
}

}  // extern "C"
