// cnn_step.cu — one SGD step of the crater CNN behind a single C call
// (remora_b200_cnn_step): the stages the Python orchestrator
// (remora_b200/cnn.py) enqueues, in the same order and with the same
// kernels, plus the data-parallel gradient sum through the caller's NCCL
// communicator.  The reference trains its CNN one example at a time through
// interpreter callables (examples/crater_train.py:239-257); its formulas
// (ReLU as select, stable BCE, p - lr * g) are those of remora_b200_cnn.h.
//
// NCCL is not linked: ncclAllReduce (and the communicator helpers) are
// looked up in the NCCL the process has already loaded -- the one that made
// the caller's communicator -- or, failing that, in libnccl.so.2.
#include <dlfcn.h>
#include <nccl.h>

#include "common.cuh"
#include "../../include/remora_b200_cnn.h"

namespace remora {
namespace {

// Flat parameter layout: w1[16,1,3,3] b1[16] w2[32,16,3,3] b2[32]
// w3[64,8192] b3[64] w4[64] b4[1] (remora_b200/crater.py)
constexpr int64_t kW1 = 0, kB1 = 144, kW2 = 160, kB2 = 4768, kW3 = 4800, kB3 = 529088, kW4 = 529152,
                  kB4 = 529216, kNParams = 529217;
constexpr int kImage = 64;

// ---------------------------------------------------------------- NCCL
using AllReduceFn = ncclResult_t (*)(const void *, void *, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                                     cudaStream_t);
using UniqueIdFn = ncclResult_t (*)(ncclUniqueId *);
using InitRankFn = ncclResult_t (*)(ncclComm_t *, int, ncclUniqueId, int);
using DestroyFn = ncclResult_t (*)(ncclComm_t);
using ErrorStringFn = const char *(*)(ncclResult_t);

void *nccl_symbol(const char *name) {
  void *f = dlsym(RTLD_DEFAULT, name);
  if (f) return f;
  static void *handle = nullptr;
  if (handle == nullptr) handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
  if (handle == nullptr) handle = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  return handle ? dlsym(handle, name) : nullptr;
}

int nccl_fail(const char *what, ncclResult_t r) {
  auto es = reinterpret_cast<ErrorStringFn>(nccl_symbol("ncclGetErrorString"));
  return fail(REMORA_ERR_CUDA, "%s failed: %s", what, es ? es(r) : "(no message)");
}

// ------------------------------------------------------------- the SGD
// p <- p - lr * g, the product and the difference rounded separately (the
// map program x0 - lr * x1 of the Python step computes the same bits).
__global__ void __launch_bounds__(256) sgd_kernel(float *__restrict__ p, const float *__restrict__ g, float lr,
                                                  long long n) {
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step)
    p[i] = __fsub_rn(p[i], __fmul_rn(lr, g[i]));
}

// ------------------------------------------------------- descriptors
RemoraMemRef1 d1(void *base, int64_t off, int64_t n) {
  RemoraMemRef1 d{};
  d.allocated = d.aligned = base;
  d.offset = off;
  d.sizes[0] = n;
  d.strides[0] = 1;
  return d;
}

RemoraMemRef2 d2(void *base, int64_t off, int64_t r, int64_t c, int64_t sr, int64_t sc) {
  RemoraMemRef2 d{};
  d.allocated = d.aligned = base;
  d.offset = off;
  d.sizes[0] = r;
  d.sizes[1] = c;
  d.strides[0] = sr;
  d.strides[1] = sc;
  return d;
}

RemoraMemRef4 d4(void *base, int64_t off, int64_t a, int64_t b, int64_t c, int64_t e) {
  RemoraMemRef4 d{};
  d.allocated = d.aligned = base;
  d.offset = off;
  d.sizes[0] = a;
  d.sizes[1] = b;
  d.sizes[2] = c;
  d.sizes[3] = e;
  d.strides[3] = 1;
  d.strides[2] = e;
  d.strides[1] = c * e;
  d.strides[0] = b * c * e;
  return d;
}

size_t align256(size_t v) { return (v + 255) & ~(size_t)255; }

}  // namespace
}  // namespace remora

using namespace remora;

extern "C" {

int remora_b200_cnn_step(RemoraB200Ctx *ctx, const RemoraCnnStepSpec *spec, RemoraMemRef1 *params,
                         RemoraMemRef1 *grads, const RemoraMemRef4 *images, const RemoraMemRef1 *labels,
                         RemoraMemRef1 *losses, void *nccl_comm, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (spec == nullptr || params == nullptr || grads == nullptr || images == nullptr || labels == nullptr)
    return fail(REMORA_ERR_ARG, "cnn_step: null argument");
  const int64_t B = spec->batch, BT = spec->batch_total;
  if (B < 1 || BT < B) return fail(REMORA_ERR_ARG, "cnn_step: batch %lld of a global %lld", (long long)B, (long long)BT);
  if (spec->precision < REMORA_CNN_MIXED || spec->precision > REMORA_CNN_TF32)
    return fail(REMORA_ERR_ARG, "cnn_step: unknown precision %d", spec->precision);
  DescView P, G, X, Y;
  REMORA_TRY(read_desc(params, 1, &P, "parameters"));
  REMORA_TRY(read_desc(grads, 1, &G, "gradients"));
  REMORA_TRY(read_desc(images, 4, &X, "images"));
  REMORA_TRY(read_desc(labels, 1, &Y, "labels"));
  if (P.sizes[0] != kNParams || G.sizes[0] != kNParams || !P.contiguous() || !G.contiguous())
    return fail(REMORA_ERR_SHAPE, "cnn_step: parameters and gradients are contiguous f32[%lld]", (long long)kNParams);
  if (X.sizes[0] != B || X.sizes[1] != 1 || X.sizes[2] != kImage || X.sizes[3] != kImage || Y.sizes[0] != B)
    return fail(REMORA_ERR_SHAPE, "cnn_step: images [%lld,1,64,64] and labels [%lld]", (long long)B, (long long)B);
  DescView LS;
  if (losses != nullptr) {
    REMORA_TRY(read_desc(losses, 1, &LS, "losses"));
    if (LS.sizes[0] != B || !LS.contiguous()) return fail(REMORA_ERR_SHAPE, "cnn_step: losses f32[%lld]", (long long)B);
  }
  AllReduceFn allreduce = nullptr;
  if (nccl_comm != nullptr) {
    allreduce = reinterpret_cast<AllReduceFn>(nccl_symbol("ncclAllReduce"));
    if (allreduce == nullptr)
      return fail(REMORA_ERR_UNSUPPORTED, "cnn_step: a communicator was given but no NCCL is loaded");
  }
  cudaStream_t s = (cudaStream_t)stream;

  // activations of this rank's shard, in the stream's activation buffer
  const size_t sz_p1 = align256((size_t)B * 16 * 32 * 32 * 4), sz_c1 = align256((size_t)B * 16 * 32 * 32);
  const size_t sz_p2 = align256((size_t)B * 32 * 16 * 16 * 4), sz_c2 = align256((size_t)B * 32 * 16 * 16);
  const size_t sz_h = align256((size_t)B * 64 * 4), sz_v = align256((size_t)B * 4);
  const size_t total = sz_p1 + sz_c1 + sz_p2 + sz_c2 + 3 * sz_h + 3 * sz_v + sz_p2 + sz_p1;
  void *act = nullptr;
  REMORA_TRY(get_activations(ctx, s, total, &act));
  char *a = static_cast<char *>(act);
  auto take = [&](size_t n) {
    char *q = a;
    a += n;
    return q;
  };
  char *p1 = take(sz_p1), *c1 = take(sz_c1), *p2 = take(sz_p2), *c2 = take(sz_c2);
  char *hpre = take(sz_h), *h = take(sz_h), *dh = take(sz_h);
  char *z = take(sz_v), *lossb = take(sz_v), *dz = take(sz_v);
  char *dp2 = take(sz_p2), *dp1 = take(sz_p1);

  // parameter and gradient views into the flat buffers
  void *pb = P.data(4), *gb = G.data(4);
  RemoraMemRef4 w1 = d4(pb, kW1, 16, 1, 3, 3), w2 = d4(pb, kW2, 32, 16, 3, 3);
  RemoraMemRef1 b1 = d1(pb, kB1, 16), b2 = d1(pb, kB2, 32), b3 = d1(pb, kB3, 64), w4 = d1(pb, kW4, 64),
                b4 = d1(pb, kB4, 1);
  RemoraMemRef2 w3 = d2(pb, kW3, 64, 8192, 8192, 1), w3t = d2(pb, kW3, 8192, 64, 1, 8192);
  RemoraMemRef4 gw1 = d4(gb, kW1, 16, 1, 3, 3), gw2 = d4(gb, kW2, 32, 16, 3, 3);
  RemoraMemRef1 gb1 = d1(gb, kB1, 16), gb2 = d1(gb, kB2, 32), gb3 = d1(gb, kB3, 64), gw4 = d1(gb, kW4, 64),
                gb4 = d1(gb, kB4, 1);
  // dense1's weight gradient as its transpose [8192, 64] (column-major in
  // the flat buffer): 64 row blocks of 128 over the 8192 features
  RemoraMemRef2 gw3t = d2(gb, kW3, 8192, 64, 1, 8192);
  // activations
  RemoraMemRef4 P1 = d4(p1, 0, B, 16, 32, 32), C1 = d4(c1, 0, B, 16, 32, 32);
  RemoraMemRef4 P2 = d4(p2, 0, B, 32, 16, 16), C2 = d4(c2, 0, B, 32, 16, 16);
  RemoraMemRef2 P2f = d2(p2, 0, B, 8192, 8192, 1), DP2f = d2(dp2, 0, B, 8192, 8192, 1),
                P2ft = d2(p2, 0, 8192, B, 1, 8192);
  RemoraMemRef4 DP2 = d4(dp2, 0, B, 32, 16, 16), DP1 = d4(dp1, 0, B, 16, 32, 32);
  RemoraMemRef2 Hpre = d2(hpre, 0, B, 64, 64, 1), H = d2(h, 0, B, 64, 64, 1), DH = d2(dh, 0, B, 64, 64, 1);
  RemoraMemRef1 Z = d1(z, 0, B), DZ = d1(dz, 0, B);
  RemoraMemRef1 LB = losses != nullptr ? *losses : d1(lossb, 0, B);

  const int fwd = spec->precision == REMORA_CNN_TF32 ? REMORA_PREC_TF32 : REMORA_PREC_3XTF32;
  const int bwd = spec->precision == REMORA_CNN_MIXED ? REMORA_PREC_2XTF32 : fwd;
  const RemoraConvSpec cf{1, 1, fwd, 0}, cb{1, 1, bwd, 0};
  const RemoraGemmSpec gs{fwd, 0};

  // forward
  REMORA_TRY(remora_b200_conv1_relu_pool(ctx, images, &w1, &b1, &P1, &C1, stream));
  REMORA_TRY(remora_b200_conv2d_fwd_relu_pool(ctx, &cf, &P1, &w2, &b2, &P2, &C2, stream));
  REMORA_TRY(remora_b200_gemm(ctx, &gs, &P2f, &w3t, &Hpre, 2, stream));
  REMORA_TRY(remora_b200_dense_bias_relu_bce(ctx, &Hpre, &b3, &H, &w4, &b4, labels, &Z, &LB, &DZ,
                                             1.0f / (float)BT, stream));
  // backward
  REMORA_TRY(remora_b200_dense_relu_bwd(ctx, &H, &w4, &DZ, &DH, &gw4, &gb4, &gb3, stream));
  REMORA_TRY(remora_b200_gemm(ctx, &gs, &P2ft, &DH, &gw3t, 2, stream));
  REMORA_TRY(remora_b200_gemm(ctx, &gs, &DH, &w3, &DP2f, 2, stream));
  REMORA_TRY(remora_b200_conv2d_wgrad_bias_unpool(ctx, &cb, &P1, &DP2, &C2, &gw2, &gb2, stream));
  REMORA_TRY(remora_b200_conv2d_dgrad_unpool(ctx, &cb, &DP2, &C2, &w2, &DP1, stream));
  REMORA_TRY(remora_b200_conv1_wgrad_pooled(ctx, images, &DP1, &C1, &gw1, &gb1, stream));
  // the gradient summed over the ranks (each already carries 1/global batch)
  if (allreduce != nullptr) {
    float *g = static_cast<float *>(gb);
    const ncclResult_t r = allreduce(g, g, (size_t)kNParams, ncclFloat32, ncclSum,
                                     static_cast<ncclComm_t>(nccl_comm), s);
    if (r != ncclSuccess) return nccl_fail("ncclAllReduce", r);
  }
  note_launch();
  sgd_kernel<<<(int)std::min<long long>((kNParams + 255) / 256, (long long)ctx->sm_count * 8), 256, 0, s>>>(
      static_cast<float *>(pb), static_cast<const float *>(gb), spec->lr, kNParams);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_nccl_unique_id(void *id_out) {
  if (id_out == nullptr) return fail(REMORA_ERR_ARG, "nccl_unique_id: null output");
  auto fn = reinterpret_cast<UniqueIdFn>(nccl_symbol("ncclGetUniqueId"));
  if (fn == nullptr) return fail(REMORA_ERR_UNSUPPORTED, "nccl_unique_id: NCCL is not available");
  ncclUniqueId id;
  const ncclResult_t r = fn(&id);
  if (r != ncclSuccess) return nccl_fail("ncclGetUniqueId", r);
  std::memcpy(id_out, &id, sizeof(id));
  return REMORA_OK;
}

int remora_b200_nccl_comm_init(void **comm_out, int32_t nranks, const void *id, int32_t rank) {
  if (comm_out == nullptr || id == nullptr) return fail(REMORA_ERR_ARG, "nccl_comm_init: null argument");
  if (nranks < 1 || rank < 0 || rank >= nranks) return fail(REMORA_ERR_ARG, "nccl_comm_init: rank %d of %d", rank, nranks);
  auto fn = reinterpret_cast<InitRankFn>(nccl_symbol("ncclCommInitRank"));
  if (fn == nullptr) return fail(REMORA_ERR_UNSUPPORTED, "nccl_comm_init: NCCL is not available");
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  const ncclResult_t r = fn(&comm, nranks, uid, rank);
  if (r != ncclSuccess) return nccl_fail("ncclCommInitRank", r);
  *comm_out = comm;
  return REMORA_OK;
}

int remora_b200_nccl_comm_destroy(void *comm) {
  if (comm == nullptr) return REMORA_OK;
  auto fn = reinterpret_cast<DestroyFn>(nccl_symbol("ncclCommDestroy"));
  if (fn == nullptr) return fail(REMORA_ERR_UNSUPPORTED, "nccl_comm_destroy: NCCL is not available");
  const ncclResult_t r = fn(static_cast<ncclComm_t>(comm));
  if (r != ncclSuccess) return nccl_fail("ncclCommDestroy", r);
  return REMORA_OK;
}

}  // extern "C"
