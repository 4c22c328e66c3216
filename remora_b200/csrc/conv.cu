// conv.cu — NCHW convolution forward and reverse mode (remora_b200_conv2d_*).
//
// The reference's conv2d is single-channel cross-correlation built from
// im2col and a lifted dot, plus a scalar bias (examples/crater_train.py:30-36,
// remora/runtime.py:1274-1288); its reverse mode is col2im for the image
// (remora/ad.py:157-171) and the mul/fold VJPs for the kernel
// (remora/ad.py:88-110).  This file extends it to batches, channels and zero
// padding:
//   y[n,k,i,j]  = sum_c ( sum_{a,b} x[n,c,i*s+a-p, j*s+b-p] * w[k,c,a,b] ) + bias[k]
//   dx[n,c,h,q] = sum_{k,a,b} dy[n,k,(h+p-a)/s,(q+p-b)/s] * w[k,c,a,b]
//   dw[k,c,a,b] = sum_{n,i,j} dy[n,k,i,j] * x[n,c,i*s+a-p, j*s+b-p]
//
// Two paths.  The tensor-core path (conv_tc.cu) covers the 3x3 / pad 1 /
// stride 1 shapes of the benchmark and the crater CNN.  Every other shape
// runs the direct kernels below: one thread per output element, forward sums
// in the reference's order (per-channel dot over taps, then over channels;
// f32 ops rounded one by one), reverse sums in f64 like the reference's tape.
#include <algorithm>

#include "../../include/remora_b200_cnn.h"
#include "conv.cuh"

namespace remora {

namespace {

__global__ void __launch_bounds__(256) conv_fwd_direct(const float *__restrict__ x, const float *__restrict__ w,
                                                       const float *__restrict__ bias, float *__restrict__ y,
                                                       ConvGeom g) {
  const long long total = (long long)g.N * g.K * g.OH * g.OW;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += step) {
    const int j = (int)(t % g.OW);
    const int i = (int)((t / g.OW) % g.OH);
    const int k = (int)((t / ((long long)g.OW * g.OH)) % g.K);
    const long long n = t / ((long long)g.OW * g.OH * g.K);
    float total_c = 0.0f;
    for (int c = 0; c < g.C; ++c) {
      float dot = 0.0f;
      const float *xc = x + ((n * g.C + c) * g.H) * (long long)g.W;
      const float *wk = w + ((long long)k * g.C + c) * g.R * g.S;
      for (int a = 0; a < g.R; ++a) {
        const int h = i * g.stride + a - g.pad;
        for (int b = 0; b < g.S; ++b) {
          const int q = j * g.stride + b - g.pad;
          const float xv = (h >= 0 && h < g.H && q >= 0 && q < g.W) ? __ldg(xc + (long long)h * g.W + q) : 0.0f;
          dot = __fadd_rn(dot, __fmul_rn(xv, __ldg(wk + a * g.S + b)));
        }
      }
      total_c = __fadd_rn(total_c, dot);
    }
    if (bias) total_c = __fadd_rn(total_c, __ldg(bias + k));
    y[t] = total_c;
  }
}

__global__ void __launch_bounds__(256) conv_dgrad_direct(const float *__restrict__ dy, const float *__restrict__ w,
                                                         float *__restrict__ dx, ConvGeom g) {
  const long long total = (long long)g.N * g.C * g.H * g.W;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += step) {
    const int q = (int)(t % g.W);
    const int h = (int)((t / g.W) % g.H);
    const int c = (int)((t / ((long long)g.W * g.H)) % g.C);
    const long long n = t / ((long long)g.W * g.H * g.C);
    double acc = 0.0;
    for (int k = 0; k < g.K; ++k)
      for (int a = 0; a < g.R; ++a) {
        const int ti = h + g.pad - a;
        if (ti < 0 || ti % g.stride) continue;
        const int i = ti / g.stride;
        if (i >= g.OH) continue;
        for (int b = 0; b < g.S; ++b) {
          const int tj = q + g.pad - b;
          if (tj < 0 || tj % g.stride) continue;
          const int j = tj / g.stride;
          if (j >= g.OW) continue;
          acc += (double)__ldg(dy + ((n * g.K + k) * g.OH + i) * (long long)g.OW + j) *
                 (double)__ldg(w + (((long long)k * g.C + c) * g.R + a) * g.S + b);
        }
      }
    dx[t] = (float)acc;
  }
}

// One block per weight element; the block reduces over all (n, i, j) in f64
// in a fixed order (deterministic).
__global__ void __launch_bounds__(256) conv_wgrad_direct(const float *__restrict__ x, const float *__restrict__ dy,
                                                         float *__restrict__ dw, ConvGeom g) {
  __shared__ double sh[256];
  const int widx = blockIdx.x;
  const int b = widx % g.S, a = (widx / g.S) % g.R, c = (widx / (g.S * g.R)) % g.C, k = widx / (g.S * g.R * g.C);
  const long long per_img = (long long)g.OH * g.OW;
  const long long total = (long long)g.N * per_img;
  double acc = 0.0;
  for (long long t = threadIdx.x; t < total; t += blockDim.x) {
    const long long n = t / per_img;
    const int i = (int)((t % per_img) / g.OW), j = (int)(t % g.OW);
    const int h = i * g.stride + a - g.pad, q = j * g.stride + b - g.pad;
    if (h < 0 || h >= g.H || q < 0 || q >= g.W) continue;
    acc += (double)__ldg(dy + ((n * g.K + k) * g.OH + i) * (long long)g.OW + j) *
           (double)__ldg(x + ((n * g.C + c) * g.H + h) * (long long)g.W + q);
  }
  sh[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if (threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) dw[widx] = (float)sh[0];
}

// Weight (and optionally bias) gradient of a 3x3 / pad 1 / stride 1 conv.
// Work items are bands of RB output rows of one image; a block stages the
// band's dy rows and the RB+2 input rows (zero-padded border columns) in
// shared memory.  Thread (kp, c) owns dw[2kp..2kp+1][c][0..2][0..2]: it walks
// the band row by row with a 3x3 window of inputs in registers (one new
// column of three inputs and two dy values per pixel for 18 FMAs).  Each
// block keeps its sums in registers over all its items and writes one f32
// partial per weight; a second kernel adds the partials in block order in
// f64 (deterministic).
template <int RB, int W>
__global__ void __launch_bounds__(512) conv_wgrad3x3_tiled(const float *__restrict__ x, const float *__restrict__ dy,
                                                           float *__restrict__ part, ConvGeom g, int with_bias) {
  extern __shared__ float sm[];
  const int C = g.C, K = g.K;
  constexpr int XW = W + 2;
  const int xplane = (RB + 2) * XW + 1;  // odd stride: conflict-free across c
  float *xs = sm;                        // [C][RB+2][W+2]
  float *ds = sm + C * xplane;           // [K][RB][W]
  const int kp = threadIdx.x / C, c = threadIdx.x % C;
  const int bands = (g.H + RB - 1) / RB;
  const long long items = (long long)g.N * bands;
  float acc0[9], acc1[9], bsum0 = 0.f, bsum1 = 0.f;
#pragma unroll
  for (int u = 0; u < 9; ++u) acc0[u] = acc1[u] = 0.f;
  for (long long it = blockIdx.x; it < items; it += gridDim.x) {
    const int n = (int)(it / bands), band = (int)(it % bands), r0 = band * RB;
    __syncthreads();
    for (int e = threadIdx.x; e < C * (RB + 2) * XW; e += blockDim.x) {
      const int cc = e / ((RB + 2) * XW), rem = e % ((RB + 2) * XW), rr = rem / XW, col = rem % XW;
      const int h = r0 + rr - 1, q = col - 1;
      xs[cc * xplane + rr * XW + col] =
          (h >= 0 && h < g.H && q >= 0 && q < W) ? __ldg(x + (((long long)n * C + cc) * g.H + h) * W + q) : 0.f;
    }
    for (int e = threadIdx.x; e < K * RB * W; e += blockDim.x) {
      const int k = e / (RB * W), rem = e % (RB * W), rr = rem / W, col = rem % W;
      const int h = r0 + rr;
      ds[e] = h < g.H ? __ldg(dy + (((long long)n * K + k) * g.H + h) * W + col) : 0.f;
    }
    __syncthreads();
    const float *xc = xs + c * xplane;
    const float *d0p = ds + (2 * kp) * RB * W, *d1p = d0p + RB * W;
    for (int i = 0; i < RB; ++i) {
      float w0[3], w1[3];
#pragma unroll
      for (int r = 0; r < 3; ++r) {
        w0[r] = xc[(i + r) * XW];
        w1[r] = xc[(i + r) * XW + 1];
      }
#pragma unroll 4
      for (int j = 0; j < W; ++j) {
        float w2[3];
#pragma unroll
        for (int r = 0; r < 3; ++r) w2[r] = xc[(i + r) * XW + j + 2];
        const float d0 = d0p[i * W + j], d1 = d1p[i * W + j];
#pragma unroll
        for (int r = 0; r < 3; ++r) {
          acc0[r * 3 + 0] = fmaf(d0, w0[r], acc0[r * 3 + 0]);
          acc0[r * 3 + 1] = fmaf(d0, w1[r], acc0[r * 3 + 1]);
          acc0[r * 3 + 2] = fmaf(d0, w2[r], acc0[r * 3 + 2]);
          acc1[r * 3 + 0] = fmaf(d1, w0[r], acc1[r * 3 + 0]);
          acc1[r * 3 + 1] = fmaf(d1, w1[r], acc1[r * 3 + 1]);
          acc1[r * 3 + 2] = fmaf(d1, w2[r], acc1[r * 3 + 2]);
          w0[r] = w1[r];
          w1[r] = w2[r];
        }
        bsum0 += d0;
        bsum1 += d1;
      }
    }
  }
  float *pb = part + (long long)blockIdx.x * (K * C * 9 + K);
#pragma unroll
  for (int u = 0; u < 9; ++u) {
    pb[((2 * kp) * C + c) * 9 + u] = acc0[u];
    pb[((2 * kp + 1) * C + c) * 9 + u] = acc1[u];
  }
  if (with_bias && c == 0) {
    pb[K * C * 9 + 2 * kp] = bsum0;
    pb[K * C * 9 + 2 * kp + 1] = bsum1;
  }
}

__global__ void wgrad_finish(const float *__restrict__ part, int nblocks, int stride, int nw, int nb,
                             float *__restrict__ dw, float *__restrict__ db) {
  const int e = blockIdx.x * blockDim.x + threadIdx.x;
  if (e >= nw + nb) return;
  double s = 0.0;
  for (int b = 0; b < nblocks; ++b) s += (double)part[(long long)b * stride + e];
  if (e < nw) dw[e] = (float)s;
  else db[e - nw] = (float)s;
}

// Bias gradient db[k] = sum over n and pixels of dy[n,k,:,:]; one block per
// channel, f64, fixed order.
__global__ void __launch_bounds__(256) bias_grad_direct(const float *__restrict__ dy, float *__restrict__ db,
                                                        int N, int K, long long pix) {
  __shared__ double sh[256];
  const int k = blockIdx.x;
  double acc = 0.0;
  for (long long t = threadIdx.x; t < (long long)N * pix; t += blockDim.x) {
    const long long n = t / pix, p = t % pix;
    acc += (double)dy[(n * K + k) * pix + p];
  }
  sh[threadIdx.x] = acc;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) db[k] = (float)sh[0];
}

int grid_for(long long n, int sm_count) {
  return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sm_count * 32));
}

}  // namespace

// dw (and db when non-null) of a 3x3 / pad 1 / stride 1 conv with the
// register-tiled kernel; *handled = false for shapes it does not take.
int conv_wgrad3x3(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dy, float *dw, float *db,
                  cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!(g.R == 3 && g.S == 3 && g.pad == 1 && g.stride == 1 && g.K % 2 == 0)) return REMORA_OK;
  const int threads = (g.K / 2) * g.C;
  if (threads > 512 || threads % 32) return REMORA_OK;
  constexpr int RB = 4;
  int W = g.W;
  if (W != 32 && W != 64) return REMORA_OK;
  const size_t smem = ((size_t)g.C * ((RB + 2) * (W + 2) + 1) + (size_t)g.K * RB * W) * sizeof(float);
  if (smem > 200 * 1024) return REMORA_OK;
  const int blocks = std::max(1, std::min<int>(ctx->sm_count * 2, g.N * ((g.H + RB - 1) / RB)));
  const int nw = g.K * g.C * 9, nb = g.K;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, (size_t)blocks * (nw + nb) * sizeof(float) + 256, &ws));
  float *part = reinterpret_cast<float *>(ws->buf);
  if (W == 64) {
    REMORA_CUDA_TRY(cudaFuncSetAttribute(conv_wgrad3x3_tiled<RB, 64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
    note_launch();
    conv_wgrad3x3_tiled<RB, 64><<<blocks, threads, smem, stream>>>(x, dy, part, g, db != nullptr);
  } else {
    REMORA_CUDA_TRY(cudaFuncSetAttribute(conv_wgrad3x3_tiled<RB, 32>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)smem));
    note_launch();
    conv_wgrad3x3_tiled<RB, 32><<<blocks, threads, smem, stream>>>(x, dy, part, g, db != nullptr);
  }
  note_launch();
  wgrad_finish<<<(nw + nb + 255) / 256, 256, 0, stream>>>(part, blocks, nw + nb, nw, db ? nb : 0, dw, db);
  REMORA_CUDA_TRY(cudaGetLastError());
  *handled = true;
  return REMORA_OK;
}

namespace {

int read_conv(const RemoraConvSpec *spec, const RemoraMemRef4 *xin, const RemoraMemRef4 *w, const RemoraMemRef4 *yout,
              bool x_is_input, DescView *X, DescView *Wd, DescView *Y, ConvGeom *g) {
  if (spec == nullptr) return fail(REMORA_ERR_ARG, "conv: null spec");
  if (spec->stride < 1 || spec->pad < 0) return fail(REMORA_ERR_ARG, "conv: stride %d pad %d", spec->stride, spec->pad);
  if (spec->precision != REMORA_PREC_TF32 && spec->precision != REMORA_PREC_3XTF32 &&
      spec->precision != REMORA_PREC_2XTF32)
    return fail(REMORA_ERR_ARG, "conv: unknown precision %d", spec->precision);
  REMORA_TRY(read_desc(xin, 4, X, x_is_input ? "conv input" : "conv output gradient"));
  REMORA_TRY(read_desc(w, 4, Wd, "conv weights"));
  REMORA_TRY(read_desc(yout, 4, Y, "conv result"));
  for (const DescView *d : {X, Wd, Y})
    if (!d->contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "conv: operands must be contiguous NCHW / KCRS");
  g->stride = spec->stride;
  g->pad = spec->pad;
  g->K = (int)Wd->sizes[0];
  g->C = (int)Wd->sizes[1];
  g->R = (int)Wd->sizes[2];
  g->S = (int)Wd->sizes[3];
  return REMORA_OK;
}

int finish_geom(ConvGeom *g) {
  if (g->H + 2 * g->pad < g->R || g->W + 2 * g->pad < g->S)
    return fail(REMORA_ERR_SHAPE, "conv: kernel %dx%d larger than the padded %dx%d image", g->R, g->S, g->H, g->W);
  g->OH = (g->H + 2 * g->pad - g->R) / g->stride + 1;
  g->OW = (g->W + 2 * g->pad - g->S) / g->stride + 1;
  return REMORA_OK;
}

}  // namespace
}  // namespace remora

using namespace remora;

extern "C" {

int remora_b200_conv2d_fwd(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                           const RemoraMemRef4 *w, const RemoraMemRef1 *bias, RemoraMemRef4 *y,
                           remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, Wd, Y, B;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, x, w, y, true, &X, &Wd, &Y, &g));
  g.N = (int)X.sizes[0];
  g.H = (int)X.sizes[2];
  g.W = (int)X.sizes[3];
  if (X.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv: input has %lld channels, weights %d", X.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (Y.sizes[0] != g.N || Y.sizes[1] != g.K || Y.sizes[2] != g.OH || Y.sizes[3] != g.OW)
    return fail(REMORA_ERR_SHAPE, "conv: output must be [%d, %d, %d, %d]", g.N, g.K, g.OH, g.OW);
  const float *bp = nullptr;
  if (bias) {
    REMORA_TRY(read_desc(bias, 1, &B, "conv bias"));
    if (B.sizes[0] != g.K || (B.strides[0] != 1 && g.K > 1))
      return fail(REMORA_ERR_SHAPE, "conv: bias must be a contiguous [%d]", g.K);
    bp = (const float *)B.data(4);
  }
  if (Y.numel() == 0) return REMORA_OK;
  bool handled = false;
  REMORA_TRY(conv_tc_fwd(ctx, g, (const float *)X.data(4), (const float *)Wd.data(4), bp, (float *)Y.data(4),
                         spec->precision, (cudaStream_t)stream, &handled));
  if (handled) return REMORA_OK;
  note_launch();
  conv_fwd_direct<<<grid_for(Y.numel(), ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)X.data(4), (const float *)Wd.data(4), bp, (float *)Y.data(4), g);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_conv2d_dgrad(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *dy,
                             const RemoraMemRef4 *w, RemoraMemRef4 *dx, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView DY, Wd, DX;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, dy, w, dx, false, &DY, &Wd, &DX, &g));
  g.N = (int)DX.sizes[0];
  g.H = (int)DX.sizes[2];
  g.W = (int)DX.sizes[3];
  if (DX.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv dgrad: dx has %lld channels, weights %d", DX.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (DY.sizes[0] != g.N || DY.sizes[1] != g.K || DY.sizes[2] != g.OH || DY.sizes[3] != g.OW)
    return fail(REMORA_ERR_SHAPE, "conv dgrad: dy must be [%d, %d, %d, %d]", g.N, g.K, g.OH, g.OW);
  if (DX.numel() == 0) return REMORA_OK;
  bool handled = false;
  REMORA_TRY(conv_tc_dgrad(ctx, g, (const float *)DY.data(4), (const float *)Wd.data(4), (float *)DX.data(4),
                           spec->precision, (cudaStream_t)stream, &handled));
  if (handled) return REMORA_OK;
  note_launch();
  conv_dgrad_direct<<<grid_for(DX.numel(), ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)DY.data(4), (const float *)Wd.data(4), (float *)DX.data(4), g);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_conv2d_wgrad(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                             const RemoraMemRef4 *dy, RemoraMemRef4 *dw, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, DY, DW;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, x, dw, dy, true, &X, &DW, &DY, &g));
  g.N = (int)X.sizes[0];
  g.H = (int)X.sizes[2];
  g.W = (int)X.sizes[3];
  if (X.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv wgrad: x has %lld channels, dw %d", X.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (DY.sizes[0] != g.N || DY.sizes[1] != g.K || DY.sizes[2] != g.OH || DY.sizes[3] != g.OW)
    return fail(REMORA_ERR_SHAPE, "conv wgrad: dy must be [%d, %d, %d, %d]", g.N, g.K, g.OH, g.OW);
  if (DW.numel() == 0) return REMORA_OK;
  bool handled = false;
  REMORA_TRY(conv_tc_wgrad_bias(ctx, g, (const float *)X.data(4), (const float *)DY.data(4), (float *)DW.data(4),
                                nullptr, spec->precision, (cudaStream_t)stream, &handled));
  if (handled) return REMORA_OK;
  REMORA_TRY(conv_wgrad3x3(ctx, g, (const float *)X.data(4), (const float *)DY.data(4), (float *)DW.data(4), nullptr,
                           (cudaStream_t)stream, &handled));
  if (handled) return REMORA_OK;
  note_launch();
  conv_wgrad_direct<<<(unsigned)DW.numel(), 256, 0, (cudaStream_t)stream>>>(
      (const float *)X.data(4), (const float *)DY.data(4), (float *)DW.data(4), g);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_conv2d_wgrad_bias(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                                  const RemoraMemRef4 *dy, RemoraMemRef4 *dw, RemoraMemRef1 *db,
                                  remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, DY, DW, DB;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, x, dw, dy, true, &X, &DW, &DY, &g));
  REMORA_TRY(read_desc(db, 1, &DB, "conv bias gradient"));
  g.N = (int)X.sizes[0];
  g.H = (int)X.sizes[2];
  g.W = (int)X.sizes[3];
  if (X.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv wgrad: x has %lld channels, dw %d", X.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (DY.sizes[0] != g.N || DY.sizes[1] != g.K || DY.sizes[2] != g.OH || DY.sizes[3] != g.OW)
    return fail(REMORA_ERR_SHAPE, "conv wgrad: dy must be [%d, %d, %d, %d]", g.N, g.K, g.OH, g.OW);
  if (DB.sizes[0] != g.K || (DB.strides[0] != 1 && g.K > 1))
    return fail(REMORA_ERR_SHAPE, "conv wgrad: db must be a contiguous [%d]", g.K);
  bool handled = false;
  REMORA_TRY(conv_tc_wgrad_bias(ctx, g, (const float *)X.data(4), (const float *)DY.data(4), (float *)DW.data(4),
                                (float *)DB.data(4), spec->precision, (cudaStream_t)stream, &handled));
  if (handled) return REMORA_OK;
  REMORA_TRY(conv_wgrad3x3(ctx, g, (const float *)X.data(4), (const float *)DY.data(4), (float *)DW.data(4),
                           (float *)DB.data(4), (cudaStream_t)stream, &handled));
  if (handled) return REMORA_OK;
  note_launch();
  conv_wgrad_direct<<<(unsigned)DW.numel(), 256, 0, (cudaStream_t)stream>>>(
      (const float *)X.data(4), (const float *)DY.data(4), (float *)DW.data(4), g);
  note_launch();
  bias_grad_direct<<<g.K, 256, 0, (cudaStream_t)stream>>>((const float *)DY.data(4), (float *)DB.data(4), g.N, g.K,
                                                          (long long)g.OH * g.OW);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

// ---- fused conv + ReLU + 2x2 max-pool (the crater CNN's second layer) ----

namespace {
// Pooled tensor [N, C, H/2, W/2] (values) or its codes (bytes) for an
// activation of [N, C, H, W].
int read_pooled(const void *desc, int N, int C, int H, int W, DescView *out, const char *what) {
  REMORA_TRY(read_desc(desc, 4, out, what));
  if (!out->contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "%s must be contiguous", what);
  if (out->sizes[0] != N || out->sizes[1] != C || out->sizes[2] != H / 2 || out->sizes[3] != W / 2)
    return fail(REMORA_ERR_SHAPE, "%s must be [%d, %d, %d, %d]", what, N, C, H / 2, W / 2);
  return REMORA_OK;
}
}  // namespace

int remora_b200_conv2d_fwd_relu_pool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                                     const RemoraMemRef4 *w, const RemoraMemRef1 *bias, RemoraMemRef4 *pooled,
                                     RemoraMemRef4 *code, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, Wd, P, Cd, B;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, x, w, pooled, true, &X, &Wd, &P, &g));
  g.N = (int)X.sizes[0];
  g.H = (int)X.sizes[2];
  g.W = (int)X.sizes[3];
  if (X.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv: input has %lld channels, weights %d", X.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (g.OH != g.H || g.OW != g.W || (g.H | g.W) & 1)
    return fail(REMORA_ERR_SHAPE, "conv_relu_pool: needs a same-size conv on an even-sized image");
  REMORA_TRY(read_pooled(pooled, g.N, g.K, g.H, g.W, &P, "pooled output"));
  REMORA_TRY(read_pooled(code, g.N, g.K, g.H, g.W, &Cd, "pool codes"));
  REMORA_TRY(read_desc(bias, 1, &B, "conv bias"));
  if (B.sizes[0] != g.K || (B.strides[0] != 1 && g.K > 1))
    return fail(REMORA_ERR_SHAPE, "conv: bias must be a contiguous [%d]", g.K);
  if (P.numel() == 0) return REMORA_OK;
  bool handled = false;
  REMORA_TRY(conv_tc_fwd_relu_pool(ctx, g, (const float *)X.data(4), (const float *)Wd.data(4),
                                   (const float *)B.data(4), (float *)P.data(4), (uint8_t *)Cd.data(1),
                                   spec->precision, (cudaStream_t)stream, &handled));
  if (!handled)
    return fail(REMORA_ERR_UNSUPPORTED,
                "conv_relu_pool: only the tensor-core shape 3x3 / pad 1, 16 -> 17..32 channels, width 32");
  return REMORA_OK;
}

int remora_b200_conv2d_dgrad_unpool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *dpooled,
                                    const RemoraMemRef4 *code, const RemoraMemRef4 *w, RemoraMemRef4 *dx,
                                    remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView DP, Cd, Wd, DX;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, dpooled, w, dx, false, &DP, &Wd, &DX, &g));
  g.N = (int)DX.sizes[0];
  g.H = (int)DX.sizes[2];
  g.W = (int)DX.sizes[3];
  if (DX.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv dgrad: dx has %lld channels, weights %d", DX.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (g.OH != g.H || g.OW != g.W || (g.H | g.W) & 1)
    return fail(REMORA_ERR_SHAPE, "conv_dgrad_unpool: needs a same-size conv on an even-sized image");
  REMORA_TRY(read_pooled(dpooled, g.N, g.K, g.H, g.W, &DP, "pooled gradient"));
  REMORA_TRY(read_pooled(code, g.N, g.K, g.H, g.W, &Cd, "pool codes"));
  if (DX.numel() == 0) return REMORA_OK;
  bool handled = false;
  REMORA_TRY(conv_tc_dgrad_unpool(ctx, g, (const float *)DP.data(4), (const uint8_t *)Cd.data(1),
                                  (const float *)Wd.data(4), (float *)DX.data(4), spec->precision,
                                  (cudaStream_t)stream, &handled));
  if (!handled)
    return fail(REMORA_ERR_UNSUPPORTED,
                "conv_dgrad_unpool: only the tensor-core shape 3x3 / pad 1, 32 -> 16 channels, width 32");
  return REMORA_OK;
}

int remora_b200_conv2d_wgrad_bias_unpool(RemoraB200Ctx *ctx, const RemoraConvSpec *spec, const RemoraMemRef4 *x,
                                         const RemoraMemRef4 *dpooled, const RemoraMemRef4 *code,
                                         RemoraMemRef4 *dw, RemoraMemRef1 *db, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, DP, Cd, DW, DB;
  ConvGeom g{};
  REMORA_TRY(read_conv(spec, x, dw, dpooled, true, &X, &DW, &DP, &g));
  REMORA_TRY(read_desc(db, 1, &DB, "conv bias gradient"));
  g.N = (int)X.sizes[0];
  g.H = (int)X.sizes[2];
  g.W = (int)X.sizes[3];
  if (X.sizes[1] != g.C) return fail(REMORA_ERR_SHAPE, "conv wgrad: x has %lld channels, dw %d", X.sizes[1], g.C);
  REMORA_TRY(finish_geom(&g));
  if (g.OH != g.H || g.OW != g.W || (g.H | g.W) & 1)
    return fail(REMORA_ERR_SHAPE, "conv_wgrad_unpool: needs a same-size conv on an even-sized image");
  REMORA_TRY(read_pooled(dpooled, g.N, g.K, g.H, g.W, &DP, "pooled gradient"));
  REMORA_TRY(read_pooled(code, g.N, g.K, g.H, g.W, &Cd, "pool codes"));
  if (DB.sizes[0] != g.K || (DB.strides[0] != 1 && g.K > 1))
    return fail(REMORA_ERR_SHAPE, "conv wgrad: db must be a contiguous [%d]", g.K);
  bool handled = false;
  REMORA_TRY(conv_tc_wgrad_bias_unpool(ctx, g, (const float *)X.data(4), (const float *)DP.data(4),
                                       (const uint8_t *)Cd.data(1), (float *)DW.data(4), (float *)DB.data(4),
                                       spec->precision, (cudaStream_t)stream, &handled));
  if (!handled)
    return fail(REMORA_ERR_UNSUPPORTED,
                "conv_wgrad_unpool: only the tensor-core shape 3x3 / pad 1, 16 input channels, width 32");
  return REMORA_OK;
}

}  // extern "C"
