// cnn.cu — fused kernels of the crater-CNN training step.
//
// The model (conv3x3 1->16 + ReLU, 2x2 max-pool, conv3x3 16->32 + ReLU,
// 2x2 max-pool, dense 8192->64 + ReLU, dense 64->1, sigmoid BCE, SGD) is built
// from the reference's formulas: ReLU as select(v > 0, v, 0) and the stable
// BCE (examples/crater_train.py:46-54), the update p - lr * g
// (examples/crater_train.py:249-253), and the VJPs of remora/ad.py:85-179
// (select routes the adjoint to the taken branch, fold broadcasts it, mul
// multiplies by the other operand).  Max-pool, batch-mean BCE and
// multi-channel convolution have no reference counterpart.
//
// ReLU and max-pool commute (max of ReLUs = ReLU of the max), so every
// pooled output keeps one byte: the index (0..3, window order (0,0) (0,1)
// (1,0) (1,1), first maximum wins) of the element that receives its
// gradient, or 255 when the maximum is not positive and no gradient flows.
// The conv1 activation (B x 16 x 64 x 64) is never written to HBM: the
// forward kernel pools it at once and the weight gradient of conv1 is
// accumulated straight from the pooled gradient.
#include <algorithm>

#include "../../include/remora_b200_cnn.h"
#include "common.cuh"

namespace remora {

namespace {

constexpr uint8_t kNoGrad = 255;

__device__ __forceinline__ void pool4(float v0, float v1, float v2, float v3, float *out, uint8_t *code) {
  float m = v0;
  int idx = 0;
  if (v1 > m) m = v1, idx = 1;
  if (v2 > m) m = v2, idx = 2;
  if (v3 > m) m = v3, idx = 3;
  *out = m > 0.0f ? m : 0.0f;
  *code = m > 0.0f ? (uint8_t)idx : kNoGrad;
}

// conv3x3 (1 input channel, pad 1) + bias + ReLU + 2x2 max-pool.  One block
// per image: the image goes to shared memory once with a zero border, each
// thread takes four pooled positions, keeps their 4x4 input patches in
// registers and runs all K channels over them (weights broadcast from shared
// memory).  Each conv output is the oracle's dot over taps in order (f32 ops
// rounded one by one), then + bias; for one channel the lanes of a warp
// write consecutive pooled pixels.
constexpr int kConv1Threads = 256;
constexpr int kConv1MaxK = 32;

// Stage the padded input rows 2*i0-1 .. 2*i0+IR-2 of one H x W image in
// shared memory (row stride W + 2, zero outside the image).  With `vec` (the
// image starts on a 16-byte boundary) each thread issues all of its 16-byte
// reads before its first shared-memory write, so a block waits for one
// memory latency rather than one per row chunk.
template <int H, int W, int IR>
__device__ __forceinline__ void stage_rows(const float *__restrict__ xb, int i0, float *img, bool vec) {
  constexpr int PWD = W + 2, V4 = W / 4, NV = IR * V4;
  constexpr int LPT = (NV + kConv1Threads - 1) / kConv1Threads;
  static_assert(W % 4 == 0, "rows of whole 16-byte vectors");
  if (vec) {
    float4 v[LPT];
#pragma unroll
    for (int j = 0; j < LPT; ++j) {
      const int e = threadIdx.x + j * kConv1Threads, r = 2 * i0 + e / V4 - 1;
      v[j] = (e < NV && r >= 0 && r < H) ? __ldg(reinterpret_cast<const float4 *>(xb + r * W) + e % V4)
                                         : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    }
#pragma unroll
    for (int j = 0; j < LPT; ++j) {
      const int e = threadIdx.x + j * kConv1Threads;
      if (e < NV) {
        float *d = img + (e / V4) * PWD + 1 + 4 * (e % V4);
        d[0] = v[j].x;
        d[1] = v[j].y;
        d[2] = v[j].z;
        d[3] = v[j].w;
      }
    }
    for (int e = threadIdx.x; e < 2 * IR; e += kConv1Threads) img[(e >> 1) * PWD + (e & 1) * (W + 1)] = 0.0f;
  } else {
    for (int e = threadIdx.x; e < IR * PWD; e += kConv1Threads) {
      const int r = 2 * i0 + e / PWD - 1, c = e % PWD - 1;
      img[e] = (r >= 0 && r < H && c >= 0 && c < W) ? __ldg(xb + r * W + c) : 0.0f;
    }
  }
}

template <int H, int W, int PARTS>
__global__ void __launch_bounds__(kConv1Threads) conv1_relu_pool_kernel(const float *__restrict__ x,
                                                                        const float *__restrict__ w,
                                                                        const float *__restrict__ bias,
                                                                        float *__restrict__ p,
                                                                        uint8_t *__restrict__ code, int K,
                                                                        bool vec) {
  // PARTS blocks share an image, each taking RP consecutive pooled rows (and
  // the 2 * RP + 2 padded input rows they read), so that small batches
  // still fill the GPU; every output is computed the same way for any PARTS.
  constexpr int OH = H / 2, OW = W / 2, NP = OH * OW, PWD = W + 2;
  constexpr int RP = OH / PARTS, NPP = RP * OW, IR = 2 * RP + 2;
  constexpr int PER = (NPP + kConv1Threads - 1) / kConv1Threads;
  static_assert(OH % PARTS == 0, "parts split the pooled rows evenly");
  __shared__ float img[IR * PWD];
  __shared__ float ws[kConv1MaxK * 10];
  const long long b = blockIdx.x / PARTS;
  const int i0 = (blockIdx.x % PARTS) * RP;  // first pooled row of this block
  stage_rows<H, W, IR>(x + b * (long long)H * W, i0, img, vec);
  for (int e = threadIdx.x; e < K * 10; e += kConv1Threads)
    ws[e] = (e % 10) < 9 ? __ldg(w + (e / 10) * 9 + e % 10) : __ldg(bias + e / 10);
  __syncthreads();
  float patch[PER][4][4];
#pragma unroll
  for (int u = 0; u < PER; ++u) {
    const int pos = threadIdx.x + u * kConv1Threads;
    const int i = pos / OW, j = pos % OW;
#pragma unroll
    for (int a = 0; a < 4; ++a)
#pragma unroll
      for (int c = 0; c < 4; ++c) patch[u][a][c] = pos < NPP ? img[(2 * i + a) * PWD + 2 * j + c] : 0.0f;
  }
  float *pb = p + b * (long long)K * NP + i0 * OW;
  uint8_t *cb = code + b * (long long)K * NP + i0 * OW;
#pragma unroll 1
  for (int k = 0; k < K; ++k) {
    float wk[9];
#pragma unroll
    for (int t = 0; t < 9; ++t) wk[t] = ws[k * 10 + t];
    const float bk = ws[k * 10 + 9];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int pos = threadIdx.x + u * kConv1Threads;
      float v[4];
#pragma unroll
      for (int di = 0; di < 2; ++di)
#pragma unroll
        for (int dj = 0; dj < 2; ++dj) {
          // 0 + p0*w0 only differs from p0*w0 by the sign of a zero, which no
          // later sum keeps once 0 + dot is taken: the first add is skipped.
          float dot = __fmul_rn(patch[u][di][dj], wk[0]);
#pragma unroll
          for (int t = 1; t < 9; ++t)
            dot = __fadd_rn(dot, __fmul_rn(patch[u][di + t / 3][dj + t % 3], wk[t]));
          v[di * 2 + dj] = __fadd_rn(__fadd_rn(0.0f, dot), bk);
        }
      if (pos < NPP) pool4(v[0], v[1], v[2], v[3], pb + (long long)k * NP + pos, cb + (long long)k * NP + pos);
    }
  }
}

// ReLU + 2x2 max-pool of an NCHW tensor (the conv2 activation, bias added).
__global__ void __launch_bounds__(256) relu_pool_kernel(const float *__restrict__ a, float *__restrict__ p,
                                                        uint8_t *__restrict__ code, long long planes, int H, int W) {
  const int OH = H / 2, OW = W / 2;
  const long long total = planes * OH * OW;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += step) {
    const int j = (int)(t % OW), i = (int)((t / OW) % OH);
    const long long pl = t / ((long long)OW * OH);
    const float *ap = a + (pl * H + 2 * i) * W + 2 * j;
    const float2 r0 = *reinterpret_cast<const float2 *>(ap);
    const float2 r1 = *reinterpret_cast<const float2 *>(ap + W);
    pool4(r0.x, r0.y, r1.x, r1.y, p + t, code + t);
  }
}

// Adjoint of ReLU + max-pool: the pooled gradient goes to the recorded
// element, every other element of the window gets 0.
__global__ void __launch_bounds__(256) unpool_kernel(const float *__restrict__ dp, const uint8_t *__restrict__ code,
                                                     float *__restrict__ da, long long planes, int H, int W) {
  const int OH = H / 2, OW = W / 2;
  const long long total = planes * OH * OW;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long t = (long long)blockIdx.x * blockDim.x + threadIdx.x; t < total; t += step) {
    const int j = (int)(t % OW), i = (int)((t / OW) % OH);
    const long long pl = t / ((long long)OW * OH);
    const uint8_t c = code[t];
    const float g = dp[t];
    float2 r0 = make_float2(0.f, 0.f), r1 = make_float2(0.f, 0.f);
    if (c == 0) r0.x = g;
    else if (c == 1) r0.y = g;
    else if (c == 2) r1.x = g;
    else if (c == 3) r1.y = g;
    float *ap = da + (pl * H + 2 * i) * W + 2 * j;
    *reinterpret_cast<float2 *>(ap) = r0;
    *reinterpret_cast<float2 *>(ap + W) = r1;
  }
}

// Dense 64 -> 1 on the ReLU'd hidden layer, the stable BCE and its gradient.
// One warp per sample.  loss[b] = bce(z, y); dz[b] = (sigmoid(z) - y) * inv.
// With hb non-null, h is computed first from hpre: h = relu(hpre + hb),
// stored to h_out, and used in place of a stored hidden layer.
__global__ void __launch_bounds__(256) dense_bce_kernel(const float *__restrict__ h, const float *__restrict__ hb,
                                                        float *__restrict__ h_out, const float *__restrict__ w4,
                                                        const float *__restrict__ b4, const float *__restrict__ y,
                                                        float *__restrict__ z_out, float *__restrict__ loss,
                                                        float *__restrict__ dz, int B, int D, float inv) {
  const int lane = threadIdx.x & 31;
  const long long warp = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  for (long long b = warp; b < B; b += nwarps) {
    float acc = 0.0f;
    for (int o = lane; o < D; o += 32) {
      float hv = h[b * D + o];
      if (hb) {
        const float s = __fadd_rn(hv, __ldg(hb + o));
        hv = s > 0.0f ? s : 0.0f;
        h_out[b * D + o] = hv;
      }
      acc = __fadd_rn(acc, __fmul_rn(__ldg(w4 + o), hv));
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, s));
    if (lane == 0) {
      const float z = __fadd_rn(acc, __ldg(b4));
      const float yy = y[b];
      const float pos = z > 0.0f ? z : 0.0f;
      const float absz = z > 0.0f ? z : __fsub_rn(0.0f, z);
      const float l = __fadd_rn(pos, __fadd_rn(__fmul_rn(-1.0f, __fmul_rn(z, yy)),
                                               logf(__fadd_rn(1.0f, expf(__fsub_rn(0.0f, absz))))));
      float s;
      if (z > 0.0f) {
        s = __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-z)));
      } else {
        const float e = expf(z);
        s = __fdiv_rn(e, __fadd_rn(1.0f, e));
      }
      z_out[b] = z;
      loss[b] = l;
      dz[b] = __fmul_rn(__fsub_rn(s, yy), inv);
    }
  }
}

// Backward of dense 64 -> 1 and the hidden ReLU.  Block o: dw4[o] =
// sum_b dz[b] h[b,o] (fixed order), dh[b,o] = h[b,o] > 0 ? dz[b] w4[o] : 0,
// and (when dsum is non-null) dsum[o] = sum_b dh[b,o], the gradient of the
// hidden layer's bias; block D (one extra) sums db4 = sum_b dz[b].  Sums in
// f64, combined in a fixed tree order.
__global__ void __launch_bounds__(256) dense_bwd_kernel(const float *__restrict__ h, const float *__restrict__ w4,
                                                        const float *__restrict__ dz, float *__restrict__ dh,
                                                        float *__restrict__ dw4, float *__restrict__ db4,
                                                        float *__restrict__ dsum, int B, int D) {
  __shared__ double sh[2][256];
  const int o = blockIdx.x;
  double acc = 0.0, acc2 = 0.0;
  if (o < D) {
    const float wo = __ldg(w4 + o);
    for (int b = threadIdx.x; b < B; b += blockDim.x) {
      const float hv = h[(long long)b * D + o];
      const float g = dz[b];
      acc += (double)g * (double)hv;
      const float d = hv > 0.0f ? __fmul_rn(g, wo) : 0.0f;
      dh[(long long)b * D + o] = d;
      acc2 += (double)d;
    }
  } else {
    for (int b = threadIdx.x; b < B; b += blockDim.x) acc += (double)dz[b];
  }
  sh[0][threadIdx.x] = acc;
  sh[1][threadIdx.x] = acc2;
  __syncthreads();
  for (int s = 128; s > 0; s >>= 1) {
    if ((int)threadIdx.x < s) {
      sh[0][threadIdx.x] += sh[0][threadIdx.x + s];
      sh[1][threadIdx.x] += sh[1][threadIdx.x + s];
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (o < D) {
      dw4[o] = (float)sh[0][0];
      if (dsum) dsum[o] = (float)sh[1][0];
    } else {
      *db4 = (float)sh[0][0];
    }
  }
}

// conv1 weight and bias gradients straight from the pooled gradient: each
// pooled output with a recorded element (h, q) contributes
// dp * x[h + a - 1, q + b - 1] to dw1[k][a][b] and dp to db1[k].  PARTS
// blocks per image, each over RP consecutive pooled rows (its input rows in
// shared memory with a zero border).  The 16 lanes of a half-warp share a
// channel k; lane l reads pooled positions 64 j + 4 l .. 64 j + 4 l + 3 as one
// 16-byte gradient vector and one 4-byte code word, four such groups in
// flight at a time.  A group of 16 positions is summed in f32 (fused
// multiply-adds), each group sum is added in f64, and the 16 lanes combine
// with a fixed shuffle tree into
// part[((b * PARTS + part) * K + k) * 10 + {0..8: taps, 9: bias}]: the weight
// gradient adds every pixel of the batch with heavy cancellation, and f32
// sums of whole rows lose about 1e-4 of the result.  The finish kernel adds
// the partials in (image, part) order in f64.
template <int H, int W, int PARTS>
__global__ void __launch_bounds__(kConv1Threads) conv1_wgrad_pool_kernel(const float *__restrict__ x,
                                                                         const float *__restrict__ dp,
                                                                         const uint8_t *__restrict__ code,
                                                                         double *__restrict__ part, int K,
                                                                         bool vec) {
  constexpr int OW = W / 2, NP = (H / 2) * OW, PWD = W + 2;
  constexpr int RP = (H / 2) / PARTS, NPP = RP * OW, IR = 2 * RP + 2;
  constexpr int GROUPS = NPP / 64;  // 4-position groups per lane and channel
  static_assert((H / 2) % PARTS == 0, "parts split the pooled rows evenly");
  static_assert(NPP % 256 == 0 && OW % 4 == 0, "whole batches of four groups, groups inside one row");
  __shared__ float img[IR * PWD];
  const long long b = blockIdx.x / PARTS;
  const int i0 = (blockIdx.x % PARTS) * RP;
  stage_rows<H, W, IR>(x + b * (long long)H * W, i0, img, vec);
  __syncthreads();
  const int lane16 = threadIdx.x & 15;
  for (int k = threadIdx.x >> 4; k < K; k += kConv1Threads / 16) {
    double acc[10];
#pragma unroll
    for (int u = 0; u < 10; ++u) acc[u] = 0.0;
    const long long base = (b * K + k) * (long long)NP + i0 * OW;
    const float *dpk = dp + base;
    const uint8_t *ck = code + base;
#pragma unroll 1
    for (int j0 = 0; j0 < GROUPS; j0 += 4) {
      float g[4][4];
      uint32_t cw[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int p0 = 64 * (j0 + j) + 4 * lane16;
        if (vec) {
          const float4 t = __ldg(reinterpret_cast<const float4 *>(dpk + p0));
          g[j][0] = t.x, g[j][1] = t.y, g[j][2] = t.z, g[j][3] = t.w;
          cw[j] = __ldg(reinterpret_cast<const unsigned int *>(ck + p0));
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) g[j][e] = __ldg(dpk + p0 + e);
          cw[j] = (uint32_t)ck[p0] | (uint32_t)ck[p0 + 1] << 8 | (uint32_t)ck[p0 + 2] << 16 |
                  (uint32_t)ck[p0 + 3] << 24;
        }
      }
      float sum[10];
#pragma unroll
      for (int u = 0; u < 10; ++u) sum[u] = 0.0f;
#pragma unroll
      for (int j = 0; j < 4; ++j)
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int pos = 64 * (j0 + j) + 4 * lane16 + e;
          const uint32_t c0 = (cw[j] >> (8 * e)) & 0xFFu;
          const float gv = c0 == kNoGrad ? 0.0f : g[j][e];
          const int c = (int)(c0 & 3u);  // window index; a no-gradient code still reads inside the border
          const float *ip = img + (2 * (pos / OW) + (c >> 1)) * PWD + 2 * (pos % OW) + (c & 1);
#pragma unroll
          for (int a = 0; a < 3; ++a)
#pragma unroll
            for (int bb = 0; bb < 3; ++bb) sum[a * 3 + bb] = fmaf(gv, ip[a * PWD + bb], sum[a * 3 + bb]);
          sum[9] += gv;
        }
#pragma unroll
      for (int u = 0; u < 10; ++u) acc[u] += (double)sum[u];
    }
#pragma unroll
    for (int u = 0; u < 10; ++u) {
      double v = acc[u];
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
      if (lane16 == 0) part[((long long)blockIdx.x * K + k) * 10 + u] = v;
    }
  }
}

// Blocks per image for the conv1 kernels: enough blocks for several waves
// on small batches, one block per image on large ones.
int conv1_parts(int B, int H) {
  if (H != 64) return 1;
  // 512 images (one rank of eight at a global batch of 4096): two blocks
  // per image measured faster than four (294 vs 300 us per step)
  return B <= 128 ? 4 : (B <= 2048 ? 2 : 1);
}

// dw1, db1 = sums of the n per-block partials, in block order, f64.  One
// block per output value.
__global__ void __launch_bounds__(256) conv1_wgrad_finish_kernel(const double *__restrict__ part,
                                                                 float *__restrict__ dw, float *__restrict__ db,
                                                                 int B, int K) {
  __shared__ double sh[256];
  const int k = blockIdx.x / 10, u = blockIdx.x % 10;
  double s = 0.0;
  for (int b = threadIdx.x; b < B; b += 256) s += part[((long long)b * K + k) * 10 + u];
  sh[threadIdx.x] = s;
  __syncthreads();
  for (int o = 128; o > 0; o >>= 1) {
    if ((int)threadIdx.x < o) sh[threadIdx.x] += sh[threadIdx.x + o];
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    if (u < 9) dw[k * 9 + u] = (float)sh[0];
    else db[k] = (float)sh[0];
  }
}

int grid_for(long long n, int sm_count) {
  return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sm_count * 32));
}

bool aligned(const void *p, uintptr_t bytes) { return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0; }

int need4(const void *desc, DescView *v, const char *what) {
  REMORA_TRY(read_desc(desc, 4, v, what));
  if (!v->contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "%s must be contiguous", what);
  return REMORA_OK;
}

}  // namespace

}  // namespace remora

using namespace remora;

extern "C" {

int remora_b200_conv1_relu_pool(RemoraB200Ctx *ctx, const RemoraMemRef4 *x, const RemoraMemRef4 *w,
                                const RemoraMemRef1 *bias, RemoraMemRef4 *pooled, RemoraMemRef4 *code,
                                remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, Wd, Bd, P, C;
  REMORA_TRY(need4(x, &X, "conv1 input"));
  REMORA_TRY(need4(w, &Wd, "conv1 weights"));
  REMORA_TRY(read_desc(bias, 1, &Bd, "conv1 bias"));
  REMORA_TRY(need4(pooled, &P, "pooled output"));
  REMORA_TRY(need4(code, &C, "pool codes"));
  const int B = (int)X.sizes[0], H = (int)X.sizes[2], W = (int)X.sizes[3], K = (int)Wd.sizes[0];
  if (X.sizes[1] != 1 || Wd.sizes[1] != 1 || Wd.sizes[2] != 3 || Wd.sizes[3] != 3 || (H | W) & 1)
    return fail(REMORA_ERR_SHAPE, "conv1_relu_pool: needs x [B,1,H,W] (H, W even) and w [K,1,3,3]");
  if (Bd.sizes[0] != K || P.sizes[0] != B || P.sizes[1] != K || P.sizes[2] != H / 2 || P.sizes[3] != W / 2)
    return fail(REMORA_ERR_SHAPE, "conv1_relu_pool: pooled output must be [B,K,H/2,W/2]");
  for (int d = 0; d < 4; ++d)
    if (C.sizes[d] != P.sizes[d]) return fail(REMORA_ERR_SHAPE, "conv1_relu_pool: codes must match pooled shape");
  if (P.numel() == 0) return REMORA_OK;
  if (!((H == 64 && W == 64) || (H == 32 && W == 32)) || K > kConv1MaxK)
    return fail(REMORA_ERR_UNSUPPORTED, "conv1_relu_pool: images of 64x64 or 32x32 and at most %d channels",
                kConv1MaxK);
  const int parts = conv1_parts(B, H);
  auto kern = H != 64      ? conv1_relu_pool_kernel<32, 32, 1>
              : parts == 4 ? conv1_relu_pool_kernel<64, 64, 4>
              : parts == 2 ? conv1_relu_pool_kernel<64, 64, 2>
                           : conv1_relu_pool_kernel<64, 64, 1>;
  note_launch();
  kern<<<B * parts, kConv1Threads, 0, (cudaStream_t)stream>>>((const float *)X.data(4), (const float *)Wd.data(4),
                                                      (const float *)Bd.data(4), (float *)P.data(4),
                                                      (uint8_t *)C.data(1), K, aligned(X.data(4), 16));
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_relu_pool(RemoraB200Ctx *ctx, const RemoraMemRef4 *a, RemoraMemRef4 *pooled, RemoraMemRef4 *code,
                          remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView A, P, C;
  REMORA_TRY(need4(a, &A, "relu_pool input"));
  REMORA_TRY(need4(pooled, &P, "relu_pool output"));
  REMORA_TRY(need4(code, &C, "relu_pool codes"));
  const int H = (int)A.sizes[2], W = (int)A.sizes[3];
  if ((H | W) & 1 || P.sizes[0] != A.sizes[0] || P.sizes[1] != A.sizes[1] || P.sizes[2] != H / 2 ||
      P.sizes[3] != W / 2)
    return fail(REMORA_ERR_SHAPE, "relu_pool: output must be [N,C,H/2,W/2] with H, W even");
  for (int d = 0; d < 4; ++d)
    if (C.sizes[d] != P.sizes[d]) return fail(REMORA_ERR_SHAPE, "relu_pool: codes must match pooled shape");
  if (P.numel() == 0) return REMORA_OK;
  note_launch();
  relu_pool_kernel<<<grid_for(P.numel(), ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)A.data(4), (float *)P.data(4), (uint8_t *)C.data(1), A.sizes[0] * A.sizes[1], H, W);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_unpool(RemoraB200Ctx *ctx, const RemoraMemRef4 *dpooled, const RemoraMemRef4 *code,
                       RemoraMemRef4 *da, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView P, C, A;
  REMORA_TRY(need4(dpooled, &P, "unpool gradient"));
  REMORA_TRY(need4(code, &C, "unpool codes"));
  REMORA_TRY(need4(da, &A, "unpool output"));
  const int H = (int)A.sizes[2], W = (int)A.sizes[3];
  if ((H | W) & 1 || P.sizes[0] != A.sizes[0] || P.sizes[1] != A.sizes[1] || P.sizes[2] != H / 2 ||
      P.sizes[3] != W / 2)
    return fail(REMORA_ERR_SHAPE, "unpool: gradient must be [N,C,H/2,W/2] of the [N,C,H,W] output");
  for (int d = 0; d < 4; ++d)
    if (C.sizes[d] != P.sizes[d]) return fail(REMORA_ERR_SHAPE, "unpool: codes must match the pooled shape");
  if (P.numel() == 0) return REMORA_OK;
  note_launch();
  unpool_kernel<<<grid_for(P.numel(), ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)P.data(4), (const uint8_t *)C.data(1), (float *)A.data(4), A.sizes[0] * A.sizes[1], H, W);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_dense_bce(RemoraB200Ctx *ctx, const RemoraMemRef2 *h, const RemoraMemRef1 *w, const RemoraMemRef1 *b,
                          const RemoraMemRef1 *y, RemoraMemRef1 *z, RemoraMemRef1 *loss, RemoraMemRef1 *dz,
                          float grad_scale, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView Hd, Wd, Bd, Y, Z, Lo, Dz;
  REMORA_TRY(read_desc(h, 2, &Hd, "hidden"));
  REMORA_TRY(read_desc(w, 1, &Wd, "dense weights"));
  REMORA_TRY(read_desc(b, 1, &Bd, "dense bias"));
  REMORA_TRY(read_desc(y, 1, &Y, "labels"));
  REMORA_TRY(read_desc(z, 1, &Z, "logits"));
  REMORA_TRY(read_desc(loss, 1, &Lo, "losses"));
  REMORA_TRY(read_desc(dz, 1, &Dz, "logit gradients"));
  for (const DescView *d : {&Hd, &Wd, &Bd, &Y, &Z, &Lo, &Dz})
    if (!d->contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "dense_bce: operands must be contiguous");
  const int B = (int)Hd.sizes[0], D = (int)Hd.sizes[1];
  if (Wd.sizes[0] != D || Bd.sizes[0] != 1 || Y.sizes[0] != B || Z.sizes[0] != B || Lo.sizes[0] != B ||
      Dz.sizes[0] != B)
    return fail(REMORA_ERR_SHAPE, "dense_bce: shapes must be h [B,D], w [D], b [1], y/z/loss/dz [B]");
  if (B == 0) return REMORA_OK;
  note_launch();
  dense_bce_kernel<<<grid_for((long long)B * 32, ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)Hd.data(4), nullptr, nullptr, (const float *)Wd.data(4), (const float *)Bd.data(4),
      (const float *)Y.data(4), (float *)Z.data(4), (float *)Lo.data(4), (float *)Dz.data(4), B, D, grad_scale);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_dense_bias_relu_bce(RemoraB200Ctx *ctx, const RemoraMemRef2 *hpre, const RemoraMemRef1 *hb,
                                    RemoraMemRef2 *h, const RemoraMemRef1 *w, const RemoraMemRef1 *b,
                                    const RemoraMemRef1 *y, RemoraMemRef1 *z, RemoraMemRef1 *loss, RemoraMemRef1 *dz,
                                    float grad_scale, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView Hp, Hb, Hd, Wd, Bd, Y, Z, Lo, Dz;
  REMORA_TRY(read_desc(hpre, 2, &Hp, "hidden pre-activation"));
  REMORA_TRY(read_desc(hb, 1, &Hb, "hidden bias"));
  REMORA_TRY(read_desc(h, 2, &Hd, "hidden"));
  REMORA_TRY(read_desc(w, 1, &Wd, "dense weights"));
  REMORA_TRY(read_desc(b, 1, &Bd, "dense bias"));
  REMORA_TRY(read_desc(y, 1, &Y, "labels"));
  REMORA_TRY(read_desc(z, 1, &Z, "logits"));
  REMORA_TRY(read_desc(loss, 1, &Lo, "losses"));
  REMORA_TRY(read_desc(dz, 1, &Dz, "logit gradients"));
  for (const DescView *d : {&Hp, &Hb, &Hd, &Wd, &Bd, &Y, &Z, &Lo, &Dz})
    if (!d->contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "dense_bias_relu_bce: operands must be contiguous");
  const int B = (int)Hp.sizes[0], D = (int)Hp.sizes[1];
  if (Hd.sizes[0] != B || Hd.sizes[1] != D || Hb.sizes[0] != D || Wd.sizes[0] != D || Bd.sizes[0] != 1 ||
      Y.sizes[0] != B || Z.sizes[0] != B || Lo.sizes[0] != B || Dz.sizes[0] != B)
    return fail(REMORA_ERR_SHAPE,
                "dense_bias_relu_bce: shapes must be hpre/h [B,D], hb/w [D], b [1], y/z/loss/dz [B]");
  if (B == 0) return REMORA_OK;
  note_launch();
  dense_bce_kernel<<<grid_for((long long)B * 32, ctx->sm_count), 256, 0, (cudaStream_t)stream>>>(
      (const float *)Hp.data(4), (const float *)Hb.data(4), (float *)Hd.data(4), (const float *)Wd.data(4),
      (const float *)Bd.data(4), (const float *)Y.data(4), (float *)Z.data(4), (float *)Lo.data(4),
      (float *)Dz.data(4), B, D, grad_scale);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_dense_relu_bwd(RemoraB200Ctx *ctx, const RemoraMemRef2 *h, const RemoraMemRef1 *w,
                               const RemoraMemRef1 *dz, RemoraMemRef2 *dh, RemoraMemRef1 *dw, RemoraMemRef1 *db,
                               RemoraMemRef1 *dh_colsum, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView Hd, Wd, Dz, Dh, Dw, Db;
  REMORA_TRY(read_desc(h, 2, &Hd, "hidden"));
  REMORA_TRY(read_desc(w, 1, &Wd, "dense weights"));
  REMORA_TRY(read_desc(dz, 1, &Dz, "logit gradients"));
  REMORA_TRY(read_desc(dh, 2, &Dh, "hidden gradients"));
  REMORA_TRY(read_desc(dw, 1, &Dw, "weight gradients"));
  REMORA_TRY(read_desc(db, 1, &Db, "bias gradient"));
  for (const DescView *d : {&Hd, &Wd, &Dz, &Dh, &Dw, &Db})
    if (!d->contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "dense_relu_bwd: operands must be contiguous");
  const int B = (int)Hd.sizes[0], D = (int)Hd.sizes[1];
  if (Wd.sizes[0] != D || Dz.sizes[0] != B || Dh.sizes[0] != B || Dh.sizes[1] != D || Dw.sizes[0] != D ||
      Db.sizes[0] != 1)
    return fail(REMORA_ERR_SHAPE, "dense_relu_bwd: shapes must be h/dh [B,D], w/dw [D], dz [B], db [1]");
  float *ds = nullptr;
  if (dh_colsum) {
    DescView Ds;
    REMORA_TRY(read_desc(dh_colsum, 1, &Ds, "hidden-bias gradient"));
    if (Ds.sizes[0] != D || !Ds.contiguous())
      return fail(REMORA_ERR_SHAPE, "dense_relu_bwd: dh_colsum must be a contiguous [%d]", D);
    ds = (float *)Ds.data(4);
  }
  note_launch();
  dense_bwd_kernel<<<D + 1, 256, 0, (cudaStream_t)stream>>>(
      (const float *)Hd.data(4), (const float *)Wd.data(4), (const float *)Dz.data(4), (float *)Dh.data(4),
      (float *)Dw.data(4), (float *)Db.data(4), ds, B, D);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int remora_b200_conv1_wgrad_pooled(RemoraB200Ctx *ctx, const RemoraMemRef4 *x, const RemoraMemRef4 *dpooled,
                                   const RemoraMemRef4 *code, RemoraMemRef4 *dw, RemoraMemRef1 *db,
                                   remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView X, P, C, Dw, Db;
  REMORA_TRY(need4(x, &X, "conv1 input"));
  REMORA_TRY(need4(dpooled, &P, "pooled gradient"));
  REMORA_TRY(need4(code, &C, "pool codes"));
  REMORA_TRY(need4(dw, &Dw, "conv1 weight gradient"));
  REMORA_TRY(read_desc(db, 1, &Db, "conv1 bias gradient"));
  const int B = (int)X.sizes[0], H = (int)X.sizes[2], W = (int)X.sizes[3], K = (int)Dw.sizes[0];
  if (X.sizes[1] != 1 || Dw.sizes[1] != 1 || Dw.sizes[2] != 3 || Dw.sizes[3] != 3 || Db.sizes[0] != K ||
      P.sizes[0] != B || P.sizes[1] != K || P.sizes[2] != H / 2 || P.sizes[3] != W / 2)
    return fail(REMORA_ERR_SHAPE, "conv1_wgrad_pooled: x [B,1,H,W], dpooled/codes [B,K,H/2,W/2], dw [K,1,3,3]");
  if (!((H == 64 && W == 64) || (H == 32 && W == 32)))
    return fail(REMORA_ERR_UNSUPPORTED, "conv1_wgrad_pooled: images of 64x64 or 32x32");
  if (K == 0) return REMORA_OK;
  if (B == 0) {
    REMORA_CUDA_TRY(cudaMemsetAsync(Dw.data(4), 0, (size_t)K * 9 * 4, (cudaStream_t)stream));
    REMORA_CUDA_TRY(cudaMemsetAsync(Db.data(4), 0, (size_t)K * 4, (cudaStream_t)stream));
    return REMORA_OK;
  }
  const int parts = conv1_parts(B, H);
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, (cudaStream_t)stream, (size_t)B * parts * K * 10 * sizeof(double) + 256, &ws));
  double *part = reinterpret_cast<double *>(ws->buf);
  auto kern = H != 64      ? conv1_wgrad_pool_kernel<32, 32, 1>
              : parts == 4 ? conv1_wgrad_pool_kernel<64, 64, 4>
              : parts == 2 ? conv1_wgrad_pool_kernel<64, 64, 2>
                           : conv1_wgrad_pool_kernel<64, 64, 1>;
  const bool vec = aligned(X.data(4), 16) && aligned(P.data(4), 16) && aligned(C.data(1), 4);
  note_launch();
  kern<<<B * parts, kConv1Threads, 0, (cudaStream_t)stream>>>((const float *)X.data(4), (const float *)P.data(4),
                                                              (const uint8_t *)C.data(1), part, K, vec);
  note_launch();
  conv1_wgrad_finish_kernel<<<K * 10, 256, 0, (cudaStream_t)stream>>>(part, (float *)Dw.data(4),
                                                                      (float *)Db.data(4), B * parts, K);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

}  // extern "C"
