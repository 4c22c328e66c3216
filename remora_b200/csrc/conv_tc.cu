// conv_tc.cu — tcgen05 implicit-GEMM convolution for 3x3 / pad 1 / stride 1
// (the benchmark layer [256,16,64,64] * [32,16,3,3] and the crater CNN's
// second layer), forward and input gradient.
//
// GEMM view of one tile: M = 128-pixel blocks of the output (TH rows x W
// columns of one image), N = 32 output channels (zero-padded weights when
// there are fewer), K = input channels, accumulated over the 9 taps.
// im2col never touches HBM: the loader warps stage the TH+2 input rows of
// the tile once per channel and write them to shared memory three times,
// shifted by -1, 0, +1 columns (zero at the image border).  Each copy is an
// MN-major SWIZZLE_128B_BASE32B operand (32 pixels per 128-byte row, one row
// per channel), so the A operand of tap (r, s) is copy s starting r*W pixels
// further — a descriptor offset, no data movement.  Weights stay resident
// in shared memory for the whole kernel in the same MN-major form.
//
// Roles (416 threads): warps 0-7 load and shift the input rows (all of a
// tile's 128-bit loads in flight at once, then generic stores +
// fence.proxy.async and an mbarrier arrive), warp 12 lane 0 issues
// 9 * CIN/8 tcgen05.mma (M=128, N=32, K=8) per 128-pixel block into a TMEM
// accumulator, warps 8-11 read TMEM (32 lanes x 32 channels per warp), add
// the bias and store NCHW rows (for one channel a warp writes 32 consecutive
// pixels).  Two TMEM accumulators and up to two input stages overlap load,
// MMA and epilogue of consecutive tiles.  Input gradient: the same kernel
// on dY with w'[c][k][r][s] = w[k][c][2-r][2-s].
#include <algorithm>

#include "conv.cuh"
#include "tcgen05.cuh"

namespace remora {

namespace {

template <int CIN, int IMG_W, int MT, int STAGES>
struct ConvCfg {
  static constexpr int PIX = 128 * MT;
  static constexpr int TH = PIX / IMG_W;
  static constexpr int ROWS = TH + 2;
  static constexpr uint32_t LBO = CIN * 128;  // bytes between 32-pixel chunks
  static constexpr uint32_t COPY_BYTES = (uint32_t)ROWS * IMG_W * CIN * 4;
  static constexpr uint32_t STAGE_BYTES = 3 * COPY_BYTES;
  static constexpr uint32_t W_BYTES = 9 * CIN * 128;
  static constexpr size_t SMEM = W_BYTES + (size_t)STAGES * STAGE_BYTES + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * MT * 32 <= 64 ? 64 : 128;
  static constexpr int NVEC = CIN * ROWS * (IMG_W / 4);
  static constexpr int NV = NVEC / 256;  // 16-byte loads per loader thread per tile
  static_assert(NVEC % 256 == 0, "loads split evenly over the 256 loader threads");
  static_assert(PIX % IMG_W == 0, "tile must hold whole rows");
  static_assert(COPY_BYTES % 1024 == 0 && W_BYTES % 1024 == 0, "1 KB aligned operand regions");
  static_assert(CIN % 8 == 0, "K steps of 8 channels");
};

struct ConvTCParams {
  const float *x;
  const float *w;
  const float *bias;
  float *y;
  int N, H, COUT;
  int mode;  // 0: forward, w is [COUT][CIN][3][3]; 1: input gradient, w is [CIN][COUT][3][3] (forward weights)
  int tiles_per_img;
  int *err;
};

// warps 0-7 load, 8-11 epilogue (lane quarters 0-3), 12 MMA + TMEM alloc
constexpr int kConvThreads = 416;
constexpr int kLoaders = 256;

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

template <int CIN, int IMG_W, int MT, int STAGES>
__global__ void __launch_bounds__(kConvThreads, 1) conv3x3_tc_kernel(ConvTCParams p) {
  using Cf = ConvCfg<CIN, IMG_W, MT, STAGES>;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  uint8_t *wsm = smem;
  uint8_t *stg = smem + Cf::W_BYTES;
  __shared__ __align__(8) uint64_t afull[STAGES], aempty[STAGES], tfull[2], tempty[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ float bias_s[32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&afull[s], kLoaders);
      tc::mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 4);
    }
    tc::mbar_init(&drain, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (threadIdx.x < 32) bias_s[threadIdx.x] = (p.bias && (int)threadIdx.x < p.COUT) ? p.bias[threadIdx.x] : 0.0f;
  // Resident weights, one MN-major [CIN][32] tile per tap.
  for (int idx = threadIdx.x; idx < 9 * CIN * 32; idx += kConvThreads) {
    const int co = idx & 31, ci = (idx >> 5) % CIN, tap = idx / (CIN * 32);
    const int r = tap / 3, s = tap % 3;
    float v = 0.0f;
    if (co < p.COUT)
      v = p.mode == 0 ? __ldg(p.w + ((co * CIN + ci) * 3 + r) * 3 + s)
                      : __ldg(p.w + ((ci * p.COUT + co) * 3 + (2 - r)) * 3 + (2 - s));
    const uint32_t off = tap * CIN * 128 + (ci >> 2) * 512 + (ci & 3) * 128 + (((co >> 3) ^ (ci & 3)) << 5) +
                         (co & 7) * 4;
    *reinterpret_cast<float *>(wsm + off) = v;
  }
  fence_proxy_async_smem();
  if (warp == 12) tc::tmem_alloc(&tmem_base, Cf::TMEM_COLS);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const int ntiles = p.N * p.tiles_per_img;
  volatile int *abort_v = &abort_flag;

  if (warp < 8) {
    // --------------------------------------------- input rows -> 3 copies
    // All of a tile's loads go to registers first, before the stage is known
    // to be free, so their latency overlaps the previous tile's MMAs.
    const uint32_t stg_u = tc::smem_u32(stg);
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int st = it % STAGES;
      const uint32_t ph = (it / STAGES) & 1;
      const int n = t / p.tiles_per_img, oh0 = (t % p.tiles_per_img) * Cf::TH;
      float4 val[Cf::NV];
#pragma unroll
      for (int u = 0; u < Cf::NV; ++u) {
        const int v = u * kLoaders + warp * 32 + lane;
        const int q = v % (IMG_W / 4), rl = v / (IMG_W / 4);
        const int c = rl / Cf::ROWS, r = rl % Cf::ROWS;
        const int ih = oh0 - 1 + r;
        val[u] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (ih >= 0 && ih < p.H)
          val[u] = __ldg(reinterpret_cast<const float4 *>(p.x + (((long long)n * CIN + c) * p.H + ih) * IMG_W) + q);
      }
      if (!tc::mbar_wait(&aempty[st], ph ^ 1, abort_v, p.err, 201)) break;
      const uint32_t base = stg_u + st * Cf::STAGE_BYTES;
#pragma unroll
      for (int u = 0; u < Cf::NV; ++u) {
        const int v = u * kLoaders + warp * 32 + lane;
        const int q = v % (IMG_W / 4), rl = v / (IMG_W / 4);
        const int c = rl / Cf::ROWS, r = rl % Cf::ROWS;
        float left = __shfl_up_sync(0xffffffffu, val[u].w, 1);
        float right = __shfl_down_sync(0xffffffffu, val[u].x, 1);
        if (q == 0) left = 0.0f;
        if (q == IMG_W / 4 - 1) right = 0.0f;
        const int px = r * IMG_W + 4 * q;
        const uint32_t off = (px >> 5) * Cf::LBO + (c >> 2) * 512 + (c & 3) * 128 +
                             ((((px & 31) >> 3) ^ (c & 3)) << 5) + ((px & 7) ? 16 : 0);
        st_shared_v4(base + off, left, val[u].x, val[u].y, val[u].z);                       // column - 1
        st_shared_v4(base + Cf::COPY_BYTES + off, val[u].x, val[u].y, val[u].z, val[u].w);  // column
        st_shared_v4(base + 2 * Cf::COPY_BYTES + off, val[u].y, val[u].z, val[u].w, right);  // column + 1
      }
      fence_proxy_async_smem();
      tc::mbar_arrive(&afull[st]);
    }
  } else if (warp == 12 && lane == 0) {
    // ---------------------------------------------------------- MMA issue
    const uint32_t idesc = tc::idesc_tf32(128, 32, 1, 1);
    const uint32_t stg_u = tc::smem_u32(stg), w_u = tc::smem_u32(wsm);
    int it = 0;
    bool issued = false;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int st = it % STAGES;
      const uint32_t ph = (it / STAGES) & 1;
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!tc::mbar_wait(&afull[st], ph, abort_v, p.err, 202)) break;
      if (!tc::mbar_wait(&tempty[acc], aph ^ 1, abort_v, p.err, 203)) break;
      tc::fence_after_sync();
      const uint32_t abase = stg_u + st * Cf::STAGE_BYTES;
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        const uint32_t d = tbase + acc * (MT * 32) + mt * 32;
        uint32_t first = 1;
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const int r = tap / 3, s = tap % 3;
          const uint32_t a0 = abase + s * Cf::COPY_BYTES + ((mt * 128 + r * IMG_W) >> 5) * Cf::LBO;
          const uint32_t b0 = w_u + tap * CIN * 128;
#pragma unroll
          for (int kk = 0; kk < CIN / 8; ++kk) {
            tc::mma_tf32(d, tc::desc_mnmajor(a0, Cf::LBO, kk), tc::desc_mnmajor(b0, CIN * 128, kk), idesc,
                         first ? 0u : 1u);
            first = 0;
          }
        }
      }
      issued = true;
      tc::mma_commit(&aempty[st]);
      tc::mma_commit(&tfull[acc]);
    }
    if (issued) {
      tc::mma_commit(&drain);
      const long long t0 = clock64();
      while (!tc::mbar_test(&drain, 0) && clock64() - t0 < tc::kWaitCycles) {
      }
    }
  } else if (warp >= 8 && warp < 12) {
    // ----------------------------------------------------------- epilogue
    const int q = warp - 8;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aph, abort_v, p.err, 204)) break;
      tc::fence_after_sync();
      const int n = t / p.tiles_per_img, oh0 = (t % p.tiles_per_img) * Cf::TH;
#pragma unroll 1
      for (int mt = 0; mt < MT; ++mt) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(tbase + acc * (MT * 32) + mt * 32 + ((uint32_t)(q * 32) << 16), r);
        tc::tmem_ld_wait();
        const int px = mt * 128 + q * 32 + lane;
        const int oh = oh0 + px / IMG_W, col = px % IMG_W;
        if (oh < p.H) {
          float *yp = p.y + ((long long)n * p.COUT * p.H + oh) * IMG_W + col;
#pragma unroll
          for (int co = 0; co < 32; ++co)
            if (co < p.COUT) yp[(long long)co * p.H * IMG_W] = __fadd_rn(__uint_as_float(r[co]), bias_s[co]);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[acc]);
    }
  }
  __syncthreads();
  if (warp == 12) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, Cf::TMEM_COLS);
  }
}

template <int CIN, int IMG_W, int MT, int STAGES>
int launch_conv(const ConvTCParams &p, int sm_count, cudaStream_t stream) {
  using Cf = ConvCfg<CIN, IMG_W, MT, STAGES>;
  static bool attr = false;
  if (!attr) {
    REMORA_CUDA_TRY(cudaFuncSetAttribute(conv3x3_tc_kernel<CIN, IMG_W, MT, STAGES>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::SMEM));
    attr = true;
  }
  ConvTCParams q = p;
  q.tiles_per_img = (p.H + Cf::TH - 1) / Cf::TH;
  const int ntiles = p.N * q.tiles_per_img;
  const int grid = std::min(ntiles, sm_count);
  conv3x3_tc_kernel<CIN, IMG_W, MT, STAGES><<<grid, kConvThreads, Cf::SMEM, stream>>>(q);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

// Picks the instantiation for (input channels, width); false if none.
int dispatch(const ConvTCParams &p, int cin, int width, int sm_count, cudaStream_t stream, bool *handled) {
  *handled = true;
  if (cin == 16 && width == 64) return launch_conv<16, 64, 2, 2>(p, sm_count, stream);
  if (cin == 32 && width == 64) return launch_conv<32, 64, 1, 1>(p, sm_count, stream);
  if (cin == 16 && width == 32) return launch_conv<16, 32, 2, 2>(p, sm_count, stream);
  if (cin == 32 && width == 32) return launch_conv<32, 32, 1, 2>(p, sm_count, stream);
  *handled = false;
  return REMORA_OK;
}

bool shape_ok(const ConvGeom &g, const void *x, int precision) {
  return precision == REMORA_PREC_TF32 && g.R == 3 && g.S == 3 && g.pad == 1 && g.stride == 1 &&
         (reinterpret_cast<uintptr_t>(x) & 15) == 0 && g.N > 0 && g.H > 0;
}

}  // namespace

int conv_tc_fwd(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *w, const float *bias, float *y,
                int precision, cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!shape_ok(g, x, precision) || g.K > 32) return REMORA_OK;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  ConvTCParams p{x, w, bias, y, g.N, g.H, g.K, 0, 0, ws->err};
  return dispatch(p, g.C, g.W, ctx->sm_count, stream, handled);
}

int conv_tc_dgrad(RemoraB200Ctx *ctx, const ConvGeom &g, const float *dy, const float *w, float *dx, int precision,
                  cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!shape_ok(g, dy, precision) || g.C > 32) return REMORA_OK;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  // forward conv of dy (K channels) into dx (C channels) with flipped weights
  ConvTCParams p{dy, w, nullptr, dx, g.N, g.H, g.C, 1, 0, ws->err};
  return dispatch(p, g.K, g.W, ctx->sm_count, stream, handled);
}

int conv_tc_wgrad(RemoraB200Ctx *, const ConvGeom &, const float *, const float *, float *, int, cudaStream_t,
                  bool *handled) {
  *handled = false;
  return REMORA_OK;
}

}  // namespace remora
