// conv_wgrad_tc.cu — tcgen05 weight (and bias) gradient of a 3x3 / pad 1 /
// stride 1 convolution, one launch per group of 16 input channels and at
// most 32 output channels (the benchmark layer and the crater CNN's second
// layer are one group each), TF32, 3xTF32 or 2xTF32:
//   dw[co][ci][r][s] = sum_pixels dy[co][p] * x[ci][p + (r - 1, s - 1)]
//   db[co]           = sum_pixels dy[co][p]
// GEMM view: M = 64 rows (dy channels 0..31, then 32 more rows: zero for
// TF32, the low halves of dy for 3xTF32), N = 160 columns (the 9 x 16
// shifted input channels, then a row of ones that yields db, then zeros),
// K = the pixels of the batch.  Each CTA owns one accumulator for its whole
// share of the pixels; the per-CTA partials are added in CTA order in f64
// by a second kernel (deterministic).
//
// Pixels are consumed in tiles of R image rows.  Per tile:
//   warp 0 lane 0   TMA: x rows h0-1 .. h0+R (zero outside the image) and
//                   dy rows h0 .. h0+R-1, raw NCHW, into a raw stage
//   warps 2-13      transform: the K-major interleaved operands, 4 pixels
//                   (16 bytes) per row and K chunk: A[chunk][co] from dy
//                   rows, B[chunk][tap * 16 + ci] from x rows shifted by the
//                   tap (left/right image borders read as zero)
//   warp 1 lane 0   one tcgen05.mma (M = 64, N = 160, K = 8) per 8 pixels;
//                   3xTF32 adds a second one against the low halves of x:
//                   [dy_hi; dy_lo] x x_hi + [dy_hi; dy_lo] x x_lo covers
//                   hi*hi, lo*hi, hi*lo (and lo*lo) in one accumulator whose
//                   two 32-row halves the epilogue adds.  2xTF32 keeps the
//                   split rows of dy and the first MMA only:
//                   [dy_hi; dy_lo] x x (x as TF32).
//   warps 2-5       epilogue, once after their last transform tile:
//                   TMEM -> shared -> partials.
// Chunks of the operands are 16 bytes longer than their rows so that the
// lanes of the transform, which walk consecutive chunks, hit different
// shared-memory banks.
#include <cudaTypedefs.h>

#include <algorithm>

#include "conv.cuh"
#include "tcgen05.cuh"

namespace remora {

namespace {

constexpr uint32_t wg_align1k(uint32_t v) { return (v + 1023u) & ~1023u; }

constexpr int kWgCin = 16;
constexpr int kWgRowsA = 64;                // M
constexpr int kWgRowsB = 9 * kWgCin + 16;   // N = 160
constexpr int kWgOnesRow = 9 * kWgCin;      // B row of ones: column 144 of D is db
constexpr int kWgOutCols = 9 * kWgCin + 1;  // 145 columns kept per partial
constexpr int kWgThreads = 448;
constexpr int kWgTransformWarp0 = 2, kWgTransformWarps = 12;  // warps 2-5 also run the epilogue
constexpr int kWgTransformThreads = kWgTransformWarps * 32;

// UNPOOL: dy is given as a pooled gradient and its 2x2 max-pool codes
// ([COUT][H/2][W/2] each); the transform expands it (the pooled value goes
// to the recorded window element, the others are 0).
// PREC: 0 TF32, 1 3xTF32 (dy and x split), 2 2xTF32 (dy split, x TF32).
template <int W, int R, int PREC, int RAW_ST, int OP_ST, bool UNPOOL = false>
struct WgCfg {
  static constexpr bool SPLIT_A = PREC >= 1;  // dy as [hi; lo] rows
  static constexpr bool SPLIT_B = PREC == 1;  // x hi and lo copies
  static constexpr int CPR = W / 4;     // 4-pixel chunks per image row
  static constexpr int NCH = R * CPR;   // chunks per tile
  static constexpr uint32_t A_CH = kWgRowsA * 16 + 16;
  static constexpr uint32_t B_CH = kWgRowsB * 16 + 16;
  static constexpr uint32_t A_BYTES = NCH * A_CH;
  static constexpr uint32_t B_BYTES = NCH * B_CH;
  static constexpr uint32_t OP_STAGE = wg_align1k(A_BYTES + B_BYTES * (SPLIT_B ? 2 : 1));
  static constexpr uint32_t RAWX = kWgCin * (R + 2) * W * 4;
  static constexpr uint32_t RAWD = UNPOOL ? 32 * (R / 2) * (W / 2) * 4 : 32 * R * W * 4;
  static constexpr uint32_t RAWC = UNPOOL ? 32 * (R / 2) * (W / 2) : 0;  // codes
  static constexpr uint32_t RAWX_AL = wg_align1k(RAWX);  // dy raw rows start here
  static constexpr uint32_t RAWC_OFF = RAWX_AL + wg_align1k(RAWD);
  static constexpr uint32_t RAW_STAGE = RAWC_OFF + wg_align1k(RAWC);
  static constexpr uint32_t OFF_RAW = OP_ST * OP_STAGE;
  static constexpr size_t SMEM = (size_t)OFF_RAW + (size_t)RAW_ST * RAW_STAGE + 1024;
  static constexpr int ITEMS_A = 32 * NCH;
  static constexpr int ITEMS_B = 3 * kWgCin * NCH;
  static_assert(NCH % 2 == 0, "K steps of 8 pixels");
  static_assert(!UNPOOL || (R % 2 == 0 && W % 32 == 0), "pooled rows are 16-byte TMA boxes");
  static_assert(SMEM <= 230 * 1024, "shared memory per block");
  static_assert(kWgRowsA * kWgRowsB * 4 <= OP_STAGE, "the epilogue reuses an operand stage");
  static_assert(A_CH / 16 < 16384 && B_CH / 16 < 16384, "descriptor offsets");
};

struct WgParams {
  int N, H, COUT;  // COUT: the output channels of this launch (at most 32)
  int tiles_per_img;
  float *part;  // [gridDim.x][32][kWgOutCols]
  int *err;
  // this launch's channels: input channels ci0 .. ci0 + 15 of cin_total and
  // output channels co0 .. co0 + COUT - 1 of cout_total (a layer with more
  // channels runs one launch per group)
  int ci0, cin_total, co0, cout_total;
};

__device__ __forceinline__ void wg_st4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}
__device__ __forceinline__ float4 wg_ld4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}
__device__ __forceinline__ float wg_ld1(uint32_t addr) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(addr) : "memory");
  return v;
}
__device__ __forceinline__ float wg_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// Writes v (4 pixels of one operand row), or for 3xTF32 its high half at
// `hi` and its low half at `lo`.
template <bool SPLIT3>
__device__ __forceinline__ void wg_put(uint32_t hi, uint32_t lo, float4 v) {
  if (SPLIT3) {
    const float a = wg_hi(v.x), b = wg_hi(v.y), c = wg_hi(v.z), d = wg_hi(v.w);
    wg_st4(hi, a, b, c, d);
    wg_st4(lo, __fsub_rn(v.x, a), __fsub_rn(v.y, b), __fsub_rn(v.z, c), __fsub_rn(v.w, d));
  } else {
    wg_st4(hi, v.x, v.y, v.z, v.w);
  }
}

template <int W, int R, int PREC, int RAW_ST, int OP_ST, bool UNPOOL>
__global__ void __launch_bounds__(kWgThreads, 1)
    conv_wgrad_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmd,
                         const __grid_constant__ CUtensorMap tmc, WgParams p) {
  // tmd: dy rows, or with UNPOOL the pooled gradient; tmc: its codes
  using Cf = WgCfg<W, R, PREC, RAW_ST, OP_ST, UNPOOL>;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t rfull[RAW_ST], rempty[RAW_ST], ofull[OP_ST], oempty[OP_ST], drain, efull;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t s_base = tc::smem_u32(smem);
  const uint32_t raw_bytes = UNPOOL ? Cf::RAWX + (uint32_t)p.COUT * (R / 2) * (W / 2) * 5
                                    : Cf::RAWX + (uint32_t)p.COUT * R * W * 4;
  if (threadIdx.x == 0) {
    for (int s = 0; s < RAW_ST; ++s) {
      tc::mbar_init(&rfull[s], 1);
      tc::mbar_init(&rempty[s], kWgTransformWarps);
    }
    for (int s = 0; s < OP_ST; ++s) {
      tc::mbar_init(&ofull[s], kWgTransformWarps);
      tc::mbar_init(&oempty[s], 1);
    }
    tc::mbar_init(&drain, 1);
    tc::mbar_init(&efull, 4);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  // Operand stages start zero; the ones row of B (high copy) is set once.
  for (uint32_t off = threadIdx.x * 16; off < OP_ST * Cf::OP_STAGE; off += kWgThreads * 16)
    wg_st4(s_base + off, 0.f, 0.f, 0.f, 0.f);
  __syncthreads();
  for (int e = threadIdx.x; e < OP_ST * Cf::NCH; e += kWgThreads) {
    const int st = e / Cf::NCH, kc = e % Cf::NCH;
    wg_st4(s_base + st * Cf::OP_STAGE + Cf::A_BYTES + kc * Cf::B_CH + kWgOnesRow * 16, 1.f, 1.f, 1.f, 1.f);
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  if (warp == 1) tc::tmem_alloc(&tmem_base, 256);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const int ntiles = p.N * p.tiles_per_img;
  volatile int *abort_v = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ------------------------------------------------------- TMA producer
      tc::prefetch_tmap(&tmx);
      tc::prefetch_tmap(&tmd);
      int it = 0, issued = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int st = it % RAW_ST;
        if (!tc::mbar_wait(&rempty[st], ((it / RAW_ST) & 1) ^ 1, abort_v, p.err, 211)) break;
        const int n = t / p.tiles_per_img, h0 = (t % p.tiles_per_img) * R;
        uint8_t *raw = smem + Cf::OFF_RAW + st * Cf::RAW_STAGE;
        tc::mbar_arrive_expect_tx(&rfull[st], raw_bytes);
        tc::tma_load_3d(&tmx, &rfull[st], raw, 0, h0 - 1, n * p.cin_total + p.ci0);
        if (UNPOOL) {
          tc::tma_load_3d(&tmd, &rfull[st], raw + Cf::RAWX_AL, 0, h0 / 2, n * p.cout_total + p.co0);
          tc::tma_load_3d(&tmc, &rfull[st], raw + Cf::RAWC_OFF, 0, h0 / 2, n * p.cout_total + p.co0);
        } else {
          tc::tma_load_3d(&tmd, &rfull[st], raw + Cf::RAWX_AL, 0, h0, n * p.cout_total + p.co0);
        }
        ++issued;
      }
      for (int j = issued > RAW_ST ? issued - RAW_ST : 0; j < issued; ++j) {
        const long long t0 = clock64();
        while (!tc::mbar_test(&rfull[j % RAW_ST], (j / RAW_ST) & 1) && clock64() - t0 < tc::kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---------------------------------------------------------- MMA issue
      const uint32_t idesc = tc::idesc_tf32(kWgRowsA, kWgRowsB, 0, 0);
      int it = 0;
      bool issued = false;
      uint32_t accum = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
        const int st = it % OP_ST;
        if (!tc::mbar_wait(&ofull[st], (it / OP_ST) & 1, abort_v, p.err, 212)) break;
        tc::fence_after_sync();
        const uint32_t a0 = s_base + st * Cf::OP_STAGE, b0 = a0 + Cf::A_BYTES, bl0 = b0 + Cf::B_BYTES;
        const uint64_t ad = tc::smem_desc(a0, Cf::A_CH, 128, 0);
        const uint64_t bd = tc::smem_desc(b0, Cf::B_CH, 128, 0);
        const uint64_t bld = tc::smem_desc(bl0, Cf::B_CH, 128, 0);
#pragma unroll 4
        for (int j = 0; j < Cf::NCH / 2; ++j) {
          const uint64_t ao = (uint64_t)((2 * j * Cf::A_CH) >> 4), bo = (uint64_t)((2 * j * Cf::B_CH) >> 4);
          tc::mma_tf32(tbase, ad + ao, bd + bo, idesc, accum);
          accum = 1;
          if (Cf::SPLIT_B) tc::mma_tf32(tbase, ad + ao, bld + bo, idesc, 1);
        }
        issued = true;
        tc::mma_commit(&oempty[st]);
      }
      if (issued) tc::mma_commit(&drain);
    }
  } else {
    // Warps 2-13 build the operands of every tile; after the last one,
    // warps 2-5 also run the epilogue (they are idle until then).
    // ------------------------------------------------------------ transform
    const int tt = threadIdx.x - kWgTransformWarp0 * 32;
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int rs = it % RAW_ST, os = it % OP_ST;
      if (!tc::mbar_wait(&rfull[rs], (it / RAW_ST) & 1, abort_v, p.err, 215)) break;
      if (!tc::mbar_wait(&oempty[os], ((it / OP_ST) & 1) ^ 1, abort_v, p.err, 216)) break;
      const uint32_t rawx = s_base + Cf::OFF_RAW + rs * Cf::RAW_STAGE, rawd = rawx + Cf::RAWX_AL;
      const uint32_t a0 = s_base + os * Cf::OP_STAGE, b0 = a0 + Cf::A_BYTES, bl0 = b0 + Cf::B_BYTES;
      // A: dy rows, 4 pixels per 16 bytes (hi in rows 0..31, lo in 32..63)
      for (int item = tt; item < Cf::ITEMS_A; item += kWgTransformThreads) {
        const int kc = item % Cf::NCH, co = item / Cf::NCH;
        if (co >= p.COUT) continue;
        const int hr = kc / Cf::CPR, w0 = 4 * (kc % Cf::CPR);
        float4 v;
        if (UNPOOL) {
          // row hr of the tile: pooled row hr / 2, parity hr & 1; pixels
          // w0 .. w0+3 in pooled columns w0/2, w0/2 + 1
          const uint32_t e = (uint32_t)((co * (R / 2) + hr / 2) * (W / 2) + w0 / 2);
          float2 g;
          uint32_t cw;
          asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(g.x), "=f"(g.y) : "r"(rawd + e * 4) : "memory");
          asm volatile("ld.shared.u16 %0, [%1];" : "=r"(cw) : "r"(rawd - Cf::RAWX_AL + Cf::RAWC_OFF + e) : "memory");
          const uint32_t hp = (uint32_t)(hr & 1) * 2, c0 = cw & 0xFF, c1 = (cw >> 8) & 0xFF;
          v = make_float4(c0 == hp ? g.x : 0.0f, c0 == hp + 1 ? g.x : 0.0f, c1 == hp ? g.y : 0.0f,
                          c1 == hp + 1 ? g.y : 0.0f);
        } else {
          v = wg_ld4(rawd + (uint32_t)((co * R + hr) * W + w0) * 4);
        }
        const uint32_t dst = a0 + kc * Cf::A_CH + co * 16;
        wg_put<Cf::SPLIT_A>(dst, dst + 32 * 16, v);
      }
      // B: x rows shifted by the tap, three column shifts from one read.
      // A warp's 32 items are whole groups of NCH consecutive chunks, so the
      // pixels either side of a chunk are the neighbouring lanes' (one
      // 16-byte read per lane, no 4-byte reads that share banks).
      static_assert(Cf::ITEMS_B % kWgTransformThreads == 0 && 32 % Cf::NCH == 0,
                    "every lane runs each pass; a warp covers whole chunk groups");
      for (int item = tt; item < Cf::ITEMS_B; item += kWgTransformThreads) {
        const int kc = item % Cf::NCH, rci = item / Cf::NCH, ci = rci % kWgCin, r = rci / kWgCin;
        const int hr = kc / Cf::CPR, w0 = 4 * (kc % Cf::CPR);
        const uint32_t row = rawx + (uint32_t)((ci * (R + 2) + hr + r) * W) * 4;
        const float4 L = wg_ld4(row + w0 * 4);
        const float left = __shfl_up_sync(0xffffffffu, L.w, 1);
        const float right = __shfl_down_sync(0xffffffffu, L.x, 1);
        const float prev = w0 > 0 ? left : 0.0f;
        const float next = w0 + 4 < W ? right : 0.0f;
        const uint32_t dst = b0 + kc * Cf::B_CH + ((r * 3) * kWgCin + ci) * 16;
        wg_put<Cf::SPLIT_B>(dst, dst + Cf::B_BYTES, make_float4(prev, L.x, L.y, L.z));
        wg_put<Cf::SPLIT_B>(dst + kWgCin * 16, dst + kWgCin * 16 + Cf::B_BYTES, L);
        wg_put<Cf::SPLIT_B>(dst + 2 * kWgCin * 16, dst + 2 * kWgCin * 16 + Cf::B_BYTES,
                            make_float4(L.y, L.z, L.w, next));
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&ofull[os]);
        tc::mbar_arrive(&rempty[rs]);
      }
    }
    if (warp < kWgTransformWarp0 + 4) {
      // ------------------------------------------------------------- epilogue
      // D row m (M = 64, one CTA) lives in TMEM lane (m % 16) + 32 * (m / 16):
      // warp quarter q holds rows 16q .. 16q+15 in its first 16 lanes.
      const int q = warp & 3;
      bool ok = ntiles > (int)blockIdx.x;
      if (ok) ok = tc::mbar_wait(&drain, 0, abort_v, p.err, 213);
      if (ok) {
        tc::fence_after_sync();
        const uint32_t dsm = s_base;  // operand stage 0, idle now
#pragma unroll 1
        for (int c = 0; c < kWgRowsB / 32; ++c) {
          uint32_t r[32];
          tc::tmem_ld_32x32b_x32(tbase + c * 32 + ((uint32_t)(q * 32) << 16), r);
          tc::tmem_ld_wait();
          if (lane < 16) {
            const int m = 16 * q + lane;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              asm volatile("st.shared.f32 [%0], %1;" ::"r"(dsm + (uint32_t)(m * kWgRowsB + c * 32 + j) * 4),
                           "r"(r[j])
                           : "memory");
          }
        }
        tc::fence_before_sync();
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&efull);
        ok = tc::mbar_wait(&efull, 0, abort_v, p.err, 214);
        if (ok) {
          float *pb = p.part + (long long)blockIdx.x * 32 * kWgOutCols;
          for (int idx = (warp - 2) * 32 + lane; idx < 32 * kWgOutCols; idx += 128) {
            const int co = idx / kWgOutCols, n = idx % kWgOutCols;
            const float v = __fadd_rn(wg_ld1(dsm + (uint32_t)(co * kWgRowsB + n) * 4),
                                      wg_ld1(dsm + (uint32_t)((32 + co) * kWgRowsB + n) * 4));
            pb[idx] = v;
          }
        }
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 256);
  }
}

// dw[co][ci][r][s] and db[co] from the per-CTA partials in f64: one warp
// per value, lane l adding partials l, l+32, ... in order, then a fixed
// shuffle tree (deterministic).
__global__ void __launch_bounds__(256) wgrad_tc_finish(const float *__restrict__ part, int nblocks, int cout,
                                                       int cin_total, float *__restrict__ dw, float *__restrict__ db) {
  const int e = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (e >= cout * kWgOutCols) return;
  const int co = e / kWgOutCols, n = e % kWgOutCols;
  double s = 0.0;
  for (int b = lane; b < nblocks; b += 32) s += (double)part[((long long)b * 32 + co) * kWgOutCols + n];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if (lane != 0) return;
  if (n == kWgOnesRow) {
    if (db) db[co] = (float)s;
  } else {
    const int tap = n / kWgCin, ci = n % kWgCin;
    dw[((long long)co * cin_total + ci) * 9 + tap] = (float)s;
  }
}

int wg_encode(const void *x, int N, int C, int H, int W, int box_rows, int box_ch, CUtensorMap *map,
              bool codes = false) {
  auto fn = tensor_map_encoder();
  if (!fn) return fail(REMORA_ERR_CUDA, "conv wgrad: cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t es = codes ? 1 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N * C};
  cuuint64_t strides[2] = {(cuuint64_t)W * es, (cuuint64_t)H * W * es};
  cuuint32_t box[3] = {(cuuint32_t)W, (cuuint32_t)box_rows, (cuuint32_t)box_ch};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, codes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                  const_cast<void *>(x), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(REMORA_ERR_CUDA, "conv wgrad: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return REMORA_OK;
}

// One launch per group of 16 input channels and at most 32 output
// channels (groups of equal size); each writes its block of dw (and, the
// first input-channel group, of db).
template <int W, int R, int PREC, int RAW_ST, int OP_ST, bool UNPOOL = false>
int launch_wgrad(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dy, const uint8_t *codes,
                 float *dw, float *db, cudaStream_t stream) {
  using Cf = WgCfg<W, R, PREC, RAW_ST, OP_ST, UNPOOL>;
  auto kern = conv_wgrad_tc_kernel<W, R, PREC, RAW_ST, OP_ST, UNPOOL>;
  static bool attr = false;
  if (!attr) {
    REMORA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::SMEM));
    attr = true;
  }
  const int ng = (g.K + 31) / 32, gs = (g.K + ng - 1) / ng;
  const int tiles_per_img = (g.H + R - 1) / R;
  const int ntiles = g.N * tiles_per_img;
  const int grid = std::min(ntiles, ctx->persistent_limit());
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, (size_t)grid * 32 * kWgOutCols * sizeof(float) + 256, &ws));
  CUtensorMap mx, md, mc;
  REMORA_TRY(wg_encode(x, g.N, g.C, g.H, W, R + 2, kWgCin, &mx));
  for (int co0 = 0; co0 < g.K; co0 += gs) {
    const int cout = std::min(gs, g.K - co0);
    if (UNPOOL) {
      REMORA_TRY(wg_encode(dy, g.N, g.K, g.H / 2, W / 2, R / 2, cout, &md));
      REMORA_TRY(wg_encode(codes, g.N, g.K, g.H / 2, W / 2, R / 2, cout, &mc, true));
    } else {
      REMORA_TRY(wg_encode(dy, g.N, g.K, g.H, W, R, cout, &md));
      mc = md;
    }
    for (int ci0 = 0; ci0 < g.C; ci0 += kWgCin) {
      WgParams p{g.N, g.H, cout, tiles_per_img, reinterpret_cast<float *>(ws->buf), ws->err, ci0, g.C, co0, g.K};
      note_launch();
      kern<<<grid, kWgThreads, Cf::SMEM, stream>>>(mx, md, mc, p);
      const int outs = cout * kWgOutCols;
      note_launch();
      wgrad_tc_finish<<<(outs * 32 + 255) / 256, 256, 0, stream>>>(
          p.part, grid, cout, g.C, dw + ((long long)co0 * g.C + ci0) * 9, ci0 == 0 && db ? db + co0 : nullptr);
    }
  }
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

// 0 TF32, 1 3xTF32, 2 2xTF32; -1 for an unknown precision
int wg_prec(int precision) {
  return precision == REMORA_PREC_TF32 ? 0 : precision == REMORA_PREC_3XTF32 ? 1 : precision == REMORA_PREC_2XTF32 ? 2 : -1;
}

}  // namespace

int conv_tc_wgrad_bias(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dy, float *dw, float *db,
                       int precision, cudaStream_t stream, bool *handled) {
  *handled = false;
  const int prec = wg_prec(precision);
  if (prec < 0 || g.R != 3 || g.S != 3 || g.pad != 1 || g.stride != 1 || g.C < kWgCin || g.C % kWgCin ||
      g.K < 1 || g.N < 1 || g.H < 1 || g.OH != g.H || g.OW != g.W)
    return REMORA_OK;
  if ((reinterpret_cast<uintptr_t>(x) & 15) || (reinterpret_cast<uintptr_t>(dy) & 15)) return REMORA_OK;
  *handled = true;
  if (g.W == 16)
    return prec == 1 ? launch_wgrad<16, 4, 1, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream)
         : prec == 2 ? launch_wgrad<16, 4, 2, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream)
                     : launch_wgrad<16, 4, 0, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream);
  if (g.W == 128 && prec != 1)  // 3xTF32's hi and lo copies of x do not fit a 128-wide row
    return prec == 2 ? launch_wgrad<128, 1, 2, 2, 1>(ctx, g, x, dy, nullptr, dw, db, stream)
                     : launch_wgrad<128, 1, 0, 2, 1>(ctx, g, x, dy, nullptr, dw, db, stream);
  if (g.W == 32)
    return prec == 1 ? launch_wgrad<32, 2, 1, 1, 2>(ctx, g, x, dy, nullptr, dw, db, stream)
         : prec == 2 ? launch_wgrad<32, 2, 2, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream)
                     : launch_wgrad<32, 2, 0, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream);
  if (g.W == 64)
    return prec == 1 ? launch_wgrad<64, 1, 1, 1, 2>(ctx, g, x, dy, nullptr, dw, db, stream)
         : prec == 2 ? launch_wgrad<64, 1, 2, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream)
                     : launch_wgrad<64, 1, 0, 2, 2>(ctx, g, x, dy, nullptr, dw, db, stream);
  *handled = false;
  return REMORA_OK;
}

int conv_tc_wgrad_bias_unpool(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *dpooled,
                              const uint8_t *codes, float *dw, float *db, int precision, cudaStream_t stream,
                              bool *handled) {
  *handled = false;
  const int prec = wg_prec(precision);
  if (prec < 0 || g.R != 3 || g.S != 3 || g.pad != 1 || g.stride != 1 ||
      g.C != kWgCin || g.K < 1 || g.K > 32 || g.N < 1 || g.H < 2 || g.H % 2 || g.OH != g.H || g.OW != g.W ||
      g.W != 32)
    return REMORA_OK;
  const auto a16 = [](const void *q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!a16(x) || !a16(dpooled) || !a16(codes)) return REMORA_OK;
  *handled = true;
  return prec == 1 ? launch_wgrad<32, 2, 1, 1, 2, true>(ctx, g, x, dpooled, codes, dw, db, stream)
       : prec == 2 ? launch_wgrad<32, 2, 2, 2, 2, true>(ctx, g, x, dpooled, codes, dw, db, stream)
                   : launch_wgrad<32, 2, 0, 2, 2, true>(ctx, g, x, dpooled, codes, dw, db, stream);
}

}  // namespace remora
