// conv_tc.cu — tcgen05 implicit-GEMM convolution for 3x3 / pad 1 / stride 1
// (among them the benchmark layer [256,16,64,64] * [32,16,3,3] and the
// crater CNN's second layer), forward and input gradient, TF32, 3xTF32 and
// 2xTF32; 16, 32 or 64 input channels on 16- to 128-wide images, output
// channels in launches of at most 32 (a table of instantiations below).
//
// GEMM view of one tile: M = output pixels of TH rows of one image, N = the
// output channels (16 or 32, zero-padded weights above COUT), K = input
// channels, accumulated over the 9 taps.  im2col never touches HBM and is
// never materialised: shared memory holds the tile's TH+2 input rows ONCE,
// as a K-major "interleaved" UMMA operand (layout SWIZZLE_NONE): 16-byte
// rows of 4 channels of one pixel, one plane per 4 channels, rows of the
// image PW = W + 1 positions apart with one zero column between them.
// Output pixel (i, w) is GEMM row m = i * PW + w, and tap (r, s) reads
// operand row m + r * PW + s: every tap is the same operand at another
// 16-byte-aligned start address (a descriptor offset), and the zero column
// is the left pad of one row and the right pad of the one before.  Rows
// m with m % PW == W are discarded in the epilogue.
//
// Forward fused with ReLU + 2x2 max-pool: the operand is split by input
// row parity into two planes per 4 channels (padded rows 2r and 2r + 1 of
// the tile are row r of plane 0 and plane 1, pitch PW = W + 2), GEMM row m
// = i * PW + w stands for pooled row i, and two accumulators per M block
// hold conv rows 2i and 2i + 1: tap (r, s) of conv row 2i + a reads plane
// (a + r) & 1 at row offset (a + r) >> 1, again a descriptor offset.  A
// thread then holds both rows of its pooling window and the lane next to
// it (PW even: lanes 2k, 2k + 1 are columns 2j, 2j + 1) holds the other
// column.
//
// Roles (512 threads):
//   warp 0 lane 0    TMA: one tiled load per tile of the raw NCHW rows
//                    [CIN][TH+2][W] (rows outside the image read as zero)
//   warp 1           TMEM allocation; lane 0 issues the MMAs
//                    (M = 128, N = NOUT, K = 8) into a TMEM accumulator
//   warps 2-9        epilogue: TMEM -> registers (+ bias, ReLU + pool) ->
//                    global memory; for one channel the 32 lanes of a warp
//                    hold consecutive pixels, so every store instruction
//                    writes a contiguous run.  Two warps per TMEM lane
//                    quarter split the channel groups (or the M blocks).
//   warps 10-15      transform: raw rows -> the interleaved operand (and,
//                    for 3xTF32, its hi/lo split)
// Raw stages, operand stages and two accumulators let TMA, transform, MMA
// and epilogue of consecutive tiles overlap.  Input gradient: the same
// kernel on dY with w'[c][k][r][s] = w[k][c][2-r][2-s].
// Precision PREC: 0 TF32 (both operands as given, the tensor core reads
// their TF32 part); 1 3xTF32: hi = x with the low 13 mantissa bits
// cleared, lo = x - hi, for activations and weights, and the MMA adds
// hi*hi + hi*lo + lo*hi into one f32 accumulator; 2 2xTF32: the weights
// alone are split, their hi and lo halves stacked as the N = 2 * NOUT
// columns of one MMA against the TF32 activations, and the epilogue adds
// column c and column NOUT + c (one MMA of twice the width in place of
// three: the activation operand is read once, not three times); 3 3xTF32
// with stacked weights: the activation split into hi and lo copies, the
// weights' hi and lo rows stacked as in 2, and per K step one MMA
// act_hi x [w_hi; w_lo] (N = 2 * NOUT) and one act_lo x w_hi (N = NOUT, into
// the first NOUT columns): the same three products as 1 from two reads of
// the activation operand instead of three.  The 16 -> 32 channel forward on
// 32-wide images (the crater CNN's conv2, plain and pooled) runs this form
// with tiles of 14 rows (two 256-column accumulators fit TMEM), and so does
// the 32 -> 16 channel 3xTF32 input gradient on 32-wide images.
#include <cudaTypedefs.h>

#include <algorithm>

#include "conv.cuh"
#include "tcgen05.cuh"

namespace remora {

namespace {

constexpr uint32_t align1k(uint32_t v) { return (v + 1023u) & ~1023u; }

// Fusions of the crater CNN's second layer:
//   kFuseNone    plain conv (forward or input gradient)
//   kFusePool    forward whose epilogue applies ReLU + 2x2 max-pool and
//                stores the pooled values and the pool codes instead of y
//   kFuseUnpool  input gradient whose input dY is given pooled: the pooled
//                gradient and the codes are expanded to the full-resolution
//                dY (the adjoint of ReLU + max-pool) while the transform
//                builds the operand
constexpr int kFuseNone = 0, kFusePool = 1, kFuseUnpool = 2;
constexpr uint8_t kNoGradCode = 255;

// CSPLIT > 1: the input channels of a tile flow through the raw and operand
// stages in CSPLIT slices of CIN / CSPLIT channels (one TMA load, one
// transform and the MMAs of those channels each, accumulated into the same
// TMEM accumulator), so that a tile of many channels still double-buffers.
template <int CIN, int W, int TH, int NOUT, int PREC, int RAW_ST, int A_ST, int CG, int FUSE = kFuseNone,
          int CSPLIT = 1>
struct ConvCfg {
  static constexpr bool SPLIT_A = PREC == 1 || PREC == 3;  // hi / lo copies of the activation operand
  static constexpr bool SPLIT_W = PREC == 1;               // hi / lo copies of the weights
  static constexpr bool STACKED = PREC == 2 || PREC == 3;  // weight hi rows, then lo rows, in one operand
  static constexpr int NB = STACKED ? 2 * NOUT : NOUT;     // MMA N
  static constexpr int CH = CIN / CSPLIT;              // channels of one stage
  static constexpr bool PAR = FUSE == kFusePool;       // operand split by input row parity
  static constexpr int NPAR = PAR ? 2 : 1;
  static constexpr int PW = PAR ? W + 2 : W + 1;       // padded row pitch (positions)
  static constexpr int ROWS = TH + 2;                  // input rows per tile
  static constexpr int MROWS = PAR ? TH / 2 : TH;      // GEMM rows of pixels per tile
  static constexpr int MB = (MROWS * PW + 127) / 128;  // 128-row M blocks per tile
  static constexpr int NPOS0 = MB * 128 + (PAR ? PW : 2 * PW) + 2;  // positions any tap reads
  // planes start one 16-byte bank group apart (NPOS = 1 mod 8)
  static constexpr int NPOS = ((NPOS0 + 7) / 8) * 8 + 1;
  static constexpr uint32_t PLANE = NPOS * 16;  // bytes of one 4-channel plane
  static constexpr int NPL = CIN / 4;            // weight planes (every channel)
  static constexpr int NPLS = CH / 4;            // operand planes of one stage
  static constexpr uint32_t A_COPY = NPLS * NPAR * PLANE;
  static constexpr uint32_t A_STAGE = align1k(A_COPY * (SPLIT_A ? 2 : 1));
  // kFuseUnpool: the raw stage holds pooled rows: values, then codes
  static constexpr int PROWS = TH / 2 + 2;
  static constexpr uint32_t RAW_F32 = FUSE == kFuseUnpool ? CH * PROWS * (W / 2) * 4 : CH * ROWS * W * 4;
  static constexpr uint32_t RAW_CODES = FUSE == kFuseUnpool ? CH * PROWS * (W / 2) : 0;
  static constexpr uint32_t RAW_BYTES = RAW_F32 + RAW_CODES;
  static constexpr uint32_t RAW_CODE_OFF = align1k(RAW_F32);
  static constexpr uint32_t RAW_STAGE = align1k(RAW_CODE_OFF + RAW_CODES);
  static constexpr uint32_t BPLANE = NB * 16;
  static constexpr uint32_t W_COPY = 9 * NPL * BPLANE;
  static constexpr uint32_t W_REGION = align1k(W_COPY * (SPLIT_W ? 2 : 1));
  static constexpr uint32_t OFF_RAW = W_REGION;
  static constexpr uint32_t OFF_A = OFF_RAW + RAW_ST * RAW_STAGE;
  static constexpr size_t SMEM = (size_t)OFF_A + A_ST * A_STAGE + 1024;
  static constexpr int ACC_COLS = MB * NPAR * NB;  // TMEM columns of one accumulator
  static constexpr int ITEMS = NPLS * ROWS * (W / 4);
  static constexpr int KSTEPS = CH / 8;  // K steps of one stage
  static_assert(CIN % CSPLIT == 0 && CH % 8 == 0 && W % 16 == 0 && (NOUT == 16 || NOUT == 32), "shape");
  static_assert((CG == 8 || CG == 16 || CG == 32) && (NOUT == CG || NOUT == 2 * CG), "channel groups");
  static_assert(FUSE == kFuseNone || (TH % 2 == 0 && W % 32 == 0), "pooled rows are 16-byte TMA boxes");
  static_assert(!PAR || PW % 2 == 0, "pool partners share a lane pair");
  static_assert(2 * ACC_COLS <= 512, "two accumulators fit TMEM");
  static_assert(SMEM <= 232448, "shared memory per block");
  static_assert(ROWS <= 256 && W <= 256 && CH <= 256, "TMA box dims");
  static_assert(NPAR * PLANE / 16 < 16384 && BPLANE / 16 < 16384, "descriptor offsets");
};

struct ConvTCParams {
  const float *w;
  const float *bias;
  float *y;         // output, NCHW [N][COUT][H][W] (kFusePool: pooled [N][COUT][H/2][W/2])
  uint8_t *codes;   // kFusePool: pool codes, same shape as the pooled output
  int N, H, COUT;
  int mode;  // 0: forward, w is [COUT][CIN][3][3]; 1: input gradient, w is [CIN][COUT][3][3] (forward weights)
  int tiles_per_img;
  int *err;
  // output channels co0 .. co0 + COUT - 1 of ctot (0: COUT, one group): a
  // layer with more than 32 output channels runs one launch per group
  int co0, ctot;
};

// warp roles
// 16 warps, four per SM sub-partition: up to 128 registers a thread
constexpr int kConvThreads = 512;
constexpr int kEpiWarp0 = 2, kEpiWarps = 8;
constexpr int kTransformWarp0 = kEpiWarp0 + kEpiWarps, kTransformWarps = 6;
constexpr int kTransformThreads = kTransformWarps * 32;

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(addr)
               : "memory");
  return v;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ float tf32_hi(float v) { return __uint_as_float(__float_as_uint(v) & 0xFFFFE000u); }

// (x, y, z, w) rotated left by r in 0..3
__device__ __forceinline__ float4 rotl4(float4 v, int r) {
  if (r & 1) v = make_float4(v.y, v.z, v.w, v.x);
  if (r & 2) v = make_float4(v.z, v.w, v.x, v.y);
  return v;
}

__device__ __forceinline__ float comp(const float4 &v, int j) {
  return j == 0 ? v.x : j == 1 ? v.y : j == 2 ? v.z : v.w;
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 8 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld_32x32b_x8(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr)
               : "memory");
}

template <int CG>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[CG]) {
  if constexpr (CG == 32) tc::tmem_ld_32x32b_x32(taddr, r);
  else if constexpr (CG == 16) tmem_ld_32x32b_x16(taddr, r);
  else tmem_ld_32x32b_x8(taddr, r);
}

// K-major interleaved (SWIZZLE_NONE) operand: 8-row groups 128 B apart
// (SBO), the two 4-element K chunks of one MMA `lbo` bytes apart.
__device__ __forceinline__ uint64_t desc_interleaved(uint32_t saddr, uint32_t lbo) {
  return tc::smem_desc(saddr, lbo, 128, 0);
}

template <int CIN, int W, int TH, int NOUT, int PREC, int RAW_ST, int A_ST, int CG, int FUSE, int CSPLIT>
__global__ void __launch_bounds__(kConvThreads, 1)
    conv3x3_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmx2,
                      ConvTCParams p) {
  // tmx: input rows (kFuseUnpool: pooled gradient values), tmx2: their pool
  // codes (kFuseUnpool only)
  using Cf = ConvCfg<CIN, W, TH, NOUT, PREC, RAW_ST, A_ST, CG, FUSE, CSPLIT>;
  constexpr bool SPLIT_A = Cf::SPLIT_A, SPLIT_W = Cf::SPLIT_W, STACKED = Cf::STACKED;
  constexpr int NB = Cf::NB;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  __shared__ __align__(8) uint64_t rfull[RAW_ST], rempty[RAW_ST], afull[A_ST], aempty[A_ST], tfull[2], tempty[2],
      drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ float bias_s[32];

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t s_base = tc::smem_u32(smem);
  if (threadIdx.x == 0) {
    for (int s = 0; s < RAW_ST; ++s) {
      tc::mbar_init(&rfull[s], 1);
      tc::mbar_init(&rempty[s], kTransformWarps);
    }
    for (int s = 0; s < A_ST; ++s) {
      tc::mbar_init(&afull[s], kTransformWarps);
      tc::mbar_init(&aempty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], kEpiWarps);
    }
    tc::mbar_init(&drain, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  const int ctot = p.ctot > 0 ? p.ctot : p.COUT;
  if (threadIdx.x < 32)
    bias_s[threadIdx.x] = (p.bias && (int)threadIdx.x < p.COUT) ? p.bias[p.co0 + threadIdx.x] : 0.0f;
  // Operand stages start all zero: pad columns and the tail past the last
  // row are never written again.
  for (uint32_t off = threadIdx.x * 16; off < A_ST * Cf::A_STAGE; off += kConvThreads * 16)
    st_shared_v4(s_base + Cf::OFF_A + off, 0.f, 0.f, 0.f, 0.f);
  // Resident weights: plane (tap, ci/4), row co, 16 bytes of 4 input channels.
  for (int idx = threadIdx.x; idx < 9 * CIN * NOUT; idx += kConvThreads) {
    const int co = idx % NOUT, ci = (idx / NOUT) % CIN, tap = idx / (NOUT * CIN);
    const int r = tap / 3, s = tap % 3;
    float v = 0.0f;
    if (co < p.COUT)
      v = p.mode == 0 ? __ldg(p.w + (((p.co0 + co) * CIN + ci) * 3 + r) * 3 + s)
                      : __ldg(p.w + ((ci * ctot + p.co0 + co) * 3 + (2 - r)) * 3 + (2 - s));
    const uint32_t off = (uint32_t)(tap * Cf::NPL + (ci >> 2)) * Cf::BPLANE + co * 16 + (ci & 3) * 4;
    if (SPLIT_W) {
      const float h = tf32_hi(v);
      *reinterpret_cast<float *>(smem + off) = h;
      *reinterpret_cast<float *>(smem + Cf::W_COPY + off) = __fsub_rn(v, h);
    } else if (STACKED) {
      // hi in row co, lo in row NOUT + co of the same plane
      const float h = tf32_hi(v);
      *reinterpret_cast<float *>(smem + off) = h;
      *reinterpret_cast<float *>(smem + off + NOUT * 16) = __fsub_rn(v, h);
    } else {
      *reinterpret_cast<float *>(smem + off) = v;
    }
  }
  fence_proxy_async_smem();
  if (warp == 1) tc::tmem_alloc(&tmem_base, 512);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  const int ntiles = p.N * p.tiles_per_img;
  volatile int *abort_v = &abort_flag;

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------- TMA producer
      tc::prefetch_tmap(&tmx);
      int it = 0;
      int issued = 0;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x) {
        const int n = t / p.tiles_per_img, h0 = (t % p.tiles_per_img) * TH;
        for (int cs = 0; cs < CSPLIT; ++cs, ++it) {
          const int st = it % RAW_ST;
          const uint32_t ph = (it / RAW_ST) & 1;
          if (!tc::mbar_wait(&rempty[st], ph ^ 1, abort_v, p.err, 201)) goto producer_done;
          uint8_t *raw = smem + Cf::OFF_RAW + st * Cf::RAW_STAGE;
          const int c0 = n * CIN + cs * Cf::CH;
          tc::mbar_arrive_expect_tx(&rfull[st], Cf::RAW_BYTES);
          if (FUSE == kFuseUnpool) {
            // pooled rows h0/2 - 1 .. h0/2 + TH/2 cover input rows h0 - 1 .. h0 + TH
            tc::tma_load_3d(&tmx, &rfull[st], raw, 0, h0 / 2 - 1, c0);
            tc::tma_load_3d(&tmx2, &rfull[st], raw + Cf::RAW_CODE_OFF, 0, h0 / 2 - 1, c0);
          } else {
            tc::tma_load_3d(&tmx, &rfull[st], raw, 0, h0 - 1, c0);
          }
          ++issued;
        }
      }
    producer_done:
      // Do not leave while a TMA copy may still write this CTA's shared
      // memory: wait (bounded) for the last RAW_ST loads to land.
      for (int j = issued > RAW_ST ? issued - RAW_ST : 0; j < issued; ++j) {
        const long long t0 = clock64();
        while (!tc::mbar_test(&rfull[j % RAW_ST], (j / RAW_ST) & 1) && clock64() - t0 < tc::kWaitCycles) {
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ------------------------------------------------------ MMA issue
      const uint32_t idesc = tc::idesc_tf32(128, NB, 0, 0);
      // stacked 3xTF32: the second MMA (activation lo x weight hi) reads
      // the weight operand's first NOUT rows only
      const uint32_t idesc_hi_rows = tc::idesc_tf32(128, NOUT, 0, 0);
      // Descriptors are built once; an operand at byte offset o from a base
      // is the base descriptor plus o >> 4 (start-address field, no carry:
      // shared-memory addresses are below 2^18).
      const uint64_t bd_hi = desc_interleaved(s_base, Cf::BPLANE);
      const uint64_t bd_lo = desc_interleaved(s_base + Cf::W_COPY, Cf::BPLANE);
      int it = 0, ti = 0;
      bool issued = false;
      for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++ti) {
        const int acc = ti & 1;
        const uint32_t aph = (ti >> 1) & 1;
        // 128-row blocks that hold rows of this tile: the image's last tile
        // may have fewer rows (the epilogue stores none of the others)
        const int rows_here = min(TH, p.H - (t % p.tiles_per_img) * TH);
        const int mb_n = min(Cf::MB, ((Cf::PAR ? (rows_here + 1) / 2 : rows_here) * Cf::PW + 127) / 128);
        for (int cs = 0; cs < CSPLIT; ++cs, ++it) {
        const int st = it % A_ST;
        const uint32_t ph = (it / A_ST) & 1;
        if (!tc::mbar_wait(&afull[st], ph, abort_v, p.err, 202)) goto mma_done;
        if (cs == 0 && !tc::mbar_wait(&tempty[acc], aph ^ 1, abort_v, p.err, 203)) goto mma_done;
        tc::fence_after_sync();
        const uint32_t a_hi = s_base + Cf::OFF_A + st * Cf::A_STAGE;
        // the two 4-channel K chunks of one MMA are NPAR planes apart
        const uint64_t ad_hi0 = desc_interleaved(a_hi, Cf::NPAR * Cf::PLANE);
        const uint64_t ad_lo0 = desc_interleaved(a_hi + Cf::A_COPY, Cf::NPAR * Cf::PLANE);
#pragma unroll 1
        for (int mb = 0; mb < mb_n; ++mb) {
          const uint64_t ad_hi = ad_hi0 + (uint64_t)(mb * 128), ad_lo = ad_lo0 + (uint64_t)(mb * 128);
#pragma unroll
          for (int a = 0; a < Cf::NPAR; ++a) {
            // accumulator of conv rows with parity a (one block of NB columns each)
            const uint32_t d = tbase + acc * Cf::ACC_COLS + (mb * Cf::NPAR + a) * NB;
#pragma unroll
            for (int tap = 0; tap < 9; ++tap) {
              const int r = tap / 3, sc = tap % 3;
              // plane parity and row offset of the tap's input rows
              const int pp = Cf::PAR ? (a + r) & 1 : 0, ro = Cf::PAR ? (a + r) >> 1 : r;
#pragma unroll
              for (int kk = 0; kk < Cf::KSTEPS; ++kk) {
                // operand rows start (ro * PW + sc) positions into plane (4-channel group 2kk, parity pp)
                const uint32_t a_off =
                    (uint32_t)((ro * Cf::PW + sc) * 16 + (2 * kk * Cf::NPAR + pp) * Cf::PLANE) >> 4;
                const uint32_t b_off = ((uint32_t)(tap * Cf::NPL + cs * Cf::NPLS + 2 * kk) * Cf::BPLANE) >> 4;
                tc::mma_tf32(d, ad_hi + a_off, bd_hi + b_off, idesc, (cs | tap | kk) != 0);
                if (PREC == 3) tc::mma_tf32(d, ad_lo + a_off, bd_hi + b_off, idesc_hi_rows, 1);
                if (SPLIT_W) {
                  tc::mma_tf32(d, ad_hi + a_off, bd_lo + b_off, idesc, 1);
                  tc::mma_tf32(d, ad_lo + a_off, bd_hi + b_off, idesc, 1);
                }
              }
            }
          }
        }
        issued = true;
        tc::mma_commit(&aempty[st]);
        if (cs == CSPLIT - 1) tc::mma_commit(&tfull[acc]);
        }
      }
    mma_done:
      if (issued) {
        tc::mma_commit(&drain);
        const long long t0 = clock64();
        while (!tc::mbar_test(&drain, 0) && clock64() - t0 < tc::kWaitCycles) {
        }
      }
    }
  } else if (warp < kTransformWarp0) {
    // ------------------------------------------------------------ epilogue
    // Per M block and group of CG channels: TMEM -> registers, + bias, and
    // straight to global memory.  Lane m of the block is GEMM row m: pixel
    // (i, w) = (m / PW, m % PW) of the tile (kFusePool: pooled row i, conv
    // rows 2i and 2i + 1 in the two parity accumulators); rows with w >= W
    // or past the image are discarded.
    const int q = warp & 3;  // TMEM lane quarter this warp may read
    const uint32_t tq = (uint32_t)(q * 32) << 16;
    const long long plane_px = Cf::PAR ? (long long)(p.H / 2) * (W / 2) : (long long)p.H * W;
    // the two warps of a lane quarter: with two channel groups each takes
    // one group (all M blocks), with one group they alternate M blocks
    constexpr int NCG = NOUT / CG;
    const int half = (warp - kEpiWarp0) >> 2;
    const int cg = NCG == 2 ? half : 0;
    const int mb0 = NCG == 2 ? 0 : half, mbs = NCG == 2 ? 1 : 2;
    const bool active = cg * CG < p.COUT;
    float bias_r[CG];
#pragma unroll
    for (int c = 0; c < CG; ++c) bias_r[c] = bias_s[cg * CG + c];
    int it = 0;
    for (int t = blockIdx.x; t < ntiles; t += gridDim.x, ++it) {
      const int acc = it & 1;
      const uint32_t aph = (it >> 1) & 1;
      if (!tc::mbar_wait(&tfull[acc], aph, abort_v, p.err, 204)) break;
      tc::fence_after_sync();
      const int n = t / p.tiles_per_img, h0 = (t % p.tiles_per_img) * TH;
      const uint32_t tacc = tbase + acc * Cf::ACC_COLS + tq + cg * CG;
#pragma unroll 1
      for (int mb = mb0; mb < Cf::MB && active; mb += mbs) {
        const int m = mb * 128 + q * 32 + lane;
        const int i = m / Cf::PW, col = m % Cf::PW;
        if constexpr (Cf::PAR) {
          // ReLU + 2x2 max-pool; window order (0,0) (0,1) (1,0) (1,1), the
          // first maximum wins, code 255 when the maximum is not positive.
          // The even-column lane of each pair stores.  H is even, so conv
          // row 2i + 1 exists whenever row 2i does.
          const bool store = col < W && !(col & 1) && i < TH / 2 && h0 + 2 * i < p.H;
          const long long o = ((long long)n * ctot + p.co0 + cg * CG) * plane_px + (long long)(h0 / 2 + i) * (W / 2) +
                              col / 2;
          uint32_t top[CG], bot[CG];
          tmem_ld_cols<CG>(tacc + (mb * 2 + 0) * NB, top);
          tmem_ld_cols<CG>(tacc + (mb * 2 + 1) * NB, bot);
          if constexpr (STACKED) {
            uint32_t tl[CG], bl[CG];
            tmem_ld_cols<CG>(tacc + (mb * 2 + 0) * NB + NOUT, tl);
            tmem_ld_cols<CG>(tacc + (mb * 2 + 1) * NB + NOUT, bl);
            tc::tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < CG; ++c) {
              top[c] = __float_as_uint(__fadd_rn(__uint_as_float(top[c]), __uint_as_float(tl[c])));
              bot[c] = __float_as_uint(__fadd_rn(__uint_as_float(bot[c]), __uint_as_float(bl[c])));
            }
          }
          tc::tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < CG; ++c) {
            const float v0 = __fadd_rn(__uint_as_float(top[c]), bias_r[c]);
            const float v2 = __fadd_rn(__uint_as_float(bot[c]), bias_r[c]);
            const float v1 = __shfl_xor_sync(0xffffffffu, v0, 1);
            const float v3 = __shfl_xor_sync(0xffffffffu, v2, 1);
            if (store && cg * CG + c < p.COUT) {
              float mx = v0;
              uint32_t idx = 0;
              if (v1 > mx) mx = v1, idx = 1;
              if (v2 > mx) mx = v2, idx = 2;
              if (v3 > mx) mx = v3, idx = 3;
              p.y[o + c * plane_px] = mx > 0.0f ? mx : 0.0f;
              p.codes[o + c * plane_px] = mx > 0.0f ? (uint8_t)idx : kNoGradCode;
            }
          }
        } else {
          const bool store = col < W && i < TH && h0 + i < p.H;
          const long long o = ((long long)n * ctot + p.co0 + cg * CG) * plane_px + (long long)(h0 + i) * W + col;
          uint32_t r[CG];
          tmem_ld_cols<CG>(tacc + mb * NB, r);
          if constexpr (STACKED) {
            uint32_t rl[CG];
            tmem_ld_cols<CG>(tacc + mb * NB + NOUT, rl);
            tc::tmem_ld_wait();
#pragma unroll
            for (int c = 0; c < CG; ++c) r[c] = __float_as_uint(__fadd_rn(__uint_as_float(r[c]), __uint_as_float(rl[c])));
          }
          tc::tmem_ld_wait();
#pragma unroll
          for (int c = 0; c < CG; ++c)
            if (store && cg * CG + c < p.COUT) p.y[o + c * plane_px] = __fadd_rn(__uint_as_float(r[c]), bias_r[c]);
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[acc]);
    }
  } else {
    // ----------------------------------------------------------- transform
    // Item (plane c4, row j, pixel quad qd): four 16-byte reads (channels
    // 4c4..4c4+3 of pixels 4qd..4qd+3, consecutive lanes take consecutive
    // quads: conflict-free), a 4x4 transpose in registers, four 16-byte
    // writes (one pixel's 4 channels each).  Each lane writes its pixels in
    // an order rotated by (qd / 2) % 4 so the 8 lanes of a shared-memory
    // phase hit 8 different 16-byte bank groups.
    const int tt = threadIdx.x - kTransformWarp0 * 32;
    const int nsub = ((ntiles - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x) * CSPLIT;
    for (int it = 0; it < nsub; ++it) {
      const int rs = it % RAW_ST, as = it % A_ST;
      const uint32_t rph = (it / RAW_ST) & 1, aph = (it / A_ST) & 1;
      if (!tc::mbar_wait(&rfull[rs], rph, abort_v, p.err, 205)) break;
      if (!tc::mbar_wait(&aempty[as], aph ^ 1, abort_v, p.err, 206)) break;
      const uint32_t raw = s_base + Cf::OFF_RAW + rs * Cf::RAW_STAGE;
      const uint32_t a_hi = s_base + Cf::OFF_A + as * Cf::A_STAGE;
#pragma unroll 1
      for (int item = tt; item < Cf::ITEMS; item += kTransformThreads) {
        const int qd = item % (W / 4), j = (item / (W / 4)) % Cf::ROWS, c4 = item / ((W / 4) * Cf::ROWS);
        const int rot = (qd >> 1) & 3;
        float4 v[4];
        if (FUSE == kFuseUnpool) {
          // input row h0 - 1 + j sits in pooled row (j + 1) / 2 of the stage
          // with row parity (j + 1) & 1; pixels 4qd .. 4qd+3 in pooled
          // columns 2qd, 2qd + 1.  The pooled gradient goes to the recorded
          // window element, the others get 0.
          const int pj = (j + 1) >> 1, hp = ((j + 1) & 1) * 2;
#pragma unroll
          for (int ci = 0; ci < 4; ++ci) {
            const uint32_t e = (uint32_t)(((4 * c4 + ci) * Cf::PROWS + pj) * (W / 2) + 2 * qd);
            float2 g;
            uint32_t cw;
            asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(g.x), "=f"(g.y) : "r"(raw + e * 4) : "memory");
            asm volatile("ld.shared.u16 %0, [%1];" : "=r"(cw) : "r"(raw + Cf::RAW_CODE_OFF + e) : "memory");
            const uint32_t c0 = cw & 0xFF, c1 = (cw >> 8) & 0xFF;
            v[ci] = rotl4(make_float4(c0 == (uint32_t)hp ? g.x : 0.0f, c0 == (uint32_t)(hp + 1) ? g.x : 0.0f,
                                      c1 == (uint32_t)hp ? g.y : 0.0f, c1 == (uint32_t)(hp + 1) ? g.y : 0.0f),
                          rot);
          }
        } else {
#pragma unroll
          for (int ci = 0; ci < 4; ++ci)
            v[ci] = rotl4(ld_shared_v4(raw + (uint32_t)(((4 * c4 + ci) * Cf::ROWS + j) * W + 4 * qd) * 4), rot);
        }
        // padded row j: row j of plane c4, or (row-parity split) row j / 2
        // of plane (c4, j % 2)
        const uint32_t row0 = (uint32_t)(c4 * Cf::NPAR + (Cf::PAR ? (j & 1) : 0)) * Cf::PLANE +
                              (uint32_t)((Cf::PAR ? j >> 1 : j) * Cf::PW + 1 + 4 * qd) * 16;
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          const uint32_t dst = a_hi + row0 + (uint32_t)((jj + rot) & 3) * 16;
          const float x0 = comp(v[0], jj), x1 = comp(v[1], jj), x2 = comp(v[2], jj), x3 = comp(v[3], jj);
          if (SPLIT_A) {
            const float h0 = tf32_hi(x0), h1 = tf32_hi(x1), h2 = tf32_hi(x2), h3 = tf32_hi(x3);
            st_shared_v4(dst, h0, h1, h2, h3);
            st_shared_v4(dst + Cf::A_COPY, __fsub_rn(x0, h0), __fsub_rn(x1, h1), __fsub_rn(x2, h2),
                         __fsub_rn(x3, h3));
          } else {
            st_shared_v4(dst, x0, x1, x2, x3);
          }
        }
      }
      fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) {
        tc::mbar_arrive(&afull[as]);
        tc::mbar_arrive(&rempty[rs]);
      }
    }
  }
  __syncthreads();
  if (warp == 1) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, 512);
  }
}

// Tiled TMA view of an NCHW activation as {W, H, N*C} (innermost first),
// box {W, box_rows, box_ch}; f32, or u8 for pool codes.
int encode_activation(const void *x, int N, int C, int H, int W, int box_rows, int box_ch, CUtensorMap *map,
                      bool codes = false) {
  auto fn = tensor_map_encoder();
  if (!fn) return fail(REMORA_ERR_CUDA, "conv: cuTensorMapEncodeTiled is not available from the driver");
  const cuuint64_t es = codes ? 1 : 4;
  cuuint64_t dims[3] = {(cuuint64_t)W, (cuuint64_t)H, (cuuint64_t)N * C};
  cuuint64_t strides[2] = {(cuuint64_t)W * es, (cuuint64_t)H * W * es};
  cuuint32_t box[3] = {(cuuint32_t)W, (cuuint32_t)box_rows, (cuuint32_t)box_ch};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, codes ? CU_TENSOR_MAP_DATA_TYPE_UINT8 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3,
                  const_cast<void *>(x), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(REMORA_ERR_CUDA, "conv: cuTensorMapEncodeTiled failed (%d)", (int)r);
  return REMORA_OK;
}

// Operands of one launch: x (kFuseUnpool: the pooled gradient) and its
// codes; y (kFusePool: the pooled output) and its codes.
struct ConvIO {
  const float *x;
  const uint8_t *x_codes;
  float *y;
  uint8_t *y_codes;
};

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

template <int CIN, int W, int TH, int NOUT, int PREC, int RAW_ST, int A_ST, int CG, int FUSE = kFuseNone,
          int CSPLIT = 1>
int launch_conv(const ConvIO &io, const ConvTCParams &p, int sm_count, cudaStream_t stream, bool *handled) {
  using Cf = ConvCfg<CIN, W, TH, NOUT, PREC, RAW_ST, A_ST, CG, FUSE, CSPLIT>;
  if (!aligned16(io.x) || (FUSE == kFuseUnpool && !aligned16(io.x_codes)) ||
      (reinterpret_cast<uintptr_t>(io.y) & 3)) {
    *handled = false;  // TMA cannot address the input, or the output is not f32-aligned
    return REMORA_OK;
  }
  auto kern = conv3x3_tc_kernel<CIN, W, TH, NOUT, PREC, RAW_ST, A_ST, CG, FUSE, CSPLIT>;
  static bool attr = false;
  if (!attr) {
    REMORA_CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Cf::SMEM));
    attr = true;
  }
  CUtensorMap mx, mx2;
  if (FUSE == kFuseUnpool) {
    REMORA_TRY(encode_activation(io.x, p.N, CIN, p.H / 2, W / 2, Cf::PROWS, Cf::CH, &mx));
    REMORA_TRY(encode_activation(io.x_codes, p.N, CIN, p.H / 2, W / 2, Cf::PROWS, Cf::CH, &mx2, true));
  } else {
    REMORA_TRY(encode_activation(io.x, p.N, CIN, p.H, W, Cf::ROWS, Cf::CH, &mx));
    mx2 = mx;
  }
  ConvTCParams q = p;
  q.y = io.y;
  q.codes = io.y_codes;
  q.tiles_per_img = (p.H + TH - 1) / TH;
  const int ntiles = p.N * q.tiles_per_img;
  const int grid = std::min(ntiles, sm_count);
  note_launch();
  kern<<<grid, kConvThreads, Cf::SMEM, stream>>>(mx, mx2, q);
  REMORA_CUDA_TRY(cudaGetLastError());
  *handled = true;
  return REMORA_OK;
}

using ConvLauncher = int (*)(const ConvIO &, const ConvTCParams &, int, cudaStream_t, bool *);

// The instantiation for (input channels, width, output channels of a group
// (16: at most 16, 32: at most 32), precision 0 TF32 / 1 3xTF32 / 2 2xTF32),
// or null.  Tile rows, stages and channel slices per shape: the largest
// share of useful GEMM rows (rows of PW = W + 1 positions in 128-row blocks)
// over the image's ragged last tile that fits shared memory and two TMEM
// accumulators; the 16 -> 32 channel 3xTF32 forward on 32-wide images (the
// crater CNN's conv2) runs the stacked-weight form.
#define REMORA_UNPAREN(...) __VA_ARGS__
#define C(ci, wd, no, pr, args) \
  if (cin == ci && width == wd && nout == no && prec == pr) return &launch_conv<REMORA_UNPAREN args>;
ConvLauncher pick(int cin, int width, int nout, int prec) {
  C(16, 16, 16, 0, (16, 16, 6, 16, 0, 2, 2, 8, kFuseNone, 1))
  C(16, 16, 16, 1, (16, 16, 6, 16, 1, 2, 2, 8, kFuseNone, 1))
  C(16, 16, 16, 2, (16, 16, 6, 16, 2, 2, 2, 8, kFuseNone, 1))
  C(16, 16, 32, 0, (16, 16, 6, 32, 0, 2, 2, 16, kFuseNone, 1))
  C(16, 16, 32, 1, (16, 16, 6, 32, 1, 2, 2, 16, kFuseNone, 1))
  C(16, 16, 32, 2, (16, 16, 6, 32, 2, 2, 2, 16, kFuseNone, 1))
  C(16, 32, 16, 0, (16, 32, 32, 16, 0, 2, 1, 8, kFuseNone, 1))
  C(16, 32, 16, 1, (16, 32, 16, 16, 1, 2, 1, 8, kFuseNone, 1))
  C(16, 32, 16, 2, (16, 32, 16, 16, 2, 2, 2, 8, kFuseNone, 1))
  C(16, 32, 32, 0, (16, 32, 16, 32, 0, 2, 2, 16, kFuseNone, 1))
  C(16, 32, 32, 1, (16, 32, 14, 32, 3, 2, 1, 16, kFuseNone, 1))
  C(16, 32, 32, 2, (16, 32, 8, 32, 2, 2, 2, 16, kFuseNone, 1))
  C(16, 64, 16, 0, (16, 64, 8, 16, 0, 2, 2, 8, kFuseNone, 1))
  C(16, 64, 16, 1, (16, 64, 8, 16, 1, 2, 1, 8, kFuseNone, 1))
  C(16, 64, 16, 2, (16, 64, 8, 16, 2, 2, 2, 8, kFuseNone, 1))
  C(16, 64, 32, 0, (16, 64, 8, 32, 0, 2, 2, 16, kFuseNone, 1))
  C(16, 64, 32, 1, (16, 64, 8, 32, 1, 2, 1, 16, kFuseNone, 1))
  C(16, 64, 32, 2, (16, 64, 4, 32, 2, 2, 2, 16, kFuseNone, 1))
  C(16, 128, 16, 0, (16, 128, 4, 16, 0, 2, 2, 8, kFuseNone, 1))
  C(16, 128, 16, 1, (16, 128, 4, 16, 1, 1, 1, 8, kFuseNone, 1))
  C(16, 128, 16, 2, (16, 128, 6, 16, 2, 2, 1, 8, kFuseNone, 1))
  C(16, 128, 32, 0, (16, 128, 6, 32, 0, 2, 1, 16, kFuseNone, 1))
  C(16, 128, 32, 1, (16, 128, 4, 32, 1, 1, 1, 16, kFuseNone, 1))
  C(16, 128, 32, 2, (16, 128, 2, 32, 2, 2, 2, 16, kFuseNone, 1))
  C(32, 16, 16, 0, (32, 16, 6, 16, 0, 2, 2, 8, kFuseNone, 2))
  C(32, 16, 16, 1, (32, 16, 6, 16, 1, 2, 2, 8, kFuseNone, 2))
  C(32, 16, 16, 2, (32, 16, 6, 16, 2, 2, 2, 8, kFuseNone, 2))
  C(32, 16, 32, 0, (32, 16, 6, 32, 0, 2, 2, 16, kFuseNone, 2))
  C(32, 16, 32, 1, (32, 16, 6, 32, 1, 2, 2, 16, kFuseNone, 2))
  C(32, 16, 32, 2, (32, 16, 6, 32, 2, 2, 2, 16, kFuseNone, 2))
  C(32, 32, 16, 0, (32, 32, 16, 16, 0, 2, 2, 8, kFuseNone, 2))
  C(32, 32, 16, 1, (32, 32, 16, 16, 3, 2, 1, 8, kFuseNone, 2))
  C(32, 32, 16, 2, (32, 32, 16, 16, 2, 2, 2, 8, kFuseNone, 2))
  C(32, 32, 32, 0, (32, 32, 16, 32, 0, 2, 2, 16, kFuseNone, 2))
  C(32, 32, 32, 1, (32, 32, 16, 32, 1, 1, 1, 16, kFuseNone, 2))
  C(32, 32, 32, 2, (32, 32, 6, 32, 2, 2, 2, 16, kFuseNone, 2))
  C(32, 64, 16, 0, (32, 64, 8, 16, 0, 2, 2, 8, kFuseNone, 2))
  C(32, 64, 16, 1, (32, 64, 4, 16, 1, 2, 2, 8, kFuseNone, 2))
  C(32, 64, 16, 2, (32, 64, 8, 16, 2, 2, 2, 8, kFuseNone, 2))
  C(32, 64, 32, 0, (32, 64, 8, 32, 0, 2, 2, 16, kFuseNone, 2))
  C(32, 64, 32, 1, (32, 64, 8, 32, 1, 1, 1, 16, kFuseNone, 2))
  C(32, 64, 32, 2, (32, 64, 6, 32, 2, 2, 2, 16, kFuseNone, 2))
  C(32, 128, 16, 0, (32, 128, 8, 16, 0, 1, 1, 8, kFuseNone, 2))
  C(32, 128, 16, 1, (32, 128, 4, 16, 1, 1, 1, 8, kFuseNone, 2))
  C(32, 128, 16, 2, (32, 128, 4, 16, 2, 2, 1, 8, kFuseNone, 2))
  C(32, 128, 32, 0, (32, 128, 4, 32, 0, 2, 1, 16, kFuseNone, 2))
  C(32, 128, 32, 1, (32, 128, 2, 32, 1, 2, 1, 16, kFuseNone, 2))
  C(32, 128, 32, 2, (32, 128, 2, 32, 2, 2, 2, 16, kFuseNone, 2))
  C(64, 16, 16, 0, (64, 16, 6, 16, 0, 2, 2, 8, kFuseNone, 4))
  C(64, 16, 16, 1, (64, 16, 6, 16, 1, 2, 2, 8, kFuseNone, 4))
  C(64, 16, 16, 2, (64, 16, 6, 16, 2, 2, 2, 8, kFuseNone, 4))
  C(64, 16, 32, 0, (64, 16, 6, 32, 0, 2, 2, 16, kFuseNone, 4))
  C(64, 16, 32, 1, (64, 16, 6, 32, 1, 2, 2, 16, kFuseNone, 4))
  C(64, 16, 32, 2, (64, 16, 6, 32, 2, 2, 2, 16, kFuseNone, 4))
  C(64, 32, 16, 0, (64, 32, 16, 16, 0, 2, 2, 8, kFuseNone, 4))
  C(64, 32, 16, 1, (64, 32, 16, 16, 1, 1, 1, 8, kFuseNone, 4))
  C(64, 32, 16, 2, (64, 32, 16, 16, 2, 2, 1, 8, kFuseNone, 4))
  C(64, 32, 32, 0, (64, 32, 16, 32, 0, 2, 1, 16, kFuseNone, 4))
  C(64, 32, 32, 1, (64, 32, 6, 32, 1, 2, 1, 16, kFuseNone, 4))
  C(64, 32, 32, 2, (64, 32, 6, 32, 2, 2, 2, 16, kFuseNone, 4))
  C(64, 64, 16, 0, (64, 64, 8, 16, 0, 2, 2, 8, kFuseNone, 4))
  C(64, 64, 16, 1, (64, 64, 8, 16, 1, 1, 1, 8, kFuseNone, 4))
  C(64, 64, 16, 2, (64, 64, 8, 16, 2, 2, 1, 8, kFuseNone, 4))
  C(64, 64, 32, 0, (64, 64, 8, 32, 0, 2, 1, 16, kFuseNone, 4))
  C(64, 64, 32, 1, (64, 64, 1, 32, 1, 2, 1, 16, kFuseNone, 4))
  C(64, 64, 32, 2, (64, 64, 6, 32, 2, 1, 1, 16, kFuseNone, 4))
  C(64, 128, 16, 0, (64, 128, 8, 16, 0, 1, 1, 8, kFuseNone, 4))
  C(64, 128, 16, 1, (64, 128, 2, 16, 1, 2, 1, 8, kFuseNone, 4))
  C(64, 128, 16, 2, (64, 128, 4, 16, 2, 2, 1, 8, kFuseNone, 4))
  C(64, 128, 32, 0, (64, 128, 4, 32, 0, 2, 1, 16, kFuseNone, 4))
  C(64, 128, 32, 2, (64, 128, 2, 32, 2, 1, 1, 16, kFuseNone, 4))
  return nullptr;
}
#undef C
#undef REMORA_UNPAREN

// One launch per group of at most 32 output channels (groups of equal
// size); *handled = false (the direct kernels run instead) if no
// instantiation exists, if TMA cannot address the operands, or for fewer
// than 8 output channels.
int dispatch(const ConvIO &io, ConvTCParams p, int cin, int width, int prec, int sm_count, cudaStream_t stream,
             bool *handled) {
  *handled = false;
  const int total = p.COUT;
  // fewer than 8 output channels would leave most of an N = 16 MMA empty:
  // the direct kernels (exact f32 order) take those
  if (total < 8) return REMORA_OK;
  const int ng = (total + 31) / 32, gs = (total + ng - 1) / ng;
  const ConvLauncher launch = pick(cin, width, gs <= 16 ? 16 : 32, prec);
  if (launch == nullptr) return REMORA_OK;
  p.ctot = total;
  for (int co0 = 0; co0 < total; co0 += gs) {
    p.co0 = co0;
    p.COUT = std::min(gs, total - co0);
    REMORA_TRY(launch(io, p, sm_count, stream, handled));
    if (!*handled) return REMORA_OK;  // only the first group can decline (alignment)
  }
  return REMORA_OK;
}

// The fused forms of the crater CNN's second layer (16 -> 32 channels on
// 32 x 32 images and its input gradient).
int dispatch_pool(const ConvIO &io, const ConvTCParams &p, int cin, int width, int prec, int sm_count,
                  cudaStream_t stream, bool *handled) {
  *handled = false;
  if (cin == 16 && width == 32 && p.COUT > 16 && p.COUT <= 32 && p.H % 2 == 0)
    return prec == 1 ? launch_conv<16, 32, 14, 32, 3, 2, 1, 16, kFusePool>(io, p, sm_count, stream, handled)
         : prec == 2 ? launch_conv<16, 32, 8, 32, 2, 2, 2, 16, kFusePool>(io, p, sm_count, stream, handled)
                     : launch_conv<16, 32, 16, 32, 0, 2, 2, 16, kFusePool>(io, p, sm_count, stream, handled);
  return REMORA_OK;
}

int dispatch_unpool(const ConvIO &io, const ConvTCParams &p, int cin, int width, int prec, int sm_count,
                    cudaStream_t stream, bool *handled) {
  *handled = false;
  if (cin == 32 && width == 32 && p.COUT <= 16 && p.H % 2 == 0)
    return prec == 1 ? launch_conv<32, 32, 16, 16, 3, 2, 1, 8, kFuseUnpool, 2>(io, p, sm_count, stream, handled)
         : prec == 2 ? launch_conv<32, 32, 16, 16, 2, 2, 2, 8, kFuseUnpool, 2>(io, p, sm_count, stream, handled)
                     : launch_conv<32, 32, 16, 16, 0, 2, 2, 8, kFuseUnpool, 2>(io, p, sm_count, stream, handled);
  return REMORA_OK;
}

int prec_code(int precision) {
  return precision == REMORA_PREC_3XTF32 ? 1 : precision == REMORA_PREC_2XTF32 ? 2 : 0;
}

bool shape_ok(const ConvGeom &g, const void *x, int precision) {
  return (precision == REMORA_PREC_TF32 || precision == REMORA_PREC_3XTF32 || precision == REMORA_PREC_2XTF32) &&
         g.R == 3 && g.S == 3 &&
         g.pad == 1 && g.stride == 1 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 && g.N > 0 && g.H > 0;
}

}  // namespace

int conv_tc_fwd(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *w, const float *bias, float *y,
                int precision, cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!shape_ok(g, x, precision)) return REMORA_OK;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  ConvTCParams p{w, bias, y, nullptr, g.N, g.H, g.K, 0, 0, ws->err};
  return dispatch(ConvIO{x, nullptr, y, nullptr}, p, g.C, g.W, prec_code(precision), ctx->persistent_limit(),
                  stream, handled);
}

int conv_tc_fwd_relu_pool(RemoraB200Ctx *ctx, const ConvGeom &g, const float *x, const float *w, const float *bias,
                          float *pooled, uint8_t *codes, int precision, cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!shape_ok(g, x, precision) || g.K > 32) return REMORA_OK;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  ConvTCParams p{w, bias, pooled, codes, g.N, g.H, g.K, 0, 0, ws->err};
  return dispatch_pool(ConvIO{x, nullptr, pooled, codes}, p, g.C, g.W, prec_code(precision),
                       ctx->persistent_limit(), stream, handled);
}

int conv_tc_dgrad_unpool(RemoraB200Ctx *ctx, const ConvGeom &g, const float *dpooled, const uint8_t *codes,
                         const float *w, float *dx, int precision, cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!shape_ok(g, dpooled, precision) || g.C > 32) return REMORA_OK;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  ConvTCParams p{w, nullptr, dx, nullptr, g.N, g.H, g.C, 1, 0, ws->err};
  return dispatch_unpool(ConvIO{dpooled, codes, dx, nullptr}, p, g.K, g.W, prec_code(precision),
                         ctx->persistent_limit(), stream, handled);
}

int conv_tc_dgrad(RemoraB200Ctx *ctx, const ConvGeom &g, const float *dy, const float *w, float *dx, int precision,
                  cudaStream_t stream, bool *handled) {
  *handled = false;
  if (!shape_ok(g, dy, precision)) return REMORA_OK;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, stream, 0, &ws));
  // forward conv of dy (K channels) into dx (C channels) with flipped weights
  ConvTCParams p{w, nullptr, dx, nullptr, g.N, g.H, g.C, 1, 0, ws->err};
  return dispatch(ConvIO{dy, nullptr, dx, nullptr}, p, g.K, g.W, prec_code(precision), ctx->persistent_limit(),
                  stream, handled);
}

int conv_tc_wgrad(RemoraB200Ctx *, const ConvGeom &, const float *, const float *, float *, int, cudaStream_t,
                  bool *handled) {
  *handled = false;
  return REMORA_OK;
}

}  // namespace remora
