// gemm.cu — the dense core: C = A . B as the reference's lifted dot
// C[i,j] = fold(+, 0, map(*, A[i,:], B[:,j])) (stdlib/prelude.rem:14,
// examples/crater_train.py:38-44), on tcgen05 tensor cores for sm_100a.
//
// Kernel: persistent, warp-specialised, one CTA per SM, 128 x 256 output
// tiles, 32-deep K stages of TMA-loaded SWIZZLE_128B tiles (no multicast).
//   warp 0 lane 0  TMA producer (stage ring, full/empty mbarriers)
//   warp 1 lane 0  MMA issuer: 4 tcgen05.mma.kind::tf32 (K = 8 each) per
//                  stage into a TMEM accumulator, tcgen05.commit frees the
//                  stage; 2 accumulators of 256 columns (all 512 TMEM
//                  columns) so the epilogue of tile i overlaps tile i+1
//   warp 2         TMEM allocator
//   warps 4-7      epilogue: tcgen05.ld 32 lanes x 32 columns into a
//                  per-warp staging tile in shared memory, stored row by
//                  row as 128-byte runs of 32 columns (coalesced)
// Operands may be K-major (SWIZZLE_128B tiles) or M/N-major
// (SWIZZLE_128B_BASE32B tiles); both are native UMMA layouts.
// 3xTF32: each operand is split into hi = tf32(x) (low 13 mantissa bits
// cleared) and lo = x - hi (exact), and the MMA issues hi*hi + hi*lo +
// lo*hi per K step into the same f32 accumulator.  Small GEMMs (at most
// one tile per SM, or a short K) split in the kernel: TMA loads A and B as
// they are and warps 2-3 write each stage's lo beside it in shared memory
// (the raw tile is hi as the tensor core reads it).  Large ones take operands split by a prep pass, whose cost is
// small against their MMAs and which keeps the transform off their
// critical path.
#include <cudaTypedefs.h>

#include <algorithm>

#include "common.cuh"
#include "tcgen05.cuh"

namespace remora {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  }
  return fn;
}

namespace {

// Tiles are BM x BN_ with BN_ = 256 (the default) or 64 (for N <= 64,
// e.g. a dense layer with 64 outputs, where a 256-wide tile would compute
// 4x the needed products).
constexpr int BM = 128, BK = 32;
constexpr uint32_t A_BYTES = BM * BK * 4;
constexpr int kThreads = 256;
constexpr uint32_t kTmemCols = 512;

template <bool SPLIT3, int BN_>
struct Cfg {
  static constexpr int BN = BN_;
  static constexpr uint32_t B_BYTES = BN * BK * 4;
  static constexpr int STAGES = SPLIT3 ? (BN == 256 ? 2 : 4) : (BN == 256 ? 4 : 8);
  static constexpr uint32_t STAGE_BYTES = SPLIT3 ? 2 * (A_BYTES + B_BYTES) : (A_BYTES + B_BYTES);
  static constexpr size_t SMEM = (size_t)STAGES * STAGE_BYTES + 1024;
  static_assert(SMEM + 4 * 32 * 36 * 4 + 1024 <= 227 * 1024, "shared memory per block (dynamic + the epilogue's staging)");
  static_assert(A_BYTES % 16 == 0 && B_BYTES % 16 == 0, "split_hi_lo moves 16-byte vectors");
};
// Tile columns per group of the tile order (decode_tile).
#ifndef REMORA_GEMM_GROUP_COLS
#define REMORA_GEMM_GROUP_COLS 8
#endif
constexpr int kGroupCols = REMORA_GEMM_GROUP_COLS;
// Scratch for K-split partials: at most one 128 x 256 f32 tile per SM.
constexpr size_t kSplitPartBytes = (size_t)148 * BM * 256 * 4 + 256;

struct GemmParams {
  int M, N, K, batch;
  int a_mn, b_mn;
  int mt, nt, kt;
  float *C;
  long long ldc;  // C's row stride: element (row, col) at row * ldc + col * c_cs
  long long c_cs;  // C's column stride (1: rows contiguous)
  long long c_bstride;
  int *err;
  // Tiles from `split_from` on are split along K into `split` ranges; their
  // BM x BN partials go to `part` ([tile - split_from][split][BM][BN]) and
  // gemm_split_fixup adds them in split order.  split == 1: no split.
  // split_from == 0 splits every tile (a launch of few tiles); a larger
  // split_from splits only the tiles past the last full wave, so that the
  // persistent CTAs end together instead of a part-filled last wave.
  int split;
  int split_from;
  float *part;
  // tile order: groups of `gn` tile columns, row-major inside a group
  int gn;
};

// Work unit u -> tile, K-block range, and partial slot (-1: the whole tile).
__device__ __forceinline__ void decode_unit(int u, const GemmParams &p, int &tile, int &kb0, int &kb1,
                                            int &slot) {
  if (p.split == 1 || u < p.split_from) {
    tile = u;
    kb0 = 0;
    kb1 = p.kt;
    slot = -1;
  } else {
    const int v = u - p.split_from;
    const int part = v % p.split;
    tile = p.split_from + v / p.split;
    kb0 = (int)((long long)p.kt * part / p.split);
    kb1 = (int)((long long)p.kt * (part + 1) / p.split);
    slot = v;
  }
}

__device__ __forceinline__ void load_operand(const CUtensorMap *map, uint64_t *bar, uint8_t *dst, int mn, int row0,
                                             int rows, int k0, int b) {
  if (!mn) {
    tc::tma_load_3d(map, bar, dst, k0, row0, b);  // box {32 k, rows}
  } else {
    for (int c = 0; c < rows / 32; ++c)  // box {32 rows, 32 k} per 32-row chunk
      tc::tma_load_3d(map, bar, dst + c * 4096, row0 + 32 * c, k0, b);
  }
}

// MN-major tiles are 32-row boxes of 32 elements (4 KB) side by side.
__device__ __forceinline__ uint64_t operand_desc(uint32_t saddr, int mn, int kk) {
  return mn ? tc::desc_mnmajor(saddr, 4096, kk) : tc::desc_kmajor(saddr, kk);
}

// Tile t -> (batch, row block, column block).  Tiles run in groups of gn
// column blocks, row-major inside a group: the CTAs of one wave share few
// B column blocks and reuse each A row block across gn tiles, which keeps a
// wave's operands in L2.
__device__ __forceinline__ void decode_tile(int t, const GemmParams &p, int &b, int &mb, int &nb) {
  const int per = p.mt * p.nt;
  b = t / per;
  const int r = t - b * per;
  const int g = r / (p.mt * p.gn);
  const int gw = min(p.gn, p.nt - g * p.gn);
  const int i = r - g * p.mt * p.gn;
  mb = i / gw;
  nb = g * p.gn + (i - mb * gw);
}

// x -> (hi, lo) for the `bytes` of one operand tile at shared address t:
// lo = x - hi goes to t + bytes; hi stays where it is.  The tensor core
// reads an f32 operand of a kind::tf32 MMA as its TF32 part by dropping the
// low 13 mantissa bits, which is hi exactly, so the raw tile serves as hi
// (results bit-identical to writing hi back).  `nthreads` threads, 16 bytes
// each per pass.
__device__ __forceinline__ void split_hi_lo(uint32_t t, uint32_t bytes, int tid, int nthreads) {
  // Four 16-byte reads in flight per thread before its four writes; a
  // thread's reads are one pass (nthreads * 16 bytes) apart.
  const uint32_t pass = (uint32_t)nthreads * 16;
  for (uint32_t off0 = (uint32_t)tid * 16; off0 < bytes; off0 += 4 * pass) {
    float4 v[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t off = off0 + j * pass;
      if (off < bytes)
        asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
                     : "=f"(v[j].x), "=f"(v[j].y), "=f"(v[j].z), "=f"(v[j].w)
                     : "r"(t + off)
                     : "memory");
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t off = off0 + j * pass;
      if (off >= bytes) break;
      const float h0 = __uint_as_float(__float_as_uint(v[j].x) & 0xFFFFE000u);
      const float h1 = __uint_as_float(__float_as_uint(v[j].y) & 0xFFFFE000u);
      const float h2 = __uint_as_float(__float_as_uint(v[j].z) & 0xFFFFE000u);
      const float h3 = __uint_as_float(__float_as_uint(v[j].w) & 0xFFFFE000u);
      asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(t + bytes + off), "f"(__fsub_rn(v[j].x, h0)),
                   "f"(__fsub_rn(v[j].y, h1)), "f"(__fsub_rn(v[j].z, h2)), "f"(__fsub_rn(v[j].w, h3))
                   : "memory");
    }
  }
}

template <bool SPLIT3, int BN_, bool INK>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                     const __grid_constant__ CUtensorMap tmAl, const __grid_constant__ CUtensorMap tmBl,
                     GemmParams p) {
  using C = Cfg<SPLIT3, BN_>;
  constexpr int STAGES = C::STAGES;
  constexpr int BN = C::BN;
  constexpr uint32_t B_BYTES = C::B_BYTES;
  extern __shared__ uint8_t smem_dyn[];
  uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_dyn) + 1023) & ~uintptr_t(1023));
  // xfull: a 3xTF32 stage has been split into hi / lo (2 transform warps)
  __shared__ __align__(8) uint64_t full[STAGES], empty[STAGES], xfull[STAGES], tfull[2], tempty[2], drain;
  __shared__ uint32_t tmem_base;
  __shared__ int abort_flag;
  __shared__ __align__(16) float epi_stage[4 * 32 * 36];  // one 32 x 32 block per epilogue warp

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // A CTA with a single work unit runs its epilogue once, at the end: its
  // four epilogue warps split stages with warps 2-3 until then.
  const int ntiles = p.batch * p.mt * p.nt;
  const int nunits = p.split == 1 ? ntiles : p.split_from + (ntiles - p.split_from) * p.split;
  const bool epi_split = INK && (nunits - (int)blockIdx.x + (int)gridDim.x - 1) / (int)gridDim.x == 1;
  const int split_warps = epi_split ? 6 : 2;
  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      tc::mbar_init(&full[s], 1);
      tc::mbar_init(&empty[s], 1);
      tc::mbar_init(&xfull[s], split_warps);
    }
    for (int b = 0; b < 2; ++b) {
      tc::mbar_init(&tfull[b], 1);
      tc::mbar_init(&tempty[b], 4);
    }
    tc::mbar_init(&drain, 1);
    abort_flag = 0;
    tc::fence_barrier_init();
  }
  if (warp == 0 && lane == 0) {
    tc::prefetch_tmap(&tmA);
    tc::prefetch_tmap(&tmB);
    if (SPLIT3 && !INK) {
      tc::prefetch_tmap(&tmAl);
      tc::prefetch_tmap(&tmBl);
    }
  }
  if (warp == 2) tc::tmem_alloc(&tmem_base, kTmemCols);
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tbase = tmem_base;
  volatile int *abort_v = &abort_flag;

  // ------------------------------------------------ 3xTF32 hi/lo split
  // Elementwise: the raw tile is hi where it lies (and keeps its swizzle), lo
  // goes to the same position of the lo slot.
  auto split_stages = [&]() {
    const int tid = threadIdx.x - 64, nthreads = split_warps * 32;
    int s = 0;
    uint32_t ph = 0;
    for (int u = blockIdx.x; u < nunits && !*abort_v; u += gridDim.x) {
      int t, kb0, kb1, slot;
      decode_unit(u, p, t, kb0, kb1, slot);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait(&full[s], ph, abort_v, p.err, 105)) return;
        const uint32_t sa = tc::smem_u32(smem + (size_t)s * C::STAGE_BYTES);
        split_hi_lo(sa, A_BYTES, tid, nthreads);
        split_hi_lo(sa + 2 * A_BYTES, B_BYTES, tid, nthreads);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) tc::mbar_arrive(&xfull[s]);
        if (++s == STAGES) s = 0, ph ^= 1;
      }
    }
  };

  if (warp == 0 && lane == 0) {
    // ------------------------------------------------------ TMA producer
    int s = 0;
    uint32_t ph = 0;
    uint32_t issued_ph[STAGES];
    bool pending[STAGES];
    for (int i = 0; i < STAGES; ++i) pending[i] = false, issued_ph[i] = 0;
    for (int u = blockIdx.x; u < nunits && !*abort_v; u += gridDim.x) {
      int t, kb0, kb1, slot;
      decode_unit(u, p, t, kb0, kb1, slot);
      int b, mb, nb;
      decode_tile(t, p, b, mb, nb);
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait(&empty[s], ph ^ 1, abort_v, p.err, 101)) goto producer_done;
        uint8_t *sa = smem + (size_t)s * C::STAGE_BYTES;
        tc::mbar_arrive_expect_tx(&full[s], SPLIT3 && !INK ? C::STAGE_BYTES : A_BYTES + B_BYTES);
        load_operand(&tmA, &full[s], sa, p.a_mn, mb * BM, BM, kb * BK, b);
        if (SPLIT3 && !INK) {
          load_operand(&tmAl, &full[s], sa + A_BYTES, p.a_mn, mb * BM, BM, kb * BK, b);
          load_operand(&tmBl, &full[s], sa + 2 * A_BYTES + B_BYTES, p.b_mn, nb * BN, BN, kb * BK, b);
        }
        // 3xTF32: B goes to its hi slot (split in the kernel: raw, split there)
        load_operand(&tmB, &full[s], sa + (SPLIT3 ? 2 * A_BYTES : A_BYTES), p.b_mn, nb * BN, BN, kb * BK, b);
        issued_ph[s] = ph;
        pending[s] = true;
        if (++s == STAGES) s = 0, ph ^= 1;
      }
    }
  producer_done:
    // Do not leave while a TMA copy may still write this CTA's shared memory.
    for (int i = 0; i < STAGES; ++i) {
      if (!pending[i]) continue;
      const long long t0 = clock64();
      while (!tc::mbar_test(&full[i], issued_ph[i]) && clock64() - t0 < tc::kWaitCycles) {
      }
    }
  } else if (warp == 1 && lane == 0) {
    // ------------------------------------------------------- MMA issuer
    const uint32_t idesc = tc::idesc_tf32(BM, BN, p.a_mn, p.b_mn);
    int s = 0;
    uint32_t ph = 0;
    int local = 0;
    bool issued = false;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++local) {
      int t, kb0, kb1, slot;
      decode_unit(u, p, t, kb0, kb1, slot);
      const int buf = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!tc::mbar_wait(&tempty[buf], aph ^ 1, abort_v, p.err, 102)) break;
      tc::fence_after_sync();
      const uint32_t d = tbase + buf * BN;
      for (int kb = kb0; kb < kb1; ++kb) {
        if (!tc::mbar_wait(INK ? &xfull[s] : &full[s], ph, abort_v, p.err, 103)) goto mma_done;
        tc::fence_after_sync();
        const uint32_t sa = tc::smem_u32(smem + (size_t)s * C::STAGE_BYTES);
        const uint32_t sb = SPLIT3 ? sa + 2 * A_BYTES : sa + A_BYTES;
#pragma unroll
        for (int kk = 0; kk < BK / 8; ++kk) {
          const uint64_t ad = operand_desc(sa, p.a_mn, kk);
          const uint64_t bd = operand_desc(sb, p.b_mn, kk);
          tc::mma_tf32(d, ad, bd, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
          if (SPLIT3) {
            tc::mma_tf32(d, ad, operand_desc(sb + B_BYTES, p.b_mn, kk), idesc, 1);
            tc::mma_tf32(d, operand_desc(sa + A_BYTES, p.a_mn, kk), bd, idesc, 1);
          }
        }
        issued = true;
        tc::mma_commit(&empty[s]);
        if (++s == STAGES) s = 0, ph ^= 1;
      }
      tc::mma_commit(&tfull[buf]);
    }
  mma_done:
    if (issued) {
      // all MMAs of this CTA done before TMEM can be released
      tc::mma_commit(&drain);
      const long long t0 = clock64();
      while (!tc::mbar_test(&drain, 0) && clock64() - t0 < tc::kWaitCycles) {
      }
    }
  } else if (INK && (warp == 2 || warp == 3)) {
    split_stages();
  } else if (warp >= 4) {
    if (epi_split) split_stages();
    // --------------------------------------------------------- epilogue
    const int e = warp - 4;
    int local = 0;
    for (int u = blockIdx.x; u < nunits; u += gridDim.x, ++local) {
      int t, kb0, kb1, slot;
      decode_unit(u, p, t, kb0, kb1, slot);
      const int buf = local & 1;
      const uint32_t aph = (local >> 1) & 1;
      if (!tc::mbar_wait(&tfull[buf], aph, abort_v, p.err, 104)) break;
      tc::fence_after_sync();
      int b, mb, nb;
      decode_tile(t, p, b, mb, nb);
      // Each 32 x 32 block goes through the warp's staging tile: lane l
      // writes row l (its TMEM lane), then the warp stores the block row by
      // row, 32 consecutive columns per store (128 contiguous bytes) rather
      // than 32 rows of 16 bytes each.  Rows are padded to 36 floats, so the
      // 16-byte writes and the column reads are both free of bank conflicts.
      const uint32_t stg_s = tc::smem_u32(epi_stage + e * 32 * 36);
      const float *stg = epi_stage + e * 32 * 36;
      const int row0 = mb * BM + e * 32;
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t r[32];
        tc::tmem_ld_32x32b_x32(tbase + buf * BN + c * 32 + ((uint32_t)(e * 32) << 16), r);
        tc::tmem_ld_wait();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(stg_s + (uint32_t)(lane * 36 + 4 * j) * 4),
                       "r"(r[4 * j]), "r"(r[4 * j + 1]), "r"(r[4 * j + 2]), "r"(r[4 * j + 3])
                       : "memory");
        __syncwarp();
        const int col0 = nb * BN + c * 32;
        if (slot >= 0) {
          // one K range of a split tile: the whole BM x BN partial, unguarded
          float *dst = p.part + ((long long)slot * BM + e * 32) * BN + c * 32 + lane;
#pragma unroll 4
          for (int rr = 0; rr < 32; ++rr) dst[(long long)rr * BN] = stg[rr * 36 + lane];
        } else if (p.c_cs != 1) {
          // columns not contiguous (a column-major C: lanes hold consecutive
          // rows, so each store of the 32 lanes is one contiguous run)
          if (row0 + lane < p.M) {
            float *dst = p.C + (long long)b * p.c_bstride + (long long)(row0 + lane) * p.ldc;
            const int cols = min(32, p.N - col0);
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (j < cols) dst[(long long)(col0 + j) * p.c_cs] = __uint_as_float(r[j]);
          }
        } else if (col0 + lane < p.N) {
          float *dst = p.C + (long long)b * p.c_bstride + (long long)row0 * p.ldc + col0 + lane;
          const int rows = min(32, p.M - row0);
#pragma unroll 4
          for (int rr = 0; rr < rows; ++rr) dst[(long long)rr * p.ldc] = stg[rr * 36 + lane];
        }
        __syncwarp();
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(&tempty[buf]);
    }
  }
  __syncthreads();
  if (warp == 2) {
    tc::fence_after_sync();
    tc::tmem_dealloc(tbase, kTmemCols);
  }
}

// hi = x with the low 13 mantissa bits cleared (exactly representable in
// tf32), lo = x - hi (exact in f32).  Copies a [batch][outer][inner] view
// with arbitrary strides into contiguous [batch][outer][inner_pad] arrays,
// zero-filling inner in [inner, inner_pad).
__global__ void __launch_bounds__(256) prep_operand_kernel(const float *__restrict__ src, long long sb,
                                                           long long so, long long si, int batch, long long outer,
                                                           long long inner, long long inner_pad,
                                                           float *__restrict__ hi, float *__restrict__ lo) {
  const long long n = (long long)batch * outer * inner_pad;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const long long k = i % inner_pad;
    const long long r = (i / inner_pad) % outer;
    const long long b = i / (inner_pad * outer);
    float v = k < inner ? src[b * sb + r * so + k * si] : 0.0f;
    if (lo) {
      const float h = __uint_as_float(__float_as_uint(v) & 0xFFFFE000u);
      hi[i] = h;
      lo[i] = __fsub_rn(v, h);
    } else {
      hi[i] = v;
    }
  }
}

// C of every split tile = its partials added in split order (fixed, so the
// result is deterministic).  One thread per element of C.
template <int BN>
__global__ void __launch_bounds__(256) gemm_split_fixup(const float *__restrict__ part, GemmParams p) {
  const long long per = (long long)BM * BN;
  const long long n = ((long long)p.batch * p.mt * p.nt - p.split_from) * per;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const int st = (int)(i / per);  // index among the split tiles
    // consecutive threads walk C's contiguous direction
    const int r = p.c_cs == 1 ? (int)((i % per) / BN) : (int)(i % BM);
    const int c = p.c_cs == 1 ? (int)(i % BN) : (int)((i % per) / BM);
    int b, mb, nb;
    decode_tile(p.split_from + st, p, b, mb, nb);
    const int row = mb * BM + r, col = nb * BN + c;
    if (row >= p.M || col >= p.N) continue;
    const float *src = part + ((long long)st * p.split) * per + (long long)r * BN + c;
    float v = src[0];
    for (int s = 1; s < p.split; ++s) v = __fadd_rn(v, src[(long long)s * per]);
    p.C[(long long)b * p.c_bstride + (long long)row * p.ldc + (long long)col * p.c_cs] = v;
  }
}

__global__ void fill_zero_kernel(float *c, long long ldc, long long cs, long long bs, int batch, int M, int N) {
  const long long n = (long long)batch * M * N;
  const long long step = (long long)gridDim.x * blockDim.x;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += step) {
    const long long j = i % N, r = (i / N) % M, b = i / ((long long)N * M);
    c[b * bs + r * ldc + j * cs] = 0.0f;
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() { return tensor_map_encoder(); }

// One GEMM operand as TMA sees it: contiguous inner dimension, `ld` elements
// between outer rows, `bs` between batch entries.  `mn` says whether the
// inner dimension is M/N (1) or K (0); `rows` is the M or N extent.
struct Operand {
  const float *base;
  long long ld, bs;
  int mn;
  long long rows, K;
};

int encode_operand(const Operand &o, int box_rows, int batch, CUtensorMap *map) {
  auto fn = encode_fn();
  if (!fn) return fail(REMORA_ERR_CUDA, "gemm: cuTensorMapEncodeTiled is not available from the driver");
  cuuint64_t dims[3], strides[2];
  cuuint32_t box[3], estr[3] = {1, 1, 1};
  if (!o.mn) {
    dims[0] = (cuuint64_t)o.K;
    dims[1] = (cuuint64_t)o.rows;
    box[0] = 32;
    box[1] = (cuuint32_t)box_rows;
  } else {
    dims[0] = (cuuint64_t)o.rows;
    dims[1] = (cuuint64_t)o.K;
    box[0] = 32;
    box[1] = 32;
  }
  dims[2] = (cuuint64_t)batch;
  box[2] = 1;
  strides[0] = (cuuint64_t)o.ld * 4;
  strides[1] = (cuuint64_t)(batch > 1 ? o.bs : o.ld * (long long)dims[1]) * 4;
  // K-major tiles use the 16-byte-unit 128B swizzle, MN-major tiles the
  // 32-byte-unit one (the only MN-major layout tf32 MMAs accept).
  const CUtensorMapSwizzle swz = o.mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float *>(o.base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swz, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS)
    return fail(REMORA_ERR_CUDA, "gemm: cuTensorMapEncodeTiled failed (%d) for dims %llu x %llu x %llu", (int)r,
                (unsigned long long)dims[0], (unsigned long long)dims[1], (unsigned long long)dims[2]);
  return REMORA_OK;
}

bool tma_ok(const Operand &o, int batch) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(o.base);
  return (a & 15) == 0 && o.ld > 0 && (o.ld & 3) == 0 && (batch == 1 || ((o.bs & 3) == 0 && o.bs > 0));
}

template <bool SPLIT3, int BN, bool INK>
int launch_gemm(const Operand &A, const Operand &B, const Operand &Al, const Operand &Bl, GemmParams p,
                int sm_count, cudaStream_t stream) {
  using C = Cfg<SPLIT3, BN>;
  p.nt = (p.N + BN - 1) / BN;
  CUtensorMap ma, mb, mal, mbl;
  REMORA_TRY(encode_operand(A, BM, p.batch, &ma));
  REMORA_TRY(encode_operand(B, BN, p.batch, &mb));
  if (SPLIT3 && !INK) {
    REMORA_TRY(encode_operand(Al, BM, p.batch, &mal));
    REMORA_TRY(encode_operand(Bl, BN, p.batch, &mbl));
  } else {
    mal = ma;  // TF32, or 3xTF32 split in shared memory: no lo operands
    mbl = mb;
  }
  static bool attr_set = false;
  if (!attr_set) {
    REMORA_CUDA_TRY(cudaFuncSetAttribute(gemm_tf32_kernel<SPLIT3, BN, INK>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)C::SMEM));
    attr_set = true;
  }
  const int ntiles = p.batch * p.mt * p.nt;
  p.gn = std::max(1, std::min(p.nt, kGroupCols));
  // Few tiles and a long K (a dense layer's forward or weight gradient):
  // split K so that the launch fills the SMs.
  p.split = 1;
  p.split_from = 0;
  const long long cap = (long long)(kSplitPartBytes - 256) / ((long long)BM * BN * 4);
  if (p.part != nullptr && 2 * ntiles <= sm_count && p.kt >= 8) {
    int s = std::min(sm_count / ntiles, p.kt / 4);
    s = (int)std::min<long long>(s, cap / ntiles);
    if (s >= 2) p.split = s;
  } else if (p.part != nullptr && ntiles > sm_count && p.kt >= 16) {
    // Several waves with a part-filled last one: the tiles past the last
    // full wave are split along K over all the SMs instead (when at most
    // half a wave is left, so that each splits at least in two).
    const int rem = ntiles % sm_count;
    if (rem > 0 && 2 * rem <= sm_count) {
      int s = std::min(sm_count / rem, p.kt / 8);
      s = (int)std::min<long long>(s, cap / rem);
      if (s >= 2) {
        p.split = s;
        p.split_from = ntiles - rem;
      }
    }
  }
  const int nunits = p.split == 1 ? ntiles : p.split_from + (ntiles - p.split_from) * p.split;
  const int grid = std::min(nunits, sm_count);
  note_launch();
  gemm_tf32_kernel<SPLIT3, BN, INK><<<grid, kThreads, C::SMEM, stream>>>(ma, mb, mal, mbl, p);
  REMORA_CUDA_TRY(cudaGetLastError());
  if (p.split > 1) {
    const long long n = (long long)(ntiles - p.split_from) * BM * BN;
    note_launch();
    gemm_split_fixup<BN><<<(int)std::min<long long>((n + 255) / 256, (long long)sm_count * 16), 256, 0, stream>>>(
        p.part, p);
    REMORA_CUDA_TRY(cudaGetLastError());
  }
  return REMORA_OK;
}

int grid_for(long long n, int sm_count) {
  return (int)std::max<long long>(1, std::min<long long>((n + 255) / 256, (long long)sm_count * 16));
}

}  // namespace

size_t gemm_workspace_bytes(long long batch, long long M, long long N, long long K, bool split) {
  const long long kp = (K + 3) & ~3LL, mp = (M + 3) & ~3LL, np = (N + 3) & ~3LL;
  const size_t a = (size_t)batch * std::max(M * kp, K * mp) * 4 + 256;
  const size_t b = (size_t)batch * std::max(N * kp, K * np) * 4 + 256;
  return (split ? 2 : 1) * (a + b) + (size_t)batch * M * N * 4 + 1024 + kSplitPartBytes;
}

// Runs C = A . B with every operand given as a [batch][rows][cols] view.
// `scratch` must hold gemm_workspace_bytes(...).
int run_gemm(RemoraB200Ctx *ctx, int precision, const DescView &A, const DescView &B, const DescView &Cd, int rank,
             char *scratch, size_t scratch_bytes, int *err, cudaStream_t stream) {
  const int batch = rank == 3 ? (int)A.sizes[0] : 1;
  const int o = rank - 2;
  const long long M = A.sizes[o], K = A.sizes[o + 1], N = B.sizes[o + 1];
  if (B.sizes[o] != K) return fail(REMORA_ERR_SHAPE, "gemm: A is [%lld, %lld] but B has %lld rows", M, K, B.sizes[o]);
  if (Cd.sizes[o] != M || Cd.sizes[o + 1] != N) return fail(REMORA_ERR_SHAPE, "gemm: C must be [%lld, %lld]", M, N);
  if (rank == 3 && (B.sizes[0] != batch || Cd.sizes[0] != batch))
    return fail(REMORA_ERR_SHAPE, "gemm: batch sizes differ");
  if (M > (1LL << 30) || N > (1LL << 30) || K > (1LL << 30) || batch > 65535)
    return fail(REMORA_ERR_LIMIT, "gemm: dimension beyond the supported range");
  if (M == 0 || N == 0 || batch == 0) return REMORA_OK;
  float *cptr = reinterpret_cast<float *>(Cd.data(4));
  // any strides for C; rows contiguous (column stride 1) is the fast path,
  // columns contiguous (a column-major C) stores as fast
  const long long ldc = Cd.strides[o], ccs = N > 1 ? Cd.strides[o + 1] : 1, cbs = rank == 3 ? Cd.strides[0] : 0;
  if (K == 0) {
    note_launch();
    fill_zero_kernel<<<grid_for((long long)batch * M * N, ctx->sm_count), 256, 0, stream>>>(cptr, ldc, ccs, cbs, batch,
                                                                                              (int)M, (int)N);
    REMORA_CUDA_TRY(cudaGetLastError());
    return REMORA_OK;
  }
  const bool split = precision == REMORA_PREC_3XTF32;
  // Operand views: A [b][M][K], B [b][K][N].
  auto make = [&](const DescView &d, long long rows_axis_size, bool is_a, Operand *op) {
    const long long s_rows = is_a ? d.strides[o] : d.strides[o + 1];  // stride along M (A) / N (B)
    const long long s_k = is_a ? d.strides[o + 1] : d.strides[o];
    op->base = reinterpret_cast<const float *>(d.data(4));
    op->bs = rank == 3 ? d.strides[0] : 0;
    op->rows = rows_axis_size;
    op->K = K;
    if (s_k == 1 || K == 1) {
      op->mn = 0;
      op->ld = s_rows;
    } else if (s_rows == 1 || rows_axis_size == 1) {
      op->mn = 1;
      op->ld = s_k;
    } else {
      op->mn = 0;
      op->ld = -1;  // not TMA-addressable: staged below
    }
  };
  Operand a, b;
  make(A, M, true, &a);
  make(B, N, false, &b);
  // 3xTF32 split in the kernel for at most one tile per SM or a short K;
  // otherwise by the prep pass (a plain staging copy is still made for views
  // TMA cannot address)
  const long long tiles_est = (long long)batch * ((M + BM - 1) / BM) * ((N + (N <= 64 ? 63 : 255)) / (N <= 64 ? 64 : 256));
  const bool ink = split && (tiles_est <= ctx->sm_count || K <= 256);
  const bool prep_split = split && !ink;
  char *ws = scratch;
  size_t used = 0;
  auto take = [&](size_t bytes) -> float * {
    bytes = (bytes + 255) & ~(size_t)255;
    if (used + bytes > scratch_bytes) return nullptr;
    float *p = reinterpret_cast<float *>(ws + used);
    used += bytes;
    return p;
  };
  // Stage an operand (and split it for 3xTF32) into contiguous arrays that
  // keep its majorness, padding the inner extent to a multiple of 4.
  auto stage = [&](const DescView &d, bool is_a, Operand &op, Operand &lo) -> int {
    const long long s_rows = is_a ? d.strides[o] : d.strides[o + 1];
    const long long s_k = is_a ? d.strides[o + 1] : d.strides[o];
    const long long inner = op.mn ? op.rows : K, outer = op.mn ? K : op.rows;
    const long long si = op.mn ? s_rows : s_k, so = op.mn ? s_k : s_rows;
    const long long inner_pad = (inner + 3) & ~3LL;
    float *hi = take((size_t)batch * outer * inner_pad * 4);
    float *lp = prep_split ? take((size_t)batch * outer * inner_pad * 4) : nullptr;
    if (!hi || (prep_split && !lp)) return fail(REMORA_ERR_LIMIT, "gemm: workspace too small");
    note_launch();
    prep_operand_kernel<<<grid_for((long long)batch * outer * inner_pad, ctx->sm_count), 256, 0, stream>>>(
        reinterpret_cast<const float *>(d.data(4)), rank == 3 ? d.strides[0] : 0, so, si, batch, outer, inner,
        inner_pad, hi, lp);
    REMORA_CUDA_TRY(cudaGetLastError());
    op.base = hi;
    op.ld = inner_pad;
    op.bs = outer * inner_pad;
    if (op.mn) op.rows = inner; else op.K = K;
    lo = op;
    if (prep_split) lo.base = lp;
    return REMORA_OK;
  };
  Operand al{}, bl{};
  if (prep_split || a.ld < 0 || !tma_ok(a, batch)) {
    if (a.ld < 0) a.mn = 0;
    REMORA_TRY(stage(A, true, a, al));
  }
  if (prep_split || b.ld < 0 || !tma_ok(b, batch)) {
    if (b.ld < 0) b.mn = 0;
    REMORA_TRY(stage(B, false, b, bl));
  }
  GemmParams p{};
  p.M = (int)M;
  p.N = (int)N;
  p.K = (int)K;
  p.batch = batch;
  p.a_mn = a.mn;
  p.b_mn = b.mn;
  p.mt = (int)((M + BM - 1) / BM);
  p.nt = 0;  // set by launch_gemm for its tile width
  p.kt = (int)((K + BK - 1) / BK);
  p.C = cptr;
  p.ldc = ldc;
  p.c_cs = ccs;
  p.c_bstride = cbs;
  p.err = err;
  p.part = take(kSplitPartBytes);  // null when the workspace has no room: no split
  const bool narrow = N <= 64;
  if (prep_split)
    return narrow ? launch_gemm<true, 64, false>(a, b, al, bl, p, ctx->persistent_limit(), stream)
                  : launch_gemm<true, 256, false>(a, b, al, bl, p, ctx->persistent_limit(), stream);
  if (split)
    return narrow ? launch_gemm<true, 64, true>(a, b, a, b, p, ctx->persistent_limit(), stream)
                  : launch_gemm<true, 256, true>(a, b, a, b, p, ctx->persistent_limit(), stream);
  return narrow ? launch_gemm<false, 64, false>(a, b, a, b, p, ctx->persistent_limit(), stream)
                : launch_gemm<false, 256, false>(a, b, a, b, p, ctx->persistent_limit(), stream);
}

}  // namespace remora

using namespace remora;

extern "C" int remora_b200_gemm(RemoraB200Ctx *ctx, const RemoraGemmSpec *spec, const void *a_desc,
                                const void *b_desc, void *c_desc, int32_t rank, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (spec == nullptr) return fail(REMORA_ERR_ARG, "gemm: null spec");
  if (spec->precision != REMORA_PREC_TF32 && spec->precision != REMORA_PREC_3XTF32)
    return fail(REMORA_ERR_ARG, "gemm: unknown precision %d", spec->precision);
  if (rank != 2 && rank != 3) return fail(REMORA_ERR_RANK, "gemm: rank %d (2, or 3 for a batch)", rank);
  DescView A, B, C;
  REMORA_TRY(read_desc(a_desc, rank, &A, "gemm A"));
  REMORA_TRY(read_desc(b_desc, rank, &B, "gemm B"));
  REMORA_TRY(read_desc(c_desc, rank, &C, "gemm C"));
  const int o = rank - 2;
  const long long batch = rank == 3 ? A.sizes[0] : 1;
  const size_t need = gemm_workspace_bytes(batch, A.sizes[o], B.sizes[o + 1], A.sizes[o + 1],
                                           spec->precision == REMORA_PREC_3XTF32);
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, (cudaStream_t)stream, need, &ws));
  return run_gemm(ctx, spec->precision, A, B, C, rank, (char *)ws->buf, ws->bytes, ws->err, (cudaStream_t)stream);
}
