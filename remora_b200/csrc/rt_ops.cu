// rt_ops.cu — the reference's C runtime helpers (remora/remora_rt.c) as
// device kernels: sort and grade (stable LSD radix sort), filter and
// replicate (reduce-then-scan compaction and expansion), rotate and append
// (leading-axis segment copies).
//
// Semantics (reference file:line):
//  - sort: ascending, rank 1 or each row of a rank-2 array
//    (remora_rt.c:42-54, per-row alias :289-290; lowering
//    remora/lowering/tensor_ops.py:2505-2570).
//  - grade: ascending argsort with ties broken by index, i.e. a stable
//    argsort (remora_rt.c:56-121 `_cmp_grade_*`, per-row :291-292; interpreter
//    remora/runtime.py:1175-1177 `np.argsort(kind='stable')`).
//  - filter: keep src[i] where mask[i] != 0, in order, and return the count
//    (remora_rt.c:125-163); the lowering builds the mask from a comparison
//    against a literal (tensor_ops.py:2671-2720), which can be fused here.
//  - replicate: src[i] repeated counts[i] times, in order, and the total
//    (remora_rt.c:167-285); a count below zero writes nothing, as the fill
//    loop `for (r = 0; r < count; r++)` does.
//  - rotate: out[i] = in[(i + k) mod N] along axis 0 with a non-negative
//    modulus (remora_rt.c:324-358; interpreter np.roll(a, -k, axis=0),
//    remora/runtime.py:1135-1139).
//  - append: concatenation along axis 0 (remora_rt.c:360-388,
//    tensor_ops.py:2215-2263; interpreter
//    remora/runtime.py:1165-1166).
//
// No block waits on another anywhere in this file: every multi-block step is
// split into kernels (tile counts, one scan of the counts, tile work).
#include <algorithm>
#include <type_traits>

#include "common.cuh"

namespace remora {

int copy_to_contiguous(const DescView &src, int esize, void *dst, cudaStream_t stream, int sm_count);
int copy_from_contiguous(const void *src, const DescView &dst, int esize, cudaStream_t stream, int sm_count);

namespace {

constexpr int kT = 256;              // threads per block
constexpr int kWarps = kT / 32;      // warps per block
constexpr int kItems = 16;           // keys per thread in the large sort
constexpr int kTile = kT * kItems;   // 4096 keys per tile
constexpr int kSmallMax = kTile;     // rows up to this length sort in one block
constexpr int64_t kMaxSortLen = (int64_t)1 << 31;  // grade stores int32 indices

size_t align256(size_t b) { return (b + 255) & ~(size_t)255; }

// The counting kernels (radix_count, filter_count, rep_tile_sums) walk the
// tiles from the last to the first: the pass over the same data that
// follows them starts at the first tile, which is then the part most
// recently read and still in L2.
__device__ __forceinline__ int64_t reversed_tile() { return (int64_t)gridDim.x - 1 - blockIdx.x; }

// ------------------------------------------------------------ key order --
// Order-preserving maps of f32 / i32 bit patterns onto u32: unsigned order of
// the keys is the numeric order of the values.  For f32, -0.0 sorts before
// +0.0 unless kCanon folds -0.0 onto +0.0 (grade, where equal values must tie
// and fall back to index order); NaNs with the sign bit clear sort last and
// those with it set first.
template <int kDtype, bool kCanon>
__device__ __forceinline__ uint32_t to_key(uint32_t u) {
  if (kDtype == REMORA_F32) {
    if (kCanon && u == 0x80000000u) u = 0u;
    return u ^ ((u & 0x80000000u) ? 0xFFFFFFFFu : 0x80000000u);
  }
  return u ^ 0x80000000u;
}

template <int kDtype>
__device__ __forceinline__ uint32_t from_key(uint32_t k) {
  if (kDtype == REMORA_F32) return k ^ ((k & 0x80000000u) ? 0x80000000u : 0xFFFFFFFFu);
  return k ^ 0x80000000u;
}

// Exclusive sum of one value per thread over a kT-thread block, in thread
// order.  s_w holds kWarps words.  Ends with a barrier, so s_w is reusable.
template <typename U>
__device__ __forceinline__ U block_excl_sum(U v, U *s_w, U *total = nullptr) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  U inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const U up = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += up;
  }
  if (lane == 31) s_w[warp] = inc;
  __syncthreads();
  U pre = 0, all = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const U t = s_w[w];
    if (w < warp) pre += t;
    all += t;
  }
  if (total) *total = all;
  __syncthreads();
  return pre + inc - v;
}

// Ranks the ITEMS keys each thread holds by the 8-bit digit at `shift`.  Key
// i of a thread sits at tile position q = warp*32*ITEMS + i*32 + lane, which
// is its order in the input; positions >= valid_n are absent.  On return
// pos[i] is the key's position in the tile stably sorted by that digit.
// Within a warp the keys are ranked round by round (round i holds positions
// in lane order), so equal digits keep their input order; warps and digits
// are then laid out by exclusive sums.  The lanes sharing a digit are found
// with eight ballots (one per digit bit), which keeps the work on the
// integer pipes; the highest such lane updates the warp's counter.
template <int ITEMS>
__device__ __forceinline__ void rank_digits(const uint32_t (&k)[ITEMS], int valid_n, int shift,
                                            uint32_t (&pos)[ITEMS], uint32_t (*s_wcnt)[256], uint32_t *s_w) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t lt = (1u << lane) - 1u;
  const bool full = valid_n >= kT * ITEMS;
  for (int i = threadIdx.x; i < kWarps * 256; i += kT) (&s_wcnt[0][0])[i] = 0u;
  __syncthreads();
  uint32_t r[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int q = warp * 32 * ITEMS + i * 32 + lane;
    const bool valid = q < valid_n;
    const uint32_t d = (k[i] >> shift) & 255u;
    // a full tile (the same for the whole block) needs no validity ballot
    uint32_t peers = full ? 0xffffffffu : __ballot_sync(0xffffffffu, valid);
#pragma unroll
    for (int b = 0; b < 8; ++b) {
      const uint32_t bit = (d >> b) & 1u;
      // the ballot where this lane's bit is set, its complement where clear
      peers &= __ballot_sync(0xffffffffu, bit) ^ (bit - 1u);
    }
    const uint32_t below = __popc(peers & lt);
    const int leader = 31 - __clz(peers);  // peers is non-empty for a valid lane
    uint32_t old = 0;
    if (valid && lane == leader) {
      old = s_wcnt[warp][d];
      s_wcnt[warp][d] = old + below + 1u;
    }
    old = __shfl_sync(0xffffffffu, old, leader & 31);
    r[i] = old + below;
    __syncwarp();
  }
  __syncthreads();
  // Thread d: exclusive sum over warps of digit d, then over digits.
  const int d = threadIdx.x;  // kT == 256 digits
  uint32_t run = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) {
    const uint32_t c = s_wcnt[w][d];
    s_wcnt[w][d] = run;
    run += c;
  }
  const uint32_t start = block_excl_sum<uint32_t>(run, s_w);
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s_wcnt[w][d] += start;
  __syncthreads();
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int q = warp * 32 * ITEMS + i * 32 + lane;
    pos[i] = q < valid_n ? s_wcnt[warp][(k[i] >> shift) & 255u] + r[i] : 0u;
  }
}

// ---------------------------------------------------- small (one block) --
// Sorts one row of up to kT*ITEMS keys entirely in shared memory: four
// 8-bit passes, the keys staying on chip between them.  Grid: one block per
// row.  kGrade: write the source index of each sorted key instead of the key.
template <int kDtype, int ITEMS, bool kGrade>
__global__ void __launch_bounds__(kT) sort_rows_small(const uint32_t *__restrict__ in, int64_t in_row_stride,
                                                      uint32_t *__restrict__ out, int64_t out_row_stride,
                                                      int len) {
  __shared__ uint32_t s_keys[kT * ITEMS];
  __shared__ uint32_t s_vals[kGrade ? kT * ITEMS : 1];
  __shared__ uint32_t s_wcnt[kWarps][256];
  __shared__ uint32_t s_w[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t *src = in + (int64_t)blockIdx.x * in_row_stride;
  uint32_t k[ITEMS], v[ITEMS], pos[ITEMS];
#pragma unroll
  for (int i = 0; i < ITEMS; ++i) {
    const int q = warp * 32 * ITEMS + i * 32 + lane;
    k[i] = q < len ? to_key<kDtype, kGrade>(src[q]) : 0u;
    v[i] = (uint32_t)q;
  }
  for (int pass = 0; pass < 4; ++pass) {
    rank_digits<ITEMS>(k, len, pass * 8, pos, s_wcnt, s_w);
#pragma unroll
    for (int i = 0; i < ITEMS; ++i) {
      const int q = warp * 32 * ITEMS + i * 32 + lane;
      if (q < len && pos[i] < (uint32_t)len) {
        s_keys[pos[i]] = k[i];
        if (kGrade) s_vals[pos[i]] = v[i];
      }
    }
    __syncthreads();
    if (pass < 3) {
#pragma unroll
      for (int i = 0; i < ITEMS; ++i) {
        const int q = warp * 32 * ITEMS + i * 32 + lane;
        if (q < len) {
          k[i] = s_keys[q];
          if (kGrade) v[i] = s_vals[q];
        }
      }
      // rank_digits begins by clearing its counters and a barrier, after
      // which the shared arrays may be overwritten again.
    }
  }
  uint32_t *dst = out + (int64_t)blockIdx.x * out_row_stride;
  for (int q = threadIdx.x; q < len; q += kT) dst[q] = kGrade ? s_vals[q] : from_key<kDtype>(s_keys[q]);
}

// ---------------------------------------------------- large (multi-pass) --
// One 8-bit LSD pass over n keys is three launches: per-tile digit counts
// (digit-major: hist[d * ntiles + tile]), an exclusive scan of each digit's
// row with the row totals, and the stable scatter of every tile.

template <int kDtype, bool kFirst, bool kCanon>
__global__ void __launch_bounds__(kT) radix_count(const uint32_t *__restrict__ keys, int64_t n, int shift,
                                                  int64_t ntiles, uint32_t *__restrict__ hist) {
  __shared__ uint32_t s_cnt[kWarps][256];
  for (int i = threadIdx.x; i < kWarps * 256; i += kT) (&s_cnt[0][0])[i] = 0u;
  const int warp = threadIdx.x >> 5;
  const int64_t tile = reversed_tile();
  const int64_t base = tile * kTile;
  const int valid_n = (int)(n - base < (int64_t)kTile ? n - base : (int64_t)kTile);
  // All loads are issued before the first shared-memory atomic.
  uint32_t k[kItems];
  if (valid_n == kTile && (reinterpret_cast<uintptr_t>(keys) & 15) == 0) {
    const uint4 *v = reinterpret_cast<const uint4 *>(keys + base);
#pragma unroll
    for (int j = 0; j < kItems / 4; ++j) {
      const uint4 q = v[j * kT + threadIdx.x];
      k[4 * j] = q.x;
      k[4 * j + 1] = q.y;
      k[4 * j + 2] = q.z;
      k[4 * j + 3] = q.w;
    }
  } else {
#pragma unroll
    for (int i = 0; i < kItems; ++i) {
      const int q = (i >> 2) * kT * 4 + threadIdx.x * 4 + (i & 3);
      k[i] = q < valid_n ? keys[base + q] : 0u;
    }
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int q = (i >> 2) * kT * 4 + threadIdx.x * 4 + (i & 3);
    if (q < valid_n) {
      const uint32_t key = kFirst ? to_key<kDtype, kCanon>(k[i]) : k[i];
      atomicAdd(&s_cnt[warp][(key >> shift) & 255u], 1u);
    }
  }
  __syncthreads();
  const int d = threadIdx.x;
  uint32_t s = 0;
#pragma unroll
  for (int w = 0; w < kWarps; ++w) s += s_cnt[w][d];
  hist[(int64_t)d * ntiles + tile] = s;
}

// Exclusive sum of len values in[0..len) into out (may alias in) by one
// block, kScanItems consecutive values per thread per round; returns the
// total to every thread.
constexpr int kScanItems = 16;

template <typename In, typename Out>
__device__ __forceinline__ Out block_scan_array(const In *in, Out *out, int64_t len, Out *s_w) {
  Out run = 0;
  for (int64_t b = 0; b < len; b += (int64_t)kT * kScanItems) {
    const int64_t o = b + (int64_t)threadIdx.x * kScanItems;
    Out v[kScanItems], sum = 0;
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
      v[j] = o + j < len ? (Out)in[o + j] : Out(0);
      sum += v[j];
    }
    Out tot;
    Out r = run + block_excl_sum<Out>(sum, s_w, &tot);
#pragma unroll
    for (int j = 0; j < kScanItems; ++j) {
      if (o + j < len) out[o + j] = r;
      r += v[j];
    }
    run += tot;
  }
  return run;
}

// Block d: exclusive scan of digit d's per-tile counts in place; the row
// total goes to totals[d].
__global__ void __launch_bounds__(kT) radix_scan_rows(uint32_t *__restrict__ hist, int64_t ntiles,
                                                      uint32_t *__restrict__ totals) {
  __shared__ uint32_t s_w[kWarps];
  uint32_t *row = hist + (int64_t)blockIdx.x * ntiles;
  const uint32_t run = block_scan_array<uint32_t, uint32_t>(row, row, ntiles, s_w);
  if (threadIdx.x == 0) totals[blockIdx.x] = run;
}

// Stable scatter of one tile.  kFirst: keys come raw from the input and the
// values are generated (source indices).  kLast: keys leave in their original
// bit pattern.  kKeys / kVals: which streams are written.  Three blocks per
// SM (80 registers, a few spilled): the first pass waits on its loads, and
// 24 warps hide that latency better than 16 (2^26 f32 keys: 2.25 -> 1.84 ms
// per sort together with the leaner ranking above).
template <int kDtype, bool kFirst, bool kLast, bool kCanon, bool kKeys, bool kVals>
__global__ void __launch_bounds__(kT, 3) radix_scatter(const uint32_t *__restrict__ kin, const uint32_t *__restrict__ vin,
                                                    uint32_t *__restrict__ kout, uint32_t *__restrict__ vout,
                                                    int64_t n, int shift, int64_t ntiles,
                                                    const uint32_t *__restrict__ hist,
                                                    const uint32_t *__restrict__ totals) {
  __shared__ uint32_t s_keys[kTile];
  __shared__ uint32_t s_vals[kVals ? kTile : 1];
  __shared__ uint32_t s_wcnt[kWarps][256];
  __shared__ int64_t s_delta[256];
  __shared__ uint32_t s_w[kWarps];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t base = (int64_t)blockIdx.x * kTile;
  const int valid_n = (int)(n - base < (int64_t)kTile ? n - base : (int64_t)kTile);
  // Global start of this tile's keys of digit d.
  {
    const int d = threadIdx.x;
    const uint32_t digit_base = block_excl_sum<uint32_t>(totals[d], s_w);
    s_delta[d] = (int64_t)digit_base + hist[(int64_t)d * ntiles + blockIdx.x];
  }
  uint32_t k[kItems], v[kItems], pos[kItems];
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int q = warp * 32 * kItems + i * 32 + lane;
    const int64_t idx = base + q;
    if (q < valid_n) {
      const uint32_t raw = kin[idx];
      k[i] = kFirst ? to_key<kDtype, kCanon>(raw) : raw;
      if (kVals) v[i] = kFirst ? (uint32_t)idx : vin[idx];
    } else {
      k[i] = 0u;
      v[i] = 0u;
    }
  }
  rank_digits<kItems>(k, valid_n, shift, pos, s_wcnt, s_w);
  // s_wcnt[0][d] is now the tile-local start of digit d.
  {
    const int d = threadIdx.x;
    s_delta[d] -= (int64_t)s_wcnt[0][d];
  }
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int q = warp * 32 * kItems + i * 32 + lane;
    if (q < valid_n && pos[i] < (uint32_t)valid_n) {
      s_keys[pos[i]] = k[i];
      if (kVals) s_vals[pos[i]] = v[i];
    }
  }
  __syncthreads();
  for (int p = threadIdx.x; p < valid_n; p += kT) {
    const uint32_t key = s_keys[p];
    const int64_t g = s_delta[(key >> shift) & 255u] + p;
    if (g < 0 || g >= n) continue;  // unreachable with consistent counts; never write outside
    if (kKeys) kout[g] = kLast ? from_key<kDtype>(key) : key;
    if (kVals) vout[g] = s_vals[p];
  }
}

size_t large_sort_ws_bytes(int64_t n, bool grade) {
  const int64_t ntiles = (n + kTile - 1) / kTile;
  size_t b = align256((size_t)256 * ntiles * 4) + align256(256 * 4) + align256((size_t)n * 4);
  if (grade) b += 2 * align256((size_t)n * 4);
  return b;
}

// Sorts (or grades) one contiguous run of n keys.  sort: out receives the
// sorted values; grade: out receives int32 source indices.  `ws` holds
// large_sort_ws_bytes(n, grade) bytes.
template <int kDtype>
int large_sort(const uint32_t *in, uint32_t *out, int64_t n, bool grade, char *ws, cudaStream_t s) {
  const int64_t ntiles = (n + kTile - 1) / kTile;
  uint32_t *hist = reinterpret_cast<uint32_t *>(ws);
  uint32_t *totals = reinterpret_cast<uint32_t *>(ws + align256((size_t)256 * ntiles * 4));
  uint32_t *kw = reinterpret_cast<uint32_t *>(ws + align256((size_t)256 * ntiles * 4) + align256(256 * 4));
  uint32_t *kw2 = grade ? kw + align256((size_t)n * 4) / 4 : nullptr;
  uint32_t *vw = grade ? kw2 + align256((size_t)n * 4) / 4 : nullptr;
  const unsigned g = (unsigned)ntiles;
  auto count = [&](const uint32_t *src, int shift, bool first) {
    note_launch();
    if (first) {
      if (grade) radix_count<kDtype, true, true><<<g, kT, 0, s>>>(src, n, shift, ntiles, hist);
      else radix_count<kDtype, true, false><<<g, kT, 0, s>>>(src, n, shift, ntiles, hist);
    } else {
      radix_count<kDtype, false, false><<<g, kT, 0, s>>>(src, n, shift, ntiles, hist);
    }
    note_launch();
    radix_scan_rows<<<256, kT, 0, s>>>(hist, ntiles, totals);
  };
  if (!grade) {
    // in -> kw -> out -> kw -> out
    count(in, 0, true);
    note_launch();
    radix_scatter<kDtype, true, false, false, true, false>
        <<<g, kT, 0, s>>>(in, nullptr, kw, nullptr, n, 0, ntiles, hist, totals);
    count(kw, 8, false);
    note_launch();
    radix_scatter<kDtype, false, false, false, true, false>
        <<<g, kT, 0, s>>>(kw, nullptr, out, nullptr, n, 8, ntiles, hist, totals);
    count(out, 16, false);
    note_launch();
    radix_scatter<kDtype, false, false, false, true, false>
        <<<g, kT, 0, s>>>(out, nullptr, kw, nullptr, n, 16, ntiles, hist, totals);
    count(kw, 24, false);
    note_launch();
    radix_scatter<kDtype, false, true, false, true, false>
        <<<g, kT, 0, s>>>(kw, nullptr, out, nullptr, n, 24, ntiles, hist, totals);
  } else {
    // keys: in -> kw -> kw2 -> kw -> (dropped); indices: gen -> vw -> out -> vw -> out
    count(in, 0, true);
    note_launch();
    radix_scatter<kDtype, true, false, true, true, true>
        <<<g, kT, 0, s>>>(in, nullptr, kw, vw, n, 0, ntiles, hist, totals);
    count(kw, 8, false);
    note_launch();
    radix_scatter<kDtype, false, false, true, true, true>
        <<<g, kT, 0, s>>>(kw, vw, kw2, out, n, 8, ntiles, hist, totals);
    count(kw2, 16, false);
    note_launch();
    radix_scatter<kDtype, false, false, true, true, true>
        <<<g, kT, 0, s>>>(kw2, out, kw, vw, n, 16, ntiles, hist, totals);
    count(kw, 24, false);
    note_launch();
    radix_scatter<kDtype, false, false, true, false, true>
        <<<g, kT, 0, s>>>(kw, vw, nullptr, out, n, 24, ntiles, hist, totals);
  }
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

template <int kDtype, bool kGrade>
int small_sort(const uint32_t *in, int64_t in_stride, uint32_t *out, int64_t out_stride, int64_t rows, int len,
               cudaStream_t s) {
  note_launch();
  const unsigned g = (unsigned)rows;
  if (len <= kT) sort_rows_small<kDtype, 1, kGrade><<<g, kT, 0, s>>>(in, in_stride, out, out_stride, len);
  else if (len <= kT * 4) sort_rows_small<kDtype, 4, kGrade><<<g, kT, 0, s>>>(in, in_stride, out, out_stride, len);
  else sort_rows_small<kDtype, 16, kGrade><<<g, kT, 0, s>>>(in, in_stride, out, out_stride, len);
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

template <int kDtype>
int sort_rows(const uint32_t *in, uint32_t *out, int64_t rows, int64_t len, bool grade, char *ws,
              cudaStream_t s) {
  if (rows == 0 || len == 0) return REMORA_OK;
  if (len <= kSmallMax) {
    return grade ? small_sort<kDtype, true>(in, len, out, len, rows, (int)len, s)
                 : small_sort<kDtype, false>(in, len, out, len, rows, (int)len, s);
  }
  for (int64_t r = 0; r < rows; ++r) REMORA_TRY(large_sort<kDtype>(in + r * len, out + r * len, len, grade, ws, s));
  return REMORA_OK;
}

int sort_or_grade(RemoraB200Ctx *ctx, int32_t dtype, const void *in_desc, void *out_desc, int32_t rank,
                  bool grade, cudaStream_t s) {
  const char *what = grade ? "grade" : "sort";
  REMORA_TRY(check_ctx(ctx));
  if (dtype != REMORA_F32 && dtype != REMORA_I32)
    return fail(REMORA_ERR_UNSUPPORTED, "%s: dtype %d (f32 and i32 only, as remora_rt.c)", what, dtype);
  if (rank < 1 || rank > 2) return fail(REMORA_ERR_RANK, "%s: rank %d (ranks 1 and 2)", what, rank);
  DescView in, out;
  REMORA_TRY(read_desc(in_desc, rank, &in, what));
  REMORA_TRY(read_desc(out_desc, rank, &out, what));
  for (int d = 0; d < rank; ++d)
    if (in.sizes[d] != out.sizes[d]) return fail(REMORA_ERR_SHAPE, "%s: output shape differs from input", what);
  const int64_t len = in.sizes[rank - 1];
  const int64_t rows = rank == 2 ? in.sizes[0] : 1;
  if (len >= kMaxSortLen) return fail(REMORA_ERR_LIMIT, "%s: %lld keys per row (at most 2^31 - 1)", what, (long long)len);
  if (rows == 0 || len == 0) return REMORA_OK;
  const size_t bytes = (size_t)rows * len * 4;
  size_t need = len > kSmallMax ? large_sort_ws_bytes(len, grade) : 0;
  const size_t core = align256(need);
  if (!in.contiguous()) need = core + align256(bytes);
  if (!out.contiguous()) need = align256(need) + align256(bytes);
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, s, std::max<size_t>(need, 256), &ws));
  char *base = (char *)ws->buf;
  size_t used = core;
  const uint32_t *x = reinterpret_cast<const uint32_t *>(in.data(4));
  if (!in.contiguous()) {
    REMORA_TRY(copy_to_contiguous(in, 4, base + used, s, ctx->sm_count));
    x = reinterpret_cast<const uint32_t *>(base + used);
    used += align256(bytes);
  }
  uint32_t *y = out.contiguous() ? reinterpret_cast<uint32_t *>(out.data(4)) : reinterpret_cast<uint32_t *>(base + used);
  const int st = dtype == REMORA_F32 ? sort_rows<REMORA_F32>(x, y, rows, len, grade, base, s)
                                     : sort_rows<REMORA_I32>(x, y, rows, len, grade, base, s);
  REMORA_TRY(st);
  if (!out.contiguous()) REMORA_TRY(copy_from_contiguous(y, out, 4, s, ctx->sm_count));
  return REMORA_OK;
}

// -------------------------------------------------------------- filter --
// Keep flags: an i32 mask (remora_rt.c's form), a one-byte bool mask, or a
// comparison of the value against a literal evaluated in the kernel (the
// lowering's mask program, tensor_ops.py:2697-2706, fused away).  Float
// comparisons are ordered, like arith.cmpf o** (tensor_ops.py:2657-2663):
// NaN compares false, `!=` included.
enum { kMaskI32 = 0, kMaskU8 = 1, kMaskPred = 2 };

struct Pred {
  int op;
  float f;
  int i;
};

template <typename T>
__device__ __forceinline__ bool compare(int op, T x, T lit) {
  switch (op) {
    case REMORA_OP_LT: return x < lit;
    case REMORA_OP_LE: return x <= lit;
    case REMORA_OP_GT: return x > lit;
    case REMORA_OP_GE: return x >= lit;
    case REMORA_OP_EQ: return x == lit;
    default: return x < lit || x > lit;  // REMORA_OP_NE, ordered
  }
}

// The word a keep flag is computed from: the mask element, or the value.
template <typename T, int kMask>
__device__ __forceinline__ uint32_t flag_word(const T *__restrict__ src, const void *__restrict__ mask, int64_t i) {
  if (kMask == kMaskI32) return (uint32_t)reinterpret_cast<const int32_t *>(mask)[i];
  if (kMask == kMaskU8) return reinterpret_cast<const uint8_t *>(mask)[i];
  return *reinterpret_cast<const uint32_t *>(src + i);
}

template <typename T, int kMask>
__device__ __forceinline__ bool keep_word(uint32_t w, Pred p) {
  if (kMask != kMaskPred) return w != 0u;
  if constexpr (std::is_same<T, float>::value) return compare<float>(p.op, __uint_as_float(w), p.f);
  else return compare<int>(p.op, (int)w, p.i);
}

template <typename T, int kMask>
__global__ void __launch_bounds__(kT) filter_count(const T *__restrict__ src, const void *__restrict__ mask,
                                                   int64_t n, Pred p, uint32_t *__restrict__ tile_cnt) {
  __shared__ uint32_t s_w[kWarps];
  const int64_t tile = reversed_tile();
  const int64_t base = tile * kTile;
  uint32_t w[kItems];
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int64_t idx = base + i * kT + threadIdx.x;
    w[i] = idx < n ? flag_word<T, kMask>(src, mask, idx) : 0u;
  }
  uint32_t c = 0;
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int64_t idx = base + i * kT + threadIdx.x;
    if (idx < n && keep_word<T, kMask>(w[i], p)) ++c;
  }
  uint32_t total;
  (void)block_excl_sum<uint32_t>(c, s_w, &total);
  if (threadIdx.x == 0) tile_cnt[tile] = total;
}

// One block: exclusive scan of ntiles 32/64-bit counts into 64-bit offsets,
// and the grand total into *total.
template <typename C>
__global__ void __launch_bounds__(kT) tile_offsets(const C *__restrict__ cnt, int64_t ntiles,
                                                   unsigned long long *__restrict__ offs,
                                                   long long *__restrict__ total) {
  __shared__ unsigned long long s_w[kWarps];
  const unsigned long long run = block_scan_array<C, unsigned long long>(cnt, offs, ntiles, s_w);
  if (threadIdx.x == 0) *total = (long long)run;
}

// Compaction of one tile: keys are read in 16 rounds of kT consecutive
// elements; per (round, warp) a ballot gives the kept lanes, and one warp
// scans the 16 x 8 counts into offsets in input order.  The kept values are
// packed in shared memory and written out contiguously.
template <typename T, int kMask>
__global__ void __launch_bounds__(kT) filter_compact(const T *__restrict__ src, const void *__restrict__ mask,
                                                     int64_t n, Pred p, const unsigned long long *__restrict__ offs,
                                                     T *__restrict__ dst, int64_t cap) {
  __shared__ T s_out[kTile];
  __shared__ uint32_t s_cnt[kItems * kWarps];
  __shared__ uint32_t s_kept;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t base = (int64_t)blockIdx.x * kTile;
  T v[kItems];
  uint32_t ball[kItems];
  // All loads first, then the flags.
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int64_t idx = base + i * kT + threadIdx.x;
    v[i] = idx < n ? src[idx] : T(0);
    ball[i] = kMask == kMaskPred ? 0u : (idx < n ? flag_word<T, kMask>(src, mask, idx) : 0u);
  }
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int64_t idx = base + i * kT + threadIdx.x;
    uint32_t word = ball[i];
    if (kMask == kMaskPred) word = *reinterpret_cast<const uint32_t *>(&v[i]);
    const bool f = idx < n && keep_word<T, kMask>(word, p);
    ball[i] = __ballot_sync(0xffffffffu, f);
    if (lane == 0) s_cnt[i * kWarps + warp] = __popc(ball[i]);
  }
  __syncthreads();
  if (warp == 0) {
    // 128 counts, 4 per lane, in (round, warp) order.
    uint32_t c[4], sum = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      c[j] = s_cnt[lane * 4 + j];
      sum += c[j];
    }
    uint32_t inc = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const uint32_t up = __shfl_up_sync(0xffffffffu, inc, o);
      if (lane >= o) inc += up;
    }
    uint32_t run = inc - sum;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      s_cnt[lane * 4 + j] = run;
      run += c[j];
    }
    if (lane == 31) s_kept = inc;
  }
  __syncthreads();
  const uint32_t lt = (1u << lane) - 1u;
#pragma unroll
  for (int i = 0; i < kItems; ++i)
    if (ball[i] >> lane & 1u) s_out[s_cnt[i * kWarps + warp] + __popc(ball[i] & lt)] = v[i];
  __syncthreads();
  const int64_t o = (int64_t)offs[blockIdx.x];
  const int kept = (int)s_kept;
  for (int q = threadIdx.x; q < kept; q += kT)
    if (o + q < cap) dst[o + q] = s_out[q];
}

// ----------------------------------------------------------- replicate --
__device__ __forceinline__ unsigned long long clamp_count(int32_t c) { return c > 0 ? (unsigned long long)c : 0ull; }

__global__ void __launch_bounds__(kT) rep_tile_sums(const int32_t *__restrict__ cnt, int64_t n,
                                                    unsigned long long *__restrict__ sums) {
  __shared__ unsigned long long s_w[kWarps];
  const int64_t tile = reversed_tile();
  const int64_t base = tile * kTile;
  unsigned long long c = 0;
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int64_t idx = base + i * kT + threadIdx.x;
    if (idx < n) c += clamp_count(cnt[idx]);
  }
  unsigned long long total;
  (void)block_excl_sum<unsigned long long>(c, s_w, &total);
  if (threadIdx.x == 0) sums[tile] = total;
}

// offs[i] = sum of clamped counts before i.  The tile's counts are staged in
// shared memory (rows of kItems + 1 words, so that reading a thread's
// kItems consecutive counts spreads the lanes over the banks) and each
// thread sums kItems consecutive ones.
constexpr int kPadRow = kItems + 1;

__global__ void __launch_bounds__(kT) rep_offsets(const int32_t *__restrict__ cnt, int64_t n,
                                                  const unsigned long long *__restrict__ tile_offs,
                                                  unsigned long long *__restrict__ offs) {
  __shared__ unsigned long long s_v[kT * kPadRow];
  __shared__ unsigned long long s_w[kWarps];
  const int64_t base = (int64_t)blockIdx.x * kTile;
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int e = i * kT + threadIdx.x;
    const int64_t idx = base + e;
    s_v[(e / kItems) * kPadRow + e % kItems] = idx < n ? clamp_count(cnt[idx]) : 0ull;
  }
  __syncthreads();
  unsigned long long mine[kItems], sum = 0;
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    mine[j] = s_v[threadIdx.x * kPadRow + j];
    sum += mine[j];
  }
  unsigned long long run = tile_offs[blockIdx.x] + block_excl_sum<unsigned long long>(sum, s_w);
#pragma unroll
  for (int j = 0; j < kItems; ++j) {
    s_v[threadIdx.x * kPadRow + j] = run;
    run += mine[j];
  }
  __syncthreads();
#pragma unroll
  for (int i = 0; i < kItems; ++i) {
    const int e = i * kT + threadIdx.x;
    const int64_t idx = base + e;
    if (idx < n) offs[idx] = s_v[(e / kItems) * kPadRow + e % kItems];
  }
}

// Last index in [lo, hi] whose offset is <= j (offsets are non-decreasing
// and offs[lo] <= j).  A source with a zero count has the same offset as the
// next one, so the last such index is always a source with a count >= 1.
template <typename P>
__device__ __forceinline__ int64_t last_le(const P *offs, int64_t lo, int64_t hi, unsigned long long j) {
  while (lo < hi) {
    const int64_t mid = lo + (hi - lo + 1) / 2;
    if (offs[mid] <= j) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

// Output tiles of kTile positions, grid-strided (the total is only known on
// the device).  Each tile finds its source range with two searches; when the
// range fits in shared memory its offsets are staged there for the
// per-element searches.
template <typename T>
__global__ void __launch_bounds__(kT) rep_fill(const T *__restrict__ src, const unsigned long long *__restrict__ offs,
                                               int64_t n, const long long *__restrict__ total, int64_t cap,
                                               T *__restrict__ dst) {
  __shared__ unsigned long long s_offs[kTile];
  __shared__ int64_t s_lo, s_hi;
  const long long limit = *total < (long long)cap ? *total : (long long)cap;
  for (long long j0 = (long long)blockIdx.x * kTile; j0 < limit; j0 += (long long)gridDim.x * kTile) {
    const long long j1 = j0 + kTile < limit ? j0 + kTile : limit;
    if (threadIdx.x == 0) s_lo = last_le(offs, 0, n - 1, (unsigned long long)j0);
    if (threadIdx.x == 32) s_hi = last_le(offs, 0, n - 1, (unsigned long long)(j1 - 1));
    __syncthreads();
    const int64_t lo = s_lo, hi = s_hi;
    const bool staged = hi - lo + 1 <= kTile;
    if (staged)
      for (int64_t i = lo + threadIdx.x; i <= hi; i += kT) s_offs[i - lo] = offs[i];
    __syncthreads();
    for (long long j = j0 + threadIdx.x; j < j1; j += kT) {
      const int64_t i = staged ? lo + last_le(s_offs, 0, hi - lo, (unsigned long long)j)
                               : last_le(offs, lo, hi, (unsigned long long)j);
      dst[j] = src[i];
    }
    __syncthreads();
  }
}

// ------------------------------------------------- rotate / append copy --
// out[j] = j < split ? a[j] : b[j - split], over `total` elements of type V
// (a 16-byte vector when every address and length allows it).
template <typename V>
__global__ void __launch_bounds__(kT) two_segment_copy(const V *__restrict__ a, const V *__restrict__ b,
                                                       V *__restrict__ out, int64_t split, int64_t total) {
  const int64_t step = (int64_t)gridDim.x * kT;
  for (int64_t j = (int64_t)blockIdx.x * kT + threadIdx.x; j < total; j += step)
    out[j] = j < split ? a[j] : b[j - split];
}

int launch_two_segment(const char *a, const char *b, char *out, int64_t split_bytes, int64_t total_bytes,
                       int sm_count, cudaStream_t s) {
  if (total_bytes == 0) return REMORA_OK;
  auto grid = [&](int64_t n) {
    return (unsigned)std::max<int64_t>(1, std::min<int64_t>((n + kT - 1) / kT, (int64_t)sm_count * 8));
  };
  const bool vec = ((uintptr_t)a % 16 == 0) && ((uintptr_t)b % 16 == 0) && ((uintptr_t)out % 16 == 0) &&
                   split_bytes % 16 == 0 && total_bytes % 16 == 0;
  note_launch();
  if (vec) {
    two_segment_copy<uint4><<<grid(total_bytes / 16), kT, 0, s>>>(
        reinterpret_cast<const uint4 *>(a), reinterpret_cast<const uint4 *>(b), reinterpret_cast<uint4 *>(out),
        split_bytes / 16, total_bytes / 16);
  } else if (split_bytes % 4 == 0 && total_bytes % 4 == 0 && (uintptr_t)a % 4 == 0 && (uintptr_t)b % 4 == 0 &&
             (uintptr_t)out % 4 == 0) {
    two_segment_copy<uint32_t><<<grid(total_bytes / 4), kT, 0, s>>>(
        reinterpret_cast<const uint32_t *>(a), reinterpret_cast<const uint32_t *>(b),
        reinterpret_cast<uint32_t *>(out), split_bytes / 4, total_bytes / 4);
  } else {
    two_segment_copy<uint8_t><<<grid(total_bytes), kT, 0, s>>>(reinterpret_cast<const uint8_t *>(a),
                                                              reinterpret_cast<const uint8_t *>(b),
                                                              reinterpret_cast<uint8_t *>(out), split_bytes,
                                                              total_bytes);
  }
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

int elem_size(int32_t dtype, const char *what) {
  const int es = dtype_size(dtype);
  if (es <= 0) return fail(REMORA_ERR_UNSUPPORTED, "%s: dtype %d", what, dtype);
  return es;
}

}  // namespace
}  // namespace remora

using namespace remora;

extern "C" int remora_b200_sort(RemoraB200Ctx *ctx, int32_t dtype, const void *in_desc, void *out_desc,
                                int32_t rank, remora_stream_t stream) {
  return sort_or_grade(ctx, dtype, in_desc, out_desc, rank, false, (cudaStream_t)stream);
}

extern "C" int remora_b200_grade(RemoraB200Ctx *ctx, int32_t dtype, const void *in_desc, void *out_desc,
                                 int32_t rank, remora_stream_t stream) {
  return sort_or_grade(ctx, dtype, in_desc, out_desc, rank, true, (cudaStream_t)stream);
}

extern "C" int remora_b200_filter(RemoraB200Ctx *ctx, int32_t dtype, const void *src_desc, const void *mask_desc,
                                  int32_t mask_dtype, const RemoraFilterPred *pred, void *dst_desc,
                                  RemoraMemRef0 *count_desc, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (dtype != REMORA_F32 && dtype != REMORA_I32)
    return fail(REMORA_ERR_UNSUPPORTED, "filter: dtype %d (f32 and i32 only, as remora_rt.c)", dtype);
  if (count_desc == nullptr || count_desc->aligned == nullptr) return fail(REMORA_ERR_ARG, "filter: null count");
  if ((mask_desc == nullptr) == (pred == nullptr))
    return fail(REMORA_ERR_ARG, "filter: give exactly one of a mask and a predicate");
  Pred p{REMORA_OP_NE, 0.0f, 0};
  int kind = kMaskPred;
  if (pred) {
    if (pred->op < REMORA_OP_LT || pred->op > REMORA_OP_NE)
      return fail(REMORA_ERR_UNSUPPORTED, "filter: predicate op %d is not a comparison", pred->op);
    p = Pred{pred->op, pred->lit_f, pred->lit_i};
  } else if (mask_dtype == REMORA_I32) {
    kind = kMaskI32;
  } else if (mask_dtype == REMORA_BOOL) {
    kind = kMaskU8;
  } else {
    return fail(REMORA_ERR_UNSUPPORTED, "filter: mask dtype %d (i32 or bool)", mask_dtype);
  }
  DescView src, mask, dst;
  REMORA_TRY(read_desc(src_desc, 1, &src, "filter source"));
  REMORA_TRY(read_desc(dst_desc, 1, &dst, "filter destination"));
  if (!dst.contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "filter: the destination must be contiguous");
  if (mask_desc) {
    REMORA_TRY(read_desc(mask_desc, 1, &mask, "filter mask"));
    if (mask.sizes[0] != src.sizes[0]) return fail(REMORA_ERR_SHAPE, "filter: mask length differs from source");
  }
  const int64_t n = src.sizes[0];
  if (n >= kMaxSortLen) return fail(REMORA_ERR_LIMIT, "filter: %lld elements (at most 2^31 - 1)", (long long)n);
  const int mes = kind == kMaskU8 ? 1 : 4;
  const int64_t ntiles = std::max<int64_t>(1, (n + kTile - 1) / kTile);
  size_t need = align256((size_t)ntiles * 4) + align256((size_t)ntiles * 8);
  const size_t core = need;
  if (!src.contiguous()) need += align256((size_t)n * 4);
  if (mask_desc && !mask.contiguous()) need += align256((size_t)n * mes);
  cudaStream_t s = (cudaStream_t)stream;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, s, need, &ws));
  char *base = (char *)ws->buf;
  uint32_t *tile_cnt = reinterpret_cast<uint32_t *>(base);
  unsigned long long *offs = reinterpret_cast<unsigned long long *>(base + align256((size_t)ntiles * 4));
  size_t used = core;
  const void *x = src.data(4);
  if (!src.contiguous()) {
    REMORA_TRY(copy_to_contiguous(src, 4, base + used, s, ctx->sm_count));
    x = base + used;
    used += align256((size_t)n * 4);
  }
  const void *m = mask_desc ? (const void *)mask.data(mes) : nullptr;
  if (mask_desc && !mask.contiguous()) {
    REMORA_TRY(copy_to_contiguous(mask, mes, base + used, s, ctx->sm_count));
    m = base + used;
    used += align256((size_t)n * mes);
  }
  void *y = dst.data(4);
  long long *count = reinterpret_cast<long long *>(static_cast<char *>(count_desc->aligned) + count_desc->offset * 8);
  const unsigned g = (unsigned)ntiles;
#define REMORA_FILTER_LAUNCH(T, K)                                                                       \
  do {                                                                                                   \
    note_launch();                                                                                       \
    filter_count<T, K><<<g, kT, 0, s>>>((const T *)x, m, n, p, tile_cnt);                                \
    note_launch();                                                                                       \
    tile_offsets<uint32_t><<<1, kT, 0, s>>>(tile_cnt, ntiles, offs, count);                              \
    note_launch();                                                                                       \
    filter_compact<T, K><<<g, kT, 0, s>>>((const T *)x, m, n, p, offs, (T *)y, dst.sizes[0]);            \
  } while (0)
  if (dtype == REMORA_F32) {
    if (kind == kMaskI32) REMORA_FILTER_LAUNCH(float, kMaskI32);
    else if (kind == kMaskU8) REMORA_FILTER_LAUNCH(float, kMaskU8);
    else REMORA_FILTER_LAUNCH(float, kMaskPred);
  } else {
    if (kind == kMaskI32) REMORA_FILTER_LAUNCH(int32_t, kMaskI32);
    else if (kind == kMaskU8) REMORA_FILTER_LAUNCH(int32_t, kMaskU8);
    else REMORA_FILTER_LAUNCH(int32_t, kMaskPred);
  }
#undef REMORA_FILTER_LAUNCH
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

extern "C" int remora_b200_replicate(RemoraB200Ctx *ctx, int32_t dtype, const void *src_desc,
                                     const void *counts_desc, void *dst_desc, RemoraMemRef0 *total_desc,
                                     remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (dtype != REMORA_F32 && dtype != REMORA_I32)
    return fail(REMORA_ERR_UNSUPPORTED, "replicate: dtype %d (f32 and i32 only, as remora_rt.c)", dtype);
  if (total_desc == nullptr || total_desc->aligned == nullptr) return fail(REMORA_ERR_ARG, "replicate: null total");
  DescView src, cnt, dst;
  REMORA_TRY(read_desc(src_desc, 1, &src, "replicate source"));
  REMORA_TRY(read_desc(counts_desc, 1, &cnt, "replicate counts"));
  if (cnt.sizes[0] != src.sizes[0]) return fail(REMORA_ERR_SHAPE, "replicate: counts length differs from source");
  if (dst_desc) {
    REMORA_TRY(read_desc(dst_desc, 1, &dst, "replicate destination"));
    if (!dst.contiguous()) return fail(REMORA_ERR_UNSUPPORTED, "replicate: the destination must be contiguous");
  }
  const int64_t n = src.sizes[0];
  if (n >= kMaxSortLen) return fail(REMORA_ERR_LIMIT, "replicate: %lld elements (at most 2^31 - 1)", (long long)n);
  const int64_t ntiles = std::max<int64_t>(1, (n + kTile - 1) / kTile);
  size_t need = 2 * align256((size_t)ntiles * 8) + align256((size_t)n * 8);
  const size_t core = need;
  if (!src.contiguous()) need += align256((size_t)n * 4);
  if (!cnt.contiguous()) need += align256((size_t)n * 4);
  cudaStream_t s = (cudaStream_t)stream;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, s, need, &ws));
  char *base = (char *)ws->buf;
  unsigned long long *sums = reinterpret_cast<unsigned long long *>(base);
  unsigned long long *toffs = reinterpret_cast<unsigned long long *>(base + align256((size_t)ntiles * 8));
  unsigned long long *offs = reinterpret_cast<unsigned long long *>(base + 2 * align256((size_t)ntiles * 8));
  size_t used = core;
  const void *x = src.data(4);
  if (!src.contiguous()) {
    REMORA_TRY(copy_to_contiguous(src, 4, base + used, s, ctx->sm_count));
    x = base + used;
    used += align256((size_t)n * 4);
  }
  const int32_t *c = reinterpret_cast<const int32_t *>(cnt.data(4));
  if (!cnt.contiguous()) {
    REMORA_TRY(copy_to_contiguous(cnt, 4, base + used, s, ctx->sm_count));
    c = reinterpret_cast<const int32_t *>(base + used);
    used += align256((size_t)n * 4);
  }
  long long *total = reinterpret_cast<long long *>(static_cast<char *>(total_desc->aligned) + total_desc->offset * 8);
  const unsigned g = (unsigned)ntiles;
  note_launch();
  rep_tile_sums<<<g, kT, 0, s>>>(c, n, sums);
  note_launch();
  tile_offsets<unsigned long long><<<1, kT, 0, s>>>(sums, ntiles, toffs, total);
  if (dst_desc && n > 0 && dst.sizes[0] > 0) {
    note_launch();
    rep_offsets<<<g, kT, 0, s>>>(c, n, toffs, offs);
    const unsigned fill_grid = (unsigned)std::max<int64_t>(
        1, std::min<int64_t>((dst.sizes[0] + kTile - 1) / kTile, (int64_t)ctx->sm_count * 4));
    note_launch();
    if (dtype == REMORA_F32)
      rep_fill<float><<<fill_grid, kT, 0, s>>>((const float *)x, offs, n, total, dst.sizes[0], (float *)dst.data(4));
    else
      rep_fill<int32_t><<<fill_grid, kT, 0, s>>>((const int32_t *)x, offs, n, total, dst.sizes[0],
                                                 (int32_t *)dst.data(4));
  }
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

extern "C" int remora_b200_rotate(RemoraB200Ctx *ctx, int32_t dtype, int64_t shift, const void *in_desc,
                                  void *out_desc, int32_t rank, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  const int es = elem_size(dtype, "rotate");
  if (es < 0) return es;
  if (rank < 1 || rank > REMORA_MAX_RANK) return fail(REMORA_ERR_RANK, "rotate: rank %d (needs >= 1)", rank);
  DescView in, out;
  REMORA_TRY(read_desc(in_desc, rank, &in, "rotate input"));
  REMORA_TRY(read_desc(out_desc, rank, &out, "rotate output"));
  for (int d = 0; d < rank; ++d)
    if (in.sizes[d] != out.sizes[d]) return fail(REMORA_ERR_SHAPE, "rotate: output shape differs from input");
  const int64_t N = in.sizes[0];
  const int64_t total = in.numel();
  if (total == 0) return REMORA_OK;
  const int64_t row = total / N;
  const int64_t k = ((shift % N) + N) % N;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t bytes = (size_t)total * es;
  size_t need = 0;
  if (!in.contiguous()) need += align256(bytes);
  if (!out.contiguous()) need += align256(bytes);
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, s, std::max<size_t>(need, 256), &ws));
  char *base = (char *)ws->buf;
  const char *x = in.data(es);
  if (!in.contiguous()) {
    REMORA_TRY(copy_to_contiguous(in, es, base, s, ctx->sm_count));
    x = base;
    base += align256(bytes);
  }
  char *y = out.contiguous() ? out.data(es) : base;
  REMORA_TRY(launch_two_segment(x + k * row * es, x, y, (N - k) * row * es, total * es, ctx->sm_count, s));
  if (!out.contiguous()) REMORA_TRY(copy_from_contiguous(y, out, es, s, ctx->sm_count));
  return REMORA_OK;
}

extern "C" int remora_b200_append(RemoraB200Ctx *ctx, int32_t dtype, const void *a_desc, const void *b_desc,
                                  void *out_desc, int32_t rank, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  const int es = elem_size(dtype, "append");
  if (es < 0) return es;
  if (rank < 1 || rank > REMORA_MAX_RANK) return fail(REMORA_ERR_RANK, "append: rank %d (needs >= 1)", rank);
  DescView a, b, out;
  REMORA_TRY(read_desc(a_desc, rank, &a, "append left"));
  REMORA_TRY(read_desc(b_desc, rank, &b, "append right"));
  REMORA_TRY(read_desc(out_desc, rank, &out, "append output"));
  if (out.sizes[0] != a.sizes[0] + b.sizes[0]) return fail(REMORA_ERR_SHAPE, "append: output length is not the sum");
  for (int d = 1; d < rank; ++d)
    if (a.sizes[d] != out.sizes[d] || b.sizes[d] != out.sizes[d])
      return fail(REMORA_ERR_SHAPE, "append: operands differ in a trailing axis");
  const int64_t total = out.numel();
  if (total == 0) return REMORA_OK;
  cudaStream_t s = (cudaStream_t)stream;
  const size_t abytes = (size_t)a.numel() * es, bbytes = (size_t)b.numel() * es, obytes = (size_t)total * es;
  size_t need = 0;
  if (!a.contiguous()) need += align256(abytes);
  if (!b.contiguous()) need += align256(bbytes);
  if (!out.contiguous()) need += align256(obytes);
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, s, std::max<size_t>(need, 256), &ws));
  char *base = (char *)ws->buf;
  const char *pa = a.data(es), *pb = b.data(es);
  if (!a.contiguous() && abytes) {
    REMORA_TRY(copy_to_contiguous(a, es, base, s, ctx->sm_count));
    pa = base;
    base += align256(abytes);
  }
  if (!b.contiguous() && bbytes) {
    REMORA_TRY(copy_to_contiguous(b, es, base, s, ctx->sm_count));
    pb = base;
    base += align256(bbytes);
  }
  char *y = out.contiguous() ? out.data(es) : base;
  REMORA_TRY(launch_two_segment(pa, pb, y, (int64_t)abytes, (int64_t)obytes, ctx->sm_count, s));
  if (!out.contiguous()) REMORA_TRY(copy_from_contiguous(y, out, es, s, ctx->sm_count));
  return REMORA_OK;
}
