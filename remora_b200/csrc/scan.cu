// scan.cu — scans along the leading axis (remora_b200_scan).
//
// Semantics follow the reference's CPU lowering
// (remora/lowering/tensor_ops.py:2301-2482) and interpreter
// (remora/runtime.py:1100-1123): rank 1 inclusive / exclusive / right, rank
// >= 2 inclusive along axis 0 with the other axes as independent columns.
//
// Algorithm: three-phase reduce-then-scan.  (1) every tile (rank 1: 2048
// consecutive elements; rank >= 2: a segment of rows for 256 columns)
// reduces to an aggregate; (2) one pass scans the aggregates into per-tile
// carries, starting from init; (3) every tile rescans its elements from its
// carry.  No block ever waits on another, so there is no spin loop to bound,
// and f32 results are bitwise reproducible run to run (the combine order is
// fixed); they differ from the sequential CPU order only by rounding.
#include <algorithm>

#include "common.cuh"

namespace remora {

namespace {

constexpr int kThreads = 256;
constexpr int kItems = 8;
constexpr int kTile = kThreads * kItems;

template <typename T, bool kMul>
struct ScanOp;
template <>
struct ScanOp<float, false> {
  static __device__ __forceinline__ float apply(float a, float b) { return __fadd_rn(a, b); }
  static __device__ __forceinline__ float ident() { return 0.0f; }
};
template <>
struct ScanOp<float, true> {
  static __device__ __forceinline__ float apply(float a, float b) { return __fmul_rn(a, b); }
  static __device__ __forceinline__ float ident() { return 1.0f; }
};
template <>
struct ScanOp<int, false> {
  static __device__ __forceinline__ int apply(int a, int b) { return (int)((unsigned)a + (unsigned)b); }
  static __device__ __forceinline__ int ident() { return 0; }
};
template <>
struct ScanOp<int, true> {
  static __device__ __forceinline__ int apply(int a, int b) { return (int)((unsigned)a * (unsigned)b); }
  static __device__ __forceinline__ int ident() { return 1; }
};

// Exclusive scan of one value per thread across the block (thread order).
template <typename T, typename Op>
__device__ __forceinline__ T block_exclusive(T v, T *sh_warp, T *total) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  T inc = v;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    T up = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = Op::apply(up, inc);
  }
  if (lane == 31) sh_warp[warp] = inc;
  __syncthreads();
  if (threadIdx.x == 0) {
    T run = Op::ident();
    for (int w = 0; w < kThreads / 32; ++w) {
      T t = sh_warp[w];
      sh_warp[w] = run;
      run = Op::apply(run, t);
    }
    *total = run;
  }
  __syncthreads();
  T excl_in_warp = __shfl_up_sync(0xffffffffu, inc, 1);
  if (lane == 0) excl_in_warp = Op::ident();
  T r = Op::apply(sh_warp[warp], excl_in_warp);
  __syncthreads();
  return r;
}

__device__ __forceinline__ int64_t phys(int64_t q, int64_t n, int right) { return right ? n - 1 - q : q; }

// The kItems (8) elements q = base .. base+7 of a tile row in scan order,
// and their stores.  Where the 8 physical elements are one aligned 32-byte
// run (whole tile slot, 16-byte aligned array, and for a right scan a
// length divisible by 4) they move as two 16-byte vectors, so the lanes of
// a warp cover 1 KB contiguously per pair of instructions; else one by one.
template <typename T>
__device__ __forceinline__ bool vec8(const T *p, int64_t base, int64_t n, int right) {
  return base + kItems <= n && (reinterpret_cast<uintptr_t>(p) & 15) == 0 && (!right || (n & 3) == 0);
}

template <typename T, typename Op>
__device__ __forceinline__ void load8(const T *__restrict__ x, int64_t base, int64_t n, int right, T (&v)[kItems]) {
  if (vec8(x, base, n, right)) {
    const int64_t p0 = right ? n - base - kItems : base;
    const uint4 a = __ldcs(reinterpret_cast<const uint4 *>(x + p0));
    const uint4 b = __ldcs(reinterpret_cast<const uint4 *>(x + p0 + 4));
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int k = 0; k < kItems; ++k) v[k] = __builtin_bit_cast(T, w[right ? kItems - 1 - k : k]);
  } else {
#pragma unroll
    for (int k = 0; k < kItems; ++k) v[k] = base + k < n ? x[phys(base + k, n, right)] : Op::ident();
  }
}

template <typename T>
__device__ __forceinline__ void store8(T *__restrict__ y, int64_t base, int64_t n, int right, const T (&v)[kItems]) {
  if (vec8(y, base, n, right)) {
    const int64_t p0 = right ? n - base - kItems : base;
    uint32_t w[8];
#pragma unroll
    for (int k = 0; k < kItems; ++k) w[right ? kItems - 1 - k : k] = __builtin_bit_cast(uint32_t, v[k]);
    __stcs(reinterpret_cast<uint4 *>(y + p0), make_uint4(w[0], w[1], w[2], w[3]));
    __stcs(reinterpret_cast<uint4 *>(y + p0 + 4), make_uint4(w[4], w[5], w[6], w[7]));
  } else {
#pragma unroll
    for (int k = 0; k < kItems; ++k)
      if (base + k < n) y[phys(base + k, n, right)] = v[k];
  }
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) tile_aggregate(const T *__restrict__ x, int64_t n, int right,
                                                          T *__restrict__ agg) {
  __shared__ T sh[kThreads / 32];
  __shared__ T total;
  const int64_t base = (int64_t)blockIdx.x * kTile + (int64_t)threadIdx.x * kItems;
  T v[kItems];
  load8<T, Op>(x, base, n, right, v);
  T acc = Op::ident();
#pragma unroll
  for (int k = 0; k < kItems; ++k)
    if (base + k < n) acc = Op::apply(acc, v[k]);
  (void)block_exclusive<T, Op>(acc, sh, &total);
  if (threadIdx.x == 0) agg[blockIdx.x] = total;
}

// One block turns the tile aggregates into per-tile carries: carry[0] = init,
// carry[t] = carry[t-1] op agg[t-1].  Thread i owns the run of `per`
// consecutive aggregates from i * per (per a multiple of 4, so runs start on
// 16-byte boundaries): it reduces its run with 16-byte reads, eight in
// flight, the block scans the 1024 run totals in thread order, and each
// thread rescans its run from its prefix.  The combine order is fixed, so
// results are reproducible run to run.
constexpr int kCarryThreads = 1024;

template <typename T>
__device__ __forceinline__ void load4(const T *__restrict__ p, T (&v)[4]) {
  const uint4 w = *reinterpret_cast<const uint4 *>(p);
  v[0] = __builtin_bit_cast(T, w.x), v[1] = __builtin_bit_cast(T, w.y);
  v[2] = __builtin_bit_cast(T, w.z), v[3] = __builtin_bit_cast(T, w.w);
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kCarryThreads) carries_rank1(const T *__restrict__ agg, T *__restrict__ carry,
                                                              int64_t ntiles, T init) {
  __shared__ T sh[kCarryThreads / 32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t per = ((ntiles + kCarryThreads - 1) / kCarryThreads + 3) & ~int64_t(3);
  const int64_t b0 = min(ntiles, (int64_t)threadIdx.x * per), b1 = min(ntiles, b0 + per);
  T acc = Op::ident();
  bool any = false;
  for (int64_t i = b0; i < b1; i += 32) {
    T v[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t q = i + 4 * j;
      if (q + 4 <= b1) {
        load4(agg + q, v[j]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[j][e] = q + e < b1 ? agg[q + e] : Op::ident();
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        if (i + 4 * j + e < b1) {
          acc = any ? Op::apply(acc, v[j][e]) : v[j][e];
          any = true;
        }
  }
  // exclusive scan of the run totals in thread order: lanes, then warps
  T inc = acc;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const T up = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc = Op::apply(up, inc);
  }
  if (lane == 31) sh[warp] = inc;
  __syncthreads();
  if (warp == 0) {
    T w = sh[lane], winc = w;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const T up = __shfl_up_sync(0xffffffffu, winc, o);
      if (lane >= o) winc = Op::apply(up, winc);
    }
    T wex = __shfl_up_sync(0xffffffffu, winc, 1);
    sh[lane] = lane == 0 ? init : Op::apply(init, wex);
  }
  __syncthreads();
  T ex = __shfl_up_sync(0xffffffffu, inc, 1);
  T run = lane == 0 ? sh[warp] : Op::apply(sh[warp], ex);
  // the run again, eight 16-byte reads in flight, carries written 16 bytes
  // at a time
  for (int64_t i = b0; i < b1; i += 32) {
    T v[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t q = i + 4 * j;
      if (q + 4 <= b1) {
        load4(agg + q, v[j]);
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e) v[j][e] = q + e < b1 ? agg[q + e] : Op::ident();
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int64_t q = i + 4 * j;
      T c[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        c[e] = run;
        if (q + e < b1) run = Op::apply(run, v[j][e]);
      }
      if (q + 4 <= b1) {
        *reinterpret_cast<uint4 *>(carry + q) =
            make_uint4(__builtin_bit_cast(uint32_t, c[0]), __builtin_bit_cast(uint32_t, c[1]),
                       __builtin_bit_cast(uint32_t, c[2]), __builtin_bit_cast(uint32_t, c[3]));
      } else {
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (q + e < b1) carry[q + e] = c[e];
      }
    }
  }
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) tile_scan(const T *__restrict__ x, T *__restrict__ y, int64_t n,
                                                     int right, int exclusive, const T *__restrict__ carry) {
  __shared__ T sh[kThreads / 32];
  __shared__ T total;
  const int64_t base = (int64_t)blockIdx.x * kTile + (int64_t)threadIdx.x * kItems;
  T v[kItems];
  load8<T, Op>(x, base, n, right, v);
  T acc = Op::ident();
#pragma unroll
  for (int k = 0; k < kItems; ++k) acc = Op::apply(acc, v[k]);
  T run = Op::apply(carry[blockIdx.x], block_exclusive<T, Op>(acc, sh, &total));
  T out[kItems];
#pragma unroll
  for (int k = 0; k < kItems; ++k) {
    if (exclusive) {
      out[k] = run;
      run = Op::apply(run, v[k]);
    } else {
      run = Op::apply(run, v[k]);
      out[k] = run;
    }
  }
  store8<T>(y, base, n, right, out);
}

// ---- rank >= 2: columns t in [0, T), rows split into segments.
template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) seg_aggregate(const T *__restrict__ x, int64_t N, int64_t C,
                                                         int64_t seg_rows, T *__restrict__ agg) {
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= C) return;
  const int64_t r0 = (int64_t)blockIdx.y * seg_rows, r1 = min(N, r0 + seg_rows);
  T acc = Op::ident();
  for (int64_t r = r0; r < r1; ++r) acc = Op::apply(acc, x[r * C + t]);
  agg[(int64_t)blockIdx.y * C + t] = acc;
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) seg_carries(const T *__restrict__ agg, T *__restrict__ carry,
                                                       int64_t C, int64_t nseg, T init) {
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= C) return;
  T run = init;
  for (int64_t s = 0; s < nseg; ++s) {
    carry[s * C + t] = run;
    run = Op::apply(run, agg[s * C + t]);
  }
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) seg_scan(const T *__restrict__ x, T *__restrict__ y, int64_t N,
                                                    int64_t C, int64_t seg_rows, const T *__restrict__ carry,
                                                    T init, int has_carry) {
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= C) return;
  const int64_t r0 = (int64_t)blockIdx.y * seg_rows, r1 = min(N, r0 + seg_rows);
  T run = has_carry ? carry[(int64_t)blockIdx.y * C + t] : init;
  for (int64_t r = r0; r < r1; ++r) {
    run = Op::apply(run, x[r * C + t]);
    y[r * C + t] = run;
  }
}

template <typename T, bool kMul>
int scan_impl(const T *x, T *y, int64_t N, int64_t C, int right, int exclusive, T init, char *scratch,
              size_t scratch_bytes, int sm_count, cudaStream_t stream) {
  using Op = ScanOp<T, kMul>;
  if (N == 0 || C == 0) return REMORA_OK;
  if (C == 1) {
    const int64_t ntiles = (N + kTile - 1) / kTile;
    T *agg = reinterpret_cast<T *>(scratch);
    T *carry = agg + ((ntiles + 63) & ~int64_t(63));
    if ((size_t)(2 * ((ntiles + 63) & ~int64_t(63))) * sizeof(T) > scratch_bytes)
      return fail(REMORA_ERR_LIMIT, "scan: scratch too small");
    note_launch();
    tile_aggregate<T, Op><<<(unsigned)ntiles, kThreads, 0, stream>>>(x, N, right, agg);
    note_launch();
    carries_rank1<T, Op><<<1, kCarryThreads, 0, stream>>>(agg, carry, ntiles, init);
    note_launch();
    tile_scan<T, Op><<<(unsigned)ntiles, kThreads, 0, stream>>>(x, y, N, right, exclusive, carry);
  } else {
    const int64_t cblocks = (C + kThreads - 1) / kThreads;
    const int64_t want_threads = (int64_t)sm_count * 2048;
    int64_t nseg = std::max<int64_t>(1, std::min<int64_t>(N, want_threads / std::max<int64_t>(C, 1)));
    nseg = std::min<int64_t>(nseg, 65535);
    const int64_t seg_rows = (N + nseg - 1) / nseg;
    nseg = (N + seg_rows - 1) / seg_rows;
    dim3 grid((unsigned)cblocks, (unsigned)nseg);
    if (nseg == 1) {
      note_launch();
      seg_scan<T, Op><<<grid, kThreads, 0, stream>>>(x, y, N, C, seg_rows, nullptr, init, 0);
    } else {
      T *agg = reinterpret_cast<T *>(scratch);
      T *carry = agg + nseg * C;
      if ((size_t)(2 * nseg * C) * sizeof(T) > scratch_bytes)
        return fail(REMORA_ERR_LIMIT, "scan: scratch too small");
      note_launch();
      seg_aggregate<T, Op><<<grid, kThreads, 0, stream>>>(x, N, C, seg_rows, agg);
      note_launch();
      seg_carries<T, Op><<<(unsigned)cblocks, kThreads, 0, stream>>>(agg, carry, C, nseg, init);
      note_launch();
      seg_scan<T, Op><<<grid, kThreads, 0, stream>>>(x, y, N, C, seg_rows, carry, init, 1);
    }
  }
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

}  // namespace

int copy_to_contiguous(const DescView &src, int esize, void *dst, cudaStream_t stream, int sm_count);
int copy_from_contiguous(const void *src, const DescView &dst, int esize, cudaStream_t stream, int sm_count);

size_t scan_scratch_bytes(int64_t N, int64_t C, int sm_count) {
  if (C <= 1) return (size_t)2 * (((N + kTile - 1) / kTile + 63) & ~int64_t(63)) * 4 + 256;
  const int64_t want_threads = (int64_t)sm_count * 2048;
  int64_t nseg = std::max<int64_t>(1, std::min<int64_t>(N, want_threads / std::max<int64_t>(C, 1)));
  nseg = std::min<int64_t>(nseg, 65535);
  return (size_t)2 * nseg * C * 4 + 256;
}

int run_scan(const RemoraScanSpec &sp, const DescView &in, const DescView &out, char *scratch,
             size_t scratch_bytes, int sm_count, cudaStream_t stream) {
  const int64_t N = in.rank ? in.sizes[0] : 1;
  const int64_t C = N ? in.numel() / std::max<int64_t>(N, 1) : 0;
  const size_t core = scan_scratch_bytes(N, C, sm_count);
  char *stage = scratch + ((core + 255) & ~(size_t)255);
  size_t used = (core + 255) & ~(size_t)255;
  const void *x = in.data(4);
  void *y = out.data(4);
  const size_t bytes = (size_t)in.numel() * 4;
  if (!in.contiguous()) {
    if (used + bytes > scratch_bytes) return fail(REMORA_ERR_LIMIT, "scan: staging needs more scratch");
    REMORA_TRY(copy_to_contiguous(in, 4, stage, stream, sm_count));
    x = stage;
    used += (bytes + 255) & ~(size_t)255;
  }
  const bool out_contig = out.contiguous();
  if (!out_contig) {
    if (used + bytes > scratch_bytes) return fail(REMORA_ERR_LIMIT, "scan: staging needs more scratch");
    y = scratch + used;
  }
  int st;
  if (sp.dtype == REMORA_F32) {
    st = sp.op == REMORA_FOLD_MUL
             ? scan_impl<float, true>((const float *)x, (float *)y, N, C, sp.right, sp.exclusive, sp.init_f,
                                      scratch, core, sm_count, stream)
             : scan_impl<float, false>((const float *)x, (float *)y, N, C, sp.right, sp.exclusive, sp.init_f,
                                       scratch, core, sm_count, stream);
  } else {
    st = sp.op == REMORA_FOLD_MUL
             ? scan_impl<int, true>((const int *)x, (int *)y, N, C, sp.right, sp.exclusive, sp.init_i, scratch,
                                    core, sm_count, stream)
             : scan_impl<int, false>((const int *)x, (int *)y, N, C, sp.right, sp.exclusive, sp.init_i, scratch,
                                     core, sm_count, stream);
  }
  REMORA_TRY(st);
  if (!out_contig) REMORA_TRY(copy_from_contiguous(y, out, 4, stream, sm_count));
  return REMORA_OK;
}

int validate_scan(const RemoraScanSpec *spec, const void *in_desc, const void *out_desc, int rank,
                  DescView *in, DescView *out) {
  if (spec == nullptr) return fail(REMORA_ERR_ARG, "scan: null spec");
  if (spec->op != REMORA_FOLD_ADD && spec->op != REMORA_FOLD_MUL)
    return fail(REMORA_ERR_UNSUPPORTED, "scan: op %d is not + or *", spec->op);
  if (spec->dtype != REMORA_F32 && spec->dtype != REMORA_I32)
    return fail(REMORA_ERR_UNSUPPORTED, "scan: dtype %d (f32 and i32 only)", spec->dtype);
  if (rank < 1) return fail(REMORA_ERR_RANK, "scan: rank %d (scan needs at least rank 1)", rank);
  if (rank >= 2 && (spec->exclusive || spec->right))
    return fail(REMORA_ERR_UNSUPPORTED, "scan: exclusive and right scans with rank >= 2 are deferred");
  REMORA_TRY(read_desc(in_desc, rank, in, "scan input"));
  REMORA_TRY(read_desc(out_desc, rank, out, "scan output"));
  for (int d = 0; d < rank; ++d)
    if (in->sizes[d] != out->sizes[d]) return fail(REMORA_ERR_SHAPE, "scan: output shape differs from input");
  return REMORA_OK;
}

// ---- leading-axis fold with an array accumulator (array fold):
// out[t] = init[t] op x[0,t] op x[1,t] ...  With one segment this is the
// reference's sequential order exactly; with several, the segment
// aggregates are combined in segment order after init.
namespace {

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) array_fold_combine(const T *__restrict__ agg, const T *__restrict__ init,
                                                              int64_t init_stride, T *__restrict__ out,
                                                              int64_t C, int64_t nseg) {
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= C) return;
  T run = init[t * init_stride];
  for (int64_t s = 0; s < nseg; ++s) run = Op::apply(run, agg[s * C + t]);
  out[t] = run;
}

template <typename T, typename Op>
__global__ void __launch_bounds__(kThreads) array_fold_direct(const T *__restrict__ x, const T *__restrict__ init,
                                                             int64_t init_stride, T *__restrict__ out, int64_t N,
                                                             int64_t C) {
  const int64_t t = (int64_t)blockIdx.x * kThreads + threadIdx.x;
  if (t >= C) return;
  T run = init[t * init_stride];
  for (int64_t r = 0; r < N; ++r) run = Op::apply(run, x[r * C + t]);
  out[t] = run;
}

template <typename T, bool kMul>
int array_fold_impl(const T *x, const T *init, int64_t init_stride, T *out, int64_t N, int64_t C, char *scratch,
                    size_t scratch_bytes, int sm_count, cudaStream_t stream) {
  using Op = ScanOp<T, kMul>;
  if (C == 0) return REMORA_OK;
  const int64_t cblocks = (C + kThreads - 1) / kThreads;
  const int64_t want_threads = (int64_t)sm_count * 2048;
  int64_t nseg = std::max<int64_t>(1, std::min<int64_t>(N / 16, want_threads / std::max<int64_t>(C, 1)));
  nseg = std::min<int64_t>(nseg, 65535);
  if (nseg <= 1) {
    note_launch();
    array_fold_direct<T, Op><<<(unsigned)cblocks, kThreads, 0, stream>>>(x, init, init_stride, out, N, C);
  } else {
    const int64_t seg_rows = (N + nseg - 1) / nseg;
    nseg = (N + seg_rows - 1) / seg_rows;
    if ((size_t)(nseg * C) * sizeof(T) > scratch_bytes) return fail(REMORA_ERR_LIMIT, "array fold: scratch");
    T *agg = reinterpret_cast<T *>(scratch);
    note_launch();
    seg_aggregate<T, Op><<<dim3((unsigned)cblocks, (unsigned)nseg), kThreads, 0, stream>>>(x, N, C, seg_rows, agg);
    note_launch();
    array_fold_combine<T, Op><<<(unsigned)cblocks, kThreads, 0, stream>>>(agg, init, init_stride, out, C, nseg);
  }
  REMORA_CUDA_TRY(cudaGetLastError());
  return REMORA_OK;
}

}  // namespace

}  // namespace remora

using namespace remora;

extern "C" int remora_b200_array_fold(RemoraB200Ctx *ctx, const RemoraFoldSpec *spec, const void *in_desc,
                                      int32_t in_rank, const void *init_desc, void *out_desc,
                                      remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (spec == nullptr) return fail(REMORA_ERR_ARG, "array fold: null spec");
  if (spec->op != REMORA_FOLD_ADD && spec->op != REMORA_FOLD_MUL)
    return fail(REMORA_ERR_UNSUPPORTED, "array fold: op %d is not + or *", spec->op);
  if (spec->dtype != REMORA_F32 && spec->dtype != REMORA_I32)
    return fail(REMORA_ERR_UNSUPPORTED, "array fold: dtype %d", spec->dtype);
  if (spec->has_premap) return fail(REMORA_ERR_UNSUPPORTED, "array fold: premap programs are not supported");
  if (in_rank < 2) return fail(REMORA_ERR_RANK, "array fold: input rank %d (needs >= 2)", in_rank);
  DescView in, init, out;
  REMORA_TRY(read_desc(in_desc, in_rank, &in, "array fold input"));
  REMORA_TRY(read_desc(init_desc, in_rank - 1, &init, "array fold init"));
  REMORA_TRY(read_desc(out_desc, in_rank - 1, &out, "array fold output"));
  for (int d = 1; d < in_rank; ++d)
    if (init.sizes[d - 1] != in.sizes[d] || out.sizes[d - 1] != in.sizes[d])
      return fail(REMORA_ERR_SHAPE, "array fold: init/output shape must be the cell shape");
  const int64_t N = in.sizes[0];
  const int64_t C = init.numel();
  cudaStream_t s = (cudaStream_t)stream;
  size_t need = (size_t)std::max<int64_t>(1, (int64_t)ctx->sm_count * 2048) * 4 + 256;
  const size_t cbytes = (((size_t)C * 4) + 255) & ~(size_t)255;
  const size_t nbytes = (((size_t)in.numel() * 4) + 255) & ~(size_t)255;
  need += 3 * cbytes + nbytes;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, s, need, &ws));
  char *base = (char *)ws->buf;
  const size_t core = (size_t)std::max<int64_t>(1, (int64_t)ctx->sm_count * 2048) * 4 + 256;
  char *stage = base + ((core + 255) & ~(size_t)255);
  const void *x = in.data(4);
  if (!in.contiguous()) {
    REMORA_TRY(copy_to_contiguous(in, 4, stage, s, ctx->sm_count));
    x = stage;
    stage += nbytes;
  }
  const void *ip = init.data(4);
  if (!init.contiguous()) {
    REMORA_TRY(copy_to_contiguous(init, 4, stage, s, ctx->sm_count));
    ip = stage;
    stage += cbytes;
  }
  void *y = out.contiguous() ? out.data(4) : (void *)stage;
  int st;
  if (spec->dtype == REMORA_F32)
    st = spec->op == REMORA_FOLD_MUL
             ? array_fold_impl<float, true>((const float *)x, (const float *)ip, 1, (float *)y, N, C, base, core,
                                            ctx->sm_count, s)
             : array_fold_impl<float, false>((const float *)x, (const float *)ip, 1, (float *)y, N, C, base, core,
                                             ctx->sm_count, s);
  else
    st = spec->op == REMORA_FOLD_MUL
             ? array_fold_impl<int, true>((const int *)x, (const int *)ip, 1, (int *)y, N, C, base, core,
                                          ctx->sm_count, s)
             : array_fold_impl<int, false>((const int *)x, (const int *)ip, 1, (int *)y, N, C, base, core,
                                           ctx->sm_count, s);
  REMORA_TRY(st);
  if (!out.contiguous()) REMORA_TRY(copy_from_contiguous(y, out, 4, s, ctx->sm_count));
  return REMORA_OK;
}

// ---- scan without any allocation: the tile aggregates and carries live in
// one fixed-size device array instead of the library's cached workspace.
namespace remora {
namespace {

// Every GPU that loads the library holds this array until the process exits.
constexpr size_t kNoAllocScanBytes = (size_t)1 << 20;
__device__ __align__(256) unsigned char g_noalloc_scan_scratch[kNoAllocScanBytes];

constexpr int kMaxDevices = 64;
std::mutex g_noalloc_mu;
void *g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the fixed scratch on `device` (which must be current).
// Host code cannot use the array's name as a device address; the address is
// looked up once per device and cached.
int noalloc_scratch(int device, void **out) {
  if (device < 0 || device >= kMaxDevices) return fail(REMORA_ERR_ARG, "scan_noalloc: device %d", device);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[device] == nullptr) {
    void *p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scan_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(REMORA_ERR_CUDA, "scan_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
    g_noalloc_ptr[device] = p;
  }
  *out = g_noalloc_ptr[device];
  return REMORA_OK;
}

}  // namespace
}  // namespace remora

extern "C" int remora_b200_scan_noalloc(RemoraB200Ctx *ctx, const RemoraScanSpec *spec, const void *in_desc,
                                        void *out_desc, int32_t rank, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView in, out;
  REMORA_TRY(validate_scan(spec, in_desc, out_desc, rank, &in, &out));
  if (!in.contiguous() || !out.contiguous())
    return fail(REMORA_ERR_UNSUPPORTED,
                "scan_noalloc: input and output must be contiguous (a strided view would need a staging copy)");
  const int64_t N = in.sizes[0];
  const int64_t C = N ? in.numel() / N : 0;
  // Rank >= 2: fewer row segments so their carries fit the fixed scratch.
  int sm = ctx->sm_count;
  size_t need = 0;
  if (N > 0 && C > 0) {
    if (C == 1) {
      need = scan_scratch_bytes(N, 1, sm);
    } else {
      sm = std::max<int>(1, std::min<int>(sm, (int)((kNoAllocScanBytes - 256) / (8 * 2048))));
      const int64_t nseg = std::max<int64_t>(1, std::min<int64_t>(N, (int64_t)sm * 2048 / C));
      need = nseg == 1 ? 0 : scan_scratch_bytes(N, C, sm);
    }
  }
  if (need > kNoAllocScanBytes) {
    const long long max_tiles = (long long)((kNoAllocScanBytes - 256) / 8) & ~63LL;
    return fail(REMORA_ERR_LIMIT,
                "scan_noalloc: a rank-1 scan of %lld elements needs %zu bytes of scratch; the fixed scratch holds "
                "%zu bytes, i.e. at most %lld elements",
                (long long)N, need, kNoAllocScanBytes, max_tiles * kTile);
  }
  void *scratch = nullptr;
  REMORA_TRY(noalloc_scratch(ctx->device, &scratch));
  return run_scan(*spec, in, out, static_cast<char *>(scratch), kNoAllocScanBytes, sm, (cudaStream_t)stream);
}

extern "C" int remora_b200_scan(RemoraB200Ctx *ctx, const RemoraScanSpec *spec, const void *in_desc,
                                void *out_desc, int32_t rank, remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView in, out;
  REMORA_TRY(validate_scan(spec, in_desc, out_desc, rank, &in, &out));
  const int64_t N = in.sizes[0];
  const int64_t C = N ? in.numel() / N : 0;
  size_t need = ((scan_scratch_bytes(N, C, ctx->sm_count) + 255) & ~(size_t)255);
  if (!in.contiguous()) need += ((size_t)in.numel() * 4 + 255) & ~(size_t)255;
  if (!out.contiguous()) need += ((size_t)out.numel() * 4 + 255) & ~(size_t)255;
  Workspace *ws = nullptr;
  REMORA_TRY(get_workspace(ctx, (cudaStream_t)stream, need, &ws));
  return run_scan(*spec, in, out, (char *)ws->buf, ws->bytes, ctx->sm_count, (cudaStream_t)stream);
}
