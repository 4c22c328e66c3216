/*
 * remora_b200.h — C ABI of libremora_b200.so, the sm_100a backend for the
 * Remora Dense Core data-parallel hot path (lifted maps, cell-frame folds,
 * scans, the dense core GEMM, im2col convolution and their reverse-mode
 * kernels).
 *
 * Conventions (all taken from the reference's descriptor contract):
 *  - Every array crosses the ABI as a pointer to a rank-specialised
 *    RemoraMemRefN descriptor {allocated, aligned, offset, sizes[N],
 *    strides[N]}; offsets and strides are in ELEMENTS, view offsets live in
 *    `offset` and are never folded into `aligned`
 *    (reference docs/ABI.md:11-76, remora/abi.py:20-47).
 *  - The element type is not part of the descriptor; every entry point takes
 *    dtype tags (docs/ABI.md:78).  bool is one byte holding 0 or 1
 *    (docs/ABI.md:80-93).
 *  - Descriptor structs are HOST memory; the data pointers inside them are
 *    device pointers.  The reference copies each descriptor to the device per
 *    launch (remora/runtime.py:415-445); this library reads them on the host
 *    and passes sizes/strides by value, so no per-launch descriptor copy.
 *  - The caller owns every data buffer (remora/executor.py:60-115).  The
 *    library owns only a cached per-stream workspace (fold partials, scan
 *    tile status, split-K partials) released by remora_b200_shutdown.
 *  - Every call is asynchronous on the given stream and returns a status
 *    code; nothing aborts or throws across the ABI.  remora_b200_last_error
 *    returns the message of the last failing call on the calling thread.
 *  - Ranks 0..10 only (remora/limits.py:3).
 */
#ifndef REMORA_B200_H
#define REMORA_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Same object as cudaStream_t / CUstream; NULL is the legacy default stream. */
typedef struct CUstream_st *remora_stream_t;

/* ------------------------------------------------------------------------ */
/* Descriptors: byte-identical to remora/abi.py:_memref_fields (24 + 16*N B) */
/* ------------------------------------------------------------------------ */
#define REMORA_MAX_RANK 10

typedef struct {
  void *allocated;
  void *aligned;
  int64_t offset;
} RemoraMemRef0;

#define REMORA_DECLARE_MEMREF(N)                                               \
  typedef struct {                                                             \
    void *allocated;                                                           \
    void *aligned;                                                             \
    int64_t offset;                                                            \
    int64_t sizes[N];                                                          \
    int64_t strides[N];                                                        \
  } RemoraMemRef##N;

REMORA_DECLARE_MEMREF(1)
REMORA_DECLARE_MEMREF(2)
REMORA_DECLARE_MEMREF(3)
REMORA_DECLARE_MEMREF(4)
REMORA_DECLARE_MEMREF(5)
REMORA_DECLARE_MEMREF(6)
REMORA_DECLARE_MEMREF(7)
REMORA_DECLARE_MEMREF(8)
REMORA_DECLARE_MEMREF(9)
REMORA_DECLARE_MEMREF(10)
#undef REMORA_DECLARE_MEMREF

/* ------------------------------------------------------------------------ */
/* Status codes and dtype tags                                              */
/* ------------------------------------------------------------------------ */
enum {
  REMORA_OK = 0,
  REMORA_ERR_RANK = -1,        /* rank outside 0..10 or wrong for the op   */
  REMORA_ERR_SHAPE = -2,       /* sizes disagree between operands          */
  REMORA_ERR_UNSUPPORTED = -3, /* op/dtype/layout combination not provided */
  REMORA_ERR_CUDA = -4,        /* a CUDA runtime call failed               */
  REMORA_ERR_ARG = -5,         /* null pointer, negative size, bad field   */
  REMORA_ERR_TIMEOUT = -6,     /* a bounded device wait ran out            */
  REMORA_ERR_JIT = -7,         /* NVRTC could not compile a map program    */
  REMORA_ERR_LIMIT = -8        /* request beyond a documented maximum      */
};

enum { REMORA_F32 = 0, REMORA_I32 = 1, REMORA_BOOL = 2 };

/* ------------------------------------------------------------------------ */
/* Map programs: the expression trees of remora/_gpu_map_support.py:22-60     */
/* (Input / Constant / Binary + - * / / Cmp / Select) flattened to register  */
/* code, plus exp/log (remora/operators.py:17-23), && || and the new sqrt    */
/* epilogue.  Comparisons yield 1/0 in the program's compute type.            */
/* ------------------------------------------------------------------------ */
enum {
  REMORA_OP_INPUT = 0, /* dst = input[imm_i]                              */
  REMORA_OP_CONST = 1, /* dst = imm_f (f32 programs) or imm_i (i32/bool)  */
  REMORA_OP_ADD = 2,
  REMORA_OP_SUB = 3,
  REMORA_OP_MUL = 4,
  REMORA_OP_DIV = 5, /* f32: IEEE correctly rounded; i32: truncating     */
  REMORA_OP_LT = 6,
  REMORA_OP_LE = 7,
  REMORA_OP_GT = 8,
  REMORA_OP_GE = 9,
  REMORA_OP_EQ = 10,
  REMORA_OP_NE = 11,
  REMORA_OP_SELECT = 12, /* dst = a != 0 ? b : c  (a true select)          */
  REMORA_OP_AND = 13,
  REMORA_OP_OR = 14,
  REMORA_OP_NEG = 15,
  REMORA_OP_EXP = 16,
  REMORA_OP_LOG = 17,
  REMORA_OP_SQRT = 18,
  REMORA_OP_COUNT_ = 19
};

#define REMORA_MAP_MAX_INSTR 48
#define REMORA_MAP_MAX_INPUTS 8
#define REMORA_MAP_MAX_REGS 64

typedef struct {
  uint8_t op;  /* REMORA_OP_*                         */
  uint8_t dst; /* destination register                */
  uint8_t a;   /* operand registers                   */
  uint8_t b;
  uint8_t c;
  uint8_t pad_[3];
  float imm_f;   /* f32 constant                     */
  int32_t imm_i; /* i32/bool constant or input index */
} RemoraMapInstr; /* 16 bytes */

typedef struct {
  int32_t n_instr;
  int32_t n_inputs;
  int32_t compute_dtype; /* REMORA_F32 / REMORA_I32 / REMORA_BOOL          */
  int32_t out_dtype;     /* element type of the output descriptor           */
  int32_t result;        /* register holding the value to store            */
  int32_t in_dtype[REMORA_MAP_MAX_INPUTS];
  RemoraMapInstr code[REMORA_MAP_MAX_INSTR];
} RemoraMapProgram;

/* ------------------------------------------------------------------------ */
/* Fold / scan specs                                                        */
/* ------------------------------------------------------------------------ */
enum { REMORA_FOLD_ADD = 0, REMORA_FOLD_MUL = 1 };
enum { REMORA_FOLD_CELL = 0, REMORA_FOLD_ALL = 1 };
enum { REMORA_EPI_NONE = 0, REMORA_EPI_SQRT = 1 };

typedef struct {
  int32_t op;         /* REMORA_FOLD_ADD / REMORA_FOLD_MUL                 */
  int32_t mode;       /* CELL: fold the trailing cell_rank axes per frame
                         cell; ALL: whole array to a rank-0 result          */
  int32_t cell_rank;  /* CELL mode: number of trailing axes folded (>= 1)   */
  int32_t dtype;      /* REMORA_F32 or REMORA_I32 (i32 accumulates in i64)  */
  int32_t epilogue;   /* REMORA_EPI_*                                       */
  int32_t has_premap; /* 1: fold premap(in0[, in1]) instead of in0          */
  float init_f;       /* literal initial value (applied exactly once)      */
  int32_t init_i;
  RemoraMapProgram premap;
} RemoraFoldSpec;

typedef struct {
  int32_t op;        /* REMORA_FOLD_ADD / REMORA_FOLD_MUL                  */
  int32_t dtype;     /* REMORA_F32 / REMORA_I32                            */
  int32_t exclusive; /* 1: out[i] = init op x[0..i-1]                      */
  int32_t right;     /* 1: scan from the last element towards the first    */
  float init_f;
  int32_t init_i;
} RemoraScanSpec;

/* ------------------------------------------------------------------------ */
/* Dense core and convolution specs                                         */
/* ------------------------------------------------------------------------ */
/* Tensor-core precision.  TF32: operands as TF32 (10-bit mantissa), f32
   accumulation.  3XTF32: each operand split into hi = TF32(x) and
   lo = x - hi, products hi*hi + hi*lo + lo*hi (close to f32).  2XTF32
   (convolutions only): one operand split, the other TF32 -- the weights in
   the forward and input gradient, the output gradient in the weight
   gradient; for backward passes whose gradients must stay within 1e-3
   (an error study of the crater CNN gives 3.9e-4 for its second layer's
   backward in this mode, 2e-2 for plain TF32). */
enum { REMORA_PREC_TF32 = 0, REMORA_PREC_3XTF32 = 1, REMORA_PREC_2XTF32 = 2 };

typedef struct {
  int32_t precision; /* REMORA_PREC_TF32 or REMORA_PREC_3XTF32             */
  int32_t reserved_;
} RemoraGemmSpec;

typedef struct {
  int32_t stride; /* square stride (1 in the benchmark shape)              */
  int32_t pad;    /* zero padding on every side                            */
  int32_t precision; /* REMORA_PREC_TF32, _3XTF32 or _2XTF32             */
  int32_t reserved_;
} RemoraConvSpec;

typedef struct {
  int32_t kh, kw, stride;
  int32_t reserved_;
} RemoraIm2colSpec;

/* Filter predicate fused into the compaction: keep x where `x op literal`
   (op one of REMORA_OP_LT .. REMORA_OP_NE; f32 comparisons are ordered, so
   NaN compares false), the mask the reference's lowering builds with
   arith.cmpi / arith.cmpf (remora/lowering/tensor_ops.py:2657-2706). */
typedef struct {
  int32_t op;
  float lit_f;   /* literal of an f32 filter */
  int32_t lit_i; /* literal of an i32 filter */
  int32_t reserved_;
} RemoraFilterPred;

typedef struct RemoraB200Ctx RemoraB200Ctx;

/* ------------------------------------------------------------------------ */
/* Context and plumbing.  These replace CUDARuntime (remora/runtime.py:      */
/* 243-340): cuInit/cuCtxCreate, cuMemAlloc/Free, HtoD/DtoH, cuMemsetD32,     */
/* cuCtxSynchronize.                                                         */
/* ------------------------------------------------------------------------ */
/* replaces CUDARuntime.__init__ (remora/runtime.py:246-260) */
int remora_b200_init(int device, RemoraB200Ctx **ctx);
/* replaces CUDARuntime.close (remora/runtime.py:315-319) */
int remora_b200_shutdown(RemoraB200Ctx *ctx);
/* replaces the CUDAError message path (remora/runtime.py:477-491) */
int remora_b200_last_error(char *buf, size_t n);
/* The library's version string (no counterpart in the reference). */
const char *remora_b200_version(void);
/* Number of kernels the library has enqueued in this process (launched, or
   recorded into a CUDA graph under stream capture): the difference over a
   captured region is the kernel count of one replay.  No counterpart in the
   reference. */
unsigned long long remora_b200_launch_count(void);
/* replaces CUDARuntime.alloc / free (remora/runtime.py:270-281) */
int remora_b200_malloc(RemoraB200Ctx *ctx, size_t nbytes, void **dptr);
int remora_b200_free(RemoraB200Ctx *ctx, void *dptr);
/* replaces copy_host_bytes_to_device / copy_device_to_host
   (remora/runtime.py:283-300) */
int remora_b200_memcpy_h2d(RemoraB200Ctx *ctx, void *dst, const void *src,
                           size_t nbytes, remora_stream_t stream);
int remora_b200_memcpy_d2h(RemoraB200Ctx *ctx, void *dst, const void *src,
                           size_t nbytes, remora_stream_t stream);
/* replaces CUDARuntime.memset_d32 (remora/runtime.py:302-307) */
int remora_b200_memset_d32(RemoraB200Ctx *ctx, void *dst, uint32_t value,
                           size_t count, remora_stream_t stream);
/* replaces CUDARuntime.synchronize (remora/runtime.py:309-313); also
   reports REMORA_ERR_TIMEOUT if a bounded device wait ran out since the
   previous check on this stream's workspace. */
int remora_b200_synchronize(RemoraB200Ctx *ctx, remora_stream_t stream);
/* Failure-detection check of the bounded device waits (no counterpart in
   the reference, whose generated kernels have no device-side waits).
   Launches one block that waits, with the same bounded mbarrier wait every
   tcgen05 kernel of this library uses, for a phase that completes only when
   `signal` is 1.  With signal = 0 the wait gives up after `limit_cycles` SM
   clock cycles (0 .. 2^40), records code 900 in the stream's error word and
   returns: the next remora_b200_synchronize on that stream returns
   REMORA_ERR_TIMEOUT, and the context and the device stay usable.  Nothing
   is in flight during the wait (no copies, no MMAs, no tensor memory). */
int remora_b200_wait_check(RemoraB200Ctx *ctx, int64_t limit_cycles,
                           int32_t signal, remora_stream_t stream);
/* Caps the CTAs of this context's persistent kernels (GEMM, tensor-core
   convolutions and their gradients) at n, one per SM (n <= 0: every SM),
   for calls enqueued from now on.  A persistent CTA holds a whole SM
   (shared memory, tensor memory); when a kernel on another stream, such as
   a data-parallel gradient allreduce, holds some SMs, the CTAs scheduled
   behind it wait until it ends and the whole launch ends late.  Leaving
   those SMs free lets the two run side by side.  No counterpart in the
   reference (one stream, no collectives). */
int remora_b200_set_persistent_sms(RemoraB200Ctx *ctx, int32_t n);
/* Pins a host buffer for asynchronous copies (cudaHostRegister), and
   releases it.  No counterpart in the reference, whose copies are
   synchronous (remora/runtime.py:283-300). */
int remora_b200_host_register(void *ptr, size_t nbytes);
int remora_b200_host_unregister(void *ptr);

/* Code-generation check: validates a map program and compiles its generated
   map module (and, when fold_op >= 0 and the program has one or two inputs,
   the fused cell-fold module with it as premap) with NVRTC for sm_100a,
   without a GPU and without launching anything.  Writes the generated
   source to src_out (may be NULL).  The analogue of the reference's
   PTX-emission step (remora/codegen.py:116-257). */
int remora_b200_jit_check(const RemoraMapProgram *prog, int32_t fold_op,
                          char *src_out, size_t n);

/* ------------------------------------------------------------------------ */
/* Hot-path kernels                                                         */
/* ------------------------------------------------------------------------ */

/* Lifted rank-polymorphic map.  Replaces the f32/i32/bool descriptor-ABI map
   kernels (remora/gpu_lowering.py:459-904, launched by
   remora/executor.py:104-108).  Inputs of lower rank than the output are
   broadcast over the trailing frame axes (prefix agreement,
   remora/frame.py:188-211, remora/lowering/tensor_ops.py:644-734); rank-0
   inputs are splatted scalars. */
int remora_b200_map(RemoraB200Ctx *ctx, const RemoraMapProgram *prog,
                    const void *const *in_descs, const int32_t *in_ranks,
                    int32_t n_in, void *out_desc, int32_t out_rank,
                    remora_stream_t stream);

/* Cell-frame fold (remora/lowering/tensor_ops.py:802-874) and whole-array
   fold (remora/lowering/tensor_ops.py:1135-1204; the reference GPU kernel is
   remora/gpu_lowering.py:1021-1150), optionally fused with the producing map
   (premap over 1 or 2 same-shape inputs) and a sqrt epilogue.  Whole-array
   folds are deterministic (fixed-order two-level combine). */
int remora_b200_fold(RemoraB200Ctx *ctx, const RemoraFoldSpec *spec,
                     const void *const *in_descs, const int32_t *in_ranks,
                     int32_t n_in, void *out_desc, int32_t out_rank,
                     remora_stream_t stream);

/* Leading-axis fold with an array-valued accumulator
   (remora/lowering/tensor_ops.py:1223-1296): out = init op x[0] op x[1] ...
   over axis 0.  The AD unbroadcast-sum and bias gradients use it. */
int remora_b200_array_fold(RemoraB200Ctx *ctx, const RemoraFoldSpec *spec,
                           const void *in_desc, int32_t in_rank,
                           const void *init_desc, void *out_desc,
                           remora_stream_t stream);

/* Scans (remora/lowering/tensor_ops.py:2301-2482, interpreter
   remora/runtime.py:1100-1123, single-thread GPU kernel
   remora/gpu_lowering.py:238-304).  Rank 1: inclusive, exclusive, right.
   Rank >= 2: inclusive along axis 0 (the reference defers the others and so
   does this entry point, with REMORA_ERR_UNSUPPORTED). */
int remora_b200_scan(RemoraB200Ctx *ctx, const RemoraScanSpec *spec,
                     const void *in_desc, void *out_desc, int32_t rank,
                     remora_stream_t stream);

/* The same scans as remora_b200_scan, for callers that cannot allocate
   device memory: callers whose device memory is owned entirely by another
   allocator (a host framework's memory pool that has reserved the GPU), and
   callers on a latency-critical path where cudaMalloc, which may synchronise
   the device, is not acceptable.  This entry point allocates nothing: its
   scratch (tile aggregates and carries) is one fixed 1 MiB array in device
   memory that every GPU loading the library holds until the process exits.
   Limits: a rank-1 scan may have at most 268,304,384 elements (larger scans
   return REMORA_ERR_LIMIT before any work is queued); input and output must
   be contiguous (strided views return REMORA_ERR_UNSUPPORTED).  A rank >= 2
   scan runs on fewer row segments here (at most 63 SMs' worth of blocks, so
   that their carries fit the array), so its f32 sums may round differently
   from remora_b200_scan's by reassociation; integer results are identical.
   The first
   call on a device looks up the array's device address (cudaGetSymbolAddress)
   and caches it; make that first call before any stream capture.  Every call
   on a device shares the array: calls that overlap on the GPU (different
   streams, or different threads) race and give wrong results; serialise
   them.  The array keeps the previous call's contents; nothing in it needs
   to start at zero.  No counterpart in the reference. */
int remora_b200_scan_noalloc(RemoraB200Ctx *ctx, const RemoraScanSpec *spec,
                             const void *in_desc, void *out_desc, int32_t rank,
                             remora_stream_t stream);

/* Dense core: C = A . B as the lifted dot
   C[i,j] = fold(+, 0, map(*, A[i,:], B[:,j])) (stdlib/prelude.rem:14,
   examples/crater_train.py:38-44), rank 2 or batched rank 3, f32 storage,
   TF32 or 3xTF32 tcgen05 tensor-core arithmetic with f32 accumulation.
   A may be K-major or M-major and B K-major or N-major, as their strides say;
   C may have any strides (rows or columns contiguous store at full speed). */
int remora_b200_gemm(RemoraB200Ctx *ctx, const RemoraGemmSpec *spec,
                     const void *a_desc, const void *b_desc, void *c_desc,
                     int32_t rank, remora_stream_t stream);

/* Multi-channel NCHW convolution, cross-correlation as the reference's
   conv2d = map(dot-patch p (ravel k)) (im2col image) + b
   (examples/crater_train.py:30-36), extended with channels, batch and zero
   padding.  bias may be NULL.  3x3 / pad 1 / stride 1 layers with 16, 32
   or 64 reduction channels on 16-, 32-, 64- or 128-wide rows and at least
   8 output channels run on the tensor cores in the spec's precision (more
   than 32 output channels: one launch per group of at most 32); every
   other shape runs on CUDA-core kernels in the reference's f32 order,
   whatever the precision. */
int remora_b200_conv2d_fwd(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                           const RemoraMemRef4 *x, const RemoraMemRef4 *w,
                           const RemoraMemRef1 *bias, RemoraMemRef4 *y,
                           remora_stream_t stream);
/* Reverse mode w.r.t. the input: the im2col VJP is col2im
   (remora/ad.py:157-171). */
int remora_b200_conv2d_dgrad(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                             const RemoraMemRef4 *dy, const RemoraMemRef4 *w,
                             RemoraMemRef4 *dx, remora_stream_t stream);
/* Reverse mode w.r.t. the weights: the mul VJP adj*other summed over the
   patches (remora/ad.py:91-95 with the fold VJP at :106-110).  On the
   tensor cores for 3x3 / pad 1 / stride 1 layers whose input channels are a
   multiple of 16, on 16-, 32-, 64- or 128-wide rows (128: TF32 and 2XTF32). */
int remora_b200_conv2d_wgrad(RemoraB200Ctx *ctx, const RemoraConvSpec *spec,
                             const RemoraMemRef4 *x, const RemoraMemRef4 *dy,
                             RemoraMemRef4 *dw, remora_stream_t stream);

/* Reference-exact single-channel im2col / col2im
   (remora/runtime.py:1274-1305; patch order i*out_w+j, pixel order
   ki*kw+kj). */
int remora_b200_im2col(RemoraB200Ctx *ctx, const RemoraIm2colSpec *spec,
                       const RemoraMemRef2 *image, RemoraMemRef2 *cols,
                       remora_stream_t stream);
int remora_b200_col2im(RemoraB200Ctx *ctx, const RemoraIm2colSpec *spec,
                       const RemoraMemRef2 *cols, RemoraMemRef2 *image,
                       remora_stream_t stream);

/* Rank-2 transpose, the swapaxes(0,1) of remora/runtime.py:1052-1056 and
   its VJP (remora/ad.py:116-117). */
int remora_b200_transpose(RemoraB200Ctx *ctx, int32_t dtype,
                          const RemoraMemRef2 *in, RemoraMemRef2 *out,
                          remora_stream_t stream);

/* ------------------------------------------------------------------------ */
/* The C runtime helpers of the reference (remora/remora_rt.c) on the GPU.   */
/* f32 and i32 data, as remora_rt.c; rotate and append also take bool.      */
/* ------------------------------------------------------------------------ */

/* Ascending sort of a rank-1 array, or of every row of a rank-2 array.
   Replaces remora_sort_i32 / remora_sort_f32 (remora/remora_rt.c:42-54) and
   the per-row aliases remora_sort_1d_* (remora/remora_rt.c:289-290) used by
   the rank-2 lowering (remora/lowering/tensor_ops.py:2505-2570).  in and out
   may be the same buffer.  For f32, -0.0 is placed before +0.0 (qsort leaves
   their order open); NaNs without the sign bit go last.  Rows of up to 2^31 - 1. */
int remora_b200_sort(RemoraB200Ctx *ctx, int32_t dtype, const void *in_desc,
                     void *out_desc, int32_t rank, remora_stream_t stream);

/* Stable ascending argsort (int32 indices; equal values keep index order,
   -0.0 and +0.0 are equal) of a rank-1 array or of every row of a rank-2
   array.  Replaces remora_grade_i32 / remora_grade_f32
   (remora/remora_rt.c:56-121) and remora_grade_1d_* (:291-292). */
int remora_b200_grade(RemoraB200Ctx *ctx, int32_t dtype, const void *in_desc,
                      void *out_desc, int32_t rank, remora_stream_t stream);

/* Stream compaction of a rank-1 array: dst[0..count) = src[i] for every i in
   order where the flag is set; *count (a rank-0 int64 device scalar) gets
   the number kept.  The flag is either mask[i] != 0 (mask_dtype REMORA_I32,
   the form of remora_filter_i32 / remora_filter_f32,
   remora/remora_rt.c:125-163, or REMORA_BOOL) or the fused predicate `pred`
   (then mask_desc is NULL).  dst must be contiguous; elements past its
   length are counted but not written.  Replaces the reference's n+2 buffer
   with the count at position 0 (remora/lowering/tensor_ops.py:2707-2720,
   remora/runtime.py:663-668) by a separate count. */
int remora_b200_filter(RemoraB200Ctx *ctx, int32_t dtype, const void *src_desc,
                       const void *mask_desc, int32_t mask_dtype,
                       const RemoraFilterPred *pred, void *dst_desc,
                       RemoraMemRef0 *count_desc, remora_stream_t stream);

/* dst = src[0] repeated counts[0] times, then src[1] counts[1] times, ...
   (rank 1; counts int32; a negative count repeats nothing).  *total (rank-0
   int64 device scalar) gets the length of the result.  With dst_desc NULL
   only the total is computed: remora_replicate_*_count; otherwise
   remora_replicate_*_fill / remora_replicate_* (remora/remora_rt.c:167-285).
   dst must be contiguous; elements past its length are not written. */
int remora_b200_replicate(RemoraB200Ctx *ctx, int32_t dtype,
                          const void *src_desc, const void *counts_desc,
                          void *dst_desc, RemoraMemRef0 *total_desc,
                          remora_stream_t stream);

/* out[i, ...] = in[(i + shift) mod N, ...] along axis 0 with a non-negative
   modulus, any rank >= 1.  Replaces remora_rotate_*_1d
   (remora/remora_rt.c:324-358) and the rotate lowering
   (remora/lowering/tensor_ops.py:1968-2021; interpreter np.roll(a, -shift,
   axis=0), remora/runtime.py:1135-1139). */
int remora_b200_rotate(RemoraB200Ctx *ctx, int32_t dtype, int64_t shift,
                       const void *in_desc, void *out_desc, int32_t rank,
                       remora_stream_t stream);

/* out = a followed by b along axis 0 (trailing axes equal), any rank >= 1.
   Replaces remora_append_*_1d (remora/remora_rt.c:360-388) and the append
   lowering (remora/lowering/tensor_ops.py:2215-2263). */
int remora_b200_append(RemoraB200Ctx *ctx, int32_t dtype, const void *a_desc,
                       const void *b_desc, void *out_desc, int32_t rank,
                       remora_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* REMORA_B200_H */
