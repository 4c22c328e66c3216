// map_fold.cu — lifted maps and fused folds (remora_b200_map / _fold /
// _array_fold).  Map programs are generated per expression and compiled by
// NVRTC (jit.cu); the templates below are the kernel bodies around them.
//
// HBM design: contiguous operands stream through 128-bit loads (4 elements a
// thread, U vectors in flight per thread), results go out with streaming
// stores; cell folds give G lanes (a power of two <= 32) to each frame cell
// and finish with a warp-shuffle butterfly, so a warp covers 512 contiguous
// bytes per load instruction whatever the cell length.  Whole-array folds
// are two-level and deterministic: fixed per-block ranges, fixed-order
// combine of the block partials by the last block to finish.
#include <algorithm>
#include <unordered_map>

#include "jit.cuh"

// Cell-fold launch choices (compile-time; the defaults are the measured best).
#ifndef REMORA_FOLD_MINB
#define REMORA_FOLD_MINB 0
#endif
#ifndef REMORA_FOLD_PF
#define REMORA_FOLD_PF 1
#endif
#ifndef REMORA_FOLD_GRID
#define REMORA_FOLD_GRID 1
#endif
#ifndef REMORA_FOLD_U
#define REMORA_FOLD_U 0
#endif
#ifndef REMORA_FOLD_KC
#define REMORA_FOLD_KC 8
#endif

namespace remora {

namespace {

const char *kPrelude = R"(
typedef long long i64;
typedef unsigned long long u64;
__device__ __forceinline__ float cvt_f(float v) { return v; }
__device__ __forceinline__ float cvt_f(int v) { return (float)v; }
__device__ __forceinline__ float cvt_f(unsigned char v) { return v ? 1.0f : 0.0f; }
__device__ __forceinline__ int cvt_i(float v) { return (int)v; }
__device__ __forceinline__ int cvt_i(int v) { return v; }
__device__ __forceinline__ int cvt_i(unsigned char v) { return v ? 1 : 0; }
// Programmatic dependent launch: wait until the previous kernel in the
// stream has finished and its writes are visible, then let the next one be
// scheduled onto SMs as ours drain.  No-ops without the launch attribute.
#define PDL_PROLOGUE() do { asm volatile("griddepcontrol.wait;" ::: "memory"); \
                            asm volatile("griddepcontrol.launch_dependents;" :::); } while (0)
)";

const char *ctype(int dtype) {
  return dtype == REMORA_F32 ? "float" : dtype == REMORA_I32 ? "int" : "unsigned char";
}
const char *vtype(int dtype) {
  return dtype == REMORA_F32 ? "float4" : dtype == REMORA_I32 ? "int4" : "uchar4";
}

// Expression converting a loaded element `v` of dtype `from` to the
// program's compute type.
std::string to_compute(int compute, const std::string &v) {
  return (compute == REMORA_F32 ? "cvt_f(" : "cvt_i(") + v + ")";
}

// Expression converting compute value `v` to the output dtype.
std::string to_out(int compute, int out, const std::string &v) {
  if (out == REMORA_BOOL)
    return std::string("(unsigned char)((") + v + ") != " + (compute == REMORA_F32 ? "0.0f" : "0") + ")";
  if (out == REMORA_F32) return compute == REMORA_F32 ? v : "(float)(" + v + ")";
  return compute == REMORA_F32 ? "(int)(" + v + ")" : v;
}

enum InMode { IN_FULL = 0, IN_BCAST = 1, IN_SCALAR = 2 };

struct MapVecArgs {
  void *out;
  int64_t n;
  const void *in[REMORA_MAP_MAX_INPUTS];
  int64_t div[REMORA_MAP_MAX_INPUTS];
};

struct MapStridedArgs {
  void *out;
  int64_t n;
  int32_t rank;
  int32_t pad_;
  int64_t shape[REMORA_MAX_RANK];
  int64_t ostride[REMORA_MAX_RANK];
  const void *in[REMORA_MAP_MAX_INPUTS];
  int64_t istride[REMORA_MAP_MAX_INPUTS][REMORA_MAX_RANK];
};

constexpr int kMapUnroll = 4;

std::string map_module_source(const RemoraMapProgram &p, const int *modes) {
  const int n = p.n_inputs;
  const std::string T = p.compute_dtype == REMORA_F32 ? "float" : "int";
  std::string s = kPrelude;
  s += gen_expr(p);
  s += "struct MapVecArgs { void* out; i64 n; const void* in[8]; i64 div[8]; };\n";
  s += "struct MapStridedArgs { void* out; i64 n; int rank; int pad_; i64 shape[10]; i64 "
       "ostride[10]; const void* in[8]; i64 istride[8][10]; };\n";
  s += "#define U " + std::to_string(kMapUnroll) + "\n";

  // ---- vectorised kernel: FULL inputs as 4-vectors, BCAST (divisor a
  // multiple of 4) as one element per vector, SCALAR hoisted.
  s += "extern \"C\" __global__ void __launch_bounds__(256) remora_map_vec(MapVecArgs a) {\n";
  s += "  PDL_PROLOGUE();\n";
  s += "  const i64 nv = a.n >> 2;\n  const i64 step = (i64)gridDim.x * blockDim.x;\n";
  for (int k = 0; k < n; ++k) {
    if (modes[k] == IN_SCALAR)
      s += "  const " + T + " s" + std::to_string(k) + " = " +
           to_compute(p.compute_dtype, std::string("((const ") + ctype(p.in_dtype[k]) + "*)a.in[" +
                                           std::to_string(k) + "])[0]") + ";\n";
  }
  s += "  for (i64 v0 = (i64)blockIdx.x * blockDim.x + threadIdx.x; v0 < nv; v0 += step * U) {\n";
  for (int k = 0; k < n; ++k) {
    const std::string K = std::to_string(k);
    if (modes[k] == IN_FULL) s += "    " + T + " x" + K + "[U][4];\n";
    if (modes[k] == IN_BCAST) s += "    " + T + " b" + K + "[U];\n";
  }
  s += "#pragma unroll\n    for (int u = 0; u < U; ++u) {\n      const i64 v = v0 + u * step;\n"
       "      if (v < nv) {\n";
  for (int k = 0; k < n; ++k) {
    const std::string K = std::to_string(k);
    if (modes[k] == IN_FULL) {
      s += std::string("        const ") + vtype(p.in_dtype[k]) + " t" + K + " = __ldg((const " +
           vtype(p.in_dtype[k]) + "*)a.in[" + K + "] + v);\n";
      const char *comp[4] = {"x", "y", "z", "w"};
      for (int e = 0; e < 4; ++e)
        s += "        x" + K + "[u][" + std::to_string(e) + "] = " +
             to_compute(p.compute_dtype, "t" + K + "." + comp[e]) + ";\n";
    } else if (modes[k] == IN_BCAST) {
      s += "        b" + K + "[u] = " +
           to_compute(p.compute_dtype, std::string("__ldg((const ") + ctype(p.in_dtype[k]) +
                                           "*)a.in[" + K + "] + (v * 4) / a.div[" + K + "])") +
           ";\n";
    }
  }
  s += "      }\n    }\n";
  s += "#pragma unroll\n    for (int u = 0; u < U; ++u) {\n      const i64 v = v0 + u * step;\n"
       "      if (v < nv) {\n";
  s += std::string("        ") + vtype(p.out_dtype) + " o;\n";
  const char *comp[4] = {"x", "y", "z", "w"};
  for (int e = 0; e < 4; ++e) {
    std::string call = "remora_expr(";
    for (int k = 0; k < n; ++k) {
      const std::string K = std::to_string(k);
      call += (k ? ", " : "");
      call += modes[k] == IN_FULL ? "x" + K + "[u][" + std::to_string(e) + "]"
              : modes[k] == IN_BCAST ? "b" + K + "[u]"
                                     : "s" + K;
    }
    call += ")";
    s += std::string("        o.") + comp[e] + " = " + to_out(p.compute_dtype, p.out_dtype, call) + ";\n";
  }
  if (p.out_dtype == REMORA_BOOL)
    s += "        ((uchar4*)a.out)[v] = o;\n";
  else
    s += std::string("        __stcs((") + vtype(p.out_dtype) + "*)a.out + v, o);\n";
  s += "      }\n    }\n  }\n";
  // tail (n % 4 elements)
  s += "  for (i64 i = (nv << 2) + (i64)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += step) {\n";
  {
    std::string call = "remora_expr(";
    for (int k = 0; k < n; ++k) {
      const std::string K = std::to_string(k);
      std::string idx = modes[k] == IN_FULL ? "i" : modes[k] == IN_BCAST ? "i / a.div[" + K + "]" : "0";
      call += (k ? ", " : "");
      call += modes[k] == IN_SCALAR ? "s" + K
                                    : to_compute(p.compute_dtype, std::string("((const ") +
                                                                      ctype(p.in_dtype[k]) + "*)a.in[" +
                                                                      K + "])[" + idx + "]");
    }
    call += ")";
    s += std::string("    ((") + ctype(p.out_dtype) + "*)a.out)[i] = " +
         to_out(p.compute_dtype, p.out_dtype, call) + ";\n";
  }
  s += "  }\n}\n";

  // ---- general strided kernel (views, negative strides, broadcasting).
  s += "extern \"C\" __global__ void __launch_bounds__(256) remora_map_strided(MapStridedArgs a) {\n";
  s += "  PDL_PROLOGUE();\n";
  s += "  const i64 step = (i64)gridDim.x * blockDim.x;\n";
  s += "  for (i64 i = (i64)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += step) {\n";
  s += "    i64 rem = i, off_o = 0;\n";
  for (int k = 0; k < n; ++k) s += "    i64 off" + std::to_string(k) + " = 0;\n";
  s += "    for (int d = a.rank - 1; d >= 0; --d) {\n      const i64 q = rem % a.shape[d];\n"
       "      rem /= a.shape[d];\n      off_o += q * a.ostride[d];\n";
  for (int k = 0; k < n; ++k)
    s += "      off" + std::to_string(k) + " += q * a.istride[" + std::to_string(k) + "][d];\n";
  s += "    }\n";
  {
    std::string call = "remora_expr(";
    for (int k = 0; k < n; ++k) {
      const std::string K = std::to_string(k);
      call += (k ? ", " : "");
      call += to_compute(p.compute_dtype, std::string("((const ") + ctype(p.in_dtype[k]) +
                                              "*)a.in[" + K + "])[off" + K + "]");
    }
    call += ")";
    s += std::string("    ((") + ctype(p.out_dtype) + "*)a.out)[off_o] = " +
         to_out(p.compute_dtype, p.out_dtype, call) + ";\n";
  }
  s += "  }\n}\n";
  return s;
}

// ------------------------------------------------------------------ folds --

struct FoldCellArgs {
  void *out;
  int64_t rows;
  int64_t L;
  const void *in[2];
  float init_f;
  int32_t init_i;
};

struct FoldAllArgs {
  void *out;
  int64_t n;
  int64_t per_block;
  const void *in[2];
  void *partials;
  unsigned int *counter;
  float init_f;
  int32_t init_i;
};

// Cell-fold module for cells of G lanes x U rows per lane group.  minb > 0
// asks for at least that many resident 256-thread blocks per SM (register
// budget); kc > 0 when every lane of a group reads exactly kc 16-byte
// vectors per row (L / 4 == kc * G): the vector kernel then issues all of a
// pass's loads at once and, when a pass holds at most 4 vectors per lane,
// the next pass's loads before this pass's butterfly.
std::string fold_module_source(const RemoraFoldSpec &sp, int n_in, int G, int U, int minb = 0, int kc = 0) {
  const bool f = sp.dtype == REMORA_F32;
  std::string s = kPrelude;
  RemoraMapProgram ident{};
  const RemoraMapProgram *pm = &sp.premap;
  if (!sp.has_premap) {
    ident.n_instr = 1;
    ident.n_inputs = 1;
    ident.compute_dtype = sp.dtype;
    ident.out_dtype = sp.dtype;
    ident.in_dtype[0] = sp.dtype;
    ident.result = 0;
    ident.code[0].op = REMORA_OP_INPUT;
    ident.code[0].dst = 0;
    ident.code[0].imm_i = 0;
    pm = &ident;
  }
  s += gen_expr(*pm);
  const std::string T = pm->compute_dtype == REMORA_F32 ? "float" : "int";
  s += "#define G " + std::to_string(G) + "\n#define U " + std::to_string(U) + "\n";
  s += f ? "typedef float ACC;\n#define IDENT " + std::string(sp.op == REMORA_FOLD_MUL ? "1.0f" : "0.0f") + "\n"
         : "typedef long long ACC;\n#define IDENT " + std::string(sp.op == REMORA_FOLD_MUL ? "1LL" : "0LL") + "\n";
  if (f)
    s += std::string("__device__ __forceinline__ ACC acc_op(ACC a, ACC b) { return ") +
         (sp.op == REMORA_FOLD_MUL ? "__fmul_rn(a, b)" : "__fadd_rn(a, b)") + "; }\n";
  else
    s += std::string("__device__ __forceinline__ ACC acc_op(ACC a, ACC b) { return (ACC)((u64)a ") +
         (sp.op == REMORA_FOLD_MUL ? "*" : "+") + " (u64)b); }\n";
  // element value as ACC: premap output converted to the fold dtype
  std::string elem = "(ACC)(" + to_out(pm->compute_dtype, sp.dtype, n_in == 2 ? "remora_expr(A, B)" : "remora_expr(A)") + ")";
  s += "#define ELEM(A, B) " + elem + "\n";
  // final value: init op total, epilogue, cast
  if (f) {
    std::string fin = "__fadd_rn(__int_as_float(init_bits), t)";
    if (sp.op == REMORA_FOLD_MUL) fin = "__fmul_rn(__int_as_float(init_bits), t)";
    if (sp.epilogue == REMORA_EPI_SQRT) fin = "sqrtf(" + fin + ")";
    s += "__device__ __forceinline__ void put(void* out, i64 r, ACC t, int init_bits) { ((float*)out)[r] = " + fin + "; }\n";
  } else {
    s += std::string("__device__ __forceinline__ void put(void* out, i64 r, ACC t, int init_i) { ((int*)out)[r] = (int)acc_op((ACC)init_i, t); }\n");
  }
  const std::string inT = ctype(pm->in_dtype[0]);
  const std::string inT1 = ctype(n_in == 2 ? pm->in_dtype[1] : pm->in_dtype[0]);
  const std::string inV = vtype(pm->in_dtype[0]);
  const std::string inV1 = vtype(n_in == 2 ? pm->in_dtype[1] : pm->in_dtype[0]);
  const std::string cvt = pm->compute_dtype == REMORA_F32 ? "cvt_f" : "cvt_i";
  const std::string init_arg = f ? "__float_as_int(a.init_f)" : "a.init_i";
  s += "struct FoldCellArgs { void* out; i64 rows; i64 L; const void* in[2]; float init_f; int init_i; };\n";
  s += "struct FoldAllArgs { void* out; i64 n; i64 per_block; const void* in[2]; void* partials; unsigned int* counter; float init_f; int init_i; };\n";

  {
    int lu = 0, lg = 0;
    while ((1 << lu) < U) ++lu;
    while ((1 << lg) < G) ++lg;
    s += "#define HS " + std::to_string(std::min(lu, lg)) + "\n";  // halving steps of the butterfly
  }
  // ---- cell fold, 128-bit loads (L % 4 == 0, 16-byte aligned rows)
  const std::string lb = minb > 0 ? "__launch_bounds__(256, " + std::to_string(minb) + ")" : "__launch_bounds__(256)";
  // loads of the U rows starting at row R into (VA, VB), vector columns
  // C + k * G for k < KC (element u * KC + k)
  auto loads = [&](const std::string &VA, const std::string &VB, const std::string &R, const std::string &C) {
    std::string t = "#pragma unroll\n      for (int u = 0; u < U; ++u) {\n        const i64 r = " + R +
                    " + u;\n        if (r < a.rows) {\n#pragma unroll\n          for (int k = 0; k < KC; ++k) {\n";
    t += "            " + VA + "[u * KC + k] = __ldcs((const " + inV + "*)a.in[0] + r * nv + " + C + " + k * G);\n";
    if (n_in == 2)
      t += "            " + VB + "[u * KC + k] = __ldcs((const " + inV1 + "*)a.in[1] + r * nv + " + C + " + k * G);\n";
    else t += "            " + VB + "[u * KC + k] = " + VA + "[u * KC + k];\n";
    t += "          }\n        }\n      }\n";
    return t;
  };
  // each lane adds its vectors of a row in column order
  auto accum = [&](const std::string &VA, const std::string &VB) {
    std::string t = "#pragma unroll\n      for (int u = 0; u < U; ++u) {\n        if (r0 + u < a.rows) {\n"
                    "#pragma unroll\n          for (int k = 0; k < KC; ++k) {\n";
    for (const char *c : {"x", "y", "z", "w"})
      t += std::string("            acc[u] = acc_op(acc[u], ELEM(") + cvt + "(" + VA + "[u * KC + k]." + c + "), " +
           cvt + "(" + VB + "[u * KC + k]." + c + ")));\n";
    t += "          }\n        }\n      }\n";
    return t;
  };
  const std::string butterfly = R"(
    // Butterfly over the G lanes of a group for its U rows at once: the
    // first HS steps halve the rows a lane holds (it keeps one half and
    // sends the other), the rest are plain xor steps.  Each partial sum
    // pairs the same lanes in the same order as a separate butterfly per
    // row would, so the totals are the same bit for bit, with
    // U/2 + U/4 + ... + log2(G/U)... shuffles instead of U * log2(G).
#pragma unroll
    for (int step = 0; step < HS; ++step) {
      const int o = G >> (step + 1), h = U >> step;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < h / 2; ++j) {
        const ACC send = up ? acc[j] : acc[j + h / 2];
        const ACC keep = up ? acc[j + h / 2] : acc[j];
        acc[j] = acc_op(keep, __shfl_xor_sync(0xffffffffu, send, o));
      }
    }
#pragma unroll
    for (int o = G >> (HS + 1); o > 0; o >>= 1) {
#pragma unroll
      for (int j = 0; j < (U >> HS); ++j) acc[j] = acc_op(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], o));
    }
    if ((sub & ((G >> HS) - 1)) == 0) {
      int u0 = 0;
#pragma unroll
      for (int step = 0; step < HS; ++step)
        if (lane & (G >> (step + 1))) u0 += U >> (step + 1);
#pragma unroll
      for (int j = 0; j < (U >> HS); ++j)
        if (r0 + u0 + j < a.rows) put(a.out, r0 + u0 + j, acc[j], )" + init_arg + R"();
    }
)";
  s += "\nextern \"C\" __global__ void " + lb + " remora_fold_cell_vec(FoldCellArgs a) {\n";
  s += R"(  PDL_PROLOGUE();
  const int lane = threadIdx.x & 31, sub = lane & (G - 1), grp = lane / G;
  const i64 warp = (i64)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const i64 nwarps = (i64)gridDim.x * (blockDim.x >> 5);
  const i64 rows_per_warp = (32 / G) * U;
  const i64 nv = a.L >> 2;
)";
  if (kc > 0 && U * kc <= 4) {
    // kc vectors per lane per row: pass k+1's loads are in flight while
    // pass k's butterfly and stores run.
    s += "#define KC " + std::to_string(kc) + "\n";
    s += "  const i64 stride = nwarps * rows_per_warp;\n  i64 base = warp * rows_per_warp;\n";
    s += "  " + inV + " va[U * KC]; " + inV1 + " vb[U * KC];\n  {\n    const i64 r0 = base + (i64)grp * U;\n";
    s += loads("va", "vb", "r0", "sub");
    s += "  }\n  for (; base < a.rows; base += stride) {\n    const i64 r0 = base + (i64)grp * U;\n";
    s += "    " + inV + " na[U * KC]; " + inV1 + " nb[U * KC];\n    {\n      const i64 rn = r0 + stride;\n";
    s += loads("na", "nb", "rn", "sub");
    s += "    }\n    ACC acc[U];\n#pragma unroll\n    for (int u = 0; u < U; ++u) acc[u] = IDENT;\n";
    s += accum("va", "vb");
    s += butterfly;
    s += "#pragma unroll\n    for (int i = 0; i < U * KC; ++i) { va[i] = na[i]; vb[i] = nb[i]; }\n  }\n}\n";
  } else if (kc > 0) {
    // kc vectors per lane per row, all of a pass's loads issued at once
    s += "#define KC " + std::to_string(kc) + "\n";
    s += R"(  for (i64 base = warp * rows_per_warp; base < a.rows; base += nwarps * rows_per_warp) {
    const i64 r0 = base + (i64)grp * U;
    ACC acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = IDENT;
)";
    s += "    " + inV + " va[U * KC]; " + inV1 + " vb[U * KC];\n";
    s += loads("va", "vb", "r0", "sub");
    s += accum("va", "vb");
    s += butterfly;
    s += "  }\n}\n";
  } else {
    s += "#define KC 1\n";
    s += R"(  for (i64 base = warp * rows_per_warp; base < a.rows; base += nwarps * rows_per_warp) {
    const i64 r0 = base + (i64)grp * U;
    ACC acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = IDENT;
#pragma unroll 4
    for (i64 c = sub; c < nv; c += G) {
)";
    s += "      " + inV + " va[U]; " + inV1 + " vb[U];\n";
    s += loads("va", "vb", "r0", "c");
    s += accum("va", "vb");
    s += "    }\n";
    s += butterfly;
    s += "  }\n}\n";
  }

  // ---- cell fold, scalar loads (any L, any 4-byte alignment)
  s += R"(
extern "C" __global__ void __launch_bounds__(256) remora_fold_cell_scalar(FoldCellArgs a) {
  PDL_PROLOGUE();
  const int lane = threadIdx.x & 31, sub = lane & (G - 1), grp = lane / G;
  const i64 warp = (i64)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const i64 nwarps = (i64)gridDim.x * (blockDim.x >> 5);
  const i64 rows_per_warp = (32 / G) * U;
  for (i64 base = warp * rows_per_warp; base < a.rows; base += nwarps * rows_per_warp) {
    const i64 r0 = base + (i64)grp * U;
    ACC acc[U];
#pragma unroll
    for (int u = 0; u < U; ++u) acc[u] = IDENT;
#pragma unroll 4
    for (i64 c = sub; c < a.L; c += G) {
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const i64 r = r0 + u;
        if (r < a.rows) {
)";
  s += "          const " + inT + " xa = ((const " + inT + "*)a.in[0])[r * a.L + c];\n";
  if (n_in == 2) s += "          const " + inT1 + " xb = ((const " + inT1 + "*)a.in[1])[r * a.L + c];\n";
  else s += "          const " + inT + " xb = xa;\n";
  s += "          acc[u] = acc_op(acc[u], ELEM(" + cvt + "(xa), " + cvt + "(xb)));\n";
  s += R"(        }
      }
    }
    // Butterfly over the G lanes of a group for its U rows at once: the
    // first HS steps halve the rows a lane holds (it keeps one half and
    // sends the other), the rest are plain xor steps.  Each partial sum
    // pairs the same lanes in the same order as a separate butterfly per
    // row would, so the totals are the same bit for bit, with
    // U/2 + U/4 + ... + log2(G/U)... shuffles instead of U * log2(G).
#pragma unroll
    for (int step = 0; step < HS; ++step) {
      const int o = G >> (step + 1), h = U >> step;
      const bool up = (lane & o) != 0;
#pragma unroll
      for (int j = 0; j < h / 2; ++j) {
        const ACC send = up ? acc[j] : acc[j + h / 2];
        const ACC keep = up ? acc[j + h / 2] : acc[j];
        acc[j] = acc_op(keep, __shfl_xor_sync(0xffffffffu, send, o));
      }
    }
#pragma unroll
    for (int o = G >> (HS + 1); o > 0; o >>= 1) {
#pragma unroll
      for (int j = 0; j < (U >> HS); ++j) acc[j] = acc_op(acc[j], __shfl_xor_sync(0xffffffffu, acc[j], o));
    }
    if ((sub & ((G >> HS) - 1)) == 0) {
      int u0 = 0;
#pragma unroll
      for (int step = 0; step < HS; ++step)
        if (lane & (G >> (step + 1))) u0 += U >> (step + 1);
#pragma unroll
      for (int j = 0; j < (U >> HS); ++j)
        if (r0 + u0 + j < a.rows) put(a.out, r0 + u0 + j, acc[j], )" + init_arg + R"();
    }
  }
}
)";

  // ---- whole-array fold: fixed block ranges, last block combines in order
  s += R"(
__device__ __forceinline__ ACC block_reduce(ACC v, ACC* sh) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = acc_op(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
  if (l == 0) sh[w] = v;
  __syncthreads();
  ACC t = IDENT;
  if (threadIdx.x == 0)
    for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t = acc_op(t, sh[i]);
  __syncthreads();
  return t;
}
extern "C" __global__ void __launch_bounds__(256) remora_fold_all(FoldAllArgs a) {
  PDL_PROLOGUE();
  __shared__ ACC sh[32];
  __shared__ int is_last;
  const i64 beg = (i64)blockIdx.x * a.per_block;
  const i64 end = beg + a.per_block < a.n ? beg + a.per_block : a.n;
  ACC acc = IDENT;
  const bool vec = ((a.per_block & 3) == 0) && ((a.n & 3) == 0) &&
                   ((((u64)a.in[0]) & 15) == 0) && ((((u64)a.in[1]) & 15) == 0);
  if (vec) {
#pragma unroll 4
    for (i64 v = (beg >> 2) + threadIdx.x; v < (end >> 2); v += blockDim.x) {
)";
  s += "      const " + inV + " va = __ldcs((const " + inV + "*)a.in[0] + v);\n";
  if (n_in == 2) s += "      const " + inV1 + " vb = __ldcs((const " + inV1 + "*)a.in[1] + v);\n";
  else s += "      const " + inV + " vb = va;\n";
  for (const char *c : {"x", "y", "z", "w"})
    s += std::string("      acc = acc_op(acc, ELEM(") + cvt + "(va." + c + "), " + cvt + "(vb." + c + ")));\n";
  s += "    }\n  } else {\n    for (i64 i = beg + threadIdx.x; i < end; i += blockDim.x) {\n";
  s += "      const " + inT + " xa = ((const " + inT + "*)a.in[0])[i];\n";
  if (n_in == 2) s += "      const " + inT1 + " xb = ((const " + inT1 + "*)a.in[1])[i];\n";
  else s += "      const " + inT + " xb = xa;\n";
  s += "      acc = acc_op(acc, ELEM(" + cvt + "(xa), " + cvt + "(xb)));\n    }\n  }\n";
  s += R"(
  const ACC total = block_reduce(acc, sh);
  if (threadIdx.x == 0) {
    ((ACC*)a.partials)[blockIdx.x] = total;
    __threadfence();
    const unsigned t = atomicAdd(a.counter, 1u);
    is_last = (t == gridDim.x - 1);
  }
  __syncthreads();
  if (is_last) {
    __threadfence();
    ACC v = IDENT;
    for (int i = threadIdx.x; i < (int)gridDim.x; i += blockDim.x)
      v = acc_op(v, __ldcg((const ACC*)a.partials + i));
    const ACC t = block_reduce(v, sh);
    if (threadIdx.x == 0) {
      put(a.out, 0, t, )" + init_arg + R"();
      *a.counter = 0u;
    }
  }
}
)";
  return s;
}

int pow2_floor(int64_t v) {
  int g = 1;
  while ((int64_t)g * 2 <= v && g < 32) g *= 2;
  return g;
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// Blocks of `block` threads of kernel k that one SM holds at once (cached
// per kernel; at least 1).
int resident_blocks(cudaKernel_t k, int block) {
  static std::mutex mu;
  static std::unordered_map<const void *, int> cache;
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find((const void *)k);
  if (it != cache.end()) return it->second;
  int n = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, (const void *)k, block, 0) != cudaSuccess || n < 1) {
    cudaGetLastError();
    n = 1;
  }
  cache.emplace((const void *)k, n);
  return n;
}

// Every JIT kernel starts with PDL_PROLOGUE, so it may be launched as a
// programmatic dependent of the previous kernel in the stream: its blocks
// are scheduled while that kernel's last blocks drain, which hides most of
// the launch gap between back-to-back HBM-bound kernels.
int launch(cudaKernel_t k, int grid, int block, void *args_struct, cudaStream_t stream) {
  void *params[] = {args_struct};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  note_launch();
  cudaError_t e = cudaLaunchKernelExC(&cfg, (const void *)k, params);
  if (e != cudaSuccess) return fail(REMORA_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(e));
  return REMORA_OK;
}

}  // namespace

// Strided copy into a contiguous buffer (misc.cu).
int copy_to_contiguous(const DescView &src, int esize, void *dst, cudaStream_t stream, int sm_count);
int copy_from_contiguous(const void *src, const DescView &dst, int esize, cudaStream_t stream, int sm_count);

int run_map(RemoraB200Ctx *ctx, const RemoraMapProgram &p, const DescView *ins, int n_in,
            const DescView &out, cudaStream_t stream) {
  const int R = out.rank;
  const int64_t n = out.numel();
  // Effective strides over the output's axes (prefix-frame broadcasting).
  int modes[REMORA_MAP_MAX_INPUTS] = {0};
  int64_t div[REMORA_MAP_MAX_INPUTS] = {0};
  int64_t eff[REMORA_MAP_MAX_INPUTS][REMORA_MAX_RANK] = {{0}};
  bool vec_ok = out.contiguous() && aligned16(out.data(dtype_size(p.out_dtype)));
  if (p.out_dtype == REMORA_BOOL) vec_ok = out.contiguous() && ((uintptr_t)out.data(1) & 3) == 0;
  for (int k = 0; k < n_in; ++k) {
    const DescView &d = ins[k];
    if (d.rank > R)
      return fail(REMORA_ERR_SHAPE, "map: input %d has rank %d above the output rank %d", k, d.rank, R);
    for (int ax = 0; ax < d.rank; ++ax)
      if (d.sizes[ax] != out.sizes[ax])
        return fail(REMORA_ERR_SHAPE,
                    "map: input %d axis %d has size %lld, the frame has %lld (prefix agreement)",
                    k, ax, (long long)d.sizes[ax], (long long)out.sizes[ax]);
    for (int ax = 0; ax < d.rank; ++ax) eff[k][ax] = d.sizes[ax] == 1 ? 0 : d.strides[ax];
    int64_t inner = 1;
    for (int ax = d.rank; ax < R; ++ax) inner *= out.sizes[ax];
    const int es = dtype_size(p.in_dtype[k]);
    if (d.rank == 0 || d.numel() == 1) {
      modes[k] = IN_SCALAR;
    } else if (d.contiguous() && inner == 1) {
      modes[k] = IN_FULL;
      if (!(p.in_dtype[k] == REMORA_BOOL ? (((uintptr_t)d.data(1) & 3) == 0) : aligned16(d.data(es))))
        vec_ok = false;
    } else if (d.contiguous()) {
      modes[k] = IN_BCAST;
      div[k] = inner;
      if (inner % 4) vec_ok = false;
    } else {
      modes[k] = IN_FULL;
      vec_ok = false;
    }
  }
  if (n == 0) return REMORA_OK;
  if (!vec_ok)
    for (int k = 0; k < n_in; ++k) modes[k] = IN_FULL;  // strided kernel ignores modes
  std::string key("map");
  key_append(key, p);
  for (int k = 0; k < n_in; ++k) key_append(key, modes[k]);
  auto make = [&]() { return map_module_source(p, modes); };
  const int block = 256;
  if (vec_ok) {
    cudaKernel_t kern;
    REMORA_TRY(jit_kernel_keyed(key, "remora_map_vec", make, &kern));
    MapVecArgs a{};
    a.out = out.data(dtype_size(p.out_dtype));
    a.n = n;
    for (int k = 0; k < n_in; ++k) {
      a.in[k] = ins[k].data(dtype_size(p.in_dtype[k]));
      a.div[k] = div[k] ? div[k] : 1;
    }
    int64_t vecs = (n / 4 + kMapUnroll - 1) / kMapUnroll;
    int64_t grid = std::max<int64_t>(1, std::min<int64_t>((vecs + block - 1) / block, (int64_t)ctx->sm_count * 8));
    return launch(kern, (int)grid, block, &a, stream);
  }
  cudaKernel_t kern;
  REMORA_TRY(jit_kernel_keyed(key, "remora_map_strided", make, &kern));
  MapStridedArgs a{};
  a.out = out.data(dtype_size(p.out_dtype));
  a.n = n;
  a.rank = R;
  for (int ax = 0; ax < R; ++ax) {
    a.shape[ax] = out.sizes[ax];
    a.ostride[ax] = out.strides[ax];
  }
  for (int k = 0; k < n_in; ++k) {
    a.in[k] = ins[k].data(dtype_size(p.in_dtype[k]));
    for (int ax = 0; ax < R; ++ax) a.istride[k][ax] = eff[k][ax];
  }
  int64_t grid = std::max<int64_t>(1, std::min<int64_t>((n + block - 1) / block, (int64_t)ctx->sm_count * 16));
  return launch(kern, (int)grid, block, &a, stream);
}

int run_fold(RemoraB200Ctx *ctx, const RemoraFoldSpec &sp, const DescView *ins, int n_in,
             const DescView &out, cudaStream_t stream, void *scratch, size_t scratch_bytes,
             unsigned int *ticket, int *err, bool use_scratch_only);

}  // namespace remora

using namespace remora;

namespace remora {

// Layout of a fold's scratch: [256 B unused] [partials: kMaxFoldBlocks x 8 B]
// [contiguous staging copies of non-contiguous inputs/outputs].  The block
// ticket of the whole-array fold lives in the workspace's small zeroed block
// (Workspace::fold_ticket), not here, because other calls overwrite this
// scratch freely.
constexpr size_t kFoldHeader = 256 + (size_t)kMaxFoldBlocks * 8;

int run_fold(RemoraB200Ctx *ctx, const RemoraFoldSpec &sp, const DescView *ins_in, int n_in,
             const DescView &out_in, cudaStream_t stream, void *scratch, size_t scratch_bytes,
             unsigned int *ticket, int *err, bool no_staging) {
  DescView ins[2] = {ins_in[0], n_in == 2 ? ins_in[1] : ins_in[0]};
  const DescView &x = ins[0];
  const int in_es[2] = {dtype_size(sp.has_premap ? sp.premap.in_dtype[0] : sp.dtype),
                        dtype_size(sp.has_premap ? sp.premap.in_dtype[n_in == 2 ? 1 : 0] : sp.dtype)};
  int64_t rows, L;
  if (sp.mode == REMORA_FOLD_ALL) {
    rows = 1;
    L = x.numel();
  } else {
    const int fr = x.rank - sp.cell_rank;
    rows = 1;
    L = 1;
    for (int d = 0; d < fr; ++d) rows *= x.sizes[d];
    for (int d = fr; d < x.rank; ++d) L *= x.sizes[d];
  }
  char *stage = static_cast<char *>(scratch) + kFoldHeader;
  size_t stage_used = 0;
  const void *src[2];
  for (int k = 0; k < n_in; ++k) {
    if (ins[k].contiguous()) {
      src[k] = ins[k].data(in_es[k]);
    } else {
      if (no_staging)
        return fail(REMORA_ERR_UNSUPPORTED, "fold: input %d is not contiguous", k);
      size_t need = ((size_t)ins[k].numel() * in_es[k] + 255) & ~(size_t)255;
      if (kFoldHeader + stage_used + need > scratch_bytes)
        return fail(REMORA_ERR_LIMIT, "fold: staging needs more scratch");
      REMORA_TRY(copy_to_contiguous(ins[k], in_es[k], stage + stage_used, stream, ctx->sm_count));
      src[k] = stage + stage_used;
      stage_used += need;
    }
  }
  if (n_in == 1) src[1] = src[0];
  const int out_es = dtype_size(sp.dtype);
  void *dst = out_in.data(out_es);
  const bool out_contig = out_in.contiguous();
  if (!out_contig) {
    if (no_staging) return fail(REMORA_ERR_UNSUPPORTED, "fold: output is not contiguous");
    size_t need = ((size_t)out_in.numel() * out_es + 255) & ~(size_t)255;
    if (kFoldHeader + stage_used + need > scratch_bytes)
      return fail(REMORA_ERR_LIMIT, "fold: staging needs more scratch");
    dst = stage + stage_used;
    stage_used += need;
  }

  const int block = 256;
  if (sp.mode == REMORA_FOLD_ALL) {
    std::string key("fold");
    key_append(key, sp);
    key_append(key, n_in);
    cudaKernel_t kern;
    REMORA_TRY(jit_kernel_keyed(key, "remora_fold_all",
                                [&]() { return fold_module_source(sp, n_in, 32, 1); }, &kern));
    FoldAllArgs a{};
    a.out = dst;
    a.n = L;
    const int64_t chunk = (int64_t)block * 4 * 4;
    int64_t nblocks = std::max<int64_t>(1, std::min<int64_t>((L + chunk - 1) / chunk, kMaxFoldBlocks));
    int64_t per = (L + nblocks - 1) / nblocks;
    per = (per + 3) & ~(int64_t)3;
    nblocks = std::max<int64_t>(1, (L + per - 1) / std::max<int64_t>(per, 1));
    a.per_block = per;
    a.in[0] = src[0];
    a.in[1] = src[1];
    a.counter = ticket;
    a.partials = static_cast<char *>(scratch) + 256;
    a.init_f = sp.init_f;
    a.init_i = sp.init_i;
    REMORA_TRY(launch(kern, (int)nblocks, block, &a, stream));
  } else {
    bool vec = (L % 4) == 0;
    for (int k = 0; k < n_in; ++k)
      if (in_es[k] != 4 || !aligned16(src[k])) vec = false;
    const int64_t units = vec ? L / 4 : L;
    const int G = pow2_floor(std::max<int64_t>(units, 1));
    const int64_t per_lane = (units + G - 1) / G;
    int U = 1;
    if (per_lane < 4) U = (int)std::max<int64_t>(1, 4 / std::max<int64_t>(per_lane, 1));
    if (REMORA_FOLD_U > 0 && per_lane < 4) U = REMORA_FOLD_U;
    // vectors per lane per row when they divide evenly (at most 8)
    const int one = (vec && REMORA_FOLD_PF && units % G == 0 && units / G <= REMORA_FOLD_KC) ? (int)(units / G) : 0;
    const int minb = REMORA_FOLD_MINB;
    std::string key("fold");
    key_append(key, sp);
    key_append(key, n_in);
    key_append(key, G);
    key_append(key, U);
    key_append(key, one);
    key_append(key, minb);
    cudaKernel_t kern;
    REMORA_TRY(jit_kernel_keyed(key, vec ? "remora_fold_cell_vec" : "remora_fold_cell_scalar",
                                [&]() { return fold_module_source(sp, n_in, G, U, minb, one); }, &kern));
    FoldCellArgs a{};
    a.out = dst;
    a.rows = rows;
    a.L = L;
    a.in[0] = src[0];
    a.in[1] = src[1];
    a.init_f = sp.init_f;
    a.init_i = sp.init_i;
    const int64_t rows_per_block = (int64_t)(block / 32) * (32 / G) * U;
    // Every block resident at once: a grid of at most the blocks the SMs
    // hold together, each striding over the row blocks, so no block waits
    // for a second wave and every block makes the same number of passes
    // (to within one).
    int64_t cap = (int64_t)ctx->sm_count * 8;
    if (REMORA_FOLD_GRID) cap = (int64_t)ctx->sm_count * resident_blocks(kern, block);
    int64_t grid = std::max<int64_t>(1, std::min<int64_t>((rows + rows_per_block - 1) / rows_per_block, cap));
    if (rows > 0) REMORA_TRY(launch(kern, (int)grid, block, &a, stream));
  }
  if (!out_contig) REMORA_TRY(copy_from_contiguous(dst, out_in, out_es, stream, ctx->sm_count));
  return REMORA_OK;
}

int validate_fold(const RemoraFoldSpec *spec, const void *const *in_descs, const int32_t *in_ranks,
                  int32_t n_in, const void *out_desc, int32_t out_rank, DescView *ins, DescView *out) {
  if (spec == nullptr || in_descs == nullptr || in_ranks == nullptr)
    return fail(REMORA_ERR_ARG, "fold: null argument");
  const RemoraFoldSpec &sp = *spec;
  if (sp.op != REMORA_FOLD_ADD && sp.op != REMORA_FOLD_MUL)
    return fail(REMORA_ERR_UNSUPPORTED, "fold: op %d is not + or *", sp.op);
  if (sp.dtype != REMORA_F32 && sp.dtype != REMORA_I32)
    return fail(REMORA_ERR_UNSUPPORTED, "fold: dtype %d (f32 and i32 folds only)", sp.dtype);
  if (sp.epilogue == REMORA_EPI_SQRT && sp.dtype != REMORA_F32)
    return fail(REMORA_ERR_UNSUPPORTED, "fold: sqrt epilogue needs f32");
  if (n_in < 1 || n_in > 2) return fail(REMORA_ERR_ARG, "fold: %d inputs (1 or 2 allowed)", n_in);
  if (n_in == 2 && !sp.has_premap)
    return fail(REMORA_ERR_ARG, "fold: two inputs need a premap program combining them");
  if (sp.has_premap) REMORA_TRY(validate_program(sp.premap, n_in));
  for (int k = 0; k < n_in; ++k) REMORA_TRY(read_desc(in_descs[k], in_ranks[k], &ins[k], "fold input"));
  if (n_in == 2) {
    if (ins[0].rank != ins[1].rank) return fail(REMORA_ERR_SHAPE, "fold: inputs differ in rank");
    for (int d = 0; d < ins[0].rank; ++d)
      if (ins[0].sizes[d] != ins[1].sizes[d]) return fail(REMORA_ERR_SHAPE, "fold: inputs differ in shape");
  }
  REMORA_TRY(read_desc(out_desc, out_rank, out, "fold output"));
  if (sp.mode == REMORA_FOLD_ALL) {
    if (out_rank != 0) return fail(REMORA_ERR_RANK, "fold: a whole-array fold writes a rank-0 result");
  } else if (sp.mode == REMORA_FOLD_CELL) {
    if (sp.cell_rank < 1 || sp.cell_rank > ins[0].rank)
      return fail(REMORA_ERR_RANK, "fold: cell rank %d for an input of rank %d", sp.cell_rank, ins[0].rank);
    if (out_rank != ins[0].rank - sp.cell_rank)
      return fail(REMORA_ERR_RANK, "fold: output rank %d, frame rank %d", out_rank, ins[0].rank - sp.cell_rank);
    for (int d = 0; d < out_rank; ++d)
      if (out->sizes[d] != ins[0].sizes[d]) return fail(REMORA_ERR_SHAPE, "fold: output shape is not the frame shape");
  } else {
    return fail(REMORA_ERR_ARG, "fold: unknown mode %d", sp.mode);
  }
  if (sp.has_premap) {
    for (int k = 0; k < n_in; ++k)
      if (sp.premap.in_dtype[k] == REMORA_BOOL)
        return fail(REMORA_ERR_UNSUPPORTED, "fold: bool premap inputs are not supported");
  }
  return REMORA_OK;
}

size_t fold_staging_bytes(const DescView *ins, int n_in, const DescView &out, const RemoraFoldSpec &sp) {
  size_t need = kFoldHeader;
  for (int k = 0; k < n_in; ++k)
    if (!ins[k].contiguous()) need += (((size_t)ins[k].numel() * 4 + 255) & ~(size_t)255);
  if (!out.contiguous()) need += (((size_t)out.numel() * dtype_size(sp.dtype) + 255) & ~(size_t)255);
  return need;
}

}  // namespace remora

extern "C" {

int remora_b200_map(RemoraB200Ctx *ctx, const RemoraMapProgram *prog, const void *const *in_descs,
                    const int32_t *in_ranks, int32_t n_in, void *out_desc, int32_t out_rank,
                    remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  if (prog == nullptr) return fail(REMORA_ERR_ARG, "map: null program");
  if (n_in > 0 && (in_descs == nullptr || in_ranks == nullptr))
    return fail(REMORA_ERR_ARG, "map: null input arrays");
  REMORA_TRY(validate_program(*prog, n_in));
  DescView ins[REMORA_MAP_MAX_INPUTS], out;
  for (int k = 0; k < n_in; ++k) REMORA_TRY(read_desc(in_descs[k], in_ranks[k], &ins[k], "map input"));
  REMORA_TRY(read_desc(out_desc, out_rank, &out, "map output"));
  return run_map(ctx, *prog, ins, n_in, out, (cudaStream_t)stream);
}

int remora_b200_jit_check(const RemoraMapProgram *prog, int32_t fold_op, char *src_out, size_t n) {
  if (prog == nullptr) return fail(REMORA_ERR_ARG, "jit check: null program");
  REMORA_TRY(validate_program(*prog, prog->n_inputs));
  int modes[REMORA_MAP_MAX_INPUTS];
  for (int k = 0; k < REMORA_MAP_MAX_INPUTS; ++k) modes[k] = k == 1 ? IN_BCAST : k == 2 ? IN_SCALAR : IN_FULL;
  std::string src = map_module_source(*prog, modes);
  REMORA_TRY(nvrtc_compile(src, nullptr));
  if (fold_op >= 0 && prog->n_inputs >= 1 && prog->n_inputs <= 2) {
    RemoraFoldSpec sp{};
    sp.op = fold_op;
    sp.mode = REMORA_FOLD_CELL;
    sp.cell_rank = 1;
    sp.dtype = prog->out_dtype == REMORA_I32 ? REMORA_I32 : REMORA_F32;
    sp.epilogue = sp.dtype == REMORA_F32 ? REMORA_EPI_SQRT : REMORA_EPI_NONE;
    sp.has_premap = 1;
    sp.premap = *prog;
    src += "\n// ---- fold module\n";
    std::string fsrc = fold_module_source(sp, prog->n_inputs, 16, 4);
    REMORA_TRY(nvrtc_compile(fsrc, nullptr));
    src += fsrc;
    // the forms with a pass's loads issued at once (one vector per lane
    // and row with the next pass in flight; eight per lane and row)
    REMORA_TRY(nvrtc_compile(fold_module_source(sp, prog->n_inputs, 16, 4, 4, 1), nullptr));
    REMORA_TRY(nvrtc_compile(fold_module_source(sp, prog->n_inputs, 32, 1, 0, 8), nullptr));
  }
  if (src_out && n) std::snprintf(src_out, n, "%s", src.c_str());
  return REMORA_OK;
}

int remora_b200_fold(RemoraB200Ctx *ctx, const RemoraFoldSpec *spec, const void *const *in_descs,
                     const int32_t *in_ranks, int32_t n_in, void *out_desc, int32_t out_rank,
                     remora_stream_t stream) {
  REMORA_TRY(check_ctx(ctx));
  DescView ins[2], out;
  REMORA_TRY(validate_fold(spec, in_descs, in_ranks, n_in, out_desc, out_rank, ins, &out));
  Workspace *ws = nullptr;
  const size_t need = fold_staging_bytes(ins, n_in, out, *spec);
  REMORA_TRY(get_workspace(ctx, (cudaStream_t)stream, need, &ws));
  return run_fold(ctx, *spec, ins, n_in, out, (cudaStream_t)stream, ws->buf, ws->bytes, ws->fold_ticket(), ws->err, false);
}

}  // extern "C"
