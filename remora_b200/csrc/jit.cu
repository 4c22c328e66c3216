// jit.cu — program validation, expression code generation and the NVRTC
// compile cache (see jit.cuh).
#include <nvrtc.h>

#include <unordered_map>

#include "jit.cuh"

namespace remora {

namespace {

bool op_is_float_only(int op) {
  return op == REMORA_OP_EXP || op == REMORA_OP_LOG || op == REMORA_OP_SQRT;
}

int op_arity(int op) {
  switch (op) {
  case REMORA_OP_INPUT:
  case REMORA_OP_CONST: return 0;
  case REMORA_OP_NEG:
  case REMORA_OP_EXP:
  case REMORA_OP_LOG:
  case REMORA_OP_SQRT: return 1;
  case REMORA_OP_SELECT: return 3;
  default: return 2;
  }
}

std::string reg(int r) { return "r" + std::to_string(r); }

}  // namespace

int validate_program(const RemoraMapProgram &p, int n_inputs) {
  if (p.n_instr < 1 || p.n_instr > REMORA_MAP_MAX_INSTR)
    return fail(REMORA_ERR_ARG, "map program: n_instr %d outside 1..%d", p.n_instr,
                REMORA_MAP_MAX_INSTR);
  if (p.n_inputs != n_inputs)
    return fail(REMORA_ERR_ARG, "map program: declares %d inputs, call passes %d",
                p.n_inputs, n_inputs);
  if (n_inputs < 0 || n_inputs > REMORA_MAP_MAX_INPUTS)
    return fail(REMORA_ERR_ARG, "map program: %d inputs outside 0..%d", n_inputs,
                REMORA_MAP_MAX_INPUTS);
  if (p.compute_dtype < REMORA_F32 || p.compute_dtype > REMORA_BOOL ||
      p.out_dtype < REMORA_F32 || p.out_dtype > REMORA_BOOL)
    return fail(REMORA_ERR_ARG, "map program: bad compute/out dtype");
  for (int k = 0; k < n_inputs; ++k)
    if (p.in_dtype[k] < REMORA_F32 || p.in_dtype[k] > REMORA_BOOL)
      return fail(REMORA_ERR_ARG, "map program: bad dtype for input %d", k);
  bool written[REMORA_MAP_MAX_REGS] = {false};
  for (int i = 0; i < p.n_instr; ++i) {
    const RemoraMapInstr &in = p.code[i];
    if (in.op >= REMORA_OP_COUNT_)
      return fail(REMORA_ERR_ARG, "map program: instruction %d has unknown op %d", i, in.op);
    if (in.dst >= REMORA_MAP_MAX_REGS)
      return fail(REMORA_ERR_ARG, "map program: instruction %d writes register %d", i, in.dst);
    if (op_is_float_only(in.op) && p.compute_dtype != REMORA_F32)
      return fail(REMORA_ERR_UNSUPPORTED,
                  "map program: exp/log/sqrt need an f32 program (instruction %d)", i);
    int ar = op_arity(in.op);
    const uint8_t ops[3] = {in.a, in.b, in.c};
    for (int q = 0; q < ar; ++q) {
      if (ops[q] >= REMORA_MAP_MAX_REGS || !written[ops[q]])
        return fail(REMORA_ERR_ARG,
                    "map program: instruction %d reads register %d before it is written",
                    i, ops[q]);
    }
    if (in.op == REMORA_OP_INPUT && (in.imm_i < 0 || in.imm_i >= n_inputs))
      return fail(REMORA_ERR_ARG, "map program: instruction %d reads input %d of %d", i,
                  in.imm_i, n_inputs);
    written[in.dst] = true;
  }
  if (p.result < 0 || p.result >= REMORA_MAP_MAX_REGS || !written[p.result])
    return fail(REMORA_ERR_ARG, "map program: result register %d is never written",
                p.result);
  return REMORA_OK;
}

// Every f32 operation is an explicitly rounded intrinsic, so no multiply and
// add are ever contracted into an FMA: results match the CPU path's separate
// arith.mulf / arith.addf bit for bit (division and sqrt are the IEEE
// correctly rounded forms).  exp/log call CUDA's expf/logf.
std::string gen_expr(const RemoraMapProgram &p) {
  const bool f = p.compute_dtype == REMORA_F32;
  const std::string T = f ? "float" : "int";
  std::string s = "__device__ __forceinline__ " + T + " remora_expr(";
  for (int k = 0; k < p.n_inputs; ++k) s += (k ? ", " : "") + T + " x" + std::to_string(k);
  if (p.n_inputs == 0) s += "void";
  s += ") {\n";
  bool used[REMORA_MAP_MAX_REGS] = {false};
  for (int i = 0; i < p.n_instr; ++i) used[p.code[i].dst] = true;
  for (int r = 0; r < REMORA_MAP_MAX_REGS; ++r)
    if (used[r]) s += "  " + T + " " + reg(r) + ";\n";
  char buf[256];
  for (int i = 0; i < p.n_instr; ++i) {
    const RemoraMapInstr &in = p.code[i];
    const std::string a = reg(in.a), b = reg(in.b), c = reg(in.c), d = reg(in.dst);
    const std::string one = f ? "1.0f" : "1", zero = f ? "0.0f" : "0";
    std::string e;
    auto cmp = [&](const char *o) { return "(" + a + " " + o + " " + b + ") ? " + one + " : " + zero; };
    switch (in.op) {
    case REMORA_OP_INPUT: e = "x" + std::to_string(in.imm_i); break;
    case REMORA_OP_CONST:
      if (f) {
        uint32_t bits;
        std::memcpy(&bits, &in.imm_f, 4);
        std::snprintf(buf, sizeof buf, "__int_as_float(0x%08xu)", bits);
        e = buf;
      } else {
        std::snprintf(buf, sizeof buf, "(int)0x%08xu", (uint32_t)in.imm_i);
        e = buf;
      }
      break;
    case REMORA_OP_ADD: e = f ? "__fadd_rn(" + a + ", " + b + ")" : "(int)((unsigned)" + a + " + (unsigned)" + b + ")"; break;
    case REMORA_OP_SUB: e = f ? "__fsub_rn(" + a + ", " + b + ")" : "(int)((unsigned)" + a + " - (unsigned)" + b + ")"; break;
    case REMORA_OP_MUL: e = f ? "__fmul_rn(" + a + ", " + b + ")" : "(int)((unsigned)" + a + " * (unsigned)" + b + ")"; break;
    case REMORA_OP_DIV:
      e = f ? "__fdiv_rn(" + a + ", " + b + ")"
            : "(" + b + " == 0 ? 0 : (" + b + " == -1 ? (int)(0u - (unsigned)" + a + ") : " + a + " / " + b + "))";
      break;
    case REMORA_OP_LT: e = cmp("<"); break;
    case REMORA_OP_LE: e = cmp("<="); break;
    case REMORA_OP_GT: e = cmp(">"); break;
    case REMORA_OP_GE: e = cmp(">="); break;
    case REMORA_OP_EQ: e = cmp("=="); break;
    case REMORA_OP_NE: e = cmp("!="); break;
    case REMORA_OP_SELECT: e = "(" + a + " != " + zero + ") ? " + b + " : " + c; break;
    case REMORA_OP_AND: e = "(" + a + " != " + zero + " && " + b + " != " + zero + ") ? " + one + " : " + zero; break;
    case REMORA_OP_OR: e = "(" + a + " != " + zero + " || " + b + " != " + zero + ") ? " + one + " : " + zero; break;
    case REMORA_OP_NEG: e = f ? "-" + a : "(int)(0u - (unsigned)" + a + ")"; break;
    case REMORA_OP_EXP: e = "expf(" + a + ")"; break;
    case REMORA_OP_LOG: e = "logf(" + a + ")"; break;
    case REMORA_OP_SQRT: e = "sqrtf(" + a + ")"; break;
    }
    s += "  " + d + " = " + e + ";\n";
  }
  s += "  return " + reg(p.result) + ";\n}\n";
  return s;
}

namespace {

struct JitEntry {
  cudaLibrary_t lib = nullptr;
  std::unordered_map<std::string, cudaKernel_t> kernels;
};

std::mutex g_jit_mu;
std::unordered_map<std::string, JitEntry> g_jit_cache;

}  // namespace

int nvrtc_compile(const std::string &source, std::vector<char> *cubin) {
  nvrtcProgram prog;
  if (nvrtcCreateProgram(&prog, source.c_str(), "remora_jit.cu", 0, nullptr, nullptr) != NVRTC_SUCCESS)
    return fail(REMORA_ERR_JIT, "nvrtcCreateProgram failed");
  const char *opts[] = {"-arch=sm_100a", "-std=c++17", "-default-device", "--fmad=false", "-lineinfo"};
  nvrtcResult rc = nvrtcCompileProgram(prog, 5, opts);
  if (rc != NVRTC_SUCCESS) {
    size_t n = 0;
    nvrtcGetProgramLogSize(prog, &n);
    std::string log(n, '\0');
    nvrtcGetProgramLog(prog, &log[0]);
    nvrtcDestroyProgram(&prog);
    return fail(REMORA_ERR_JIT, "NVRTC compile failed: %s\n%.600s", nvrtcGetErrorString(rc), log.c_str());
  }
  if (cubin) {
    size_t n = 0;
    nvrtcGetCUBINSize(prog, &n);
    cubin->resize(n);
    nvrtcGetCUBIN(prog, cubin->data());
  }
  nvrtcDestroyProgram(&prog);
  return REMORA_OK;
}

int jit_kernel(const std::string &source, const char *name, cudaKernel_t *out) {
  std::lock_guard<std::mutex> lock(g_jit_mu);
  auto it = g_jit_cache.find(source);
  if (it == g_jit_cache.end()) {
    std::vector<char> cubin;
    REMORA_TRY(nvrtc_compile(source, &cubin));
    JitEntry e;
    cudaError_t ce = cudaLibraryLoadData(&e.lib, cubin.data(), nullptr, nullptr, 0, nullptr, nullptr, 0);
    if (ce != cudaSuccess)
      return fail(REMORA_ERR_CUDA, "cudaLibraryLoadData failed: %s", cudaGetErrorString(ce));
    it = g_jit_cache.emplace(source, std::move(e)).first;
  }
  JitEntry &e = it->second;
  auto kt = e.kernels.find(name);
  if (kt == e.kernels.end()) {
    cudaKernel_t k;
    cudaError_t ce = cudaLibraryGetKernel(&k, e.lib, name);
    if (ce != cudaSuccess)
      return fail(REMORA_ERR_CUDA, "cudaLibraryGetKernel(%s) failed: %s", name,
                  cudaGetErrorString(ce));
    kt = e.kernels.emplace(name, k).first;
  }
  *out = kt->second;
  return REMORA_OK;
}

namespace {
std::mutex g_key_mu;
std::unordered_map<std::string, cudaKernel_t> g_key_cache;
}  // namespace

int jit_lookup(const std::string &key, cudaKernel_t *out) {
  std::lock_guard<std::mutex> lock(g_key_mu);
  auto it = g_key_cache.find(key);
  if (it == g_key_cache.end()) return REMORA_ERR_ARG;
  *out = it->second;
  return REMORA_OK;
}

void jit_remember(const std::string &key, cudaKernel_t k) {
  std::lock_guard<std::mutex> lock(g_key_mu);
  g_key_cache[key] = k;
}

}  // namespace remora

