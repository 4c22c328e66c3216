// jit.cuh — per-program kernel generation for lifted maps and fused folds.
//
// The reference turns every map expression into its own kernel text and runs
// it through llc for sm_80 (remora/gpu_lowering.py:556-874,
// remora/pipeline.py:445-477).  Here a map program becomes a CUDA C
// expression spliced into vectorised kernel templates, compiled by NVRTC for
// sm_100a and cached per (program, template parameters).
#pragma once

#include <string>

#include "common.cuh"

namespace remora {

// Validates a program: instruction count, register and input indices,
// write-before-read, ops legal for the compute type.
int validate_program(const RemoraMapProgram &p, int n_inputs);

// CUDA C source of `__device__ T remora_expr(T x0, ..., T x{n-1})`.
std::string gen_expr(const RemoraMapProgram &p);

// NVRTC compile of `source` for sm_100a; the cubin is returned when asked.
// Needs no GPU.
int nvrtc_compile(const std::string &source, std::vector<char> *cubin);

// Cached NVRTC compile of `source`; returns the kernel `name` in it.
int jit_kernel(const std::string &source, const char *name, cudaKernel_t *out);

// Same, keyed by a compact binary `key` that identifies the source: on a hit
// the source is never generated.
template <class MakeSource>
int jit_kernel_keyed(const std::string &key, const char *name, MakeSource make, cudaKernel_t *out);

int jit_lookup(const std::string &key, cudaKernel_t *out);
void jit_remember(const std::string &key, cudaKernel_t k);

template <class MakeSource>
int jit_kernel_keyed(const std::string &key, const char *name, MakeSource make, cudaKernel_t *out) {
  std::string full = key + '\0' + name;
  if (jit_lookup(full, out) == REMORA_OK) return REMORA_OK;
  REMORA_TRY(jit_kernel(make(), name, out));
  jit_remember(full, *out);
  return REMORA_OK;
}

// Appends the raw bytes of a trivially copyable value to a key.
template <class T>
void key_append(std::string &key, const T &v) {
  key.append(reinterpret_cast<const char *>(&v), sizeof(T));
}

}  // namespace remora
