// common.cuh — shared host-side helpers of libremora_b200.so: status/error
// reporting, descriptor access, the context with its per-stream workspace.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/remora_b200.h"

namespace remora {

// ---------------------------------------------------------------- errors --
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);

#define REMORA_CUDA_TRY(expr)                                                  \
  do {                                                                         \
    cudaError_t err_ = (expr);                                                 \
    if (err_ != cudaSuccess)                                                   \
      return ::remora::fail(REMORA_ERR_CUDA, "%s failed: %s (%s:%d)", #expr,   \
                            cudaGetErrorString(err_), __FILE__, __LINE__);     \
  } while (0)

#define REMORA_TRY(expr)                                                       \
  do {                                                                         \
    int st_ = (expr);                                                          \
    if (st_ != REMORA_OK) return st_;                                          \
  } while (0)

// ----------------------------------------------------------- descriptors --
// A rank-N descriptor is {allocated, aligned, offset, sizes[N], strides[N]};
// this view reads any rank from its base pointer.
struct DescView {
  char *aligned = nullptr;
  int64_t offset = 0;
  int rank = 0;
  int64_t sizes[REMORA_MAX_RANK] = {0};
  int64_t strides[REMORA_MAX_RANK] = {0};

  int64_t numel() const {
    int64_t n = 1;
    for (int d = 0; d < rank; ++d) n *= sizes[d];
    return n;
  }
  // Address of the logical first element for an element size.
  char *data(int esize) const { return aligned + offset * esize; }
  bool contiguous() const {
    int64_t expect = 1;
    for (int d = rank - 1; d >= 0; --d) {
      if (sizes[d] != 1 && strides[d] != expect) return false;
      expect *= sizes[d];
    }
    return true;
  }
};

int read_desc(const void *desc, int rank, DescView *out, const char *what);

// Bumps the process-wide count of kernels this library has enqueued
// (launched, or recorded into a graph under stream capture); every launch
// site calls it once per kernel.
void note_launch();
int dtype_size(int dtype);

// -------------------------------------------------------------- context --
// Per-stream scratch owned by the library (fold partials, scan tile status,
// split-K partials) plus a device error word that bounded waits set.
struct Workspace {
  void *buf = nullptr;
  size_t bytes = 0;
  // 256-byte device block, zeroed at creation: word 0 is the error word
  // (nonzero after a bounded wait ran out); word 16 is the whole-array
  // fold's block ticket, which only that kernel touches and which it
  // returns to zero when it finishes.  The large buffer `buf` is scratch
  // that every call may overwrite.
  int *err = nullptr;
  unsigned int *fold_ticket() const { return reinterpret_cast<unsigned int *>(err + 16); }
  // Activations of a training step (remora_b200_cnn_step), kept apart from
  // `buf`, which the kernels of the step use as their own scratch.
  void *act = nullptr;
  size_t act_bytes = 0;
};

}  // namespace remora

struct RemoraB200Ctx {
  int device = 0;
  int sm_count = 148;
  // SMs the persistent kernels (GEMM, tensor-core convolutions) may fill;
  // 0: all of them (remora_b200_set_persistent_sms)
  std::atomic<int> persistent_sms{0};
  std::mutex mu;
  std::map<cudaStream_t, remora::Workspace> ws;
  // CTAs a persistent kernel launches at most: one per SM it may fill
  int persistent_limit() const {
    const int n = persistent_sms.load(std::memory_order_relaxed);
    return n > 0 && n < sm_count ? n : sm_count;
  }
};

namespace remora {
// Returns a workspace of at least `bytes` for `stream` (grown on demand).
int get_workspace(RemoraB200Ctx *ctx, cudaStream_t stream, size_t bytes,
                  Workspace **out);
// The stream's activation buffer, at least `bytes` (grown on demand).
int get_activations(RemoraB200Ctx *ctx, cudaStream_t stream, size_t bytes, void **out);
int check_ctx(RemoraB200Ctx *ctx);

constexpr int kMaxFoldBlocks = 1184;  // 148 SMs x 8
}  // namespace remora
