// Host-side context shared by the translation units of libmdlc_b200.so.
#pragma once

#include <cuda_runtime.h>
#include <stdarg.h>

#include <string>

#include "mdlc_b200.h"

static constexpr int kMaxEvents = 4096;
static constexpr int kMaxFences = 64;
// Device-side waits give up after this long (nanoseconds).
static constexpr unsigned long long kWaitLimitNs = 2000000000ull;

struct mdlc_ctx {
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;       // compute stream (every kernel)
  cudaStream_t copy_stream = nullptr;  // host<->device transfers overlapped with compute
  int* d_err = nullptr;  // device error word (first failure wins)
  uint8_t* d_pad = nullptr;  // 256 x 16-byte fill patterns (byte value v at v*16)
  // split-K conv scratch: per-unit partial accumulators and per-tile arrival
  // counters (kept at zero between calls); allocated with the context so no
  // conv call allocates (calls may be captured in a CUDA graph)
  uint32_t* d_split_ws = nullptr;
  int* d_split_cnt = nullptr;
  cudaGraph_t graph = nullptr;
  cudaGraphExec_t graph_exec = nullptr;
  bool capturing = false;
  long long launches = 0;           // kernels launched by this context
  long long captured_launches = 0;  // kernels inside the instantiated graph
  cudaEvent_t events[kMaxEvents] = {};
  cudaEvent_t fences[kMaxFences] = {};  // cross-stream ordering (no timing)
  std::string last_error;
};

int mdlc_set_error(mdlc_ctx* ctx, int status, const char* fmt, ...);
int mdlc_cuda_status(mdlc_ctx* ctx, cudaError_t e, const char* what);

constexpr size_t kSplitWsBytes = 8u << 20;  // split-K partials: 64 units of 128 x 256 fp32
constexpr int kSplitCounters = 1024;

inline void mdlc_note_launch(mdlc_ctx* ctx) {
  if (ctx->capturing)
    ctx->captured_launches++;
  else
    ctx->launches++;
}
