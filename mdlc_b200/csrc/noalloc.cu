// Split-K convolution without any device allocation.
//
// mdlc_conv2d_splitk_noalloc runs the split-K form of the tcgen05 convolution
// kernel (the one conv path that needs scratch memory: per-slice partial
// accumulators and per-tile arrival counters) with that scratch taken from a
// fixed array in this library's device image instead of a context's
// allocations. It is for callers that cannot call cudaMalloc: a plug-in that
// only borrows a stream from a host framework whose memory manager owns every
// device allocation, or a service whose device memory budget is fixed at
// start-up. Such callers cannot create an mdlc_ctx either (creating one
// allocates), so this entry point needs only the caller's stream on the
// current device. No reference counterpart.
#include <atomic>
#include <cstdio>

#include "runtime.h"

namespace {

// Scratch, in 32-bit words: arrival counters, the kernels' error word, then the
// partials region, which has the context workspace's size so the conv path's
// own size check applies unchanged. Every GPU that loads the library holds it
// (8 MiB + 8 KiB) until the process exits; it starts zeroed.
constexpr size_t kCntWords = kSplitCounters;
constexpr size_t kErrWords = 64;
constexpr size_t kWsWords = kSplitWsBytes / 4;
static __device__ __align__(256) uint32_t g_noalloc_scratch[kCntWords + kErrWords + kWsWords];

// The array's device address per device, looked up with that device current
// (host code naming g_noalloc_scratch gets a host-side stand-in, not a device
// address). Host threads may race on the first lookup; each stores the same
// value, through an atomic. The cache is not invalidated: after a device reset
// (cudaDeviceReset, or the primary context being destroyed and re-created) the
// cached address is stale, so such a process must not call these entry points
// again on that device.
std::atomic<void*> g_scratch_addr[64];

// This device's copy of the array, looked up on first use; null (and msg set)
// on failure.
uint32_t* scratch_of_current(int* dev_out, char* msg, size_t msg_len) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    if (msg && msg_len) snprintf(msg, msg_len, "conv2d_splitk_noalloc: no current CUDA device");
    return nullptr;
  }
  void* p = g_scratch_addr[dev].load(std::memory_order_acquire);
  if (!p) {
    // set-up, once per device with it current (the first call on a device
    // does it; that call should come before any stream capture)
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      if (msg && msg_len)
        snprintf(msg, msg_len, "conv2d_splitk_noalloc: scratch address lookup failed: %s", cudaGetErrorString(e));
      return nullptr;
    }
    g_scratch_addr[dev].store(p, std::memory_order_release);
  }
  *dev_out = dev;
  return static_cast<uint32_t*>(p);
}

}  // namespace

extern "C" int mdlc_conv2d_splitk_noalloc(const mdlc_conv_desc* desc, const void* x, const void* w_packed,
                                          const void* bias, const void* residual, void* y,
                                          const mdlc_epilogue* epi, int splits, void* stream, char* msg,
                                          size_t msg_len) {
  auto fail = [&](int status, const char* text) {
    if (msg && msg_len) snprintf(msg, msg_len, "%s", text);
    return status;
  };
  if (!desc) return fail(MDLC_ERR_INVALID, "conv2d_splitk_noalloc: null descriptor");
  if (desc->in_type != MDLC_BF16 || desc->groups != 1)
    return fail(MDLC_ERR_UNSUPPORTED, "conv2d_splitk_noalloc: bf16 inputs and groups == 1 only");
  if (splits < 2 || splits > 255) return fail(MDLC_ERR_INVALID, "conv2d_splitk_noalloc: splits must be 2..255");
  int dev = 0;
  uint32_t* scratch = scratch_of_current(&dev, msg, msg_len);
  if (!scratch) return MDLC_ERR_CUDA;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return fail(MDLC_ERR_CUDA, "conv2d_splitk_noalloc: device attribute query failed");
  // The conv path clears the arrival counters it uses on `stream` before each
  // launch (a call cut short by a bounded wait leaves them non-zero). The error
  // word is left alone: it keeps the first device-side error since the last
  // mdlc_conv2d_splitk_noalloc_status call on this device.
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // a context on the stack around the caller's stream and the fixed scratch:
  // no events, no allocations
  mdlc_ctx tmp;
  tmp.device = dev;
  tmp.num_sms = sms;
  tmp.stream = s;
  tmp.d_split_cnt = reinterpret_cast<int*>(scratch);
  tmp.d_err = reinterpret_cast<int*>(scratch + kCntWords);
  tmp.d_split_ws = scratch + kCntWords + kErrWords;
  mdlc_tile_cfg cfg{};
  cfg.flags = splits << 8;
  const int st = mdlc_conv2d(&tmp, desc, x, w_packed, bias, residual, y, epi, &cfg);
  if (st) return fail(st, tmp.last_error.c_str());
  return MDLC_OK;
}

// Reads (synchronising `stream`) and clears the error word of this device's
// fixed array: the first device-side error any mdlc_conv2d_splitk_noalloc call
// on this device recorded since the last status call, or 0. Allocates nothing.
extern "C" int mdlc_conv2d_splitk_noalloc_status(void* stream, int* flag, char* msg, size_t msg_len) {
  if (!flag) {
    if (msg && msg_len) snprintf(msg, msg_len, "conv2d_splitk_noalloc_status: null flag pointer");
    return MDLC_ERR_INVALID;
  }
  *flag = 0;
  int dev = 0;
  uint32_t* scratch = scratch_of_current(&dev, msg, msg_len);
  if (!scratch) return MDLC_ERR_CUDA;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  int* err = reinterpret_cast<int*>(scratch + kCntWords);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, err, sizeof(int), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e == cudaSuccess && v) e = cudaMemsetAsync(err, 0, sizeof(int), s);
  if (e == cudaSuccess && v) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    if (msg && msg_len) snprintf(msg, msg_len, "conv2d_splitk_noalloc_status: %s", cudaGetErrorString(e));
    return MDLC_ERR_CUDA;
  }
  *flag = v;
  return MDLC_OK;
}
