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

// The array's device address per device, looked up once with that device
// current (host code naming g_noalloc_scratch gets a host-side stand-in, not a
// device address).
void* g_scratch_addr[64] = {};

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
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
    return fail(MDLC_ERR_CUDA, "conv2d_splitk_noalloc: no current CUDA device");
  if (!g_scratch_addr[dev]) {
    // set-up, once per device with it current (the first call on a device
    // does it; that call should come before any stream capture)
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || !p) {
      char t[160];
      snprintf(t, sizeof t, "conv2d_splitk_noalloc: scratch address lookup failed: %s", cudaGetErrorString(e));
      return fail(MDLC_ERR_CUDA, t);
    }
    g_scratch_addr[dev] = p;
  }
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || sms <= 0)
    return fail(MDLC_ERR_CUDA, "conv2d_splitk_noalloc: device attribute query failed");
  uint32_t* scratch = static_cast<uint32_t*>(g_scratch_addr[dev]);
  // the arrival counters (which the kernel leaves at zero, unless a call was
  // cut short) and the error word must start at zero
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (cudaMemsetAsync(scratch, 0, (kCntWords + kErrWords) * 4, s) != cudaSuccess)
    return fail(MDLC_ERR_CUDA, "conv2d_splitk_noalloc: clearing the counters failed");
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
