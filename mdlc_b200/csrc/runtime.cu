// Context, memory, synchronisation, CUDA-graph capture and timing entry
// points of the C ABI (include/mdlc_b200.h). Replaces the reference's ctypes
// driver wrapper (mdlc/codegen/cuda/nvrtc_runtime.py:162-225).
#include <chrono>
#include <cstdio>
#include <cstring>
#include <string>
#include <thread>

#include "common.cuh"
#include "runtime.h"

using namespace mdlc;

int mdlc_set_error(mdlc_ctx* ctx, int status, const char* fmt, ...) {
  if (ctx) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    ctx->last_error = buf;
  }
  return status;
}

int mdlc_cuda_status(mdlc_ctx* ctx, cudaError_t e, const char* what) {
  if (e == cudaSuccess) return MDLC_OK;
  return mdlc_set_error(ctx, MDLC_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" {

int mdlc_version(void) { return 100; }

int mdlc_device_count(int* count) {
  if (!count) return MDLC_ERR_INVALID;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  *count = (e == cudaSuccess) ? n : 0;
  return MDLC_OK;
}

int mdlc_ctx_create(int device, mdlc_ctx** out) {
  if (!out) return MDLC_ERR_INVALID;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return MDLC_ERR_CUDA;
  if (cudaSetDevice(device) != cudaSuccess) return MDLC_ERR_CUDA;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess) return MDLC_ERR_CUDA;
  if (prop.major != 10) return MDLC_ERR_UNSUPPORTED;  // built for sm_100a only
  mdlc_ctx* ctx = new mdlc_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->copy_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&ctx->d_err, 256) != cudaSuccess ||
      cudaMemset(ctx->d_err, 0, 256) != cudaSuccess || cudaMalloc(&ctx->d_pad, 4096) != cudaSuccess ||
      cudaMalloc(&ctx->d_split_ws, kSplitWsBytes) != cudaSuccess ||
      cudaMalloc(&ctx->d_split_cnt, kSplitCounters * sizeof(int)) != cudaSuccess ||
      cudaMemset(ctx->d_split_cnt, 0, kSplitCounters * sizeof(int)) != cudaSuccess) {
    delete ctx;
    return MDLC_ERR_CUDA;
  }
  {
    uint8_t pat[4096];
    for (int i = 0; i < 4096; ++i) pat[i] = (uint8_t)(i >> 4);
    if (cudaMemcpy(ctx->d_pad, pat, sizeof(pat), cudaMemcpyHostToDevice) != cudaSuccess) {
      delete ctx;
      return MDLC_ERR_CUDA;
    }
  }
  for (int i = 0; i < kMaxEvents; ++i) cudaEventCreate(&ctx->events[i]);
  for (int i = 0; i < kMaxFences; ++i) cudaEventCreateWithFlags(&ctx->fences[i], cudaEventDisableTiming);
  *out = ctx;
  return MDLC_OK;
}

int mdlc_ctx_destroy(mdlc_ctx* ctx) {
  if (!ctx) return MDLC_OK;
  cudaSetDevice(ctx->device);
  cudaStreamSynchronize(ctx->stream);
  if (ctx->copy_stream) cudaStreamSynchronize(ctx->copy_stream);
  if (ctx->graph_exec) cudaGraphExecDestroy(ctx->graph_exec);
  if (ctx->graph) cudaGraphDestroy(ctx->graph);
  for (int i = 0; i < kMaxEvents; ++i) cudaEventDestroy(ctx->events[i]);
  for (int i = 0; i < kMaxFences; ++i)
    if (ctx->fences[i]) cudaEventDestroy(ctx->fences[i]);
  cudaFree(ctx->d_err);
  cudaFree(ctx->d_pad);
  cudaFree(ctx->d_split_ws);
  cudaFree(ctx->d_split_cnt);
  cudaStreamDestroy(ctx->stream);
  if (ctx->copy_stream) cudaStreamDestroy(ctx->copy_stream);
  delete ctx;
  return MDLC_OK;
}

const char* mdlc_last_error(mdlc_ctx* ctx) { return ctx ? ctx->last_error.c_str() : "no context"; }

int mdlc_get_stream(mdlc_ctx* ctx, void** stream) {
  if (!ctx || !stream) return MDLC_ERR_INVALID;
  *stream = (void*)ctx->stream;
  return MDLC_OK;
}

int mdlc_alloc(mdlc_ctx* ctx, size_t bytes, void** dev) {
  if (!ctx || !dev) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  *dev = nullptr;
  cudaError_t e = cudaMalloc(dev, bytes ? bytes : 256);
  if (e == cudaErrorMemoryAllocation)
    return mdlc_set_error(ctx, MDLC_ERR_NOMEM, "cudaMalloc(%zu): out of memory", bytes);
  return mdlc_cuda_status(ctx, e, "cudaMalloc");
}

int mdlc_free(mdlc_ctx* ctx, void* dev) {
  if (!ctx) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaFree(dev), "cudaFree");
}

int mdlc_host_alloc(mdlc_ctx* ctx, size_t bytes, void** host) {
  if (!ctx || !host) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaMallocHost(host, bytes ? bytes : 64), "cudaMallocHost");
}

int mdlc_host_free(mdlc_ctx* ctx, void* host) {
  if (!ctx) return MDLC_ERR_INVALID;
  return mdlc_cuda_status(ctx, cudaFreeHost(host), "cudaFreeHost");
}

int mdlc_upload(mdlc_ctx* ctx, void* dev, const void* host, size_t bytes) {
  if (!ctx || (!dev && bytes) || (!host && bytes)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(
      ctx, cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, ctx->stream), "upload");
}

int mdlc_download(mdlc_ctx* ctx, void* host, const void* dev, size_t bytes) {
  if (!ctx || (!dev && bytes) || (!host && bytes)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(
      ctx, cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, ctx->stream), "download");
}

int mdlc_memset(mdlc_ctx* ctx, void* dev, int value, size_t bytes) {
  if (!ctx) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaMemsetAsync(dev, value, bytes, ctx->stream), "memset");
}

static cudaStream_t stream_of(mdlc_ctx* ctx, int s) {
  return s == MDLC_STREAM_COPY ? ctx->copy_stream : (s == MDLC_STREAM_COMPUTE ? ctx->stream : nullptr);
}

int mdlc_upload_on(mdlc_ctx* ctx, int stream, void* dev, const void* host, size_t bytes) {
  if (!ctx || !stream_of(ctx, stream) || (!dev && bytes) || (!host && bytes)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(
      ctx, cudaMemcpyAsync(dev, host, bytes, cudaMemcpyHostToDevice, stream_of(ctx, stream)), "upload");
}

int mdlc_download_on(mdlc_ctx* ctx, int stream, void* host, const void* dev, size_t bytes) {
  if (!ctx || !stream_of(ctx, stream) || (!dev && bytes) || (!host && bytes)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(
      ctx, cudaMemcpyAsync(host, dev, bytes, cudaMemcpyDeviceToHost, stream_of(ctx, stream)), "download");
}

int mdlc_fence_record(mdlc_ctx* ctx, int id, int stream) {
  if (!ctx || id < 0 || id >= kMaxFences || !stream_of(ctx, stream)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaEventRecord(ctx->fences[id], stream_of(ctx, stream)), "fence record");
}

int mdlc_fence_wait(mdlc_ctx* ctx, int id, int stream) {
  if (!ctx || id < 0 || id >= kMaxFences || !stream_of(ctx, stream)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaStreamWaitEvent(stream_of(ctx, stream), ctx->fences[id], 0), "fence wait");
}

int mdlc_fence_sync(mdlc_ctx* ctx, int id, int timeout_ms) {
  if (!ctx || id < 0 || id >= kMaxFences) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaEventQuery(ctx->fences[id]);
    if (e == cudaSuccess) return MDLC_OK;
    if (e != cudaErrorNotReady) return mdlc_cuda_status(ctx, e, "fence sync");
    if (timeout_ms > 0 && std::chrono::duration_cast<std::chrono::milliseconds>(
                              std::chrono::steady_clock::now() - t0).count() > timeout_ms)
      return mdlc_set_error(ctx, MDLC_ERR_TIMEOUT, "fence %d not reached after %d ms", id, timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

int mdlc_sync(mdlc_ctx* ctx, int timeout_ms) {
  if (!ctx) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  if (timeout_ms <= 0) {
    cudaError_t e = cudaStreamSynchronize(ctx->copy_stream);
    if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
    return mdlc_cuda_status(ctx, e, "sync");
  }
  const auto t0 = std::chrono::steady_clock::now();
  for (;;) {
    cudaError_t e = cudaStreamQuery(ctx->copy_stream);
    if (e == cudaSuccess) e = cudaStreamQuery(ctx->stream);
    if (e == cudaSuccess) return MDLC_OK;
    if (e != cudaErrorNotReady) return mdlc_cuda_status(ctx, e, "sync");
    auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                  std::chrono::steady_clock::now() - t0)
                  .count();
    if (ms > timeout_ms)
      return mdlc_set_error(ctx, MDLC_ERR_TIMEOUT, "stream not idle after %d ms", timeout_ms);
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
}

int mdlc_check_flag(mdlc_ctx* ctx, int* flag) {
  if (!ctx || !flag) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  int v = 0;
  cudaError_t e = cudaMemcpyAsync(&v, ctx->d_err, sizeof(int), cudaMemcpyDeviceToHost, ctx->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ctx->stream);
  if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "check_flag");
  *flag = v;
  if (v) {
    cudaMemsetAsync(ctx->d_err, 0, sizeof(int), ctx->stream);
    cudaStreamSynchronize(ctx->stream);
  }
  return MDLC_OK;
}

int mdlc_graph_begin(mdlc_ctx* ctx) {
  if (!ctx) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  mdlc_graph_reset(ctx);
  ctx->capturing = true;
  ctx->captured_launches = 0;
  return mdlc_cuda_status(
      ctx, cudaStreamBeginCapture(ctx->stream, cudaStreamCaptureModeThreadLocal), "begin capture");
}

int mdlc_graph_end(mdlc_ctx* ctx) {
  if (!ctx || !ctx->capturing) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  ctx->capturing = false;
  cudaError_t e = cudaStreamEndCapture(ctx->stream, &ctx->graph);
  if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "end capture");
  return mdlc_cuda_status(ctx, cudaGraphInstantiate(&ctx->graph_exec, ctx->graph, 0),
                          "graph instantiate");
}

int mdlc_graph_launch(mdlc_ctx* ctx) {
  if (!ctx || !ctx->graph_exec) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  ctx->launches += ctx->captured_launches;
  return mdlc_cuda_status(ctx, cudaGraphLaunch(ctx->graph_exec, ctx->stream), "graph launch");
}

int mdlc_graph_reset(mdlc_ctx* ctx) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (ctx->graph_exec) cudaGraphExecDestroy(ctx->graph_exec);
  if (ctx->graph) cudaGraphDestroy(ctx->graph);
  ctx->graph_exec = nullptr;
  ctx->graph = nullptr;
  return MDLC_OK;
}

int mdlc_event_record(mdlc_ctx* ctx, int slot) {
  if (!ctx || slot < 0 || slot >= kMaxEvents) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaEventRecord(ctx->events[slot], ctx->stream), "event record");
}

int mdlc_event_record_on(mdlc_ctx* ctx, int slot, int stream) {
  if (!ctx || slot < 0 || slot >= kMaxEvents || !stream_of(ctx, stream)) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(ctx, cudaEventRecord(ctx->events[slot], stream_of(ctx, stream)), "event record");
}

int mdlc_event_elapsed(mdlc_ctx* ctx, int a, int b, float* ms) {
  if (!ctx || !ms || a < 0 || b < 0 || a >= kMaxEvents || b >= kMaxEvents) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  cudaError_t e = cudaEventSynchronize(ctx->events[b]);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, ctx->events[a], ctx->events[b]);
  return mdlc_cuda_status(ctx, e, "event elapsed");
}

int mdlc_launch_count(mdlc_ctx* ctx, long long* count) {
  if (!ctx || !count) return MDLC_ERR_INVALID;
  *count = ctx->launches;
  return MDLC_OK;
}

}  // extern "C"

// ---------------------------------------------------------------- probe
// One thread initialises an mbarrier expecting one arrival that never comes
// and waits on it with the library's bounded wait. The wait gives up after
// limit_cycles, records MDLC_DEVERR_WAIT_TIMEOUT and the kernel returns normally.
__global__ void timeout_probe_kernel(int* err, uint64_t limit_cycles) {
  __shared__ __align__(8) uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x != 0) return;
  abort_flag = 0;
  mbar_init(smem_u32(&bar), 1);
  fence_mbar_init();
  mbar_wait(smem_u32(&bar), 0, &abort_flag, err, limit_cycles);
  if (abort_flag) record_error(err, MDLC_DEVERR_WAIT_TIMEOUT);
}

extern "C" int mdlc_debug_timeout_probe(mdlc_ctx* ctx, int limit_us) {
  if (!ctx || limit_us <= 0 || limit_us > 2000000) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  timeout_probe_kernel<<<1, 32, 0, ctx->stream>>>(ctx->d_err, (uint64_t)limit_us * 2000ull);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "timeout probe launch");
}

extern "C" int mdlc_debug_poison_split_counters(mdlc_ctx* ctx, int value) {
  if (!ctx || value < 0 || value > 255) return MDLC_ERR_INVALID;
  cudaSetDevice(ctx->device);
  return mdlc_cuda_status(
      ctx, cudaMemsetAsync(ctx->d_split_cnt, value, kSplitCounters * sizeof(int), ctx->stream),
      "poison split counters");
}
