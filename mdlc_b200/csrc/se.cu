// Squeeze-excite gate: global average pool -> FC + act -> FC + act in one
// kernel (mdlc_se_fc). The pool is either done already (a pooled [n][c]
// input) or fused: the block averages its images' [hw][c] activations itself
// (16-byte loads, lanes across 8-channel groups so a warp reads whole pixel
// rows, pixel slices summed by a tree in shared memory), which saves the
// pooled tensor's round trip and one launch per gate. The two FCs act on one pixel per image, so
// as tensor-core GEMMs they were two launches of a handful of CTAs each,
// bounded by launch and load latency; here each block takes two images, so
// every weight row it reads from L2 serves two dot products, 32 warps and
// unrolled loops keep many L2 loads in flight (the loops are latency-bound),
// and the hidden layer never leaves shared memory (kept in fp32).
#include "common.cuh"
#include "runtime.h"

namespace mdlc {
namespace {

constexpr int kSeImgs = 2;       // images per block (b = 256: 128 blocks)
constexpr int kSeThreads = 1024;  // 32 warps: the FC loops are latency-bound chains of L2 loads

template <typename T>
MDLC_DEV float se_ld(const T* p);
template <>
MDLC_DEV float se_ld<float>(const float* p) { return __ldg(p); }
template <>
MDLC_DEV float se_ld<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
MDLC_DEV void se_st(T* p, float v);
template <>
MDLC_DEV void se_st<float>(float* p, float v) { *p = v; }
template <>
MDLC_DEV void se_st<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// eight consecutive channels (16 bytes of bf16, 32 of fp32) as fp32
MDLC_DEV void se_ld8(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}
MDLC_DEV void se_ld8(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p));
  const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}

template <typename T>
__global__ void __launch_bounds__(kSeThreads) se_fc_kernel(const mdlc_se_desc d, const T* p, const float* w1,
                                                           const float* b1, const float* w2t, const float* b2,
                                                           T* s, const ActParams a1, const ActParams a2) {
  pdl_wait();  // launched with programmatic serialization: nothing global before this
  pdl_trigger();
  extern __shared__ float se_smem[];
  float* ps = se_smem;                 // [kSeImgs][c] pooled inputs
  float* hs = se_smem + kSeImgs * d.c; // [kSeImgs][rd] hidden layer
  const int n0 = blockIdx.x * kSeImgs;
  const int ni = min(kSeImgs, d.n - n0);
  if (d.hw > 1) {
    // fused squeeze: thread t sums channel group t % G over the pixels of slice
    // t / G (every slices-th pixel), then the slices are added pairwise
    float* part = hs + kSeImgs * d.rd;  // [8][kSeThreads]: conflict-free columns
    const int G = d.c_stride >> 3;      // <= 512 groups of 8 channels
    const int slices = kSeThreads / G;  // >= 2
    const int g = threadIdx.x % G, sl = threadIdx.x / G;
    for (int im = 0; im < kSeImgs; ++im) {
      float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
      if (im < ni && sl < slices) {
        const T* xb = p + (long long)(n0 + im) * d.hw * d.c_stride + g * 8;
#pragma unroll 8
        for (int q = sl; q < d.hw; q += slices) {
          float v[8];
          se_ld8(xb + (long long)q * d.c_stride, v);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] += v[e];
        }
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) part[e * kSeThreads + threadIdx.x] = acc[e];
      __syncthreads();
      for (int st = 1; st < slices; st <<= 1) {
        if (sl < slices && (sl & (2 * st - 1)) == 0 && sl + st < slices) {
#pragma unroll
          for (int e = 0; e < 8; ++e) part[e * kSeThreads + threadIdx.x] += part[e * kSeThreads + threadIdx.x + st * G];
        }
        __syncthreads();
      }
      if (sl == 0) {
#pragma unroll
        for (int e = 0; e < 8; ++e)
          if (g * 8 + e < d.c) ps[im * d.c + g * 8 + e] = part[e * kSeThreads + threadIdx.x] / (float)d.hw;
      }
      __syncthreads();
    }
  } else {
    for (int i = threadIdx.x; i < kSeImgs * d.c; i += kSeThreads) {
      const int im = i / d.c, c = i - im * d.c;
      ps[i] = im < ni ? se_ld<T>(p + (long long)(n0 + im) * d.c_stride + c) : 0.0f;
    }
    __syncthreads();
  }
  // FC1: each warp takes four hidden units at a time, lanes across the input
  // channels, so every lane has four (x2 unrolled: eight) weight loads in flight
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int j0 = warp * 4; j0 < d.rd; j0 += (kSeThreads / 32) * 4) {
    const int nr = min(4, d.rd - j0);
    float acc[4][kSeImgs] = {};
#pragma unroll 2
    for (int i = lane; i < d.c; i += 32) {
      float w[4];
#pragma unroll
      for (int r = 0; r < 4; ++r) w[r] = r < nr ? __ldg(w1 + (long long)(j0 + r) * d.c + i) : 0.0f;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int im = 0; im < kSeImgs; ++im) acc[r][im] = fmaf(w[r], ps[im * d.c + i], acc[r][im]);
    }
#pragma unroll
    for (int r = 0; r < 4; ++r)
#pragma unroll
      for (int im = 0; im < kSeImgs; ++im) {
#pragma unroll
        for (int o = 16; o; o >>= 1) acc[r][im] += __shfl_xor_sync(0xffffffffu, acc[r][im], o);
      }
    if (lane == 0) {
      for (int r = 0; r < nr; ++r) {
        const float bias = b1 ? __ldg(b1 + j0 + r) : 0.0f;
#pragma unroll
        for (int im = 0; im < kSeImgs; ++im) hs[im * d.rd + j0 + r] = apply_act(acc[r][im] + bias, a1);
      }
    }
  }
  __syncthreads();
  // FC2: one thread per output channel, the transposed weights read coalesced
  for (int c = threadIdx.x; c < d.c_stride; c += kSeThreads) {
    float acc[kSeImgs] = {};
    if (c < d.c) {
      const float bias = b2 ? __ldg(b2 + c) : 0.0f;
#pragma unroll
      for (int im = 0; im < kSeImgs; ++im) acc[im] = bias;
      // the loop's L2 loads are independent of the FMAs: unrolled, sixteen are in flight
#pragma unroll 16
      for (int j = 0; j < d.rd; ++j) {
        const float w = __ldg(w2t + (long long)j * d.c + c);
#pragma unroll
        for (int im = 0; im < kSeImgs; ++im) acc[im] = fmaf(w, hs[im * d.rd + j], acc[im]);
      }
#pragma unroll
      for (int im = 0; im < kSeImgs; ++im) acc[im] = apply_act(acc[im], a2);
    }
    for (int im = 0; im < ni; ++im) se_st<T>(s + (long long)(n0 + im) * d.c_stride + c, acc[im]);
  }
}

}  // namespace
}  // namespace mdlc

using namespace mdlc;

extern "C" int mdlc_se_fc(mdlc_ctx* ctx, const mdlc_se_desc* d, const void* pooled, const float* w1,
                          const float* b1, const float* w2t, const float* b2, void* gate) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!d || !pooled || !w1 || !w2t || !gate || d->n <= 0 || d->c <= 0 || d->c > 4096 || d->rd <= 0 ||
      d->rd > 1024 || d->c_stride < d->c || d->c_stride % 8 || d->c_stride > 4096 || d->hw < 0 ||
      (d->dtype != MDLC_BF16 && d->dtype != MDLC_F32))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "se_fc: bad descriptor");
  if (d->hw > 1 && (reinterpret_cast<uintptr_t>(pooled) & 15))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "se_fc: the activations to pool must be 16-byte aligned");
  cudaSetDevice(ctx->device);
  const ActParams a1{d->act1, d->alpha1, d->beta1, d->lo1, d->hi1};
  const ActParams a2{d->act2, d->alpha2, d->beta2, d->lo2, d->hi2};
  // pooled inputs and hidden layer, and with the fused squeeze the slice partials
  const int smem = (kSeImgs * (d->c + d->rd) + (d->hw > 1 ? 8 * kSeThreads : 0)) * (int)sizeof(float);
  const unsigned grid = (unsigned)((d->n + kSeImgs - 1) / kSeImgs);
  cudaError_t e = cudaSuccess;
  if (d->dtype == MDLC_BF16) {
    if (smem > 48 * 1024)
      e = cudaFuncSetAttribute(se_fc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = launch_pdl(se_fc_kernel<__nv_bfloat16>, dim3(grid), dim3(kSeThreads), (size_t)smem, ctx->stream, *d,
                     static_cast<const __nv_bfloat16*>(pooled), w1, b1, w2t, b2, static_cast<__nv_bfloat16*>(gate),
                     a1, a2);
  } else {
    if (smem > 48 * 1024)
      e = cudaFuncSetAttribute(se_fc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      e = launch_pdl(se_fc_kernel<float>, dim3(grid), dim3(kSeThreads), (size_t)smem, ctx->stream, *d,
                     static_cast<const float*>(pooled), w1, b1, w2t, b2, static_cast<float*>(gate), a1, a2);
  }
  if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "se_fc launch");
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "se_fc launch");
}
