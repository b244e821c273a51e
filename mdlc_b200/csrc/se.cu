// Squeeze-excite gate: global-average-pooled activations -> FC + act -> FC +
// act in one kernel (mdlc_se_fc). The two FCs act on one pixel per image, so
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

template <typename T>
__global__ void __launch_bounds__(kSeThreads) se_fc_kernel(const mdlc_se_desc d, const T* p, const float* w1,
                                                           const float* b1, const float* w2t, const float* b2,
                                                           T* s, const ActParams a1, const ActParams a2) {
  extern __shared__ float se_smem[];
  float* ps = se_smem;                 // [kSeImgs][c] pooled inputs
  float* hs = se_smem + kSeImgs * d.c; // [kSeImgs][rd] hidden layer
  const int n0 = blockIdx.x * kSeImgs;
  const int ni = min(kSeImgs, d.n - n0);
  for (int i = threadIdx.x; i < kSeImgs * d.c; i += kSeThreads) {
    const int im = i / d.c, c = i - im * d.c;
    ps[i] = im < ni ? se_ld<T>(p + (long long)(n0 + im) * d.c_stride + c) : 0.0f;
  }
  __syncthreads();
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
      d->rd > 1024 || d->c_stride < d->c || d->c_stride % 8 || (d->dtype != MDLC_BF16 && d->dtype != MDLC_F32))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "se_fc: bad descriptor");
  cudaSetDevice(ctx->device);
  const ActParams a1{d->act1, d->alpha1, d->beta1, d->lo1, d->hi1};
  const ActParams a2{d->act2, d->alpha2, d->beta2, d->lo2, d->hi2};
  const int smem = kSeImgs * (d->c + d->rd) * (int)sizeof(float);
  const unsigned grid = (unsigned)((d->n + kSeImgs - 1) / kSeImgs);
  cudaError_t e = cudaSuccess;
  if (d->dtype == MDLC_BF16) {
    if (smem > 48 * 1024)
      e = cudaFuncSetAttribute(se_fc_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      se_fc_kernel<__nv_bfloat16><<<grid, kSeThreads, smem, ctx->stream>>>(
          *d, static_cast<const __nv_bfloat16*>(pooled), w1, b1, w2t, b2, static_cast<__nv_bfloat16*>(gate), a1, a2);
  } else {
    if (smem > 48 * 1024)
      e = cudaFuncSetAttribute(se_fc_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e == cudaSuccess)
      se_fc_kernel<float><<<grid, kSeThreads, smem, ctx->stream>>>(
          *d, static_cast<const float*>(pooled), w1, b1, w2t, b2, static_cast<float*>(gate), a1, a2);
  }
  if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "se_fc smem attribute");
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "se_fc launch");
}
