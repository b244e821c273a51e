// Data-movement ops (Transpose, Pad, Concat as one 4-D copy kernel) and Softmax
// over NHWC tensors addressed by their logical (n, c, h, w) index. The
// reference GPU executor bounces these to the host (mdlc/codegen/cuda/emit.py:32-35);
// here they are device kernels. Not on any benchmark path: one thread per
// element (copies) and one warp per softmax row keep them simple.
#include <cmath>

#include "common.cuh"
#include "runtime.h"

namespace mdlc {
namespace {

template <typename T>
MDLC_DEV float ldf(const T* p);
template <>
MDLC_DEV float ldf<float>(const float* p) { return *p; }
template <>
MDLC_DEV float ldf<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
MDLC_DEV void stf(T* p, float v);
template <>
MDLC_DEV void stf<float>(float* p, float v) { *p = v; }
template <>
MDLC_DEV void stf<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

// physical offset of logical (n, c, h, w) in an NHWC tensor of dims d, stride cs
MDLC_DEV long long phys(const int (&i)[4], const int32_t* d, int cs) {
  return (((long long)i[0] * d[2] + i[2]) * d[3] + i[3]) * cs + i[1];
}

// index along one source dimension after padding: -1 when it reads the fill value
MDLC_DEV int pad_index(int s, int n, int mode) {
  if ((unsigned)s < (unsigned)n) return s;
  if (mode == 1) return s < 0 ? 0 : n - 1;  // edge
  if (mode == 2 && n > 1) {                 // reflect (the edge element is not repeated)
    const int period = 2 * (n - 1);
    int m = s % period;
    if (m < 0) m += period;
    return m < n ? m : period - m;
  }
  return -1;
}

template <typename T>
__global__ void __launch_bounds__(256) copy_gather_kernel(const mdlc_copy_desc d, const T* x, T* y, long long total) {
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % d.out_cs);
    long long t = idx / d.out_cs;
    const int w = (int)(t % d.out_dims[3]);
    t /= d.out_dims[3];
    const int h = (int)(t % d.out_dims[2]);
    const int n = (int)(t / d.out_dims[2]);
    float v = 0.0f;  // padding channels stay zero
    if (c < d.out_dims[1]) {
      const int o[4] = {n, c, h, w};
      int s[4] = {0, 0, 0, 0};
      bool fill = false;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int sd = d.src_dim[i];
        const int si = pad_index(o[i] - d.offset[i], d.in_dims[sd], d.pad_mode);
        if (si < 0) fill = true;
        s[sd] = si;
      }
      v = fill ? d.value : ldf<T>(x + phys(s, d.in_dims, d.in_cs));
    }
    stf<T>(y + idx, v);
  }
}

template <typename T>
__global__ void __launch_bounds__(256) copy_scatter_kernel(const mdlc_copy_desc d, const T* x, T* y, long long total) {
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int c = (int)(idx % d.in_dims[1]);
    long long t = idx / d.in_dims[1];
    const int w = (int)(t % d.in_dims[3]);
    t /= d.in_dims[3];
    const int h = (int)(t % d.in_dims[2]);
    const int n = (int)(t / d.in_dims[2]);
    const int s[4] = {n, c, h, w};
    int o[4];
    bool inside = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[i] = s[i] + d.offset[i];
      inside = inside && (unsigned)o[i] < (unsigned)d.out_dims[i];
    }
    if (inside) y[phys(o, d.out_dims, d.out_cs)] = x[phys(s, d.in_dims, d.in_cs)];
  }
}

// one warp per row of the softmax axis; fp32 max, sum and division
template <typename T>
__global__ void __launch_bounds__(256) softmax_kernel(const mdlc_softmax_desc d, const T* x, T* y, long long rows) {
  const int lane = threadIdx.x & 31;
  const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
  const int L = d.dims[d.axis];
  // physical stride of each logical dimension
  const long long stride[4] = {(long long)d.dims[2] * d.dims[3] * d.cs, 1, (long long)d.dims[3] * d.cs, d.cs};
  for (long long r = warp0; r < rows; r += nwarps) {
    // the row's fixed indices: the other three dimensions, n outermost
    long long t = r, base = 0;
    for (int i = 3; i >= 0; --i) {
      if (i == d.axis) continue;
      const int v = (int)(t % d.dims[i]);
      t /= d.dims[i];
      base += v * stride[i];
    }
    const long long st = stride[d.axis];
    float m = -INFINITY;
    for (int k = lane; k < L; k += 32) m = fmaxf(m, ldf<T>(x + base + k * st));
#pragma unroll
    for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float sum = 0.0f;
    for (int k = lane; k < L; k += 32) sum += expf(ldf<T>(x + base + k * st) - m);
#pragma unroll
    for (int o = 16; o; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    for (int k = lane; k < L; k += 32) stf<T>(y + base + k * st, expf(ldf<T>(x + base + k * st) - m) / sum);
  }
}

unsigned grid_of(mdlc_ctx* ctx, long long work, int per_block) {
  long long b = (work + per_block - 1) / per_block;
  const long long cap = (long long)ctx->num_sms * 16;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace mdlc

using namespace mdlc;

extern "C" int mdlc_copy4d(mdlc_ctx* ctx, const mdlc_copy_desc* d, const void* x, void* y) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!d || !x || !y || (d->dtype != MDLC_F32 && d->dtype != MDLC_BF16) || (d->mode != 0 && d->mode != 1) ||
      d->pad_mode < 0 || d->pad_mode > 2)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "copy4d: bad descriptor");
  bool seen[4] = {false, false, false, false};
  for (int i = 0; i < 4; ++i) {
    if (d->in_dims[i] <= 0 || d->out_dims[i] <= 0 || d->src_dim[i] < 0 || d->src_dim[i] > 3 || seen[d->src_dim[i]])
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "copy4d: bad dims or src_dim (not a permutation)");
    seen[d->src_dim[i]] = true;
    if (d->mode == 1 && d->src_dim[i] != i)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "copy4d: scatter needs the identity src_dim");
  }
  if (d->in_cs < d->in_dims[1] || d->out_cs < d->out_dims[1] || d->in_cs % 8 || d->out_cs % 8)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "copy4d: channel strides must cover c and be multiples of 8");
  cudaSetDevice(ctx->device);
  const bool bf = d->dtype == MDLC_BF16;
  if (d->mode == 0) {
    const long long total = (long long)d->out_dims[0] * d->out_dims[2] * d->out_dims[3] * d->out_cs;
    if (bf)
      copy_gather_kernel<__nv_bfloat16><<<grid_of(ctx, total, 256), 256, 0, ctx->stream>>>(
          *d, static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), total);
    else
      copy_gather_kernel<float><<<grid_of(ctx, total, 256), 256, 0, ctx->stream>>>(
          *d, static_cast<const float*>(x), static_cast<float*>(y), total);
  } else {
    const long long total = (long long)d->in_dims[0] * d->in_dims[1] * d->in_dims[2] * d->in_dims[3];
    if (bf)
      copy_scatter_kernel<__nv_bfloat16><<<grid_of(ctx, total, 256), 256, 0, ctx->stream>>>(
          *d, static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), total);
    else
      copy_scatter_kernel<float><<<grid_of(ctx, total, 256), 256, 0, ctx->stream>>>(
          *d, static_cast<const float*>(x), static_cast<float*>(y), total);
  }
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "copy4d launch");
}

extern "C" int mdlc_softmax(mdlc_ctx* ctx, const mdlc_softmax_desc* d, const void* x, void* y) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!d || !x || !y || (d->dtype != MDLC_F32 && d->dtype != MDLC_BF16) || d->axis < 0 || d->axis > 3 ||
      d->cs < d->dims[1] || d->cs % 8)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "softmax: bad descriptor");
  for (int i = 0; i < 4; ++i)
    if (d->dims[i] <= 0) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "softmax: bad dims");
  cudaSetDevice(ctx->device);
  const int esz = d->dtype == MDLC_BF16 ? 2 : 4;
  if (d->cs != d->dims[1]) {  // padding channels of y: zero
    const cudaError_t e = cudaMemsetAsync(y, 0, (size_t)d->dims[0] * d->dims[2] * d->dims[3] * d->cs * esz,
                                          ctx->stream);
    if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "softmax padding");
  }
  const long long rows = (long long)d->dims[0] * d->dims[1] * d->dims[2] * d->dims[3] / d->dims[d->axis];
  if (esz == 2)
    softmax_kernel<__nv_bfloat16><<<grid_of(ctx, rows * 32, 256), 256, 0, ctx->stream>>>(
        *d, static_cast<const __nv_bfloat16*>(x), static_cast<__nv_bfloat16*>(y), rows);
  else
    softmax_kernel<float><<<grid_of(ctx, rows * 32, 256), 256, 0, ctx->stream>>>(
        *d, static_cast<const float*>(x), static_cast<float*>(y), rows);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "softmax launch");
}
