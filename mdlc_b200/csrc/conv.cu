// mdlc_conv2d dispatch, weight packing, and the depthwise (generic shapes) and
// grouped convolution kernels.
//
// Reference semantics: mdlc/runtime/ops.py:56-81 (conv = im2col + einsum,
// grouped conv per group), ops.py:84-92 (gemm). The reference lowering runs
// conv as explicit im2col + an fp32 FFMA GEMM for one image at a time
// (mdlc/codegen/cuda/emit.py:159-209) and grouped/depthwise conv on the host
// (emit.py:175-180); here every case is a device kernel over the whole batch.
#include <cmath>
#include <cstring>

#include "common.cuh"
#include "conv.h"

namespace mdlc {
namespace {

// ------------------------------------------------------------ depthwise
// One thread per (output pixel, 8-channel group): nine (or r*s) 16-byte
// vector loads of the input, fp32 weights [r*s][cs] and fp32 accumulation.
template <typename T>
struct Vec8;
template <>
struct Vec8<__nv_bfloat16> {
  static MDLC_DEV void load(const __nv_bfloat16* p, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
    f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
  }
  static MDLC_DEV void store(__nv_bfloat16* p, const float (&f)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                              pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
};
template <>
struct Vec8<float> {
  static MDLC_DEV void load(const float* p, float (&f)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  static MDLC_DEV void store(float* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
};

struct DwArgs {
  const void* x;
  const float* w;
  const float* bias;
  const void* res;
  void* y;
  int h, w_, cs, c, r, s, sh, sw, pt, pl, dh, dw, oh, ow, res_s;
  long long total;  // M * cs/8
  ActParams act;
};

template <typename T>
__global__ void __launch_bounds__(256) conv_dw_kernel(const DwArgs a) {
  const int G = a.cs >> 3;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < a.total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(idx % G);
    const long long m = idx / G;
    const int ohw = a.oh * a.ow;
    const int img = (int)(m / ohw);
    const int rem = (int)(m - (long long)img * ohw);
    const int oy = rem / a.ow, ox = rem - (rem / a.ow) * a.ow;
    const int c0 = g * 8;
    float acc[8];
    if (a.bias) {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = c0 + e < a.c ? __ldg(a.bias + c0 + e) : 0.0f;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = 0.0f;
    }
    const T* xb = static_cast<const T*>(a.x) + (long long)img * a.h * a.w_ * a.cs + c0;
    for (int rr = 0; rr < a.r; ++rr) {
      const int ih = oy * a.sh - a.pt + rr * a.dh;
      if ((unsigned)ih >= (unsigned)a.h) continue;
      for (int ss = 0; ss < a.s; ++ss) {
        const int iw = ox * a.sw - a.pl + ss * a.dw;
        if ((unsigned)iw >= (unsigned)a.w_) continue;
        float xv[8], wv[8];
        Vec8<T>::load(xb + ((long long)ih * a.w_ + iw) * a.cs, xv);
        Vec8<float>::load(a.w + (rr * a.s + ss) * a.cs + c0, wv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(xv[e], wv[e], acc[e]);
      }
    }
    if (a.res) {
      float rv[8];
      Vec8<T>::load(static_cast<const T*>(a.res) + m * a.res_s + c0, rv);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += rv[e];
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = (c0 + e < a.c) ? apply_act(acc[e], a.act) : 0.0f;
    Vec8<T>::store(static_cast<T*>(a.y) + m * a.cs + c0, acc);
  }
}

// Depthwise 3x3 (stride 1 or 2, dilation 1) over NHWC, 8 channels per
// thread. Each thread owns one (image, output column, 8-channel group) and
// walks a strip of kDwStrip output rows: the three input pixels of every input
// row it needs sit in a register ring (consecutive output rows share two
// (stride 1) or one (stride 2) of their three input rows), and the group's 72
// weights stay in registers. An input pixel is read from the cache hierarchy
// about three times instead of nine, a weight once per strip; at stride 1 the
// next output row's new input row is loaded before the current row is
// computed. Taps are summed in the same (row, column) order as conv_dw_kernel.
constexpr int kDwStrip = 8;
template <typename T>
struct DwPix;
template <>
struct DwPix<__nv_bfloat16> {
  uint4 v;
  MDLC_DEV void load(const __nv_bfloat16* p) { v = __ldg(reinterpret_cast<const uint4*>(p)); }
  MDLC_DEV void zero() { v = make_uint4(0, 0, 0, 0); }
  MDLC_DEV void get(float (&f)[8]) const {
    f[0] = bf16_lo(v.x); f[1] = bf16_hi(v.x); f[2] = bf16_lo(v.y); f[3] = bf16_hi(v.y);
    f[4] = bf16_lo(v.z); f[5] = bf16_hi(v.z); f[6] = bf16_lo(v.w); f[7] = bf16_hi(v.w);
  }
};
template <>
struct DwPix<float> {
  float4 a, b;
  MDLC_DEV void load(const float* p) {
    a = __ldg(reinterpret_cast<const float4*>(p));
    b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  }
  MDLC_DEV void zero() { a = b = make_float4(0.f, 0.f, 0.f, 0.f); }
  MDLC_DEV void get(float (&f)[8]) const {
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
};

template <typename T, int SH>
__global__ void __launch_bounds__(128) conv_dw3_kernel(const DwArgs a, int strips, int total) {
  const int G = a.cs >> 3;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int g = idx % G;
    int t = idx / G;
    const int ox = t % a.ow;
    t /= a.ow;
    const int strip = t % strips;
    const int img = t / strips;
    const int c0 = g * 8;
    float w[9][8];
#pragma unroll
    for (int tap = 0; tap < 9; ++tap) Vec8<float>::load(a.w + tap * a.cs + c0, w[tap]);
    float bias[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) bias[e] = (a.bias && c0 + e < a.c) ? __ldg(a.bias + c0 + e) : 0.0f;
    const int iw0 = ox * a.sw - a.pl;
    const bool cv0 = (unsigned)iw0 < (unsigned)a.w_, cv1 = (unsigned)(iw0 + 1) < (unsigned)a.w_,
               cv2 = (unsigned)(iw0 + 2) < (unsigned)a.w_;
    const T* xi = static_cast<const T*>(a.x) + (long long)img * a.h * a.w_ * a.cs + c0;
    auto load_row = [&](int ih, DwPix<T> (&r)[3]) {
      if ((unsigned)ih < (unsigned)a.h) {
        const T* p = xi + ((long long)ih * a.w_ + iw0) * a.cs;
        if (cv0) r[0].load(p); else r[0].zero();
        if (cv1) r[1].load(p + a.cs); else r[1].zero();
        if (cv2) r[2].load(p + 2 * a.cs); else r[2].zero();
      } else {
        r[0].zero(); r[1].zero(); r[2].zero();
      }
    };
    auto accumulate = [&](const DwPix<T> (&r)[3], int row, float (&acc)[8]) {
#pragma unroll
      for (int s = 0; s < 3; ++s) {
        float xv[8];
        r[s].get(xv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = fmaf(xv[e], w[row * 3 + s][e], acc[e]);
      }
    };
    const int oy0 = strip * kDwStrip;
    const int oy1 = min(oy0 + kDwStrip, a.oh);
    int ih = oy0 * SH - a.pt;
    // r0..r2: the current output row's input rows; n0 (stride 1): the next
    // output row's new input row, loaded before the current row is computed so
    // the load overlaps the arithmetic
    DwPix<T> r0[3], r1[3], r2[3], n0[3];
    load_row(ih, r0);
    load_row(ih + 1, r1);
    load_row(ih + 2, r2);
    for (int oy = oy0; oy < oy1; ++oy) {
      const bool more = oy + 1 < oy1;
      if (SH == 1 && more) load_row(ih + 3, n0);
      float acc[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = bias[e];
      accumulate(r0, 0, acc);
      accumulate(r1, 1, acc);
      accumulate(r2, 2, acc);
      const long long m = ((long long)img * a.oh + oy) * a.ow + ox;
      if (a.res) {
        float rv[8];
        Vec8<T>::load(static_cast<const T*>(a.res) + m * a.res_s + c0, rv);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] += rv[e];
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = (c0 + e < a.c) ? apply_act(acc[e], a.act) : 0.0f;
      Vec8<T>::store(static_cast<T*>(a.y) + m * a.cs + c0, acc);
      if (more) {
        if (SH == 1) {
#pragma unroll
          for (int s = 0; s < 3; ++s) { r0[s] = r1[s]; r1[s] = r2[s]; r2[s] = n0[s]; }
          ih += 1;
        } else {
          // stride 2: the two new rows are loaded here (prefetching them costs more
          // registers than it saves)
#pragma unroll
          for (int s = 0; s < 3; ++s) r0[s] = r2[s];
          load_row(ih + 3, r1);
          load_row(ih + 4, r2);
          ih += 2;
        }
      }
    }
  }
}

// ------------------------------------------------------------ grouped
// General grouped convolution (1 < groups < c; reference: the per-group loop
// of mdlc/runtime/ops.py:68-78, which the reference GPU lowering sends to the
// host, emit.py:175-180). One thread per (output pixel, output channel); the
// threads of a warp take consecutive output channels of one pixel, so the
// weights, packed [r*s][c/g][k_stride] fp32, are read coalesced and the
// input channels of a group are broadcast to the threads of that group. fp32
// accumulation over taps (row, column) then group channels in order.
struct GroupedArgs {
  const void* x;
  const float* w;
  const float* bias;
  const void* res;
  void* y;
  int h, w_, cs, k, ks, icg, ocg, r, s, sh, sw, pt, pl, dh, dw, oh, ow, res_s;
  long long total;  // M * ks
  ActParams act;
  int* err;
  long long x_elems, w_elems, res_elems;  // element extents (checked build)
};

template <typename T>
MDLC_DEV float ld_f(const T* p);
template <>
MDLC_DEV float ld_f<float>(const float* p) { return __ldg(p); }
template <>
MDLC_DEV float ld_f<__nv_bfloat16>(const __nv_bfloat16* p) { return __bfloat162float(*p); }
template <typename T>
MDLC_DEV void st_f(T* p, float v);
template <>
MDLC_DEV void st_f<float>(float* p, float v) { *p = v; }
template <>
MDLC_DEV void st_f<__nv_bfloat16>(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

template <typename T>
__global__ void __launch_bounds__(256) conv_grouped_kernel(const GroupedArgs a) {
  const int ohw = a.oh * a.ow;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < a.total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int o = (int)(idx % a.ks);
    const long long m = idx / a.ks;
    T* yp = static_cast<T*>(a.y) + m * a.ks + o;
    if (o >= a.k) {
      st_f<T>(yp, 0.0f);
      continue;
    }
    const int img = (int)(m / ohw);
    const int rem = (int)(m - (long long)img * ohw);
    const int oy = rem / a.ow, ox = rem - (rem / a.ow) * a.ow;
    const int c0 = (o / a.ocg) * a.icg;
    float acc = a.bias ? __ldg(a.bias + o) : 0.0f;
    const T* xb = static_cast<const T*>(a.x) + (long long)img * a.h * a.w_ * a.cs + c0;
    for (int rr = 0; rr < a.r; ++rr) {
      const int ih = oy * a.sh - a.pt + rr * a.dh;
      if ((unsigned)ih >= (unsigned)a.h) continue;
      for (int ss = 0; ss < a.s; ++ss) {
        const int iw = ox * a.sw - a.pl + ss * a.dw;
        if ((unsigned)iw >= (unsigned)a.w_) continue;
        const T* xp = xb + ((long long)ih * a.w_ + iw) * a.cs;
        const float* wp = a.w + (long long)(rr * a.s + ss) * a.icg * a.ks + o;
        if (!MDLC_CHECK_IDX(a.err, (xp + a.icg - 1) - static_cast<const T*>(a.x), a.x_elems) ||
            !MDLC_CHECK_IDX(a.err, (wp - a.w) + (long long)(a.icg - 1) * a.ks, a.w_elems))
          continue;
        for (int c = 0; c < a.icg; ++c) acc = fmaf(ld_f<T>(xp + c), __ldg(wp + (long long)c * a.ks), acc);
      }
    }
    if (a.res && MDLC_CHECK_IDX(a.err, m * a.res_s + o, a.res_elems))
      acc += ld_f<T>(static_cast<const T*>(a.res) + m * a.res_s + o);
    st_f<T>(yp, apply_act(acc, a.act));
  }
}

ActParams act_of(const mdlc_epilogue* epi) {
  if (!epi) return ActParams{MDLC_ACT_NONE, 0.f, 0.f, -INFINITY, INFINITY};
  return ActParams{epi->act, epi->alpha, epi->beta, epi->clip_lo, epi->clip_hi};
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

uint16_t f32_to_bf16_rne(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  if ((u & 0x7F800000u) == 0x7F800000u && (u & 0x7FFFFFu)) return (uint16_t)((u >> 16) | 0x40);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}

int validate(mdlc_ctx* ctx, const mdlc_conv_desc* d) {
  if (!d) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: null descriptor");
  if (d->n <= 0 || d->h <= 0 || d->w <= 0 || d->c <= 0 || d->k <= 0 || d->r <= 0 || d->s <= 0 ||
      d->oh <= 0 || d->ow <= 0 || d->stride_h <= 0 || d->stride_w <= 0 || d->dil_h <= 0 ||
      d->dil_w <= 0 || d->pad_t < 0 || d->pad_l < 0 || d->groups <= 0)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: non-positive dimension");
  const bool i8 = d->in_type == MDLC_U8 || d->in_type == MDLC_S8;
  const int align = i8 ? 16 : 8;
  if (d->c_stride < d->c || d->c_stride % align)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: c_stride %d must be >= c and a multiple of %d",
                          d->c_stride, align);
  const bool o8 = d->out_type == MDLC_U8 || d->out_type == MDLC_S8;
  if (d->k_stride < d->k || d->k_stride % (o8 ? 16 : 8))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: k_stride %d must be >= k and a multiple of %d",
                          d->k_stride, o8 ? 16 : 8);
  if (d->res_stride && (d->res_stride < d->k || d->res_stride % (o8 ? 16 : 8)))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: bad res_stride %d", d->res_stride);
  const long long pixels = (long long)d->n * d->h * d->w;
  if (pixels * d->c_stride >= (1ll << 40) || (long long)d->n * d->oh * d->ow >= (1ll << 31) - 256)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: tensor too large");
  return MDLC_OK;
}

enum Path { kPathTC, kPathDW, kPathGrouped, kPathNone };

Path path_of(const mdlc_conv_desc& d) {
  if (d.groups == 1) {
    if (d.in_type == MDLC_BF16 && (d.out_type == MDLC_BF16 || d.out_type == MDLC_F32)) return kPathTC;
    if ((d.in_type == MDLC_U8 || d.in_type == MDLC_S8) &&
        (d.out_type == MDLC_U8 || d.out_type == MDLC_S8 || d.out_type == MDLC_F32 || d.out_type == MDLC_S32))
      return kPathTC;
    if (d.in_type == MDLC_F32 && d.out_type == MDLC_F32) return kPathTC;  // 3xTF32
    return kPathNone;
  }
  if (d.groups == d.c && d.c == d.k && d.in_type == d.out_type &&
      (d.in_type == MDLC_BF16 || d.in_type == MDLC_F32))
    return kPathDW;
  if (d.groups > 1 && d.c % d.groups == 0 && d.k % d.groups == 0 && d.in_type == d.out_type &&
      (d.in_type == MDLC_BF16 || d.in_type == MDLC_F32))
    return kPathGrouped;
  return kPathNone;
}

}  // namespace

int conv_dw(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
            const void* res, void* y, const mdlc_epilogue* epi) {
  DwArgs a{};
  a.x = x; a.w = w; a.bias = bias; a.res = res; a.y = y;
  a.h = d.h; a.w_ = d.w; a.cs = d.c_stride; a.c = d.c; a.r = d.r; a.s = d.s;
  a.sh = d.stride_h; a.sw = d.stride_w; a.pt = d.pad_t; a.pl = d.pad_l; a.dh = d.dil_h; a.dw = d.dil_w;
  a.oh = d.oh; a.ow = d.ow; a.res_s = d.res_stride ? d.res_stride : d.c_stride;
  a.total = (long long)d.n * d.oh * d.ow * (d.c_stride / 8);
  a.act = act_of(epi);
  // 3x3 stride 1 / 2: the TMA halo-staged kernel (csrc/dwconv.cu)
  {
    const int st = conv_dw_tma(ctx, d, x, w, bias, res, y, epi);
    if (st != MDLC_ERR_UNSUPPORTED) return st;
  }
  const int strips = (d.oh + kDwStrip - 1) / kDwStrip;
  const long long strip_total = (long long)d.n * strips * d.ow * (d.c_stride / 8);
  if (d.r == 3 && d.s == 3 && d.dil_h == 1 && d.dil_w == 1 && d.stride_h == d.stride_w &&
      (d.stride_h == 1 || d.stride_h == 2) && strip_total < (1LL << 31)) {
    long long blocks = (strip_total + 127) / 128;
    const long long cap = (long long)ctx->num_sms * 32;
    if (blocks > cap) blocks = cap;
    const bool bf = d.in_type == MDLC_BF16;
    if (d.stride_h == 1) {
      if (bf) conv_dw3_kernel<__nv_bfloat16, 1><<<(unsigned)blocks, 128, 0, ctx->stream>>>(a, strips, (int)strip_total);
      else conv_dw3_kernel<float, 1><<<(unsigned)blocks, 128, 0, ctx->stream>>>(a, strips, (int)strip_total);
    } else {
      if (bf) conv_dw3_kernel<__nv_bfloat16, 2><<<(unsigned)blocks, 128, 0, ctx->stream>>>(a, strips, (int)strip_total);
      else conv_dw3_kernel<float, 2><<<(unsigned)blocks, 128, 0, ctx->stream>>>(a, strips, (int)strip_total);
    }
    mdlc_note_launch(ctx);
    return mdlc_cuda_status(ctx, cudaGetLastError(), "conv_dw3 launch");
  }
  long long blocks = (a.total + 255) / 256;
  const long long cap = (long long)ctx->num_sms * 16;
  if (blocks > cap) blocks = cap;
  if (d.in_type == MDLC_BF16)
    conv_dw_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, ctx->stream>>>(a);
  else
    conv_dw_kernel<float><<<(unsigned)blocks, 256, 0, ctx->stream>>>(a);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "conv_dw launch");
}

int conv_grouped(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
                 const void* res, void* y, const mdlc_epilogue* epi) {
  GroupedArgs a{};
  a.x = x; a.w = w; a.bias = bias; a.res = res; a.y = y;
  a.h = d.h; a.w_ = d.w; a.cs = d.c_stride; a.k = d.k; a.ks = d.k_stride;
  a.icg = d.c / d.groups; a.ocg = d.k / d.groups;
  a.r = d.r; a.s = d.s; a.sh = d.stride_h; a.sw = d.stride_w; a.pt = d.pad_t; a.pl = d.pad_l;
  a.dh = d.dil_h; a.dw = d.dil_w; a.oh = d.oh; a.ow = d.ow;
  a.res_s = d.res_stride ? d.res_stride : d.k_stride;
  a.total = (long long)d.n * d.oh * d.ow * d.k_stride;
  a.act = act_of(epi);
  a.err = ctx->d_err;
  a.x_elems = (long long)d.n * d.h * d.w * d.c_stride;
  a.w_elems = (long long)d.r * d.s * a.icg * d.k_stride;
  a.res_elems = (long long)d.n * d.oh * d.ow * a.res_s;
  long long blocks = (a.total + 255) / 256;
  const long long cap = (long long)ctx->num_sms * 16;
  if (blocks > cap) blocks = cap;
  if (d.in_type == MDLC_BF16)
    conv_grouped_kernel<__nv_bfloat16><<<(unsigned)blocks, 256, 0, ctx->stream>>>(a);
  else
    conv_grouped_kernel<float><<<(unsigned)blocks, 256, 0, ctx->stream>>>(a);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "conv_grouped launch");
}

}  // namespace mdlc

using namespace mdlc;

extern "C" int mdlc_conv_weight_bytes(const mdlc_conv_desc* d, size_t* bytes) {
  if (!d || !bytes) return MDLC_ERR_INVALID;
  const long long kg = (long long)d->r * d->s * d->c_stride;
  switch (path_of(*d)) {
    case kPathTC: {
      const int esz = d->in_type == MDLC_BF16 ? 2 : (d->in_type == MDLC_F32 ? 4 : 1);
      const long long kb = 128 / esz;
      // fp32: a tf32 hi matrix and a lo matrix
      *bytes = (size_t)(((kg + kb - 1) / kb) * 128) * (size_t)d->k * (esz == 4 ? 2 : 1);
      return MDLC_OK;
    }
    case kPathDW:
      *bytes = (size_t)d->r * d->s * d->c_stride * sizeof(float);
      return MDLC_OK;
    case kPathGrouped:
      *bytes = (size_t)d->r * d->s * (d->c / d->groups) * d->k_stride * sizeof(float);
      return MDLC_OK;
    default:
      return MDLC_ERR_UNSUPPORTED;
  }
}

extern "C" int mdlc_pack_conv_weights(const mdlc_conv_desc* d, const float* w, void* out) {
  if (!d || !w || !out) return MDLC_ERR_INVALID;
  size_t bytes = 0;
  int st = mdlc_conv_weight_bytes(d, &bytes);
  if (st) return st;
  std::memset(out, 0, bytes);
  const int C = d->c, K = d->k, R = d->r, S = d->s, cs = d->c_stride;
  const int icg = C / d->groups;
  auto W = [&](int o, int c, int r, int s) { return w[(((long long)o * icg + c) * R + r) * S + s]; };
  switch (path_of(*d)) {
    case kPathTC: {
      const int esz = d->in_type == MDLC_BF16 ? 2 : (d->in_type == MDLC_F32 ? 4 : 1);
      const long long kb = 128 / esz;
      const long long kg_pad = ((1ll * R * S * cs + kb - 1) / kb) * kb;
      for (int o = 0; o < K; ++o)
        for (int r = 0; r < R; ++r)
          for (int s = 0; s < S; ++s)
            for (int c = 0; c < C; ++c) {
              const long long idx = (long long)o * kg_pad + (long long)(r * S + s) * cs + c;
              const float v = W(o, c, r, s);
              if (esz == 4) {
                // tf32 split: hi keeps the top 10 mantissa bits (the rest cleared),
                // lo = v - hi exactly; [hi matrix][lo matrix], each [k][kg_pad]
                uint32_t u;
                std::memcpy(&u, &v, 4);
                u &= 0xFFFFE000u;
                float hi;
                std::memcpy(&hi, &u, 4);
                static_cast<float*>(out)[idx] = hi;
                static_cast<float*>(out)[(long long)K * kg_pad + idx] = v - hi;
              } else if (esz == 2) {
                static_cast<uint16_t*>(out)[idx] = f32_to_bf16_rne(v);
              } else {
                static_cast<int8_t*>(out)[idx] = (int8_t)lrintf(v);
              }
            }
      return MDLC_OK;
    }
    case kPathDW: {
      float* o_ = static_cast<float*>(out);
      for (int c = 0; c < C; ++c)
        for (int r = 0; r < R; ++r)
          for (int s = 0; s < S; ++s) o_[(r * S + s) * cs + c] = W(c, 0, r, s);
      return MDLC_OK;
    }
    case kPathGrouped: {
      // [r*s][c/g][k_stride]: output channel fastest (coalesced across a warp)
      float* o_ = static_cast<float*>(out);
      for (int o = 0; o < K; ++o)
        for (int r = 0; r < R; ++r)
          for (int s = 0; s < S; ++s)
            for (int c = 0; c < icg; ++c)
              o_[((long long)(r * S + s) * icg + c) * d->k_stride + o] = W(o, c, r, s);
      return MDLC_OK;
    }
    default:
      return MDLC_ERR_UNSUPPORTED;
  }
}

extern "C" int mdlc_conv2d(mdlc_ctx* ctx, const mdlc_conv_desc* d, const void* x, const void* w,
                           const void* bias, const void* res, void* y, const mdlc_epilogue* epi,
                           const mdlc_tile_cfg* cfg) {
  if (!ctx) return MDLC_ERR_INVALID;
  int st = validate(ctx, d);
  if (st) return st;
  if (!x || !w || !y) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: null tensor pointer");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (bias && !aligned16(bias)) ||
      (res && !aligned16(res)))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: pointers must be 16-byte aligned");
  cudaSetDevice(ctx->device);
  switch (path_of(*d)) {
    case kPathTC:
      if (d->out_type == MDLC_S32 && res)
        return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv int8: no residual with int32 accumulator output");
      if ((d->in_type == MDLC_U8 || d->in_type == MDLC_S8) && d->out_type != MDLC_F32 &&
          d->out_type != MDLC_S32 && (!epi || (!epi->rq_scale && !epi->rq_mult)))
        return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv int8: requantisation scales or multipliers required");
      if (epi && epi->rq_mult && (!epi->rq_shift || (res && !epi->rq_res_mult)))
        return mdlc_set_error(ctx, MDLC_ERR_INVALID,
                              "conv int8: fixed-point requantisation needs rq_shift (and rq_res_mult with a residual)");
      if ((d->in_type == MDLC_U8 || d->in_type == MDLC_S8) && d->out_type == MDLC_F32 &&
          (!epi || !epi->deq_scale))
        return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv int8: deq_scale required for float output");
      return conv_tc(ctx, *d, x, w, bias, res, y, epi, cfg);
    case kPathDW:
      return conv_dw(ctx, *d, x, static_cast<const float*>(w), static_cast<const float*>(bias), res, y, epi);
    case kPathGrouped:
      return conv_grouped(ctx, *d, x, static_cast<const float*>(w), static_cast<const float*>(bias), res, y, epi);
    default:
      return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED,
                            "conv: groups=%d in_type=%d out_type=%d not supported", d->groups, d->in_type,
                            d->out_type);
  }
}
