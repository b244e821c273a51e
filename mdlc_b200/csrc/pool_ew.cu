// Memory-bound kernels: max / average / global-average pooling and the fused
// elementwise interpreter, all over NHWC with 16-byte vectors of 8 channels.
//
// Reference semantics: mdlc/runtime/ops.py:109-150 (pools), ops.py:155-205
// (activations and broadcasting binary ops), the FusedElementwise subgraph
// evaluation of mdlc/runtime/reference.py:186-195. The reference runs pools on
// the host (mdlc/codegen/cuda/emit.py:32-35) and generates one CUDA kernel per
// elementwise group (templates.py:209-269); here one prebuilt interpreter
// kernel runs any group whose program fits mdlc_ew_prog.
#include <cmath>

#include "common.cuh"
#include "runtime.h"

namespace mdlc {
namespace {

template <typename T>
struct V8;
template <>
struct V8<__nv_bfloat16> {
  static MDLC_DEV void load(const void* p, float (&f)[8]) {
    const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
    f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
    f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
  }
  static MDLC_DEV void store(void* p, const float (&f)[8]) {
    *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                              pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
  }
  static constexpr int kBytes = 2;
};
template <>
struct V8<float> {
  static MDLC_DEV void load(const void* p, float (&f)[8]) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(p));
    const float4 b = __ldg(reinterpret_cast<const float4*>(p) + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  static MDLC_DEV void store(void* p, const float (&f)[8]) {
    reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
    reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
  static constexpr int kBytes = 4;
};

// ------------------------------------------------------------ max / avg pool
template <typename T>
__global__ void __launch_bounds__(256) pool_kernel(const mdlc_pool_desc d, const void* x, void* y,
                                                   long long total) {
  const int G = d.c_stride >> 3;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(idx % G);
    const long long m = idx / G;
    const int ohw = d.oh * d.ow;
    const int img = (int)(m / ohw);
    const int rem = (int)(m - (long long)img * ohw);
    const int oy = rem / d.ow, ox = rem - oy * d.ow;
    float acc[8];
    const bool is_max = d.kind == 0;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[e] = is_max ? -INFINITY : 0.0f;
    int cnt = 0;
    const char* xb = static_cast<const char*>(x) +
                     ((long long)img * d.h * d.w * d.c_stride + g * 8) * V8<T>::kBytes;
    for (int ky = 0; ky < d.kh; ++ky) {
      const int ih = oy * d.stride_h - d.pad_t + ky;
      if ((unsigned)ih >= (unsigned)d.h) continue;
      for (int kx = 0; kx < d.kw; ++kx) {
        const int iw = ox * d.stride_w - d.pad_l + kx;
        if ((unsigned)iw >= (unsigned)d.w) continue;
        float v[8];
        V8<T>::load(xb + ((long long)ih * d.w + iw) * d.c_stride * V8<T>::kBytes, v);
        ++cnt;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = is_max ? fmaxf(acc[e], v[e]) : acc[e] + v[e];
      }
    }
    if (!is_max) {
      // count_include_pad counts the whole window, clipped to the padded input
      // extent as ONNX/ops.averagepool do
      float den = (float)(cnt > 0 ? cnt : 1);
      if (d.count_include_pad) den = (float)(d.kh * d.kw);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] = acc[e] / den;
    }
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (g * 8 + e >= d.c) acc[e] = 0.0f;
    V8<T>::store(static_cast<char*>(y) + (m * d.c_stride + g * 8) * V8<T>::kBytes, acc);
  }
}

// Packed 8-channel max: bf16 pairs through __hmax2, fp32 through fmaxf.
template <typename T>
struct MaxV8;
template <>
struct MaxV8<__nv_bfloat16> {
  using V = uint4;
  static MDLC_DEV V lowest() {
    const uint32_t ni = 0xFF80FF80u;  // two bf16 -inf
    return make_uint4(ni, ni, ni, ni);
  }
  static MDLC_DEV V load(const char* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
  static MDLC_DEV uint32_t m2(uint32_t a, uint32_t b) {
    __nv_bfloat162 r = __hmax2(*reinterpret_cast<__nv_bfloat162*>(&a), *reinterpret_cast<__nv_bfloat162*>(&b));
    return *reinterpret_cast<uint32_t*>(&r);
  }
  static MDLC_DEV V max(V a, V b) { return make_uint4(m2(a.x, b.x), m2(a.y, b.y), m2(a.z, b.z), m2(a.w, b.w)); }
  static MDLC_DEV void store(char* p, V v) { *reinterpret_cast<uint4*>(p) = v; }
  static constexpr int kBytes = 2;
  static constexpr int kVec = 8;  // channels per vector
};
// 8-bit codes: 16 channels per vector, byte-wise max (exact on codes).
template <>
struct MaxV8<uint8_t> {
  using V = uint4;
  static MDLC_DEV V lowest() { return make_uint4(0, 0, 0, 0); }
  static MDLC_DEV V load(const char* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
  static MDLC_DEV V max(V a, V b) {
    return make_uint4(__vmaxu4(a.x, b.x), __vmaxu4(a.y, b.y), __vmaxu4(a.z, b.z), __vmaxu4(a.w, b.w));
  }
  static MDLC_DEV void store(char* p, V v) { *reinterpret_cast<uint4*>(p) = v; }
  static constexpr int kBytes = 1;
  static constexpr int kVec = 16;
};
template <>
struct MaxV8<int8_t> {
  using V = uint4;
  static MDLC_DEV V lowest() {
    const uint32_t m = 0x80808080u;
    return make_uint4(m, m, m, m);
  }
  static MDLC_DEV V load(const char* p) { return __ldg(reinterpret_cast<const uint4*>(p)); }
  static MDLC_DEV V max(V a, V b) {
    return make_uint4(__vmaxs4(a.x, b.x), __vmaxs4(a.y, b.y), __vmaxs4(a.z, b.z), __vmaxs4(a.w, b.w));
  }
  static MDLC_DEV void store(char* p, V v) { *reinterpret_cast<uint4*>(p) = v; }
  static constexpr int kBytes = 1;
  static constexpr int kVec = 16;
};
template <>
struct MaxV8<float> {
  struct V { float4 a, b; };
  static MDLC_DEV V lowest() {
    return V{make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY),
             make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY)};
  }
  static MDLC_DEV V load(const char* p) {
    return V{__ldg(reinterpret_cast<const float4*>(p)), __ldg(reinterpret_cast<const float4*>(p) + 1)};
  }
  static MDLC_DEV float4 m4(float4 a, float4 b) {
    return make_float4(fmaxf(a.x, b.x), fmaxf(a.y, b.y), fmaxf(a.z, b.z), fmaxf(a.w, b.w));
  }
  static MDLC_DEV V max(V a, V b) { return V{m4(a.a, b.a), m4(a.b, b.b)}; }
  static MDLC_DEV void store(char* p, V v) {
    reinterpret_cast<float4*>(p)[0] = v.a;
    reinterpret_cast<float4*>(p)[1] = v.b;
  }
  static constexpr int kBytes = 4;
  static constexpr int kVec = 8;
};

// 3x3 / stride-2 max pool (the ResNet stem pool). Each thread owns one
// (image, output column, 16-byte channel group) and walks kStrip output rows: the
// horizontal max of every input row is taken once and the row shared by
// vertically adjacent windows is carried over, so an output row costs two
// input rows of three 16-byte loads. Channel group fastest: a warp reads whole
// pixels. Padded channels are zero in the input, so they stay zero.
template <typename T, int kStrip>
__global__ void __launch_bounds__(256) maxpool3s2_kernel(const mdlc_pool_desc d, const void* x, void* y,
                                                         int strips, int total) {
  // launched the ordinary way (programmatic serialization measured 1% slower
  // on ResNet-18 b=256); the trigger lets the next conv stage its prologue
  pdl_wait();
  pdl_trigger();
  using M = MaxV8<T>;
  const int G = d.c_stride / M::kVec;
  const long long row_bytes = (long long)d.w * d.c_stride * M::kBytes;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int g = idx % G;
    int t = idx / G;
    const int ox = t % d.ow;
    t /= d.ow;
    const int strip = t % strips;
    const int img = t / strips;
    const int iw0 = ox * 2 - d.pad_l;
    const char* xi = static_cast<const char*>(x) + (long long)img * d.h * row_bytes + (long long)g * M::kVec * M::kBytes;
    const long long px = (long long)d.c_stride * M::kBytes;
    auto hrow = [&](int ih) {
      typename M::V r = M::lowest();
      if ((unsigned)ih < (unsigned)d.h) {
        const char* rp = xi + ih * row_bytes;
#pragma unroll
        for (int kx = 0; kx < 3; ++kx) {
          const int iw = iw0 + kx;
          if ((unsigned)iw < (unsigned)d.w) r = M::max(r, M::load(rp + iw * px));
        }
      }
      return r;
    };
    const int oy0 = strip * kStrip;
    typename M::V carry = hrow(oy0 * 2 - d.pad_t);
    char* yo = static_cast<char*>(y) + (((long long)img * d.oh + oy0) * d.ow + ox) * px + (long long)g * M::kVec * M::kBytes;
    const long long orow = (long long)d.ow * px;
#pragma unroll
    for (int j = 0; j < kStrip; ++j) {
      const int oy = oy0 + j;
      if (oy >= d.oh) break;
      const typename M::V a = hrow(oy * 2 - d.pad_t + 1);
      const typename M::V b = hrow(oy * 2 - d.pad_t + 2);
      M::store(yo + j * orow, M::max(carry, M::max(a, b)));
      carry = b;
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) pool_max_u8_kernel(const mdlc_pool_desc d, const uint8_t* x,
                                                          uint8_t* y, long long total) {
  // 8-bit max pool on 16-channel vectors; max commutes with the monotone
  // quantisation map, so it is exact on the codes.
  const int G = d.c_stride >> 4;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(idx % G);
    const long long m = idx / G;
    const int ohw = d.oh * d.ow;
    const int img = (int)(m / ohw);
    const int rem = (int)(m - (long long)img * ohw);
    const int oy = rem / d.ow, ox = rem - oy * d.ow;
    T best[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) best[e] = (T)(sizeof(T) == 1 && (T)-1 < 0 ? -128 : 0);
    for (int ky = 0; ky < d.kh; ++ky) {
      const int ih = oy * d.stride_h - d.pad_t + ky;
      if ((unsigned)ih >= (unsigned)d.h) continue;
      for (int kx = 0; kx < d.kw; ++kx) {
        const int iw = ox * d.stride_w - d.pad_l + kx;
        if ((unsigned)iw >= (unsigned)d.w) continue;
        const uint4 u = __ldg(reinterpret_cast<const uint4*>(
            x + (((long long)img * d.h + ih) * d.w + iw) * d.c_stride + g * 16));
        const T* t = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int e = 0; e < 16; ++e) best[e] = t[e] > best[e] ? t[e] : best[e];
      }
    }
    *reinterpret_cast<uint4*>(y + m * d.c_stride + g * 16) = *reinterpret_cast<const uint4*>(best);
  }
}

// ------------------------------------------------------------ global average
// One block per (image, up to 32 channel groups): the 256 threads split the
// pixels over however many groups the block holds (a 56-channel tensor keeps
// every thread busy, not 7 of 32 lanes), fp32 sums, then reduce the slices in
// shared memory. (1024 threads per block measured slower: the serial
// reduction over the slices grows with them.)
constexpr int kGapThreads = 256;
template <typename T>
__global__ void __launch_bounds__(kGapThreads) gap_kernel(const mdlc_pool_desc d, const void* x, void* y) {
  pdl_wait();  // a no-op: launched the ordinary way, like the max pool
  pdl_trigger();
  __shared__ float part[kGapThreads][8];
  const int img = blockIdx.x;
  const int g0 = blockIdx.y * 32;
  const int gb = min(32, (d.c_stride >> 3) - g0);  // channel groups in this block
  const int slices = kGapThreads / gb;
  const int t = threadIdx.x;
  const int gl = t % gb, slice = t / gb;
  const int hw = d.h * d.w;
  float acc[8] = {0, 0, 0, 0, 0, 0, 0, 0};
  if (slice < slices) {
    const char* xb =
        static_cast<const char*>(x) + ((long long)img * hw * d.c_stride + (g0 + gl) * 8) * V8<T>::kBytes;
    // unrolled: several independent 16-byte loads in flight per thread (the
    // reduction is latency-bound at one image per block)
#pragma unroll 4
    for (int p = slice; p < hw; p += slices) {
      float v[8];
      V8<T>::load(xb + (long long)p * d.c_stride * V8<T>::kBytes, v);
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[e] += v[e];
    }
  }
#pragma unroll
  for (int e = 0; e < 8; ++e) part[t][e] = acc[e];
  __syncthreads();
  if (t < gb) {
    const int g = g0 + t;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      float s = 0.0f;
      for (int q = 0; q < slices; ++q) s += part[q * gb + t][e];
      acc[e] = (g * 8 + e < d.c) ? s / (float)hw : 0.0f;
    }
    V8<T>::store(static_cast<char*>(y) + ((long long)img * d.c_stride + g * 8) * V8<T>::kBytes, acc);
  }
}

// int8 global average: int32 sum of (q - in_zp), requantised to the output scale
template <typename T>
__global__ void __launch_bounds__(256) gap_q_kernel(const mdlc_pool_desc d, const uint8_t* x, uint8_t* y) {
  const int img = blockIdx.x;
  const int c = blockIdx.y * 256 + threadIdx.x;
  if (c >= d.c_stride) return;
  const int hw = d.h * d.w;
  int32_t s = 0;
  const T* xb = reinterpret_cast<const T*>(x) + (long long)img * hw * d.c_stride + c;
  for (int p = 0; p < hw; ++p) s += (int32_t)xb[(long long)p * d.c_stride] - d.in_zp;
  int32_t q = 0;
  if (c < d.c) {
    q = d.out_zp + requant(s, d.rq_mult, d.rq_shift);
    const int lo = (T)-1 < 0 ? -128 : 0, hi = (T)-1 < 0 ? 127 : 255;
    q = min(max(q, lo), hi);
  }
  reinterpret_cast<T*>(y)[(long long)img * d.c_stride + c] = (T)q;
}

// ------------------------------------------------------------ elementwise
MDLC_DEV float ew_unary(int op, float v, float i0, float i1) {
  switch (op) {
    case MDLC_EW_RELU: return fmaxf(v, 0.0f);
    case MDLC_EW_CLIP: return fminf(fmaxf(v, i0), i1);
    case MDLC_EW_SIGMOID: return 1.0f / (1.0f + expf(-v));
    case MDLC_EW_TANH: return tanhf(v);
    case MDLC_EW_LEAKY_RELU: return v >= 0.0f ? v : i0 * v;
    case MDLC_EW_HARD_SIGMOID: return fminf(fmaxf(i0 * v + i1, 0.0f), 1.0f);
    case MDLC_EW_HARD_SWISH: return v * fminf(fmaxf(v / 6.0f + 0.5f, 0.0f), 1.0f);
    case MDLC_EW_ERF: return erff(v);
    case MDLC_EW_GELU: return gelu_f(v);
    case MDLC_EW_ADDI: return v + i0;
    case MDLC_EW_SUBI: return v - i0;
    case MDLC_EW_RSUBI: return i0 - v;
    case MDLC_EW_MULI: return v * i0;
    case MDLC_EW_DIVI: return v / i0;
    case MDLC_EW_RDIVI: return i0 / v;
    default: return v;
  }
}

template <typename T>
__global__ void __launch_bounds__(256) eltwise_kernel(const __grid_constant__ mdlc_ew_prog p,
                                                      const void* in0, const void* in1, const void* in2,
                                                      const void* in3, void* out0, void* out1,
                                                      long long total) {
  pdl_wait();  // launched with programmatic serialization: nothing global before this
  pdl_trigger();
  const void* ins[4] = {in0, in1, in2, in3};
  const int G = p.c_stride >> 3;
  const long long hwG = (long long)p.hw * G;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(idx % G);
    const long long img = idx / hwG;
    float reg[8][8];
#pragma unroll
    for (int i = 0; i < MDLC_EW_MAX_INPUTS; ++i) {
      if (i >= p.n_inputs) break;
      const int mode = p.bcast[i];
      if (mode == MDLC_BC_SCALAR) {
        const float s = (sizeof(T) == 2) ? __bfloat162float(*static_cast<const __nv_bfloat16*>(ins[i]))
                                         : *static_cast<const float*>(ins[i]);
#pragma unroll
        for (int e = 0; e < 8; ++e) reg[i][e] = s;
      } else {
        long long off = idx * 8;
        if (mode == MDLC_BC_NC) off = (img * p.c_stride) + g * 8;
        if (mode == MDLC_BC_C) off = g * 8;
        V8<T>::load(static_cast<const char*>(ins[i]) + off * V8<T>::kBytes, reg[i]);
      }
    }
    for (int q = 0; q < p.n_instr; ++q) {
      const mdlc_ew_instr in = p.code[q];
      float r[8];
      if (in.op <= MDLC_EW_DIV || in.op == MDLC_EW_MAX || in.op == MDLC_EW_MIN) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float a = reg[in.src0 & 7][e], b = reg[in.src1 & 7][e];
          switch (in.op) {
            case MDLC_EW_ADD: r[e] = a + b; break;
            case MDLC_EW_SUB: r[e] = a - b; break;
            case MDLC_EW_MUL: r[e] = a * b; break;
            case MDLC_EW_DIV: r[e] = a / b; break;
            case MDLC_EW_MAX: r[e] = fmaxf(a, b); break;
            default: r[e] = fminf(a, b); break;
          }
        }
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) r[e] = ew_unary(in.op, reg[in.src0 & 7][e], in.imm0, in.imm1);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) reg[in.dst & 7][e] = r[e];
    }
    void* outs[2] = {out0, out1};
    for (int o = 0; o < p.n_outputs; ++o) {
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = (g * 8 + e < p.c) ? reg[p.out_reg[o] & 7][e] : 0.0f;
      V8<T>::store(static_cast<char*>(outs[o]) + idx * 8 * V8<T>::kBytes, v);
    }
  }
}

unsigned grid_for(mdlc_ctx* ctx, long long total) {
  long long b = (total + 255) / 256;
  const long long cap = (long long)ctx->num_sms * 16;
  return (unsigned)(b < 1 ? 1 : (b > cap ? cap : b));
}

}  // namespace
}  // namespace mdlc

using namespace mdlc;

extern "C" int mdlc_pool2d(mdlc_ctx* ctx, const mdlc_pool_desc* d, const void* x, void* y) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!d || !x || !y) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "pool: null argument");
  const bool q = d->dtype == MDLC_U8 || d->dtype == MDLC_S8;
  if (d->n <= 0 || d->h <= 0 || d->w <= 0 || d->c <= 0 || d->c_stride < d->c ||
      d->c_stride % (q ? 16 : 8))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "pool: bad geometry");
  if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "pool: pointers must be 16-byte aligned");
  cudaSetDevice(ctx->device);
  if (d->kind == 2) {
    if (q) {
      dim3 grid(d->n, (d->c_stride + 255) / 256);
      if (d->dtype == MDLC_U8)
        gap_q_kernel<uint8_t><<<grid, 256, 0, ctx->stream>>>(*d, static_cast<const uint8_t*>(x),
                                                             static_cast<uint8_t*>(y));
      else
        gap_q_kernel<int8_t><<<grid, 256, 0, ctx->stream>>>(*d, static_cast<const uint8_t*>(x),
                                                            static_cast<uint8_t*>(y));
    } else {
      dim3 grid(d->n, (d->c_stride / 8 + 31) / 32);
      if (d->dtype == MDLC_BF16)
        gap_kernel<__nv_bfloat16><<<grid, kGapThreads, 0, ctx->stream>>>(*d, x, y);
      else if (d->dtype == MDLC_F32)
        gap_kernel<float><<<grid, kGapThreads, 0, ctx->stream>>>(*d, x, y);
      else
        return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "pool: dtype %d", d->dtype);
    }
  } else {
    if (d->oh <= 0 || d->ow <= 0 || d->kh <= 0 || d->kw <= 0 || d->stride_h <= 0 || d->stride_w <= 0)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "pool: bad window");
    constexpr int kStrip = 8;
    const int strips = (d->oh + kStrip - 1) / kStrip;
    const long long strip_total = (long long)d->n * strips * d->ow * (d->c_stride / (q ? 16 : 8));
    const bool s32 = d->kind == 0 && d->kh == 3 && d->kw == 3 && d->stride_h == 2 && d->stride_w == 2 &&
                     d->pad_t <= 1 && d->pad_l <= 1 && strip_total < (1LL << 31) &&
                     (d->oh - 1) * 2 - d->pad_t < d->h && (d->ow - 1) * 2 - d->pad_l < d->w;
    if (q) {
      if (d->kind != 0) return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "pool: int8 average pool");
      const long long total = (long long)d->n * d->oh * d->ow * (d->c_stride / 16);
      if (s32 && d->dtype == MDLC_U8)
        maxpool3s2_kernel<uint8_t, kStrip><<<grid_for(ctx, strip_total), 256, 0, ctx->stream>>>(
            *d, x, y, strips, (int)strip_total);
      else if (s32)
        maxpool3s2_kernel<int8_t, kStrip><<<grid_for(ctx, strip_total), 256, 0, ctx->stream>>>(
            *d, x, y, strips, (int)strip_total);
      else if (d->dtype == MDLC_U8)
        pool_max_u8_kernel<uint8_t><<<grid_for(ctx, total), 256, 0, ctx->stream>>>(
            *d, static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), total);
      else
        pool_max_u8_kernel<int8_t><<<grid_for(ctx, total), 256, 0, ctx->stream>>>(
            *d, static_cast<const uint8_t*>(x), static_cast<uint8_t*>(y), total);
    } else {
      const long long total = (long long)d->n * d->oh * d->ow * (d->c_stride / 8);
      if (s32 && d->dtype == MDLC_BF16)
        maxpool3s2_kernel<__nv_bfloat16, kStrip><<<grid_for(ctx, strip_total), 256, 0, ctx->stream>>>(
            *d, x, y, strips, (int)strip_total);
      else if (s32 && d->dtype == MDLC_F32)
        maxpool3s2_kernel<float, kStrip><<<grid_for(ctx, strip_total), 256, 0, ctx->stream>>>(
            *d, x, y, strips, (int)strip_total);
      else if (d->dtype == MDLC_BF16)
        pool_kernel<__nv_bfloat16><<<grid_for(ctx, total), 256, 0, ctx->stream>>>(*d, x, y, total);
      else if (d->dtype == MDLC_F32)
        pool_kernel<float><<<grid_for(ctx, total), 256, 0, ctx->stream>>>(*d, x, y, total);
      else
        return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "pool: dtype %d", d->dtype);
    }
  }
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "pool launch");
}

namespace mdlc {
namespace {

// Fast path of the interpreter for out = [unary](in0 (op) in1): two inputs, in0
// full, in1 broadcast per the given mode, one binary instruction and at most
// one unary one after it (the squeeze-excite multiply, a residual add + act
// not absorbed into a conv). Values stay in registers (the interpreter's
// register file is indexed at run time and lives in local memory).
template <typename T, int BC>
__global__ void __launch_bounds__(256) eltwise_binary_kernel(const mdlc_ew_prog p, const void* in0, const void* in1,
                                                             void* out0, int bop, int uop, float u0, float u1,
                                                             long long total) {
  pdl_wait();  // launched with programmatic serialization: nothing global before this
  pdl_trigger();
  const int G = p.c_stride >> 3;
  const long long hwG = (long long)p.hw * G;
  float bs = 0.0f;
  if (BC == MDLC_BC_SCALAR)
    bs = (sizeof(T) == 2) ? __bfloat162float(*static_cast<const __nv_bfloat16*>(in1)) : *static_cast<const float*>(in1);
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int g = (int)(idx % G);
    float a[8], b[8];
    V8<T>::load(static_cast<const char*>(in0) + idx * 8 * V8<T>::kBytes, a);
    if (BC == MDLC_BC_SCALAR) {
#pragma unroll
      for (int e = 0; e < 8; ++e) b[e] = bs;
    } else {
      const long long off = BC == MDLC_BC_FULL ? idx * 8 : (BC == MDLC_BC_NC ? (idx / hwG) * p.c_stride + g * 8 : g * 8);
      V8<T>::load(static_cast<const char*>(in1) + off * V8<T>::kBytes, b);
    }
    float r[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      switch (bop) {
        case MDLC_EW_ADD: r[e] = a[e] + b[e]; break;
        case MDLC_EW_SUB: r[e] = a[e] - b[e]; break;
        case MDLC_EW_MUL: r[e] = a[e] * b[e]; break;
        case MDLC_EW_DIV: r[e] = a[e] / b[e]; break;
        case MDLC_EW_MAX: r[e] = fmaxf(a[e], b[e]); break;
        default: r[e] = fminf(a[e], b[e]); break;
      }
    }
    if (uop >= 0) {
#pragma unroll
      for (int e = 0; e < 8; ++e) r[e] = ew_unary(uop, r[e], u0, u1);
    }
#pragma unroll
    for (int e = 0; e < 8; ++e) r[e] = (g * 8 + e < p.c) ? r[e] : 0.0f;
    V8<T>::store(static_cast<char*>(out0) + idx * 8 * V8<T>::kBytes, r);
  }
}

bool is_binary(int op) { return op <= MDLC_EW_DIV || op == MDLC_EW_MAX || op == MDLC_EW_MIN; }

// Runs the program on the fast path when it has that shape; false otherwise.
template <typename T>
bool eltwise_fast(mdlc_ctx* ctx, const mdlc_ew_prog* p, const void* const* in, void* const* out, long long total) {
  if (p->n_inputs != 2 || p->n_outputs != 1 || p->bcast[0] != MDLC_BC_FULL || p->n_instr < 1 || p->n_instr > 2)
    return false;
  const mdlc_ew_instr& b = p->code[0];
  if (!is_binary(b.op) || b.src0 != 0 || b.src1 != 1 || b.dst < 2) return false;
  int uop = -1;
  float u0 = 0.0f, u1 = 0.0f;
  int last = b.dst;
  if (p->n_instr == 2) {
    const mdlc_ew_instr& u = p->code[1];
    if (is_binary(u.op) || u.src0 != b.dst) return false;
    uop = u.op, u0 = u.imm0, u1 = u.imm1, last = u.dst;
  }
  if (p->out_reg[0] != last) return false;
  const unsigned grid = grid_for(ctx, total);
  switch (p->bcast[1]) {
    case MDLC_BC_FULL:
      launch_pdl(eltwise_binary_kernel<T, MDLC_BC_FULL>, dim3(grid), dim3(256), 0, ctx->stream, *p, in[0], in[1], out[0], b.op, uop,
                 u0, u1, total);
      break;
    case MDLC_BC_NC:
      launch_pdl(eltwise_binary_kernel<T, MDLC_BC_NC>, dim3(grid), dim3(256), 0, ctx->stream, *p, in[0], in[1], out[0], b.op, uop,
                 u0, u1, total);
      break;
    case MDLC_BC_C:
      launch_pdl(eltwise_binary_kernel<T, MDLC_BC_C>, dim3(grid), dim3(256), 0, ctx->stream, *p, in[0], in[1], out[0], b.op, uop,
                 u0, u1, total);
      break;
    default:
      launch_pdl(eltwise_binary_kernel<T, MDLC_BC_SCALAR>, dim3(grid), dim3(256), 0, ctx->stream, *p, in[0], in[1], out[0], b.op, uop,
                 u0, u1, total);
      break;
  }
  return true;
}

}  // namespace
}  // namespace mdlc

extern "C" int mdlc_eltwise(mdlc_ctx* ctx, const mdlc_ew_prog* p, const void* const* inputs,
                            void* const* outputs) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!p || !inputs || !outputs) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "eltwise: null argument");
  if (p->n_inputs < 1 || p->n_inputs > MDLC_EW_MAX_INPUTS || p->n_outputs < 1 ||
      p->n_outputs > MDLC_EW_MAX_OUTPUTS || p->n_instr < 0 || p->n_instr > MDLC_EW_MAX_INSTR ||
      p->c_stride % 8 || p->c_stride < p->c || p->n <= 0 || p->hw <= 0)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "eltwise: bad program header");
  for (int i = 0; i < p->n_instr; ++i) {
    const mdlc_ew_instr& in = p->code[i];
    if (in.dst < 0 || in.dst > 7 || in.src0 < 0 || in.src0 > 7 || in.src1 < 0 || in.src1 > 7 || in.op < 0 ||
        in.op > MDLC_EW_MIN)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "eltwise: bad instruction %d", i);
  }
  const void* in[4] = {nullptr, nullptr, nullptr, nullptr};
  void* out[2] = {nullptr, nullptr};
  for (int i = 0; i < p->n_inputs; ++i) {
    in[i] = inputs[i];
    if (!in[i] || (reinterpret_cast<uintptr_t>(in[i]) & 15 && p->bcast[i] != MDLC_BC_SCALAR))
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "eltwise: input %d null or misaligned", i);
  }
  for (int i = 0; i < p->n_outputs; ++i) {
    out[i] = outputs[i];
    if (!out[i] || reinterpret_cast<uintptr_t>(out[i]) & 15)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "eltwise: output %d null or misaligned", i);
  }
  cudaSetDevice(ctx->device);
  const long long total = (long long)p->n * p->hw * (p->c_stride / 8);
  if ((p->dtype == MDLC_BF16 && eltwise_fast<__nv_bfloat16>(ctx, p, in, out, total)) ||
      (p->dtype == MDLC_F32 && eltwise_fast<float>(ctx, p, in, out, total))) {
    mdlc_note_launch(ctx);
    return mdlc_cuda_status(ctx, cudaGetLastError(), "eltwise launch");
  }
  if (p->dtype == MDLC_BF16)
    launch_pdl(eltwise_kernel<__nv_bfloat16>, dim3(grid_for(ctx, total)), dim3(256), 0, ctx->stream, *p, in[0], in[1],
               in[2], in[3], out[0], out[1], total);
  else if (p->dtype == MDLC_F32)
    launch_pdl(eltwise_kernel<float>, dim3(grid_for(ctx, total)), dim3(256), 0, ctx->stream, *p, in[0], in[1], in[2],
               in[3], out[0], out[1], total);
  else
    return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "eltwise: dtype %d", p->dtype);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "eltwise launch");
}

// ------------------------------------------------------------ layout
namespace mdlc {
namespace {

// NCHW fp32 -> NHWC (channel stride cs): one thread per (image, pixel,
// 8-channel group) with the pixel index fastest, so reads of each channel
// plane are coalesced across the warp and each thread writes one 16-byte (or
// 8-byte for 8-bit types) vector.
template <int DT>
__global__ void __launch_bounds__(256) to_nhwc_kernel(const float* x, int n, int c, int hw, void* y, int cs,
                                                      float inv_scale, int zp, long long total) {
  const int G = (cs + 7) >> 3;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(idx % hw);
    const long long t = idx / hw;
    const int g = (int)(t % G);
    const int img = (int)(t / G);
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int ch = g * 8 + e;
      v[e] = ch < c ? __ldg(x + ((long long)img * c + ch) * hw + p) : 0.0f;
    }
    const long long o = ((long long)img * hw + p) * cs + g * 8;
    if constexpr (DT == MDLC_F32) {
      V8<float>::store(static_cast<float*>(y) + o, v);
    } else if constexpr (DT == MDLC_BF16) {
      V8<__nv_bfloat16>::store(static_cast<__nv_bfloat16*>(y) + o, v);
    } else {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int q = 0;
        if (g * 8 + e < c) {
          q = __float2int_rn(__fmul_rn(v[e], inv_scale)) + zp;
          q = DT == MDLC_S8 ? min(max(q, -128), 127) : min(max(q, 0), 255);
        } else {
          q = 0;
        }
        const uint32_t b = (uint32_t)(q & 0xFF) << (8 * (e & 3));
        if (e < 4) lo |= b; else hi |= b;
      }
      *reinterpret_cast<uint2*>(static_cast<uint8_t*>(y) + o) = make_uint2(lo, hi);
    }
  }
}

// NCHW fp32 -> 2x2 space-to-depth NHWC; one thread per (image, output pixel,
// 8-channel group), output pixel index fastest.
template <int DT>
__global__ void __launch_bounds__(256) to_s2d_kernel(const float* x, int c, int h, int w, void* y, int cs,
                                                     float inv_scale, int zp, long long total) {
  const int G = cs >> 3;
  const int h2 = h >> 1, w2 = w >> 1, hw2 = h2 * w2;
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(idx % hw2);
    const long long t = idx / hw2;
    const int g = (int)(t % G);
    const int img = (int)(t / G);
    const int Y = p / w2, X = p - (p / w2) * w2;
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const int cc = g * 8 + e;
      v[e] = 0.0f;
      if (cc < 4 * c) {
        const int q = cc / c, ci = cc - q * c;
        const int dy = q >> 1, dx = q & 1;
        v[e] = __ldg(x + (((long long)img * c + ci) * h + 2 * Y + dy) * w + 2 * X + dx);
      }
    }
    const long long o = ((long long)img * hw2 + p) * cs + g * 8;
    if constexpr (DT == MDLC_F32) {
      V8<float>::store(static_cast<float*>(y) + o, v);
    } else if constexpr (DT == MDLC_BF16) {
      V8<__nv_bfloat16>::store(static_cast<__nv_bfloat16*>(y) + o, v);
    } else {
      uint32_t lo = 0, hi = 0;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        int q = 0;
        if (g * 8 + e < 4 * c) {
          q = __float2int_rn(__fmul_rn(v[e], inv_scale)) + zp;
          q = DT == MDLC_S8 ? min(max(q, -128), 127) : min(max(q, 0), 255);
        }
        const uint32_t b = (uint32_t)(q & 0xFF) << (8 * (e & 3));
        if (e < 4) lo |= b; else hi |= b;
      }
      *reinterpret_cast<uint2*>(static_cast<uint8_t*>(y) + o) = make_uint2(lo, hi);
    }
  }
}

// The image-stem case of the above: at most 4 input channels into CS = 16 or
// 32 output channels. One thread per PX horizontally adjacent output pixels
// reads one 2*PX-float vector (float2 / float4) per (channel, row) --
// coalesced across the warp -- and writes each pixel's CS channels with
// full-width vector stores, so the input is read once and every byte written
// is a whole 32-byte sector. PX = 2 (when the output row width is even)
// halves the index arithmetic per pixel and doubles the bytes per load.
template <int DT, int CS>
MDLC_DEV void s2d_store_pixel(void* y, long long pix, const float (&v)[16], float inv_scale, int zp, int nvals) {
  const long long o = pix * CS;
  if constexpr (DT == MDLC_F32) {
    float4* yo = reinterpret_cast<float4*>(static_cast<float*>(y) + o);
#pragma unroll
    for (int j = 0; j < CS / 4; ++j)
      yo[j] = j < 4 ? make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]) : make_float4(0, 0, 0, 0);
  } else if constexpr (DT == MDLC_BF16) {
    uint32_t u[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) u[j] = pack_bf16x2(v[2 * j], v[2 * j + 1]);
    uint4* yo = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(y) + o);
    yo[0] = make_uint4(u[0], u[1], u[2], u[3]);
    yo[1] = make_uint4(u[4], u[5], u[6], u[7]);
#pragma unroll
    for (int j = 2; j < CS / 8; ++j) yo[j] = make_uint4(0, 0, 0, 0);
  } else {
    uint32_t u[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      if (e < nvals) {
        int q = __float2int_rn(__fmul_rn(v[e], inv_scale)) + zp;
        q = DT == MDLC_S8 ? min(max(q, -128), 127) : min(max(q, 0), 255);
        u[e >> 2] |= (uint32_t)(q & 0xFF) << (8 * (e & 3));
      }
    }
    uint4* yo = reinterpret_cast<uint4*>(static_cast<uint8_t*>(y) + o);
    yo[0] = make_uint4(u[0], u[1], u[2], u[3]);
#pragma unroll
    for (int j = 1; j < CS / 16; ++j) yo[j] = make_uint4(0, 0, 0, 0);
  }
}

template <int DT, int C, int CS, int PX>
__global__ void __launch_bounds__(256) to_s2d16_kernel(const float* x, int h, int w, void* y, float inv_scale,
                                                       int zp, int total) {
  // total: output pixels / PX; a thread's pixels are (Y, PX*Xg .. PX*Xg + PX-1)
  const int w2 = w >> 1, wg = w2 / PX, hwg = (h >> 1) * wg;
  for (int idx = blockIdx.x * blockDim.x + threadIdx.x; idx < total; idx += gridDim.x * blockDim.x) {
    const int img = idx / hwg;
    const int p = idx - img * hwg;
    const int Y = p / wg, Xg = p - Y * wg;
    float v[PX][16];
#pragma unroll
    for (int q = 0; q < PX; ++q)
#pragma unroll
      for (int e = 0; e < 16; ++e) v[q][e] = 0.0f;
#pragma unroll
    for (int ci = 0; ci < C; ++ci)
#pragma unroll
      for (int dy = 0; dy < 2; ++dy) {
        const float* src = x + (((long long)img * C + ci) * h + 2 * Y + dy) * w + 2 * PX * Xg;
        if constexpr (PX == 2) {
          const float4 f = __ldg(reinterpret_cast<const float4*>(src));
          v[0][(2 * dy) * C + ci] = f.x;
          v[0][(2 * dy + 1) * C + ci] = f.y;
          v[1][(2 * dy) * C + ci] = f.z;
          v[1][(2 * dy + 1) * C + ci] = f.w;
        } else {
          const float2 f = __ldg(reinterpret_cast<const float2*>(src));
          v[0][(2 * dy) * C + ci] = f.x;
          v[0][(2 * dy + 1) * C + ci] = f.y;
        }
      }
    const long long pix0 = ((long long)img * (h >> 1) + Y) * w2 + (long long)PX * Xg;
#pragma unroll
    for (int q = 0; q < PX; ++q) s2d_store_pixel<DT, CS>(y, pix0 + q, v[q], inv_scale, zp, 4 * C);
  }
}

template <int DT, int CS, int PX>
void launch_s2d16_px(mdlc_ctx* ctx, const float* x, int c, int h, int w, void* y, float inv_scale, int zp,
                     int total) {
  const unsigned grid = grid_for(ctx, total);
  switch (c) {
    case 1: to_s2d16_kernel<DT, 1, CS, PX><<<grid, 256, 0, ctx->stream>>>(x, h, w, y, inv_scale, zp, total); break;
    case 2: to_s2d16_kernel<DT, 2, CS, PX><<<grid, 256, 0, ctx->stream>>>(x, h, w, y, inv_scale, zp, total); break;
    case 3: to_s2d16_kernel<DT, 3, CS, PX><<<grid, 256, 0, ctx->stream>>>(x, h, w, y, inv_scale, zp, total); break;
    default: to_s2d16_kernel<DT, 4, CS, PX><<<grid, 256, 0, ctx->stream>>>(x, h, w, y, inv_scale, zp, total); break;
  }
}

template <int DT, int CS>
void launch_s2d16(mdlc_ctx* ctx, const float* x, int c, int h, int w, void* y, float inv_scale, int zp,
                  int total) {
  // two pixels per thread when every thread's float4 is 16-byte aligned: rows
  // of w floats with w % 4 == 0 (the output row width w / 2 is even)
  if (w % 4 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0)
    launch_s2d16_px<DT, CS, 2>(ctx, x, c, h, w, y, inv_scale, zp, total / 2);
  else
    launch_s2d16_px<DT, CS, 1>(ctx, x, c, h, w, y, inv_scale, zp, total);
}

template <int DT>
void launch_s2d_stem(mdlc_ctx* ctx, const float* x, int c, int h, int w, void* y, int cs, float inv_scale,
                     int zp, int total) {
  if (cs == 16)
    launch_s2d16<DT, 16>(ctx, x, c, h, w, y, inv_scale, zp, total);
  else
    launch_s2d16<DT, 32>(ctx, x, c, h, w, y, inv_scale, zp, total);
}

template <int DT>
__global__ void __launch_bounds__(256) to_nchw_kernel(const void* x, int n, int c, int hw, int cs, float* y,
                                                      float scale, int zp, long long total) {
  for (long long idx = (long long)blockIdx.x * blockDim.x + threadIdx.x; idx < total;
       idx += (long long)gridDim.x * blockDim.x) {
    const int p = (int)(idx % hw);
    const long long t = idx / hw;
    const int ch = (int)(t % c);
    const int img = (int)(t / c);
    const long long i = ((long long)img * hw + p) * cs + ch;
    float v;
    if constexpr (DT == MDLC_F32) v = static_cast<const float*>(x)[i];
    else if constexpr (DT == MDLC_BF16) v = __bfloat162float(static_cast<const __nv_bfloat16*>(x)[i]);
    else if constexpr (DT == MDLC_S8) v = __fmul_rn((float)((int)static_cast<const int8_t*>(x)[i] - zp), scale);
    else v = __fmul_rn((float)((int)static_cast<const uint8_t*>(x)[i] - zp), scale);
    y[idx] = v;
  }
}

}  // namespace
}  // namespace mdlc

extern "C" int mdlc_nchw_to_nhwc(mdlc_ctx* ctx, const float* x, int n, int c, int h, int w, void* y, int cs,
                                 int dtype, float inv_scale, int zp) {
  if (!ctx) return MDLC_ERR_INVALID;
  const bool q = dtype == MDLC_U8 || dtype == MDLC_S8;
  if (!x || !y || n <= 0 || c <= 0 || h <= 0 || w <= 0 || cs < c || cs % (q ? 16 : 8))
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "nchw_to_nhwc: bad arguments");
  cudaSetDevice(ctx->device);
  const int hw = h * w;
  const long long total = (long long)n * hw * (cs / 8);
  const unsigned grid = grid_for(ctx, total);
  switch (dtype) {
    case MDLC_F32: to_nhwc_kernel<MDLC_F32><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, y, cs, inv_scale, zp, total); break;
    case MDLC_BF16: to_nhwc_kernel<MDLC_BF16><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, y, cs, inv_scale, zp, total); break;
    case MDLC_S8: to_nhwc_kernel<MDLC_S8><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, y, cs, inv_scale, zp, total); break;
    case MDLC_U8: to_nhwc_kernel<MDLC_U8><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, y, cs, inv_scale, zp, total); break;
    default: return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "nchw_to_nhwc: dtype %d", dtype);
  }
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "nchw_to_nhwc launch");
}

extern "C" int mdlc_nchw_to_s2d(mdlc_ctx* ctx, const float* x, int n, int c, int h, int w, void* y, int cs,
                                int dtype, float inv_scale, int zp) {
  if (!ctx) return MDLC_ERR_INVALID;
  const int align = (dtype == MDLC_U8 || dtype == MDLC_S8) ? 16 : 8;
  if (!x || !y || n <= 0 || c <= 0 || h <= 0 || w <= 0 || (h & 1) || (w & 1) || cs < 4 * c || cs % align)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "nchw_to_s2d: bad arguments");
  cudaSetDevice(ctx->device);
  const long long pixels = (long long)n * (h / 2) * (w / 2);
  if ((cs == 16 || cs == 32) && c <= 4 && pixels < (1LL << 31) && !(reinterpret_cast<uintptr_t>(x) & 7) &&
      !(reinterpret_cast<uintptr_t>(y) & 15)) {
    switch (dtype) {
      case MDLC_BF16: launch_s2d_stem<MDLC_BF16>(ctx, x, c, h, w, y, cs, inv_scale, zp, (int)pixels); break;
      case MDLC_F32: launch_s2d_stem<MDLC_F32>(ctx, x, c, h, w, y, cs, inv_scale, zp, (int)pixels); break;
      case MDLC_U8: launch_s2d_stem<MDLC_U8>(ctx, x, c, h, w, y, cs, inv_scale, zp, (int)pixels); break;
      case MDLC_S8: launch_s2d_stem<MDLC_S8>(ctx, x, c, h, w, y, cs, inv_scale, zp, (int)pixels); break;
      default: return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "nchw_to_s2d: dtype %d", dtype);
    }
    mdlc_note_launch(ctx);
    return mdlc_cuda_status(ctx, cudaGetLastError(), "nchw_to_s2d launch");
  }
  const long long total = pixels * (cs / 8);
  const unsigned grid = grid_for(ctx, total);
  switch (dtype) {
    case MDLC_BF16: to_s2d_kernel<MDLC_BF16><<<grid, 256, 0, ctx->stream>>>(x, c, h, w, y, cs, inv_scale, zp, total); break;
    case MDLC_F32: to_s2d_kernel<MDLC_F32><<<grid, 256, 0, ctx->stream>>>(x, c, h, w, y, cs, inv_scale, zp, total); break;
    case MDLC_U8: to_s2d_kernel<MDLC_U8><<<grid, 256, 0, ctx->stream>>>(x, c, h, w, y, cs, inv_scale, zp, total); break;
    case MDLC_S8: to_s2d_kernel<MDLC_S8><<<grid, 256, 0, ctx->stream>>>(x, c, h, w, y, cs, inv_scale, zp, total); break;
    default: return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "nchw_to_s2d: dtype %d", dtype);
  }
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "nchw_to_s2d launch");
}

extern "C" int mdlc_nhwc_to_nchw(mdlc_ctx* ctx, const void* x, int n, int c, int h, int w, int cs, int dtype,
                                 float* y, float scale, int zp) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!x || !y || n <= 0 || c <= 0 || h <= 0 || w <= 0 || cs < c)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "nhwc_to_nchw: bad arguments");
  cudaSetDevice(ctx->device);
  const int hw = h * w;
  const long long total = (long long)n * c * hw;
  const unsigned grid = grid_for(ctx, total);
  switch (dtype) {
    case MDLC_F32: to_nchw_kernel<MDLC_F32><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, cs, y, scale, zp, total); break;
    case MDLC_BF16: to_nchw_kernel<MDLC_BF16><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, cs, y, scale, zp, total); break;
    case MDLC_S8: to_nchw_kernel<MDLC_S8><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, cs, y, scale, zp, total); break;
    case MDLC_U8: to_nchw_kernel<MDLC_U8><<<grid, 256, 0, ctx->stream>>>(x, n, c, hw, cs, y, scale, zp, total); break;
    default: return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "nhwc_to_nchw: dtype %d", dtype);
  }
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "nhwc_to_nchw launch");
}
