// Depthwise 3x3 convolution with the input halo staged in shared memory by TMA.
//
// Reference semantics: the grouped conv of mdlc/runtime/ops.py:68-78 with
// groups == C == K, which the reference GPU lowering runs on the host
// (mdlc/codegen/cuda/emit.py:175-180).
//
// HBM-bound (9 multiply-adds per output element against 2 bytes read and 2
// written in bf16), so the design is about keeping enough bytes in flight:
// persistent CTAs, one per SM, walk output tiles (16 x 16 pixels at stride 1,
// 8 x 8 at stride 2) x channel blocks of up to 128 bytes per pixel. One thread
// issues ONE tiled 4-D TMA load per tile for the tile's padded input window
// ((TH-1)*S+3 rows x (TW-1)*S+3 columns x the channel block); out-of-image
// pixels arrive as zeros, so padding costs nothing. Three shared-memory
// stages: two windows load while the current one is computed. Each thread
// owns one 8-channel vector of one output column and walks a run of output
// rows with a register ring of the three input rows it needs (one or two new
// rows per output row, unpacked to fp32 once), weights and bias in registers,
// paired fp32 multiply-adds (fma.rn.f32x2), fused bias + residual +
// activation, 16-byte stores.
#include "common.cuh"
#include "conv.h"

namespace mdlc {
namespace {

constexpr int kDwThreads = 256;
constexpr int kDwMaxBlockBytes = 128;  // channel block per pixel in shared memory

template <int SH>
struct DwTile {
  static constexpr int TH = SH == 1 ? 16 : 8;
  static constexpr int TW = SH == 1 ? 16 : 8;
  static constexpr int IH = (TH - 1) * SH + 3;  // input window rows
  static constexpr int IW = (TW - 1) * SH + 3;  // input window columns
  static constexpr int kStage = IH * IW * kDwMaxBlockBytes;
  static constexpr int kStages = 3;                     // input windows in flight per CTA
  static constexpr int kSmem = kStages * kStage + 64 + 128;  // + barriers, alignment slack
};

struct DwTmaArgs {
  const float* w;  // [9][cs] fp32
  const float* bias;
  const void* res;
  void* y;
  int* err;
  int cs, c, res_s, oh, ow, pt, pl;
  int cb_elems, vecs, cblocks;  // channel block (elements), 8-channel vectors in it, blocks per pixel
  int tiles_x, tiles_y, total;  // tiles per image row / column, total tiles
  long long y_elems, res_elems; // element extents (checked build)
  unsigned long long wait_cycles;
  ActParams act;
};

// Paired fp32 multiply-add (one fma.rn.f32x2: two IEEE fmas), on float2 kept
// in a 64-bit register pair.
MDLC_DEV void ffma2(float2& d, const float2 a, const float2 b) {
  unsigned long long dd = *reinterpret_cast<unsigned long long*>(&d);
  asm("fma.rn.f32x2 %0, %1, %2, %0;"
      : "+l"(dd)
      : "l"(*reinterpret_cast<const unsigned long long*>(&a)), "l"(*reinterpret_cast<const unsigned long long*>(&b)));
  d = *reinterpret_cast<float2*>(&dd);
}

// 8 channels of one pixel from shared memory, as four fp32 pairs
template <typename T>
MDLC_DEV void lds8(const uint8_t* p, float2 (&f)[4]);
template <>
MDLC_DEV void lds8<__nv_bfloat16>(const uint8_t* p, float2 (&f)[4]) {
  const uint4 v = *reinterpret_cast<const uint4*>(p);
  f[0] = make_float2(bf16_lo(v.x), bf16_hi(v.x));
  f[1] = make_float2(bf16_lo(v.y), bf16_hi(v.y));
  f[2] = make_float2(bf16_lo(v.z), bf16_hi(v.z));
  f[3] = make_float2(bf16_lo(v.w), bf16_hi(v.w));
}
template <>
MDLC_DEV void lds8<float>(const uint8_t* p, float2 (&f)[4]) {
  const float4 a = reinterpret_cast<const float4*>(p)[0], b = reinterpret_cast<const float4*>(p)[1];
  f[0] = make_float2(a.x, a.y); f[1] = make_float2(a.z, a.w);
  f[2] = make_float2(b.x, b.y); f[3] = make_float2(b.z, b.w);
}

template <typename T>
MDLC_DEV void load8(const T* p, float (&f)[8]);
template <>
MDLC_DEV void load8<__nv_bfloat16>(const __nv_bfloat16* p, float (&f)[8]) {
  const uint4 u = __ldg(reinterpret_cast<const uint4*>(p));
  f[0] = bf16_lo(u.x); f[1] = bf16_hi(u.x); f[2] = bf16_lo(u.y); f[3] = bf16_hi(u.y);
  f[4] = bf16_lo(u.z); f[5] = bf16_hi(u.z); f[6] = bf16_lo(u.w); f[7] = bf16_hi(u.w);
}
template <>
MDLC_DEV void load8<float>(const float* p, float (&f)[8]) {
  const float4 a = __ldg(reinterpret_cast<const float4*>(p)), b = __ldg(reinterpret_cast<const float4*>(p) + 1);
  f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
}
template <typename T>
MDLC_DEV void store8(T* p, const float (&f)[8]);
template <>
MDLC_DEV void store8<__nv_bfloat16>(__nv_bfloat16* p, const float (&f)[8]) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f[0], f[1]), pack_bf16x2(f[2], f[3]),
                                            pack_bf16x2(f[4], f[5]), pack_bf16x2(f[6], f[7]));
}
template <>
MDLC_DEV void store8<float>(float* p, const float (&f)[8]) {
  reinterpret_cast<float4*>(p)[0] = make_float4(f[0], f[1], f[2], f[3]);
  reinterpret_cast<float4*>(p)[1] = make_float4(f[4], f[5], f[6], f[7]);
}

template <typename T, int SH>
__global__ void __launch_bounds__(kDwThreads, 1)
    conv_dw3_tma_kernel(const __grid_constant__ CUtensorMap tmap, const DwTmaArgs a) {
  using Tl = DwTile<SH>;
  constexpr int TH = Tl::TH, TW = Tl::TW, IW = Tl::IW, NS = Tl::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bar0 = sbase + NS * Tl::kStage;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + NS * Tl::kStage + 8 * NS + 8);
  const int tid = threadIdx.x;
  const int esz = (int)sizeof(T);
  const int cb_bytes = a.cb_elems * esz;
  const int per_img = a.tiles_x * a.tiles_y;
  const int per_cb = a.total / a.cblocks;  // tiles of one channel block
  auto decode = [&](int tile, int& cb, int& img, int& ty, int& tx) {
    cb = tile / per_cb;
    int t = tile - cb * per_cb;
    img = t / per_img;
    t -= img * per_img;
    ty = t / a.tiles_x;
    tx = t - ty * a.tiles_x;
  };
  auto issue = [&](int tile, int stage) {
    int cb, img, ty, tx;
    decode(tile, cb, img, ty, tx);
    const uint32_t bar = bar0 + 8u * stage;
    mbar_arrive_expect_tx(bar, (uint32_t)(Tl::IH * IW * cb_bytes));
    tma_load_4d(sbase + stage * Tl::kStage, &tmap, cb * a.cb_elems, tx * TW * SH - a.pl, ty * TH * SH - a.pt, img,
                bar);
  };
  if (tid == 0) {
    for (int q = 0; q < NS; ++q) mbar_init(bar0 + 8u * q, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap);
  }
  __syncthreads();
  // the first NS - 1 windows of this CTA
  if (tid == 0)
    for (int q = 0; q < NS - 1; ++q)
      if ((int)blockIdx.x + q * (int)gridDim.x < a.total) issue(blockIdx.x + q * gridDim.x, q);

  // thread -> (8-channel vector, output column, run of output rows)
  const int V = a.vecs;
  const int groups = kDwThreads / (V * TW);           // row groups (>= 2 for V <= 8)
  const int rpt = (TH + groups - 1) / groups;         // output rows per thread
  const int v = tid % V, col = (tid / V) % TW, rg = tid / (V * TW);
  const bool active = rg < groups;
  const int oy0 = rg * rpt, oy1 = min(oy0 + rpt, TH);
  float2 w[9][4], bias[4];
  int cur_cb = -1;
  int i = 0;
  for (int tile = blockIdx.x; tile < a.total; tile += gridDim.x, ++i) {
    const int stage = i % NS;
    const int ahead = tile + (NS - 1) * gridDim.x;
    if (tid == 0 && ahead < a.total) {
      // that stage was last read in iteration i - 1, before its closing barrier
      fence_proxy_async_smem();
      issue(ahead, (i + NS - 1) % NS);
    }
    const bool ok = mbar_wait(bar0 + 8u * stage, (i / NS) & 1, abort_flag, a.err, a.wait_cycles);
    if (__syncthreads_or(!ok)) break;  // a timed-out wait ends every thread's loop together
    int cb, img, ty, tx;
    decode(tile, cb, img, ty, tx);
    const int c0 = cb * a.cb_elems + v * 8;
    if (active && oy0 < oy1) {
      if (cb != cur_cb) {
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const float4 w0 = __ldg(reinterpret_cast<const float4*>(a.w + tap * a.cs + c0));
          const float4 w1 = __ldg(reinterpret_cast<const float4*>(a.w + tap * a.cs + c0) + 1);
          w[tap][0] = make_float2(w0.x, w0.y); w[tap][1] = make_float2(w0.z, w0.w);
          w[tap][2] = make_float2(w1.x, w1.y); w[tap][3] = make_float2(w1.z, w1.w);
        }
        if (a.bias) {
          const float4 b0 = __ldg(reinterpret_cast<const float4*>(a.bias + c0));
          const float4 b1 = __ldg(reinterpret_cast<const float4*>(a.bias + c0) + 1);
          bias[0] = make_float2(b0.x, b0.y); bias[1] = make_float2(b0.z, b0.w);
          bias[2] = make_float2(b1.x, b1.y); bias[3] = make_float2(b1.z, b1.w);
        } else {
#pragma unroll
          for (int e = 0; e < 4; ++e) bias[e] = make_float2(0.0f, 0.0f);
        }
        cur_cb = cb;
      }
      const uint8_t* st = smem + stage * Tl::kStage + v * 8 * esz;
      auto px_at = [&](int r, int c) { return st + (r * IW + c) * cb_bytes; };
      float2 p[3][3][4];  // the three input rows of the current output row, unpacked
      const int c_in = col * SH;
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int c = 0; c < 3; ++c) lds8<T>(px_at(oy0 * SH + r, c_in + c), p[r][c]);
      const int gx = tx * TW + col;
      for (int oy = oy0; oy < oy1; ++oy) {
        float2 acc[4] = {bias[0], bias[1], bias[2], bias[3]};
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int c = 0; c < 3; ++c)
#pragma unroll
            for (int e = 0; e < 4; ++e) ffma2(acc[e], p[r][c][e], w[r * 3 + c][e]);
        const int gy = ty * TH + oy;
        const long long m = ((long long)img * a.oh + gy) * a.ow + gx;
        if (gy < a.oh && gx < a.ow && MDLC_CHECK_IDX(a.err, m * a.cs + c0 + 7, a.y_elems) &&
            (!a.res || MDLC_CHECK_IDX(a.err, m * a.res_s + c0 + 7, a.res_elems))) {
          float f[8] = {acc[0].x, acc[0].y, acc[1].x, acc[1].y, acc[2].x, acc[2].y, acc[3].x, acc[3].y};
          if (a.res) {
            float rv[8];
            load8<T>(static_cast<const T*>(a.res) + m * a.res_s + c0, rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) f[e] += rv[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) f[e] = (c0 + e < a.c) ? apply_act(f[e], a.act) : 0.0f;
          store8<T>(static_cast<T*>(a.y) + m * a.cs + c0, f);
        }
        if (oy + 1 < oy1) {
          if (SH == 1) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                p[0][c][e] = p[1][c][e];
                p[1][c][e] = p[2][c][e];
              }
              lds8<T>(px_at(oy + 3, c_in + c), p[2][c]);
            }
          } else {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
#pragma unroll
              for (int e = 0; e < 4; ++e) p[0][c][e] = p[2][c][e];
              lds8<T>(px_at(oy * 2 + 3, c_in + c), p[1][c]);
              lds8<T>(px_at(oy * 2 + 4, c_in + c), p[2][c]);
            }
          }
        }
      }
    }
    __syncthreads();  // every thread is done with this stage before it is reloaded
  }
  // loads still in flight (the loop was left on a timed-out wait at iteration
  // i: that window's load and the NS - 2 after it) must land before the CTA's
  // shared memory is released; these waits are bounded too
  if (tid == 0 && *abort_flag) {
    for (int j = i; j < i + NS - 1 + 1; ++j)
      if ((int)blockIdx.x + j * (int)gridDim.x < a.total)
        mbar_wait(bar0 + 8u * (j % NS), (j / NS) & 1, nullptr, a.err, 2000000ull);
  }
}

}  // namespace
}  // namespace mdlc

namespace mdlc {

int conv_dw_tma(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
                const void* res, void* y, const mdlc_epilogue* epi) {
  if (d.r != 3 || d.s != 3 || d.dil_h != 1 || d.dil_w != 1 || d.stride_h != d.stride_w ||
      (d.stride_h != 1 && d.stride_h != 2))
    return MDLC_ERR_UNSUPPORTED;
  const bool bf = d.in_type == MDLC_BF16;
  const int esz = bf ? 2 : 4;
  // channel block: the largest multiple of 8 channels of at most 128 bytes dividing the stride
  int cb = 0;
  for (int c = kDwMaxBlockBytes / esz; c >= 8; c -= 8)
    if (d.c_stride % c == 0) {
      cb = c;
      break;
    }
  auto encode = tensor_map_encoder();
  if (!cb || !encode) return MDLC_ERR_UNSUPPORTED;
  const int SH = d.stride_h;
  const int TH = SH == 1 ? DwTile<1>::TH : DwTile<2>::TH, TW = SH == 1 ? DwTile<1>::TW : DwTile<2>::TW;
  const int IH = SH == 1 ? DwTile<1>::IH : DwTile<2>::IH, IW = SH == 1 ? DwTile<1>::IW : DwTile<2>::IW;
  const long long tiles_x = (d.ow + TW - 1) / TW, tiles_y = (d.oh + TH - 1) / TH;
  const long long total = (long long)(d.c_stride / cb) * d.n * tiles_x * tiles_y;
  if (total >= (1ll << 31)) return MDLC_ERR_UNSUPPORTED;
  CUtensorMap tmap;
  const cuuint64_t gd[4] = {(cuuint64_t)d.c_stride, (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
  const cuuint64_t gs[3] = {(cuuint64_t)d.c_stride * esz, (cuuint64_t)d.w * d.c_stride * esz,
                            (cuuint64_t)d.h * d.w * d.c_stride * esz};
  const cuuint32_t box[4] = {(cuuint32_t)cb, (cuuint32_t)IW, (cuuint32_t)IH, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  if (encode(&tmap, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(x),
             gd, gs, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return MDLC_ERR_UNSUPPORTED;
  DwTmaArgs a{};
  a.w = w; a.bias = bias; a.res = res; a.y = y; a.err = ctx->d_err;
  a.cs = d.c_stride; a.c = d.c; a.res_s = d.res_stride ? d.res_stride : d.c_stride;
  a.oh = d.oh; a.ow = d.ow; a.pt = d.pad_t; a.pl = d.pad_l;
  a.cb_elems = cb; a.vecs = cb / 8; a.cblocks = d.c_stride / cb;
  a.tiles_x = (int)tiles_x; a.tiles_y = (int)tiles_y; a.total = (int)total;
  a.y_elems = (long long)d.n * d.oh * d.ow * d.c_stride;
  a.res_elems = (long long)d.n * d.oh * d.ow * a.res_s;
  a.wait_cycles = 2 * kWaitLimitNs;
  a.act = epi ? ActParams{epi->act, epi->alpha, epi->beta, epi->clip_lo, epi->clip_hi}
              : ActParams{MDLC_ACT_NONE, 0.f, 0.f, -INFINITY, INFINITY};
  const long long slots = (long long)ctx->num_sms;  // one CTA per SM (register budget)
  const unsigned grid = (unsigned)(total < slots ? total : slots);
  void (*kern)(const CUtensorMap, const DwTmaArgs);
  int smem;
  if (SH == 1) {
    kern = bf ? conv_dw3_tma_kernel<__nv_bfloat16, 1> : conv_dw3_tma_kernel<float, 1>;
    smem = DwTile<1>::kSmem;
  } else {
    kern = bf ? conv_dw3_tma_kernel<__nv_bfloat16, 2> : conv_dw3_tma_kernel<float, 2>;
    smem = DwTile<2>::kSmem;
  }
  static bool attr_set[64][4] = {};
  const int which = (SH - 1) * 2 + (bf ? 1 : 0);
  if (!attr_set[ctx->device & 63][which]) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "conv_dw3_tma smem attribute");
    attr_set[ctx->device & 63][which] = true;
  }
  kern<<<grid, kDwThreads, smem, ctx->stream>>>(tmap, a);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, cudaGetLastError(), "conv_dw3_tma launch");
}

}  // namespace mdlc
