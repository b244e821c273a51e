// Depthwise 3x3 convolution with the input halo staged in shared memory by TMA.
//
// Reference semantics: the grouped conv of mdlc/runtime/ops.py:68-78 with
// groups == C == K, which the reference GPU lowering runs on the host
// (mdlc/codegen/cuda/emit.py:175-180).
//
// HBM-bound (9 multiply-adds per output element against 2 bytes read and 2
// written in bf16), so the design is about keeping enough bytes in flight:
// persistent CTAs, two per SM, walk output tiles (16 x 16 pixels at stride 1,
// 8 x 8 at stride 2) x channel blocks of up to 128 bytes per pixel. One thread
// issues ONE tiled 4-D TMA load per tile for the tile's padded input window
// ((TH-1)*S+3 rows x (TW-1)*S+3 columns x the channel block); out-of-image
// pixels arrive as zeros, so padding costs nothing. Two shared-memory stages:
// the next tile's window loads while the current one is computed. Each thread
// owns one 8-channel vector of one output column and walks a run of output
// rows with a register ring of the three input rows it needs (one or two new
// rows per output row), weights and bias in registers, fp32 accumulation,
// fused bias + residual + activation, 16-byte stores.
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
  static constexpr int kWeights = 9 * 64 * 4;           // fp32 3x3 taps of one channel block
  static constexpr int kSmem = 2 * kStage + kWeights + 64 + 128;  // + barriers, alignment slack
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
  unsigned long long wait_cycles;
  ActParams act;
};

// 8 channels of one pixel, packed as in memory
template <typename T>
struct Px;
template <>
struct Px<__nv_bfloat16> {
  uint4 v;
  MDLC_DEV void lds(const uint8_t* p) { v = *reinterpret_cast<const uint4*>(p); }
  MDLC_DEV void fma(const float (&w)[8], float (&acc)[8]) const {
    acc[0] = fmaf(bf16_lo(v.x), w[0], acc[0]); acc[1] = fmaf(bf16_hi(v.x), w[1], acc[1]);
    acc[2] = fmaf(bf16_lo(v.y), w[2], acc[2]); acc[3] = fmaf(bf16_hi(v.y), w[3], acc[3]);
    acc[4] = fmaf(bf16_lo(v.z), w[4], acc[4]); acc[5] = fmaf(bf16_hi(v.z), w[5], acc[5]);
    acc[6] = fmaf(bf16_lo(v.w), w[6], acc[6]); acc[7] = fmaf(bf16_hi(v.w), w[7], acc[7]);
  }
};
template <>
struct Px<float> {
  float4 a, b;
  MDLC_DEV void lds(const uint8_t* p) {
    a = reinterpret_cast<const float4*>(p)[0];
    b = reinterpret_cast<const float4*>(p)[1];
  }
  MDLC_DEV void fma(const float (&w)[8], float (&acc)[8]) const {
    acc[0] = fmaf(a.x, w[0], acc[0]); acc[1] = fmaf(a.y, w[1], acc[1]);
    acc[2] = fmaf(a.z, w[2], acc[2]); acc[3] = fmaf(a.w, w[3], acc[3]);
    acc[4] = fmaf(b.x, w[4], acc[4]); acc[5] = fmaf(b.y, w[5], acc[5]);
    acc[6] = fmaf(b.z, w[6], acc[6]); acc[7] = fmaf(b.w, w[7], acc[7]);
  }
};

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
__global__ void __launch_bounds__(kDwThreads, 2)
    conv_dw3_tma_kernel(const __grid_constant__ CUtensorMap tmap, const DwTmaArgs a) {
  using Tl = DwTile<SH>;
  constexpr int TH = Tl::TH, TW = Tl::TW, IW = Tl::IW;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const uint32_t sbase = smem_u32(smem);
  float* sw = reinterpret_cast<float*>(smem + 2 * Tl::kStage);  // [9][cb_elems]
  const uint32_t bar0 = sbase + 2 * Tl::kStage + Tl::kWeights;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + 2 * Tl::kStage + Tl::kWeights + 16);
  const int tid = threadIdx.x;
  const int esz = (int)sizeof(T);
  const int cb_bytes = a.cb_elems * esz;
  const int per_img = a.tiles_x * a.tiles_y;
  const int per_cb = per_img * (a.total / (a.cblocks * per_img));  // tiles of one channel block
  auto issue = [&](int tile, int stage) {
    const int cb = tile / per_cb;
    int t = tile - cb * per_cb;
    const int img = t / per_img;
    t -= img * per_img;
    const int ty = t / a.tiles_x, tx = t - ty * a.tiles_x;
    const uint32_t bar = bar0 + 8u * stage;
    mbar_arrive_expect_tx(bar, (uint32_t)(Tl::IH * IW * cb_bytes));
    tma_load_4d(sbase + stage * Tl::kStage, &tmap, cb * a.cb_elems, tx * TW * SH - a.pl, ty * TH * SH - a.pt, img,
                bar);
  };
  if (tid == 0) {
    mbar_init(bar0, 1);
    mbar_init(bar0 + 8, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmap);
  }
  __syncthreads();
  if (tid == 0 && (int)blockIdx.x < a.total) issue(blockIdx.x, 0);

  // thread -> (8-channel vector, output column, run of output rows)
  const int V = a.vecs;
  const int groups = kDwThreads / (V * TW);           // row groups (>= 2 for V <= 8)
  const int rpt = (TH + groups - 1) / groups;         // output rows per thread
  const int v = tid % V, col = (tid / V) % TW, rg = tid / (V * TW);
  const bool active = rg < groups;
  const int oy0 = rg * rpt, oy1 = min(oy0 + rpt, TH);
  float bias[8];
  int cur_cb = -1;
  int i = 0;
  for (int tile = blockIdx.x; tile < a.total; tile += gridDim.x, ++i) {
    const int stage = i & 1;
    const int next = tile + gridDim.x;
    if (tid == 0 && next < a.total) {
      // the other stage was last read before the previous iteration's barrier
      fence_proxy_async_smem();
      issue(next, stage ^ 1);
    }
    const int cb = tile / per_cb;
    const bool new_cb = cb != cur_cb;  // block-uniform
    if (new_cb) {
      // this channel block's taps into shared memory (last read before the
      // previous iteration's barrier), and this thread's bias into registers
      for (int j = tid; j < 9 * a.cb_elems; j += kDwThreads) {
        const int tap = j / a.cb_elems;
        sw[j] = __ldg(a.w + tap * a.cs + cb * a.cb_elems + (j - tap * a.cb_elems));
      }
      const int cc = cb * a.cb_elems + v * 8;
      if (a.bias && active) {
        load8<float>(a.bias + cc, bias);
      } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) bias[e] = 0.0f;
      }
      cur_cb = cb;
    }
    const bool ok = mbar_wait(bar0 + 8u * stage, (i >> 1) & 1, abort_flag, a.err, a.wait_cycles);
    if (__syncthreads_or(!ok)) break;  // a timed-out wait ends every thread's loop together
    int t = tile - cb * per_cb;
    const int img = t / per_img;
    t -= img * per_img;
    const int ty = t / a.tiles_x, tx = t - ty * a.tiles_x;
    const int c0 = cb * a.cb_elems + v * 8;
    const float* wv = sw + v * 8;  // tap j of this vector at wv + j * cb_elems
    if (active && oy0 < oy1) {
      const uint8_t* st = smem + stage * Tl::kStage + v * 8 * esz;
      auto px_at = [&](int r, int c) { return st + (r * IW + c) * cb_bytes; };
      Px<T> p[3][3];
      const int c_in = col * SH;
#pragma unroll
      for (int r = 0; r < 3; ++r)
#pragma unroll
        for (int c = 0; c < 3; ++c) p[r][c].lds(px_at(oy0 * SH + r, c_in + c));
      const int gx = tx * TW + col;
      for (int oy = oy0; oy < oy1; ++oy) {
        float acc[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[e] = bias[e];
#pragma unroll
        for (int r = 0; r < 3; ++r)
#pragma unroll
          for (int c = 0; c < 3; ++c) {
            const float4 w0 = *reinterpret_cast<const float4*>(wv + (r * 3 + c) * a.cb_elems);
            const float4 w1 = *reinterpret_cast<const float4*>(wv + (r * 3 + c) * a.cb_elems + 4);
            const float wt[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
            p[r][c].fma(wt, acc);
          }
        const int gy = ty * TH + oy;
        if (gy < a.oh && gx < a.ow) {
          const long long m = ((long long)img * a.oh + gy) * a.ow + gx;
          if (a.res) {
            float rv[8];
            load8<T>(static_cast<const T*>(a.res) + m * a.res_s + c0, rv);
#pragma unroll
            for (int e = 0; e < 8; ++e) acc[e] += rv[e];
          }
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[e] = (c0 + e < a.c) ? apply_act(acc[e], a.act) : 0.0f;
          store8<T>(static_cast<T*>(a.y) + m * a.cs + c0, acc);
        }
        if (oy + 1 < oy1) {
          if (SH == 1) {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
              p[0][c] = p[1][c];
              p[1][c] = p[2][c];
              p[2][c].lds(px_at(oy + 3, c_in + c));
            }
          } else {
#pragma unroll
            for (int c = 0; c < 3; ++c) {
              p[0][c] = p[2][c];
              p[1][c].lds(px_at(oy * 2 + 3, c_in + c));
              p[2][c].lds(px_at(oy * 2 + 4, c_in + c));
            }
          }
        }
      }
    }
    __syncthreads();  // every thread is done with this stage before it is reloaded
  }
  // loads still in flight (the loop was left on a timed-out wait at iteration
  // i: that tile's load and the next one's) must land before the CTA's shared
  // memory is released; these waits are bounded too
  if (tid == 0 && *abort_flag) {
    for (int j = i; j <= i + 1; ++j)
      if ((int)blockIdx.x + j * (int)gridDim.x < a.total)
        mbar_wait(bar0 + 8u * (j & 1), (j >> 1) & 1, nullptr, a.err, 2000000ull);
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
  a.wait_cycles = 2 * kWaitLimitNs;
  a.act = epi ? ActParams{epi->act, epi->alpha, epi->beta, epi->clip_lo, epi->clip_hi}
              : ActParams{MDLC_ACT_NONE, 0.f, 0.f, -INFINITY, INFINITY};
  const long long slots = (long long)ctx->num_sms * 2;
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
