// Host side of the tcgen05 implicit-GEMM convolution (kernel: conv_tc_kernel.cuh):
// tile-configuration choice, A-operand mode, tensor maps (weights, im2col /
// pointwise / halo input, TMA-stored output and residual), split-K set-up,
// then the launcher of the element type's translation unit.
#include <cudaTypedefs.h>

#include <cmath>
#include <cstring>
#include <mutex>

#include "conv_tc_kernel.cuh"

namespace mdlc {
namespace {

// ---------------------------------------------------------------- host side
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

PFN_cuTensorMapEncodeIm2col_v12000 get_im2col_fn() {
  static PFN_cuTensorMapEncodeIm2col_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeIm2col", &p, 12000, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeIm2col_v12000>(p);
  });
  return fn;
}

// im2col-mode tensor map over the NHWC input: 128 output pixels x one
// 128-byte channel block per load. The pixel box corners follow from the
// padding and the output extent: lower = -pad, upper = pad_end - (R-1)*dil
// with pad_end chosen so the traversal yields exactly oh x ow positions.
// Returns false when the layer does not fit the hardware's limits (channel
// stride not a multiple of the block, corners outside [-128, 127], traversal
// stride above 8, offsets of 128 or more) or is small (< 128 KiB), in which
// case the kernel gathers A with cp.async instead.
// v as a bf16 pair (both halves) when v is exactly representable in bf16
bool bf16_pair_exact(float v, uint32_t* pair) {
  uint32_t u;
  memcpy(&u, &v, 4);
  if ((u & 0xFFFFu) != 0 || v != v) return false;
  *pair = (u >> 16) | (u & 0xFFFF0000u);
  return true;
}

int encode_im2col(CUtensorMap* m, const mdlc_conv_desc& d, const void* x, int esz) {
  const int kb_elems = 128 / esz;
  // mode 1: 128-byte channel blocks; modes 2/3: the whole pixel (bf16 cs 16 / 32) per load
  int mode = 0, cpp = kb_elems;
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const int pixel_bytes = d.c_stride * esz;
  if (d.c_stride % kb_elems == 0) {
    mode = 1;
  } else if (pixel_bytes == 32) {
    mode = 2, cpp = d.c_stride, sw = CU_TENSOR_MAP_SWIZZLE_32B;
  } else if (pixel_bytes == 64) {
    mode = 3, cpp = d.c_stride, sw = CU_TENSOR_MAP_SWIZZLE_64B;
  } else {
    return 0;
  }
  if (d.stride_h > 8 || d.stride_w > 8) return 0;
  if ((d.r - 1) * d.dil_h >= 128 || (d.s - 1) * d.dil_w >= 128) return 0;
  const long long bytes = (long long)d.n * d.h * d.w * d.c_stride * esz;
  if (bytes < 131072) return 0;
  const int lower_w = -d.pad_l, lower_h = -d.pad_t;
  const int upper_w = (d.ow - 1) * d.stride_w + 1 - d.w - d.pad_l;
  const int upper_h = (d.oh - 1) * d.stride_h + 1 - d.h - d.pad_t;
  for (int v : {lower_w, lower_h, upper_w, upper_h})
    if (v < -128 || v > 127) return 0;
  auto fn = get_im2col_fn();
  if (!fn) return 0;
  const cuuint64_t gdim[4] = {(cuuint64_t)d.c_stride, (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
  const cuuint64_t gstride[3] = {(cuuint64_t)d.c_stride * esz, (cuuint64_t)d.w * d.c_stride * esz,
                                 (cuuint64_t)d.h * d.w * d.c_stride * esz};
  const int lower[2] = {lower_w, lower_h};
  const int upper[2] = {upper_w, upper_h};
  const cuuint32_t estride[4] = {1, (cuuint32_t)d.stride_w, (cuuint32_t)d.stride_h, 1};
  const bool ok = fn(m, esz == 2 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                 : (esz == 4 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_UINT8), 4,
                     const_cast<void*>(x), gdim, gstride, lower, upper, (cuuint32_t)cpp, (cuuint32_t)kBM, estride,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
  return ok ? mode : 0;
}

}  // namespace

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() { return get_encode_fn(); }

int conv_tc(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const void* w, const void* bias,
            const void* res, void* y, const mdlc_epilogue* epi, const mdlc_tile_cfg* cfg) {
  const bool int8 = d.in_type == MDLC_U8 || d.in_type == MDLC_S8;
  const bool fp32 = d.in_type == MDLC_F32;  // 3xTF32 on kind::tf32
  const int esz = int8 ? 1 : (fp32 ? 4 : 2);
  const int kb_elems = 128 / esz;
  const long long kg = (long long)d.r * d.s * d.c_stride;
  const int num_kb = (int)((kg + kb_elems - 1) / kb_elems);
  const long long M = (long long)d.n * d.oh * d.ow;
  if (M <= 0 || M > (1ll << 31) - 256) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: bad M=%lld", M);

  // halo mode (AMODE 4): stride-1 convs with a TMA-stored output on images
  // large enough that 16x8 tiles waste little, on request (flags bit 2): it
  // moves fewer bytes, but the per-tap loads are not what bounds these layers
  // on this part (single-CTA MMA rate and TMA issue rate are), so the per-tap
  // modes are the default.
  const bool out8 = d.out_type == MDLC_U8 || d.out_type == MDLC_S8;
  const bool out_tma = (!int8 && d.out_type == MDLC_BF16) || (int8 && out8);
  const int pixel_bytes = d.c_stride * esz;
  const int band_px = pixel_bytes % 128 == 0 ? 128 : (pixel_bytes == 32 || pixel_bytes == 64 ? pixel_bytes : 0);
  const bool halo_shape = out_tma && band_px && d.stride_h == 1 && d.stride_w == 1 && d.dil_h == 1 &&
                          d.dil_w == 1 && d.r * d.s > 1 && d.r <= kHaloMaxR && d.s <= kHaloSlots - kHaloTW + 1 &&
                          d.oh >= 14 && d.ow >= 14 && (!int8 || d.in_zp == 0) && !(cfg && (cfg->flags & 3)) &&
                          !fp32;
  // resident weights (flags bit 3): bf16 halo layers with 128-byte channel
  // blocks whose whole packed weight matrix -- at most 64 output channels and
  // kResidentKb k-blocks (64 -> 64 3x3: 72 KB) -- stays in shared memory, one
  // CTA per SM, no split-K
  const bool resident = halo_shape && cfg && (cfg->flags & 8) && esz == 2 && band_px == 128 &&
                        d.k_stride <= 64 && num_kb <= kResidentKb && ((cfg->flags >> 8) & 0xFF) <= 1;
  const bool halo = halo_shape && cfg && ((cfg->flags & 4) || resident);
  const int tiles_x = (d.ow + kHaloTW - 1) / kHaloTW, tiles_y = (d.oh + kHaloTH - 1) / kHaloTH;

  int bn = cfg && cfg->bn ? cfg->bn : 0;
  int stages = cfg && cfg->stages ? cfg->stages : 0;
  if (resident) {
    bn = 64;
    stages = kResidentKb;
  }
  const long long num_m_ll = halo ? (long long)d.n * tiles_x * tiles_y : (M + kBM - 1) / kBM;
  if (num_m_ll > (1ll << 30)) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv: too many tiles");
  const int num_m = (int)num_m_ll;
  if (!bn && fp32) {
    // fp32 tiles: 64, 128 or 256 wide (shared memory holds hi and lo stages)
    bn = d.k_stride > 128 ? 256 : (d.k_stride > 64 ? 128 : 64);
    while (bn > 64 && (long long)num_m * ((d.k_stride + bn - 1) / bn) < ctx->num_sms) bn /= 2;
  }
  if (!bn) {
    bn = d.k_stride > 128 ? 256 : (d.k_stride > 64 ? 128 : 64);
    // keep enough tiles in flight for the whole GPU
    while (bn > 64 && (long long)num_m * ((d.k_stride + bn - 1) / bn) < ctx->num_sms) bn /= 2;
    if (bn == 256) {
      // 192-wide tiles when they fill the last wave better: compare the
      // busiest SM's output columns, ceil(tiles / SMs) x tile width
      auto busiest = [&](int w) {
        const long long tiles = (long long)num_m * ((d.k_stride + w - 1) / w);
        return (tiles + ctx->num_sms - 1) / ctx->num_sms * w;
      };
      if (busiest(192) < busiest(256)) bn = 192;
    }
  }
  // 64- and 128-wide tiles: the two-CTAs-per-SM configurations (see Occ)
  // when every SM gets more than one tile; otherwise each CTA runs alone on
  // its SM and the deep single-CTA pipelines are faster
  // fp32 ring depth left to the library: settled below, once the A mode is
  // known (the deeper rings are built for the TMA modes of 128-byte blocks)
  const bool f32_auto_stages = fp32 && !stages;
  if (!stages && fp32) stages = bn == 64 ? 3 : 2;
  if (!stages) {
    const long long tiles = (long long)num_m * ((d.k_stride + bn - 1) / bn);
    const bool pair = tiles > ctx->num_sms;
    stages = bn >= 192 ? 3 : (bn == 128 ? (pair ? 2 : 4) : (pair ? 3 : 8));
  }
  if (fp32 && !((bn == 64 && (stages == 3 || stages == 4)) || (bn == 128 && (stages == 2 || stages == 3)) ||
                 (bn == 256 && stages == 2)))
    return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED,
                          "conv_tc fp32: tile configurations (64, 3), (64, 4), (128, 2), (128, 3), (256, 2) only, "
                          "got (%d, %d)", bn, stages);
  if (bn != 64 && bn != 128 && bn != 192 && bn != 256)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "conv_tc: bn must be 64/128/192/256, got %d", bn);

  auto encode = get_encode_fn();
  if (!encode) return mdlc_set_error(ctx, MDLC_ERR_CUDA, "cuTensorMapEncodeTiled unavailable");
  CUtensorMap tmap;
  const cuuint64_t gdim[3] = {(cuuint64_t)num_kb * kb_elems, (cuuint64_t)d.k, 2};
  const cuuint64_t gstride[2] = {(cuuint64_t)num_kb * 128, (cuuint64_t)num_kb * 128 * d.k};
  const cuuint32_t box[3] = {(cuuint32_t)kb_elems, (cuuint32_t)bn, 2};
  const cuuint32_t estride[3] = {1, 1, 1};
  // fp32: the packed weights are the tf32 hi matrix then the lo matrix ([2][k][k_pad]);
  // one 3-D box brings a k-block of both, hi tile then lo tile
  const auto wdt = int8 ? CU_TENSOR_MAP_DATA_TYPE_UINT8
                        : (fp32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16);
  CUresult cr = encode(&tmap, wdt, fp32 ? 3 : 2, const_cast<void*>(w), gdim, gstride, box, estride,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (cr != CUDA_SUCCESS) return mdlc_set_error(ctx, MDLC_ERR_INVALID, "weight tensor map: CUresult %d", (int)cr);

  TcArgs a{};
  a.x = static_cast<const uint8_t*>(x);
  a.y = y;
  a.bias = bias;
  a.res = static_cast<const uint8_t*>(res);
  a.pad_src = nullptr;
  a.err = ctx->d_err;
  a.n = d.n; a.h = d.h; a.w = d.w; a.cs = d.c_stride;
  a.k = d.k; a.ks = d.k_stride; a.res_s = d.res_stride ? d.res_stride : d.k_stride;
  a.r = d.r; a.s = d.s; a.sh = d.stride_h; a.sw = d.stride_w; a.pt = d.pad_t; a.pl = d.pad_l;
  a.dh = d.dil_h; a.dw = d.dil_w; a.oh = d.oh; a.ow = d.ow;
  a.M = (int)M;
  a.x_elems = (long long)d.n * d.h * d.w * d.c_stride;
  a.y_elems = M * d.k_stride;
  a.res_elems = M * (d.res_stride ? d.res_stride : d.k_stride);
  a.num_kb = num_kb;
  a.num_m_tiles = num_m;
  a.tiles_x = tiles_x; a.tiles_y = tiles_y;
  a.halo_rows = kHaloTH + d.r - 1;
  a.band_px = band_px;
  a.cpb = band_px == 128 ? pixel_bytes / 128 : 1;
  a.b_resident = resident ? 1 : 0;
  a.num_n_tiles = (d.k_stride + bn - 1) / bn;
  a.out_type = d.out_type;
  a.a_signed = d.in_type == MDLC_S8;
  a.wait_cycles = 2 * kWaitLimitNs;  // cycles: >= the nanosecond limit at clocks up to 2 GHz
  if (epi) {
    a.act = ActParams{epi->act, epi->alpha, epi->beta, epi->clip_lo, epi->clip_hi};
    a.rq_scale = epi->rq_scale;
    a.out_zp = epi->out_zp; a.qlo = epi->qmin - epi->out_zp; a.qhi = epi->qmax - epi->out_zp;
    a.res_zp = epi->res_zp; a.res_scale = epi->res_scale; a.res_signed = epi->res_signed;
    a.deq_scale = epi->deq_scale; a.deq_bias = epi->deq_bias;
    a.rq_mult = epi->rq_mult; a.rq_res_mult = epi->rq_res_mult; a.rq_shift = epi->rq_shift;
    a.rq_fixed = epi->rq_mult != nullptr;
  }
  if (int8) a.pad_src = ctx->d_pad + 16 * (d.in_zp & 0xFF);

  // A operand: im2col-mode TMA when the layer qualifies (zero padding only, so
  // not for int8 inputs with a non-zero zero point), else the cp.async gather
  CUtensorMap tmap_x = tmap;
  const auto dt = wdt;
  int amode = 0;
  if (halo) {
    // the input band of a tile: one channel block (band_px bytes) x kHaloSlots
    // pixels x halo_rows rows of one image, swizzled at band_px bytes;
    // out-of-image pixels read 0
    const cuuint64_t gd[4] = {(cuuint64_t)d.c_stride, (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
    const cuuint64_t gs[3] = {(cuuint64_t)d.c_stride * esz, (cuuint64_t)d.w * d.c_stride * esz,
                              (cuuint64_t)d.h * d.w * d.c_stride * esz};
    const cuuint32_t bx[4] = {(cuuint32_t)(band_px / esz), (cuuint32_t)kHaloSlots, (cuuint32_t)a.halo_rows, 1};
    const cuuint32_t es4[4] = {1, 1, 1, 1};
    const auto bsw = band_px == 32 ? CU_TENSOR_MAP_SWIZZLE_32B
                                   : (band_px == 64 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B);
    if (encode(&tmap_x, dt, 4, const_cast<void*>(x), gd, gs, bx, es4, CU_TENSOR_MAP_INTERLEAVE_NONE, bsw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "halo input tensor map encode failed");
    amode = 4;
  } else if (d.r == 1 && d.s == 1 && d.stride_h == 1 && d.stride_w == 1 && d.pad_t == 0 && d.pad_l == 0 &&
             d.oh == d.h && d.ow == d.w && !(cfg && (cfg->flags & 1))) {
    // pointwise conv / GEMM: A is the [M, cs] activation matrix; a 2-D tiled
    // load fetches each 128-row x 128-byte k-block (channels past cs read 0,
    // and no padding exists, so any input zero point is exact)
    const cuuint64_t gd[2] = {(cuuint64_t)d.c_stride, (cuuint64_t)M};
    const cuuint64_t gs[1] = {(cuuint64_t)d.c_stride * esz};
    const cuuint32_t bx[2] = {(cuuint32_t)kb_elems, (cuuint32_t)kBM};
    if (encode(&tmap_x, dt, 2, const_cast<void*>(x), gd, gs, bx, estride, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "pointwise input tensor map encode failed");
    amode = 5;
  } else if ((!int8 || d.in_zp == 0) && !(cfg && (cfg->flags & 1))) {
    amode = encode_im2col(&tmap_x, d, x, esz);
  }
  // fp32 layers fed by TMA in 128-byte channel blocks: the deeper rings (64, 4)
  // and (128, 3) (measured on ResNet-18 b=256: 3x3 layers 6-23% faster than
  // (64, 3) / (128, 2), the paired stem 1375 -> 1353 us)
  if (f32_auto_stages && (amode == 1 || amode == 5) && bn <= 128) stages = bn == 64 ? 4 : 3;

  // split-K on request (flags bits 8-15 = number of K slices): the tile's
  // reduction is cut into slices run by different CTAs, each writing its raw
  // accumulators to the context's workspace, and the tile's last slice to
  // finish sums them in slice order (deterministic; exact for int8) and runs
  // the epilogue. Measured on ResNet-18 at b=1 it shortened the 512-channel
  // 7x7 layers (43 -> 35 us) but not the forward, so no layer splits by
  // default. Not in halo mode.
  a.split = 1;
  a.kps = num_kb;
  // fp32: promote the accumulator every 4 k-blocks (128 reduction elements)
  // when the reduction is deeper than 1152: the truncation error of the
  // tensor cores' accumulation grows like K^1.5, and at K <= 1152 it stays
  // near the fp32 rounding error of the sum itself
  a.kchunk = (esz == 4 && num_kb > 36) ? 4 : 0;
  a.ws = ctx->d_split_ws;
  a.counters = ctx->d_split_cnt;
  if (cfg && ((cfg->flags >> 8) & 0xFF) > 1) {
    const long long tiles = (long long)a.num_m_tiles * a.num_n_tiles;
    int s = (cfg->flags >> 8) & 0xFF;
    if (s > num_kb) s = num_kb;
    if (amode == 4) return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "conv_tc: split-K is not built for halo mode");
    a.kps = (num_kb + s - 1) / s;
    a.split = (num_kb + a.kps - 1) / a.kps;  // no empty slice
    if ((size_t)tiles * a.split * kBM * bn * 4 > kSplitWsBytes || tiles > kSplitCounters)
      return mdlc_set_error(ctx, MDLC_ERR_INVALID,
                            "conv_tc: split-K needs %lld tiles x %d slices of %d x %d accumulators, over the "
                            "%zu-byte workspace", tiles, a.split, kBM, bn, kSplitWsBytes);
    // The kernel leaves every counter at zero, except on a call whose CTAs gave
    // up on a bounded wait: that tile's counter keeps its partial count, and
    // the next split-K call would take a tile's last slice for early. So the
    // counters this launch uses are cleared on the stream first.
    if (a.split > 1) {
      const cudaError_t e = cudaMemsetAsync(a.counters, 0, (size_t)tiles * sizeof(int), ctx->stream);
      if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "conv_tc: clearing split-K counters");
    }
  }

  // bf16 / 8-bit output: the epilogue stages 32x64 tiles in shared memory and
  // writes them with TMA stores; a residual is brought in by TMA loads of the
  // same tile shape. Boxes hanging over the tensor are clipped by TMA.
  CUtensorMap tmap_y = tmap, tmap_r = tmap;
  if (out_tma) {
    // 32 rows x 64 columns: 128-byte rows with 128-byte swizzle (bf16), 64-byte
    // rows with 64-byte swizzle (8-bit). Halo mode addresses the same 32 rows
    // as 4 output rows x 8 columns of one image (4-D box).
    const auto swz = int8 ? CU_TENSOR_MAP_SWIZZLE_64B : CU_TENSOR_MAP_SWIZZLE_128B;
    auto encode_out = [&](CUtensorMap* m, const void* base, int inner) {
      if (amode == 4) {
        const cuuint64_t gd[4] = {(cuuint64_t)inner, (cuuint64_t)d.ow, (cuuint64_t)d.oh, (cuuint64_t)d.n};
        const cuuint64_t gs[3] = {(cuuint64_t)inner * esz, (cuuint64_t)d.ow * inner * esz,
                                  (cuuint64_t)d.oh * d.ow * inner * esz};
        const cuuint32_t bx[4] = {64, (cuuint32_t)kHaloTW, (cuuint32_t)(32 / kHaloTW), 1};
        const cuuint32_t es4[4] = {1, 1, 1, 1};
        return encode(m, dt, 4, const_cast<void*>(base), gd, gs, bx, es4, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
      }
      const cuuint64_t gd[2] = {(cuuint64_t)inner, (cuuint64_t)M};
      const cuuint64_t gs[1] = {(cuuint64_t)inner * esz};
      const cuuint32_t bx[2] = {64, 32};
      return encode(m, dt, 2, const_cast<void*>(base), gd, gs, bx, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    };
    if (encode_out(&tmap_y, y, d.k_stride) != CUDA_SUCCESS ||
        (res && encode_out(&tmap_r, res, a.res_s) != CUDA_SUCCESS))
      return mdlc_set_error(ctx, MDLC_ERR_INVALID, "output/residual tensor map encode failed");
    a.tma_epi = 1;
  }

// Activation specialisations of the bf16 TMA epilogue: none, ReLU, Clip
// (ReLU6), GELU, sigmoid; anything else (and the int8 / fp32-output paths)
// uses the run-time switch.
  const int act = a.act.act;
  const int act_t = (!int8 && !fp32 && a.tma_epi &&
                     (act == MDLC_ACT_NONE || act == MDLC_ACT_RELU || act == MDLC_ACT_CLIP ||
                      act == MDLC_ACT_GELU || act == MDLC_ACT_SIGMOID)) ? act : -1;
  // none / ReLU / clip with bounds exact in bf16: applied to packed bf16 pairs
  if (act_t == MDLC_ACT_NONE || act_t == MDLC_ACT_RELU || act_t == MDLC_ACT_CLIP) {
    const float lo = act_t == MDLC_ACT_CLIP ? a.act.lo : (act_t == MDLC_ACT_RELU ? 0.0f : -INFINITY);
    const float hi = act_t == MDLC_ACT_CLIP ? a.act.hi : INFINITY;
    uint32_t lo2 = 0, hi2 = 0;
    if (bf16_pair_exact(lo, &lo2) && bf16_pair_exact(hi, &hi2) && lo <= hi) {
      a.act_packed = 1;
      a.act_lo2 = lo2;
      a.act_hi2 = hi2;
    }
  }
  const TcLaunch l{&tmap, &tmap_y, &tmap_r, &tmap_x, &a, bn, stages, amode, act_t};
  if (fp32) return launch_tc_f32(ctx, l);
  if (int8) return launch_tc_i8(ctx, l);
  if ((bn == 64 && stages == 3) || (bn == 128 && stages == 2) || (bn == 256 && stages == 3))
    return launch_tc_bf16_a(ctx, l);
  return launch_tc_bf16_b(ctx, l);
}

}  // namespace mdlc
