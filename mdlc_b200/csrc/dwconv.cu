// Depthwise 3x3 convolution with the input window staged in shared memory by TMA.
//
// Reference semantics: the grouped conv of mdlc/runtime/ops.py:68-78 with
// groups == C == K, which the reference GPU lowering runs on the host
// (mdlc/codegen/cuda/emit.py:175-180).
//
// HBM-bound (9 multiply-adds per output element against 2 bytes read and 2
// written in bf16), so the kernel has two jobs: keep enough bytes in flight
// to stream HBM, and spend few enough instructions per output that the SM's
// issue rate is not the limit. Bytes in flight come from TMA: persistent
// CTAs (one per SM, 12 warps) walk tiles of TH x TW output pixels x one
// channel block, and one thread keeps up to four tile windows ((TH-1)*S+3 x
// (TW-1)*S+3 input pixels x the block; out-of-image pixels arrive as zeros,
// so padding costs nothing) loading into shared memory while the current one
// is computed. Instructions: each thread owns four channels of TWO adjacent
// output columns and walks R output rows of the tile with a register ring of
// the input rows they need (per output row, one new input row of four pixels
// at stride 1: 2 new input pixels per output instead of 3), weights and bias
// in registers, 9 fp32 multiply-adds per output, and for bf16 outputs the
// clamp activations (none / ReLU / ReLU6-style clip) applied to the packed
// bf16 pairs (max/min.bf16x2).
// The host picks the channel block, the tile and R per layer so that a layer
// of any spatial size keeps most threads on real pixels.
#include <cmath>

#include "common.cuh"
#include "conv.h"

namespace mdlc {
namespace {

constexpr int kDwThreads = 384;
constexpr int kDwMaxStages = 4;
constexpr int kDwSmemBudget = 200 * 1024;  // stage ring (one CTA per SM)
constexpr int kDwMaxStageBytes = 64 * 1024;

struct DwTmaArgs {
  const float* w;  // [9][cs] fp32
  const float* bias;
  const void* res;
  void* y;
  int* err;
  int cs, c, res_s, oh, ow, pt, pl;
  int cb_elems, cblocks;            // channel block (elements), blocks per pixel
  int quads, pairs, groups, rows;   // threads: quads x column pairs x row groups; rows per thread
  int th, tw, ih, iw;               // output tile and input window extents
  int stage_bytes, stages;
  int tiles_x, tiles_y, total;      // tiles per image row / column, total tiles
  long long y_elems, res_elems;     // element extents (checked build)
  unsigned long long wait_cycles;
  ActParams act;
  int act_kind;                     // 0 identity, 1 clamp to [lo, hi], 2 general (apply_act)
  uint32_t lo2, hi2;                // bf16 output: the clamp bounds as bf16 pairs
};

// 4 channels of one pixel from shared memory, as two fp32 pairs
template <typename T>
MDLC_DEV void lds4(const uint8_t* p, float2 (&f)[2]);
template <>
MDLC_DEV void lds4<__nv_bfloat16>(const uint8_t* p, float2 (&f)[2]) {
  const uint2 v = *reinterpret_cast<const uint2*>(p);
  f[0] = make_float2(bf16_lo(v.x), bf16_hi(v.x));
  f[1] = make_float2(bf16_lo(v.y), bf16_hi(v.y));
}
template <>
MDLC_DEV void lds4<float>(const uint8_t* p, float2 (&f)[2]) {
  const float4 v = *reinterpret_cast<const float4*>(p);
  f[0] = make_float2(v.x, v.y);
  f[1] = make_float2(v.z, v.w);
}

// 4 channels of a global tensor as two fp32 pairs (the residual)
template <typename T>
MDLC_DEV void ldg4(const T* p, float2 (&f)[2]);
template <>
MDLC_DEV void ldg4<__nv_bfloat16>(const __nv_bfloat16* p, float2 (&f)[2]) {
  const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
  f[0] = make_float2(bf16_lo(v.x), bf16_hi(v.x));
  f[1] = make_float2(bf16_lo(v.y), bf16_hi(v.y));
}
template <>
MDLC_DEV void ldg4<float>(const float* p, float2 (&f)[2]) {
  const float4 v = __ldg(reinterpret_cast<const float4*>(p));
  f[0] = make_float2(v.x, v.y);
  f[1] = make_float2(v.z, v.w);
}

// bias + taps (+ residual) of 4 channels -> activation -> 4 output elements;
// channels at or past c (the padding of the channel stride) are written as 0
template <typename T, bool GEN>
MDLC_DEV void store4(const DwTmaArgs& a, T* yp, float2 (&f)[2], bool full, int c0) {
  if constexpr (sizeof(T) == 4) {
    float v[4] = {f[0].x, f[0].y, f[1].x, f[1].y};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if constexpr (GEN) v[e] = apply_act(v[e], a.act);
      else if (a.act_kind == 1) v[e] = fminf(fmaxf(v[e], a.act.lo), a.act.hi);
      if (!full && c0 + e >= a.c) v[e] = 0.0f;
    }
    *reinterpret_cast<float4*>(yp) = make_float4(v[0], v[1], v[2], v[3]);
    return;
  }
  if constexpr (GEN) {
    f[0] = make_float2(apply_act(f[0].x, a.act), apply_act(f[0].y, a.act));
    f[1] = make_float2(apply_act(f[1].x, a.act), apply_act(f[1].y, a.act));
  }
  if (!full) {
    f[0] = make_float2(c0 < a.c ? f[0].x : 0.0f, c0 + 1 < a.c ? f[0].y : 0.0f);
    f[1] = make_float2(c0 + 2 < a.c ? f[1].x : 0.0f, c0 + 3 < a.c ? f[1].y : 0.0f);
  }
  uint32_t w0 = pack_bf16x2(f[0].x, f[0].y), w1 = pack_bf16x2(f[1].x, f[1].y);
  // clamp bounds are exact in bf16 (the host checks), and rounding is
  // monotonic, so clamping the rounded pair equals rounding the clamped one;
  // a zero padding channel stays zero as every clamp range holds 0
  if (!GEN && a.act_kind == 1) {
    w0 = clamp_bf16x2(w0, a.lo2, a.hi2);
    w1 = clamp_bf16x2(w1, a.lo2, a.hi2);
  }
  *reinterpret_cast<uint2*>(yp) = make_uint2(w0, w1);
}

// GEN: the activation is not a clamp (apply_act per element)
template <typename T, int SH, bool GEN>
__global__ void __launch_bounds__(kDwThreads, 1)
    conv_dw3_tma_kernel(const __grid_constant__ CUtensorMap tmap, const DwTmaArgs a) {
  pdl_wait();  // launched with programmatic serialization: nothing global before this
  pdl_trigger();
  constexpr int NC = SH == 1 ? 4 : 5;  // input columns under a thread's two output columns
  constexpr int esz = (int)sizeof(T);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 127) & ~uintptr_t(127));
  const uint32_t sbase = smem_u32(smem);
  const int NS = a.stages;
  const int ring_bytes = NS * a.stage_bytes;
  const uint32_t bar0 = sbase + ring_bytes;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + ring_bytes + 8 * kDwMaxStages);
  const int tid = threadIdx.x;
  const int cb_bytes = a.cb_elems * esz;
  const int per_img = a.tiles_x * a.tiles_y;
  // tiles are numbered channel block minor and the grid is a multiple of the
  // block count, so a CTA keeps one channel block (its weights stay in
  // registers) while the CTAs of the other blocks work on the same pixels at
  // the same time: the 64-byte DRAM bursts and halo pixels they share are L2 hits
  auto decode = [&](int tile, int& cb, int& img, int& ty, int& tx) {
    int t = tile / a.cblocks;
    cb = tile - t * a.cblocks;
    img = t / per_img;
    t -= img * per_img;
    ty = t / a.tiles_x;
    tx = t - ty * a.tiles_x;
  };
  auto issue = [&](int tile, int stage) {
    int cb, img, ty, tx;
    decode(tile, cb, img, ty, tx);
    const uint32_t bar = bar0 + 8u * stage;
    mbar_arrive_expect_tx(bar, (uint32_t)(a.ih * a.iw * cb_bytes));
    tma_load_4d(sbase + stage * a.stage_bytes, &tmap, cb * a.cb_elems, tx * a.tw * SH - a.pl,
                ty * a.th * SH - a.pt, img, bar);
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

  // thread -> (4-channel quad, output column pair, row group of R rows)
  const int Q = a.quads, P = a.pairs;
  const int qd = tid % Q, pr = (tid / Q) % P, rg = tid / (Q * P);
  const bool active = rg < a.groups;
  const int ox = 2 * pr;            // tile-local first output column
  const int oy0 = rg * a.rows;      // tile-local first output row
  const int row_bytes = a.iw * cb_bytes;
  float2 w[9][2], bias[2];
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
    const int c0 = cb * a.cb_elems + qd * 4;
    const int gx = tx * a.tw + ox;
    const int gy0 = ty * a.th + oy0;
    if (active && gx < a.ow && gy0 < a.oh) {
      if (cb != cur_cb) {
#pragma unroll
        for (int tap = 0; tap < 9; ++tap) {
          const float4 w4 = __ldg(reinterpret_cast<const float4*>(a.w + tap * a.cs + c0));
          w[tap][0] = make_float2(w4.x, w4.y);
          w[tap][1] = make_float2(w4.z, w4.w);
        }
        // bias holds c floats (not necessarily the padded stride)
        float b4[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) b4[e] = (a.bias && c0 + e < a.c) ? __ldg(a.bias + c0 + e) : 0.0f;
        bias[0] = make_float2(b4[0], b4[1]);
        bias[1] = make_float2(b4[2], b4[3]);
        cur_cb = cb;
      }
      const bool full = c0 + 4 <= a.c;
      const bool v1 = gx + 1 < a.ow;
      const uint8_t* colp = smem + stage * a.stage_bytes + (ox * SH) * cb_bytes + qd * 4 * esz;
      float2 x[3][NC][2];  // the input rows under the current output row, unpacked
      auto load_row = [&](int wr, float2 (&dst)[NC][2]) {
        const uint8_t* rp = colp + wr * row_bytes;
#pragma unroll
        for (int c = 0; c < NC; ++c) lds4<T>(rp + c * cb_bytes, dst[c]);
      };
#pragma unroll
      for (int r = 0; r < 3; ++r) load_row(oy0 * SH + r, x[r]);
      const int nrows = min(a.rows, a.oh - gy0);
      const long long m0 = ((long long)img * a.oh + gy0) * a.ow + gx;
      // output row r from the ring (xa, xb, xc) = its input rows; then the
      // oldest slot(s) take the next row's new input rows. The row loop is
      // unrolled by three with the slots rotated, so the ring never moves.
      auto step = [&](float2 (&xa)[NC][2], float2 (&xb)[NC][2], float2 (&xc)[NC][2], int r) {
        float2 acc[2][2] = {{bias[0], bias[1]}, {bias[0], bias[1]}};
#pragma unroll
        for (int kx = 0; kx < 3; ++kx)
#pragma unroll
          for (int j = 0; j < 2; ++j)
#pragma unroll
            for (int e = 0; e < 2; ++e) {
              // scalar fmas: measured faster than forcing fma.rn.f32x2 through
              // inline asm (MobileNetV2 depthwise 65.5 vs 71.5 us per launch)
              acc[j][e].x = fmaf(xa[j * SH + kx][e].x, w[kx][e].x, acc[j][e].x);
              acc[j][e].y = fmaf(xa[j * SH + kx][e].y, w[kx][e].y, acc[j][e].y);
              acc[j][e].x = fmaf(xb[j * SH + kx][e].x, w[3 + kx][e].x, acc[j][e].x);
              acc[j][e].y = fmaf(xb[j * SH + kx][e].y, w[3 + kx][e].y, acc[j][e].y);
              acc[j][e].x = fmaf(xc[j * SH + kx][e].x, w[6 + kx][e].x, acc[j][e].x);
              acc[j][e].y = fmaf(xc[j * SH + kx][e].y, w[6 + kx][e].y, acc[j][e].y);
            }
        const long long m = m0 + (long long)r * a.ow;
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          if (j == 1 && !v1) break;
          const long long mj = m + j;
          if (!MDLC_CHECK_IDX(a.err, mj * a.cs + c0 + 3, a.y_elems)) continue;
          if (a.res) {
            if (!MDLC_CHECK_IDX(a.err, mj * a.res_s + c0 + 3, a.res_elems)) continue;
            float2 rv[2];
            ldg4<T>(static_cast<const T*>(a.res) + mj * a.res_s + c0, rv);
            acc[j][0].x += rv[0].x; acc[j][0].y += rv[0].y;
            acc[j][1].x += rv[1].x; acc[j][1].y += rv[1].y;
          }
          store4<T, GEN>(a, static_cast<T*>(a.y) + mj * a.cs + c0, acc[j], full, c0);
        }
        if (r + 1 >= nrows) return false;
        const int oy = oy0 + r;
        if (SH == 1) {
          load_row(oy + 3, xa);  // next: (xb, xc, xa)
        } else {
          load_row(oy * 2 + 3, xa);  // next: (xc, xa, xb)
          load_row(oy * 2 + 4, xb);
        }
        return true;
      };
      if (SH == 1) {
        for (int r = 0;; r += 3)
          if (!step(x[0], x[1], x[2], r) || !step(x[1], x[2], x[0], r + 1) || !step(x[2], x[0], x[1], r + 2)) break;
      } else {
        for (int r = 0;; r += 3)
          if (!step(x[0], x[1], x[2], r) || !step(x[2], x[0], x[1], r + 1) || !step(x[1], x[2], x[0], r + 2)) break;
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

uint16_t bf16_bits_rn(float f) {
  uint32_t u;
  memcpy(&u, &f, 4);
  if (std::isnan(f)) return 0x7FC0;
  return (uint16_t)((u + 0x7FFFu + ((u >> 16) & 1u)) >> 16);
}

}  // namespace

// Tile choice for one layer (host): channel block, column pairs, rows per
// thread. Score = the fraction of threads on real output pixels (and of
// enough tiles to occupy every SM) over a per-output instruction estimate:
// 4.5 paired FMAs + ~2 for the epilogue + the ring loads (an input row of
// NC pixels is 5 instructions a pixel in bf16 -- one shared load, four
// unpacks -- and a thread loads R + 2 rows at stride 1, 2R + 1 at stride 2,
// for 8 outputs a row) + ~100 instructions of per-tile overhead (barrier,
// tile decode) spread over the thread's 8R outputs.
DwTileChoice choose_dw_tile(int c_stride, int esz, int oh, int ow, int n, int sh) {
  DwTileChoice best{};
  double best_score = -1.0;
  for (int cbb = 256; cbb >= 16; cbb -= 16) {  // channel block bytes
    const int cb = cbb / esz;
    if (cb % 4 || c_stride % cb) continue;
    const int Q = cb / 4;
    for (int P = 8; P >= 2; --P) {
      if (Q * P > kDwThreads) continue;
      const int G = kDwThreads / (Q * P);
      for (int R = 8; R >= 1; --R) {
        const int th = G * R, tw = 2 * P;
        const int ih = (th - 1) * sh + 3, iw = (tw - 1) * sh + 3;
        if (ih > 256 || iw > 256) continue;
        const int stage = (ih * iw * cbb + 127) / 128 * 128;
        if (stage > kDwMaxStageBytes) continue;
        int stages = kDwSmemBudget / stage;
        if (stages > kDwMaxStages) stages = kDwMaxStages;
        if (stages < 2) continue;
        const long long tx = (ow + tw - 1) / tw, ty = (oh + th - 1) / th;
        const double used = (double)oh * ow / ((double)tx * tw * ty * th) * (double)(Q * P * G) / kDwThreads;
        const double load = sh == 1 ? (R + 2.0) / R * 2.5 : (2.0 * R + 1.0) / R * 3.125;
        const double cost = 6.5 + load + 100.0 / (8.0 * R);
        const long long tiles = (long long)(c_stride / cb) * n * tx * ty;
        const double spread = tiles >= 4 * 148 ? 1.0 : (double)tiles / (4 * 148);
        const double score = used * spread / cost;
        if (score > best_score + 1e-9) {
          best_score = score;
          best = DwTileChoice{cb, Q, P, G, R, th, tw, ih, iw, stage, stages};
        }
      }
    }
  }
  return best;
}

int conv_dw_tma(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
                const void* res, void* y, const mdlc_epilogue* epi) {
  if (d.r != 3 || d.s != 3 || d.dil_h != 1 || d.dil_w != 1 || d.stride_h != d.stride_w ||
      (d.stride_h != 1 && d.stride_h != 2))
    return MDLC_ERR_UNSUPPORTED;
  const bool bf = d.in_type == MDLC_BF16;
  const int esz = bf ? 2 : 4;
  auto encode = tensor_map_encoder();
  const int SH = d.stride_h;
  const DwTileChoice t = choose_dw_tile(d.c_stride, esz, d.oh, d.ow, d.n, SH);
  if (!t.cb || !encode) return MDLC_ERR_UNSUPPORTED;
  const long long tiles_x = (d.ow + t.tw - 1) / t.tw, tiles_y = (d.oh + t.th - 1) / t.th;
  const long long total = (long long)(d.c_stride / t.cb) * d.n * tiles_x * tiles_y;
  if (total >= (1ll << 31)) return MDLC_ERR_UNSUPPORTED;
  CUtensorMap tmap;
  const cuuint64_t gd[4] = {(cuuint64_t)d.c_stride, (cuuint64_t)d.w, (cuuint64_t)d.h, (cuuint64_t)d.n};
  const cuuint64_t gs[3] = {(cuuint64_t)d.c_stride * esz, (cuuint64_t)d.w * d.c_stride * esz,
                            (cuuint64_t)d.h * d.w * d.c_stride * esz};
  const cuuint32_t box[4] = {(cuuint32_t)t.cb, (cuuint32_t)t.iw, (cuuint32_t)t.ih, 1};
  const cuuint32_t es[4] = {1, 1, 1, 1};
  if (encode(&tmap, bf ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<void*>(x),
             gd, gs, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return MDLC_ERR_UNSUPPORTED;
  DwTmaArgs a{};
  a.w = w; a.bias = bias; a.res = res; a.y = y; a.err = ctx->d_err;
  a.cs = d.c_stride; a.c = d.c; a.res_s = d.res_stride ? d.res_stride : d.c_stride;
  a.oh = d.oh; a.ow = d.ow; a.pt = d.pad_t; a.pl = d.pad_l;
  a.cb_elems = t.cb; a.cblocks = d.c_stride / t.cb;
  a.quads = t.quads; a.pairs = t.pairs; a.groups = t.groups; a.rows = t.rows;
  a.th = t.th; a.tw = t.tw; a.ih = t.ih; a.iw = t.iw;
  a.stage_bytes = t.stage_bytes; a.stages = t.stages;
  a.tiles_x = (int)tiles_x; a.tiles_y = (int)tiles_y; a.total = (int)total;
  a.y_elems = (long long)d.n * d.oh * d.ow * d.c_stride;
  a.res_elems = (long long)d.n * d.oh * d.ow * a.res_s;
  a.wait_cycles = 2 * kWaitLimitNs;
  a.act = epi ? ActParams{epi->act, epi->alpha, epi->beta, epi->clip_lo, epi->clip_hi}
              : ActParams{MDLC_ACT_NONE, 0.f, 0.f, -INFINITY, INFINITY};
  // activations that are a clamp: none (kind 0), ReLU, and clip with bounds
  // exact in the output type
  a.act_kind = 2;
  if (a.act.act == MDLC_ACT_NONE) {
    a.act_kind = 0;
  } else if (a.act.act == MDLC_ACT_RELU || a.act.act == MDLC_ACT_CLIP) {
    const float lo = a.act.act == MDLC_ACT_RELU ? 0.0f : a.act.lo;
    const float hi = a.act.act == MDLC_ACT_RELU ? INFINITY : a.act.hi;
    const uint16_t lb = bf16_bits_rn(lo), hb = bf16_bits_rn(hi);
    uint32_t lu, hu;
    memcpy(&lu, &lo, 4);
    memcpy(&hu, &hi, 4);
    const bool exact = !bf || (((uint32_t)lb << 16) == lu && ((uint32_t)hb << 16) == hu);
    if (exact && lo <= 0.0f && hi >= 0.0f && !std::isnan(lo) && !std::isnan(hi)) {
      a.act_kind = 1;
      a.act.lo = lo;
      a.act.hi = hi;
      a.lo2 = (uint32_t)lb | ((uint32_t)lb << 16);
      a.hi2 = (uint32_t)hb | ((uint32_t)hb << 16);
    }
  }
  // one CTA per SM, a multiple of the channel block count (see decode)
  const long long per_block = total / a.cblocks;
  long long ctas_per_block = ctx->num_sms / a.cblocks;
  if (ctas_per_block < 1) ctas_per_block = 1;
  if (ctas_per_block > per_block) ctas_per_block = per_block;
  const unsigned grid = (unsigned)(ctas_per_block * a.cblocks);
  void (*kern)(const CUtensorMap, const DwTmaArgs);
  const bool gen = a.act_kind == 2;
  if (SH == 1) {
    if (bf) kern = gen ? conv_dw3_tma_kernel<__nv_bfloat16, 1, true> : conv_dw3_tma_kernel<__nv_bfloat16, 1, false>;
    else kern = gen ? conv_dw3_tma_kernel<float, 1, true> : conv_dw3_tma_kernel<float, 1, false>;
  } else {
    if (bf) kern = gen ? conv_dw3_tma_kernel<__nv_bfloat16, 2, true> : conv_dw3_tma_kernel<__nv_bfloat16, 2, false>;
    else kern = gen ? conv_dw3_tma_kernel<float, 2, true> : conv_dw3_tma_kernel<float, 2, false>;
  }
  const int smem = t.stages * t.stage_bytes + 8 * kDwMaxStages + 16 + 128;  // + barriers, flag, alignment slack
  static int attr_set[64][8] = {};
  const int which = (SH - 1) * 4 + (bf ? 2 : 0) + (gen ? 1 : 0);
  if (attr_set[ctx->device & 63][which] < smem) {
    const cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return mdlc_cuda_status(ctx, e, "conv_dw3_tma smem attribute");
    attr_set[ctx->device & 63][which] = smem;
  }
  const cudaError_t e = launch_pdl(kern, dim3(grid), dim3(kDwThreads), (size_t)smem, ctx->stream, tmap, a);
  mdlc_note_launch(ctx);
  return mdlc_cuda_status(ctx, e != cudaSuccess ? e : cudaGetLastError(), "conv_dw3_tma launch");
}

}  // namespace mdlc
