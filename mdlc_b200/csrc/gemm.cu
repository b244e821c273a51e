// GEMM and depthwise entry points of the C ABI, expressed on the convolution
// kernels. A GEMM y[m, n] = a[m, k] . op(b) is a 1x1 convolution over m
// images of one pixel with k input and n output channels, so it runs on the
// tcgen05 implicit-GEMM kernel (a loaded as a plain 2-D tile): bf16, 8-bit, and
// fp32 as 3xTF32. Reference: the Gemm / MatMul lowering of
// mdlc/codegen/cuda/emit.py:211-244 and ops.gemm (mdlc/runtime/ops.py:84-92).
#include <cstring>
#include <vector>

#include "runtime.h"

namespace {

bool is8(int t) { return t == MDLC_U8 || t == MDLC_S8; }

int to_conv(const mdlc_gemm_desc* g, mdlc_conv_desc* d) {
  if (!g || g->m <= 0 || g->n <= 0 || g->k <= 0) return MDLC_ERR_INVALID;
  if (g->trans_a) return MDLC_ERR_UNSUPPORTED;
  const int a8 = is8(g->in_type) ? 16 : 8;
  const int o8 = is8(g->out_type) ? 16 : 8;
  std::memset(d, 0, sizeof(*d));
  d->n = g->m;
  d->h = d->w = d->oh = d->ow = 1;
  d->c = g->k;
  d->c_stride = g->lda ? g->lda : (g->k + a8 - 1) / a8 * a8;
  d->k = g->n;
  d->k_stride = (g->n + o8 - 1) / o8 * o8;
  d->r = d->s = 1;
  d->stride_h = d->stride_w = 1;
  d->dil_h = d->dil_w = 1;
  d->groups = 1;
  d->in_type = g->in_type;
  d->out_type = g->out_type;
  return MDLC_OK;
}

}  // namespace

extern "C" int mdlc_gemm_weight_bytes(const mdlc_gemm_desc* g, size_t* bytes) {
  mdlc_conv_desc d;
  const int st = to_conv(g, &d);
  if (st) return st;
  return mdlc_conv_weight_bytes(&d, bytes);
}

extern "C" int mdlc_pack_gemm_weights(const mdlc_gemm_desc* g, const float* b, void* out) {
  mdlc_conv_desc d;
  const int st = to_conv(g, &d);
  if (st) return st;
  if (!b || !out) return MDLC_ERR_INVALID;
  // OIHW [n][k][1][1] = alpha * op(b)^T
  std::vector<float> w((size_t)g->n * g->k);
  for (int o = 0; o < g->n; ++o)
    for (int i = 0; i < g->k; ++i)
      w[(size_t)o * g->k + i] = g->alpha * (g->trans_b ? b[(size_t)o * g->k + i] : b[(size_t)i * g->n + o]);
  return mdlc_pack_conv_weights(&d, w.data(), out);
}

extern "C" int mdlc_gemm(mdlc_ctx* ctx, const mdlc_gemm_desc* g, const void* a, const void* b, const void* bias,
                         void* y, const mdlc_epilogue* epi, const mdlc_tile_cfg* cfg) {
  if (!ctx) return MDLC_ERR_INVALID;
  mdlc_conv_desc d;
  const int st = to_conv(g, &d);
  if (st == MDLC_ERR_UNSUPPORTED) return mdlc_set_error(ctx, st, "gemm: trans_a = 1 is not supported");
  if (st) return mdlc_set_error(ctx, st, "gemm: bad descriptor");
  return mdlc_conv2d(ctx, &d, a, b, bias, nullptr, y, epi, cfg);
}

extern "C" int mdlc_dwconv2d(mdlc_ctx* ctx, const mdlc_conv_desc* d, const void* x, const void* w,
                             const void* bias, const void* res, void* y, const mdlc_epilogue* epi) {
  if (!ctx) return MDLC_ERR_INVALID;
  if (!d || d->groups != d->c || d->k != d->c)
    return mdlc_set_error(ctx, MDLC_ERR_INVALID, "dwconv: needs groups == c == k");
  return mdlc_conv2d(ctx, d, x, w, bias, res, y, epi, nullptr);
}
