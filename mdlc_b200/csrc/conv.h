// Internal entry points of the convolution kernels (not part of the C ABI).
#pragma once

#include <cudaTypedefs.h>

#include "mdlc_b200.h"
#include "runtime.h"

namespace mdlc {

// tcgen05 implicit GEMM (bf16, int8, fp32 as 3xTF32), groups == 1
int conv_tc(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const void* w, const void* bias,
            const void* res, void* y, const mdlc_epilogue* epi, const mdlc_tile_cfg* cfg);
// depthwise (groups == c == k), bf16 or fp32 activations, fp32 weights
int conv_dw(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
            const void* res, void* y, const mdlc_epilogue* epi);

// grouped (1 < groups, not depthwise), bf16 or fp32 activations, fp32 weights
int conv_grouped(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
                 const void* res, void* y, const mdlc_epilogue* epi);

// depthwise 3x3 with TMA halo staging; MDLC_ERR_UNSUPPORTED when the layer
// does not fit it (the caller then uses conv_dw)
int conv_dw_tma(mdlc_ctx* ctx, const mdlc_conv_desc& d, const void* x, const float* w, const float* bias,
                const void* res, void* y, const mdlc_epilogue* epi);
// its tile for one layer: channel block (elements), threads as quads x column
// pairs x row groups, rows per thread, output tile, input window, stage ring
struct DwTileChoice {
  int cb, quads, pairs, groups, rows, th, tw, ih, iw, stage_bytes, stages;
};
DwTileChoice choose_dw_tile(int c_stride, int esz, int oh, int ow, int n, int sh);
// cuTensorMapEncodeTiled from the driver (null when unavailable)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

}  // namespace mdlc
