// 8-bit (kind::i8) instantiations of the tcgen05 convolution kernel, every tile
// configuration; the epilogue requantises (fixed point or fp32) at run time.
#include "conv_tc_kernel.cuh"

namespace mdlc {

#define MDLC_TC_LAUNCH(BN_, ST_, E_, A_)                                                                      \
  switch (l.amode) {                                                                                        \
    case 1: return launch_tc<BN_, ST_, E_, A_, 1>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    case 4: return launch_tc<BN_, ST_, E_, A_, 4>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    case 5: return launch_tc<BN_, ST_, E_, A_, 5>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    case 2: if (BN_ <= 128) return launch_tc<BN_, ST_, E_, A_, 2>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); break; \
    case 3: if (BN_ <= 128) return launch_tc<BN_, ST_, E_, A_, 3>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); break; \
    default: break;                                                                                         \
  }                                                                                                         \
  return launch_tc<BN_, ST_, E_, A_, 0>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args);

int launch_tc_i8(mdlc_ctx* ctx, const TcLaunch& l) {
  if (l.bn == 64 && l.stages == 3) { MDLC_TC_LAUNCH(64, 3, 1, -1) }
  if (l.bn == 128 && l.stages == 2) { MDLC_TC_LAUNCH(128, 2, 1, -1) }
  if (l.bn == 256 && l.stages == 3) { MDLC_TC_LAUNCH(256, 3, 1, -1) }
  if (l.bn == 192 && l.stages == 3) { MDLC_TC_LAUNCH(192, 3, 1, -1) }
  if (l.bn == 64 && l.stages == 8) { MDLC_TC_LAUNCH(64, 8, 1, -1) }
  if (l.bn == 128 && l.stages == 4) { MDLC_TC_LAUNCH(128, 4, 1, -1) }
  return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "conv_tc: no int8 kernel for bn=%d stages=%d", l.bn, l.stages);
}

}  // namespace mdlc
