// bf16 instantiations of the tcgen05 convolution kernel, tiles (64, 3), (128, 2), (256, 3):
// each activation the TMA epilogue specialises, and the run-time switch.
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

int launch_tc_bf16_a(mdlc_ctx* ctx, const TcLaunch& l) {
  if (l.bn == 64 && l.stages == 3) {
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_LAUNCH(64, 3, 2, MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_LAUNCH(64, 3, 2, MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_LAUNCH(64, 3, 2, MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_LAUNCH(64, 3, 2, MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_LAUNCH(64, 3, 2, MDLC_ACT_SIGMOID) }
    MDLC_TC_LAUNCH(64, 3, 2, -1)
  }
  if (l.bn == 128 && l.stages == 2) {
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_LAUNCH(128, 2, 2, MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_LAUNCH(128, 2, 2, MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_LAUNCH(128, 2, 2, MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_LAUNCH(128, 2, 2, MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_LAUNCH(128, 2, 2, MDLC_ACT_SIGMOID) }
    MDLC_TC_LAUNCH(128, 2, 2, -1)
  }
  if (l.bn == 256 && l.stages == 3) {
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_LAUNCH(256, 3, 2, MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_LAUNCH(256, 3, 2, MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_LAUNCH(256, 3, 2, MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_LAUNCH(256, 3, 2, MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_LAUNCH(256, 3, 2, MDLC_ACT_SIGMOID) }
    MDLC_TC_LAUNCH(256, 3, 2, -1)
  }
  return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "conv_tc: no bf16 kernel for bn=%d stages=%d", l.bn, l.stages);
}

}  // namespace mdlc
