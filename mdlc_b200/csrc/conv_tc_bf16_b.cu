// bf16 instantiations of the tcgen05 convolution kernel, tiles (192, 3), (64, 8), (128, 4)
// and the resident-weight halo tile (64, kResidentKb):
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

int launch_tc_bf16_b(mdlc_ctx* ctx, const TcLaunch& l) {
  if (l.bn == 192 && l.stages == 3) {
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_LAUNCH(192, 3, 2, MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_LAUNCH(192, 3, 2, MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_LAUNCH(192, 3, 2, MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_LAUNCH(192, 3, 2, MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_LAUNCH(192, 3, 2, MDLC_ACT_SIGMOID) }
    MDLC_TC_LAUNCH(192, 3, 2, -1)
  }
  if (l.bn == 64 && l.stages == 8) {
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_LAUNCH(64, 8, 2, MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_LAUNCH(64, 8, 2, MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_LAUNCH(64, 8, 2, MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_LAUNCH(64, 8, 2, MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_LAUNCH(64, 8, 2, MDLC_ACT_SIGMOID) }
    MDLC_TC_LAUNCH(64, 8, 2, -1)
  }
  if (l.bn == 128 && l.stages == 4) {
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_LAUNCH(128, 4, 2, MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_LAUNCH(128, 4, 2, MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_LAUNCH(128, 4, 2, MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_LAUNCH(128, 4, 2, MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_LAUNCH(128, 4, 2, MDLC_ACT_SIGMOID) }
    MDLC_TC_LAUNCH(128, 4, 2, -1)
  }
  if (l.bn == 64 && l.stages == kResidentKb && l.amode == 4) {
    // resident-weight halo mode: the halo band main loop only
#define MDLC_TC_RESIDENT(A_) return launch_tc<64, kResidentKb, 2, A_, 4>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args);
    if (l.act == MDLC_ACT_NONE) { MDLC_TC_RESIDENT(MDLC_ACT_NONE) }
    if (l.act == MDLC_ACT_RELU) { MDLC_TC_RESIDENT(MDLC_ACT_RELU) }
    if (l.act == MDLC_ACT_CLIP) { MDLC_TC_RESIDENT(MDLC_ACT_CLIP) }
    if (l.act == MDLC_ACT_GELU) { MDLC_TC_RESIDENT(MDLC_ACT_GELU) }
    if (l.act == MDLC_ACT_SIGMOID) { MDLC_TC_RESIDENT(MDLC_ACT_SIGMOID) }
    MDLC_TC_RESIDENT(-1)
#undef MDLC_TC_RESIDENT
  }
  return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "conv_tc: no bf16 kernel for bn=%d stages=%d", l.bn, l.stages);
}

}  // namespace mdlc
