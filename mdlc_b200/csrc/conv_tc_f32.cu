// fp32 (3xTF32, kind::tf32) instantiations of the tcgen05 convolution kernel:
// tiles (64, 3), (128, 2), (256, 2) in every A mode but the halo band; the
// deeper rings (64, 4) and (128, 3) (194 / 199 KB of shared memory: hi, lo
// and weight stages) for the TMA modes of 128-byte channel blocks only.
#include "conv_tc_kernel.cuh"

namespace mdlc {

#define MDLC_TC_LAUNCH_F32(BN_, ST_)                                                                      \
  switch (l.amode) {                                                                                      \
    case 1: return launch_tc<BN_, ST_, 4, -1, 1>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    case 5: return launch_tc<BN_, ST_, 4, -1, 5>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    case 2: if (BN_ <= 128) return launch_tc<BN_, ST_, 4, -1, 2>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); break; \
    case 3: if (BN_ <= 128) return launch_tc<BN_, ST_, 4, -1, 3>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); break; \
    default: break;                                                                                       \
  }                                                                                                       \
  return launch_tc<BN_, ST_, 4, -1, 0>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args);

#define MDLC_TC_LAUNCH_F32_DEEP(BN_, ST_)                                                                 \
  switch (l.amode) {                                                                                      \
    case 1: return launch_tc<BN_, ST_, 4, -1, 1>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    case 5: return launch_tc<BN_, ST_, 4, -1, 5>(ctx, *l.tmap_w, *l.tmap_y, *l.tmap_r, *l.tmap_x, *l.args); \
    default: break;                                                                                       \
  }                                                                                                       \
  return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "conv_tc: fp32 tile (%d, %d) needs 128-byte channel blocks", BN_, ST_);

int launch_tc_f32(mdlc_ctx* ctx, const TcLaunch& l) {
  if (l.bn == 64 && l.stages == 3) { MDLC_TC_LAUNCH_F32(64, 3) }
  if (l.bn == 128 && l.stages == 2) { MDLC_TC_LAUNCH_F32(128, 2) }
  if (l.bn == 256 && l.stages == 2) { MDLC_TC_LAUNCH_F32(256, 2) }
  if (l.bn == 64 && l.stages == 4) { MDLC_TC_LAUNCH_F32_DEEP(64, 4) }
  if (l.bn == 128 && l.stages == 3) { MDLC_TC_LAUNCH_F32_DEEP(128, 3) }
  return mdlc_set_error(ctx, MDLC_ERR_UNSUPPORTED, "conv_tc: no fp32 kernel for bn=%d stages=%d", l.bn, l.stages);
}

}  // namespace mdlc
