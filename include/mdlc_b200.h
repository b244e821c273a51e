/*
 * mdlc_b200 — C ABI of the B200 (sm_100a) execution library for mdlc graphs.
 *
 * This library replaces the reference compiler's code generation + GPU runtime
 * hot path: NVRTC compilation of generated CUDA C (mdlc/codegen/cuda/
 * nvrtc_runtime.py:97-159), the per-launch argument marshalling of the GPU
 * executor (mdlc/codegen/cuda/gpu_executor.py:38-98) and its host fallbacks
 * (gpu_executor.py:100-114). Every kernel is prebuilt for sm_100a; there is no
 * JIT and no host fallback.
 *
 * Conventions
 *   - Every function returns MDLC_OK (0) or a negative MDLC_ERR_* status; no
 *     C++ exception or abort crosses this boundary. mdlc_last_error() gives
 *     the message of the last failure on a context.
 *   - Pointers are device pointers unless named host_*. Kernels never free or
 *     retain caller pointers.
 *   - Activations are NHWC. A tensor's channel stride (c_stride / k_stride) is
 *     its channel count rounded up to a multiple of 8 (16 for 8-bit types);
 *     padding channels hold zeros and kernels keep them zero.
 *   - One context per device and host thread; calls on different contexts are
 *     independent. All work is issued on the context's stream.
 *   - Device-side waits are bounded (~2 s); on expiry a kernel records an error
 *     code in the context's device error word (read with mdlc_check_flag),
 *     releases its tensor memory and returns instead of hanging.
 */
#ifndef MDLC_B200_H
#define MDLC_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct mdlc_ctx mdlc_ctx;

/* ---- status codes ------------------------------------------------------ */
#define MDLC_OK 0
#define MDLC_ERR_INVALID (-1)     /* bad argument / shape / alignment */
#define MDLC_ERR_CUDA (-2)        /* a CUDA runtime call failed */
#define MDLC_ERR_UNSUPPORTED (-3) /* valid request this build does not implement */
#define MDLC_ERR_TIMEOUT (-4)     /* host-side wait exceeded its limit */
#define MDLC_ERR_DEVICE (-5)      /* a kernel reported a device-side error */
#define MDLC_ERR_NOMEM (-6)

/* device-side error word values (mdlc_check_flag) */
#define MDLC_DEVERR_NONE 0
#define MDLC_DEVERR_WAIT_TIMEOUT 1 /* an mbarrier wait ran out of time */
#define MDLC_DEVERR_BOUNDS 2       /* a checked index was out of range */
#define MDLC_DEVERR_INJECTED 3     /* raised by mdlc_debug_timeout_probe */

/* ---- element types ----------------------------------------------------- */
enum { MDLC_F32 = 0, MDLC_BF16 = 1, MDLC_S8 = 2, MDLC_U8 = 3, MDLC_S32 = 4 };

/* ---- epilogue activations (reference: mdlc/codegen/cuda/templates.py:24-51,
 *      mdlc/runtime/reference.py:19-38; GELU is an extension) ------------- */
enum {
  MDLC_ACT_NONE = 0,
  MDLC_ACT_RELU = 1,
  MDLC_ACT_CLIP = 2,
  MDLC_ACT_SIGMOID = 3,
  MDLC_ACT_TANH = 4,
  MDLC_ACT_LEAKY_RELU = 5,
  MDLC_ACT_HARD_SIGMOID = 6,
  MDLC_ACT_HARD_SWISH = 7,
  MDLC_ACT_GELU = 8
};

/* Fused epilogue applied to every conv / GEMM output element:
 *   float path: y = act(acc + bias[k] (+ residual))
 *   int8 path, fixed point (rq_mult set; the default of int8 executables):
 *               y = out_zp + clamp(t, qmin - out_zp, qmax - out_zp) with
 *               t = ((acc + bias32[k]) * rq_mult[k] (+ (residual - res_zp) * rq_res_mult[k])
 *                    + 2^(rq_shift[k] - 1)) >> rq_shift[k]
 *               in 64-bit integers, one rounding (half up): the single-rounding form of
 *               TFLite's MultiplyByQuantizedMultiplier, the two products sharing the shift
 *   int8 path, fp32 (rq_mult null, rq_scale set):
 *               y = out_zp + clamp(rint(f), qmin - out_zp, qmax - out_zp) with
 *               f = fp32(acc + bias32[k]) * rq_scale[k] (+ fp32(residual - res_zp) * res_scale),
 *               every product and sum one IEEE fp32 rounding (no fused multiply-add),
 *               rint = round half to even; bias is int32 for the int8 path
 *   int8 path with out_type F32: y = act(deq_scale[k] * (acc + bias32[k]) + deq_bias[k]
 *                                       (+ res_scale * (residual - res_zp)))  */
typedef struct {
  int32_t act;
  float alpha;    /* LeakyRelu slope / HardSigmoid alpha */
  float beta;     /* HardSigmoid beta */
  float clip_lo;  /* Clip bounds (use +-INFINITY for one-sided) */
  float clip_hi;
  const float* rq_scale;  /* [k] requantisation scales s_x * s_w[k] / s_y (int8 path, 8-bit output) */
  int32_t out_zp, qmin, qmax;
  int32_t res_zp;
  float res_scale;        /* residual scale: s_res / s_y (8-bit output) or s_res (float output) */
  int32_t res_signed;     /* int8 path: residual codes are signed int8 (else uint8) */
  const float* deq_scale; /* [k] (int8 path, float output) */
  const float* deq_bias;  /* [k] (int8 path, float output) */
  const int32_t* rq_mult;     /* [k] fixed-point multipliers (int8 path, 8-bit output); null: fp32 form */
  const int32_t* rq_res_mult; /* [k] residual multipliers sharing rq_shift (with a residual) */
  const int32_t* rq_shift;    /* [k] right shifts, 1..62 */
} mdlc_epilogue;

/* 2-D convolution over NHWC tensors (groups == 1: implicit GEMM; groups == c
 * == k: depthwise). A GEMM y[M,N] = x[M,K] * W[N,K]^T is the 1x1 conv with
 * n = M, h = w = 1. Reference semantics: mdlc/runtime/ops.py:56-81. */
typedef struct {
  int32_t n, h, w, c, c_stride; /* input */
  int32_t k, k_stride;          /* output channels and output channel stride */
  int32_t r, s;                 /* filter height / width */
  int32_t stride_h, stride_w;
  int32_t pad_t, pad_l;         /* top / left padding (bottom/right follow from oh/ow) */
  int32_t dil_h, dil_w;
  int32_t oh, ow;
  int32_t groups;
  int32_t in_type, out_type;    /* MDLC_BF16 -> MDLC_BF16|MDLC_F32; MDLC_F32 -> MDLC_F32;
                                   MDLC_U8|MDLC_S8 -> MDLC_U8|MDLC_S8|MDLC_F32|MDLC_S32, where
                                   MDLC_S32 writes the int32 accumulator + bias32 (no
                                   requantisation, no residual; k_stride a multiple of 8) */
  int32_t res_stride;           /* residual channel stride (0: same as k_stride) */
  int32_t in_zp;                /* 8-bit input zero point: padded taps read this value */
} mdlc_conv_desc;

/* Tile configuration for the tensor-core implicit GEMM (0 = library default). */
typedef struct {
  int32_t bn;     /* output channels per CTA: 64, 128, 192 or 256 */
  int32_t stages; /* shared-memory pipeline depth; built pairs: (64, 3), (128, 2) (two CTAs per SM), (256, 3), (192, 3), (64, 8), (128, 4);
                     fp32 (3xTF32): (64, 3), (128, 2), (256, 2), and (64, 4), (128, 3) for layers fed by TMA
                     in 128-byte channel blocks */
  int32_t flags;  /* bit 0: gather the A operand with cp.async even when the layer
                     qualifies for TMA loads; bit 1: per-tap TMA loads (im2col mode)
                     instead of the halo band of stride-1 layers; bit 2: load one halo band
                     per tile for stride-1 layers instead of one load per tap; bit 3: the
                     halo band with the whole weight matrix resident in shared memory, one
                     CTA per SM (bf16, channel stride a multiple of 64, at most 64 output
                     channels and 9 k-blocks of 128 bytes, e.g. 64 -> 64 3x3; bn and
                     stages are then chosen by the library; ignored otherwise); bits 8-15:
                     split-K, the reduction cut into that many slices on different CTAs,
                     the last one to finish a tile summing them in slice order (at most
                     8 MiB of fp32 / int32 partials: tiles x slices x 128 x bn x 4 bytes) */
} mdlc_tile_cfg;

/* Pooling over NHWC (reference: ops.py:109-150). kind: 0 max, 1 average,
 * 2 global average (kernel/stride/pad ignored). */
typedef struct {
  int32_t kind;
  int32_t n, h, w, c, c_stride;
  int32_t kh, kw, stride_h, stride_w, pad_t, pad_l, oh, ow;
  int32_t count_include_pad;
  int32_t dtype; /* MDLC_F32 | MDLC_BF16 | MDLC_U8 | MDLC_S8 */
  /* int8 average pooling requantisation (ignored for float types) */
  int32_t in_zp, out_zp, rq_mult, rq_shift;
} mdlc_pool_desc;

/* Fused elementwise program (reference: FusedElementwise groups,
 * mdlc/passes/fuse_elementwise.py:111-118, evaluated per element like
 * mdlc/codegen/cuda/templates.py:209-269 but interpreted, not generated).
 * Registers 0..n_inputs-1 are preloaded with the inputs; each instruction
 * writes register dst = op(src0, src1) or op(src0) or src0 `op` imm. */
enum {
  MDLC_EW_ADD = 0, MDLC_EW_SUB, MDLC_EW_MUL, MDLC_EW_DIV,
  MDLC_EW_ADDI, MDLC_EW_SUBI, MDLC_EW_RSUBI, MDLC_EW_MULI, MDLC_EW_DIVI, MDLC_EW_RDIVI,
  MDLC_EW_RELU, MDLC_EW_CLIP, MDLC_EW_SIGMOID, MDLC_EW_TANH, MDLC_EW_LEAKY_RELU,
  MDLC_EW_HARD_SIGMOID, MDLC_EW_HARD_SWISH, MDLC_EW_ERF, MDLC_EW_GELU, MDLC_EW_MAX, MDLC_EW_MIN
};
#define MDLC_EW_MAX_INPUTS 4
#define MDLC_EW_MAX_OUTPUTS 2
#define MDLC_EW_MAX_INSTR 24
/* input broadcast modes over an NHWC output of shape [n, hw, c] */
enum { MDLC_BC_FULL = 0, MDLC_BC_NC = 1, MDLC_BC_C = 2, MDLC_BC_SCALAR = 3 };

typedef struct {
  int8_t op, dst, src0, src1;
  float imm0, imm1;
} mdlc_ew_instr;

typedef struct {
  int32_t n, hw, c, c_stride; /* output geometry; every tensor uses c_stride */
  int32_t dtype;              /* MDLC_F32 | MDLC_BF16 */
  int32_t n_inputs, n_outputs, n_instr;
  int32_t bcast[MDLC_EW_MAX_INPUTS];
  int32_t out_reg[MDLC_EW_MAX_OUTPUTS];
  mdlc_ew_instr code[MDLC_EW_MAX_INSTR];
} mdlc_ew_prog;

/* ---- library / context ------------------------------------------------- */
int mdlc_version(void);
int mdlc_device_count(int* count);
int mdlc_ctx_create(int device, mdlc_ctx** out);
int mdlc_ctx_destroy(mdlc_ctx* ctx);
const char* mdlc_last_error(mdlc_ctx* ctx);
int mdlc_get_stream(mdlc_ctx* ctx, void** stream); /* cudaStream_t of the context */

/* ---- memory (the C side owns device and pinned host allocations) ------- */
int mdlc_alloc(mdlc_ctx* ctx, size_t bytes, void** dev);
int mdlc_free(mdlc_ctx* ctx, void* dev);
int mdlc_host_alloc(mdlc_ctx* ctx, size_t bytes, void** host);
int mdlc_host_free(mdlc_ctx* ctx, void* host);
int mdlc_upload(mdlc_ctx* ctx, void* dev, const void* host, size_t bytes);      /* async on the stream */
int mdlc_download(mdlc_ctx* ctx, void* host, const void* dev, size_t bytes);    /* async on the stream */
int mdlc_memset(mdlc_ctx* ctx, void* dev, int value, size_t bytes);
int mdlc_sync(mdlc_ctx* ctx, int timeout_ms);   /* waits for both streams of the context */
int mdlc_check_flag(mdlc_ctx* ctx, int* flag); /* reads and clears the device error word */

/* ---- copy stream: overlap host<->device transfers with compute ---------
 * Every context owns a compute stream (all kernels) and a copy stream.
 * Transfers may go on either; ordering between the two goes through fences:
 * mdlc_fence_record(ctx, id, s) marks the current end of stream s as fence id
 * (in [0, 64)), mdlc_fence_wait(ctx, id, s) makes later work on stream s wait
 * for the last recorded fence id (a fence never recorded is already passed),
 * and mdlc_fence_sync blocks the host on it. */
enum { MDLC_STREAM_COMPUTE = 0, MDLC_STREAM_COPY = 1 };
int mdlc_upload_on(mdlc_ctx* ctx, int stream, void* dev, const void* host, size_t bytes);
int mdlc_download_on(mdlc_ctx* ctx, int stream, void* host, const void* dev, size_t bytes);
int mdlc_fence_record(mdlc_ctx* ctx, int id, int stream);
int mdlc_fence_wait(mdlc_ctx* ctx, int id, int stream);
int mdlc_fence_sync(mdlc_ctx* ctx, int id, int timeout_ms);

/* ---- kernels (all asynchronous on the context stream) ------------------ */
/* Replaces conv lowering (mdlc/codegen/cuda/emit.py:159-209: im2col + gemm),
 * Gemm/MatMul lowering (emit.py:211-244) and grouped-conv host fallback
 * (emit.py:175-180). Weights must be packed with mdlc_pack_conv_weights. */
int mdlc_conv2d(mdlc_ctx* ctx, const mdlc_conv_desc* desc, const void* x, const void* w_packed,
                const void* bias, const void* residual, void* y, const mdlc_epilogue* epi,
                const mdlc_tile_cfg* cfg);
/* Size in bytes of the packed weight buffer for desc (host helper). */
int mdlc_conv_weight_bytes(const mdlc_conv_desc* desc, size_t* bytes);
/* Pack OIHW fp32 weights (reference layout, mdlc/runtime/ops.py:57) into the
 * layout the kernel for desc reads; int8 paths take already-quantised int8
 * values stored as float. Host-only. */
int mdlc_pack_conv_weights(const mdlc_conv_desc* desc, const float* host_w_oihw, void* host_out);
/* Split-K convolution that allocates nothing. No counterpart in the reference.
 * For callers that cannot call cudaMalloc -- a plug-in that only borrows a
 * stream from a host framework whose memory manager owns every device
 * allocation, or a service whose device memory budget is fixed at start-up --
 * and so cannot create an mdlc_ctx either. Runs mdlc_conv2d's tcgen05 kernel
 * with the reduction cut into `splits` (2..255) slices, as tile-config flags
 * bits 8-15 do, on `stream` (a cudaStream_t of the current device), with its
 * scratch (per-slice partials, per-tile arrival counters, error word) in a
 * fixed array of this library's device image: 8 MiB + 8 KiB, held by every GPU
 * that loads the library until the process exits. Layers needing more partials
 * than 8 MiB (tiles x splits x 128 x bn x 4 bytes) are rejected with
 * MDLC_ERR_INVALID; only bf16 inputs and groups == 1. The first call on a device
 * looks up the array's device address and should come before any stream
 * capture; each call clears the arrival counters it uses with cudaMemsetAsync
 * on `stream`. All calls on one GPU share that GPU's copy of the array, which
 * keeps the last call's contents: calls whose work can overlap on the GPU
 * (issued to different streams, or from host threads without ordering between
 * them) race on it and must be serialised by the caller. A device-side error
 * (a bounded wait that ran out: the output is then incomplete) is kept in the
 * array's error word, which mdlc_conv2d_splitk_noalloc_status reads. The
 * array's device address is cached per device for the life of the process:
 * after a device reset these entry points must not be called again.
 * On failure `msg` (may be null) receives a message. */
int mdlc_conv2d_splitk_noalloc(const mdlc_conv_desc* desc, const void* x, const void* w_packed,
                               const void* bias, const void* residual, void* y, const mdlc_epilogue* epi,
                               int splits, void* stream, char* msg, size_t msg_len);
/* Companion of mdlc_conv2d_splitk_noalloc, also allocation-free and with no
 * reference counterpart: synchronises `stream`, then reads and clears the
 * current device's error word into *flag (MDLC_DEVERR_* of the first
 * device-side error any call on this device recorded since the last status
 * call, or MDLC_DEVERR_NONE). */
int mdlc_conv2d_splitk_noalloc_status(void* stream, int* flag, char* msg, size_t msg_len);

/* Depthwise convolution (groups == c == k): the entry point of
 * mdlc_conv2d's depthwise path with the shape checked. Replaces the grouped
 * conv host fallback (emit.py:175-180, ops.py:68-78). Weights packed by
 * mdlc_pack_conv_weights. */
int mdlc_dwconv2d(mdlc_ctx* ctx, const mdlc_conv_desc* desc, const void* x, const void* w_packed,
                  const void* bias, const void* residual, void* y, const mdlc_epilogue* epi);

/* GEMM y[m, n] = act(a[m, k] . op(b) + bias) on the convolution kernels (a
 * 1x1 convolution over m one-pixel images). Replaces the Gemm / MatMul
 * lowering (emit.py:211-244, ops.py:84-92). a is row-major with row stride lda
 * elements (>= k; a multiple of 8, or 16 for 8-bit types); y is row-major with
 * row stride round_up(n, 8) (16 for 8-bit outputs), pad columns written as 0.
 * op(b) = b^T when trans_b (b stored [n, k], ONNX transB = 1, the FC layout),
 * else b ([k, n]); alpha is folded into the packed weights by
 * mdlc_pack_gemm_weights and beta into bias by the caller (bias: n floats, or
 * int32 for 8-bit types). trans_a = 1 is rejected (MDLC_ERR_UNSUPPORTED). */
typedef struct {
  int32_t m, n, k;
  int32_t lda;
  int32_t trans_a, trans_b;
  float alpha;
  int32_t in_type, out_type;
} mdlc_gemm_desc;
int mdlc_gemm_weight_bytes(const mdlc_gemm_desc* desc, size_t* bytes);
int mdlc_pack_gemm_weights(const mdlc_gemm_desc* desc, const float* host_b, void* host_out); /* host-only */
int mdlc_gemm(mdlc_ctx* ctx, const mdlc_gemm_desc* desc, const void* a, const void* b_packed, const void* bias,
              void* y, const mdlc_epilogue* epi, const mdlc_tile_cfg* cfg);

/* Replaces the MaxPool / AveragePool / GlobalAveragePool host fallbacks
 * (emit.py:32-35, ops.py:109-150). */
int mdlc_pool2d(mdlc_ctx* ctx, const mdlc_pool_desc* desc, const void* x, void* y);
/* Replaces the generated elementwise kernel (emit.py:246-278, templates.py:209-269). */
int mdlc_eltwise(mdlc_ctx* ctx, const mdlc_ew_prog* prog, const void* const* inputs,
                 void* const* outputs);

/* Graph-boundary layout conversion (the reference stages feeds and reads
 * outputs as NCHW fp32, gpu_executor.py:48-55,94). to_nhwc converts an NCHW
 * fp32 tensor to NHWC with channel stride cs (pad channels zeroed) in dtype;
 * for 8-bit dtypes q = clamp(rint(x * inv_scale) + zp). to_nchw is the
 * inverse (8-bit: x = (q - zp) * scale, with scale = 1 / inv_scale given). */
int mdlc_nchw_to_nhwc(mdlc_ctx* ctx, const float* x, int n, int c, int h, int w, void* y, int cs,
                      int dtype, float inv_scale, int zp);
int mdlc_nhwc_to_nchw(mdlc_ctx* ctx, const void* x, int n, int c, int h, int w, int cs, int dtype,
                      float* y, float scale, int zp);
/* NCHW fp32 (h, w even) -> 2x2 space-to-depth NHWC: y[n][Y][X][(dy*2+dx)*c + ci]
 * = x[n][ci][2Y+dy][2X+dx], channel stride cs >= 4c (pad channels zeroed); 8-bit
 * dtypes quantise like mdlc_nchw_to_nhwc.
 * Feeds a stride-2 stem conv rewritten as a stride-1 conv (no reference
 * counterpart: a layout choice of this backend). */
int mdlc_nchw_to_s2d(mdlc_ctx* ctx, const float* x, int n, int c, int h, int w, void* y, int cs, int dtype,
                     float inv_scale, int zp);

/* Data-movement ops over NHWC tensors addressed by their logical 4-D index
 * (n, c, h, w) (rank-2 [n, c] and rank-3 [n, c, h] tensors use h = w = 1 / w = 1).
 * Replaces the Transpose / Concat / Pad host bounces of the reference GPU
 * executor (mdlc/codegen/cuda/emit.py:32-35; semantics mdlc/runtime/ops.py:229-255).
 * Gather (mode 0): every output element, padding channels included, reads the
 * source element whose index along source dimension src_dim[i] is
 * out_index[i] - offset[i]; an index outside the source is filled per
 * pad_mode: 0 constant (value), 1 edge (clamped), 2 reflect (no edge repeat).
 * Scatter (mode 1): every source element is written to the output element at
 * index + offset (src_dim must be the identity); other output elements are
 * left as they are. Transpose = gather with src_dim = the inverse permutation;
 * Pad = gather with offset = the leading pads; Concat = gather of the first
 * input (zero fill) then a scatter of each other input at its offset. */
typedef struct {
  int32_t dtype;        /* MDLC_F32 | MDLC_BF16 */
  int32_t in_dims[4];   /* logical n, c, h, w of the source */
  int32_t in_cs;        /* source channel stride */
  int32_t out_dims[4];
  int32_t out_cs;
  int32_t src_dim[4];
  int32_t offset[4];
  int32_t mode, pad_mode;
  float value;
} mdlc_copy_desc;
int mdlc_copy4d(mdlc_ctx* ctx, const mdlc_copy_desc* desc, const void* x, void* y);

/* Softmax along one logical axis (0..3 of n, c, h, w) of an NHWC tensor:
 * y = exp(x - max) / sum(exp(x - max)) over that axis, fp32 arithmetic.
 * Replaces the Softmax host bounce (reference ops.py:188-191). */
typedef struct {
  int32_t dtype;   /* MDLC_F32 | MDLC_BF16 */
  int32_t dims[4]; /* logical n, c, h, w */
  int32_t cs;      /* channel stride of x and y */
  int32_t axis;
} mdlc_softmax_desc;
int mdlc_softmax(mdlc_ctx* ctx, const mdlc_softmax_desc* desc, const void* x, void* y);

/* Squeeze-excite gate: a global average pool and the two 1x1 convolutions on
 * the 1x1 map that follow it (FC, act, FC, act), which the reference runs as a
 * GlobalAveragePool (runtime/reference.py:134) and two FusedConvAct GEMM
 * launches (emit.py:159-209), in one kernel:
 *   p[n, i] = mean over the hw pixels of x[n, :, i]          (hw > 1)
 *   h[n, j] = act1(b1[j] + sum_i w1[j, i] * p[n, i])       j < rd
 *   s[n, i] = act2(b2[i] + sum_j w2t[j, i] * h[n, j])      i < c
 * With hw 0 or 1 the input is the pooled p, [n][c_stride]; with hw > 1 it is
 * the NHWC activation x, [n][hw][c_stride] (16-byte aligned), averaged in fp32
 * (kept in fp32, not rounded to dtype). s: [n][c_stride] in dtype (bf16 or
 * fp32; the padding channels are written as zero); w1, w2t: [rd][c] fp32 (w2t
 * is the second conv's [c][rd] weight transposed); b1 [rd], b2 [c] fp32 or
 * null. fp32 accumulation, h kept in fp32. c <= c_stride <= 4096, rd <= 1024. */
typedef struct {
  int32_t n, c, c_stride, rd;
  int32_t dtype;                  /* MDLC_BF16 or MDLC_F32 */
  int32_t act1, act2;             /* MDLC_ACT_* */
  float alpha1, beta1, lo1, hi1;  /* act1 parameters (leaky / hard-sigmoid / clip) */
  float alpha2, beta2, lo2, hi2;  /* act2 parameters */
  int32_t hw;                     /* pixels per image of the input: 0 / 1 pooled, > 1 pool fused */
} mdlc_se_desc;
int mdlc_se_fc(mdlc_ctx* ctx, const mdlc_se_desc* desc, const void* pooled, const float* w1, const float* b1,
               const float* w2t, const float* b2, void* gate);

/* ---- CUDA graph capture of a whole run (b=1 latency) ------------------- */
int mdlc_graph_begin(mdlc_ctx* ctx);
int mdlc_graph_end(mdlc_ctx* ctx);    /* instantiates the captured graph */
int mdlc_graph_launch(mdlc_ctx* ctx);
int mdlc_graph_reset(mdlc_ctx* ctx);

/* ---- timing on the context stream (replaces nvrtc_runtime.py:211-225) -- */
int mdlc_event_record(mdlc_ctx* ctx, int slot); /* slot in [0, 4096), on the compute stream */
int mdlc_event_record_on(mdlc_ctx* ctx, int slot, int stream);
int mdlc_event_elapsed(mdlc_ctx* ctx, int start_slot, int stop_slot, float* ms);
/* number of kernels this context has launched (including graph replays) */
int mdlc_launch_count(mdlc_ctx* ctx, long long* count);

/* ---- fault handling self-test ----------------------------------------- */
/* Launches a one-thread kernel that waits on an mbarrier nothing will ever
 * complete, with the given time limit in microseconds; the wait gives up, the
 * kernel records MDLC_DEVERR_WAIT_TIMEOUT in the error word and returns. Used
 * to test the bounded-wait path without faulting or hanging the GPU. */
int mdlc_debug_timeout_probe(mdlc_ctx* ctx, int limit_us);
/* Fills the context's split-K arrival counters with the byte `value` (on the
 * stream), reproducing the state a split-K call that gave up on a bounded wait
 * leaves behind, so tests can check that the next split-K call is unaffected. */
int mdlc_debug_poison_split_counters(mdlc_ctx* ctx, int value);

#ifdef __cplusplus
}
#endif
#endif /* MDLC_B200_H */
