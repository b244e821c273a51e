// Device-side helpers shared by the sm_100a kernels: inline PTX wrappers for
// mbarriers, cp.async, TMA tile loads and tcgen05 (TMEM alloc, UMMA issue,
// commit, TMEM->register loads), bounded waits, activation math and bf16
// packing. Written against the PTX ISA for sm_100a; no CUTLASS types.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "mdlc_b200.h"

#define MDLC_DEV __device__ __forceinline__

namespace mdlc {

// ------------------------------------------------------------ programmatic dependent launch
// A kernel started by launch_pdl may begin while the previous kernel in the
// stream is still running (its launch and prologue overlap that kernel's
// tail). It must call pdl_wait() before its first global-memory access: the
// wait returns once the previous grid has completed and its writes are
// visible (in a kernel launched the ordinary way it returns at once).
// pdl_trigger() then lets the next kernel in the stream be scheduled; it
// starts only after every CTA of this grid has triggered or exited.
MDLC_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MDLC_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t stream,
                              Args... args) {
  cudaLaunchConfig_t lc = {};
  lc.gridDim = grid;
  lc.blockDim = block;
  lc.dynamicSmemBytes = smem;
  lc.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  lc.attrs = attr;
  lc.numAttrs = 1;
  return cudaLaunchKernelEx(&lc, kern, args...);
}

// ------------------------------------------------------------ error word
// Each context owns one int in device memory; kernels record the first
// device-side failure with atomicCAS so the first cause is kept.
MDLC_DEV void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// Bounds checks of computed global-memory indices, compiled in only by the
// checked build (-DMDLC_CHECK, libmdlc_b200_check.so): an index outside
// [0, extent) records MDLC_DEVERR_BOUNDS in the error word and the access is
// skipped; nothing traps. In the normal build the check is the constant true.
#ifdef MDLC_CHECK
#define MDLC_CHECK_IDX(err, idx, extent) \
  (((unsigned long long)(idx) < (unsigned long long)(extent)) ? true \
                                                              : (mdlc::record_error((err), MDLC_DEVERR_BOUNDS), false))
#else
#define MDLC_CHECK_IDX(err, idx, extent) true
#endif

MDLC_DEV uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
  return t;
}

MDLC_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------ mbarrier
MDLC_DEV void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
MDLC_DEV void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
MDLC_DEV void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
MDLC_DEV void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
MDLC_DEV bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(1000000u)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete. Gives up when
// another role of the CTA has already given up (*abort != 0) or after
// limit_cycles SM clock cycles (clock64, cheap to read; the library passes 2x
// the nanosecond limit, i.e. at least the limit at any clock up to 2 GHz); on
// time-out it records MDLC_DEVERR_WAIT_TIMEOUT and raises *abort. Returns true
// when the phase completed.
MDLC_DEV bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err,
                        uint64_t limit_cycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 3u) == 0) {
      if (abort && *abort) return false;
      if ((unsigned long long)(clock64() - t0) > limit_cycles) {
        record_error(err, MDLC_DEVERR_WAIT_TIMEOUT);
        if (abort) *abort = 1;
        return false;
      }
    }
  }
}

MDLC_DEV void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------ cp.async
// 16-byte global->shared copy; src_bytes < 16 zero-fills the remainder
// (src_bytes == 0 reads nothing and writes 16 zero bytes).
MDLC_DEV void cp_async_16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src),
               "r"(src_bytes)
               : "memory");
}
MDLC_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
MDLC_DEV void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
MDLC_DEV void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// Arrive on the mbarrier once every cp.async this thread issued so far has
// landed; .noinc: the arrival counts against the barrier's expected count.
MDLC_DEV void cp_async_mbar_arrive_noinc(uint32_t bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar) : "memory");
}

// ------------------------------------------------------------ TMA
MDLC_DEV void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(tmap)) : "memory");
}
// 2-D tiled load into this CTA's shared memory, completing on an mbarrier transaction count.
MDLC_DEV void tma_load_2d(uint32_t dst, const void* tmap, int32_t x, int32_t y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(x), "r"(y)
      : "memory");
}

// 3-D tiled load into this CTA's shared memory.
MDLC_DEV void tma_load_3d(uint32_t dst, const void* tmap, int32_t x, int32_t y, int32_t z, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 4-D im2col-mode load (NHWC tensor map): 128 consecutive output pixels
// starting at spatial coordinate (w, h) of image n, channels [c, c + box), with
// the filter-tap offsets (off_w, off_h) added; padding reads as zero.
MDLC_DEV void tma_load_im2col_4d(uint32_t dst, const void* tmap, int32_t c, int32_t w, int32_t h, int32_t n,
                                 uint16_t off_w, uint16_t off_h, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.im2col.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2], {%7, %8};" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c), "r"(w), "r"(h), "r"(n), "h"(off_w), "h"(off_h)
      : "memory");
}

// 4-D tiled load into this CTA's shared memory; coordinates may be negative or past the end
// (those elements read as zero).
MDLC_DEV void tma_load_4d(uint32_t dst, const void* tmap, int32_t c0, int32_t c1, int32_t c2, int32_t c3,
                          uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(tmap)), "r"(bar), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// 4-D tiled store shared -> global; box elements past the end of the tensor
// are not written (coordinates must be non-negative).
MDLC_DEV void tma_store_4d(const void* tmap, int32_t c0, int32_t c1, int32_t c2, int32_t c3, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}

// 2-D tiled store shared -> global (bulk-group completion); out-of-range rows
// and columns of the box are not written.
MDLC_DEV void tma_store_2d(const void* tmap, int32_t x, int32_t y, uint32_t src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(tmap)),
               "r"(src), "r"(x), "r"(y)
               : "memory");
}
MDLC_DEV void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// wait until at most N committed bulk groups still read their shared source
template <int N>
MDLC_DEV void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
template <int N>
MDLC_DEV void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// ------------------------------------------------------------ tcgen05
MDLC_DEV void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
MDLC_DEV void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MDLC_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
MDLC_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MDLC_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// Shared-memory matrix descriptor for a K-major operand stored in 128-byte
// swizzled rows: 8-row groups 1024 bytes apart (SBO), LBO unused (1),
// descriptor version 1 (sm_100), layout type 2 = SWIZZLE_128B.
MDLC_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
         ((uint64_t)(1024 >> 4) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// 128-byte swizzled K-major operand whose 8-row groups are sbo_bytes apart
// (a multiple of 1024, so every group starts at the same swizzle phase). The
// start may sit at any 128-byte row inside the swizzle atom: the swizzle is a
// function of the shared-memory address bits, which the tensor memory
// accelerator used when it wrote the rows.
MDLC_DEV uint64_t umma_desc_sw128_sbo(uint32_t saddr, uint32_t sbo_bytes) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

// Same for the narrower K-major swizzles: layout 6 = SWIZZLE_32B (8 rows x
// 32 bytes per atom, SBO 256), layout 4 = SWIZZLE_64B (8 x 64 bytes, SBO 512).
MDLC_DEV uint64_t umma_desc_k(uint32_t saddr, uint32_t sbo_bytes, uint32_t layout) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) |
         ((uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32) | ((uint64_t)1 << 46) | ((uint64_t)layout << 61);
}

// Instruction descriptor, kind::f16 with bf16 operands and fp32 accumulator.
__host__ __device__ constexpr uint32_t idesc_bf16(int M, int N) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}
// Instruction descriptor, kind::tf32 (A and B tf32, format 2; fp32 accumulator).
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
// Instruction descriptor, kind::i8 with int32 accumulator; a_signed/b_signed
// select s8 (1) or u8 (0) operands.
__host__ __device__ constexpr uint32_t idesc_i8(int M, int N, int a_signed, int b_signed) {
  return (2u << 4) | ((uint32_t)a_signed << 7) | ((uint32_t)b_signed << 10) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

MDLC_DEV void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
MDLC_DEV void umma_i8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                      uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
MDLC_DEV void umma_tf32(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on an mbarrier once all previously issued tcgen05 async operations
// of this thread have completed.
MDLC_DEV void umma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32-bit, 16 consecutive columns per thread.
MDLC_DEV void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}
MDLC_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 32-bit, 16 consecutive columns per thread, registers -> TMEM.
MDLC_DEV void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]),
      "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
MDLC_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------ activations
struct ActParams {
  int act;
  float alpha, beta, lo, hi;
};

MDLC_DEV float apply_act(float v, const ActParams& p);

// Paired fp32 arithmetic (mul / fma .rn.f32x2: two IEEE
// round-to-nearest operations in one instruction) on float2 values kept in
// 64-bit register pairs.
MDLC_DEV unsigned long long f2_bits(const float2 v) { return *reinterpret_cast<const unsigned long long*>(&v); }
MDLC_DEV float2 f2_from(unsigned long long b) { return *reinterpret_cast<float2*>(&b); }
MDLC_DEV float2 fmul2(const float2 a, const float2 b) {
  unsigned long long d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_from(d);
}
// a * b + c
MDLC_DEV float2 fma2(const float2 a, const float2 b, const float2 c) {
  unsigned long long d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_from(d);
}
// d += a * b
MDLC_DEV void ffma2(float2& d, const float2 a, const float2 b) { d = fma2(a, b, d); }
MDLC_DEV float2 splat2(float v) { return make_float2(v, v); }

// GELU(x) = x * Phi(x) = 0.5 x (1 + erf(x / sqrt 2)), branch-free so the
// independent elements of an epilogue chunk interleave (erff branches on |x|,
// which left the epilogue one latency chain at a time). erfc(z), z >= 0, is the
// Chebyshev-fitted erfcc of Numerical Recipes (Press et al., 2nd ed., sec. 6.2:
// erfc(z) ~ t exp(-z^2 + P(t)), t = 1 / (1 + z / 2), fractional error < 1.2e-7);
// then 1 + erf(z) = 2 - erfc(z) for x >= 0 and erfc(|z|) for x < 0.
MDLC_DEV float gelu_f(float x) {
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = __fdividef(1.0f, fmaf(0.5f, z, 1.0f));
  float p = fmaf(t, 0.17087277f, -0.82215223f);
  p = fmaf(t, p, 1.48851587f);
  p = fmaf(t, p, -1.13520398f);
  p = fmaf(t, p, 0.27886807f);
  p = fmaf(t, p, -0.18628806f);
  p = fmaf(t, p, 0.09678418f);
  p = fmaf(t, p, 0.37409196f);
  p = fmaf(t, p, 1.00002368f);
  p = fmaf(t, p, -1.26551223f);
  const float e = t * __expf(fmaf(-z, z, p));
  return 0.5f * x * (x >= 0.0f ? 2.0f - e : e);
}

// Eight elements at once, each stage of the formula applied to all eight
// before the next, so the eight dependency chains interleave (one epilogue
// warp per scheduler has no other warps to hide their latency).
MDLC_DEV void gelu8(float (&x)[8]) {
  // the same evaluation as gelu_f, two elements per instruction where the
  // operation pairs (f32x2 multiply / fma), scalar for reciprocal and exp2
  constexpr float kC[10] = {0.17087277f, -0.82215223f, 1.48851587f, -1.13520398f, 0.27886807f,
                            -0.18628806f, 0.09678418f, 0.37409196f, 1.00002368f, -1.26551223f};
  float2 z[4], t[4], p[4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
    z[i] = fmul2(make_float2(fabsf(x[2 * i]), fabsf(x[2 * i + 1])), splat2(0.70710678118654752f));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 d = fma2(splat2(0.5f), z[i], splat2(1.0f));
    t[i] = make_float2(__fdividef(1.0f, d.x), __fdividef(1.0f, d.y));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) p[i] = fma2(t[i], splat2(kC[0]), splat2(kC[1]));
#pragma unroll
  for (int c = 2; c < 10; ++c)
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = fma2(t[i], p[i], splat2(kC[c]));
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // t * exp(p - z^2), exp(v) = 2^(v log2 e)
    const float2 v = fmul2(fma2(fmul2(z[i], splat2(-1.0f)), z[i], p[i]), splat2(1.4426950408889634f));
    float e0, e1;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e0) : "f"(v.x));
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e1) : "f"(v.y));
    p[i] = fmul2(t[i], make_float2(e0, e1));
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    // 1 + erf(x / sqrt 2) = 2 - erfc for x >= 0, erfc(|z|) for x < 0
    const float2 q2 = fma2(p[i], splat2(-1.0f), splat2(2.0f));
    const float2 q = make_float2(x[2 * i] >= 0.0f ? q2.x : p[i].x, x[2 * i + 1] >= 0.0f ? q2.y : p[i].y);
    const float2 r = fmul2(fmul2(make_float2(x[2 * i], x[2 * i + 1]), splat2(0.5f)), q);
    x[2 * i] = r.x;
    x[2 * i + 1] = r.y;
  }
}
MDLC_DEV void sigmoid8(float (&x)[8]) {
  float e[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = __expf(-x[i]);
#pragma unroll
  for (int i = 0; i < 8; ++i) x[i] = __fdividef(1.0f, 1.0f + e[i]);
}

// Activation fixed at compile time (ACT >= 0) or chosen at run time (ACT == -1).
// Fixing it keeps the unrolled epilogue small: every inlined copy of the
// run-time switch carries the exp/tanh/erf paths.
template <int ACT>
MDLC_DEV float act_fn(float v, const ActParams& p) {
  if constexpr (ACT == -1) return apply_act(v, p);
  else if constexpr (ACT == MDLC_ACT_NONE) return v;
  else if constexpr (ACT == MDLC_ACT_RELU) return fmaxf(v, 0.0f);
  else if constexpr (ACT == MDLC_ACT_CLIP) return fminf(fmaxf(v, p.lo), p.hi);
  else if constexpr (ACT == MDLC_ACT_GELU) return gelu_f(v);
  else if constexpr (ACT == MDLC_ACT_SIGMOID) return 1.0f / (1.0f + expf(-v));
  else return apply_act(v, p);
}

MDLC_DEV float apply_act(float v, const ActParams& p) {
  switch (p.act) {
    case MDLC_ACT_RELU: return fmaxf(v, 0.0f);
    case MDLC_ACT_CLIP: return fminf(fmaxf(v, p.lo), p.hi);
    case MDLC_ACT_SIGMOID: return 1.0f / (1.0f + expf(-v));
    case MDLC_ACT_TANH: return tanhf(v);
    case MDLC_ACT_LEAKY_RELU: return v >= 0.0f ? v : p.alpha * v;
    case MDLC_ACT_HARD_SIGMOID: return fminf(fmaxf(p.alpha * v + p.beta, 0.0f), 1.0f);
    case MDLC_ACT_HARD_SWISH: return v * fminf(fmaxf(v / 6.0f + 0.5f, 0.0f), 1.0f);
    case MDLC_ACT_GELU: return gelu_f(v);
    default: return v;
  }
}

// ------------------------------------------------------------ bf16 packing
MDLC_DEV uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}
MDLC_DEV float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
// Clamp both halves of a bf16 pair to [lo, hi] (given as bf16 pairs). With
// bounds exact in bf16, clamping after rounding to bf16 equals rounding after
// clamping in fp32 (rounding is monotonic); NaN becomes lo, as with
// fminf(fmaxf(x, lo), hi).
MDLC_DEV uint32_t clamp_bf16x2(uint32_t v, uint32_t lo2, uint32_t hi2) {
  asm("max.bf16x2 %0, %0, %1;" : "+r"(v) : "r"(lo2));
  asm("min.bf16x2 %0, %0, %1;" : "+r"(v) : "r"(hi2));
  return v;
}
MDLC_DEV float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

// ------------------------------------------------------------ int8 requant
// gemmlowp / TFLite fixed point: SaturatingRoundingDoublingHighMul followed
// by RoundingDivideByPOT (round half away from zero).
MDLC_DEV int32_t sat_rdh_mul(int32_t a, int32_t b) {
  if (a == INT32_MIN && b == INT32_MIN) return INT32_MAX;
  const long long ab = (long long)a * (long long)b;
  const long long nudge = ab >= 0 ? (1ll << 30) : (1 - (1ll << 30));
  return (int32_t)((ab + nudge) / (1ll << 31));
}
MDLC_DEV int32_t rounding_rshift(int32_t x, int shift) {
  if (shift <= 0) return x;
  const int32_t mask = (int32_t)((1ll << shift) - 1);
  const int32_t rem = x & mask;
  const int32_t threshold = (mask >> 1) + (x < 0 ? 1 : 0);
  return (x >> shift) + (rem > threshold ? 1 : 0);
}
// MultiplyByQuantizedMultiplier: shift > 0 right-shifts after the high
// multiply; shift < 0 left-shifts the input first (saturated to int32).
MDLC_DEV int32_t requant(int32_t acc, int32_t mult, int32_t shift) {
  if (shift < 0) {
    long long v = (long long)acc << (-shift);
    v = v > INT32_MAX ? INT32_MAX : (v < INT32_MIN ? INT32_MIN : v);
    return sat_rdh_mul((int32_t)v, mult);
  }
  return rounding_rshift(sat_rdh_mul(acc, mult), shift);
}

}  // namespace mdlc
