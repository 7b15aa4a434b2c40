// Inline-PTX helpers for sm_100a: mbarriers, TMA (cp.async.bulk.tensor into this CTA's shared memory),
// tcgen05 (TMEM alloc, MMA, commit, ld) and shared-memory matrix descriptors.
//
// Every wait on an mbarrier is bounded: after kSpinLimit polls it records an error
// code in the library's device error word and reports failure to the caller, which
// then skips the rest of its work, frees TMEM and returns.  No kernel in this library
// spins without a limit.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace svla {

// error codes written to the device error word (first nonzero wins)
enum DeviceError : int {
  kErrNone = 0,
  kErrMbarTimeout = 101,   // an mbarrier wait ran out of polls
  kErrBadShape = 102,      // a kernel saw a shape its launcher should have rejected
};

constexpr uint32_t kSpinLimit = 1u << 22;  // ~4M polls of try_wait (each may block ~1 µs): seconds, then error

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

// ------------------------------------------------------------------ programmatic dependent launch
// Kernels are launched with programmatic stream serialisation: a kernel may start while the previous one
// in the stream is still running.  Every kernel calls pdl_wait() before it reads anything an earlier
// kernel wrote or writes anything an earlier kernel may still read (pdl_wait returns once the previous
// grid has completed and its memory is visible), and only then pdl_trigger(), so that when a kernel
// starts, every kernel before its immediate predecessor has completed.  Without the launch attribute
// both are no-ops.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false (and
// records kErrMbarTimeout) when the poll budget runs out.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
  }
  record_error(err, kErrMbarTimeout);
  return false;
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3-D tile (x = column, y = row, z = batch); rows past the tensor's extent read as zeros
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
          "r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// 4-D tile (x, y, z, w); coordinates past the tensor's extent read as zeros
__device__ __forceinline__ void tma_load_4d(void* smem_dst, const CUtensorMap* map, uint64_t* bar, int x, int y,
                                            int z, int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// generic-proxy writes to shared memory -> visible to the async proxy (tensor core / TMA)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::i8 (s8 x s8 -> s32)
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 x bf16 -> f32)
__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// all prior tcgen05.mma of this thread -> one arrive on the mbarrier when they complete
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns -> 16 registers per thread
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 bit, 32 consecutive columns -> 32 registers per thread
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// registers -> 32 lanes x 32 bit, 16 consecutive columns
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[tmem] * B[smem], kind::f16 with the A operand (K-major, M rows = TMEM lanes, two bf16 per
// 32-bit column) read from tensor memory; no output lanes disabled
__device__ __forceinline__ void mma_bf16_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0u)
      : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle (8-row x 128-byte atoms, atoms stacked every 1024 bytes along M/N).
//   bits  0-13 start address >> 4      bits 16-29 leading byte offset >> 4 (unused here: 1)
//   bits 32-45 stride byte offset >> 4 (1024 B between 8-row groups)
//   bits 46-47 descriptor version (1 on sm_100)   bits 61-63 layout (2 = 128B swizzle)
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFF) >> 4);
  d |= static_cast<uint64_t>(1) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// The same descriptor with a leading byte offset: for an MN-major operand, the distance between successive
// 64-element (128-byte) blocks along M/N, each an 8-row x 128-byte atom stack like the first.
__device__ __forceinline__ uint64_t smem_desc_sw128_lbo(uint32_t saddr, uint32_t lbo_bytes) {
  return (smem_desc_sw128(saddr) & ~(static_cast<uint64_t>(0x3FFF) << 16)) |
         (static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFF) << 16);
}

// Instruction descriptors (cta_group::1, both operands K-major, dense).
//   bits 4-5 D format (1 = f32, 2 = s32)   bits 7-9 / 10-12 A / B format
//   bits 17-22 N >> 3                       bits 24-28 M >> 4
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ bool elect_lane0() { return (threadIdx.x & 31) == 0; }

// ------------------------------------------------------------------ CTA pairs (tcgen05 cta_group::2)
// Two CTAs of a cluster of two share one MMA: the even CTA issues tcgen05.mma with M = 256, whose A rows
// 0..127 come from its own shared memory and 128..255 from its peer's, and whose B (N columns) is split
// in halves between them; each CTA's TMEM receives its own 128 rows of the accumulator.  Only plain
// (non-multicast) TMA loads are used: each CTA loads its own operand tiles.
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// all threads of both CTAs; release / acquire orders shared-memory writes (barrier initialisation) across them
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// address of the same shared-memory offset in CTA `rank` of the cluster (shared::cluster window)
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// arrive on an mbarrier of a CTA of the cluster (release at cluster scope)
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// TMA tile load into this CTA's shared memory whose completion counts on an mbarrier that may be in the peer
// CTA of the pair (cluster address); no multicast
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, uint32_t bar_cluster_addr,
                                                 int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
      : "memory");
}
// TMEM allocation for a CTA pair: issued by the same warp in both CTAs, same slot offset
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void mma_i8_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// all prior pair MMAs of this thread -> one arrive on an mbarrier of either CTA (cluster address)
__device__ __forceinline__ void mma_commit_pair(uint32_t bar_cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar_cluster_addr)
               : "memory");
}

// ------------------------------------------------------------------ numeric helpers
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
// two fp32 values rounded to bf16 (RN) and packed: lo in the low half
__device__ __forceinline__ uint32_t pack_bf16_rn(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The same rounding with integer operations only (for loops where the conversion unit is the bottleneck):
// round-to-nearest-even of a finite fp32 to bf16, as the fp32 bit pattern with the low 16 bits clear.
__device__ __forceinline__ uint32_t bf16_rn_bits(float x) {
  const uint32_t u = __float_as_uint(x);
  return (u + 0x7FFFu + ((u >> 16) & 1u)) & 0xFFFF0000u;
}
// exact int32 -> fp32 for |i| < 2^22 without a conversion instruction: 0x4B400000 is 1.5 * 2^23, where
// the fp32 spacing is exactly 1
__device__ __forceinline__ float small_int_to_f32(int i) { return __int_as_float(0x4B400000 + i) - 12582912.0f; }

// Round-half-even of |y| < 2^22 to an integer with one fp32 add (the sum lands where the spacing is 1).
__device__ __forceinline__ int round_rn_small(float y, float& r) {
  const float t = __fadd_rn(y, 12582912.0f);
  r = __fsub_rn(t, 12582912.0f);
  return __float_as_int(t) - 0x4B400000;
}

// round-half-even then clamp, the torch.round(..).clamp(lo, hi) rule
__device__ __forceinline__ int quant_rn_clamp(float v, int lo, int hi) {
  float r = rintf(v);
  r = fminf(fmaxf(r, static_cast<float>(lo)), static_cast<float>(hi));
  return static_cast<int>(r);
}

// SmoothQuant activation quantize: round((x / s) / a).clamp(-128, 127) with two IEEE divides
__device__ __forceinline__ int8_t smooth_quant(float x, float s, float a) {
  return static_cast<int8_t>(quant_rn_clamp(__fdiv_rn(__fdiv_rn(x, s), a), -128, 127));
}
// the same, kept out of line: the rare fallback of smooth_quant_fast (one copy instead of one per element)
__device__ __noinline__ int smooth_quant_slow(float x, float s, float a) { return smooth_quant(x, s, a); }

// The same result as smooth_quant, cheaper: y = (x * rs) * ra with rs = 1/s, ra = 1/a (correctly rounded
// reciprocals) differs from fl(fl(x / s) / a) by at most 6 * 2^-24 * |y| (< 1e-4 for |y| < 256).  Away
// from a rounding boundary (fraction more than 2^-12 from .5) and inside |y| < 256, round(y) therefore
// equals the two-divide result; beyond 256 both clamp to the same end.  Everything else -- values within
// 2^-12 of a .5 boundary, NaN, infinities -- takes the exact two-divide path.
__device__ __forceinline__ int8_t smooth_quant_fast(float x, float s, float rs, float a, float ra) {
  const float y = __fmul_rn(__fmul_rn(x, rs), ra);
  const float ay = fabsf(y);
  if (ay < 256.0f) {
    float r;
    const int i = round_rn_small(y, r);
    if (fabsf(__fsub_rn(y, r)) <= 0.5f - 0.000244140625f) return static_cast<int8_t>(i < -128 ? -128 : (i > 127 ? 127 : i));
  } else if (ay < 3.0e38f) {
    return static_cast<int8_t>(y > 0.0f ? 127 : -128);
  }
  return static_cast<int8_t>(smooth_quant_slow(x, s, a));
}

// Branch-free form of smooth_quant_fast for four values, packed as four int8 bytes (x[0] in the low byte).
// y is clamped to [-128, 127] before rounding -- the same result as rounding first and clamping after
// (a NaN also lands on -128, as in smooth_quant) -- then rounded with one add: t = y + 1.5 * 2^23 holds
// round(y) in its low mantissa bits, so the low byte of t's bit pattern is the int8 two's complement.
// The fast y differs from the two-divide y by at most 6 * 2^-24 * 128.5 < 4.6e-5 inside the clamp range,
// so only values within 2^-12 (5x that) of a .5 boundary can round differently: bit e of the returned
// `slow` mask (bit 4k+e of the caller's group) marks those, and the caller recomputes them with smooth_quant.
__device__ __forceinline__ uint32_t smooth_quant4_fast(const float* x, float4 rs, float ra, uint32_t& slow, int bit0) {
  // Pairs through the packed fp32 pipe (FMUL2 / FADD2 / FFMA2): each lane of a packed op is the IEEE
  // round-to-nearest result of the scalar op, so y, t and the fraction are bit-identical to the scalar form
  // fmin(fmax((x * rs) * ra)), t = y + C, y - (t - C); t - C is written t + (-C) and y - r as fma(r, -1, y),
  // both exactly the same roundings.
  constexpr float kC = 12582912.0f;
  const float2 ra2 = make_float2(ra, ra);
  float2 y[2] = {__fmul2_rn(__fmul2_rn(make_float2(x[0], x[1]), make_float2(rs.x, rs.y)), ra2),
                 __fmul2_rn(__fmul2_rn(make_float2(x[2], x[3]), make_float2(rs.z, rs.w)), ra2)};
  uint32_t b[4];
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    y[h].x = fminf(fmaxf(y[h].x, -128.0f), 127.0f);
    y[h].y = fminf(fmaxf(y[h].y, -128.0f), 127.0f);
    const float2 t = __fadd2_rn(y[h], make_float2(kC, kC));
    const float2 f = __ffma2_rn(__fadd2_rn(t, make_float2(-kC, -kC)), make_float2(-1.0f, -1.0f), y[h]);
    if (fabsf(f.x) > 0.5f - 0.000244140625f) slow |= 1u << (bit0 + 2 * h);
    if (fabsf(f.y) > 0.5f - 0.000244140625f) slow |= 1u << (bit0 + 2 * h + 1);
    b[2 * h] = __float_as_uint(t.x);
    b[2 * h + 1] = __float_as_uint(t.y);
  }
  return __byte_perm(__byte_perm(b[0], b[1], 0x0040), __byte_perm(b[2], b[3], 0x0040), 0x5410);
}

// Hardware approximations (PTX ex2.approx / rcp.approx, flush-to-zero): 2^x and 1/x with relative
// errors around 2^-22, far below the bf16 rounding that follows every use here.
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Round two fp32 values to bf16 (RN) and return them as fp32: one packed conversion for both.
__device__ __forceinline__ void bf16_round2(float& a, float& b) {
  const uint32_t p = pack_bf16_rn(a, b);
  a = __uint_as_float(p << 16);
  b = __uint_as_float(p & 0xFFFF0000u);
}

}  // namespace svla
