// The action expert's flow-matching loop as ONE persistent kernel, for calls with at most 64 action rows
// (batch x chunk; batch 1 at chunk 50).  lerobot VLAFlowMatching.sample_actions / denoise_step:
//   x_t = noise;  for step: v = expert(x_t, t_step, prefix KV);  x_t += dt * v      (dt = -1 / num_steps)
// with, per step, action_in_proj, the time MLP (SiLU), 16 expert layers (RMSNorm, q/k/v + RoPE, attention
// over the cached prefix K/V [+ the chunk's own K/V on self-attention layers], o_proj + residual, RMSNorm,
// SiLU-gated MLP, down_proj + residual), the final RMSNorm and action_out_proj.
//
// At these sizes every launch of the per-layer kernels is latency-bound (a few CTAs, short K loops); here
// the ~84 phases of one step run back to back inside one cooperative grid (one CTA per SM), separated by
// grid barriers, so a phase costs a barrier instead of a kernel launch with its prologue and drain.
//
// Phases are GEMMs of row blocks (32 rows; 64 for gate/up) against 16-column slices of a weight (a task = a
// slice x a row block, tasks spread over the CTAs; the 8 warps of a CTA split K and add their partial tiles in
// a fixed order), mma.sync m16n8k16 bf16 with fp32 accumulators, the A rows staged in shared memory by bulk
// copies (RMSNorm applied there with the stand-alone norm kernel's arithmetic and operation order), weights
// read straight from global memory in MMA fragment order (pack_fragments_kernel): one k16 step of a 16-column
// slice is 32 lanes x 8 elements, so a warp's load is one contiguous 256-byte (int8) or 512-byte (bf16) run.
// The expert layers' W8A16 weights stay int8 and are dequantised in registers to bf16(q * w_s), the bf16
// weight of the per-layer path bit for bit, at half the bytes.  Epilogues round exactly where the GEMM kernel's epilogues do (bias, SiLU,
// RoPE, residual, SiLU-gate, Euler update), so the only difference from the per-layer launch list is the
// fp32 summation order inside each dot product.
// Attention: one CTA per (sample, query head, 16-query tile); the 8 warps take consecutive key ranges with
// an online softmax each and their partial (max, sum, O) are merged in a fixed order.  The prefix keys /
// values of a CTA's first task are copied into shared memory before the grid barrier that precedes the
// phase (they are final before the kernel starts).
//
// Grid barrier: a monotonic 64-bit arrival counter in a caller-provided 8-byte buffer (zero before first use;
// every completed launch leaves it at a multiple of the grid size); each CTA arrives with a release reduction
// and polls for its own precomputed target.  Every wait is bounded: a barrier that
// does not open within spin_limit polls (kSpinLimit unless the caller sets a shorter one) records kErrFlowBarrier in the device error word; the other CTAs see
// the error word at their next wait and return, so the kernel always ends (and later launches refuse to run
// while the error word is set).  A rows are staged with bulk copies completing on an mbarrier, also waited
// for with a bound.
#pragma once

#include <type_traits>

#include "attention.cuh"
#include "gemm.cuh"
#include "norm.cuh"
#include "ptx.cuh"

namespace svla {

constexpr int kFlowMaxLayers = 32;
constexpr int kFlowThreads = 256;
constexpr int kFlowWarps = kFlowThreads / 32;
constexpr int kFlowRows = 64;             // most action rows per call (four m16 tiles)
constexpr int kFlowKC = 1024;             // A columns staged for 64 rows (twice as many for 32-row blocks)
constexpr int kFlowLda = kFlowKC + 16;    // largest staged row stride (elements) of 64 rows
constexpr int kFlowRedStride = 40;        // fp32 row stride of the per-warp partial tiles (conflict-free)
constexpr int kFlowMaxSlices = kFlowKC / 16;  // 16-column slices of a row of E
constexpr int kFlowAttnStride = 72;       // fp32 row stride of the per-warp attention partials
constexpr int kErrFlowBarrier = 103;

// int8 weights in fragment order, each with its per-output-channel scales
struct FlowLayer {
  const __nv_bfloat16* ln1;  // input RMSNorm weight [E]
  const __nv_bfloat16* ln2;  // post-attention RMSNorm weight [E]
  const uint8_t* wq;         // [q_dim, E]
  const uint8_t* wk;         // [kv_dim, E] (self-attention layers)
  const uint8_t* wv;
  const uint8_t* wo;         // [E, q_dim]
  const uint8_t* wg;         // [mlp, E]
  const uint8_t* wu;
  const uint8_t* wd;         // [E, mlp]
  const float *sq, *sk, *sv, *so, *sg, *su, *sd;
  const __nv_bfloat16* k1;   // prefix keys [B * Lp, kv_dim]: the KV cache (self) or its cross projection
  const __nv_bfloat16* v1;
  int cross;
};

struct FlowArgs {
  int B, S, Lp, E, A, Hq, Hkv, mlp, n_layers, n_steps;
  float eps, dt, scale;
  const float* noise;
  float* xt;
  __nv_bfloat16* xt_bf;
  // bf16 weights in fragment order
  const uint8_t* w_in;         // action_in_proj [E, A] + bias [E]
  const __nv_bfloat16* b_in;
  const uint8_t* w_tin;        // action_time_mlp_in, its first E columns [E, E]
  const float* c_step;         // [n_steps, E]: W_tin[:, E:] . time_emb(t_step) + b_tin
  const uint8_t* w_tout;       // action_time_mlp_out [E, E] + bias
  const __nv_bfloat16* b_tout;
  const __nv_bfloat16* ln_f;   // final RMSNorm [E]
  const uint8_t* w_out;        // action_out_proj [A, E] + bias [A]
  const __nv_bfloat16* b_out;
  const uint8_t* key_mask;     // prefix key flags, row b at key_mask + b * key_mask_bs
  long long key_mask_bs;
  const int* suffix_pos;       // [B * S] RoPE positions (self- / cross-attention layers)
  const int* cross_pos;
  const float* rope_cs;        // [max_pos][32] (cos, sin)
  int max_pos;
  __nv_bfloat16 *a_emb, *a_t, *eh, *eq, *ek, *ev, *ectx, *emlp;  // scratch rows
  float* norm_part;            // [kFlowRows][kFlowMaxSlices]: per row and 16-column slice, sum of squares of eh
  unsigned long long* sync;    // monotonic arrival counter (a multiple of gridDim.x between launches)
  uint32_t spin_limit;         // polls of a grid barrier before it gives up (kErrFlowBarrier)
  int* err;
  unsigned long long* dbg;     // profiling: (event, globaltimer ns) pairs of CTA 0 and the last CTA, or nullptr
  FlowLayer layer[kFlowMaxLayers];
};

// profiling events (FlowArgs::dbg): kFlowDbgEvents (code, ns) pairs for CTA 0, then as many for the last CTA
constexpr int kFlowDbgEvents = 1024;
enum FlowEvent : int {
  kEvBarrierIn = 1, kEvBarrierOut = 2, kEvStaged = 3, kEvMma = 4, kEvEpilogue = 5, kEvAttn = 6,
  kEvCopied = 7,     // A rows landed in shared memory (before the row norm)
  kEvKeys = 8,       // attention: warp 0's first keys / values landed
  kEvAttnDone = 9,   // attention: warp 0's partial done (before the merge)
};

struct FlowSmem {
  uint64_t bar;                                          // completion of the bulk copies that stage A
  uint64_t pad_;
  __nv_bfloat16 a[kFlowRows * kFlowLda];                 // A rows (bf16)
  float red[kFlowWarps * kFlowRows * kFlowRedStride];    // per-warp partial tiles / attention partials
  float ml[kFlowWarps * 32];                             // attention: per-warp row max (16) and sum (16)
  uint8_t kf[kFlowWarps * 32];                           // attention: the staged keys' padding flags
  float rstd[kFlowRows];                                 // RMSNorm: 1 / rms of the staged rows
  unsigned long long target;                             // arrival count that opens the next grid barrier
  int ok;
  int n_ev;                                              // profiling events recorded by this CTA
};

namespace flow_detail {

using attn_detail::cp_async16;
using attn_detail::cp_async_commit;
using attn_detail::cp_async_wait;
using attn_detail::ex2;
using attn_detail::ldmatrix_x4_trans;
using attn_detail::kLog2e;
using attn_detail::kMaskedScore;
using attn_detail::ldmatrix_x4;
using attn_detail::mma16816;

__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
// bulk copy (no tensor map, no multicast) of `bytes` from global memory into this CTA's shared memory,
// completing on `bar`; 16-byte aligned addresses, bytes a multiple of 16
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ uint32_t ldcg_u32(const __nv_bfloat16* p) {
  return __ldcg(reinterpret_cast<const unsigned int*>(p));
}
__device__ __forceinline__ void store2(__nv_bfloat16* p, float x, float y) {
  *reinterpret_cast<uint32_t*>(p) = pack_bf16_rn(x, y);
}
// store2, returning the sum of squares of the two stored (bf16) values: a row's RMSNorm statistics
__device__ __forceinline__ float store2_ss(__nv_bfloat16* p, float x, float y) {
  const float xr = bf16_round(x), yr = bf16_round(y);
  store2(p, xr, yr);
  return __fmaf_rn(yr, yr, __fmul_rn(xr, xr));
}

// profiling: thread 0 of CTA 0 and of the last CTA append (event, globaltimer) while there is room
__device__ __forceinline__ void event(const FlowArgs& a, FlowSmem& sm, int code) {
  if (a.dbg == nullptr || threadIdx.x != 0) return;
  const int sel = blockIdx.x == 0 ? 0 : (blockIdx.x == gridDim.x - 1 ? 1 : -1);
  if (sel < 0 || sm.n_ev >= kFlowDbgEvents) return;
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  unsigned long long* d = a.dbg + (static_cast<size_t>(sel) * kFlowDbgEvents + sm.n_ev) * 2;
  d[0] = static_cast<unsigned long long>(code);
  d[1] = t;
  ++sm.n_ev;
}

// Grid barrier on a monotonic 64-bit arrival counter: barrier k (1, 2, ...) of a launch opens when the counter
// reaches base + k * gridDim.x, base = the counter at launch (a multiple of gridDim.x: no barrier of this launch
// can open before every CTA has read it, since each must arrive first).  False when it timed out or another CTA recorded an
// error (then the caller returns).
// during(): work of every thread between its CTA's arrival and its wait that depends on no other CTA's writes
// of the phase (L2 prefetches of the next phase's weights, staging of constant keys).
template <typename During>
__device__ bool grid_sync(const FlowArgs& a, FlowSmem& sm, During&& during) {
  __syncthreads();
  event(a, sm, kEvBarrierIn);
  // arrive: a release reduction publishes this CTA's writes (ordered before it by the CTA barrier)
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(a.sync) : "memory");
  during();
  if (threadIdx.x == 0) {
    int ok = 1;
    const unsigned long long target = sm.target;
    sm.target = target + gridDim.x;
    uint32_t spins = 0;
    while (ld_acquire_u64(a.sync) < target) {
      if (++spins >= a.spin_limit) {
        record_error(a.err, kErrFlowBarrier);
        ok = 0;
        break;
      }
      if ((spins & 63u) == 0 && *reinterpret_cast<volatile int*>(a.err) != 0) {
        ok = 0;
        break;
      }
    }
    sm.ok = ok;
  }
  __syncthreads();
  event(a, sm, kEvBarrierOut);
  return sm.ok != 0;
}
__device__ __forceinline__ bool grid_sync(const FlowArgs& a, FlowSmem& sm) {
  return grid_sync(a, sm, [] {});
}

// L2 prefetch of the weight slices of this CTA's first task of a GEMM phase (n_col slices x row blocks of
// rows_t rows, K columns), issued while it waits at the barrier before the phase
template <int G, bool I8, typename WFn>
__device__ __forceinline__ void prefetch_first(WFn&& wslices, int n_col, int M, int rows_t, int K) {
  const int blocks = (M + rows_t - 1) / rows_t;
  if (static_cast<int>(blockIdx.x) >= n_col * blocks || static_cast<int>(threadIdx.x) >= G) return;
  const uint8_t* w[G];
  const float* sc[G];
  wslices(static_cast<int>(blockIdx.x) / blocks, w, sc);
  const uint32_t bytes = static_cast<uint32_t>(K) * 16u * (I8 ? 1u : 2u);
#pragma unroll
  for (int gi = 0; gi < G; ++gi)
    if (gi == static_cast<int>(threadIdx.x))
      asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(w[gi]), "r"(bytes) : "memory");
}

// row stride (elements) of a staged chunk of kc columns: 16-byte rows whose 8-row ldmatrix groups hit
// distinct bank groups ((stride / 8) odd)
__device__ __forceinline__ int staged_ld(int kc) {
  int s = kc + 8;
  if (((s / 8) & 1) == 0) s += 8;
  return s;
}

// rows [0, M) x columns [k0, k0 + kc) of A (row stride lda) into shared memory: one bulk copy per row, all in
// flight at once, completing on the CTA's mbarrier (stage_wait: bounded; a timeout records an error that ends
// the kernel at its next grid barrier).  Rows M..63 are left as they are: they only feed output rows that are
// not stored.
__device__ void stage_issue(FlowSmem& sm, const __nv_bfloat16* A, int lda, int M, int k0, int kc, int ldsa,
                            const float* part = nullptr) {
  const uint32_t part_bytes = part != nullptr ? static_cast<uint32_t>(M * kFlowMaxSlices * 4) : 0u;
  if (threadIdx.x == 0) mbar_arrive_expect_tx(&sm.bar, static_cast<uint32_t>(M * kc * 2) + part_bytes);
  __syncthreads();
  const bool row = static_cast<int>(threadIdx.x) < M, parts = part != nullptr && threadIdx.x == kFlowRows;
  if (row || parts) {
    // order other CTAs' earlier (generic) writes of A and this CTA's earlier reads of the buffer before the copy
    asm volatile("fence.proxy.async.global;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (row)
    bulk_g2s(&sm.a[threadIdx.x * ldsa], A + static_cast<size_t>(threadIdx.x) * lda + k0, static_cast<uint32_t>(kc * 2),
             &sm.bar);
  if (parts) bulk_g2s(sm.red, part, part_bytes, &sm.bar);  // the rows' slice sums of squares (RMSNorm phases)
}
__device__ __forceinline__ void stage_wait(FlowSmem& sm, uint32_t& parity, int* err) {
  mbar_wait(&sm.bar, parity, err);
  parity ^= 1u;
}


// RMSNorm of the staged rows, folded into the GEMM: the phase that wrote the rows left, per row and 16-column
// slice, the sum of squares of the stored bf16 values (reduce_tiles, a fixed butterfly over the slice); they are
// staged with the rows (stage_issue), added here in a fixed order (4 threads per row, consecutive slice runs,
// then a butterfly) into rstd = 1 / sqrt(ss / K + eps), and mma_w applies y = bf16(w * bf16(x * rstd)) to each
// A fragment it loads -- the rounding points of the stand-alone norm kernel's RMSNorm rows (norm_quant_row); only
// the fp32 order of the sum of squares differs.  Rows M.. of the tile get rstd 0 (they feed no stored output).
__device__ void rstd_from_parts(FlowSmem& sm, int K, float eps, int M, int tile_rows) {
  const int m = threadIdx.x >> 2, q = threadIdx.x & 3, ns = K / 16, nq = (ns + 3) / 4;
  float ss = 0.f;
  if (m < M) {
    const float* p = sm.red + m * kFlowMaxSlices;
    const int end = (q + 1) * nq < ns ? (q + 1) * nq : ns;
    for (int sl = q * nq; sl < end; ++sl) ss = __fadd_rn(ss, p[sl]);
  }
  ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, 1));
  ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, 2));
  if (q == 0 && m < tile_rows) {
    const float var = __fdiv_rn(ss, static_cast<float>(K));
    sm.rstd[m] = m < M ? __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps))) : 0.f;
  }
}
// y = bf16(w * bf16(x * r)) of a bf16x2 pair x with weights w (the product of two bf16 values is exact in fp32,
// so one bf16x2 multiply rounds it exactly as bf16(fp32(w) * fp32(h)) does)
__device__ __forceinline__ uint32_t norm_pair(uint32_t x, float r, uint32_t w) {
  const __nv_bfloat162 xb = *reinterpret_cast<const __nv_bfloat162*>(&x);
  const __nv_bfloat162 wb = *reinterpret_cast<const __nv_bfloat162*>(&w);
  const __nv_bfloat162 h = __float22bfloat162_rn(__fmul2_rn(__bfloat1622float2(xb), make_float2(r, r)));
  const __nv_bfloat162 y = __hmul2(wb, h);
  return *reinterpret_cast<const uint32_t*>(&y);
}

// One lane's weight fragments of one k16 step of a 16-column slice: the B fragments (b0, b1) of the slice's two
// 8-column tiles, as int8 (8 bytes) or bf16 (16 bytes).
template <bool I8>
using Frag = typename std::conditional<I8, uint2, uint4>::type;

// bf16x2 of two int8 weights (bytes sh / 8 and sh / 8 + 1 of w) dequantised as bf16(float(q) * s): the rounding
// of the bf16 weight the per-layer path multiplies by
__device__ __forceinline__ uint32_t deq_pair(uint32_t w, int sh, float s) {
  const float q0 = static_cast<float>(static_cast<int8_t>((w >> sh) & 0xFFu));
  const float q1 = static_cast<float>(static_cast<int8_t>((w >> (sh + 8)) & 0xFFu));
  return pack_bf16_rn(__fmul_rn(q0, s), __fmul_rn(q1, s));
}

// the four bf16x2 B registers (tile 0: b0, b1; tile 1: b0, b1) of a fragment; sc: the scales of the lane's
// columns in tiles 0 and 1 (int8 only)
__device__ __forceinline__ void frag_regs(const uint2& f, const float (&sc)[2], uint32_t (&r)[4]) {
  r[0] = deq_pair(f.x, 0, sc[0]);
  r[1] = deq_pair(f.x, 16, sc[0]);
  r[2] = deq_pair(f.y, 0, sc[1]);
  r[3] = deq_pair(f.y, 16, sc[1]);
}
__device__ __forceinline__ void frag_regs(const uint4& f, const float (&)[2], uint32_t (&r)[4]) {
  r[0] = f.x;
  r[1] = f.y;
  r[2] = f.z;
  r[3] = f.w;
}

// this warp's weight fragments of one chunk (k16 steps w, w + 8, ..., at most U) of the slices ws[G], loaded
// before they are needed so that their latency overlaps the staging of A
template <int G, int U, bool I8>
__device__ __forceinline__ void load_w(const uint8_t* const (&ws)[G], int k0, int kc, Frag<I8> (&b)[U][G]) {
  constexpr int kLaneBytes = I8 ? 8 : 16;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int steps = kc / 16, s0 = k0 / 16;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int s = warp + u * kFlowWarps;
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      if (s < steps) {
        b[u][gi] = __ldg(reinterpret_cast<const Frag<I8>*>(ws[gi] + (static_cast<size_t>(s0 + s) * 32 + lane) * kLaneBytes));
      } else {
        b[u][gi] = Frag<I8>{};
      }
    }
  }
}

// the norm weights of this warp's k16 steps (columns k0 + s*16 + 2t, + 1 and + 8, + 9), loaded with the weights
template <int U>
__device__ __forceinline__ void load_nw(const __nv_bfloat16* nw, int k0, int kc, uint32_t (&nv)[U][2]) {
  const int warp = threadIdx.x >> 5, t = threadIdx.x & 3;
  const int steps = kc / 16;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int s = warp + u * kFlowWarps;
    if (s < steps) {
      nv[u][0] = __ldg(reinterpret_cast<const unsigned int*>(nw + k0 + s * 16 + 2 * t));
      nv[u][1] = __ldg(reinterpret_cast<const unsigned int*>(nw + k0 + s * 16 + 2 * t + 8));
    } else {
      nv[u][0] = nv[u][1] = 0u;
    }
  }
}

// this warp's partial products over its k16 steps of the staged chunk; NORM: RMSNorm each A fragment first
// (norm weights nv from load_nw, the fragment rows' rstd in rs[mt][0 / 1] for rows g / g + 8)
template <int G, int MT, int U, bool I8, bool NORM>
__device__ __forceinline__ void mma_w(const FlowSmem& sm, int ldsa, int kc, const Frag<I8> (&b)[U][G],
                                      const float (&sc)[G][2], float (&acc)[G][2][MT][4],
                                      const uint32_t (&nv)[U][2], const float (&rs)[MT][2]) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int steps = kc / 16;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int s = warp + u * kFlowWarps;
    if (s >= steps) break;
    uint32_t r[G][4];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) frag_regs(b[u][gi], sc[gi], r[gi]);
    const uint32_t w_lo = nv[u][0], w_hi = nv[u][1];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
      uint32_t af[4];
      ldmatrix_x4(af, &sm.a[(mt * 16 + (lane & 15)) * ldsa + s * 16 + (lane >> 4) * 8]);
      if constexpr (NORM) {  // a0: row g, k 2t | a1: row g + 8 | a2: row g, k 2t + 8 | a3: row g + 8, k 2t + 8
        af[0] = norm_pair(af[0], rs[mt][0], w_lo);
        af[1] = norm_pair(af[1], rs[mt][1], w_lo);
        af[2] = norm_pair(af[2], rs[mt][0], w_hi);
        af[3] = norm_pair(af[3], rs[mt][1], w_hi);
      }
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        mma16816(acc[gi][0][mt], af, r[gi][0], r[gi][1]);
        mma16816(acc[gi][1][mt], af, r[gi][2], r[gi][3]);
      }
    }
  }
}

// adds the 8 warps' partial tiles (warp order) and hands each (row, column pair) to the epilogue together
// with the four words pre(m, j) fetched for it before the partial tiles were exchanged (residuals, biases:
// their load latency overlaps the exchange).  An epilogue that returns a SqSums<G> returns, per group, the sum of
// squares of the two values it stored: the 8 pairs of a row of each group's 16 columns are then added by a fixed
// butterfly and handed to stat(m, gi, ss) -- the RMSNorm statistics of the rows for the next phase.
template <int G>
struct SqSums {
  float s[G];
};
template <int G, int MT, typename Pre, typename Epi, typename Stat>
__device__ __forceinline__ void reduce_tiles(FlowSmem& sm, int M, const float (&acc)[G][2][MT][4], Pre&& pre,
                                             Epi&& epi, Stat&& stat) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  constexpr int kItems = (MT * 16 * 8 + kFlowThreads - 1) / kFlowThreads;  // (row, column pair) items per thread
  using R = decltype(epi(0, 0, std::declval<float (&)[G][2]>(), std::declval<const uint4&>()));
  constexpr bool kStats = std::is_same<R, SqSums<G>>::value;
  uint4 pv[kItems];
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const int idx = threadIdx.x + u * kFlowThreads;
    pv[u] = idx < M * 8 ? pre(idx >> 3, (idx & 7) * 2) : make_uint4(0u, 0u, 0u, 0u);
  }
  float* red = sm.red + warp * kFlowRows * kFlowRedStride;
#pragma unroll
  for (int gi = 0; gi < G; ++gi) {
#pragma unroll
    for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
      for (int mt = 0; mt < MT; ++mt) {
        const int col = gi * 16 + nt * 8 + 2 * t, r0 = mt * 16 + g;
        *reinterpret_cast<float2*>(&red[r0 * kFlowRedStride + col]) =
            make_float2(acc[gi][nt][mt][0], acc[gi][nt][mt][1]);
        *reinterpret_cast<float2*>(&red[(r0 + 8) * kFlowRedStride + col]) =
            make_float2(acc[gi][nt][mt][2], acc[gi][nt][mt][3]);
      }
    }
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const int idx = threadIdx.x + u * kFlowThreads;
    const bool valid = idx < M * 8;  // every thread takes every u (the butterfly below needs whole warps)
    const int m = idx >> 3, j = (idx & 7) * 2;
    SqSums<G> ss{};
    if (valid) {
      float v[G][2];
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        v[gi][0] = v[gi][1] = 0.f;
#pragma unroll
        for (int w = 0; w < kFlowWarps; ++w) {
          const float2 p = *reinterpret_cast<const float2*>(
              &sm.red[(w * kFlowRows + m) * kFlowRedStride + gi * 16 + j]);
          v[gi][0] = __fadd_rn(v[gi][0], p.x);
          v[gi][1] = __fadd_rn(v[gi][1], p.y);
        }
      }
      if constexpr (kStats) {
        ss = epi(m, j, v, pv[u]);
      } else {
        epi(m, j, v, pv[u]);
      }
    }
    if constexpr (kStats) {
#pragma unroll
      for (int gi = 0; gi < G; ++gi) {
        float x = ss.s[gi];
        x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, 1));
        x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, 2));
        x = __fadd_rn(x, __shfl_xor_sync(0xffffffffu, x, 4));
        if (valid && (idx & 7) == 0) stat(m, gi, x);
      }
    }
  }
  __syncthreads();
}

// One GEMM phase: out[rows, slice] = epi(A[rows, :K] . W[slice, :K]^T) for n_col slices of G x 16 columns,
// each split into blocks of MT * 16 rows (a task = a slice x a row block: with MT = 2 a CTA stages, normalises
// and multiplies half of the rows, at twice the tasks); wslices(slice, w, s) gives each group's packed 16-column
// slice (K * 16 elements, int8 when I8, else bf16) and, for int8, the slice's 16 per-column scales.
// NORM: RMSNorm the A rows with norm_w (K <= 1024; rstd_from_parts).  An epilogue that returns SqSums<G> leaves
// the RMSNorm statistics of its rows for the next phase: group gi of task ct is slice ct * G + gi of the output.
template <int G, int MT, bool I8, bool NORM, typename WFn, typename PreFn, typename EpiFn>
__device__ void gemm_phase(const FlowArgs& fa, FlowSmem& sm, uint32_t& parity, int M, const __nv_bfloat16* A, int K,
                           const __nv_bfloat16* norm_w, float eps, int n_col, WFn&& wslices, PreFn&& pre,
                           EpiFn&& epi) {
  constexpr int kRowsT = MT * 16;
  // columns staged per chunk: as many as the A buffer holds for kRowsT rows, at most U k16 steps per warp
  constexpr int U = G == 1 ? 16 : 8;
  constexpr int KC0 = U * 16 * kFlowWarps, KC1 = (kFlowRows * kFlowLda) / kRowsT - 16;
  constexpr int KC = KC0 < KC1 ? KC0 : KC1;
  static_assert(KC % 16 == 0 && KC >= 1024, "chunk width");
  if (NORM && K > KC) return;  // a normed phase stages its rows whole (svla_flow checks K <= 1024)
  const int blocks = (M + kRowsT - 1) / kRowsT;
  const int n_tasks = n_col * blocks;
  if (static_cast<int>(blockIdx.x) >= n_tasks) return;
  const bool single = K <= KC;
  const int ldsa = staged_ld(single ? K : KC);
  float rs[MT][2] = {};
  uint32_t nv[U][2] = {};
  int staged = -1;  // row block in shared memory (single-chunk phases)
  Frag<I8> b[U][G];
  const int g8 = (threadIdx.x & 31) >> 2;
  for (int task = blockIdx.x; task < n_tasks; task += gridDim.x) {
    const int ct = task / blocks, rb = task % blocks;
    const int row0 = rb * kRowsT, rows = (M - row0) < kRowsT ? (M - row0) : kRowsT;
    const __nv_bfloat16* Ab = A + static_cast<size_t>(row0) * K;
    const uint8_t* wr[G];
    const float* wsc[G];
    wslices(ct, wr, wsc);
    float sc[G][2];
#pragma unroll
    for (int gi = 0; gi < G; ++gi) {
      sc[gi][0] = I8 ? __ldg(wsc[gi] + g8) : 0.f;
      sc[gi][1] = I8 ? __ldg(wsc[gi] + 8 + g8) : 0.f;
    }
    float acc[G][2][MT][4];
#pragma unroll
    for (int gi = 0; gi < G; ++gi)
#pragma unroll
      for (int nt = 0; nt < 2; ++nt)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) acc[gi][nt][mt][0] = acc[gi][nt][mt][1] = acc[gi][nt][mt][2] = acc[gi][nt][mt][3] = 0.f;
    for (int k0 = 0; k0 < K; k0 += KC) {
      const int kc = (K - k0) < KC ? (K - k0) : KC;
      // the rows are requested before the weights, whose loads would otherwise queue ahead of them
      const bool stage = !single || staged != rb;
      if (stage) {
        if (!single) __syncthreads();  // every warp is done with the previous chunk
        stage_issue(sm, Ab, K, rows, k0, kc, ldsa,
                    NORM ? fa.norm_part + static_cast<size_t>(row0) * kFlowMaxSlices : nullptr);
      }
      load_w<G, U, I8>(wr, k0, kc, b);
      if constexpr (NORM) load_nw<U>(norm_w, k0, kc, nv);
      if (stage) {
        stage_wait(sm, parity, fa.err);
        event(fa, sm, kEvCopied);
        if (single) staged = rb;
        if constexpr (NORM) {
          rstd_from_parts(sm, K, eps, rows, kRowsT);
          __syncthreads();
#pragma unroll
          for (int mt = 0; mt < MT; ++mt) {
            rs[mt][0] = sm.rstd[mt * 16 + g8];
            rs[mt][1] = sm.rstd[mt * 16 + 8 + g8];
          }
        }
        event(fa, sm, kEvStaged);
      }
      mma_w<G, MT, U, I8, NORM>(sm, ldsa, kc, b, sc, acc, nv, rs);
    }
    event(fa, sm, kEvMma);
    reduce_tiles<G, MT>(
        sm, rows, acc, [&](int m, int j) { return pre(ct, row0 + m, j); },
        [&](int m, int j, float (&v)[G][2], const uint4& p) { return epi(ct, row0 + m, j, v, p); },
        [&](int m, int gi, float ss) {
          fa.norm_part[static_cast<size_t>(row0 + m) * kFlowMaxSlices + ct * G + gi] = ss;
        });
    event(fa, sm, kEvEpilogue);
  }
}

constexpr int kAttnSub = 32;  // keys a warp stages at a time
constexpr int kAttnRs = 72;   // bf16 row stride of the staged keys / values (conflict-free ldmatrix)
enum { kKeysAll = 0, kKeysPrefix = 1, kKeysSuffix = 2 };

// Warp-level asynchronous copies of keys [sub0, sub0 + 32) of kv head kh of sample b (and their padding flags)
// into this warp's slice of shared memory; keys at or past kend are zero-filled.  part: all keys, or only those
// of the prefix (keys < Lp: the KV cache / cross projections, final before the flow kernel starts) with the
// flags, or only the chunk's own keys (written by the QKV phase).
__device__ void stage_keys(FlowSmem& sm, const FlowArgs& a, const FlowLayer& L, int b, int kh, int sub0, int kend,
                           int part) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, kvd = a.Hkv * 64, L1 = a.Lp;
  __nv_bfloat16* sk = sm.a + warp * (2 * kAttnSub * kAttnRs);
  __nv_bfloat16* sv = sk + kAttnSub * kAttnRs;
  for (int idx = lane; idx < kAttnSub * 8; idx += 32) {
    const int r = idx >> 3, c = (idx & 7) * 8;
    const int key = sub0 + r;
    if ((part == kKeysPrefix && key >= L1) || (part == kKeysSuffix && key < L1)) continue;
    const bool in = key < kend;
    const __nv_bfloat16* kp = L.k1;
    const __nv_bfloat16* vp = L.v1;
    if (in) {
      if (key < L1) {
        const size_t off = (static_cast<size_t>(b) * a.Lp + key) * kvd + kh * 64 + c;
        kp = L.k1 + off;
        vp = L.v1 + off;
      } else {
        const size_t off = (static_cast<size_t>(b) * a.S + (key - L1)) * kvd + kh * 64 + c;
        kp = a.ek + off;
        vp = a.ev + off;
      }
    }
    cp_async16(&sk[r * kAttnRs + c], kp, in ? 16 : 0);
    cp_async16(&sv[r * kAttnRs + c], vp, in ? 16 : 0);
  }
  // padding flags of the prefix keys among them (16-byte runs; runs at or past the prefix read as 0)
  if (part != kKeysSuffix && lane < kAttnSub / 16) {
    const int key = sub0 + lane * 16;
    const bool in = a.key_mask != nullptr && key < a.Lp;
    const void* src = in ? static_cast<const void*>(a.key_mask + static_cast<size_t>(b) * a.key_mask_bs + key)
                         : static_cast<const void*>(L.k1);
    cp_async16(sm.kf + warp * kAttnSub + lane * 16, src, in ? 16 : 0);
  }
  cp_async_commit();
}

// Before the grid barrier that precedes attention: the prefix part of every warp's first keys of this CTA's
// first attention task (the same decomposition as attention_phase)
__device__ void attention_prestage(FlowSmem& sm, const FlowArgs& a, const FlowLayer& L) {
  const int qtiles = (a.S + 15) / 16;
  const int task = blockIdx.x;
  if (task >= a.B * a.Hq * qtiles) return;
  const int Lk = a.Lp + (L.cross ? 0 : a.S);
  const int ks = ((Lk + kFlowWarps - 1) / kFlowWarps + 15) / 16 * 16;
  const int warp = threadIdx.x >> 5;
  const int h = (task / qtiles) % a.Hq, b = task / (qtiles * a.Hq), kh = h / (a.Hq / a.Hkv);
  const int kbeg = warp * ks, kend = (kbeg + ks) < Lk ? (kbeg + ks) : Lk;
  if (kbeg < kend) stage_keys(sm, a, L, b, kh, kbeg, kend, kKeysPrefix);
}

// attention of one expert layer; o -> ectx (bf16).  Each warp stages its keys / values 32 at a time in its
// own slice of shared memory (asynchronous copies, all in flight at once) and reads MMA fragments with
// ldmatrix; keys past the warp's range or past the last key are zero-filled and masked.
__device__ void attention_phase(FlowSmem& sm, const FlowArgs& a, const FlowLayer& L) {
  constexpr int kSub = kAttnSub, kRs = kAttnRs;
  const int qd = a.Hq * 64, grp = a.Hq / a.Hkv;
  const int qtiles = (a.S + 15) / 16;
  const int n_tasks = a.B * a.Hq * qtiles;
  const int L1 = a.Lp, Lk = L1 + (L.cross ? 0 : a.S);
  const int ks = ((Lk + kFlowWarps - 1) / kFlowWarps + 15) / 16 * 16;  // keys per warp
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
  const __nv_bfloat16* sk = sm.a + warp * (2 * kSub * kRs);
  const __nv_bfloat16* sv = sk + kSub * kRs;
  for (int task = blockIdx.x; task < n_tasks; task += gridDim.x) {
    const int qt = task % qtiles, h = (task / qtiles) % a.Hq, b = task / (qtiles * a.Hq);
    const int kh = h / grp;
    const int s0 = qt * 16 + g, s1 = s0 + 8;
    const int kbeg = warp * ks, kend = (kbeg + ks) < Lk ? (kbeg + ks) : Lk;
    const uint8_t* kflags = a.key_mask;
    const uint8_t* kf = sm.kf + warp * kSub;
    // the first keys of the CTA's first task had their prefix part (and flags) staged before the grid barrier
    // (attention_prestage): only the chunk's own keys are left
    const bool prestaged = task == static_cast<int>(blockIdx.x);
    if (kbeg < kend) stage_keys(sm, a, L, b, kh, kbeg, kend, prestaged ? kKeysSuffix : kKeysAll);
    uint32_t qa[4][4];
    {
      const __nv_bfloat16* q0 = a.eq + static_cast<size_t>(b * a.S + s0) * qd + h * 64;
      const __nv_bfloat16* q1 = a.eq + static_cast<size_t>(b * a.S + s1) * qd + h * 64;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        qa[kk][0] = s0 < a.S ? ldcg_u32(q0 + kk * 16 + 2 * t) : 0u;
        qa[kk][1] = s1 < a.S ? ldcg_u32(q1 + kk * 16 + 2 * t) : 0u;
        qa[kk][2] = s0 < a.S ? ldcg_u32(q0 + kk * 16 + 8 + 2 * t) : 0u;
        qa[kk][3] = s1 < a.S ? ldcg_u32(q1 + kk * 16 + 8 + 2 * t) : 0u;
      }
    }
    float o[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float mx[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
    for (int sub0 = kbeg; sub0 < kend; sub0 += kSub) {
      if (sub0 != kbeg) {
        __syncwarp();  // the previous keys' fragments have been read
        stage_keys(sm, a, L, b, kh, sub0, kend, kKeysAll);
      }
      cp_async_wait<0>();
      __syncwarp();
      if (sub0 == kbeg) event(a, sm, kEvKeys);
      const int sub_end = (sub0 + kSub) < kend ? (sub0 + kSub) : kend;
      for (int key0 = sub0; key0 < sub_end; key0 += 16) {
        const int rb = key0 - sub0;
        float s[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {
          // B fragments of the two 8-key n-tiles: keys rb + 0..7 | 8..15, head dims kk*16 + 0..7 | 8..15
          uint32_t kb[4];
          ldmatrix_x4(kb, &sk[(rb + (lane & 7) + ((lane >> 4) << 3)) * kRs + kk * 16 + ((lane >> 3) & 1) * 8]);
          mma16816(s[0], qa[kk], kb[0], kb[1]);
          mma16816(s[1], qa[kk], kb[2], kb[3]);
        }
        // scale, mask (key padding over the prefix, causal order over the chunk), online softmax
        float tmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int key = key0 + nt * 8 + 2 * t + (e & 1);
            const int query = (e >> 1) ? s1 : s0;
            float v = __fmul_rn(s[nt][e], a.scale);
            if (key >= Lk) {
              v = -INFINITY;
            } else if (key < a.Lp) {
              if (kflags != nullptr && kf[key - sub0] == 0) v = kMaskedScore;
            } else if (key - a.Lp > query) {
              v = kMaskedScore;
            }
            s[nt][e] = v;
            tmax[e >> 1] = fmaxf(tmax[e >> 1], v);
          }
        }
        float alpha[2];
#pragma unroll
        for (int hr = 0; hr < 2; ++hr) {
          tmax[hr] = fmaxf(tmax[hr], __shfl_xor_sync(0xffffffffu, tmax[hr], 1));
          tmax[hr] = fmaxf(tmax[hr], __shfl_xor_sync(0xffffffffu, tmax[hr], 2));
          const float nm = fmaxf(mx[hr], tmax[hr]);
          alpha[hr] = (mx[hr] == -INFINITY) ? 0.f : ex2((mx[hr] - nm) * kLog2e);
          mx[hr] = nm;
          l[hr] *= alpha[hr];
        }
#pragma unroll
        for (int n = 0; n < 8; ++n) {
          o[n][0] *= alpha[0];
          o[n][1] *= alpha[0];
          o[n][2] *= alpha[1];
          o[n][3] *= alpha[1];
        }
        uint32_t pa[4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
          const float p0 = ex2((s[nt][0] - mx[0]) * kLog2e), p1 = ex2((s[nt][1] - mx[0]) * kLog2e);
          const float p2 = ex2((s[nt][2] - mx[1]) * kLog2e), p3 = ex2((s[nt][3] - mx[1]) * kLog2e);
          l[0] += p0 + p1;
          l[1] += p2 + p3;
          pa[2 * nt] = pack_bf16_rn(p0, p1);
          pa[2 * nt + 1] = pack_bf16_rn(p2, p3);
        }
#pragma unroll
        for (int np = 0; np < 4; ++np) {
          // V^T fragments: keys rb + 0..15, head dims np*16 + 0..7 | 8..15
          uint32_t vb[4];
          ldmatrix_x4_trans(vb, &sv[(rb + (lane & 15)) * kRs + np * 16 + ((lane >> 4) << 3)]);
          mma16816(o[2 * np], pa, vb[0], vb[1]);
          mma16816(o[2 * np + 1], pa, vb[2], vb[3]);
        }
      }
    }
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 1);
      l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 2);
    }
    event(a, sm, kEvAttnDone);
    // this warp's partial (max, sum, unnormalised O) -> shared memory; merged in warp order
    float* po = sm.red + warp * 16 * kFlowAttnStride;
#pragma unroll
    for (int nd = 0; nd < 8; ++nd) {
      const int d = nd * 8 + 2 * t;
      *reinterpret_cast<float2*>(&po[g * kFlowAttnStride + d]) = make_float2(o[nd][0], o[nd][1]);
      *reinterpret_cast<float2*>(&po[(g + 8) * kFlowAttnStride + d]) = make_float2(o[nd][2], o[nd][3]);
    }
    if (t == 0) {
      sm.ml[warp * 32 + g] = mx[0];
      sm.ml[warp * 32 + g + 8] = mx[1];
      sm.ml[warp * 32 + 16 + g] = l[0];
      sm.ml[warp * 32 + 16 + g + 8] = l[1];
    }
    __syncthreads();
    for (int idx = threadIdx.x; idx < 16 * 32; idx += kFlowThreads) {
      const int r = idx >> 5, d = (idx & 31) * 2;
      const int s = qt * 16 + r;
      if (s >= a.S) continue;
      float M = -INFINITY;
#pragma unroll
      for (int w = 0; w < kFlowWarps; ++w) M = fmaxf(M, sm.ml[w * 32 + r]);
      float Ls = 0.f, o0 = 0.f, o1 = 0.f;
#pragma unroll
      for (int w = 0; w < kFlowWarps; ++w) {
        const float mw = sm.ml[w * 32 + r];
        if (mw == -INFINITY) continue;  // a warp without keys
        const float f = ex2((mw - M) * kLog2e);
        const float2 ow = *reinterpret_cast<const float2*>(&sm.red[(w * 16 + r) * kFlowAttnStride + d]);
        Ls = __fmaf_rn(sm.ml[w * 32 + 16 + r], f, Ls);
        o0 = __fmaf_rn(ow.x, f, o0);
        o1 = __fmaf_rn(ow.y, f, o1);
      }
      const float inv = __frcp_rn(Ls);
      store2(a.ectx + static_cast<size_t>(b * a.S + s) * qd + h * 64 + d, bf16_round(o0 * inv), bf16_round(o1 * inv));
    }
    __syncthreads();
    event(a, sm, kEvAttn);
  }
}

}  // namespace flow_detail

// Fragment-order copy of a weight w [n, k] (row stride ld elements of eb bytes; n, k multiples of 16), the
// layout the flow kernel's weight loads read: thread i writes lane (i % 32) of k16 step s of 16-row slice sl
// (i / 32 = sl * k / 16 + s), 8 elements: rows sl*16 + g (e < 4) or + 8 + g (e >= 4), g = lane / 4, columns
// s*16 + 2 (lane % 4) + (e % 2) + 8 ((e / 2) % 2) -- the B fragments b0, b1 of mma.m16n8k16 for both 8-row tiles.
__global__ void pack_fragments_kernel(const uint8_t* w, int eb, long long ld, int n, int k, uint8_t* out) {
  const long long total = static_cast<long long>(n) * k / 8;
  const int ks = k / 16;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const int lane = static_cast<int>(i % 32);
    const long long r = i / 32;
    const int s = static_cast<int>(r % ks), sl = static_cast<int>(r / ks);
    const int g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const long long row = sl * 16 + (e >= 4 ? 8 : 0) + g;
      const long long col = s * 16 + 2 * t + (e & 1) + ((e >> 1) & 1) * 8;
      const uint8_t* src = w + (row * ld + col) * eb;
      uint8_t* dst = out + (i * 8 + e) * eb;
      for (int bb = 0; bb < eb; ++bb) dst[bb] = src[bb];
    }
  }
}

__global__ void __launch_bounds__(kFlowThreads, 1) flow_kernel(const FlowArgs a) {
  using namespace flow_detail;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  FlowSmem& sm = *reinterpret_cast<FlowSmem*>(smem_raw);
  uint32_t parity = 0;  // phase parity of the staging mbarrier
  if (threadIdx.x == 0) {
    sm.n_ev = 0;
    mbar_init(&sm.bar, 1);
    fence_mbar_init();
    // a device error left by an earlier launch may have left the barrier counter between multiples: do not run
    sm.ok = *reinterpret_cast<volatile int*>(a.err) == 0;
    const unsigned long long n = gridDim.x;
    sm.target = (ld_acquire_u64(a.sync) / n + 1ull) * n;
  }
  __syncthreads();
  if (!sm.ok) return;
  const int M = a.B * a.S, E = a.E, Ad = a.A, qd = a.Hq * 64, kvd = a.Hkv * 64;

  // x_t = noise
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < M * Ad; i += gridDim.x * blockDim.x) {
    const float x = a.noise[i];
    a.xt[i] = x;
    a.xt_bf[i] = __float2bfloat16_rn(x);
  }

  // 16-column slice `i` of a fragment-packed weight with k columns
  auto slice_i8 = [](const uint8_t* w, int i, int k) { return w + static_cast<size_t>(i) * 16 * k; };
  auto slice_bf16 = [](const uint8_t* w, int i, int k) { return w + static_cast<size_t>(i) * 32 * k; };
  auto no_pre = [](int, int, int) { return make_uint4(0u, 0u, 0u, 0u); };
  // two bf16 biases of columns c, c + 1 (one word)
  auto bias_pre = [](const __nv_bfloat16* bias, int c) {
    return make_uint4(__ldg(reinterpret_cast<const unsigned int*>(bias + c)), 0u, 0u, 0u);
  };
  auto lo = [](uint32_t w) { return __uint_as_float(w << 16); };          // bf16 in the low half
  auto hi = [](uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); };  // bf16 in the high half
  // residual epilogue: p.x holds eh[m, c..c+1]
  auto resid_store = [&](int c, int m, const float (&v)[1][2], const uint4& p) {
    return SqSums<1>{{store2_ss(a.eh + static_cast<size_t>(m) * E + c, __fadd_rn(bf16_round(v[0][0]), lo(p.x)),
                                __fadd_rn(bf16_round(v[0][1]), hi(p.x)))}};
  };

  // weight slices of each GEMM phase: task -> the packed 16-column slices of its G groups (and their scales)
  auto w_in = [&](int task, const uint8_t* (&w)[1], const float* (&s)[1]) {
    w[0] = slice_bf16(a.w_in, task, Ad);
    s[0] = nullptr;
  };
  auto w_tin = [&](int task, const uint8_t* (&w)[1], const float* (&s)[1]) {
    w[0] = slice_bf16(a.w_tin, task, E);
    s[0] = nullptr;
  };
  auto w_tout = [&](int task, const uint8_t* (&w)[1], const float* (&s)[1]) {
    w[0] = slice_bf16(a.w_tout, task, E);
    s[0] = nullptr;
  };
  auto w_out = [&](int task, const uint8_t* (&w)[1], const float* (&s)[1]) {
    w[0] = slice_bf16(a.w_out, task, E);
    s[0] = nullptr;
  };
  // q (and k, v on self-attention layers) with RoPE; a task is the column pairs (c, c + 32) of 16 consecutive
  // rotation pairs of one head: c0 = head * 64 + half * 16
  auto qkv_cols = [&](const FlowLayer& L) { return 2 * a.Hq + (L.cross ? 0 : 4 * a.Hkv); };
  auto qkv_seg = [&](const FlowLayer& L, int task, int& seg, int& c0) {
    const int q_tasks = 2 * a.Hq, kv_tasks = L.cross ? 0 : 2 * a.Hkv;
    int t = task;
    seg = 0;
    if (t >= q_tasks) {
      t -= q_tasks;
      seg = 1;
      if (t >= kv_tasks) {
        t -= kv_tasks;
        seg = 2;
      }
    }
    c0 = (t >> 1) * 64 + (t & 1) * 16;
  };
  auto w_qkv = [&](const FlowLayer& L, int task, const uint8_t* (&w)[2], const float* (&s)[2]) {
    int seg, c0;
    qkv_seg(L, task, seg, c0);
    const uint8_t* W = seg == 0 ? L.wq : (seg == 1 ? L.wk : L.wv);
    const float* S = seg == 0 ? L.sq : (seg == 1 ? L.sk : L.sv);
    w[0] = slice_i8(W, c0 / 16, E);
    w[1] = slice_i8(W, (c0 + 32) / 16, E);
    s[0] = S + c0;
    s[1] = S + c0 + 32;
  };
  auto w_o = [&](const FlowLayer& L, int task, const uint8_t* (&w)[1], const float* (&s)[1]) {
    w[0] = slice_i8(L.wo, task, qd);
    s[0] = L.so + task * 16;
  };
  auto w_gu = [&](const FlowLayer& L, int task, const uint8_t* (&w)[2], const float* (&s)[2]) {
    w[0] = slice_i8(L.wg, task, E);
    w[1] = slice_i8(L.wu, task, E);
    s[0] = L.sg + task * 16;
    s[1] = L.su + task * 16;
  };
  auto w_d = [&](const FlowLayer& L, int task, const uint8_t* (&w)[1], const float* (&s)[1]) {
    w[0] = slice_i8(L.wd, task, a.mlp);
    s[0] = L.sd + task * 16;
  };
  auto bind = [](auto& f, const FlowLayer& L) { return [&f, &L](int t, auto& w, auto& s) { f(L, t, w, s); }; };
  // L2 prefetches of a phase's first-task weights, issued while waiting at the barrier before it
  auto pf_in = [&] { prefetch_first<1, false>(w_in, E / 16, M, 32, Ad); };
  auto pf_qkv = [&](const FlowLayer& L) { prefetch_first<2, true>(bind(w_qkv, L), qkv_cols(L), M, 32, E); };
  auto pf_o = [&](const FlowLayer& L) { prefetch_first<1, true>(bind(w_o, L), E / 16, M, 32, qd); };
  auto pf_gu = [&](const FlowLayer& L) { prefetch_first<2, true>(bind(w_gu, L), a.mlp / 16, M, 64, E); };
  auto pf_d = [&](const FlowLayer& L) { prefetch_first<1, true>(bind(w_d, L), E / 16, M, 32, a.mlp); };

  if (!grid_sync(a, sm, pf_in)) return;

  for (int step = 0; step < a.n_steps; ++step) {
    // action_in_proj: a_emb = bf16(x_t . W_in^T + b)
    gemm_phase<1, 2, false, false>(
        a, sm, parity, M, a.xt_bf, Ad, nullptr, 0.f, E / 16, w_in,
        [&](int task, int, int j) { return bias_pre(a.b_in, task * 16 + j); },
        [&](int task, int m, int j, float (&v)[1][2], const uint4& p) {
          store2(a.a_emb + static_cast<size_t>(m) * E + task * 16 + j, __fadd_rn(v[0][0], lo(p.x)),
                 __fadd_rn(v[0][1], hi(p.x)));
        });
    if (!grid_sync(a, sm, [&] { prefetch_first<1, false>(w_tin, E / 16, M, 32, E); })) return;
    // time MLP in: a_t = bf16(silu(bf16(a_emb . W_tin[:, :E]^T + c_step)))
    const float* cst = a.c_step + static_cast<size_t>(step) * E;
    gemm_phase<1, 2, false, false>(
        a, sm, parity, M, a.a_emb, E, nullptr, 0.f, E / 16, w_tin,
        [&](int task, int, int j) {
          const float2 c2 = __ldg(reinterpret_cast<const float2*>(cst + task * 16 + j));
          return make_uint4(__float_as_uint(c2.x), __float_as_uint(c2.y), 0u, 0u);
        },
        [&](int task, int m, int j, float (&v)[1][2], const uint4& p) {
          const float x0 = bf16_round(__fadd_rn(v[0][0], __uint_as_float(p.x)));
          const float x1 = bf16_round(__fadd_rn(v[0][1], __uint_as_float(p.y)));
          store2(a.a_t + static_cast<size_t>(m) * E + task * 16 + j, silu_f(x0), silu_f(x1));
        });
    if (!grid_sync(a, sm, [&] { prefetch_first<1, false>(w_tout, E / 16, M, 32, E); })) return;
    // time MLP out: eh = bf16(a_t . W_tout^T + b)
    gemm_phase<1, 2, false, false>(
        a, sm, parity, M, a.a_t, E, nullptr, 0.f, E / 16, w_tout,
        [&](int task, int, int j) { return bias_pre(a.b_tout, task * 16 + j); },
        [&](int task, int m, int j, float (&v)[1][2], const uint4& p) {
          return SqSums<1>{{store2_ss(a.eh + static_cast<size_t>(m) * E + task * 16 + j, __fadd_rn(v[0][0], lo(p.x)),
                                      __fadd_rn(v[0][1], hi(p.x)))}};
        });
    if (!grid_sync(a, sm, [&] { pf_qkv(a.layer[0]); })) return;

    for (int li = 0; li < a.n_layers; ++li) {
      const FlowLayer& L = a.layer[li];
      const int* pos = L.cross ? a.cross_pos : a.suffix_pos;
      gemm_phase<2, 2, true, true>(
          a, sm, parity, M, a.eh, E, L.ln1, a.eps, qkv_cols(L), bind(w_qkv, L),
          [&](int task, int m, int j) {
            // (cos, sin) of rotation pairs i0, i0 + 1 at this row's position
            int seg, c0;
            qkv_seg(L, task, seg, c0);
            if (seg == 2) return make_uint4(0u, 0u, 0u, 0u);
            int ps = pos[m];
            ps = ps < 0 ? 0 : (ps >= a.max_pos ? a.max_pos - 1 : ps);
            const int i0 = (c0 & 63) + j;
            const float4 cs = __ldg(reinterpret_cast<const float4*>(a.rope_cs + (static_cast<size_t>(ps) * 32 + i0) * 2));
            return make_uint4(__float_as_uint(cs.x), __float_as_uint(cs.y), __float_as_uint(cs.z), __float_as_uint(cs.w));
          },
          [&](int task, int m, int j, float (&v)[2][2], const uint4& p) {
            int seg, c0;
            qkv_seg(L, task, seg, c0);
            __nv_bfloat16* out = seg == 0 ? a.eq : (seg == 1 ? a.ek : a.ev);
            const int ld = seg == 0 ? qd : kvd;
            float x1a = bf16_round(v[0][0]), x1b = bf16_round(v[0][1]);
            float x2a = bf16_round(v[1][0]), x2b = bf16_round(v[1][1]);
            if (seg < 2) {
              const float ca = __uint_as_float(p.x), sa = __uint_as_float(p.y);
              const float cb = __uint_as_float(p.z), sb = __uint_as_float(p.w);
              const float y1a = __fsub_rn(__fmul_rn(x1a, ca), __fmul_rn(x2a, sa));
              const float y2a = __fadd_rn(__fmul_rn(x2a, ca), __fmul_rn(x1a, sa));
              const float y1b = __fsub_rn(__fmul_rn(x1b, cb), __fmul_rn(x2b, sb));
              const float y2b = __fadd_rn(__fmul_rn(x2b, cb), __fmul_rn(x1b, sb));
              x1a = y1a;
              x2a = y2a;
              x1b = y1b;
              x2b = y2b;
            }
            store2(out + static_cast<size_t>(m) * ld + c0 + j, x1a, x1b);
            store2(out + static_cast<size_t>(m) * ld + c0 + 32 + j, x2a, x2b);
          });
      // the prefix keys / values do not depend on this phase: staged while waiting at the barrier
      if (!grid_sync(a, sm, [&] { attention_prestage(sm, a, L); })) return;
      attention_phase(sm, a, L);
      if (!grid_sync(a, sm, [&] { pf_o(L); })) return;
      // o_proj + residual: eh = bf16(bf16(ectx . W_o^T) + eh)
      gemm_phase<1, 2, true, false>(
          a, sm, parity, M, a.ectx, qd, nullptr, 0.f, E / 16, bind(w_o, L),
          [&](int task, int m, int j) {
            return make_uint4(ldcg_u32(a.eh + static_cast<size_t>(m) * E + task * 16 + j), 0u, 0u, 0u);
          },
          [&](int task, int m, int j, float (&v)[1][2], const uint4& p) { return resid_store(task * 16 + j, m, v, p); });
      if (!grid_sync(a, sm, [&] { pf_gu(L); })) return;
      // gate / up + SiLU gate: emlp = bf16(bf16(silu(bf16(gate))) * bf16(up))
      gemm_phase<2, 4, true, true>(
          a, sm, parity, M, a.eh, E, L.ln2, a.eps, a.mlp / 16, bind(w_gu, L), no_pre,
          [&](int task, int m, int j, float (&v)[2][2], const uint4&) {
            const float g0 = bf16_round(silu_f(bf16_round(v[0][0])));
            const float g1 = bf16_round(silu_f(bf16_round(v[0][1])));
            store2(a.emlp + static_cast<size_t>(m) * a.mlp + task * 16 + j, __fmul_rn(g0, bf16_round(v[1][0])),
                   __fmul_rn(g1, bf16_round(v[1][1])));
          });
      if (!grid_sync(a, sm, [&] { pf_d(L); })) return;
      // down_proj + residual
      gemm_phase<1, 2, true, false>(
          a, sm, parity, M, a.emlp, a.mlp, nullptr, 0.f, E / 16, bind(w_d, L),
          [&](int task, int m, int j) {
            return make_uint4(ldcg_u32(a.eh + static_cast<size_t>(m) * E + task * 16 + j), 0u, 0u, 0u);
          },
          [&](int task, int m, int j, float (&v)[1][2], const uint4& p) { return resid_store(task * 16 + j, m, v, p); });
      const bool last = li + 1 == a.n_layers;
      if (!grid_sync(a, sm, [&] {
            if (last) prefetch_first<1, false>(w_out, Ad / 16, M, 32, E);
            else pf_qkv(a.layer[li + 1]);
          }))
        return;
    }
    // final RMSNorm + action_out_proj + Euler: x_t += dt * (y . W_out^T + b), x_t_bf16 = bf16(x_t)
    gemm_phase<1, 2, false, true>(
        a, sm, parity, M, a.eh, E, a.ln_f, a.eps, Ad / 16, w_out,
        [&](int task, int m, int j) {
          const int c = task * 16 + j;
          const float2 x = __ldcg(reinterpret_cast<const float2*>(a.xt + static_cast<size_t>(m) * Ad + c));
          return make_uint4(__float_as_uint(x.x), __float_as_uint(x.y),
                            __ldg(reinterpret_cast<const unsigned int*>(a.b_out + c)), 0u);
        },
        [&](int task, int m, int j, float (&v)[1][2], const uint4& p) {
          const size_t i = static_cast<size_t>(m) * Ad + task * 16 + j;
          const float x0 = __fadd_rn(__uint_as_float(p.x), __fmul_rn(a.dt, __fadd_rn(v[0][0], lo(p.z))));
          const float x1 = __fadd_rn(__uint_as_float(p.y), __fmul_rn(a.dt, __fadd_rn(v[0][1], hi(p.z))));
          *reinterpret_cast<float2*>(a.xt + i) = make_float2(x0, x1);
          store2(a.xt_bf + i, x0, x1);
        });
    if (!grid_sync(a, sm, [&] {
          if (step + 1 < a.n_steps) pf_in();
        }))
      return;
  }
}

}  // namespace svla
