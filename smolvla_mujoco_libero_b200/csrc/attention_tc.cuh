// Unmasked attention on the 5th-generation tensor cores (tcgen05), head_dim 64, bf16 in / bf16 out:
// the SigLIP encoder's self-attention (deploy/export_6f_layer0_attention_tensors.py:100-119 semantics,
// without a mask):  o = bf16(softmax((q . k) * scale) @ v), fp32 scores, softmax and accumulation.
//
// CTA: one 128-query tile of one (batch, head); 192 threads; two CTAs per SM.
//   warp 0       TMA: the Q tile once, then K and V tiles of 64 keys through a 3-stage ring
//   warp 1       TMEM owner (256 columns) and MMA issuer (one lane):
//                  S_j = Q K_j^T   (M 128, N 64, K 64; both operands from shared memory, K-major)
//                  O  += P_j [V_j | 1]  (M 128, N 80, K 64; P_j from tensor memory, V_j MN-major in shared
//                                        memory next to a tile of ones: columns 64..79 of O accumulate the row
//                                        sums of the bf16 P, so the softmax threads do no additions for them)
//   warps 2-5    softmax: thread t owns TMEM lane t = query row t, so the row max and row sum need no
//                shuffles; the row's 64 scores of a key tile are held in registers (one TMEM read per tile).
//                Lane 0 of each warp polls the mbarriers and broadcasts the result, so 128 threads do not
//                contend for the barrier unit while the MMA warp waits on it too.
// TMEM columns: two S buffers [0,64) and [64,128) (key tile j uses buffer j % 2), O [128,208) (64 output
// columns, then the row sums).  P_j (bf16 pairs) is written over the first 32 columns of its S buffer.
//
// The score tile is double-buffered, so the MMA issue order is QK_0, QK_1, then per key tile j: [P_j ready]
// PV_j, QK_{j+2} into the buffer PV_j has just consumed (the tensor pipe runs one thread's MMAs in order).
// When softmax j ends, S_{j+1} is already computed, so the softmax warps do not wait for the MMA chain; the
// other CTA on the SM fills the gaps between their exponentials.  The softmax is bound by instruction
// latency (about 6.6 cycles per issued instruction per warp), so its loop is kept short: packed FFMA2 for
// the exponent arguments, one exponential per score, one conversion per pair, no per-score additions.
//
// Online softmax with a lazily updated running max (the rescale of O and l happens only when the row max
// grows by more than 8 in log2 units; otherwise the stale max stays and the probabilities, at most 2^8,
// are still exact in bf16's exponent range).  A rescale first waits for the P.V of the previous key tile
// (o_done[(j - 1) % 2]), since that MMA may still be accumulating into O (and the row sums).  The final O / l
// uses the same max for both, so the result is the softmax regardless.  Probabilities exp2(s * scale * log2 e
// - m) are rounded to bf16 for the P.V product, as in the mma.sync kernel, and the row sum is the sum of
// those same bf16 weights (accumulated in fp32), so O / l is exactly their weighted mean of V.
#pragma once

#include <type_traits>

#include "ptx.cuh"

namespace svla {

struct AttnTcArgs {
  CUtensorMap tq;          // 3-D map (column, row, batch), box 64 x 128 x 1, 128-byte swizzle
  CUtensorMap tk, tv;      // 3-D maps, box 64 x 64 x 1, 128-byte swizzle
  __nv_bfloat16* o;        long long o_bs; int o_rs;
  int8_t* qo;              long long qo_bs; int qo_rs;
  const float* qo_smooth;  const float* qo_rsmooth;  float qo_act;
  int Lq, Lk, Hq, Hkv;
  float scale_log2;  // scale * log2(e)
  unsigned long long* dbg;  // optional phase clock stamps of the CTA (0, 0, batch / 2) (profiling)
  int* err;
};

// max of three floats in one instruction (the three-input form of max.f32, sm_100)
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

namespace atc {
constexpr int kKeys = 64;                   // keys per tile
constexpr int kQBytes = 128 * 128;          // 128 query rows x 64 bf16
constexpr int kKVBytes = kKeys * 128;       // 64 key rows x 64 bf16
constexpr int kStages = 3;
constexpr int kVStage = 2 * kKVBytes;  // V tile, then a tile of bf16 ones (the row-sum columns of the P.V MMA)
constexpr int kQ = 0, kK = kQBytes, kV = kK + kStages * kKVBytes, kBar = kV + kStages * kVStage;
constexpr int kSmemBytes = kBar + 256 + 1024;  // + barriers + alignment slack
constexpr int kThreads = 192;
constexpr int kSBufs = 2;
constexpr uint32_t kS = 0, kO = kSBufs * kKeys, kTmemCols = 256;  // O: 64 columns + 16 row-sum columns
}  // namespace atc

// warp-uniform bounded wait with one polling lane
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, int* err) {
  bool ok = true;
  if ((threadIdx.x & 31) == 0) ok = mbar_wait(bar, parity, err);
  return __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
}

__global__ void __launch_bounds__(atc::kThreads, 2) attention_tc_kernel(const __grid_constant__ AttnTcArgs a) {
  using namespace atc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + kBar);
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [kSBufs] score buffer holds S_j
  uint64_t* p_full = s_full + kSBufs;     // [kSBufs] score buffer holds P_j
  uint64_t* o_done = p_full + kSBufs;     // [2] P.V of key tile j (and all before it) done: o_done[j % 2]
  uint64_t* o_full = o_done + 2;          // the last P.V has completed
  uint64_t* mma_done = o_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (a.Hq / a.Hkv);
  const int q0 = blockIdx.x * 128;
  const int n_kv = (a.Lk + kKeys - 1) / kKeys;
  unsigned long long* dbg = (a.dbg && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == gridDim.z / 2) ? a.dbg : nullptr;
  auto stamp = [&](int slot) {
    if (dbg) dbg[slot] = clock64();
  };
  if (threadIdx.x == 0) stamp(0);

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&kv_empty[s], 1);
    }
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrive per softmax warp
    }
    mbar_init(&o_done[0], 1);
    mbar_init(&o_done[1], 1);
    mbar_init(o_full, 1);
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
  }
  if (warp >= 2) {  // the ones tiles beside the V stages (bf16 1.0 everywhere, so the swizzle is moot)
    for (int i = threadIdx.x - 64; i < kStages * kKVBytes / 16; i += 128) {
      const int st = i / (kKVBytes / 16), w = i % (kKVBytes / 16);
      *reinterpret_cast<int4*>(smem + kV + st * kVStage + kKVBytes + w * 16) =
          make_int4(0x3F803F80, 0x3F803F80, 0x3F803F80, 0x3F803F80);
    }
    fence_proxy_async_smem();  // generic-proxy writes -> visible to the tensor core
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  pdl_wait();  // q, k, v are written by the previous kernel
  pdl_trigger();
  if (threadIdx.x == 0) stamp(1);

  if (warp == 0) {
    // ---------------- TMA producer
    if (lane == 0) {
      prefetch_tmap(&a.tq);
      prefetch_tmap(&a.tk);
      prefetch_tmap(&a.tv);
      mbar_arrive_expect_tx(q_full, kQBytes);
      tma_load_3d(smem + kQ, &a.tq, q_full, h * 64, q0, b);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, a.err)) break;
        mbar_arrive_expect_tx(&k_full[s], kKVBytes);
        tma_load_3d(smem + kK + s * kKVBytes, &a.tk, &k_full[s], kh * 64, j * kKeys, b);
        mbar_arrive_expect_tx(&v_full[s], kKVBytes);
        tma_load_3d(smem + kV + s * kVStage, &a.tv, &v_full[s], kh * 64, j * kKeys, b);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_bf16(128, kKeys);
      const uint32_t id_pv = idesc_bf16(128, 80) | (1u << 16);  // B ([V | 1]) MN-major, N 80
      bool issued = false;
      const uint32_t qa = smem_u32(smem + kQ);
      auto qk = [&](int j) -> bool {  // S_j into buffer j % 3
        const int s = j % kStages;
        if (!mbar_wait(&k_full[s], (j / kStages) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t ka = smem_u32(smem + kK + s * kKVBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 16 head dims (32 bytes) per MMA
          mma_bf16(tmem + kS + (j % kSBufs) * kKeys, smem_desc_sw128(qa + kk * 32), smem_desc_sw128(ka + kk * 32),
                   id_qk, kk > 0 ? 1u : 0u);
        mma_commit(&s_full[j % kSBufs]);
        issued = true;
        return true;
      };
      auto pv = [&](int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&v_full[s], (j / kStages) & 1, a.err)) return false;
        if (!mbar_wait(&p_full[j % kSBufs], (j / kSBufs) & 1, a.err)) return false;
        if (j < 8) stamp(8 + j);
        tc_fence_after();
        const uint32_t va = smem_u32(smem + kV + s * kVStage);
#pragma unroll
        for (int kk = 0; kk < kKeys / 16; ++kk)  // 16 keys per MMA: 8 TMEM columns of P, 16 rows (2048 bytes) of V;
                                                 // columns 64.. of B are the ones tile kKVBytes further on
          mma_bf16_tmem_a(tmem + kO, tmem + kS + (j % kSBufs) * kKeys + kk * 8,
                          smem_desc_sw128_lbo(va + kk * 2048, kKVBytes), id_pv, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&o_done[j & 1]);
        mma_commit(&kv_empty[s]);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, a.err);
      stamp(2);
      for (int j = 0; j < kSBufs && j < n_kv && ok; ++j) ok = qk(j);
      for (int j = 0; j < n_kv && ok; ++j) {
        ok = pv(j);
        if (j < 8) stamp(16 + j);
        if (ok && j + kSBufs < n_kv) ok = qk(j + kSBufs);
      }
      if (ok) mma_commit(o_full);
      // every issued MMA completes before the TMEM is released
      if (issued) {
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, a.err);
      }
    }
  } else {
    // ---------------- softmax warpgroup
    const int wq = warp & 3;  // TMEM lane quarter
    const int row = q0 + wq * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tO = tmem + lanes + kO;
    const float c = a.scale_log2;
    float m = -INFINITY;
    bool ok = true;
    for (int j = 0; j < n_kv && ok; ++j) {
      const uint32_t tS = tmem + lanes + kS + (j % kSBufs) * kKeys;
      ok = mbar_wait_warp(&s_full[j % kSBufs], (j / kSBufs) & 1, a.err);
      if (!ok) break;
      const bool st0 = (wq == 0 && lane == 0 && j < 8);
      if (st0) stamp(32 + j);
      tc_fence_after();
      const int kvalid = a.Lk - j * kKeys;  // keys of this tile inside Lk
      uint32_t r[kKeys];
#pragma unroll
      for (int ch = 0; ch < kKeys / 32; ++ch) tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[ch * 32]));
      tmem_ld_wait();
      if (st0) stamp(56 + j);
      // row max with 8 independent partial maxima (short dependency chains); the three-input max does two
      // comparisons per instruction at the two-input rate
      float mp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mp[u] = -INFINITY;
      if (kvalid >= kKeys) {
#pragma unroll
        for (int e = 0; e < kKeys; e += 2) mp[(e >> 1) & 7] = max3f(mp[(e >> 1) & 7], __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
      } else {
#pragma unroll
        for (int e = 0; e < kKeys; ++e) mp[e & 7] = (e < kvalid) ? fmaxf(mp[e & 7], __uint_as_float(r[e])) : mp[e & 7];
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      const float m_new = fmaxf(m, __fmul_rn(mx, c));  // max of s * c (rounding is monotonic)
      float alpha = 1.0f;
      bool grow = false;
      if (st0) stamp(64 + j);
      if (j == 0) {
        m = m_new;  // the first P.V overwrites O
      } else if (m_new > m + 8.0f) {
        grow = true;
        alpha = ex2_approx(m - m_new);
        m = m_new;
      }
      // O rescale (rare after the first tiles): wait for the previous key tile's P.V, which may still be
      // accumulating into O; the next P.V waits for this warpgroup's arrival below.  o_done[(j-1) % 2]
      // completes once per two key tiles; the P.V of tile j - 2 had completed before S_j was computed, so the
      // phase for tile j - 1 is the one pending or just completed.  The row-sum columns are rescaled too.
      if (__any_sync(0xffffffffu, grow)) {
        ok = mbar_wait_warp(&o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, a.err);
        if (!ok) break;
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t o32[32];
          tmem_ld32(tO + ch * 32, o32);
          tmem_ld_wait();
          uint32_t w0[16], w1[16];
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            w0[e] = __float_as_uint(__fmul_rn(__uint_as_float(o32[e]), alpha));
            w1[e] = __float_as_uint(__fmul_rn(__uint_as_float(o32[16 + e]), alpha));
          }
          tmem_st16(tO + ch * 32, w0);
          tmem_st16(tO + ch * 32 + 16, w1);
        }
        uint32_t l16[16];
        tmem_ld16(tO + 64, l16);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 16; ++e) l16[e] = __float_as_uint(__fmul_rn(__uint_as_float(l16[e]), alpha));
        tmem_st16(tO + 64, l16);
      }
      // probabilities: bf16 P over the first 32 columns of the S buffer, the exponent arguments through the
      // packed fp32 pipe (FFMA2).  Keys past Lk (last tile only) get probability 0; full tiles take a loop
      // without those selects.
      const float2 c2 = make_float2(c, c), nm2 = make_float2(-m, -m);
      auto exps = [&](auto masked) {
#pragma unroll
        for (int ch = 0; ch < kKeys / 32; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const int k0 = ch * 32 + e;
            const float2 z = __ffma2_rn(make_float2(__uint_as_float(r[k0]), __uint_as_float(r[k0 + 1])), c2, nm2);
            float p0 = ex2_approx(z.x);
            float p1 = ex2_approx(z.y);
            if constexpr (decltype(masked)::value) {
              p0 = (k0 < kvalid) ? p0 : 0.f;
              p1 = (k0 + 1 < kvalid) ? p1 : 0.f;
            }
            pk[e / 2] = pack_bf16_rn(p0, p1);
          }
          tmem_st16(tS + ch * 16, pk);
        }
      };
      if (kvalid >= kKeys)
        exps(std::false_type{});
      else
        exps(std::true_type{});
      if (st0) stamp(72 + j);
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[j % kSBufs]);
      if (st0) stamp(48 + j);
    }
    // epilogue: O / l -> bf16 (and the int8 input of the next W8A8 linear)
    if (ok) {
      ok = mbar_wait_warp(o_full, 0, a.err);
      tc_fence_after();
      if (wq == 0 && lane == 0) stamp(90);
      if (ok) {
        uint32_t l16[16];
        tmem_ld16(tO + 64, l16);  // the row sum of the bf16 weights (every one of these columns holds it)
        tmem_ld_wait();
        const float inv = __frcp_rn(__uint_as_float(l16[0]));
        const float ra = (a.qo && a.qo_rsmooth) ? __frcp_rn(a.qo_act) : 0.f;
        const bool in = row < a.Lq;
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t r[32];
          tmem_ld32(tO + ch * 32, r);
          tmem_ld_wait();
          if (!in) continue;
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            v[e] = __fmul_rn(__uint_as_float(r[e]), inv);
            v[e + 1] = __fmul_rn(__uint_as_float(r[e + 1]), inv);
            bf16_round2(v[e], v[e + 1]);
          }
          const int col = h * 64 + ch * 32;
          if (a.o) {
            __nv_bfloat16* op = a.o + static_cast<size_t>(b) * a.o_bs + static_cast<size_t>(row) * a.o_rs + col;
#pragma unroll
            for (int u = 0; u < 4; ++u)
              *reinterpret_cast<int4*>(op + u * 8) =
                  make_int4(pack_bf16_rn(v[8 * u], v[8 * u + 1]), pack_bf16_rn(v[8 * u + 2], v[8 * u + 3]),
                            pack_bf16_rn(v[8 * u + 4], v[8 * u + 5]), pack_bf16_rn(v[8 * u + 6], v[8 * u + 7]));
          }
          if (a.qo) {
            uint32_t w[8] = {0u, 0u, 0u, 0u, 0u, 0u, 0u, 0u};
            uint32_t slow = a.qo_rsmooth ? 0u : 0xFFFFFFFFu;
            if (a.qo_rsmooth) {
#pragma unroll
              for (int k = 0; k < 8; ++k) {
                uint32_t sk = 0u;
                w[k] = smooth_quant4_fast(&v[4 * k], *reinterpret_cast<const float4*>(a.qo_rsmooth + col + 4 * k), ra,
                                          sk, 0);
                slow |= sk << (4 * k);
              }
            }
            if (slow != 0u) {  // rare: values near a rounding boundary take the two-divide path one by one
#pragma unroll
              for (int e = 0; e < 32; ++e) {
                if (slow & (1u << e)) {
                  const uint32_t q8 = static_cast<uint32_t>(smooth_quant_slow(v[e], a.qo_smooth[col + e], a.qo_act) & 0xFF);
                  w[e / 4] = (w[e / 4] & ~(0xFFu << (8 * (e % 4)))) | (q8 << (8 * (e % 4)));
                }
              }
            }
            int8_t* qp = a.qo + static_cast<size_t>(b) * a.qo_bs + static_cast<size_t>(row) * a.qo_rs + col;
            *reinterpret_cast<int4*>(qp) = make_int4(w[0], w[1], w[2], w[3]);
            *reinterpret_cast<int4*>(qp + 16) = make_int4(w[4], w[5], w[6], w[7]);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0) stamp(95);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace svla
