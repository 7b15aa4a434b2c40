// Unmasked attention on the 5th-generation tensor cores (tcgen05), head_dim 64, bf16 in / bf16 out:
// the SigLIP encoder's self-attention (deploy/export_6f_layer0_attention_tensors.py:100-119 semantics,
// without a mask):  o = bf16(softmax((q . k) * scale) @ v), fp32 scores, softmax and accumulation.
//
// CTA: two 128-query tiles of one (batch, head), 320 threads.
//   warp 0       TMA: both Q tiles once, then K and V tiles of 128 keys through a 4-stage ring
//   warp 1       TMEM owner (512 columns) and MMA issuer (one lane):
//                  S_i = Q_i K_j^T   (M 128, N 128, K 64; both operands from shared memory, K-major)
//                  O_i += P_i V_j    (M 128, N 64, K 128; P_i from tensor memory, V_j MN-major in smem)
//   warps 2-5    softmax of query tile 0, warps 6-9 of tile 1 (warp w reads TMEM lanes 32*(w%4)..+31):
//                thread t owns TMEM lane t = query row t, so the row max and row sum need no shuffles; the
//                row's 128 scores of a key tile are held in registers (one TMEM read per tile).
// TMEM columns: S_0 [0,128)  S_1 [128,256)  O_0 [256,320)  O_1 [320,384).  P_i (bf16 pairs) is written over
// the first 64 columns of S_i.  The MMA issue order (P.V of tile 0, next Q.K^T of tile 0, P.V of tile 1,
// next Q.K^T of tile 1) lets the two softmax warpgroups settle half a period apart, so the MMAs of one
// query tile run while the other's softmax computes.
//
// The library launches the single-tile form (PAIR = false): one 128-query tile per CTA, 192 threads
// (warps 0, 1 and one softmax warpgroup), a 2-stage K/V ring, 256 TMEM columns (S_0 [0,128), O_0 [128,192)),
// 83 KB of shared memory, so two CTAs share an SM.  The two CTAs take the ping-pong role of the two tiles
// without a common MMA issue order, and one CTA's set-up (TMEM allocation, Q load) and epilogue overlap the
// other's key loop: measured 957 -> 854 us for 128 images x 12 heads x 1024^2 against the pair form.
//
// Online softmax with a lazily updated running max (the rescale of O and l happens only when the row max
// grows by more than 8 in log2 units; otherwise the stale max stays and the probabilities, at most 2^8,
// are still exact in bf16's exponent range).  The final O / l uses the same max for both, so the result
// is the softmax regardless.  Probabilities exp2(s * scale * log2 e - m) are rounded to bf16 for the
// P.V product, as in the mma.sync kernel; the row sum uses the unrounded values.
#pragma once

#include "ptx.cuh"

namespace svla {

struct AttnTcArgs {
  CUtensorMap tq, tk, tv;  // 3-D maps (column, row, batch), box 64 x 128 x 1, 128-byte swizzle
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
constexpr int kTileBytes = 128 * 128;  // 128 rows x 64 bf16
// PAIR: two 128-query tiles per CTA (320 threads, 4 K/V stages, 512 TMEM columns, one CTA per SM);
// otherwise one tile per CTA (192 threads, 2 K/V stages, 256 TMEM columns) so that two CTAs share an SM
template <bool PAIR>
struct Cfg {
  static constexpr int kStages = PAIR ? 4 : 2;
  static constexpr int kQTiles = PAIR ? 2 : 1;
  static constexpr int kQ0 = 0, kQ1 = kTileBytes, kK = kQTiles * kTileBytes, kV = kK + kStages * kTileBytes;
  static constexpr int kBar = kV + kStages * kTileBytes;
  static constexpr int kSmemBytes = kBar + 256 + 1024;  // + barriers + alignment slack
  static constexpr int kThreads = PAIR ? 320 : 192;
  static constexpr uint32_t kS0 = 0, kS1 = 128, kO0 = PAIR ? 256 : 128, kO1 = 320, kTmemCols = PAIR ? 512 : 256;
};
}  // namespace atc

template <bool PAIR>
__global__ void __launch_bounds__(atc::Cfg<PAIR>::kThreads, PAIR ? 1 : 2)
    attention_tc_kernel(const __grid_constant__ AttnTcArgs a) {
  using C = atc::Cfg<PAIR>;
  constexpr int kTileBytes = atc::kTileBytes, kStages = C::kStages;
  constexpr int kQ0 = C::kQ0, kQ1 = C::kQ1, kK = C::kK, kV = C::kV, kBar = C::kBar;
  constexpr uint32_t kS0 = C::kS0, kS1 = C::kS1, kO0 = C::kO0, kO1 = C::kO1, kTmemCols = C::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* q_full = reinterpret_cast<uint64_t*>(smem + kBar);
  uint64_t* k_full = q_full + 1;
  uint64_t* v_full = k_full + kStages;
  uint64_t* kv_empty = v_full + kStages;
  uint64_t* s_full = kv_empty + kStages;  // [2]
  uint64_t* p_full = s_full + 2;          // [2]
  uint64_t* o_full = p_full + 2;          // [2]
  uint64_t* mma_done = o_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(mma_done + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (a.Hq / a.Hkv);
  const int q0 = blockIdx.x * 128 * C::kQTiles;
  const bool two = PAIR && q0 + 128 < a.Lq;  // the second query tile has rows
  const int n_kv = (a.Lk + 127) / 128;
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
    for (int i = 0; i < 2; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);  // one arrive per softmax warp
      mbar_init(&o_full[i], 1);
    }
    mbar_init(mma_done, 1);
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, kTmemCols);
    tmem_relinquish();
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
      mbar_arrive_expect_tx(q_full, (two ? 2 : 1) * kTileBytes);
      tma_load_3d(smem + kQ0, &a.tq, q_full, h * 64, q0, b);
      if (two) tma_load_3d(smem + kQ1, &a.tq, q_full, h * 64, q0 + 128, b);
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % kStages;
        if (j >= kStages && !mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, a.err)) break;
        mbar_arrive_expect_tx(&k_full[s], kTileBytes);
        tma_load_3d(smem + kK + s * kTileBytes, &a.tk, &k_full[s], kh * 64, j * 128, b);
        mbar_arrive_expect_tx(&v_full[s], kTileBytes);
        tma_load_3d(smem + kV + s * kTileBytes, &a.tv, &v_full[s], kh * 64, j * 128, b);
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer
    if (lane == 0) {
      const uint32_t id_qk = idesc_bf16(128, 128);
      const uint32_t id_pv = idesc_bf16(128, 64) | (1u << 16);  // B (V) MN-major
      bool issued = false;
      auto qk = [&](int i, int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&k_full[s], (j / kStages) & 1, a.err)) return false;
        tc_fence_after();
        const uint32_t qa = smem_u32(smem + (i ? kQ1 : kQ0)), ka = smem_u32(smem + kK + s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)  // 16 head dims (32 bytes) per MMA
          mma_bf16(tmem + (i ? kS1 : kS0), smem_desc_sw128(qa + kk * 32), smem_desc_sw128(ka + kk * 32), id_qk,
                   kk > 0 ? 1u : 0u);
        mma_commit(&s_full[i]);
        issued = true;
        return true;
      };
      auto pv = [&](int i, int j) -> bool {
        const int s = j % kStages;
        if (!mbar_wait(&v_full[s], (j / kStages) & 1, a.err)) return false;
        if (!mbar_wait(&p_full[i], j & 1, a.err)) return false;
        if (i == 0 && j < 8) stamp(8 + j);
        tc_fence_after();
        const uint32_t va = smem_u32(smem + kV + s * kTileBytes);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)  // 16 keys per MMA: 8 TMEM columns of P, 16 rows (2048 bytes) of V
          mma_bf16_tmem_a(tmem + (i ? kO1 : kO0), tmem + (i ? kS1 : kS0) + kk * 8, smem_desc_sw128(va + kk * 2048),
                          id_pv, (j > 0 || kk > 0) ? 1u : 0u);
        return true;
      };
      bool ok = mbar_wait(q_full, 0, a.err);
      stamp(2);
      ok = ok && qk(0, 0) && (!two || qk(1, 0));
      for (int j = 0; j < n_kv && ok; ++j) {
        ok = pv(0, j);
        if (j < 8) stamp(16 + j);
        if (ok && j + 1 < n_kv) ok = qk(0, j + 1);
        if (ok && two) ok = pv(1, j);
        if (j < 8) stamp(24 + j);
        if (ok) mma_commit(&kv_empty[j % kStages]);
        if (ok && two && j + 1 < n_kv) ok = qk(1, j + 1);
      }
      if (ok) {
        mma_commit(&o_full[0]);
        if (two) mma_commit(&o_full[1]);
      }
      // every issued MMA completes before the TMEM is released
      if (issued) {
        mma_commit(mma_done);
        mbar_wait(mma_done, 0, a.err);
      }
    }
  } else {
    // ---------------- softmax warpgroups
    const int i = (warp - 2) >> 2;  // query tile
    const int wq = warp & 3;        // TMEM lane quarter
    const int row = q0 + i * 128 + wq * 32 + lane;
    const uint32_t lanes = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lanes + (i ? kS1 : kS0);
    const uint32_t tO = tmem + lanes + (i ? kO1 : kO0);
    const float c = a.scale_log2;
    float m = -INFINITY, l = 0.f;
    bool ok = (i == 0) || two;
    const bool active = ok;
    for (int j = 0; j < n_kv && ok; ++j) {
      ok = __all_sync(0xffffffffu, mbar_wait(&s_full[i], j & 1, a.err));
      if (!ok) break;
      const bool st0 = (wq == 0 && lane == 0 && j < 8);
      if (st0) stamp(i ? 56 + j : 32 + j);
      tc_fence_after();
      const int kvalid = a.Lk - j * 128;  // keys of this tile inside Lk
      uint32_t r[128];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[ch * 32]));
      tmem_ld_wait();
      // row max with 8 independent partial maxima (short dependency chains)
      float mp[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) mp[u] = -INFINITY;
      if (kvalid >= 128) {
#pragma unroll
        for (int e = 0; e < 128; e += 2) mp[(e >> 1) & 7] = max3f(mp[(e >> 1) & 7], __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
      } else {
#pragma unroll
        for (int e = 0; e < 128; ++e) mp[e & 7] = (e < kvalid) ? fmaxf(mp[e & 7], __uint_as_float(r[e])) : mp[e & 7];
      }
      const float mx = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
      const float m_new = fmaxf(m, __fmul_rn(mx, c));  // max of s * c (rounding is monotonic)
      float alpha = 1.0f;
      bool grow = false;
      if (j == 0) {
        m = m_new;  // the first P.V overwrites O
      } else if (m_new > m + 8.0f) {
        grow = true;
        alpha = ex2_approx(m - m_new);
        m = m_new;
      }
      // probabilities and row sum; bf16 P over the first 64 columns of S (all of S is in registers).
      // Pairs of scores go through the packed fp32 pipe (FFMA2 for the exponent arguments, FADD2 for the
      // row sum, kept as 8 partial sums in 4 packed accumulators).
      float2 lp[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) lp[u] = make_float2(0.f, 0.f);
      const float2 c2 = make_float2(c, c), nm2 = make_float2(-m, -m);
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int k0 = ch * 32 + e;
          const float2 z = __ffma2_rn(make_float2(__uint_as_float(r[k0]), __uint_as_float(r[k0 + 1])), c2, nm2);
          float p0 = ex2_approx(z.x);
          float p1 = ex2_approx(z.y);
          if (kvalid < 128) {
            p0 = (k0 < kvalid) ? p0 : 0.f;
            p1 = (k0 + 1 < kvalid) ? p1 : 0.f;
          }
          lp[(e / 2) & 3] = __fadd2_rn(lp[(e / 2) & 3], make_float2(p0, p1));
          pk[e / 2] = pack_bf16_rn(p0, p1);
        }
        tmem_st16(tS + ch * 16, pk);
      }
      const float ls = ((lp[0].x + lp[0].y) + (lp[1].x + lp[1].y)) + ((lp[2].x + lp[2].y) + (lp[3].x + lp[3].y));
      l = __fmaf_rn(l, alpha, ls);
      // O rescale (rare after the first tiles): the previous P.V has completed -- its commit preceded the
      // S of this tile -- and the next one waits for this warpgroup's arrival below
      if (__any_sync(0xffffffffu, grow)) {
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
      }
      tmem_st_wait();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&p_full[i]);
      if (st0) stamp(i ? 64 + j : 48 + j);
      if (lane == 0 && j < 2) stamp((i ? 72 : 40) + 4 * j + wq);
    }
    // epilogue: O / l -> bf16 (and the int8 input of the next W8A8 linear)
    if (active && ok) {
      ok = __all_sync(0xffffffffu, mbar_wait(&o_full[i], 0, a.err));
      tc_fence_after();
      if (wq == 0 && lane == 0) stamp(90 + 2 * i);
      if (ok) {
        const float inv = __frcp_rn(l);
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
