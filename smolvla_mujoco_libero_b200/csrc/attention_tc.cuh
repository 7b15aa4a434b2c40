// Attention on the 5th-generation tensor cores (tcgen05), head_dim 64, bf16 in / bf16 (or int8) out, with the
// semantics of the reference's eager attention (deploy/export_6f_layer0_attention_tensors.py:100-119):
//   s = (q . k) * scale (fp32);  s = mask ? s : finfo(f32).min;  o = bf16(softmax(s) @ v)
// (a fully masked row becomes uniform over all keys).  MASK: none (the SigLIP encoder), a byte mask
// [B, Lq, Lk] (the VLM prefix), or the structured mask of the action expert (key padding flags over the first
// mask_keys keys, causal order over the rest).
//
// CTA: 128 packed rows of one (batch, kv head): its G = Hq / Hkv query heads x QT = 128 / G consecutive
// queries, row r = (query q0 + r / G, head kh * G + r % G) -- one 4-D TMA box (dim, head, query, batch) of Q,
// so every key / value tile is loaded once for the whole GQA group.  Keys come from up to two sources (the
// cached prefix, then the current suffix), each a sequence of 64-key tiles.  192 threads; two CTAs per SM.
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
  CUtensorMap tq;          // 4-D map (dim, head, query, batch), box 64 x G x QT x 1, 128-byte swizzle
  CUtensorMap tk, tv;      // source 1: 3-D maps (column, key, batch), box 64 x 64 x 1, 128-byte swizzle
  CUtensorMap tk2, tv2;    // source 2 (L2 > 0)
  const uint8_t* mask;     long long mask_bs; int mask_rs;   // byte mask (single source), rows 16-byte padded
  const uint8_t* key_mask; long long key_mask_bs; int mask_keys;  // structured mask
  __nv_bfloat16* o;        long long o_bs; int o_rs;
  int8_t* qo;              long long qo_bs; int qo_rs;
  const float* qo_smooth;  const float* qo_rsmooth;  float qo_act;
  int Lq, L1, L2, Hq, Hkv, G, QT;
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
constexpr int kKeepBytes = 128 * 8;  // byte mask: one 64-bit keep mask per packed row of a key tile
constexpr int kQ = 0, kK = kQBytes, kV = kK + kStages * kKVBytes, kKeep = kV + kStages * kVStage;
constexpr int kBar = kKeep + kStages * kKeepBytes;
constexpr int kSmemBytes = kBar + 256 + 1024;  // + barriers + alignment slack
// the scaled (log2-domain) score of a masked key: below any real score by far, exactly representable, and
// exp2(kMaskedLog2 - m) is 0 for any real running max m and 1 for m == kMaskedLog2
constexpr float kMaskedLog2 = -1.0e30f;
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

enum TcMask : int { kTcMaskNone = 0, kTcMaskBytes = 1, kTcMaskStructured = 2 };

template <int MASK>
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
  uint64_t* m_full = mma_done + 1;        // [kStages] byte mask: the keep masks of key tile j are in the ring
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(m_full + kStages);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kh = blockIdx.y, b = blockIdx.z;
  const int q0 = blockIdx.x * a.QT;
  const int n1 = (a.L1 + kKeys - 1) / kKeys, n_kv = n1 + (a.L2 + kKeys - 1) / kKeys;
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
    for (int s = 0; s < kStages; ++s) mbar_init(&m_full[s], 1);
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
    // ---------------- TMA producer (lane 0); with a byte mask the whole warp also turns each key tile's mask
    // bytes into one 64-bit keep mask per packed row (lane l: rows 4l .. 4l + 3)
    if (lane == 0) {
      prefetch_tmap(&a.tq);
      prefetch_tmap(&a.tk);
      prefetch_tmap(&a.tv);
      // rows G * QT.. of the Q tile are not loaded: they feed only rows that are never stored
      mbar_arrive_expect_tx(q_full, static_cast<uint32_t>(a.G * a.QT * 128));
      tma_load_4d(smem + kQ, &a.tq, q_full, 0, kh * a.G, q0, b);
    }
    for (int j = 0; j < n_kv; ++j) {
      const int s = j % kStages;
      bool ok = true;
      if (lane == 0 && j >= kStages) ok = mbar_wait(&kv_empty[s], ((j / kStages) - 1) & 1, a.err);
      if (__shfl_sync(0xffffffffu, ok ? 1 : 0, 0) == 0) break;
      const bool src1 = j < n1;
      const int key = (src1 ? j : j - n1) * kKeys;
      if constexpr (MASK == kTcMaskBytes) {
        // single key source: key j * 64 + e of row (query q0 + r / G); the host checked 16-byte aligned rows
        // padded to a multiple of 16 keys, so every 16-key run below L1 is one aligned load
        uint64_t* keep = reinterpret_cast<uint64_t*>(smem + kKeep + s * kKeepBytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int rr = lane * 4 + i, qi = q0 + rr / a.G;
          uint64_t kb = ~0ull;
          if (rr < a.G * a.QT && qi < a.Lq) {
            const uint8_t* mrow = a.mask + static_cast<size_t>(b) * a.mask_bs + static_cast<size_t>(qi) * a.mask_rs;
            kb = 0ull;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
              if (key + c * 16 >= a.L1) continue;
              const uint4 w = __ldg(reinterpret_cast<const uint4*>(mrow + key + c * 16));
              const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint32_t nz = __vcmpne4(ww[u], 0u) & 0x08040201u;  // bit b of byte b: key nonzero
                const uint32_t b4 = (nz | (nz >> 8) | (nz >> 16) | (nz >> 24)) & 0xFu;
                kb |= static_cast<uint64_t>(b4) << (c * 16 + u * 4);
              }
            }
          }
          keep[rr] = kb;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&m_full[s]);
      }
      if (lane == 0) {
        mbar_arrive_expect_tx(&k_full[s], kKVBytes);
        tma_load_3d(smem + kK + s * kKVBytes, src1 ? &a.tk : &a.tk2, &k_full[s], kh * 64, key, b);
        mbar_arrive_expect_tx(&v_full[s], kKVBytes);
        tma_load_3d(smem + kV + s * kVStage, src1 ? &a.tv : &a.tv2, &v_full[s], kh * 64, key, b);
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
    const int rr = wq * 32 + lane;  // packed row: query q0 + rr / G of head kh * G + rr % G
    const int qi = q0 + rr / a.G, hq = kh * a.G + rr % a.G;
    const bool row_in = rr < a.G * a.QT && qi < a.Lq;
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
      const bool src1 = j < n1;
      const int kvalid = src1 ? a.L1 - j * kKeys : a.L2 - (j - n1) * kKeys;  // keys of this tile in its source
      uint64_t keep = ~0ull;  // keys of the tile this row may see (bits past kvalid: don't care, set)
      if constexpr (MASK == kTcMaskStructured) {
        // global key index kg0 + e: flags below kend, causal order (kg - mask_keys <= query) from mask_keys on
        const int kg0 = src1 ? j * kKeys : a.L1 + (j - n1) * kKeys;
        const int kend = a.mask_keys < a.L1 + a.L2 ? a.mask_keys : a.L1 + a.L2;
        const uint8_t* fl = a.key_mask + static_cast<size_t>(b) * a.key_mask_bs;
        keep = 0ull;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int k16 = kg0 + c * 16;
          uint32_t bits = 0u;
          if (k16 < kend) {
            if (((k16 & 15) == 0) && (k16 + 16 <= kend || a.key_mask_bs >= ((kend + 15) & ~15))) {
              const uint4 w = __ldg(reinterpret_cast<const uint4*>(fl + k16));
              const uint32_t ww[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
              for (int u = 0; u < 4; ++u) {
                const uint32_t nz = __vcmpne4(ww[u], 0u) & 0x08040201u;
                bits |= ((nz | (nz >> 8) | (nz >> 16) | (nz >> 24)) & 0xFu) << (u * 4);
              }
            } else {
              for (int e = 0; e < 16 && k16 + e < kend; ++e) bits |= (fl[k16 + e] != 0 ? 1u : 0u) << e;
            }
            if (k16 + 16 > kend) bits &= (1u << (kend - k16)) - 1u;  // keys from kend on: causal rule below
          }
          keep |= static_cast<uint64_t>(bits) << (c * 16);
        }
        // causal part: keys kg >= kend with kg - mask_keys <= qi, i.e. e <= qi + mask_keys - kg0
        const int lo = kend - kg0, hi = qi + a.mask_keys - kg0;  // e in [max(lo, 0), hi]
        const int e0 = lo > 0 ? lo : 0;
        if (hi >= e0 && e0 < kKeys) {
          const int e1 = hi < kKeys - 1 ? hi : kKeys - 1;
          const uint64_t upto = e1 >= 63 ? ~0ull : ((2ull << e1) - 1ull);
          const uint64_t from = (e0 >= 64) ? 0ull : ~((1ull << e0) - 1ull);
          keep |= upto & from;
        }
      } else if constexpr (MASK == kTcMaskBytes) {
        if (!mbar_wait_warp(&m_full[j % kStages], (j / kStages) & 1, a.err)) {
          ok = false;
          break;
        }
        keep = reinterpret_cast<const uint64_t*>(smem + kKeep + (j % kStages) * kKeepBytes)[rr];
      }
      // valid: the tile's keys inside its source; keep: the valid keys this row may see.  A masked key has the
      // score finfo.min in the reference, i.e. probability exp(min - max) = 0 unless every key so far is
      // masked, where all scores tie and the weights are uniform: masked keys take the scaled score
      // kMaskedLog2 below (far under any real score) through the running max, probability
      // exp2(kMaskedLog2 - m) -- 0 against a real maximum, 1 while the row has seen only masked keys.
      const uint64_t valid = kvalid >= kKeys ? ~0ull : ((1ull << kvalid) - 1ull);
      keep &= valid;
      const bool any_masked = keep != valid;
      uint32_t r[kKeys];
#pragma unroll
      for (int ch = 0; ch < kKeys / 32; ++ch) tmem_ld32(tS + ch * 32, *reinterpret_cast<uint32_t(*)[32]>(&r[ch * 32]));
      tmem_ld_wait();
      if constexpr (MASK != kTcMaskNone) {
        if (any_masked) {  // masked keys leave the max and the exponentials (their weight is set below)
          const uint32_t klo = static_cast<uint32_t>(keep), khi = static_cast<uint32_t>(keep >> 32);
#pragma unroll
          for (int e = 0; e < kKeys; ++e) {
            const uint32_t kw = e < 32 ? klo : khi;
            if (((kw >> (e & 31)) & 1u) == 0u) r[e] = __float_as_uint(-INFINITY);
          }
        }
      }
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
      float m_new = fmaxf(m, __fmul_rn(mx, c));  // max of s * c (rounding is monotonic)
      if (MASK != kTcMaskNone && any_masked) m_new = fmaxf(m_new, kMaskedLog2);
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
      const float pm = (MASK != kTcMaskNone && any_masked) ? ex2_approx(kMaskedLog2 - m) : 0.f;
      const uint32_t klo = static_cast<uint32_t>(keep), khi = static_cast<uint32_t>(keep >> 32);
      const uint32_t vlo = static_cast<uint32_t>(valid), vhi = static_cast<uint32_t>(valid >> 32);
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
              // kept: its own weight; masked but valid: pm; past the source's keys: 0
              const uint32_t kw = k0 < 32 ? klo : khi, vw = k0 < 32 ? vlo : vhi;
              const int b0 = k0 & 31;
              p0 = ((kw >> b0) & 1u) ? p0 : (((vw >> b0) & 1u) ? pm : 0.f);
              p1 = ((kw >> (b0 + 1)) & 1u) ? p1 : (((vw >> (b0 + 1)) & 1u) ? pm : 0.f);
            }
            pk[e / 2] = pack_bf16_rn(p0, p1);
          }
          tmem_st16(tS + ch * 16, pk);
        }
      };
      // the choice is warp-uniform: each variant's tcgen05.st is a warp-collective instruction, and the rows of
      // a warp may differ in whether they see a masked key
      if (__all_sync(0xffffffffu, kvalid >= kKeys && !any_masked))
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
        const bool in = row_in;
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
          const int col = hq * 64 + ch * 32;
          if (a.o) {
            __nv_bfloat16* op = a.o + static_cast<size_t>(b) * a.o_bs + static_cast<size_t>(qi) * a.o_rs + col;
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
            int8_t* qp = a.qo + static_cast<size_t>(b) * a.qo_bs + static_cast<size_t>(qi) * a.qo_rs + col;
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
