// Masked GQA attention, head_dim 64, bf16 in / bf16 out, fp32 scores and softmax.
//
// Semantics follow the reference's eager attention (deploy/export_6f_layer0_attention_tensors.py:100-119;
// lerobot eager_attention_forward):
//   s = (q . k) * d^-1/2                    (fp32)
//   s = mask ? s : finfo(f32).min           (a fully masked row therefore becomes uniform over ALL keys)
//   o = bf16(softmax(s) @ v)                (fp32 accumulation)
// Query head h reads key/value head h / (Hq / Hkv).
//
// One pass over the keys with an online softmax (running max m, running sum l, O rescaled when m grows):
// probabilities exp(s - m) are rounded to bf16 for the tensor-core P.V and O is divided by l at the end.
// The reference rounds the already-normalised probabilities instead; both roundings are 2^-9 relative
// per term (bf16), well inside the stated tolerance.
//
// CTA: one (row tile, kv head, batch).  The rows of a kv head are its G = Hq / Hkv query heads' queries
// packed head-major (row r = query head kh*G + r / Lq, query r % Lq), so every key/value tile is loaded
// once for the whole group and short query lengths fill the tiles; a tile is 16 x warps rows, up to 128.
// Keys stream in tiles of 64 through a two-stage cp.async pipeline; keys may come from two sources (the
// cached prefix followed by the current suffix).  Tensor-core work is mma.sync m16n8k16 with ldmatrix
// fragments; exponentials are ex2.approx.
//
// Optional fused output quantisation (the o_proj input of a W8A8 layer):
//   qo[m, h*64 + d] = round((o / s[h*64+d]) / a).clamp(-128, 127).
#pragma once

#include "ptx.cuh"

namespace svla {

struct AttnArgs {
  const __nv_bfloat16* q;  long long q_bs; int q_rs;       // q[b*q_bs + i*q_rs + h*64 + d]
  const __nv_bfloat16* k1; const __nv_bfloat16* v1; long long kv1_bs; int kv1_rs; int L1;
  const __nv_bfloat16* k2; const __nv_bfloat16* v2; long long kv2_bs; int kv2_rs; int L2;
  const uint8_t* mask;     long long mask_bs; int mask_rs;  // mask[b*mask_bs + i*mask_rs + key] or nullptr
  // structured mask (instead of `mask`): key < mask_keys ? key_mask[b*key_mask_bs + key] : key - mask_keys <= i
  const uint8_t* key_mask; long long key_mask_bs; int mask_keys;
  __nv_bfloat16* o;        long long o_bs; int o_rs;        // optional bf16 output
  int8_t* qo;              long long qo_bs; int qo_rs;      // optional int8 output
  const float* qo_smooth;  const float* qo_rsmooth;  float qo_act;
  int Lq, Hq, Hkv;
  float scale;
  int rows;  // packed rows per CTA: 16 x warps, at most 128
};

namespace attn_detail {
constexpr int kD = 64;
constexpr int kRows = 128;    // most packed rows per CTA
constexpr int kWarps = kRows / 16;
constexpr int kKeys = 64;     // keys per tile
constexpr int kPad = 72;      // smem row (bf16): 144 bytes -> conflict-free ldmatrix
constexpr float kMaskedScore = -3.4028234663852886e38f;  // torch.finfo(torch.float32).min
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// 16-byte cp.async; src_bytes = 0 fills the destination with zeros
__device__ __forceinline__ void cp_async16(void* dst, const void* src, int src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) { return pack_bf16_rn(lo, hi); }

struct Smem {
  __nv_bfloat16 q[kRows * kPad];
  __nv_bfloat16 k[2][kKeys * kPad];
  __nv_bfloat16 v[2][kKeys * kPad];
  uint8_t m[2][kRows * kKeys];
};

// Mask kinds, a template parameter of the kernel so that the per-score mask test is resolved at compile time
enum MaskKind : int { kMaskNone = 0, kMaskBytes = 1, kMaskStructured = 2 };

// issue the cp.async copies of key tile `tile` (keys key0 .. key0+63) of kv head kh into stage st
template <int MK>
__device__ __forceinline__ void load_kv_tile(const AttnArgs& a, Smem& sm, int st, int b, int kh, int key0) {
  const int Lk = a.L1 + a.L2;
  for (int idx = threadIdx.x; idx < kKeys * 8; idx += blockDim.x) {
    const int r = idx >> 3, c = (idx & 7) * 8;
    const int key = key0 + r;
    const __nv_bfloat16* kp = a.k1;
    const __nv_bfloat16* vp = a.v1;
    int bytes = 0;
    if (key < Lk) {
      bytes = 16;
      if (key < a.L1) {
        const size_t off = static_cast<size_t>(b) * a.kv1_bs + static_cast<size_t>(key) * a.kv1_rs + kh * kD + c;
        kp = a.k1 + off;
        vp = a.v1 + off;
      } else {
        const size_t off =
            static_cast<size_t>(b) * a.kv2_bs + static_cast<size_t>(key - a.L1) * a.kv2_rs + kh * kD + c;
        kp = a.k2 + off;
        vp = a.v2 + off;
      }
    }
    cp_async16(&sm.k[st][r * kPad + c], kp, bytes);
    cp_async16(&sm.v[st][r * kPad + c], vp, bytes);
  }
  if constexpr (MK == kMaskStructured) {
    // structured mask: one row of key flags (keys below mask_keys) for every query of the tile
    if (threadIdx.x < 4) {
      const int c = threadIdx.x * 16, key = key0 + c;
      const int kend = a.mask_keys < Lk ? a.mask_keys : Lk;
      const uint8_t* src = a.key_mask + static_cast<size_t>(b) * a.key_mask_bs;
      uint8_t* dst = &sm.m[st][c];
      // a whole aligned 16-key run is one async copy when it lies inside the flags or inside the row's storage
      // (row stride covering the flags rounded up to 16); runs past the flags are zero-filled
      const bool padded = a.key_mask_bs >= ((kend + 15) & ~15);
      if (key >= kend) {
        cp_async16(dst, src, 0);
      } else if ((key + 16 <= kend || padded) && ((reinterpret_cast<uintptr_t>(src + key) & 15) == 0)) {
        cp_async16(dst, src + key, 16);
      } else {
        for (int j = 0; j < 16; ++j) dst[j] = (key + j < kend) ? src[key + j] : 0;
      }
    }
  } else if constexpr (MK == kMaskBytes) {
    // mask bytes [128 rows x 64 keys]; rows past Lq and keys past Lk are left as whatever they read:
    // the scores of keys past Lk are forced to -inf and rows past Lq are never stored.  A 16-key run is
    // one 16-byte copy when it is aligned and lies inside the row's storage (the row stride covers Lk
    // rounded up to 16: then even the last, partial run stays in bounds); runs past Lk are zero-filled.
    const int r0 = blockIdx.x * a.rows, R = a.Lq * (a.Hq / a.Hkv);
    const bool padded_rows = a.mask_rs >= ((Lk + 15) & ~15);
    for (int idx = threadIdx.x; idx < a.rows * 4; idx += blockDim.x) {
      const int r = idx >> 2, c = (idx & 3) * 16;
      const int query = (r0 + r < R) ? (r0 + r) % a.Lq : 0, key = key0 + c;
      const uint8_t* src = a.mask + static_cast<size_t>(b) * a.mask_bs + static_cast<size_t>(query) * a.mask_rs;
      uint8_t* dst = &sm.m[st][r * kKeys + c];
      if (key >= Lk) {
        cp_async16(dst, src, 0);
      } else if ((key + 16 <= Lk || padded_rows) && ((reinterpret_cast<uintptr_t>(src + key) & 15) == 0)) {
        cp_async16(dst, src + key, 16);
      } else {
        for (int j = 0; j < 16; ++j) dst[j] = (key + j < Lk) ? src[key + j] : 0;
      }
    }
  }
}
}  // namespace attn_detail

template <int MK>
__global__ void __launch_bounds__(attn_detail::kRows * 2, 2) attention_kernel(const AttnArgs a) {
  pdl_wait();
  pdl_trigger();
  using namespace attn_detail;
  extern __shared__ __align__(16) uint8_t smem_raw[];
  Smem& sm = *reinterpret_cast<Smem*>(smem_raw);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int kh = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.Hkv, R = G * a.Lq;  // packed rows of this kv head
  const int r0 = blockIdx.x * a.rows;
  const int Lk = a.L1 + a.L2;
  const int n_tiles = (Lk + kKeys - 1) / kKeys;

  // Q tile -> smem (zero rows beyond the packed rows), first K/V tile in flight
  {
    const __nv_bfloat16* qb = a.q + static_cast<size_t>(b) * a.q_bs + kh * G * kD;
    for (int idx = threadIdx.x; idx < a.rows * 8; idx += blockDim.x) {
      const int r = idx >> 3, c = (idx & 7) * 8;
      const int pr = r0 + r;
      const bool in = pr < R;
      const int hg = in ? pr / a.Lq : 0, query = in ? pr % a.Lq : 0;
      cp_async16(&sm.q[r * kPad + c], qb + static_cast<size_t>(query) * a.q_rs + hg * kD + c, in ? 16 : 0);
    }
  }
  load_kv_tile<MK>(a, sm, 0, b, kh, 0);
  cp_async_commit();

  uint32_t qa[4][4];
  float o[8][4];
  int query[2];  // query index of this thread's two rows (structured mask)
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int pr = r0 + warp * 16 + g + hr * 8;
    query[hr] = pr < R ? pr % a.Lq : 0;
  }
#pragma unroll
  for (int n = 0; n < 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mx[2] = {-INFINITY, -INFINITY}, l[2] = {0.f, 0.f};
  const int wr = warp * 16;  // this warp's first row inside the CTA tile

  for (int tile = 0; tile < n_tiles; ++tile) {
    const int st = tile & 1;
    if (tile + 1 < n_tiles) {
      load_kv_tile<MK>(a, sm, st ^ 1, b, kh, (tile + 1) * kKeys);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    if (tile == 0) {
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        // A fragments: rows wr + (lane & 15), columns kk*16 + (lane >> 4) * 8
        ldmatrix_x4(qa[kk], &sm.q[(wr + (lane & 15)) * kPad + kk * 16 + (lane >> 4) * 8]);
      }
    }
    const int key0 = tile * kKeys;
    // ---- S = Q K^T for 16 rows x 64 keys (8 n-tiles of 8 keys)
    float s[8][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        // B fragments of two 8-key n-tiles: matrices (keys np*16 + 0..7 | 8..15) x (d kk*16 + 0..7 | 8..15)
        uint32_t kb[4];
        const int key_r = np * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int col = kk * 16 + ((lane >> 3) & 1) * 8;
        ldmatrix_x4(kb, &sm.k[st][key_r * kPad + col]);
        mma16816(s[2 * np], qa[kk], kb[0], kb[1]);
        mma16816(s[2 * np + 1], qa[kk], kb[2], kb[3]);
      }
    }
    // ---- scale, mask, online softmax (rows g and g + 8 of this warp)
    float tmax[2] = {-INFINITY, -INFINITY};
    // structured mask: this thread's 16 key flags (keys n*8 + 2t and n*8 + 2t + 1, two per 16-bit load) as
    // bits 2n and 2n + 1 of one word
    uint32_t kf = 0u;
    if constexpr (MK == kMaskStructured) {
#pragma unroll
      for (int n = 0; n < 8; ++n) {
        const uint32_t w = *reinterpret_cast<const uint16_t*>(&sm.m[st][n * 8 + 2 * t]);
        kf |= ((w & 0xFFu) != 0u ? 1u : 0u) << (2 * n);
        kf |= ((w >> 8) != 0u ? 1u : 0u) << (2 * n + 1);
      }
    }
#pragma unroll
    for (int n = 0; n < 8; ++n) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int kc = n * 8 + 2 * t + (e & 1);  // key inside the tile
        const int key = key0 + kc;
        float v = __fmul_rn(s[n][e], a.scale);
        bool allowed = true;
        if constexpr (MK == kMaskStructured) {
          allowed = (key < a.mask_keys) ? ((kf >> (2 * n + (e & 1))) & 1u) != 0u : (key - a.mask_keys <= query[e >> 1]);
        } else if constexpr (MK == kMaskBytes) {
          const int rl = wr + g + ((e >> 1) << 3);  // row inside the CTA tile
          allowed = sm.m[st][rl * kKeys + kc] != 0;
        }
        if (!allowed) v = kMaskedScore;
        if (key >= Lk) v = -INFINITY;  // not a key at all
        s[n][e] = v;
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
    uint32_t pa[4][4];
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = ex2((s[n][0] - mx[0]) * kLog2e), p1 = ex2((s[n][1] - mx[0]) * kLog2e);
      const float p2 = ex2((s[n][2] - mx[1]) * kLog2e), p3 = ex2((s[n][3] - mx[1]) * kLog2e);
      l[0] += p0 + p1;
      l[1] += p2 + p3;
      const int kk = n >> 1;
      if ((n & 1) == 0) {
        pa[kk][0] = pack_bf16(p0, p1);
        pa[kk][1] = pack_bf16(p2, p3);
      } else {
        pa[kk][2] = pack_bf16(p0, p1);
        pa[kk][3] = pack_bf16(p2, p3);
      }
    }
    // ---- O += P V
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {
        uint32_t vb[4];
        const int r = kk * 16 + (lane & 15);
        const int c = np * 16 + ((lane >> 4) << 3);
        ldmatrix_x4_trans(vb, &sm.v[st][r * kPad + c]);
        mma16816(o[2 * np], pa[kk], vb[0], vb[1]);
        mma16816(o[2 * np + 1], pa[kk], vb[2], vb[3]);
      }
    }
    __syncthreads();  // stage st is refilled by the next iteration's prefetch
  }

  // ---- epilogue: O / l, bf16, optional int8 for the next W8A8 linear
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 1);
    l[hr] += __shfl_xor_sync(0xffffffffu, l[hr], 2);
  }
  const float inv[2] = {__frcp_rn(l[0]), __frcp_rn(l[1])};
  const float ra = (a.qo && a.qo_rsmooth) ? __frcp_rn(a.qo_act) : 0.f;
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int pr = r0 + wr + g + hr * 8;
    if (pr >= R) continue;
    const int h = kh * G + pr / a.Lq, row = pr % a.Lq;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int d = n * 8 + 2 * t;
      const float o0 = bf16_round(o[n][2 * hr] * inv[hr]), o1 = bf16_round(o[n][2 * hr + 1] * inv[hr]);
      if (a.o) {
        *reinterpret_cast<uint32_t*>(a.o + static_cast<size_t>(b) * a.o_bs + static_cast<size_t>(row) * a.o_rs +
                                     h * kD + d) = pack_bf16(o0, o1);
      }
      if (a.qo) {
        const int col = h * kD + d;
        int8_t q2[2];
        if (a.qo_rsmooth) {
          q2[0] = smooth_quant_fast(o0, a.qo_smooth[col], a.qo_rsmooth[col], a.qo_act, ra);
          q2[1] = smooth_quant_fast(o1, a.qo_smooth[col + 1], a.qo_rsmooth[col + 1], a.qo_act, ra);
        } else {
          q2[0] = smooth_quant(o0, a.qo_smooth[col], a.qo_act);
          q2[1] = smooth_quant(o1, a.qo_smooth[col + 1], a.qo_act);
        }
        *reinterpret_cast<int16_t*>(a.qo + static_cast<size_t>(b) * a.qo_bs + static_cast<size_t>(row) * a.qo_rs + col) =
            *reinterpret_cast<int16_t*>(q2);
      }
    }
  }
}

}  // namespace svla
