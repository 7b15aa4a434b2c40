// Masked GQA attention, head_dim 64, bf16 in / bf16 out, fp32 scores and softmax.
//
// Semantics follow the reference's eager attention (deploy/export_6f_layer0_attention_tensors.py:100-119;
// lerobot eager_attention_forward):
//   s = (q . k) * d^-1/2                    (fp32)
//   s = mask ? s : finfo(f32).min           (a fully masked row therefore becomes uniform over ALL keys)
//   p = bf16(softmax(s))                    (normalised in fp32, then rounded to bf16)
//   o = bf16(p @ v)                         (fp32 accumulation)
// Query head h reads key/value head h / (Hq / Hkv).
//
// Two passes over the keys: pass 1 finds each row's max and sum, pass 2 recomputes the scores, forms
// the normalised bf16 probabilities and accumulates P.V.  This keeps the reference's rounding of the
// normalised probabilities for any key length.
//
// Keys may come from two sources (the cached prefix followed by the current suffix); each CTA handles
// 64 queries of one (batch, head) with 4 warps of 16 rows; tensor-core work is mma.sync m16n8k16.
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
  __nv_bfloat16* o;        long long o_bs; int o_rs;        // optional bf16 output
  int8_t* qo;              long long qo_bs; int qo_rs;      // optional int8 output
  const float* qo_smooth;  float qo_act;
  int Lq, Hq, Hkv;
  float scale;
};

namespace attn_detail {
constexpr int kD = 64;
constexpr int kKP = 72;  // padded smem row (bf16) -> conflict-free fragment loads
constexpr int kChunk = 64;
constexpr float kMaskedScore = -3.4028234663852886e38f;  // torch.finfo(torch.float32).min

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t (&r)[4], const void* p) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(smem_u32(p)));
}

// load one 64-key chunk of K (and V) for kv head `kh` into padded shared tiles (zero beyond Lk)
__device__ __forceinline__ void load_kv_chunk(const AttnArgs& a, int b, int kh, int key0, __nv_bfloat16* ks,
                                              __nv_bfloat16* vs, bool load_v) {
  const int Lk = a.L1 + a.L2;
  for (int idx = threadIdx.x; idx < kChunk * 8; idx += blockDim.x) {
    const int r = idx >> 3, c = (idx & 7) * 8;
    const int key = key0 + r;
    int4 kv = make_int4(0, 0, 0, 0), vv = make_int4(0, 0, 0, 0);
    if (key < Lk) {
      const __nv_bfloat16 *kp, *vp;
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
      kv = *reinterpret_cast<const int4*>(kp);
      if (load_v) vv = *reinterpret_cast<const int4*>(vp);
    }
    *reinterpret_cast<int4*>(ks + r * kKP + c) = kv;
    if (load_v) *reinterpret_cast<int4*>(vs + r * kKP + c) = vv;
  }
}
}  // namespace attn_detail

__global__ void __launch_bounds__(128) attention_kernel(const AttnArgs a) {
  using namespace attn_detail;
  __shared__ __align__(16) __nv_bfloat16 ks[kChunk * kKP];
  __shared__ __align__(16) __nv_bfloat16 vs[kChunk * kKP];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (a.Hq / a.Hkv);
  const int q0 = blockIdx.x * 64 + warp * 16;
  const int Lk = a.L1 + a.L2;

  // Q fragments (16 rows x 64 dims per warp), rows beyond Lq read as zero
  uint32_t qa[4][4];
  {
    const int r0 = q0 + g, r1 = q0 + g + 8;
    const __nv_bfloat16* qb = a.q + static_cast<size_t>(b) * a.q_bs + h * kD;
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      const int c = kk * 16 + 2 * t;
      auto ld = [&](int r, int cc) -> uint32_t {
        if (r >= a.Lq) return 0u;
        return *reinterpret_cast<const uint32_t*>(qb + static_cast<size_t>(r) * a.q_rs + cc);
      };
      qa[kk][0] = ld(r0, c);
      qa[kk][1] = ld(r1, c);
      qa[kk][2] = ld(r0, c + 8);
      qa[kk][3] = ld(r1, c + 8);
    }
  }
  const int row0 = q0 + g, row1 = q0 + g + 8;
  const uint8_t* mrow0 = (a.mask && row0 < a.Lq) ? a.mask + static_cast<size_t>(b) * a.mask_bs + static_cast<size_t>(row0) * a.mask_rs : nullptr;
  const uint8_t* mrow1 = (a.mask && row1 < a.Lq) ? a.mask + static_cast<size_t>(b) * a.mask_bs + static_cast<size_t>(row1) * a.mask_rs : nullptr;

  // scores for one chunk: s[n][0..3] for key columns key0 + n*8 + 2t (+1), rows g / g+8
  auto chunk_scores = [&](int key0, float (&s)[8][4]) {
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      s[n][0] = s[n][1] = s[n][2] = s[n][3] = 0.f;
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        const __nv_bfloat16* kr = ks + (n * 8 + g) * kKP + kk * 16 + 2 * t;
        const uint32_t b0 = *reinterpret_cast<const uint32_t*>(kr);
        const uint32_t b1 = *reinterpret_cast<const uint32_t*>(kr + 8);
        mma16816(s[n], qa[kk], b0, b1);
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int key = key0 + n * 8 + 2 * t + (e & 1);
        const uint8_t* mr = (e < 2) ? mrow0 : mrow1;
        float v = __fmul_rn(s[n][e], a.scale);
        if (key >= Lk) {
          v = -INFINITY;  // not a key at all
        } else if (a.mask) {
          const bool allowed = mr ? (mr[key] != 0) : false;
          if (!allowed) v = kMaskedScore;
        }
        s[n][e] = v;
      }
    }
  };

  // ---------------- pass 1: row max and sum
  float mx[2] = {-INFINITY, -INFINITY}, sm[2] = {0.f, 0.f};
  for (int key0 = 0; key0 < Lk; key0 += kChunk) {
    __syncthreads();
    load_kv_chunk(a, b, kh, key0, ks, vs, false);
    __syncthreads();
    float s[8][4];
    chunk_scores(key0, s);
#pragma unroll
    for (int hr = 0; hr < 2; ++hr) {
      float cm = -INFINITY;
#pragma unroll
      for (int n = 0; n < 8; ++n) cm = fmaxf(cm, fmaxf(s[n][2 * hr], s[n][2 * hr + 1]));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 1));
      cm = fmaxf(cm, __shfl_xor_sync(0xffffffffu, cm, 2));
      const float nm = fmaxf(mx[hr], cm);
      float cs = 0.f;
#pragma unroll
      for (int n = 0; n < 8; ++n) cs += expf(s[n][2 * hr] - nm) + expf(s[n][2 * hr + 1] - nm);
      cs += __shfl_xor_sync(0xffffffffu, cs, 1);
      cs += __shfl_xor_sync(0xffffffffu, cs, 2);
      sm[hr] = (mx[hr] == -INFINITY ? 0.f : sm[hr] * expf(mx[hr] - nm)) + cs;
      mx[hr] = nm;
    }
  }

  // ---------------- pass 2: normalised bf16 probabilities, O = P V
  float oacc[8][4];
#pragma unroll
  for (int n = 0; n < 8; ++n) oacc[n][0] = oacc[n][1] = oacc[n][2] = oacc[n][3] = 0.f;
  for (int key0 = 0; key0 < Lk; key0 += kChunk) {
    __syncthreads();
    load_kv_chunk(a, b, kh, key0, ks, vs, true);
    __syncthreads();
    float s[8][4];
    chunk_scores(key0, s);
    uint32_t pa[4][4];  // A fragments of P for 4 k16 steps
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const float p0 = __fdiv_rn(expf(s[n][0] - mx[0]), sm[0]);
      const float p1 = __fdiv_rn(expf(s[n][1] - mx[0]), sm[0]);
      const float p2 = __fdiv_rn(expf(s[n][2] - mx[1]), sm[1]);
      const float p3 = __fdiv_rn(expf(s[n][3] - mx[1]), sm[1]);
      const int kk = n >> 1;
      if ((n & 1) == 0) {
        pa[kk][0] = pack_bf16(p0, p1);
        pa[kk][1] = pack_bf16(p2, p3);
      } else {
        pa[kk][2] = pack_bf16(p0, p1);
        pa[kk][3] = pack_bf16(p2, p3);
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int np = 0; np < 4; ++np) {  // pairs of 8-wide d tiles
        uint32_t vb[4];
        const int r = kk * 16 + (lane & 15);
        const int c = np * 16 + ((lane >> 4) << 3);
        ldmatrix_x4_trans(vb, vs + r * kKP + c);
        mma16816(oacc[2 * np], pa[kk], vb[0], vb[1]);
        mma16816(oacc[2 * np + 1], pa[kk], vb[2], vb[3]);
      }
    }
  }

  // ---------------- epilogue
#pragma unroll
  for (int hr = 0; hr < 2; ++hr) {
    const int row = hr ? row1 : row0;
    if (row >= a.Lq) continue;
#pragma unroll
    for (int n = 0; n < 8; ++n) {
      const int d = n * 8 + 2 * t;
      const float o0 = bf16_round(oacc[n][2 * hr]), o1 = bf16_round(oacc[n][2 * hr + 1]);
      if (a.o) {
        *reinterpret_cast<uint32_t*>(a.o + static_cast<size_t>(b) * a.o_bs + static_cast<size_t>(row) * a.o_rs +
                                     h * kD + d) = pack_bf16(o0, o1);
      }
      if (a.qo) {
        const int col = h * kD + d;
        int8_t q2[2] = {smooth_quant(o0, a.qo_smooth[col], a.qo_act), smooth_quant(o1, a.qo_smooth[col + 1], a.qo_act)};
        *reinterpret_cast<int16_t*>(a.qo + static_cast<size_t>(b) * a.qo_bs + static_cast<size_t>(row) * a.qo_rs + col) =
            *reinterpret_cast<int16_t*>(q2);
      }
    }
  }
}

}  // namespace svla
