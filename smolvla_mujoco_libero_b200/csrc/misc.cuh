// Small kernels around the GEMMs: RoPE tables, prefix / suffix masks and positions, token embedding
// gather, SigLIP patch extraction, dtype conversions.
#pragma once

#include "ptx.cuh"

namespace svla {

// cs[p][i] = (cos(p / w^(2i/64)), sin(p / w^(2i/64))), fp32 like the reference's apply_rope
// (deploy/validate_fused_rope_layout_math.py:28-42): freq = (2/64)*i, timescale = w^freq,
// radians = p / timescale.
__global__ void rope_table_kernel(float2* cs, int max_pos, float max_wavelength) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= max_pos * 32) return;
  const int p = idx / 32, i = idx % 32;
  const float freq = __fmul_rn(2.0f / 64.0f, static_cast<float>(i));
  const float ts = powf(max_wavelength, freq);
  const float rad = __fdiv_rn(static_cast<float>(p), ts);
  cs[idx] = make_float2(cosf(rad), sinf(rad));
}

// Masks and positions for one sample_actions call (deploy/diagnose_3_4_numeric_baseline.py:42-46,
// :117-146, :171-172).  Prefix tokens: 2 x n_img image tokens, n_lang language tokens, 1 state token.
//   pad   = [img0_mask]*n_img + [img1_mask]*n_img + lang_mask + [1]
//   att   = 0 ... 0, 1 (state)            cum = cumsum(att)
//   prefix_mask[q, k] = cum[k] <= cum[q] && pad[q] && pad[k]           [B, Lp, Lp]
//   prefix_pos[i]     = cumsum(pad)[i] - 1                              [B, Lp]
//   suffix (chunk tokens, all att = 1, all pad = 1):
//   self_mask[q, k]   = k < Lp ? pad[k] : (k - Lp) <= q                  [B, Ls, Lp + Ls]
//   cross_mask[q, k]  = pad[k]                                          [B, Ls, Lp]
//   suffix_pos[i]     = sum(pad) + i;   cross_pos[i] = i
// Mask rows are stored at a stride of the row length rounded up to 16 bytes (padding bytes 0), so the
// attention kernel can copy every 16-key run of a row with one aligned 16-byte transfer.
struct MaskArgs {
  const uint8_t* img_mask0;  // [B]
  const uint8_t* img_mask1;  // [B]
  const uint8_t* lang_mask;  // [B, n_lang]
  int B, n_img, n_lang, Ls;
  uint8_t* prefix_mask;  // [B, Lp, mask_ld(Lp)]
  int* prefix_pos;       // [B * Lp]
  uint8_t* self_mask;    // [B, Ls, mask_ld(Lp + Ls)]
  uint8_t* cross_mask;   // [B, Ls, mask_ld(Lp)]
  int* suffix_pos;       // [B * Ls]
  int* cross_pos;        // [B * Ls]
};

// row stride of a mask over L keys
__host__ __device__ constexpr int mask_ld(int L) { return (L + 15) & ~15; }

__device__ __forceinline__ int prefix_pad(const MaskArgs& a, int b, int i) {
  if (i < a.n_img) return a.img_mask0[b] != 0;
  if (i < 2 * a.n_img) return a.img_mask1[b] != 0;
  if (i < 2 * a.n_img + a.n_lang) return a.lang_mask[b * a.n_lang + (i - 2 * a.n_img)] != 0;
  return 1;
}

// grid (ceil((Lp + 2 Ls) / 8), B): one warp per mask row (prefix rows, then the suffix's self-attention rows,
// then its cross-attention rows), 16 bytes per lane and store; warp 0 of block (0, b) also writes the
// positions (a warp prefix sum of the padding flags)
__global__ void masks_kernel(const MaskArgs a) {
  pdl_wait();
  pdl_trigger();
  const int b = blockIdx.y;
  const int Lp = 2 * a.n_img + a.n_lang + 1, Lt = Lp + a.Ls;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (blockIdx.x == 0 && warp == 0) {
    int c = 0;  // cumsum(pad) before this run of 32
    for (int base = 0; base < Lp; base += 32) {
      const int i = base + lane;
      int x = i < Lp ? prefix_pad(a, b, i) : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += t;
      }
      if (i < Lp) a.prefix_pos[b * Lp + i] = c + x - 1;
      c += __shfl_sync(0xffffffffu, x, 31);
    }
    for (int i = lane; i < a.Ls; i += 32) {
      a.suffix_pos[b * a.Ls + i] = c + i;
      a.cross_pos[b * a.Ls + i] = i;
    }
  }
  const int row = blockIdx.x * 8 + warp;
  if (row >= Lp + 2 * a.Ls) return;
  // att cumsum: only the state token (the last prefix token) has att = 1, so cum[k] <= cum[q] fails only for
  // k = Lp - 1 with q != Lp - 1
  int kind, q, ld;
  uint8_t* dst;
  if (row < Lp) {
    kind = 0, q = row, ld = mask_ld(Lp);
    dst = a.prefix_mask + (static_cast<size_t>(b) * Lp + q) * ld;
  } else if (row < Lp + a.Ls) {
    kind = 1, q = row - Lp, ld = mask_ld(Lt);
    dst = a.self_mask + (static_cast<size_t>(b) * a.Ls + q) * ld;
  } else {
    kind = 2, q = row - Lp - a.Ls, ld = mask_ld(Lp);
    dst = a.cross_mask + (static_cast<size_t>(b) * a.Ls + q) * ld;
  }
  const int pad_q = kind == 0 ? prefix_pad(a, b, q) : 1;
  for (int c0 = lane * 16; c0 < ld; c0 += 32 * 16) {
    uint32_t w[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int k = c0 + j;
      int v;
      if (kind == 0)
        v = (k < Lp) && !(k == Lp - 1 && q != Lp - 1) && pad_q && prefix_pad(a, b, k);
      else if (kind == 1)
        v = (k < Lp) ? prefix_pad(a, b, k) : (k < Lt && (k - Lp) <= q);
      else
        v = (k < Lp) && prefix_pad(a, b, k);
      w[j / 4] |= static_cast<uint32_t>(v != 0) << (8 * (j % 4));
    }
    *reinterpret_cast<int4*>(dst + c0) = make_int4(w[0], w[1], w[2], w[3]);
  }
}

// out[b*row_stride + row_offset + t] = bf16(float(E[tok[b, t]]) * scale) ; one warp per token, 8 per lane
__global__ void embed_tokens_kernel(const long long* tokens, int B, int T, const __nv_bfloat16* table, int vocab,
                                    int H, float scale, __nv_bfloat16* out, int rows_per_batch, int row_offset,
                                    int* err) {
  pdl_wait();
  pdl_trigger();
  const int w = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  if (w >= B * T) return;
  const int b = w / T, t = w % T;
  long long tok = tokens[w];
  if (tok < 0 || tok >= vocab) {
    record_error(err, kErrBadShape);
    tok = 0;
  }
  const __nv_bfloat16* src = table + static_cast<size_t>(tok) * H;
  __nv_bfloat16* dst = out + (static_cast<size_t>(b) * rows_per_batch + row_offset + t) * H;
  for (int k = lane * 8; k < H; k += 256) {
    const int4 raw = *reinterpret_cast<const int4*>(src + k);
    const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
    uint32_t pk[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      __nv_bfloat162 v = __floats2bfloat162_rn(__fmul_rn(__bfloat162float(h[2 * u]), scale),
                                               __fmul_rn(__bfloat162float(h[2 * u + 1]), scale));
      pk[u] = *reinterpret_cast<uint32_t*>(&v);
    }
    *reinterpret_cast<int4*>(dst + k) = make_int4(pk[0], pk[1], pk[2], pk[3]);
  }
}

// SigLIP patch extraction: images fp32 [N, C, S, S] -> bf16 patches [N * (S/P)^2, C*P*P] in the
// (c, kh, kw) order of a Conv2d weight [out, C, P, P] flattened.  One thread per 8 outputs (8 kw).
__global__ void im2col_kernel(const float* img, int N, int C, int S, int P, __nv_bfloat16* out) {
  pdl_wait();
  pdl_trigger();
  const int G = S / P;
  const long long total = static_cast<long long>(N) * G * G * C * P * (P / 8);
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= total) return;
  long long r = idx;
  const int kw8 = static_cast<int>(r % (P / 8)); r /= (P / 8);
  const int kh = static_cast<int>(r % P); r /= P;
  const int c = static_cast<int>(r % C); r /= C;
  const int px = static_cast<int>(r % G); r /= G;
  const int py = static_cast<int>(r % G); r /= G;
  const int n = static_cast<int>(r);
  const float* src = img + ((static_cast<size_t>(n) * C + c) * S + (py * P + kh)) * S + px * P + kw8 * 8;
  const float4 a0 = *reinterpret_cast<const float4*>(src);
  const float4 a1 = *reinterpret_cast<const float4*>(src + 4);
  uint32_t pk[4] = {0, 0, 0, 0};
  {
    __nv_bfloat162 h0 = __floats2bfloat162_rn(a0.x, a0.y), h1 = __floats2bfloat162_rn(a0.z, a0.w);
    __nv_bfloat162 h2 = __floats2bfloat162_rn(a1.x, a1.y), h3 = __floats2bfloat162_rn(a1.z, a1.w);
    pk[0] = *reinterpret_cast<uint32_t*>(&h0);
    pk[1] = *reinterpret_cast<uint32_t*>(&h1);
    pk[2] = *reinterpret_cast<uint32_t*>(&h2);
    pk[3] = *reinterpret_cast<uint32_t*>(&h3);
  }
  const size_t row = (static_cast<size_t>(n) * G + py) * G + px;
  const int col = (c * P + kh) * P + kw8 * 8;
  *reinterpret_cast<int4*>(out + row * (C * P * P) + col) = make_int4(pk[0], pk[1], pk[2], pk[3]);
}

__global__ void f32_to_bf16_kernel(const float* x, __nv_bfloat16* y, long long n) {
  pdl_wait();
  pdl_trigger();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __float2bfloat16_rn(x[i]);
}

// y = 1 / x, correctly rounded
__global__ void reciprocal_kernel(const float* x, float* y, long long n) {
  pdl_wait();
  pdl_trigger();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) y[i] = __frcp_rn(x[i]);
}

// x_t = noise (fp32 copy) and its bf16 image
__global__ void euler_init_kernel(const float* noise, float* xt, __nv_bfloat16* xt_bf16, long long n) {
  pdl_wait();
  pdl_trigger();
  const long long i = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i < n) {
    const float v = noise[i];
    xt[i] = v;
    xt_bf16[i] = __float2bfloat16_rn(v);
  }
}

}  // namespace svla
