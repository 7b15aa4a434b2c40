// Plugin-semantics RoPE kernels: the operators of the reference's SmolVLAFusedRopeLayout and
// SmolVLAFusedRopeAttention TensorRT plugins (deploy/cuda/fused_rope_layout.h:24-50), for the data types and
// position types those plugins take (fp32 / fp16 / bf16 data, int32 / int64 positions, any even head_dim).
//
// Both rotate with rotate-half RoPE in fp32:  theta_i = pos / max_wavelength^(2i / head_dim),
//   out[i] = x[i] cos - x[i + d/2] sin,   out[i + d/2] = x[i + d/2] cos + x[i] sin   (i < d/2),
// the arithmetic of deploy/validate_fused_rope_layout_math.py:28-42 and lerobot's apply_rope.
//
// These are the plugin-compatible entry points.  The sample_actions path itself never materialises raw q / k:
// RoPE is applied in the QKV GEMM epilogue and attention reads the rotated rows directly.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "ptx.cuh"

namespace svla {
namespace rope {

__device__ __forceinline__ float load(const float* p, size_t i) { return p[i]; }
__device__ __forceinline__ float load(const __half* p, size_t i) { return __half2float(p[i]); }
__device__ __forceinline__ float load(const __nv_bfloat16* p, size_t i) { return __bfloat162float(p[i]); }
__device__ __forceinline__ void store(float* p, size_t i, float v) { p[i] = v; }
__device__ __forceinline__ void store(__half* p, size_t i, float v) { p[i] = __float2half_rn(v); }
__device__ __forceinline__ void store(__nv_bfloat16* p, size_t i, float v) { p[i] = __float2bfloat16_rn(v); }

// position of token l of sample b: from the position tensor, or l itself when there is none
template <typename PosT>
__device__ __forceinline__ float position(const PosT* pos, int b, int L, int l) {
  return pos ? static_cast<float>(pos[static_cast<size_t>(b) * L + l]) : static_cast<float>(l);
}

// (cos, sin) of the angle of rotation pair i at position p for head width d
__device__ __forceinline__ float2 angle(float p, int i, int d, float max_wavelength) {
  const float freq = __fmul_rn(__fdiv_rn(2.0f, static_cast<float>(d)), static_cast<float>(i));
  const float rad = __fdiv_rn(p, powf(max_wavelength, freq));
  float s, c;
  sincosf(rad, &s, &c);
  return make_float2(c, s);
}

}  // namespace rope

// q_raw [B, L, Hq*D] -> q_out [B, Hq, L, D];  k_raw [B, L, Hkv*D] -> k_out [B, Hq, D, L] (GQA-expanded,
// transposed), same data type in and out.  One thread per rotation pair (i, i + D/2) of one head of one token.
template <typename T, typename PosT>
__global__ void rope_layout_kernel(const T* q_raw, const T* k_raw, const PosT* pos, T* q_out, T* k_out, int B,
                                   int L, int Hq, int Hkv, int D, float max_wavelength) {
  pdl_wait();
  pdl_trigger();
  const int half = D / 2;
  const long long nq = static_cast<long long>(B) * L * Hq * half;
  const long long nk = static_cast<long long>(B) * L * Hkv * half;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= nq + nk) return;
  const bool is_q = idx < nq;
  long long r = is_q ? idx : idx - nq;
  const int H = is_q ? Hq : Hkv;
  const int i = static_cast<int>(r % half); r /= half;
  const int h = static_cast<int>(r % H); r /= H;
  const int l = static_cast<int>(r % L);
  const int b = static_cast<int>(r / L);
  const float2 cs = rope::angle(rope::position(pos, b, L, l), i, D, max_wavelength);
  const T* src = (is_q ? q_raw : k_raw) + (static_cast<size_t>(b) * L + l) * H * D + static_cast<size_t>(h) * D;
  const float x1 = rope::load(src, i), x2 = rope::load(src, i + half);
  const float o1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
  const float o2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
  if (is_q) {
    T* dst = q_out + ((static_cast<size_t>(b) * Hq + h) * L + l) * D;
    rope::store(dst, i, o1);
    rope::store(dst, i + half, o2);
  } else {
    const int g = Hq / Hkv;
    for (int j = 0; j < g; ++j) {
      T* dst = k_out + (static_cast<size_t>(b) * Hq + h * g + j) * D * L;
      rope::store(dst, static_cast<size_t>(i) * L + l, o1);
      rope::store(dst, static_cast<size_t>(i + half) * L + l, o2);
    }
  }
}

// ---------------------------------------------------------------------------------------------------------
// Fused RoPE attention with the plugin's contract (deploy/cuda/fused_rope_layout.cu:271-431, launcher
// :768-800): raw q [B, L, Hq*D], raw k / v [B, L, Hkv*D], positions [B, L] (or implicit 0..L-1), keep-mask
// [B, L, L] (bool bytes, or fp32 with keep = value > 0.5) -> fp32 context [B, Hq, L, D].  All arithmetic in
// fp32: rotated q / k, scores * D^-1/2, masked scores excluded, softmax, P.V.  A query whose every key is
// masked gets the mean of V over all keys (the plugin's rule, and softmax over a row of equal finfo.min).
//
// One CTA per (qpc query positions, kv head, sample) serves the kv head's g query heads (qpc * g <= 64 rows,
// qpc = 64 / g), so the keys and values of that kv head are rotated and staged once per key tile and shared
// by the g heads.  Keys are streamed in tiles of 64 through shared memory with an online softmax (running max
// and sum per row); each warp owns rows, each lane two keys of a tile for the scores and D/32 output columns
// for P.V.
constexpr int kRopeAttnRows = 64;   // query rows (position, head) per CTA
constexpr int kRopeAttnKeys = 64;   // keys per shared-memory tile
constexpr int kRopeAttnWarps = 8;
constexpr int kRopeAttnMaxD = 128;
constexpr int kRopeAttnMaxRows = kRopeAttnRows / kRopeAttnWarps;  // rows per warp

struct RopeAttnArgs {
  const void* q;
  const void* k;
  const void* v;
  const void* pos;
  const void* mask;
  int mask_f32;  // 0: bool bytes, 1: fp32 (keep = value > 0.5)
  float* ctx;
  int B, L, Hq, Hkv, D;
  int qpc;  // query positions per CTA (64 / g)
  float max_wavelength;
  float scale;
};

template <typename T, typename PosT>
__global__ void __launch_bounds__(kRopeAttnWarps * 32) rope_attention_kernel(RopeAttnArgs a) {
  extern __shared__ __align__(16) float rsm[];
  const int D = a.D, half = D / 2, g = a.Hq / a.Hkv;
  const int qpc = a.qpc;
  const int q0 = blockIdx.x * qpc, kvh = blockIdx.y, b = blockIdx.z;
  const int rows = qpc * g;  // row r: query position q0 + r % qpc of head kvh * g + r / qpc
  const int ldk = D + 1;     // padded key rows: lanes reading different keys hit different banks
  float* qs = rsm;                                  // [rows][D]     rotated queries
  float* ks = qs + kRopeAttnRows * kRopeAttnMaxD;   // [64][D + 1]   rotated keys
  float* vs = ks + kRopeAttnKeys * (kRopeAttnMaxD + 1);  // [64][D]  values
  const T* qr = static_cast<const T*>(a.q);
  const T* kr = static_cast<const T*>(a.k);
  const T* vr = static_cast<const T*>(a.v);
  const PosT* pos = static_cast<const PosT*>(a.pos);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  pdl_wait();
  pdl_trigger();
  // rotated queries of the CTA's rows
  for (int e = tid; e < rows * half; e += blockDim.x) {
    const int i = e % half, r = e / half;
    const int l = q0 + (r % qpc), h = kvh * g + r / qpc;
    float o1 = 0.f, o2 = 0.f;
    if (l < a.L) {
      const float2 cs = rope::angle(rope::position(pos, b, a.L, l), i, D, a.max_wavelength);
      const size_t base = (static_cast<size_t>(b) * a.L + l) * a.Hq * D + static_cast<size_t>(h) * D;
      const float x1 = rope::load(qr, base + i), x2 = rope::load(qr, base + i + half);
      o1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
      o2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
    }
    qs[r * D + i] = o1;
    qs[r * D + i + half] = o2;
  }
  // per-row online-softmax state of this warp's rows (row r = warp + 8 j)
  const int cols = D / 32;  // output columns per lane: lane + 32 c
  float m[kRopeAttnMaxRows], lsum[kRopeAttnMaxRows], acc[kRopeAttnMaxRows][kRopeAttnMaxD / 32];
#pragma unroll
  for (int j = 0; j < kRopeAttnMaxRows; ++j) {
    m[j] = -FLT_MAX;
    lsum[j] = 0.f;
#pragma unroll
    for (int c = 0; c < kRopeAttnMaxD / 32; ++c) acc[j][c] = 0.f;
  }
  const unsigned char* mask8 = static_cast<const unsigned char*>(a.mask);
  const float* maskf = static_cast<const float*>(a.mask);
  for (int k0 = 0; k0 < a.L; k0 += kRopeAttnKeys) {
    __syncthreads();  // the previous tile's keys and values are no longer read
    for (int e = tid; e < kRopeAttnKeys * half; e += blockDim.x) {
      const int i = e % half, kk = e / half, l = k0 + kk;
      float o1 = 0.f, o2 = 0.f, v1 = 0.f, v2 = 0.f;
      if (l < a.L) {
        const float2 cs = rope::angle(rope::position(pos, b, a.L, l), i, D, a.max_wavelength);
        const size_t base = (static_cast<size_t>(b) * a.L + l) * a.Hkv * D + static_cast<size_t>(kvh) * D;
        const float x1 = rope::load(kr, base + i), x2 = rope::load(kr, base + i + half);
        o1 = __fsub_rn(__fmul_rn(x1, cs.x), __fmul_rn(x2, cs.y));
        o2 = __fadd_rn(__fmul_rn(x2, cs.x), __fmul_rn(x1, cs.y));
        v1 = rope::load(vr, base + i);
        v2 = rope::load(vr, base + i + half);
      }
      ks[kk * ldk + i] = o1;
      ks[kk * ldk + i + half] = o2;
      vs[kk * D + i] = v1;
      vs[kk * D + i + half] = v2;
    }
    __syncthreads();
#pragma unroll
    for (int j = 0; j < kRopeAttnMaxRows; ++j) {
      const int r = warp + kRopeAttnWarps * j;
      if (r >= rows) break;
      const int l = q0 + (r % qpc);
      if (l >= a.L) continue;
      // scores of keys k0 + lane and k0 + lane + 32
      float s[2];
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const int kk = lane + 32 * u, key = k0 + kk;
        float dot = 0.f;
        for (int d = 0; d < D; ++d) dot = fmaf(qs[r * D + d], ks[kk * ldk + d], dot);
        bool keep = false;
        if (key < a.L) {
          const size_t mi = (static_cast<size_t>(b) * a.L + l) * a.L + key;
          keep = a.mask == nullptr || (a.mask_f32 ? maskf[mi] > 0.5f : mask8[mi] != 0);
        }
        // masked keys score finfo.min: exp(min - max) is 0 unless every key of the row is masked
        s[u] = key < a.L ? (keep ? __fmul_rn(dot, a.scale) : -FLT_MAX) : -INFINITY;
      }
      float tmax = fmaxf(s[0], s[1]);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) tmax = fmaxf(tmax, __shfl_xor_sync(0xffffffffu, tmax, o));
      const float mnew = fmaxf(m[j], tmax);
      const float alpha = expf(m[j] - mnew);
      const float p0 = expf(s[0] - mnew), p1 = expf(s[1] - mnew);
      float psum = p0 + p1;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) psum += __shfl_xor_sync(0xffffffffu, psum, o);
      lsum[j] = fmaf(lsum[j], alpha, psum);
      m[j] = mnew;
#pragma unroll
      for (int c = 0; c < kRopeAttnMaxD / 32; ++c) acc[j][c] *= alpha;
      for (int kk = 0; kk < kRopeAttnKeys && k0 + kk < a.L; ++kk) {
        const float p = __shfl_sync(0xffffffffu, kk < 32 ? p0 : p1, kk & 31);
#pragma unroll
        for (int c = 0; c < kRopeAttnMaxD / 32; ++c)
          if (c < cols) acc[j][c] = fmaf(p, vs[kk * D + lane + 32 * c], acc[j][c]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < kRopeAttnMaxRows; ++j) {
    const int r = warp + kRopeAttnWarps * j;
    if (r >= rows) break;
    const int l = q0 + (r % qpc), h = kvh * g + r / qpc;
    if (l >= a.L) continue;
    const float inv = 1.0f / lsum[j];
    float* out = a.ctx + ((static_cast<size_t>(b) * a.Hq + h) * a.L + l) * D;
#pragma unroll
    for (int c = 0; c < kRopeAttnMaxD / 32; ++c)
      if (c < cols) out[lane + 32 * c] = acc[j][c] * inv;
  }
}

inline size_t rope_attention_smem() {
  return sizeof(float) * (static_cast<size_t>(kRopeAttnRows) * kRopeAttnMaxD +
                          static_cast<size_t>(kRopeAttnKeys) * (kRopeAttnMaxD + 1) +
                          static_cast<size_t>(kRopeAttnKeys) * kRopeAttnMaxD);
}

}  // namespace svla
