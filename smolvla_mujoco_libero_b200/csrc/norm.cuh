// Row normalisation fused with SmoothQuant activation quantisation.
//
// One warp per row; each lane holds NV vectors of 8 bf16 in registers (K <= NV * 256).
//   RMSNorm  (SmolVLM2 text / expert, transformers LlamaRMSNorm):
//       h = bf16(x * (1 / sqrt(mean(x^2) + eps)));  y = bf16(w * h)
//   LayerNorm (SigLIP):  y = bf16((x - mean) * rstd * w + b)
// Outputs (any subset): y in bf16, and up to three int8 tensors
//       q_i = round((y / s_i[k]) / a_i).clamp(-128, 127)
// each with its own smooth vector s_i and activation scale a_i -- the per-projection SmoothQuant
// of q/k/v (or gate/up) that W8A8Linear.forward applies (deploy/linear_only_quant.py:104-116).
// The smooth divide runs on the bf16-rounded y, exactly as the unfused reference does.
//
// Optional pixel-shuffle remap of the outputs (SmolVLM connector, scale 4 on a 32x32 grid):
// input token t = hh*32 + ww of image i goes to output row i*64 + (hh/4)*8 + ww/4, columns
// ((hh%4)*4 + ww%4) * K ..., with the smooth vector indexed by the output column.
#pragma once

#include "ptx.cuh"

namespace svla {

struct NormQuantArgs {
  const __nv_bfloat16* x;  // [M, ldx]
  int ldx;
  const __nv_bfloat16* w;  // [K]
  const __nv_bfloat16* b;  // [K] (LayerNorm) or nullptr
  float eps;
  int M, K;
  __nv_bfloat16* y;        // optional [M, ldy]
  int ldy;
  int nq;                  // number of int8 outputs (0..3)
  int8_t* q[3];
  int ldq;
  const float* smooth[3];
  const float* rsmooth[3];  // optional reciprocals of smooth (fast path, same result)
  float act[3];
  int pixel_shuffle;       // 0 or the shuffle factor (4)
  int ps_grid;             // tokens per side of the input grid (32)
};

// one row m, its bf16 input already in registers (raw[i] = columns (i*32 + lane)*8 .. +7)
template <int NV, bool LAYERNORM>
__device__ __forceinline__ void norm_quant_row(const NormQuantArgs& a, int m, int lane, const int4 (&raw_in)[NV]) {
  float v[NV][8];
  float ss = 0.f, sum = 0.f;
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = (i * 32 + lane) * 8;
    if (k < a.K) {
      const int4 raw = raw_in[i];
      const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        v[i][j] = __bfloat162float(h[j]);
        sum += v[i][j];
      }
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) v[i][j] = 0.f;
    }
  }
  float mean = 0.f;
  if constexpr (LAYERNORM) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    mean = __fdiv_rn(sum, static_cast<float>(a.K));
  }
#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = (i * 32 + lane) * 8;
    if (k < a.K) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float d = LAYERNORM ? (v[i][j] - mean) : v[i][j];
        ss = fmaf(d, d, ss);
      }
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float var = __fdiv_rn(ss, static_cast<float>(a.K));
  const float rstd = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, a.eps)));

  // output row / column remap for the pixel shuffle
  int qrow = m, qcol0 = 0;
  if (a.pixel_shuffle > 0) {
    const int s = a.pixel_shuffle, g = a.ps_grid;
    const int per_img = g * g;
    const int img = m / per_img, t = m % per_img;
    const int hh = t / g, ww = t % g;
    const int out_side = g / s;
    qrow = img * out_side * out_side + (hh / s) * out_side + (ww / s);
    qcol0 = ((hh % s) * s + (ww % s)) * a.K;
  }

  float ra[3];  // 1 / act_i, for the multiply form of the quantiser
#pragma unroll
  for (int qi = 0; qi < 3; ++qi) ra[qi] = (qi < a.nq && a.rsmooth[qi]) ? __frcp_rn(a.act[qi]) : 0.f;

#pragma unroll
  for (int i = 0; i < NV; ++i) {
    const int k = (i * 32 + lane) * 8;
    if (k >= a.K) continue;
    const int4 wr = *reinterpret_cast<const int4*>(a.w + k);
    const __nv_bfloat16* wh = reinterpret_cast<const __nv_bfloat16*>(&wr);
    float y[8];
    if constexpr (LAYERNORM) {
      const int4 br = *reinterpret_cast<const int4*>(a.b + k);
      const __nv_bfloat16* bh = reinterpret_cast<const __nv_bfloat16*>(&br);
      // pairs through the packed fp32 pipe, each lane rounded exactly as the scalar op (x - mean is
      // x + (-mean), the same rounding)
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 d = __fadd2_rn(make_float2(v[i][j], v[i][j + 1]), make_float2(-mean, -mean));
        const float2 t = __fmul2_rn(__fmul2_rn(d, make_float2(rstd, rstd)),
                                    make_float2(__bfloat162float(wh[j]), __bfloat162float(wh[j + 1])));
        const float2 r = __fadd2_rn(t, make_float2(__bfloat162float(bh[j]), __bfloat162float(bh[j + 1])));
        y[j] = r.x;
        y[j + 1] = r.y;
      }
    } else {
      float h[8];
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 t = __fmul2_rn(make_float2(v[i][j], v[i][j + 1]), make_float2(rstd, rstd));
        h[j] = t.x;
        h[j + 1] = t.y;
      }
#pragma unroll
      for (int j = 0; j < 8; j += 2) bf16_round2(h[j], h[j + 1]);
#pragma unroll
      for (int j = 0; j < 8; j += 2) {
        const float2 t = __fmul2_rn(make_float2(__bfloat162float(wh[j]), __bfloat162float(wh[j + 1])),
                                    make_float2(h[j], h[j + 1]));
        y[j] = t.x;
        y[j + 1] = t.y;
      }
    }
#pragma unroll
    for (int j = 0; j < 8; j += 2) bf16_round2(y[j], y[j + 1]);
    if (a.y) {
      uint32_t pk[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) pk[u] = pack_bf16_rn(y[2 * u], y[2 * u + 1]);
      *reinterpret_cast<int4*>(a.y + static_cast<size_t>(qrow) * a.ldy + qcol0 + k) =
          make_int4(pk[0], pk[1], pk[2], pk[3]);
    }
#pragma unroll
    for (int qi = 0; qi < 3; ++qi) {
      if (qi >= a.nq) break;
      const int col = qcol0 + k;
      uint32_t w[2] = {0u, 0u};
      uint32_t slow = 0xFFu;  // every element exact without a reciprocal smooth vector
      if (a.rsmooth[qi]) {
        slow = 0u;
        w[0] = smooth_quant4_fast(&y[0], *reinterpret_cast<const float4*>(a.rsmooth[qi] + col), ra[qi], slow, 0);
        w[1] = smooth_quant4_fast(&y[4], *reinterpret_cast<const float4*>(a.rsmooth[qi] + col + 4), ra[qi], slow, 4);
      }
      if (slow != 0u) {  // rare: values near a rounding boundary take the two-divide path one by one
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          if (slow & (1u << j)) {
            const uint32_t q8 = static_cast<uint32_t>(smooth_quant_slow(y[j], a.smooth[qi][col + j], a.act[qi]) & 0xFF);
            w[j / 4] = (w[j / 4] & ~(0xFFu << (8 * (j % 4)))) | (q8 << (8 * (j % 4)));
          }
        }
      }
      *reinterpret_cast<int2*>(a.q[qi] + static_cast<size_t>(qrow) * a.ldq + col) = make_int2(w[0], w[1]);
    }
  }
}

// Warps stream rows (grid-stride); the next row's input is requested before the current row is processed,
// so each warp keeps two rows of loads in flight.
template <int NV, bool LAYERNORM>
__global__ void __launch_bounds__(256) norm_quant_kernel(const NormQuantArgs a) {
  // the row constants (norm weight, bias, reciprocal smooth vectors) do not depend on the previous kernel:
  // their cache lines are requested into L1 before waiting for it, one 128-byte line per thread
  {
    const int line = threadIdx.x, wl = (a.K * 2 + 127) / 128, fl = (a.K * 4 + 127) / 128;
    const void* p = nullptr;
    if (line < wl) {
      p = reinterpret_cast<const char*>(a.w) + line * 128;
    } else if (LAYERNORM && line < 2 * wl) {
      p = reinterpret_cast<const char*>(a.b) + (line - wl) * 128;
    } else {
      const int r = line - (LAYERNORM ? 2 : 1) * wl, qi = r / fl;
      if (r >= 0 && qi < a.nq && a.rsmooth[qi] != nullptr)
        p = reinterpret_cast<const char*>(a.rsmooth[qi]) + (r - qi * fl) * 128;
    }
    if (p != nullptr) asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
  }
  pdl_wait();
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const int warp0 = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int nwarps = (gridDim.x * blockDim.x) >> 5;
  auto load_row = [&](int m, int4 (&r)[NV]) {
    const __nv_bfloat16* xr = a.x + static_cast<size_t>(m) * a.ldx;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int k = (i * 32 + lane) * 8;
      r[i] = (k < a.K) ? *reinterpret_cast<const int4*>(xr + k) : make_int4(0, 0, 0, 0);
    }
  };
  int4 next[NV];
  if (warp0 < a.M) load_row(warp0, next);
  for (int m = warp0; m < a.M; m += nwarps) {
    int4 cur[NV];
#pragma unroll
    for (int i = 0; i < NV; ++i) cur[i] = next[i];
    if (m + nwarps < a.M) load_row(m + nwarps, next);
    norm_quant_row<NV, LAYERNORM>(a, m, lane, cur);
  }
}

// Standalone SmoothQuant activation quantiser (deploy/cuda/smoothquant_linear_epilogue.cu:108-119):
// q[m, k] = round((x[m, k] / s[k]) / a).clamp(-128, 127), x in bf16.  8 elements per thread.
__global__ void smooth_quant_kernel(const __nv_bfloat16* x, int ldx, const float* s, float act, int8_t* q, int ldq,
                                    int M, int K) {
  pdl_wait();
  pdl_trigger();
  const int kv = K / 8;
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= static_cast<long long>(M) * kv) return;
  const int m = static_cast<int>(idx / kv), k = static_cast<int>(idx % kv) * 8;
  const int4 raw = *reinterpret_cast<const int4*>(x + static_cast<size_t>(m) * ldx + k);
  const __nv_bfloat16* h = reinterpret_cast<const __nv_bfloat16*>(&raw);
  int8_t qv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) qv[j] = smooth_quant(__bfloat162float(h[j]), s ? s[k + j] : 1.0f, act);
  *reinterpret_cast<int2*>(q + static_cast<size_t>(m) * ldq + k) = *reinterpret_cast<int2*>(qv);
}

// Per-output-channel int8 weight packing with an optional SmoothQuant fold
// (deploy/linear_only_quant.py:43-53, :140-144):  W' = W * s[None, :];
// w_s[n] = max(max_k |W'[n, k]|, 1e-8) / 127;  q = round(W' / w_s[n]).clamp(-127, 127).
// One block per output row.
__global__ void __launch_bounds__(256) pack_weight_kernel(const __nv_bfloat16* w, int K, const float* smooth,
                                                          int8_t* q, float* wscale) {
  pdl_wait();
  pdl_trigger();
  const int n = blockIdx.x;
  const __nv_bfloat16* wr = w + static_cast<size_t>(n) * K;
  float amax = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = __bfloat162float(wr[k]);
    if (smooth) v = __fmul_rn(v, fmaxf(smooth[k], 1e-8f));
    amax = fmaxf(amax, fabsf(v));
  }
  __shared__ float red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float scale = __fdiv_rn(fmaxf(red[0], 1e-8f), 127.0f);
  if (threadIdx.x == 0) wscale[n] = scale;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = __bfloat162float(wr[k]);
    if (smooth) v = __fmul_rn(v, fmaxf(smooth[k], 1e-8f));
    q[static_cast<size_t>(n) * K + k] = static_cast<int8_t>(quant_rn_clamp(__fdiv_rn(v, scale), -127, 127));
  }
}

// out[n, k] = bf16(float(q[n, k]) * wscale[n]) -- the bf16 weight a W8A16 linear multiplies by
// (dequantize_weight(...).to(bfloat16), deploy/linear_only_quant.py:122-124, :147-148).  8 per thread.
__global__ void __launch_bounds__(256) dequant_weight_kernel(const int8_t* q, const float* wscale, int N, int K,
                                                             __nv_bfloat16* out) {
  pdl_wait();
  pdl_trigger();
  const long long i8 = (static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x) * 8;
  if (i8 >= static_cast<long long>(N) * K) return;
  const int n = static_cast<int>(i8 / K);
  const float ws = wscale[n];
  const int2 raw = *reinterpret_cast<const int2*>(q + i8);
  const int8_t* b = reinterpret_cast<const int8_t*>(&raw);
  uint32_t pk[4];
#pragma unroll
  for (int j = 0; j < 4; ++j)
    pk[j] = pack_bf16_rn(__fmul_rn(static_cast<float>(b[2 * j]), ws), __fmul_rn(static_cast<float>(b[2 * j + 1]), ws));
  *reinterpret_cast<int4*>(out + i8) = make_int4(pk[0], pk[1], pk[2], pk[3]);
}

}  // namespace svla
