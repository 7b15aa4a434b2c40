// Per-channel activation statistics for SmoothQuant calibration: the forward-pre-hook statistics of the
// reference's PerChannelLinearInputCollector (deploy/calibrate_smolvla_activation_channel_scales.py:68-84)
// for a batch of calls at once.  For every call (one sample's pass through a linear: `rows` tokens) and
// channel k:
//   amax[k]  = max_calls max(max_t |x[t, k]|, 1e-8)
//   pamax[k] = max_calls max(torch.quantile(|x[:, k]|, q), 1e-8)
// with torch.quantile's linear interpolation: rank = q * (rows - 1) in fp32, lo / hi its floor / ceiling,
// w = rank - lo, and lerp(sorted[lo], sorted[hi], w) computed as fma(w, hi - lo, lo) for w < 1/2, else
// fma(-(hi - lo), 1 - w, hi) -- bit-identical to torch.quantile on the CPU.
//
// One CTA per (8 channels, call): the call's |x| of those channels are staged in shared memory (one column
// per warp), then each warp finds the two order statistics it needs by walking the distinct values down
// from the maximum (max below a threshold, and how many equal it, per step): the p99.99 calibration needs the
// top two values of a column, so that is one or two steps; any q works, with up to `rows` steps.  The
// results are max-accumulated into amax / pamax (non-negative floats order like their bit patterns).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cfloat>
#include <cstdint>

#include "ptx.cuh"

namespace svla {

constexpr int kPctCols = 8;         // channels per CTA, one warp each
constexpr int kPctMaxRows = 4096;   // tokens per call (shared memory: kPctCols * (rows + 1) floats)

inline size_t percentile_smem(int rows) { return static_cast<size_t>(kPctCols) * (rows + 1) * sizeof(float); }

struct PercentileArgs {
  const __nv_bfloat16* x;  // [calls * rows, ldx]
  long long ldx;
  int calls, rows, K;
  int lo, hi;              // floor / ceil of rank
  float w;                 // rank - lo
  float* amax;             // [K], max-accumulated
  float* pamax;            // [K], max-accumulated
};

__global__ void __launch_bounds__(kPctCols * 32) channel_percentile_kernel(PercentileArgs a) {
  extern __shared__ float pv[];  // [kPctCols][rows + 1]: the odd column stride keeps the staging stores conflict-free
  const int c0 = blockIdx.x * kPctCols, call = blockIdx.y;
  const __nv_bfloat16* xb = a.x + static_cast<size_t>(call) * a.rows * a.ldx;
  pdl_wait();
  pdl_trigger();
  for (int i = threadIdx.x; i < a.rows * kPctCols; i += blockDim.x) {
    const int r = i / kPctCols, c = i % kPctCols;
    float v = 0.f;
    if (c0 + c < a.K) v = fabsf(__bfloat162float(xb[static_cast<size_t>(r) * a.ldx + c0 + c]));
    pv[c * (a.rows + 1) + r] = v;
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int col = c0 + warp;
  if (col >= a.K) return;
  const float* v = pv + warp * (a.rows + 1);
  // ranks counted from the top: sorted[hi] is the (rows - 1 - hi)-th largest (0 = the maximum)
  const int top_hi = a.rows - 1 - a.hi, top_lo = a.rows - 1 - a.lo;
  float thr = INFINITY, v_hi = 0.f, v_lo = 0.f, amax = 0.f;
  int taken = 0;
  bool have_hi = false;
  for (int step = 0; step < a.rows; ++step) {
    float m = -1.0f;  // every value is >= 0
    for (int r = lane; r < a.rows; r += 32) {
      const float x = v[r];
      if (x < thr) m = fmaxf(m, x);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    int cnt = 0;
    for (int r = lane; r < a.rows; r += 32) cnt += (v[r] == m) ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) cnt += __shfl_xor_sync(0xffffffffu, cnt, o);
    if (step == 0) amax = m;
    if (!have_hi && taken + cnt > top_hi) {
      v_hi = m;
      have_hi = true;
    }
    if (taken + cnt > top_lo) {
      v_lo = m;
      break;
    }
    taken += cnt;
    thr = m;
  }
  const float d = __fsub_rn(v_hi, v_lo);
  const float p = (a.w < 0.5f) ? __fmaf_rn(a.w, d, v_lo) : __fmaf_rn(-d, __fsub_rn(1.0f, a.w), v_hi);
  if (lane == 0) {
    atomicMax(reinterpret_cast<unsigned int*>(a.amax + col), __float_as_uint(fmaxf(amax, 1e-8f)));
    atomicMax(reinterpret_cast<unsigned int*>(a.pamax + col), __float_as_uint(fmaxf(p, 1e-8f)));
  }
}

}  // namespace svla
