// Policy-side pre- and post-processing around sample_actions (lerobot SmolVLA prepare_images /
// prepare_state and the action unnormalisation of predict_action_chunk, called at
// deploy/calibrate_smolvla_activation_channel_scales.py:138-139):
//   images : resize keeping the aspect ratio (bilinear, half-pixel source index: src = (dst + 0.5) * in / out
//            - 0.5, clamped at 0 -- torch's interpolate with align_corners=False), pad on the top and left to
//            the model's square size, then map [0, 1] to [-1, 1] (x * 2 - 1) as SigLIP expects
//   state  : MEAN_STD (x - mean) / (std + 1e-8) or MIN_MAX ((x - min) / (max - min + 1e-8)) * 2 - 1,
//            zero-padded to max_state_dim
//   actions: on the first action_dim channels, MEAN_STD x * std + mean, MIN_MAX (x + 1) / 2 * (max - min) + min
#pragma once

#include "ptx.cuh"

namespace svla {

struct ResizeArgs {
  const void* src;  // fp32 [N, C, H, W] in [0, 1], or uint8 [N, H, W, C] (value / 255)
  int u8_hwc;
  int N, C, H, W;
  int rh, rw;       // resized size (the image part of the output), computed on the host
  int OH, OW;       // output size; the top OH - rh rows and left OW - rw columns are padding
  float pad_value;  // in [0, 1] units, before the [-1, 1] map
  float* out;       // out[n * out_stride + (c * OH + y) * OW + x]
  long long out_stride;
};

__device__ __forceinline__ float resize_src(const ResizeArgs& a, int n, int c, int y, int x) {
  if (a.u8_hwc) {
    const uint8_t* s = static_cast<const uint8_t*>(a.src);
    return __fdiv_rn(static_cast<float>(s[((static_cast<size_t>(n) * a.H + y) * a.W + x) * a.C + c]), 255.0f);
  }
  const float* s = static_cast<const float*>(a.src);
  return s[((static_cast<size_t>(n) * a.C + c) * a.H + y) * a.W + x];
}

__global__ void resize_pad_kernel(const ResizeArgs a) {
  pdl_wait();
  pdl_trigger();
  const long long idx = static_cast<long long>(blockIdx.x) * blockDim.x + threadIdx.x;
  const long long total = static_cast<long long>(a.N) * a.C * a.OH * a.OW;
  if (idx >= total) return;
  const int ox = static_cast<int>(idx % a.OW);
  const int oy = static_cast<int>((idx / a.OW) % a.OH);
  const int c = static_cast<int>((idx / (static_cast<long long>(a.OW) * a.OH)) % a.C);
  const int n = static_cast<int>(idx / (static_cast<long long>(a.OW) * a.OH * a.C));
  const int py = a.OH - a.rh, px = a.OW - a.rw;
  float v;
  if (oy < py || ox < px) {
    v = a.pad_value;
  } else {
    const int y = oy - py, x = ox - px;
    const float sh = static_cast<float>(a.H) / static_cast<float>(a.rh);
    const float sw = static_cast<float>(a.W) / static_cast<float>(a.rw);
    const float fy = fmaxf(__fsub_rn(__fmul_rn(sh, __fadd_rn(static_cast<float>(y), 0.5f)), 0.5f), 0.0f);
    const float fx = fmaxf(__fsub_rn(__fmul_rn(sw, __fadd_rn(static_cast<float>(x), 0.5f)), 0.5f), 0.0f);
    const int y0 = static_cast<int>(fy), x0 = static_cast<int>(fx);
    const int y1 = y0 + (y0 < a.H - 1 ? 1 : 0), x1 = x0 + (x0 < a.W - 1 ? 1 : 0);
    const float ly = fminf(fmaxf(__fsub_rn(fy, static_cast<float>(y0)), 0.0f), 1.0f);
    const float lx = fminf(fmaxf(__fsub_rn(fx, static_cast<float>(x0)), 0.0f), 1.0f);
    const float hy = __fsub_rn(1.0f, ly), hx = __fsub_rn(1.0f, lx);
    const float top = __fadd_rn(__fmul_rn(hx, resize_src(a, n, c, y0, x0)), __fmul_rn(lx, resize_src(a, n, c, y0, x1)));
    const float bot = __fadd_rn(__fmul_rn(hx, resize_src(a, n, c, y1, x0)), __fmul_rn(lx, resize_src(a, n, c, y1, x1)));
    v = __fadd_rn(__fmul_rn(hy, top), __fmul_rn(ly, bot));
  }
  a.out[static_cast<size_t>(n) * a.out_stride + (static_cast<size_t>(c) * a.OH + oy) * a.OW + ox] =
      __fsub_rn(__fmul_rn(v, 2.0f), 1.0f);
}

// state [B, dim] (row stride ld) -> normalised and zero-padded [B, out_dim]; mode 0 MEAN_STD (p0 mean, p1 std),
// 1 MIN_MAX (p0 min, p1 max)
__global__ void normalize_state_kernel(const float* x, int B, int dim, int ld, const float* p0, const float* p1,
                                       int mode, int out_dim, float* out) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= B * out_dim) return;
  const int b = idx / out_dim, j = idx % out_dim;
  float v = 0.0f;
  if (j < dim) {
    const float s = x[static_cast<size_t>(b) * ld + j];
    if (mode == 0) {
      v = __fdiv_rn(__fsub_rn(s, p0[j]), __fadd_rn(p1[j], 1e-8f));
    } else {
      v = __fdiv_rn(__fsub_rn(s, p0[j]), __fadd_rn(__fsub_rn(p1[j], p0[j]), 1e-8f));
      v = __fsub_rn(__fmul_rn(v, 2.0f), 1.0f);
    }
  }
  out[idx] = v;
}

// actions [B, chunk, ld] (the first action_dim channels) -> unnormalised [B, chunk, action_dim]
__global__ void unnormalize_actions_kernel(const float* a, int rows, int ld, int action_dim, const float* p0,
                                           const float* p1, int mode, float* out) {
  pdl_wait();
  pdl_trigger();
  const int idx = blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= rows * action_dim) return;
  const int r = idx / action_dim, j = idx % action_dim;
  float v = a[static_cast<size_t>(r) * ld + j];
  if (mode == 0) {
    v = __fadd_rn(__fmul_rn(v, p1[j]), p0[j]);
  } else {
    v = __fdiv_rn(__fadd_rn(v, 1.0f), 2.0f);
    v = __fadd_rn(__fmul_rn(v, __fsub_rn(p1[j], p0[j])), p0[j]);
  }
  out[idx] = v;
}

}  // namespace svla
