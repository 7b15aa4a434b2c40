"""CPU restatement of the SmolVLA sample_actions core with SmoothQuant fake-dequant linears (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The model code (VLAFlowMatching, SmolVLMWithExpertModel) lives in lerobot 0.5.1, which the reference does
not ship; everything here that lerobot computes is restated from the reference's call sites and
restatements and is therefore UNPINNED:
  * prefix embed, masks, positions, denoise loop: deploy/diagnose_3_4_numeric_baseline.py:42-206
  * attention: deploy/export_6f_layer0_attention_tensors.py:100-119, expand_kv
    deploy/diagnose_5i_attention_error_propagation.py:205-226
  * RoPE: deploy/validate_fused_rope_layout_math.py:28-42 (the only part pinned: tests/golden/rope_kat.npz)
  * SigLIP encoder, pixel-shuffle connector, Llama RMSNorm / MLP: transformers SmolVLM / Llama semantics
  * action expert, embed_suffix, cross-attention: lerobot 0.5.1 semantics (expert layers interleave
    self-attention over [prefix KV ; suffix] with cross-attention whose K/V are the expert's k_proj / v_proj
    applied to the cached prefix K (post-RoPE) and V; cross-attention queries use positions 0..49).
Linears follow deploy/linear_only_quant.py through oracle.quant (pinned by the golden fixtures).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

MASKED = torch.finfo(torch.float32).min


# ----------------------------------------------------------------------------- primitives

def apply_rope(x: torch.Tensor, positions: torch.Tensor, max_wavelength: float = 10_000.0) -> torch.Tensor:
    """Rotate-half RoPE on x [B, L, H, D] (deploy/validate_fused_rope_layout_math.py:28-42)."""
    d_half = x.shape[-1] // 2
    dtype = x.dtype
    xf = x.to(torch.float32)
    freq_exponents = (2.0 / x.shape[-1]) * torch.arange(d_half, dtype=torch.float32)
    timescale = max_wavelength ** freq_exponents
    radians = positions[..., None].to(torch.float32) / timescale[None, None, :]
    radians = radians[..., None, :]
    sin, cos = torch.sin(radians), torch.cos(radians)
    x1, x2 = xf.split(d_half, dim=-1)
    out = torch.empty_like(xf)
    out[..., :d_half] = x1 * cos - x2 * sin
    out[..., d_half:] = x2 * cos + x1 * sin
    return out.to(dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """transformers LlamaRMSNorm: weight * bf16(x * rsqrt(mean(x^2) + eps))."""
    dtype = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return weight * h.to(dtype)


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def pixel_shuffle(x: torch.Tensor, scale: int) -> torch.Tensor:
    """SmolVLM connector pixel shuffle: [B, S, D] -> [B, S / scale^2, D * scale^2]."""
    bsz, seq, dim = x.shape
    side = int(seq ** 0.5)
    x = x.view(bsz, side, side, dim)
    x = x.view(bsz, side, side // scale, dim * scale)
    x = x.permute(0, 2, 1, 3)
    x = x.reshape(bsz, side // scale, side // scale, dim * scale * scale)
    x = x.permute(0, 2, 1, 3)
    return x.reshape(bsz, seq // (scale * scale), dim * scale * scale)


def eager_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None, hq: int,
                    hkv: int) -> torch.Tensor:
    """q [B, Lq, hq*64], k/v [B, Lk, hkv*64] (bf16, post-RoPE), mask bool [B, Lq, Lk] -> bf16 [B, Lq, hq*64].

    deploy/export_6f_layer0_attention_tensors.py:100-119 with the GQA expansion of
    deploy/diagnose_5i_attention_error_propagation.py:205-226."""
    b, lq, _ = q.shape
    lk = k.shape[1]
    d = 64
    groups = hq // hkv
    qh = q.view(b, lq, hq, d)
    kh = k.view(b, lk, hkv, 1, d).expand(b, lk, hkv, groups, d).reshape(b, lk, hq, d)
    vh = v.view(b, lk, hkv, 1, d).expand(b, lk, hkv, groups, d).reshape(b, lk, hq, d)
    qt = qh.to(torch.float32).transpose(1, 2)
    kt = kh.to(torch.float32).transpose(1, 2)
    scores = torch.matmul(qt, kt.transpose(2, 3)) * (d ** -0.5)
    if mask is not None:
        scores = torch.where(mask[:, None, :, :], scores, MASKED)
    probs = torch.softmax(scores, dim=-1)
    ctx = torch.matmul(probs.to(vh.dtype), vh.permute(0, 2, 1, 3))
    return ctx.permute(0, 2, 1, 3).reshape(b, lq, hq * d)


def make_att_2d_masks(pad_masks: torch.Tensor, att_masks: torch.Tensor) -> torch.Tensor:
    """deploy/diagnose_3_4_numeric_baseline.py:42-46."""
    cumsum = torch.cumsum(att_masks.to(torch.int64), dim=1)
    att_2d = cumsum[:, None, :] <= cumsum[:, :, None]
    pad_2d = pad_masks[:, None, :] & pad_masks[:, :, None]
    return att_2d & pad_2d


def sinusoidal_time_embedding(t: torch.Tensor, dim: int, min_period: float, max_period: float) -> torch.Tensor:
    """lerobot create_sinusoidal_pos_embedding (float64 internally)."""
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = min_period * (max_period / min_period) ** fraction
    scaling = 1.0 / period * 2 * math.pi
    sin_input = scaling[None, :] * t.to(torch.float64)[:, None]
    return torch.cat([torch.sin(sin_input), torch.cos(sin_input)], dim=1)
