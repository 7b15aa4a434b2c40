"""Policy-side pre- and post-processing of ``sample_actions`` on the device (libsvla kernels).

``prepare_images`` / ``prepare_state`` / ``unnormalize_actions`` are what lerobot's SmolVLA policy applies
before and after ``sample_actions`` in ``predict_action_chunk`` (``prepare_images`` / ``prepare_state``
are called at deploy/calibrate_smolvla_activation_channel_scales.py:138-139): aspect-preserving resize with
top/left padding to the model's square size and the [0, 1] -> [-1, 1] map SigLIP expects, state
normalisation with the dataset statistics and zero padding to ``max_state_dim``, and the inverse
normalisation of the first ``action_dim`` action channels.  Statistics are ``{"mean": .., "std": ..}``
(MEAN_STD) or ``{"min": .., "max": ..}`` (MIN_MAX) tensors of the feature width.
"""

from __future__ import annotations

import torch

from ._lib import check, lib
from .ops import _p, _stream


def _mode(stats: dict) -> tuple[int, torch.Tensor, torch.Tensor]:
    if "mean" in stats:
        return 0, stats["mean"], stats["std"]
    if "min" in stats:
        return 1, stats["min"], stats["max"]
    raise ValueError("stats need mean/std or min/max")


def prepare_images(images: torch.Tensor, size: int = 512, pad_value: float = 0.0, out: torch.Tensor | None = None):
    """images: fp32 [N, C, H, W] in [0, 1], or uint8 [N, H, W, C] camera frames -> fp32 [N, C, size, size] in
    [-1, 1].  ``out`` may be any [N, C, size, size] view whose images are contiguous (e.g. one camera of the
    runner's input buffer)."""
    if images.dtype == torch.uint8:
        n, h, w, c = images.shape
        u8 = 1
    elif images.dtype == torch.float32:
        n, c, h, w = images.shape
        u8 = 0
    else:
        raise TypeError("images must be fp32 NCHW or uint8 NHWC")
    images = images.contiguous()
    if out is None:
        out = torch.empty(n, c, size, size, dtype=torch.float32, device=images.device)
    if out.shape != (n, c, size, size) or out[0].stride() != (size * size, size, 1):
        raise ValueError("out must be [N, C, size, size] with contiguous images")
    check(lib().svla_resize_pad_images(_p(images), u8, n, c, h, w, _p(out), out.stride(0), size, size,
                                       float(pad_value), _stream()), "prepare_images")
    return out


def prepare_state(state: torch.Tensor, stats: dict, max_state_dim: int = 32) -> torch.Tensor:
    """state fp32 [B, dim] -> normalised and zero-padded fp32 [B, max_state_dim]."""
    mode, p0, p1 = _mode(stats)
    state = state.float().contiguous()
    b, dim = state.shape
    out = torch.empty(b, max_state_dim, dtype=torch.float32, device=state.device)
    check(lib().svla_normalize_state(_p(state), b, dim, dim, _p(p0.float().contiguous()), _p(p1.float().contiguous()),
                                     mode, max_state_dim, _p(out), _stream()), "prepare_state")
    return out


def unnormalize_actions(actions: torch.Tensor, stats: dict, action_dim: int) -> torch.Tensor:
    """actions fp32 [B, chunk, >= action_dim] (normalised) -> fp32 [B, chunk, action_dim]."""
    mode, p0, p1 = _mode(stats)
    a = actions.float().contiguous()
    b, t, ld = a.shape
    out = torch.empty(b, t, action_dim, dtype=torch.float32, device=a.device)
    check(lib().svla_unnormalize_actions(_p(a), b * t, ld, action_dim, _p(p0.float().contiguous()),
                                         _p(p1.float().contiguous()), mode, _p(out), _stream()), "unnormalize_actions")
    return out
