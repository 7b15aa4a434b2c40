"""CPU oracle of the policy-side processing (test infrastructure only).

lerobot's SmolVLA ``prepare_images`` (resize_with_pad to 512 with pad value 0, then x * 2 - 1),
``prepare_state`` (Normalize then pad_vector) and the output Unnormalize, which the reference calls at
deploy/calibrate_smolvla_activation_channel_scales.py:138-139 but does not ship (lerobot 0.5.1 is absent):
restated from that published algorithm with torch's own interpolate / pad.  Parity unpinned (no golden
vectors exist for these in the reference).
"""

from __future__ import annotations

import torch
import torch.nn.functional as F


def resize_with_pad(img: torch.Tensor, width: int, height: int, pad_value: float = 0.0) -> torch.Tensor:
    cur_h, cur_w = img.shape[2:]
    ratio = max(cur_w / width, cur_h / height)
    rh, rw = int(cur_h / ratio), int(cur_w / ratio)
    resized = F.interpolate(img, size=(rh, rw), mode="bilinear", align_corners=False)
    return F.pad(resized, (max(0, width - rw), 0, max(0, height - rh), 0), value=pad_value)


def prepare_images(images: torch.Tensor, size: int = 512) -> torch.Tensor:
    if images.dtype == torch.uint8:  # camera frames HWC -> CHW in [0, 1]
        images = images.permute(0, 3, 1, 2).float() / 255.0
    return resize_with_pad(images.float(), size, size, pad_value=0.0) * 2.0 - 1.0


def prepare_state(state: torch.Tensor, stats: dict, max_state_dim: int) -> torch.Tensor:
    if "mean" in stats:
        x = (state - stats["mean"]) / (stats["std"] + 1e-8)
    else:
        x = (state - stats["min"]) / (stats["max"] - stats["min"] + 1e-8) * 2 - 1
    return F.pad(x, (0, max_state_dim - x.shape[1]))


def unnormalize_actions(actions: torch.Tensor, stats: dict, action_dim: int) -> torch.Tensor:
    a = actions[..., :action_dim]
    if "mean" in stats:
        return a * stats["std"] + stats["mean"]
    return (a + 1) / 2 * (stats["max"] - stats["min"]) + stats["min"]
