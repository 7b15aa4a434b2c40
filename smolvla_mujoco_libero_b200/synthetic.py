"""Seeded synthetic inputs with the shapes and value distributions of the benchmark workloads.

LIBERO rollouts (the reference's calibration and evaluation data,
deploy/calibrate_smolvla_activation_channel_scales.py:181-229) need a simulator
that cannot run here, so every workload uses these generators instead.  All
random draws use a CPU ``torch.Generator`` so that the same seed gives the same
bytes on any host with this torch version.

Workloads
---------
single SmoothQuant linear   X bf16 [177, 960] ~ N(0,1) with 8 seeded outlier
                            channels x30, W bf16 [2560, 960] ~ N(0, 0.02),
                            32 calibration batches from the same distribution.
decoder layer               hidden N(0,1) with outlier channels, L = 177.
observations                two fp32 [B,3,512,512] images U[0,1], 48 token ids
                            U[0, 49280), 8-dim state padded to 32,
                            noise N(0,1) [B, 50, 32].
"""

from __future__ import annotations

from dataclasses import dataclass

import torch

DEFAULT_SEED = 1000  # the reference's default seed (e.g. calibrate_smolvla_activation_channel_scales.py:34)


def generator(seed: int) -> torch.Generator:
    return torch.Generator(device="cpu").manual_seed(int(seed))


def outlier_channels(k: int, n_outliers: int, g: torch.Generator) -> torch.Tensor:
    return torch.randperm(k, generator=g)[:n_outliers].sort().values


def outlier_activations(m: int, k: int, channels: torch.Tensor, scale: float, g: torch.Generator,
                        dtype=torch.bfloat16) -> torch.Tensor:
    x = torch.randn(m, k, generator=g, dtype=torch.float32)
    x[:, channels] *= scale
    return x.to(dtype)


@dataclass
class LinearCase:
    x: torch.Tensor            # bf16 [M, K]
    weight: torch.Tensor       # bf16 [N, K]
    bias: torch.Tensor | None  # bf16 [N] or None
    calib: list[torch.Tensor]  # bf16 [M, K] each
    outliers: torch.Tensor     # int64 channel ids


def smoothquant_linear_case(seed: int = DEFAULT_SEED, m: int = 177, k: int = 960, n: int = 2560,
                            n_outliers: int = 8, outlier_scale: float = 30.0, n_calib: int = 32,
                            with_bias: bool = False, weight_std: float = 0.02) -> LinearCase:
    """The single-linear workload: X, W and the calibration batches, all seeded."""
    g = generator(seed)
    ch = outlier_channels(k, n_outliers, g)
    weight = (torch.randn(n, k, generator=g) * weight_std).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * weight_std).to(torch.bfloat16) if with_bias else None
    x = outlier_activations(m, k, ch, outlier_scale, g)
    calib = [outlier_activations(m, k, ch, outlier_scale, g) for _ in range(n_calib)]
    return LinearCase(x=x, weight=weight, bias=bias, calib=calib, outliers=ch)


@dataclass
class Observation:
    images: list[torch.Tensor]      # 2 x fp32 [B,3,H,W] in [0,1]
    img_masks: list[torch.Tensor]   # 2 x bool [B]
    lang_tokens: torch.Tensor       # int64 [B, T]
    lang_masks: torch.Tensor        # bool [B, T]
    state: torch.Tensor             # fp32 [B, max_state_dim]
    noise: torch.Tensor             # fp32 [B, chunk, max_action_dim]


def observations(batch: int, seed: int = DEFAULT_SEED, image_size: int = 512, n_tokens: int = 48,
                 vocab: int = 49280, state_dim: int = 8, max_state_dim: int = 32, chunk: int = 50,
                 max_action_dim: int = 32, n_valid_tokens: int | None = None) -> Observation:
    """Independent seeded observations (one generator stream per batch, sample b uses seed + b)."""
    imgs0, imgs1, toks, states, noises = [], [], [], [], []
    for b in range(batch):
        g = generator(seed + b)
        imgs0.append(torch.rand(3, image_size, image_size, generator=g))
        imgs1.append(torch.rand(3, image_size, image_size, generator=g))
        toks.append(torch.randint(0, vocab, (n_tokens,), generator=g))
        s = torch.zeros(max_state_dim)
        s[:state_dim] = torch.randn(state_dim, generator=g)
        states.append(s)
        noises.append(torch.randn(chunk, max_action_dim, generator=g))
    lang_masks = torch.ones(batch, n_tokens, dtype=torch.bool)
    if n_valid_tokens is not None:
        lang_masks[:, n_valid_tokens:] = False
    return Observation(
        images=[torch.stack(imgs0), torch.stack(imgs1)],
        img_masks=[torch.ones(batch, dtype=torch.bool), torch.ones(batch, dtype=torch.bool)],
        lang_tokens=torch.stack(toks),
        lang_masks=lang_masks,
        state=torch.stack(states),
        noise=torch.stack(noises),
    )
