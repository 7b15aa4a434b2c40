"""Weight naming and seeded random initialisation for the SmolVLA sample_actions path.

Names follow the reference checkpoint's module paths (the keys the scale JSON uses, e.g.
``model.vlm_with_expert.vlm.model.text_model.layers.3.self_attn.q_proj``), with ``.weight`` / ``.bias``
suffixes.  There is no network and no checkpoint here, so the benchmark uses random-init weights of the
architecture: linear weights and biases N(0, 0.02), norm weights 1 + N(0, 0.1), LayerNorm biases N(0, 0.02),
embedding tables N(0, 0.02).  All draws come from one CPU generator, so a seed fixes the bytes.
"""

from __future__ import annotations

import torch

from .config import CONNECTOR, EXPERT, TEXT, VISION, SmolVLAConfig


def linear_specs(cfg: SmolVLAConfig) -> list[tuple[str, int, int, bool, str]]:
    """(module, out_features, in_features, has_bias, quantization) for every linear on the path.

    quantization: "w8a8" (SmoothQuant static per-tensor), "w8a16" or "bf16" -- the production recipe of
    deploy/6Nalpha085-vlm-a8w8-lm-expert-w8a16-deploy-eval.sh:37-45 (text q/k/v/o/gate/up W8A8, down and
    every expert linear W8A16) extended to the vision tower and connector (W8A8)."""
    s: list[tuple[str, int, int, bool, str]] = []
    for i in range(cfg.vis_layers):
        p = f"{VISION}.encoder.layers.{i}"
        for n in ("q_proj", "k_proj", "v_proj", "out_proj"):
            s.append((f"{p}.self_attn.{n}", cfg.vis_hidden, cfg.vis_hidden, True, "w8a8"))
        s.append((f"{p}.mlp.fc1", cfg.vis_mlp, cfg.vis_hidden, True, "w8a8"))
        s.append((f"{p}.mlp.fc2", cfg.vis_hidden, cfg.vis_mlp, True, "w8a8"))
    s.append((CONNECTOR, cfg.hidden, cfg.vis_hidden * cfg.scale_factor ** 2, False, "w8a8"))
    for i in range(cfg.text_layers):
        p = f"{TEXT}.layers.{i}"
        s.append((f"{p}.self_attn.q_proj", cfg.q_dim, cfg.hidden, False, "w8a8"))
        s.append((f"{p}.self_attn.k_proj", cfg.kv_dim, cfg.hidden, False, "w8a8"))
        s.append((f"{p}.self_attn.v_proj", cfg.kv_dim, cfg.hidden, False, "w8a8"))
        s.append((f"{p}.self_attn.o_proj", cfg.hidden, cfg.q_dim, False, "w8a8"))
        s.append((f"{p}.mlp.gate_proj", cfg.mlp, cfg.hidden, False, "w8a8"))
        s.append((f"{p}.mlp.up_proj", cfg.mlp, cfg.hidden, False, "w8a8"))
        s.append((f"{p}.mlp.down_proj", cfg.hidden, cfg.mlp, False, "w8a16"))
    for i in range(cfg.expert_layers):
        p = f"{EXPERT}.layers.{i}"
        kv_in = cfg.kv_dim if cfg.is_cross_layer(i) else cfg.expert_hidden
        s.append((f"{p}.self_attn.q_proj", cfg.q_dim, cfg.expert_hidden, False, "w8a16"))
        s.append((f"{p}.self_attn.k_proj", cfg.kv_dim, kv_in, False, "w8a16"))
        s.append((f"{p}.self_attn.v_proj", cfg.kv_dim, kv_in, False, "w8a16"))
        s.append((f"{p}.self_attn.o_proj", cfg.expert_hidden, cfg.q_dim, False, "w8a16"))
        s.append((f"{p}.mlp.gate_proj", cfg.expert_mlp, cfg.expert_hidden, False, "w8a16"))
        s.append((f"{p}.mlp.up_proj", cfg.expert_mlp, cfg.expert_hidden, False, "w8a16"))
        s.append((f"{p}.mlp.down_proj", cfg.expert_hidden, cfg.expert_mlp, False, "w8a16"))
    e = cfg.expert_hidden
    s.append(("model.state_proj", cfg.hidden, cfg.max_state_dim, True, "bf16"))
    s.append(("model.action_in_proj", e, cfg.max_action_dim, True, "bf16"))
    s.append(("model.action_out_proj", cfg.max_action_dim, e, True, "bf16"))
    s.append(("model.action_time_mlp_in", e, 2 * e, True, "bf16"))
    s.append(("model.action_time_mlp_out", e, e, True, "bf16"))
    return s


def other_specs(cfg: SmolVLAConfig) -> list[tuple[str, tuple[int, ...], str]]:
    """(name, shape, init) for the non-linear parameters.  init: "w" N(0,0.02), "norm" 1+N(0,0.1), "bias"."""
    s: list[tuple[str, tuple[int, ...], str]] = []
    p = f"{VISION}.embeddings"
    s.append((f"{p}.patch_embedding.weight", (cfg.vis_hidden, cfg.channels, cfg.patch, cfg.patch), "w"))
    s.append((f"{p}.patch_embedding.bias", (cfg.vis_hidden,), "w"))
    s.append((f"{p}.position_embedding.weight", (cfg.n_patches, cfg.vis_hidden), "w"))
    for i in range(cfg.vis_layers):
        q = f"{VISION}.encoder.layers.{i}"
        for ln in ("layer_norm1", "layer_norm2"):
            s.append((f"{q}.{ln}.weight", (cfg.vis_hidden,), "norm"))
            s.append((f"{q}.{ln}.bias", (cfg.vis_hidden,), "w"))
    s.append((f"{VISION}.post_layernorm.weight", (cfg.vis_hidden,), "norm"))
    s.append((f"{VISION}.post_layernorm.bias", (cfg.vis_hidden,), "w"))
    s.append((f"{TEXT}.embed_tokens.weight", (cfg.vocab, cfg.hidden), "w"))
    for i in range(cfg.text_layers):
        s.append((f"{TEXT}.layers.{i}.input_layernorm.weight", (cfg.hidden,), "norm"))
        s.append((f"{TEXT}.layers.{i}.post_attention_layernorm.weight", (cfg.hidden,), "norm"))
    s.append((f"{TEXT}.norm.weight", (cfg.hidden,), "norm"))
    for i in range(cfg.expert_layers):
        s.append((f"{EXPERT}.layers.{i}.input_layernorm.weight", (cfg.expert_hidden,), "norm"))
        s.append((f"{EXPERT}.layers.{i}.post_attention_layernorm.weight", (cfg.expert_hidden,), "norm"))
    s.append((f"{EXPERT}.norm.weight", (cfg.expert_hidden,), "norm"))
    return s


def random_weights(cfg: SmolVLAConfig, seed: int = 0, std: float = 0.02) -> dict[str, torch.Tensor]:
    """Seeded bf16 state dict on the CPU."""
    g = torch.Generator(device="cpu").manual_seed(int(seed))
    out: dict[str, torch.Tensor] = {}
    for name, n, k, bias, _ in linear_specs(cfg):
        out[f"{name}.weight"] = (torch.randn(n, k, generator=g) * std).to(torch.bfloat16)
        if bias:
            out[f"{name}.bias"] = (torch.randn(n, generator=g) * std).to(torch.bfloat16)
    for name, shape, kind in other_specs(cfg):
        t = torch.randn(*shape, generator=g)
        t = 1.0 + 0.1 * t if kind == "norm" else t * std
        out[name] = t.to(torch.bfloat16)
    return out


def w8a8_modules(cfg: SmolVLAConfig) -> list[str]:
    return [name for name, _, _, _, q in linear_specs(cfg) if q == "w8a8"]
