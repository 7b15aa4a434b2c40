"""Checkpoint -> packed weights.

``load_checkpoint`` reads a SmolVLA policy checkpoint (one ``.safetensors`` file, or a directory of shards,
with the policy's state-dict keys: ``model.vlm_with_expert.vlm.model.text_model.layers.{i}...``, the names
the reference's scale JSON and module regexes use, deploy/5Osmoothquant-alpha085-full-w8a8-deploy-eval.sh:40-42)
and infers the architecture from the tensor shapes (``infer_config``): layer counts, widths, heads, the
image size, the pixel-shuffle factor, and which expert layers cross-attend (their k_proj reads the VLM's
KV width instead of the expert width).

``save_packed`` / ``load_packed`` store the device-packed form (int8 weights with their per-channel scales,
SmoothQuant smooth vectors and reciprocals, activation scales, the bf16 weights of W8A16 linears and every
other tensor) in one safetensors file, so a deployment packs once and later loads without the scale JSON.
"""

from __future__ import annotations

import json
import math
import re
from pathlib import Path

import torch

from .config import BENCH, CONNECTOR, EXPERT, TEXT, VISION, SmolVLAConfig
from .model import DeviceWeights, PackedLinear, time_embedding_bf16
from .weights import linear_specs, other_specs


def load_checkpoint(path: str | Path) -> dict[str, torch.Tensor]:
    """All tensors of a safetensors file, or of every ``*.safetensors`` file of a directory (CPU)."""
    from safetensors.torch import load_file
    p = Path(path)
    files = sorted(p.glob("*.safetensors")) if p.is_dir() else [p]
    if not files:
        raise FileNotFoundError(f"no .safetensors file at {p}")
    state: dict[str, torch.Tensor] = {}
    for f in files:
        part = load_file(str(f))
        dup = set(part) & set(state)
        if dup:
            raise ValueError(f"{f}: keys repeated across shards: {sorted(dup)[:3]}")
        state.update(part)
    # lerobot saves the policy's state dict ("model." + module name); a bare VLAFlowMatching dict lacks the prefix
    if not any(k.startswith("model.") for k in state):
        state = {f"model.{k}": v for k, v in state.items()}
    return state


def _count_layers(state: dict, prefix: str) -> int:
    pat = re.compile(re.escape(prefix) + r"\.layers\.(\d+)\.")
    idx = {int(m.group(1)) for k in state for m in [pat.match(k)] if m}
    if not idx:
        return 0
    if idx != set(range(max(idx) + 1)):
        raise ValueError(f"{prefix}: layer indices are not contiguous: {sorted(idx)}")
    return max(idx) + 1


def infer_config(state: dict[str, torch.Tensor], base: SmolVLAConfig = BENCH) -> SmolVLAConfig:
    """The architecture of a checkpoint from its tensor shapes (fields no tensor determines keep ``base``:
    epsilons, RoPE wavelength, chunk, number of flow steps, language length, action_dim)."""
    def shape(k):
        if k not in state:
            raise KeyError(f"checkpoint has no {k}")
        return tuple(state[k].shape)

    hd = base.head_dim
    pe = shape(f"{VISION}.embeddings.patch_embedding.weight")  # [vis_hidden, channels, patch, patch]
    vis_hidden, channels, patch = pe[0], pe[1], pe[2]
    n_patches = shape(f"{VISION}.embeddings.position_embedding.weight")[0]
    grid = math.isqrt(n_patches)
    if grid * grid != n_patches:
        raise ValueError(f"position embedding of {n_patches} patches is not a square grid")
    vis_layers = _count_layers(state, f"{VISION}.encoder")
    vis_mlp = shape(f"{VISION}.encoder.layers.0.mlp.fc1.weight")[0]
    vis_heads = vis_hidden // hd
    conn = shape(f"{CONNECTOR}.weight")  # [hidden, vis_hidden * sf^2]
    sf = math.isqrt(conn[1] // vis_hidden)
    if sf * sf * vis_hidden != conn[1]:
        raise ValueError(f"connector input {conn[1]} is not vis_hidden * scale_factor^2")
    vocab, hidden = shape(f"{TEXT}.embed_tokens.weight")
    text_layers = _count_layers(state, TEXT)
    q = shape(f"{TEXT}.layers.0.self_attn.q_proj.weight")[0]
    kv = shape(f"{TEXT}.layers.0.self_attn.k_proj.weight")[0]
    mlp = shape(f"{TEXT}.layers.0.mlp.gate_proj.weight")[0]
    expert_layers = _count_layers(state, EXPERT)
    expert_hidden = shape(f"{EXPERT}.layers.0.input_layernorm.weight")[0]
    expert_mlp = shape(f"{EXPERT}.layers.0.mlp.gate_proj.weight")[0]
    # cross-attention layers project the VLM's cached K/V (width kv) instead of the expert hidden state
    cross = [shape(f"{EXPERT}.layers.{i}.self_attn.k_proj.weight")[1] == kv and kv != expert_hidden
             for i in range(expert_layers)]
    if not any(cross):
        every = 1  # every layer self-attends
    else:
        selfs = [i for i, c in enumerate(cross) if not c]
        every = selfs[1] - selfs[0] if len(selfs) > 1 else expert_layers
        if any((i % every == 0) == cross[i] for i in range(expert_layers)):
            raise ValueError(f"expert cross-attention layers {cross} do not follow one period")
    cfg = base.with_(image_size=grid * patch, patch=patch, channels=channels, vis_hidden=vis_hidden,
                     vis_layers=vis_layers, vis_heads=vis_heads, vis_mlp=vis_mlp, scale_factor=sf,
                     hidden=hidden, text_layers=text_layers, heads=q // hd, kv_heads=kv // hd, mlp=mlp,
                     vocab=vocab, expert_hidden=expert_hidden, expert_layers=expert_layers,
                     expert_mlp=expert_mlp, self_attn_every_n_layers=every,
                     max_state_dim=shape("model.state_proj.weight")[1],
                     max_action_dim=shape("model.action_in_proj.weight")[1])
    missing = [k for k in required_keys(cfg) if k not in state]
    if missing:
        raise KeyError(f"checkpoint lacks {len(missing)} tensors of the inferred architecture, e.g. {missing[:3]}")
    return cfg


def required_keys(cfg: SmolVLAConfig) -> list[str]:
    keys = []
    for name, _n, _k, has_bias, _kind in linear_specs(cfg):
        keys.append(f"{name}.weight")
        if has_bias:
            keys.append(f"{name}.bias")
    keys += [name for name, _shape, _kind in other_specs(cfg)]
    return keys


# ----------------------------------------------------------------------------- packed form

_FIELDS = ("weight", "wscale", "bias", "smooth", "rsmooth", "weight_deq")


def save_packed(weights: DeviceWeights, path: str | Path) -> None:
    """Write the device-packed weights (and the configuration) to one safetensors file."""
    from safetensors.torch import save_file
    tensors: dict[str, torch.Tensor] = {}
    meta = {"config": json.dumps(weights.cfg.as_dict()), "linears": {}}
    for name, p in weights.lin.items():
        meta["linears"][name] = {"n": p.n, "k": p.k, "kind": p.kind, "act_scale": p.act_scale}
        for f in _FIELDS:
            t = getattr(p, f)
            if t is not None:
                tensors[f"lin/{name}/{f}"] = t.detach().cpu().contiguous()
    for key, t in weights.t.items():
        # a copy: some tensors are views of others (patch_w2d reshapes the patch-embedding weight)
        tensors[f"t/{key}"] = t.detach().cpu().contiguous().clone()
    # derived constant the native engine reads instead of recomputing it (float64 on the host)
    tensors["t/time_embedding"] = time_embedding_bf16(weights.cfg).contiguous()
    save_file(tensors, str(path), metadata={"svla_packed": "1", "config": meta["config"],
                                            "linears": json.dumps(meta["linears"])})


def load_packed(path: str | Path, device="cuda") -> DeviceWeights:
    """DeviceWeights from a file written by ``save_packed`` (no packing kernels run)."""
    from safetensors import safe_open
    with safe_open(str(path), framework="pt") as f:
        meta = f.metadata() or {}
        if meta.get("svla_packed") != "1":
            raise ValueError(f"{path} is not a packed-weights file")
        cfg = SmolVLAConfig(**json.loads(meta["config"]))
        lin_meta = json.loads(meta["linears"])
        tensors = {k: f.get_tensor(k) for k in f.keys()}
    dev = torch.device(device)
    w = DeviceWeights.__new__(DeviceWeights)
    w.cfg, w.device = cfg, dev
    w.lin = {}
    for name, m in lin_meta.items():
        get = lambda f: tensors[f"lin/{name}/{f}"].to(dev) if f"lin/{name}/{f}" in tensors else None  # noqa: E731
        w.lin[name] = PackedLinear(m["n"], m["k"], m["kind"], get("weight"), get("wscale"), get("bias"),
                                   get("smooth"), get("rsmooth"), float(m["act_scale"]),
                                   weight_bf16=get("weight") if m["kind"] == "bf16" else None,
                                   weight_deq=get("weight_deq"))
    w.t = {k[2:]: v.to(dev) for k, v in tensors.items() if k.startswith("t/") and k != "t/time_embedding"}
    w.quantized = any(p.kind == "w8a8" for p in w.lin.values())
    torch.cuda.synchronize(dev)
    return w
