"""SmoothQuant calibration on the GPU, producing the reference's scale JSON.

Runs the unquantised (bf16) model through the same kernels as the deployed path (``SmolVLARunner`` in
mode "bf16") and observes the input of every W8A8-recipe linear, with the semantics of
  * PerChannelLinearInputCollector (deploy/calibrate_smolvla_activation_channel_scales.py:53-134):
    per call, per channel amax and torch.quantile(|x|, p/100) over all tokens, clamped at 1e-8;
    elementwise max over samples; scale = percentile_amax / 127 (clamp 1e-8);
  * build_entry (deploy/build_smoothquant_scales.py:55-106):
    amax_x = scale * 127; s = clamp(amax_x^alpha / amax_w^(1-alpha), 1e-4, 1e4);
    a = max(amax_x / s) / 127.
One "call" is one sample's pass through a module, as the reference hook sees it: per image for the vision
tower and connector (embed_image runs once per camera, deploy/trt_sample_actions_core_deploy.py:296-297),
per sample for the text layers.  The statistics run on the GPU (svla_channel_percentile).
"""

from __future__ import annotations

import json
from pathlib import Path
from typing import Any, Iterable

import torch

from . import ops
from .config import SmolVLAConfig
from .model import DeviceWeights, SmolVLARunner
from .weights import linear_specs


class ChannelStats:
    """Per module: elementwise max over calls of the per-call channel amax / percentile-amax, each call's
    statistics computed by the channel-percentile kernel (exact torch.quantile interpolation)."""

    def __init__(self, percentile: float):
        self.p = percentile
        self.calls: dict[str, dict[str, Any]] = {}

    def observe(self, modules: Iterable[str], x: torch.Tensor, rows_per_call: int) -> None:
        """x: [calls * rows_per_call, K] bf16, the input every module in `modules` sees."""
        k = x.shape[-1]
        amax = torch.zeros(k, dtype=torch.float32, device=x.device)
        pamax = torch.zeros_like(amax)
        ops.channel_percentile(x.reshape(-1, k), rows_per_call, self.p / 100.0, amax, pamax)
        n = x.reshape(-1, k).shape[0] // rows_per_call
        for module in modules:
            c = self.calls.get(module)
            if c is None:
                self.calls[module] = {"amax": amax, "pamax": pamax, "n": n, "shape": [rows_per_call, k]}
            else:
                c["amax"] = torch.maximum(c["amax"], amax)
                c["pamax"] = torch.maximum(c["pamax"], pamax)
                c["n"] += n


def smoothquant_entry(module: str, scale_list: torch.Tensor, weight: torch.Tensor, alpha: float,
                      smin: float = 1e-4, smax: float = 1e4, num_samples: int | None = None) -> dict:
    act_amax = (scale_list.to(torch.float32).cpu() * 127.0).clamp_min(1e-8)
    w_amax = weight.detach().to(torch.float32).cpu().abs().amax(dim=0).clamp_min(1e-8)
    smooth = (act_amax.pow(alpha) / w_amax.pow(1.0 - alpha)).clamp(min=smin, max=smax)
    smoothed = (act_amax / smooth).clamp_min(1e-8)
    scale = float((smoothed.max() / 127.0).item())
    return {
        "module": module,
        "channels": int(act_amax.numel()),
        "num_samples": num_samples,
        "scale": max(scale, 1e-8),
        "scale_source": f"smoothquant_alpha_{alpha:g}_from_per_channel",
        "quantization": "smoothquant_symmetric_static_per_tensor",
        "smoothquant_alpha": alpha,
        "smooth_scale": smooth.tolist(),
    }


def calibrate(cfg: SmolVLAConfig, state: dict[str, torch.Tensor], observations: Iterable, device="cuda",
              percentile: float | None = None, alpha: float | None = None) -> dict:
    """Scale JSON (dict) for every W8A8 linear of the path from bf16-model activations on the GPU."""
    percentile = cfg.percentile if percentile is None else percentile
    alpha = cfg.alpha if alpha is None else alpha
    dw = DeviceWeights(cfg, state, scales=None, device=device, keep_bf16=True)
    runner = None
    stats = ChannelStats(percentile)
    for obs in observations:
        b = obs.state.shape[0]
        if runner is None or runner.B != b:
            runner = SmolVLARunner(dw, b, mode="bf16")
        def observe(mods, buf, runner=runner, b=b):
            rows = buf.shape[0]
            if buf is runner.conn_in:
                per = cfg.n_img_tokens
            elif rows == b * cfg.n_cams * cfg.n_patches:
                per = cfg.n_patches
            else:
                per = cfg.prefix_len
            stats.observe(mods, buf, per)

        runner(obs.images, obs.img_masks, obs.lang_tokens, obs.lang_masks, obs.state, obs.noise, observer=observe)
    torch.cuda.synchronize()
    specs = {name: (n, k) for name, n, k, _, q in linear_specs(cfg) if q == "w8a8"}
    entries = []
    for module, c in stats.calls.items():
        if module not in specs:
            continue
        # on the CPU: a CUDA tensor divided by a Python scalar is multiplied by the scalar's reciprocal, which
        # can differ by one ulp from the division the collector's arithmetic (and the golden fixtures) use
        scale_list = (c["pamax"].cpu() / 127.0).clamp_min(1e-8)
        entries.append(smoothquant_entry(module, scale_list, state[f"{module}.weight"], alpha, num_samples=c["n"]))
    missing = set(specs) - {e["module"] for e in entries}
    if missing:
        raise RuntimeError(f"calibration did not observe {sorted(missing)[:4]} ...")
    return {
        "scale_granularity": "smoothquant_per_tensor_activation_with_per_input_channel_smoothing",
        "smoothquant_formula": "s = activation_amax**alpha / weight_input_amax**(1-alpha); x'=x/s; W'=W*s",
        "smoothquant_alpha": alpha,
        "percentile": percentile,
        "linear_call_scales": entries,
    }


def load_scale_json(src: str | Path | dict) -> dict[str, Any]:
    """module -> entry, the SmoothQuant / symmetric cases of load_activation_scales_by_module
    (deploy/linear_only_quant.py:208-246); duplicate module entries become a list."""
    data = src if isinstance(src, dict) else json.loads(Path(src).read_text())
    out: dict[str, Any] = {}
    for e in data.get("linear_call_scales", []):
        name = str(e.get("module", ""))
        if not name:
            continue
        q = str(e.get("quantization", ""))
        if q == "smoothquant_symmetric_static_per_tensor":
            if not isinstance(e.get("smooth_scale"), list):
                raise ValueError(f"missing smooth_scale list for SmoothQuant module: {name}")
            val = {"quantization": q, "scale": max(float(e.get("scale", 1e-8)), 1e-8),
                   "smooth_scale": [max(float(v), 1e-8) for v in e["smooth_scale"]],
                   "smoothquant_alpha": e.get("smoothquant_alpha")}
        elif q in ("asymmetric_static_per_tensor", "smoothquant_asymmetric_static_per_tensor"):
            raise ValueError(f"{name}: asymmetric activation quantisation is not part of the deployed recipe")
        else:
            val = e.get("scale")
        prev = out.get(name)
        if prev is None:
            out[name] = val
        elif isinstance(prev, list) and prev and isinstance(prev[0], dict):
            prev.append(val)
        else:
            out[name] = [prev, val]
    return out
