"""SmoothQuant W8A8 / W8A16 fake-dequant arithmetic, restated on CPU (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Every function cites the reference line it restates.  The rounding rules
that the CUDA path must match bit-exactly are:

* weights   (deploy/linear_only_quant.py:140-144)
      w_s[n] = max_k |W'[n,k]|  (clamp 1e-8)  / 127          (fp32, IEEE divide)
      qw     = round_half_even(W' / w_s[n]).clamp(-127, 127)  (int8)
  with W' = W.f32 * s[None, :] when a SmoothQuant smooth vector s is given
  (deploy/linear_only_quant.py:43-53).
* activations (deploy/linear_only_quant.py:104-116, :158-162)
      x_s = x.f32 / s[k]                                        (IEEE divide)
      qx  = round_half_even(x_s / a).clamp(-128, 127)           (IEEE divide)
* fake-dequant output (deploy/linear_only_quant.py:116)
      y = F.linear(bf16(qx * a), bf16(qw * w_s), bias_bf16)     (bf16 GEMM)
* integer-dequant fp32 form (deploy/export_6g_smoothquant_linear_tensors.py:121-125,
  deploy/cuda/smoothquant_linear_epilogue.cu:139-149)
      y = (acc_i32 * a) * w_s[n] + b[n]                         (fp32)
"""

from __future__ import annotations

import json
import re
from pathlib import Path
from typing import Any

import torch
import torch.nn.functional as F

SCALE_FLOOR = 1.0e-8


# ---------------------------------------------------------------------------
# weights
# ---------------------------------------------------------------------------

def quantize_weight_per_out_channel(weight: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """deploy/linear_only_quant.py:140-144."""
    w = weight.detach().to(torch.float32)
    scale = w.abs().amax(dim=1, keepdim=True).clamp_min(SCALE_FLOOR) / 127.0
    qweight = torch.round(w / scale).clamp(-127, 127).to(torch.int8)
    return qweight, scale.squeeze(1)


def dequantize_weight(qweight: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    """deploy/linear_only_quant.py:147-148 (fp32 result; callers cast to bf16)."""
    return qweight.to(torch.float32) * scale[:, None].to(torch.float32)


def smooth_weight(weight: torch.Tensor, smooth_scale: torch.Tensor | None) -> torch.Tensor:
    """The smoothing fold of W8A8Linear.__init__ (deploy/linear_only_quant.py:43-51)."""
    w = weight.detach().to(torch.float32)
    if smooth_scale is None:
        return w
    s = torch.as_tensor(smooth_scale, dtype=torch.float32).clamp_min(SCALE_FLOOR)
    if s.ndim != 1 or s.numel() != w.shape[1]:
        raise ValueError(f"smooth_scale shape {tuple(s.shape)} does not match Linear in_features {w.shape[1]}")
    return w * s[None, :]


def pack_w8a8_weight(weight: torch.Tensor, smooth_scale: torch.Tensor | None):
    """W8A8Linear.__init__ weight path: fold s, then per-out-channel int8 (linear_only_quant.py:43-54)."""
    return quantize_weight_per_out_channel(smooth_weight(weight, smooth_scale))


# ---------------------------------------------------------------------------
# activations
# ---------------------------------------------------------------------------

def quantize_activation_static(x: torch.Tensor, scale: float | torch.Tensor) -> torch.Tensor:
    """The quantize half of quantize_dequantize_activation_static (linear_only_quant.py:158-161)."""
    xf = x.to(torch.float32)
    a = torch.as_tensor(scale, dtype=torch.float32).clamp_min(SCALE_FLOOR)
    return torch.round(xf / a).clamp(-128, 127).to(torch.int8)


def smooth_quantize_activation(x: torch.Tensor, smooth_scale: torch.Tensor | None, act_scale: float) -> torch.Tensor:
    """W8A8Linear.forward up to the int8 tensor (linear_only_quant.py:105-107 then :158-161).

    The divide by s happens on x.float32 (two IEEE divides, no reciprocal)."""
    xf = x.to(torch.float32)
    if smooth_scale is not None:
        xf = xf / torch.as_tensor(smooth_scale, dtype=torch.float32).clamp_min(SCALE_FLOOR)
    return quantize_activation_static(xf, act_scale)


# ---------------------------------------------------------------------------
# linear forms
# ---------------------------------------------------------------------------

def int_gemm(qx: torch.Tensor, qw: torch.Tensor) -> torch.Tensor:
    """Exact int32 accumulators  acc[m,n] = sum_k qx[m,k] * qw[n,k]  (smoothquant_linear_epilogue.cu:121-137)."""
    acc = qx.to(torch.int64) @ qw.to(torch.int64).t()
    assert acc.abs().max() < 2**31
    return acc.to(torch.int32)


def w8a8_int_dequant(acc: torch.Tensor, act_scale: float, weight_scale: torch.Tensor,
                     bias: torch.Tensor | None) -> torch.Tensor:
    """fp32 integer-dequant form  (acc*a)*w_s[n] + b[n]  (smoothquant_linear_epilogue.cu:139-149)."""
    a = torch.tensor(act_scale, dtype=torch.float32)
    y = (acc.to(torch.float32) * a) * weight_scale.to(torch.float32)[None, :]
    if bias is not None:
        y = y + bias.to(torch.float32)[None, :]
    return y


def w8a8_fake_dequant(qx: torch.Tensor, act_scale: float, qweight: torch.Tensor, weight_scale: torch.Tensor,
                      bias: torch.Tensor | None) -> torch.Tensor:
    """bf16 fake-dequant output of W8A8Linear.forward (linear_only_quant.py:54, :109-116)."""
    a = torch.tensor(act_scale, dtype=torch.float32).clamp_min(SCALE_FLOOR)
    x_deq = (qx.to(torch.float32) * a).to(torch.bfloat16)
    w_deq = dequantize_weight(qweight, weight_scale).to(torch.bfloat16)
    b = None if bias is None else bias.to(torch.bfloat16)
    return F.linear(x_deq, w_deq, b)


class W8A8Linear:
    """Restatement of deploy/linear_only_quant.py:40-116 (static symmetric per-tensor SmoothQuant case)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None, act_scale: float,
                 smooth_scale: torch.Tensor | None):
        self.smooth_scale = None if smooth_scale is None else \
            torch.as_tensor(smooth_scale, dtype=torch.float32).clamp_min(SCALE_FLOOR)
        self.qweight, self.weight_scale = pack_w8a8_weight(weight, self.smooth_scale)
        self.weight = dequantize_weight(self.qweight, self.weight_scale).to(torch.bfloat16)
        self.bias = None if bias is None else bias.detach().to(torch.bfloat16)
        self.act_scale = max(float(act_scale), SCALE_FLOOR)
        self.in_features = int(weight.shape[1])
        self.out_features = int(weight.shape[0])

    def quantize_input(self, x: torch.Tensor) -> torch.Tensor:
        return smooth_quantize_activation(x, self.smooth_scale, self.act_scale)

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        shape = x.shape
        qx = self.quantize_input(x.reshape(-1, shape[-1]))
        a = torch.tensor(self.act_scale, dtype=torch.float32)
        x_deq = (qx.to(torch.float32) * a).to(torch.bfloat16)
        y = F.linear(x_deq, self.weight, self.bias)
        return y.reshape(*shape[:-1], self.out_features)


class W8A16Linear:
    """Restatement of deploy/linear_only_quant.py:119-137."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None):
        self.qweight, self.weight_scale = quantize_weight_per_out_channel(weight)
        self.weight = dequantize_weight(self.qweight, self.weight_scale).to(torch.bfloat16)
        self.bias = None if bias is None else bias.detach().to(torch.bfloat16)
        self.in_features = int(weight.shape[1])
        self.out_features = int(weight.shape[0])

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x.to(torch.bfloat16), self.weight, self.bias)


class Bf16Linear:
    """A plain bf16 nn.Linear (the modules the production recipe leaves unquantized)."""

    def __init__(self, weight: torch.Tensor, bias: torch.Tensor | None):
        self.weight = weight.detach().to(torch.bfloat16)
        self.bias = None if bias is None else bias.detach().to(torch.bfloat16)
        self.in_features = int(weight.shape[1])
        self.out_features = int(weight.shape[0])

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return F.linear(x.to(torch.bfloat16), self.weight, self.bias)


# ---------------------------------------------------------------------------
# calibration and SmoothQuant scale building
# ---------------------------------------------------------------------------

def per_channel_percentile_amax(x: torch.Tensor, percentile: float) -> tuple[torch.Tensor, torch.Tensor]:
    """The forward-pre-hook of PerChannelLinearInputCollector
    (deploy/calibrate_smolvla_activation_channel_scales.py:68-84): per-channel amax and
    torch.quantile(|x|, p/100, dim=0) over all tokens, both clamped at 1e-8."""
    t = x.detach().to(torch.float32)
    flat = t.abs().reshape(-1, t.shape[-1])
    amax = flat.amax(dim=0).clamp_min(SCALE_FLOOR)
    pamax = torch.quantile(flat, percentile / 100.0, dim=0).clamp_min(SCALE_FLOOR)
    return amax, pamax


class PerChannelCollector:
    """Running elementwise max over samples (calibrate_smolvla_activation_channel_scales.py:86-134)."""

    def __init__(self, percentile: float = 99.99):
        self.percentile = percentile
        self.calls: dict[str, dict[str, Any]] = {}

    def observe(self, module: str, x: torch.Tensor) -> None:
        amax, pamax = per_channel_percentile_amax(x, self.percentile)
        call = self.calls.get(module)
        if call is None:
            self.calls[module] = {"module": module, "shape": list(x.shape), "amax": amax,
                                  "percentile_amax": pamax, "num_samples": 1}
        else:
            call["amax"] = torch.maximum(call["amax"], amax)
            call["percentile_amax"] = torch.maximum(call["percentile_amax"], pamax)
            call["num_samples"] += 1

    def rows(self) -> list[dict[str, Any]]:
        out = []
        for idx, call in enumerate(self.calls.values()):
            p = call["percentile_amax"].to(torch.float32)
            a = call["amax"].to(torch.float32)
            out.append({
                "index": idx,
                "module": call["module"],
                "shape": call["shape"],
                "channels": int(p.numel()),
                "amax_max": float(a.max()),
                "percentile_amax_max": float(p.max()),
                "num_samples": call["num_samples"],
                "scale": (p / 127.0).clamp_min(SCALE_FLOOR).tolist(),
                "scale_source": f"per_channel_p{self.percentile}",
                "amax_scale": (a / 127.0).clamp_min(SCALE_FLOOR).tolist(),
            })
        return out


def activation_amax_from_entry(entry: dict[str, Any]) -> torch.Tensor:
    """deploy/build_smoothquant_scales.py:55-61."""
    if "percentile_amax" in entry and isinstance(entry["percentile_amax"], list):
        return torch.as_tensor(entry["percentile_amax"], dtype=torch.float32).clamp_min(SCALE_FLOOR)
    scale = entry.get("scale")
    if not isinstance(scale, list):
        raise ValueError(f"SmoothQuant requires per-channel activation scale list for {entry.get('module')}")
    return (torch.as_tensor(scale, dtype=torch.float32) * 127.0).clamp_min(SCALE_FLOOR)


def build_smoothquant_entry(source_entry: dict[str, Any], weight: torch.Tensor, alpha: float,
                            smooth_scale_min: float = 1.0e-4, smooth_scale_max: float = 1.0e4) -> dict[str, Any]:
    """deploy/build_smoothquant_scales.py:64-106:
    s = clamp(amax_x^alpha / amax_w^(1-alpha), min, max);  a = max(amax_x / s) / 127."""
    act_amax = activation_amax_from_entry(source_entry)
    w = weight.detach().to(torch.float32)
    weight_amax = w.abs().amax(dim=0).clamp_min(SCALE_FLOOR)
    if act_amax.numel() != weight_amax.numel():
        raise ValueError(f"activation channels {act_amax.numel()} do not match weight input channels "
                         f"{weight_amax.numel()} for {source_entry.get('module')}")
    smooth = (act_amax.pow(alpha) / weight_amax.pow(1.0 - alpha)).clamp(min=smooth_scale_min, max=smooth_scale_max)
    smoothed = (act_amax / smooth).clamp_min(SCALE_FLOOR)
    scale = float((smoothed.max() / 127.0).item())
    return {
        "index": source_entry.get("index"),
        "module": source_entry["module"],
        "shape": source_entry.get("shape"),
        "channels": int(act_amax.numel()),
        "num_samples": source_entry.get("num_samples"),
        "scale": max(scale, SCALE_FLOOR),
        "scale_source": f"smoothquant_alpha_{alpha:g}_from_{source_entry.get('scale_source', 'per_channel')}",
        "quantization": "smoothquant_symmetric_static_per_tensor",
        "smoothquant_alpha": alpha,
        "smooth_scale": smooth.tolist(),
    }


def load_activation_scales_by_module(scales_json: str | Path | dict,
                                     include_regexes: tuple[str, ...] | None = None) -> dict[str, Any]:
    """deploy/linear_only_quant.py:175-246 (symmetric and SmoothQuant entries)."""
    if isinstance(scales_json, dict):
        calibration = scales_json
    else:
        with open(scales_json) as f:
            calibration = json.load(f)
    patterns = tuple(re.compile(p) for p in (include_regexes or ()))
    scales: dict[str, Any] = {}

    def append(name: str, value: Any) -> None:
        existing = scales.get(name)
        if existing is None:
            scales[name] = value
        elif isinstance(existing, list) and existing and isinstance(existing[0], dict):
            existing.append(value)
        else:
            scales[name] = [existing, value]

    for entry in calibration.get("linear_call_scales", []):
        name = str(entry.get("module", ""))
        if patterns and not any(p.search(name) for p in patterns):
            continue
        if not name:
            continue
        quantization = str(entry.get("quantization", ""))
        scale = entry.get("scale", SCALE_FLOOR)
        if quantization in {"smoothquant_symmetric_static_per_tensor", "smoothquant_asymmetric_static_per_tensor"}:
            smooth = entry.get("smooth_scale")
            if not isinstance(smooth, list):
                raise ValueError(f"missing smooth_scale list for SmoothQuant module: {name}")
            value = {"quantization": quantization, "scale": max(float(scale), SCALE_FLOOR),
                     "smooth_scale": [max(float(v), SCALE_FLOOR) for v in smooth],
                     "smoothquant_alpha": entry.get("smoothquant_alpha")}
            if quantization == "smoothquant_asymmetric_static_per_tensor":
                value["zero_point"] = int(entry.get("zero_point", 0))
            append(name, value)
        elif quantization == "asymmetric_static_per_tensor":
            append(name, {"quantization": quantization, "scale": max(float(scale), SCALE_FLOOR),
                          "zero_point": int(entry.get("zero_point", 0))})
        elif isinstance(scale, list):
            append(name, [max(float(v), SCALE_FLOOR) for v in scale])
        else:
            append(name, max(float(scale), SCALE_FLOOR))
    return scales


def select_activation_scale_for_linear(value: Any, in_features: int) -> Any:
    """deploy/linear_only_quant.py:185-205: duplicates resolved by in_features."""
    def channels(v: Any) -> int | None:
        if isinstance(v, dict):
            if isinstance(v.get("smooth_scale"), list):
                return len(v["smooth_scale"])
            if isinstance(v.get("scale"), list):
                return len(v["scale"])
            return None
        if isinstance(v, list):
            return len(v)
        return None

    if isinstance(value, list) and value and isinstance(value[0], dict):
        for cand in value:
            if channels(cand) == in_features:
                return cand
        return value[0]
    return value
