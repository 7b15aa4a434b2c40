#!/usr/bin/env python3
"""Generate the golden fixtures under tests/golden/ from the reference's OWN code.

Run in a container that has a checkout of the reference (read-only is enough), naming its root
with --reference or the SVLA_REFERENCE environment variable:

    python tests/golden/make_golden.py --reference <reference checkout>

The reference modules are imported unchanged from <reference>/deploy:
  * linear_only_quant.W8A8Linear / W8A16Linear / quantize_weight_per_out_channel
    / quantize_dequantize_activation_static      (deploy/linear_only_quant.py:40-172)
  * build_smoothquant_scales.build_entry           (deploy/build_smoothquant_scales.py:64-106)
  * calibrate_smolvla_activation_channel_scales.PerChannelLinearInputCollector
                                                   (deploy/calibrate_smolvla_activation_channel_scales.py:53-134)
  * validate_fused_rope_layout_math.apply_rope_ref / fused_ref
                                                   (deploy/validate_fused_rope_layout_math.py:28-54)
Their top-level ``lerobot`` imports are satisfied by empty stub modules; none of
the stubbed names is called.  Inputs come from smolvla_mujoco_libero_b200.synthetic
(seeded CPU generators), so the fixtures hold digests of the full-size tensors and
complete tensors only for the small cases.
"""

from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO))

from smolvla_mujoco_libero_b200 import synthetic  # noqa: E402


def install_lerobot_stubs() -> None:
    names = [
        "lerobot", "lerobot.configs", "lerobot.envs", "lerobot.envs.factory", "lerobot.policies",
        "lerobot.policies.factory", "lerobot.scripts", "lerobot.scripts.lerobot_eval", "lerobot.utils",
        "lerobot.utils.constants", "lerobot.utils.random_utils",
    ]
    attrs = {
        "lerobot.configs": ["FeatureType", "PreTrainedConfig"],
        "lerobot.envs": ["close_envs", "make_env", "make_env_pre_post_processors", "preprocess_observation"],
        "lerobot.envs.factory": ["make_env_config"],
        "lerobot.policies": ["make_pre_post_processors"],
        "lerobot.policies.factory": ["get_policy_class", "make_pre_post_processors"],
        "lerobot.scripts.lerobot_eval": ["eval_policy_all"],
        "lerobot.utils.constants": ["ACTION", "OBS_STATE", "OBS_LANGUAGE_ATTENTION_MASK", "OBS_LANGUAGE_TOKENS"],
        "lerobot.utils.random_utils": ["set_seed"],
    }
    for name in names:
        mod = types.ModuleType(name)
        for attr in attrs.get(name, []):
            setattr(mod, attr, object())
        sys.modules[name] = mod


def digest(t: torch.Tensor) -> str:
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        b = t.view(torch.int16).numpy().tobytes()
    else:
        b = t.numpy().tobytes()
    return hashlib.sha256(b).hexdigest()


def run_reference_linear(ref, case: synthetic.LinearCase, alpha: float, percentile: float):
    """Calibrate + build SmoothQuant scales + run W8A8Linear, all with the reference's code."""
    lq, bss, cal = ref["linear_only_quant"], ref["build_smoothquant_scales"], ref["calib"]
    n, k = case.weight.shape
    linear = torch.nn.Linear(k, n, bias=case.bias is not None).to(torch.bfloat16)
    with torch.no_grad():
        linear.weight.copy_(case.weight)
        if case.bias is not None:
            linear.bias.copy_(case.bias)
    collector = cal.PerChannelLinearInputCollector(percentile, r".*")
    holder = torch.nn.Module()
    holder.add_module("proj", linear)
    collector.hook_modules(holder)
    with torch.no_grad():
        for xb in case.calib:
            collector.begin_sample()
            linear(xb)
            collector.end_sample()
    collector.close()
    rows = collector.scales()
    assert len(rows) == 1
    entry = bss.build_entry(rows[0], linear, alpha, 1.0e-4, 1.0e4)
    scales = {"linear_call_scales": [entry]}
    mod = lq.W8A8Linear.from_float(linear, {
        "quantization": entry["quantization"], "scale": entry["scale"], "smooth_scale": entry["smooth_scale"]})
    with torch.no_grad():
        y = mod.forward(case.x)
        smooth = torch.as_tensor(entry["smooth_scale"], dtype=torch.float32).clamp_min(1e-8)
        x_smooth = case.x.to(torch.float32) / smooth
        x_deq = lq.quantize_dequantize_activation_static(x_smooth, torch.tensor(entry["scale"]))
        qweight, wscale = lq.quantize_weight_per_out_channel(case.weight.to(torch.float32) * smooth[None, :])
    return rows[0], entry, scales, mod, y, x_deq, qweight, wscale


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--reference", default=os.environ.get("SVLA_REFERENCE"),
                    help="root of the reference checkout (default: $SVLA_REFERENCE)")
    args = ap.parse_args()
    if not args.reference:
        ap.error("name the reference checkout with --reference or SVLA_REFERENCE")
    deploy = Path(args.reference) / "deploy"
    sys.path.insert(0, str(deploy))
    install_lerobot_stubs()
    import build_smoothquant_scales  # noqa: E402
    import calibrate_smolvla_activation_channel_scales as calib  # noqa: E402
    import linear_only_quant  # noqa: E402
    import validate_fused_rope_layout_math as rope_kat  # noqa: E402
    ref = {"linear_only_quant": linear_only_quant, "build_smoothquant_scales": build_smoothquant_scales,
           "calib": calib}
    torch.set_num_threads(8)
    out: dict = {"generator": "tests/golden/make_golden.py", "torch": torch.__version__}

    # -- 1. single SmoothQuant W8A8 linear, full size: digests -------------------------------
    case = synthetic.smoothquant_linear_case()
    row, entry, _, mod, y, x_deq, qweight, wscale = run_reference_linear(ref, case, 0.85, 99.99)
    out["linear_full"] = {
        "shape": {"m": 177, "k": 960, "n": 2560}, "seed": synthetic.DEFAULT_SEED, "alpha": 0.85,
        "percentile": 99.99, "n_calib": 32,
        "outliers": case.outliers.tolist(),
        "act_scale": entry["scale"],
        "smooth_scale": entry["smooth_scale"],
        "calib_percentile_amax_scale": row["scale"],
        "sha256": {
            "x": digest(case.x), "weight": digest(case.weight),
            "qweight": digest(qweight), "weight_scale": digest(wscale),
            "weight_deq_bf16": digest(mod.weight), "x_deq_fp32": digest(x_deq), "y_bf16": digest(y),
        },
    }

    # -- 2. small SmoothQuant linear with bias: full tensors -------------------------------------
    small = synthetic.smoothquant_linear_case(seed=1234, m=37, k=256, n=96, n_outliers=4, n_calib=8,
                                              with_bias=True)
    row_s, entry_s, _, mod_s, y_s, x_deq_s, qw_s, ws_s = run_reference_linear(ref, small, 0.85, 99.99)
    np.savez_compressed(
        HERE / "linear_small.npz",
        x_bf16=small.x.view(torch.int16).numpy(), weight_bf16=small.weight.view(torch.int16).numpy(),
        bias_bf16=small.bias.view(torch.int16).numpy(),
        smooth_scale=np.asarray(entry_s["smooth_scale"], dtype=np.float32),
        act_scale=np.asarray([entry_s["scale"]], dtype=np.float64),
        qweight=qw_s.numpy(), weight_scale=ws_s.numpy(), x_deq=x_deq_s.numpy(),
        weight_deq_bf16=mod_s.weight.view(torch.int16).numpy(), y_bf16=y_s.view(torch.int16).numpy(),
    )
    out["linear_small"] = {"file": "linear_small.npz", "shape": {"m": 37, "k": 256, "n": 96}, "seed": 1234}

    # -- 3. W8A16 weight path (down_proj / expert linears) -----------------------------------------
    g = synthetic.generator(77)
    w16 = (torch.randn(64, 160, generator=g) * 0.02).to(torch.bfloat16)
    b16 = (torch.randn(64, generator=g) * 0.02).to(torch.bfloat16)
    x16 = torch.randn(19, 160, generator=g).to(torch.bfloat16)
    lin = torch.nn.Linear(160, 64).to(torch.bfloat16)
    with torch.no_grad():
        lin.weight.copy_(w16)
        lin.bias.copy_(b16)
        m16 = linear_only_quant.W8A16Linear.from_float(lin)
        y16 = m16.forward(x16)
    np.savez_compressed(HERE / "w8a16_small.npz", x_bf16=x16.view(torch.int16).numpy(),
                        weight_bf16=w16.view(torch.int16).numpy(), bias_bf16=b16.view(torch.int16).numpy(),
                        weight_deq_bf16=m16.weight.view(torch.int16).numpy(), y_bf16=y16.view(torch.int16).numpy())
    out["w8a16_small"] = {"file": "w8a16_small.npz", "shape": {"m": 19, "k": 160, "n": 64}, "seed": 77}

    # -- 4. RoPE / layout KAT (validate_fused_rope_layout_math.py, seed 1000, L=177) ---------------
    torch.manual_seed(1000)
    q_raw = torch.randn(1, 177, 15 * 64)
    k_raw = torch.randn(1, 177, 5 * 64)
    pos = torch.arange(177, dtype=torch.int64).unsqueeze(0)
    q_rot = rope_kat.apply_rope_ref(q_raw.view(1, 177, 15, 64), pos)
    k_rot = rope_kat.apply_rope_ref(k_raw.view(1, 177, 5, 64), pos)
    q_lay, k_lay = rope_kat.fused_ref(q_raw, k_raw, pos, 15, 5, 64)
    rows = list(range(0, 8)) + list(range(170, 177))
    np.savez_compressed(HERE / "rope_kat.npz", rows=np.asarray(rows), q_rot=q_rot[0, rows].numpy(),
                        k_rot=k_rot[0, rows].numpy())
    out["rope_kat"] = {"file": "rope_kat.npz", "seed": 1000, "seq_len": 177, "max_wavelength": 10000.0,
                       "inputs": "torch.manual_seed(1000); q_raw = randn(1,177,960); k_raw = randn(1,177,320)",
                       "sha256": {"q_layout": digest(q_lay), "k_layout": digest(k_lay)}}
    (HERE / "golden.json").write_text(json.dumps(out, indent=1))
    print("wrote", HERE / "golden.json")


if __name__ == "__main__":
    main()
