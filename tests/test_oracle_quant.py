"""The oracle's SmoothQuant arithmetic against golden vectors made by the reference's own code
(tests/golden/make_golden.py imports deploy/linear_only_quant.py, build_smoothquant_scales.py and
calibrate_smolvla_activation_channel_scales.py unchanged)."""

import hashlib

import numpy as np
import torch

from oracle import quant as Q
from smolvla_mujoco_libero_b200 import synthetic


def _digest(t):
    t = t.detach().contiguous().cpu()
    if t.dtype == torch.bfloat16:
        return hashlib.sha256(t.view(torch.int16).numpy().tobytes()).hexdigest()
    return hashlib.sha256(t.numpy().tobytes()).hexdigest()


def _bf16(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16)


def test_inputs_are_reproducible(golden):
    g = golden["linear_full"]
    case = synthetic.smoothquant_linear_case()
    assert case.outliers.tolist() == g["outliers"]
    assert _digest(case.x) == g["sha256"]["x"]
    assert _digest(case.weight) == g["sha256"]["weight"]


def test_calibration_and_smoothquant_scales_match_reference(golden):
    g = golden["linear_full"]
    case = synthetic.smoothquant_linear_case()
    col = Q.PerChannelCollector(99.99)
    for xb in case.calib:
        col.observe("proj", xb)
    row = col.rows()[0]
    assert row["scale"] == g["calib_percentile_amax_scale"]
    entry = Q.build_smoothquant_entry(row, case.weight, 0.85)
    assert entry["scale"] == g["act_scale"]
    assert entry["smooth_scale"] == g["smooth_scale"]


def test_full_linear_bit_exact_against_reference(golden):
    g = golden["linear_full"]
    case = synthetic.smoothquant_linear_case()
    smooth = torch.tensor(g["smooth_scale"], dtype=torch.float32)
    lin = Q.W8A8Linear(case.weight, None, g["act_scale"], smooth)
    assert _digest(lin.qweight) == g["sha256"]["qweight"]
    assert _digest(lin.weight_scale) == g["sha256"]["weight_scale"]
    assert _digest(lin.weight) == g["sha256"]["weight_deq_bf16"]
    qx = lin.quantize_input(case.x)
    x_deq = qx.to(torch.float32) * torch.tensor(g["act_scale"], dtype=torch.float32)
    assert _digest(x_deq) == g["sha256"]["x_deq_fp32"]
    assert _digest(lin(case.x)) == g["sha256"]["y_bf16"]


def test_small_linear_with_bias_against_reference(golden_dir):
    d = np.load(golden_dir / "linear_small.npz")
    x, w, b = _bf16(d["x_bf16"]), _bf16(d["weight_bf16"]), _bf16(d["bias_bf16"])
    a = float(d["act_scale"][0])
    lin = Q.W8A8Linear(w, b, a, torch.from_numpy(d["smooth_scale"]))
    assert torch.equal(lin.qweight, torch.from_numpy(d["qweight"]))
    assert torch.equal(lin.weight_scale, torch.from_numpy(d["weight_scale"]))
    qx = lin.quantize_input(x)
    assert torch.equal(qx.float() * torch.tensor(a, dtype=torch.float32), torch.from_numpy(d["x_deq"]))
    assert torch.equal(lin(x).view(torch.int16), torch.from_numpy(d["y_bf16"]))
    # integer identity: y_int = (acc*a)*w_s + b is the fp32 form the CUDA epilogue computes
    acc = Q.int_gemm(qx, lin.qweight)
    y_int = Q.w8a8_int_dequant(acc, a, lin.weight_scale, b)
    ref = lin(x).float()
    cos = torch.nn.functional.cosine_similarity(y_int.flatten(), ref.flatten(), dim=0)
    assert cos > 0.9999


def test_w8a16_against_reference(golden_dir):
    d = np.load(golden_dir / "w8a16_small.npz")
    x, w, b = _bf16(d["x_bf16"]), _bf16(d["weight_bf16"]), _bf16(d["bias_bf16"])
    lin = Q.W8A16Linear(w, b)
    assert torch.equal(lin.weight.view(torch.int16), torch.from_numpy(d["weight_deq_bf16"]))
    assert torch.equal(lin(x).view(torch.int16), torch.from_numpy(d["y_bf16"]))


def test_scale_json_roundtrip_and_duplicate_resolution():
    entries = {"linear_call_scales": [
        {"module": "m.a", "quantization": "smoothquant_symmetric_static_per_tensor", "scale": 0.5,
         "smooth_scale": [1.0, 2.0, 0.0]},
        {"module": "m.a", "quantization": "smoothquant_symmetric_static_per_tensor", "scale": 0.25,
         "smooth_scale": [1.0, 2.0]},
        {"module": "m.b", "scale": 0.0},
    ]}
    s = Q.load_activation_scales_by_module(entries)
    assert isinstance(s["m.a"], list) and len(s["m.a"]) == 2
    assert s["m.a"][0]["smooth_scale"][2] == 1e-8
    assert Q.select_activation_scale_for_linear(s["m.a"], 2)["scale"] == 0.25
    assert Q.select_activation_scale_for_linear(s["m.a"], 7)["scale"] == 0.5
    assert s["m.b"] == 1e-8
