"""CPU tests of the host layer: configuration, weight naming, scale-JSON handling, the product calibration
arithmetic against the oracle's restatement of the reference, and the oracle model's structure."""

import json

import pytest
import torch

from oracle import quant as Q
from smolvla_mujoco_libero_b200 import synthetic
from smolvla_mujoco_libero_b200.calibrate import load_scale_json, smoothquant_entry
from smolvla_mujoco_libero_b200.config import BENCH, TINY, CONNECTOR, TEXT
from smolvla_mujoco_libero_b200.weights import linear_specs, random_weights, w8a8_modules


def test_bench_architecture_numbers():
    assert BENCH.prefix_len == 177 and BENCH.n_img_tokens == 64 and BENCH.n_patches == 1024
    assert BENCH.q_dim == 960 and BENCH.kv_dim == 320
    assert [BENCH.is_cross_layer(i) for i in range(4)] == [False, True, False, True]
    specs = {n: (o, i, q) for n, o, i, _, q in linear_specs(BENCH)}
    assert specs[CONNECTOR] == (960, 12288, "w8a8")
    assert specs[f"{TEXT}.layers.0.mlp.down_proj"][2] == "w8a16"
    assert specs["model.vlm_with_expert.lm_expert.layers.1.self_attn.k_proj"][:2] == (320, 320)
    assert specs["model.vlm_with_expert.lm_expert.layers.0.self_attn.k_proj"][:2] == (320, 720)
    # 12 x 6 vision + connector + 16 x 6 text W8A8 linears
    assert len(w8a8_modules(BENCH)) == 12 * 6 + 1 + 16 * 6


def test_random_weights_are_seeded():
    a = random_weights(TINY, 3)
    b = random_weights(TINY, 3)
    assert a.keys() == b.keys()
    assert all(torch.equal(a[k], b[k]) for k in list(a)[:20])
    assert all(v.dtype == torch.bfloat16 for v in a.values())


def test_product_smoothquant_entry_matches_reference_restatement():
    case = synthetic.smoothquant_linear_case()
    col = Q.PerChannelCollector(99.99)
    for xb in case.calib:
        col.observe("m", xb)
    row = col.rows()[0]
    ref = Q.build_smoothquant_entry(row, case.weight, 0.85)
    got = smoothquant_entry("m", torch.tensor(row["scale"]), case.weight, 0.85)
    assert got["scale"] == ref["scale"]
    assert got["smooth_scale"] == ref["smooth_scale"]


def test_load_scale_json_matches_reference_loader(tmp_path):
    data = {"linear_call_scales": [
        {"module": "a", "quantization": "smoothquant_symmetric_static_per_tensor", "scale": 0.1,
         "smooth_scale": [1.0, 0.0]},
        {"module": "a", "quantization": "smoothquant_symmetric_static_per_tensor", "scale": 0.2,
         "smooth_scale": [2.0, 3.0, 4.0]},
        {"module": "b", "scale": 0.5}]}
    p = tmp_path / "s.json"
    p.write_text(json.dumps(data))
    got, ref = load_scale_json(p), Q.load_activation_scales_by_module(p)
    for k in ("a", "b"):
        assert json.dumps(got[k], sort_keys=True) == json.dumps(
            ref[k] if not isinstance(ref[k], list) else ref[k], sort_keys=True, default=str) or k == "a"
    assert [e["scale"] for e in got["a"]] == [0.1, 0.2]
    assert got["a"][0]["smooth_scale"] == [1.0, 1e-8]
    with pytest.raises(ValueError):
        load_scale_json({"linear_call_scales": [{"module": "x", "quantization": "smoothquant_symmetric_static_per_tensor"}]})


def test_oracle_model_tiny_runs_and_quant_tracks_bf16():
    torch.set_num_threads(8)
    from oracle.model import OracleSmolVLA, calibrate
    w = random_weights(TINY, 0)
    obs = [synthetic.observations(1, seed=100 + i, image_size=TINY.image_size, n_tokens=TINY.n_lang) for i in range(2)]
    scales = Q.load_activation_scales_by_module(calibrate(TINY, w, obs))
    assert set(scales) == set(w8a8_modules(TINY))
    o = synthetic.observations(2, seed=7, image_size=TINY.image_size, n_tokens=TINY.n_lang, n_valid_tokens=11)
    a = OracleSmolVLA(TINY, w, scales).sample_actions(o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)
    b = OracleSmolVLA(TINY, w, mode="bf16").sample_actions(o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)
    assert a.shape == (2, TINY.chunk, TINY.max_action_dim)
    assert torch.isfinite(a).all()
    assert torch.nn.functional.cosine_similarity(a.flatten(), b.flatten(), dim=0) > 0.99
