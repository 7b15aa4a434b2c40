"""End-to-end parity of the sm_100a sample_actions path with the CPU oracle.

Bar: on the same seeded inputs, weights and scale JSON, the final chunk matches the
oracle's SmoothQuant fake-dequant restatement with cosine >= 0.999 and max-abs <= 2e-2.  Batch rows are
independent: a row's result is bit-identical whether it runs alone or in a batch.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import quant as Q
from oracle.model import OracleSmolVLA, calibrate as oracle_calibrate
from smolvla_mujoco_libero_b200 import _lib as L
from smolvla_mujoco_libero_b200 import synthetic
from smolvla_mujoco_libero_b200.calibrate import calibrate as gpu_calibrate, load_scale_json
from smolvla_mujoco_libero_b200.config import BENCH, TINY
from smolvla_mujoco_libero_b200.model import DeviceWeights
from smolvla_mujoco_libero_b200.policy import SampleActions
from smolvla_mujoco_libero_b200.weights import random_weights

pytestmark = pytest.mark.gpu


def _obs(cfg, b, seed, **kw):
    return synthetic.observations(b, seed=seed, image_size=cfg.image_size, n_tokens=cfg.n_lang, **kw)


def _close(got, ref, cos=0.999, max_abs=2e-2):
    got, ref = got.float().cpu(), ref.float().cpu()
    c = float(F.cosine_similarity(got.flatten(), ref.flatten(), dim=0))
    m = float((got - ref).abs().max())
    assert c >= cos and m <= max_abs, (c, m)
    return c, m


def _run(sa, o):
    dev = "cuda"
    return sa([im.to(dev) for im in o.images], [m.to(dev) for m in o.img_masks], o.lang_tokens.to(dev),
              o.lang_masks.to(dev), o.state.to(dev), o.noise.to(dev))


@pytest.fixture(scope="module")
def tiny():
    torch.set_num_threads(8)
    w = random_weights(TINY, 0)
    cal = [_obs(TINY, 1, 100 + i) for i in range(2)]
    js = oracle_calibrate(TINY, w, cal)
    return w, js


def test_tiny_sample_actions_matches_oracle(tiny):
    w, js = tiny
    scales = load_scale_json(js)
    sa = SampleActions(TINY, DeviceWeights(TINY, w, scales))
    o = _obs(TINY, 2, 7, n_valid_tokens=11)
    got = _run(sa, o)
    ref = OracleSmolVLA(TINY, w, Q.load_activation_scales_by_module(js)).sample_actions(
        o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)[:, :, :TINY.action_dim]
    _close(got, ref)
    torch.cuda.synchronize()
    assert L.device_error() == 0


@pytest.mark.parametrize("split_k", [False, True])
def test_batch_rows_are_independent(tiny, split_k):
    """Without split-K (and on one path: the batch-1 call would otherwise take the persistent flow kernel) each
    batch row is bit-identical at any batch size; with split-K and the flow kernel (the defaults) a single row
    sums its fp32 partials in another order, so rows agree within the tolerance."""
    w, js = tiny
    sa = SampleActions(TINY, DeviceWeights(TINY, w, load_scale_json(js)), split_k=split_k,
                       flow=None if split_k else False)
    o = _obs(TINY, 3, 21)
    full = _run(sa, o)
    for i in range(3):
        one = synthetic.Observation(images=[im[i:i + 1] for im in o.images], img_masks=[m[i:i + 1] for m in o.img_masks],
                                    lang_tokens=o.lang_tokens[i:i + 1], lang_masks=o.lang_masks[i:i + 1],
                                    state=o.state[i:i + 1], noise=o.noise[i:i + 1])
        if split_k:
            _close(_run(sa, one), full[i:i + 1], cos=0.9999, max_abs=2e-2)
        else:
            assert torch.equal(_run(sa, one), full[i:i + 1])


def test_graph_replay_equals_direct_launches(tiny):
    w, js = tiny
    dw = DeviceWeights(TINY, w, load_scale_json(js))
    o = _obs(TINY, 1, 5)
    a = _run(SampleActions(TINY, dw, use_cuda_graph=True), o)
    b = _run(SampleActions(TINY, dw, use_cuda_graph=False), o)
    assert torch.equal(a, b)


def test_gpu_calibration_tracks_oracle_calibration(tiny):
    w, js = tiny
    cal = [_obs(TINY, 1, 100 + i) for i in range(2)]
    gj = gpu_calibrate(TINY, w, cal)
    ref = {e["module"]: e for e in js["linear_call_scales"]}
    assert {e["module"] for e in gj["linear_call_scales"]} == set(ref)
    for e in gj["linear_call_scales"]:
        r = ref[e["module"]]
        assert abs(e["scale"] - r["scale"]) <= 0.02 * r["scale"], e["module"]
        s, rs = torch.tensor(e["smooth_scale"]), torch.tensor(r["smooth_scale"])
        assert float(((s - rs).abs() / rs).max()) < 0.05, e["module"]


def test_gpu_calibration_equals_the_oracle_collector_on_the_same_activations(tiny, monkeypatch):
    """Given the same activations, the GPU calibration equals the reference's collector and SmoothQuant builder
    exactly (deploy/calibrate_smolvla_activation_channel_scales.py:68-134, deploy/build_smoothquant_scales.py:
    64-106 as restated in the oracle): every W8A8 input the GPU collector sees is also fed, one call at a time,
    to the oracle collector, and each module's scale and smooth vector must match bit for bit."""
    from oracle import quant as Q
    from smolvla_mujoco_libero_b200 import calibrate as C
    w, _js = tiny
    seen = []
    observe = C.ChannelStats.observe

    def spy(self, modules, x, rows_per_call):
        seen.append((list(modules), x.detach().reshape(-1, x.shape[-1]).cpu().clone(), rows_per_call))
        return observe(self, modules, x, rows_per_call)

    monkeypatch.setattr(C.ChannelStats, "observe", spy)
    gj = C.calibrate(TINY, w, [_obs(TINY, 1, 100 + i) for i in range(2)])
    col = Q.PerChannelCollector(TINY.percentile)
    for mods, x, per in seen:
        for r0 in range(0, x.shape[0], per):
            for m in mods:
                col.observe(m, x[r0:r0 + per])
    rows = {r["module"]: r for r in col.rows()}
    assert gj["linear_call_scales"]
    for e in gj["linear_call_scales"]:
        ref = Q.build_smoothquant_entry(rows[e["module"]], w[f"{e['module']}.weight"], gj["smoothquant_alpha"])
        assert e["scale"] == ref["scale"], e["module"]
        assert e["smooth_scale"] == ref["smooth_scale"], e["module"]
        assert e["num_samples"] == ref["num_samples"], e["module"]


def test_bench_architecture_batch1_matches_oracle():
    """The full benchmark architecture (SigLIP 12x768, text 16x960, expert 16x720, 10 steps) at batch 1."""
    torch.set_num_threads(8)
    w = random_weights(BENCH, 0)
    cal = [_obs(BENCH, 1, 100 + i) for i in range(2)]
    js = gpu_calibrate(BENCH, w, cal)
    sa = SampleActions(BENCH, DeviceWeights(BENCH, w, load_scale_json(js)))
    o = _obs(BENCH, 1, 1000)
    got = _run(sa, o)
    ref = OracleSmolVLA(BENCH, w, Q.load_activation_scales_by_module(js)).sample_actions(
        o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)[:, :, :BENCH.action_dim]
    _close(got, ref)


def test_prefix_features_match_oracle(tiny):
    """The RL-token features (prefix prefill only): final-layer prefix hidden states and the KV cache against
    the oracle's prefix forward; the padding mask and image-token count as the reference extractor's."""
    from smolvla_mujoco_libero_b200.policy import PrefixFeatures
    w, js = tiny
    pf = PrefixFeatures(TINY, DeviceWeights(TINY, w, load_scale_json(js)))
    o = _obs(TINY, 2, 11, n_valid_tokens=9)
    dev = "cuda"
    feats = pf.extract([im.to(dev) for im in o.images], [m.to(dev) for m in o.img_masks], o.lang_tokens.to(dev),
                       o.lang_masks.to(dev), o.state.to(dev))
    taps = {}
    OracleSmolVLA(TINY, w, Q.load_activation_scales_by_module(js)).sample_actions(
        o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise, taps=taps)
    ref = taps["prefix_out"].float()
    z = feats["z"].cpu()
    assert z.shape == ref.shape
    # relative bar: the prefix hidden states are O(1) after the final RMSNorm
    c = float(F.cosine_similarity(z.flatten(), ref.flatten(), dim=0))
    assert c >= 0.999, c
    assert float((z - ref).abs().max()) <= 2e-2 * float(ref.abs().max()) + 2e-2
    for (k, v), (rk, rv) in zip(feats["kv_cache"], taps["kv"]):
        for got, want in ((k, rk), (v, rv)):
            g, r = got.cpu().float().flatten(), want.float().reshape(got.shape).flatten()
            assert float(F.cosine_similarity(g, r, dim=0)) >= 0.999
    n_img = TINY.n_cams * TINY.n_img_tokens
    assert feats["n_img_tokens"] == n_img
    pad = feats["pad_mask"].cpu()
    assert bool(pad[:, n_img + 9:n_img + TINY.n_lang].sum() == 0) and bool(pad[:, -1].all())
