"""The persistent flow-matching kernel (svla_flow) against the per-layer launch list it replaces.

The two compute the same arithmetic with the same rounding points; only fp32 summation order inside dot
products differs, so results agree to within bf16 rounding noise carried through the steps."""

import pytest
import torch
import torch.nn.functional as F

from smolvla_mujoco_libero_b200 import _lib
from smolvla_mujoco_libero_b200.config import TINY

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def tiny():
    from oracle.model import calibrate as oracle_calibrate
    from smolvla_mujoco_libero_b200 import synthetic
    from smolvla_mujoco_libero_b200.calibrate import load_scale_json
    from smolvla_mujoco_libero_b200.model import DeviceWeights
    from smolvla_mujoco_libero_b200.weights import random_weights
    w = random_weights(TINY, 0)
    js = oracle_calibrate(TINY, w, [synthetic.observations(1, seed=100, image_size=TINY.image_size,
                                                           n_tokens=TINY.n_lang)])
    return w, js, load_scale_json(js)


def _args(cfg, b, seed):
    from smolvla_mujoco_libero_b200 import synthetic
    o = synthetic.observations(b, seed=seed, image_size=cfg.image_size, n_tokens=cfg.n_lang)
    return o, ([im.cuda() for im in o.images], [m.cuda() for m in o.img_masks], o.lang_tokens.cuda(),
               o.lang_masks.cuda(), o.state.cuda(), o.noise.cuda())


def _run(weights, cfg_batch, args, flow):
    from smolvla_mujoco_libero_b200.model import SmolVLARunner
    r = SmolVLARunner(weights, cfg_batch, flow=flow)
    assert r.flow == flow
    out = r(*args).clone()
    torch.cuda.synchronize()
    return r, out


def _close(got, want, cos_min, max_abs):
    cos = float(F.cosine_similarity(got.flatten().double(), want.flatten().double(), dim=0))
    mx = float((got - want).abs().max())
    assert cos >= cos_min and mx <= max_abs, (cos, mx)
    return cos, mx


@pytest.mark.parametrize("steps", [1, 3])
def test_flow_kernel_matches_launch_list(tiny, steps):
    from smolvla_mujoco_libero_b200.model import DeviceWeights
    w, _js, scales = tiny
    cfg = TINY.with_(num_steps=steps)
    dw = DeviceWeights(cfg, w, scales)
    _o, args = _args(cfg, 1, 21)
    r_ref, want = _run(dw, 1, args, flow=False)
    r_flow, got = _run(dw, 1, args, flow=True)
    assert _lib.device_error() == 0
    # the flow loop (Euler init + per step: 3 + 7 per layer + 2 launches) becomes one launch
    assert r_flow.n_launches == r_ref.n_launches - steps * (5 + 7 * TINY.expert_layers)
    assert torch.isfinite(got).all()
    # the last expert hidden state and the actions
    _close(r_flow.eh.float(), r_ref.eh.float(), 0.9999, 0.1)
    _close(got, want, 0.9999, 2e-2)


def test_flow_kernel_meets_the_oracle_bar(tiny):
    from oracle import quant as Q
    from oracle.model import OracleSmolVLA
    from smolvla_mujoco_libero_b200.model import DeviceWeights
    w, js, scales = tiny
    o, args = _args(TINY, 1, 22)
    _r, got = _run(DeviceWeights(TINY, w, scales), 1, args, flow=True)
    ref = OracleSmolVLA(TINY, w, Q.load_activation_scales_by_module(js)).sample_actions(
        o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)
    _close(got.cpu()[:, :, :TINY.action_dim], ref[:, :, :TINY.action_dim], 0.999, 2e-2)


def test_flow_kernel_graph_replay_is_deterministic(tiny):
    from smolvla_mujoco_libero_b200.model import DeviceWeights, SmolVLARunner
    w, _js, scales = tiny
    dw = DeviceWeights(TINY, w, scales)
    _o, args = _args(TINY, 1, 23)
    r = SmolVLARunner(dw, 1)
    assert r.flow
    first = r(*args).clone()
    r.capture()
    for _ in range(3):
        r.run()
    torch.cuda.synchronize()
    assert torch.equal(r.actions(), first)
    assert _lib.device_error() == 0


def test_engine_uses_the_flow_kernel_at_batch_one(tiny, tmp_path):
    from smolvla_mujoco_libero_b200.checkpoint import save_packed
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    from smolvla_mujoco_libero_b200.model import DeviceWeights
    w, _js, scales = tiny
    dw = DeviceWeights(TINY, w, scales)
    path = tmp_path / "tiny.safetensors"
    save_packed(dw, path)
    _o, args = _args(TINY, 1, 24)
    eng = NativeSampleActions(path, max_batch=1)
    eng_off = NativeSampleActions(path, max_batch=1, flow=False)
    assert eng.launches_per_call == eng_off.launches_per_call - TINY.num_steps * (5 + 7 * TINY.expert_layers)
    got = eng.sample_actions(*args).clone()
    again = eng.sample_actions(*args)  # graph replay
    _r, want = _run(dw, 1, args, flow=True)
    assert torch.equal(got, want) and torch.equal(again, want)
    _close(got, eng_off.sample_actions(*args), 0.9999, 2e-2)
    assert _lib.device_error() == 0


def test_flow_grid_barrier_that_runs_out_reports_an_error_and_the_context_survives(tiny):
    """Every wait in the flow kernel is bounded.  With a poll limit of 1 the first CTA to reach a grid barrier
    gives up before the others arrive: it records device error 103 (kErrFlowBarrier), every CTA returns at
    its next barrier, and the launch ends.  The host reads the error, clears it and the arrival counter, and
    the next call on the same context gives the same actions as before."""
    import ctypes

    from smolvla_mujoco_libero_b200.model import DeviceWeights
    w, _js, scales = tiny
    dw = DeviceWeights(TINY, w, scales)
    _o, args = _args(TINY, 1, 25)
    r, want = _run(dw, 1, args, flow=True)
    assert _lib.device_error() == 0
    d = next(a[0] for fn, a in r.launches if fn is _lib.lib().svla_flow)
    d.spin_limit = 1
    stream = torch.cuda.current_stream().cuda_stream
    _lib.check(_lib.lib().svla_flow(ctypes.byref(d), stream), "svla_flow")
    torch.cuda.synchronize()
    assert _lib.device_error(reset=True) == _lib.ERR_FLOW_BARRIER
    assert _lib.device_error() == 0
    d.spin_limit = 0
    r.flow_sync.zero_()
    got = r(*args).clone()
    torch.cuda.synchronize()
    assert _lib.device_error() == 0
    assert torch.equal(got, want)
