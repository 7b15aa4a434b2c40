"""The native whole-path engine (svla_engine_*): packed-file parsing and validation on the CPU, and on the GPU
bit-identical actions to the Python runner over the same kernels (device and host inputs, graph replay,
padding of short language / state rows, batch sizes below the engine's maximum)."""

import ctypes
import json

import pytest
import torch

from smolvla_mujoco_libero_b200 import _lib
from smolvla_mujoco_libero_b200.config import TINY
from smolvla_mujoco_libero_b200.engine import inspect
from smolvla_mujoco_libero_b200.weights import linear_specs, other_specs


def _fake_packed(cfg, path, seed=0, drop=None, retype=None):
    """A packed-weights file of the right names, dtypes and shapes made on the CPU (random contents), through
    the package's own writer."""
    from smolvla_mujoco_libero_b200.checkpoint import save_packed
    from smolvla_mujoco_libero_b200.model import DeviceWeights, PackedLinear
    g = torch.Generator().manual_seed(seed)
    bf = lambda *s: torch.randn(*s, generator=g).to(torch.bfloat16)  # noqa: E731
    i8 = lambda *s: torch.randint(-127, 128, s, generator=g, dtype=torch.int8)  # noqa: E731
    f32 = lambda *s: torch.rand(*s, generator=g) + 0.5  # noqa: E731
    w = DeviceWeights.__new__(DeviceWeights)
    w.cfg, w.lin, w.t = cfg, {}, {}
    for name, n, k, has_bias, kind in linear_specs(cfg):
        b = bf(n) if has_bias else None
        if kind == "w8a8":
            sm = f32(k)
            w.lin[name] = PackedLinear(n, k, kind, i8(n, k), f32(n), b, sm, 1.0 / sm, 0.01)
        elif kind == "w8a16":
            w.lin[name] = PackedLinear(n, k, kind, i8(n, k), f32(n), b, weight_deq=bf(n, k))
        else:
            w.lin[name] = PackedLinear(n, k, kind, bf(n, k), None, b)
    for name, shape, _ in other_specs(cfg):
        w.t[name] = bf(*shape)
    w.t["patch_w2d"] = w.t[f"{'model.vlm_with_expert.vlm.model.vision_model'}.embeddings.patch_embedding.weight"] \
        .reshape(cfg.vis_hidden, -1).contiguous()
    if drop:
        w.t.pop(drop, None)
    if retype:
        p = w.lin[retype]
        p.weight = p.weight.to(torch.bfloat16)
    save_packed(w, path)
    return w


def test_inspect_reads_the_config_and_counts(tmp_path):
    p = tmp_path / "tiny.safetensors"
    w = _fake_packed(TINY, p)
    info = inspect(p)
    c = TINY
    assert (info["n_cams"], info["channels"], info["image_size"], info["n_lang"]) == (2, 3, c.image_size, c.n_lang)
    assert info["prefix_len"] == c.prefix_len and info["chunk"] == c.chunk and info["num_steps"] == c.num_steps
    assert (info["vis_layers"], info["text_layers"], info["expert_layers"]) == (c.vis_layers, c.text_layers,
                                                                                c.expert_layers)
    assert info["n_linears"] == len(linear_specs(c))
    n_tensors = sum(1 for p_ in w.lin.values() for f in ("weight", "wscale", "bias", "smooth", "rsmooth",
                                                          "weight_deq") if getattr(p_, f) is not None)
    assert info["n_tensors"] == n_tensors + len(w.t) + 1  # + the time embedding
    assert info["weight_bytes"] >= sum(t.numel() * t.element_size() for t in w.t.values())
    assert info["max_batch"] == 0 and info["launches_per_call"] == 0


def _rc_and_message(path):
    info = _lib.EngineInfo()
    rc = _lib.lib().svla_engine_inspect(str(path).encode(), ctypes.byref(info))
    return rc, _lib.lib().svla_last_error().decode()


def test_inspect_rejects_missing_and_mistyped_tensors(tmp_path):
    ln = "model.vlm_with_expert.lm_expert.layers.1.post_attention_layernorm.weight"
    _fake_packed(TINY, tmp_path / "a.safetensors", drop=ln)
    rc, msg = _rc_and_message(tmp_path / "a.safetensors")
    assert rc == 1 and ln in msg
    q = "model.vlm_with_expert.vlm.model.text_model.layers.0.self_attn.q_proj"
    _fake_packed(TINY, tmp_path / "b.safetensors", retype=q)
    rc, msg = _rc_and_message(tmp_path / "b.safetensors")
    assert rc == 1 and q in msg and "BF16" in msg


def test_inspect_rejects_files_that_are_not_packed_weights(tmp_path):
    from safetensors.torch import save_file
    rc, msg = _rc_and_message(tmp_path / "missing.safetensors")
    assert rc == 1 and "cannot open" in msg
    (tmp_path / "short").write_bytes(b"\x05\x00")
    assert _rc_and_message(tmp_path / "short")[0] == 1
    (tmp_path / "len").write_bytes((10 ** 12).to_bytes(8, "little") + b"{}")
    rc, msg = _rc_and_message(tmp_path / "len")
    assert rc == 1 and "header length" in msg
    bad_json = b'{"__metadata__": {"svla_packed": "1"'
    (tmp_path / "json").write_bytes(len(bad_json).to_bytes(8, "little") + bad_json)
    rc, msg = _rc_and_message(tmp_path / "json")
    assert rc == 1 and "header" in msg
    save_file({"x": torch.zeros(4)}, str(tmp_path / "plain.safetensors"))
    rc, msg = _rc_and_message(tmp_path / "plain.safetensors")
    assert rc == 1 and "packed" in msg
    save_file({"x": torch.zeros(4)}, str(tmp_path / "cfg.safetensors"),
              metadata={"svla_packed": "1", "config": json.dumps({"image_size": 128}), "linears": "{}"})
    rc, msg = _rc_and_message(tmp_path / "cfg.safetensors")
    assert rc == 1 and "config field" in msg


def test_inspect_checks_data_offsets_against_the_file(tmp_path):
    p = tmp_path / "t.safetensors"
    _fake_packed(TINY, p)
    data = p.read_bytes()
    (tmp_path / "cut.safetensors").write_bytes(data[: len(data) - 1000])
    rc, msg = _rc_and_message(tmp_path / "cut.safetensors")
    assert rc == 1 and "offsets" in msg


def test_engine_create_rejects_bad_arguments_before_touching_the_gpu(tmp_path):
    h = ctypes.c_void_p()
    lib = _lib.lib()
    assert lib.svla_engine_create(b"/nonexistent", 0, 0, None, ctypes.byref(h)) == 1
    assert lib.svla_engine_create(b"/nonexistent", 1, 0x100, None, ctypes.byref(h)) == 1
    assert "flags" in lib.svla_last_error().decode()
    assert lib.svla_engine_create(b"/nonexistent", 1, 0, None, ctypes.byref(h)) == 1
    assert h.value is None
    assert lib.svla_engine_destroy(None) == 0


# ----------------------------------------------------------------------------------------------- GPU

@pytest.fixture(scope="module")
def packed(tmp_path_factory):
    from oracle.model import calibrate as oracle_calibrate
    from smolvla_mujoco_libero_b200 import synthetic
    from smolvla_mujoco_libero_b200.calibrate import load_scale_json
    from smolvla_mujoco_libero_b200.checkpoint import save_packed
    from smolvla_mujoco_libero_b200.model import DeviceWeights
    from smolvla_mujoco_libero_b200.weights import random_weights
    w = random_weights(TINY, 0)
    js = oracle_calibrate(TINY, w, [synthetic.observations(1, seed=100, image_size=TINY.image_size,
                                                           n_tokens=TINY.n_lang)])
    path = tmp_path_factory.mktemp("engine") / "tiny_packed.safetensors"
    save_packed(DeviceWeights(TINY, w, load_scale_json(js)), path)
    return path


def _obs(b, seed, n_tokens=TINY.n_lang):
    from smolvla_mujoco_libero_b200 import synthetic
    return synthetic.observations(b, seed=seed, image_size=TINY.image_size, n_tokens=n_tokens)


def _args(o, device="cuda"):
    return ([im.to(device) for im in o.images], [m.to(device) for m in o.img_masks], o.lang_tokens.to(device),
            o.lang_masks.to(device), o.state.to(device), o.noise.to(device))


def _runner_actions(path, args, split_k=True):
    from smolvla_mujoco_libero_b200.checkpoint import load_packed
    from smolvla_mujoco_libero_b200.model import SmolVLARunner
    r = SmolVLARunner(load_packed(path), args[4].shape[0], split_k=split_k)
    return r(*args).clone()


@pytest.mark.gpu
@pytest.mark.parametrize("batch", [1, 3])
def test_engine_matches_runner_bitwise(packed, batch):
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    eng = NativeSampleActions(packed, max_batch=3)
    assert eng.launches_per_call > 0
    args = _args(_obs(batch, 11))
    want = _runner_actions(packed, args)
    first = eng.sample_actions(*args)   # eager run, then recorded as a graph
    second = eng.sample_actions(*args)  # graph replay
    assert torch.equal(first, want)
    assert torch.equal(second, want)
    assert _lib.device_error() == 0
    eng.close()


@pytest.mark.gpu
def test_engine_host_inputs_and_output(packed):
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    eng = NativeSampleActions(packed, max_batch=2)
    o = _obs(2, 12)
    want = eng.sample_actions(*_args(o)).cpu()
    host = _args(o, "cpu")
    out = torch.empty(want.shape, dtype=torch.float32).pin_memory()
    eng.sample_actions(*host, out=out)
    torch.cuda.synchronize()
    assert torch.equal(out, want)
    pinned = [x.pin_memory() for x in host[0]], [m.pin_memory() for m in host[1]], *[t.pin_memory() for t in host[2:]]
    out2 = torch.empty_like(out)
    eng.sample_actions(*pinned, out=out2)
    torch.cuda.synchronize()
    assert torch.equal(out2, want)


@pytest.mark.gpu
def test_engine_pads_short_language_and_state_like_the_runner(packed):
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    eng = NativeSampleActions(packed, max_batch=2)
    o = _obs(2, 13, n_tokens=TINY.n_lang - 5)
    args = list(_args(o))
    args[4] = args[4][:, :8].contiguous()  # state narrower than max_state_dim
    want = _runner_actions(packed, tuple(args))
    got = eng.sample_actions(*args)
    assert torch.equal(got, want)


@pytest.mark.gpu
def test_engine_without_split_k_is_batch_independent(packed):
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    eng = NativeSampleActions(packed, max_batch=3, split_k=False, use_cuda_graph=False, flow=False)
    args = _args(_obs(3, 14))
    full = eng.sample_actions(*args).clone()
    one = eng.sample_actions(*[[x[1:2] for x in a] if isinstance(a, list) else a[1:2] for a in args])
    assert torch.equal(one[0], full[1])
    assert torch.equal(full, _runner_actions(packed, args, split_k=False))
    # the persistent flow kernel (batch 1 by default) differs only in fp32 summation order
    flow_one = NativeSampleActions(packed, max_batch=1, split_k=False).sample_actions(
        *[[x[1:2] for x in a] if isinstance(a, list) else a[1:2] for a in args])
    cos = float(torch.nn.functional.cosine_similarity(flow_one.flatten(), full[1].flatten(), dim=0))
    assert cos >= 0.9999 and float((flow_one[0] - full[1]).abs().max()) <= 2e-2


@pytest.mark.gpu
def test_engine_rejects_batches_above_its_maximum(packed):
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    eng = NativeSampleActions(packed, max_batch=1)
    with pytest.raises(_lib.SvlaError, match="batch 2 outside"):
        eng.sample_actions(*_args(_obs(2, 15)))
    info = eng.info
    assert info["max_batch"] == 1 and info["buffer_bytes"] > 0 and info["weight_bytes"] > 0
