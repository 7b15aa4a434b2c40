"""Checkpoint reading and architecture inference (CPU), packed-weights round trip (GPU)."""

import pytest
import torch

from smolvla_mujoco_libero_b200.checkpoint import infer_config, load_checkpoint, required_keys
from smolvla_mujoco_libero_b200.config import BENCH, EXPERT, TINY
from smolvla_mujoco_libero_b200.weights import random_weights


def _save(state, path):
    from safetensors.torch import save_file
    save_file({k: v.contiguous() for k, v in state.items()}, str(path))


@pytest.mark.parametrize("sharded", [False, True])
def test_infer_config_from_checkpoint(tmp_path, sharded):
    state = random_weights(TINY, 3)
    if sharded:
        keys = sorted(state)
        _save({k: state[k] for k in keys[: len(keys) // 2]}, tmp_path / "a.safetensors")
        _save({k: state[k] for k in keys[len(keys) // 2:]}, tmp_path / "b.safetensors")
        loaded = load_checkpoint(tmp_path)
    else:
        _save(state, tmp_path / "m.safetensors")
        loaded = load_checkpoint(tmp_path / "m.safetensors")
    assert set(loaded) == set(state)
    assert all(torch.equal(loaded[k], state[k]) for k in state)
    cfg = infer_config(loaded, base=TINY.with_(image_size=512, vis_layers=12, text_layers=16, expert_layers=16))
    assert cfg == TINY


def test_infer_config_reads_cross_attention_period_and_widths():
    cfg = TINY.with_(self_attn_every_n_layers=4, expert_layers=8, expert_hidden=480, expert_mlp=1280)
    state = random_weights(cfg, 1)
    got = infer_config(state, base=TINY)
    assert got.self_attn_every_n_layers == 4 and got.expert_hidden == 480 and got.expert_mlp == 1280
    assert got.expert_layers == 8
    assert set(required_keys(got)) <= set(state)


def test_missing_tensor_is_reported():
    state = random_weights(TINY, 2)
    del state[f"{EXPERT}.layers.1.mlp.down_proj.weight"]
    with pytest.raises(KeyError):
        infer_config(state, base=TINY)


def test_bare_model_keys_get_the_policy_prefix(tmp_path):
    state = random_weights(TINY, 4)
    _save({k[len("model."):]: v for k, v in state.items()}, tmp_path / "m.safetensors")
    assert set(load_checkpoint(tmp_path / "m.safetensors")) == set(state)


@pytest.mark.gpu
def test_packed_round_trip_gives_identical_actions(tmp_path):
    from oracle.model import calibrate as oracle_calibrate
    from smolvla_mujoco_libero_b200 import synthetic
    from smolvla_mujoco_libero_b200.calibrate import load_scale_json
    from smolvla_mujoco_libero_b200.checkpoint import load_packed, save_packed
    from smolvla_mujoco_libero_b200.model import DeviceWeights
    from smolvla_mujoco_libero_b200.policy import SampleActions
    w = random_weights(TINY, 0)
    obs = lambda b, s: synthetic.observations(b, seed=s, image_size=TINY.image_size, n_tokens=TINY.n_lang)  # noqa: E731
    js = oracle_calibrate(TINY, w, [obs(1, 100)])
    dw = DeviceWeights(TINY, w, load_scale_json(js))
    save_packed(dw, tmp_path / "packed.safetensors")
    dw2 = load_packed(tmp_path / "packed.safetensors")
    assert dw2.cfg == TINY and set(dw2.lin) == set(dw.lin)
    o = obs(2, 9)
    args = ([im.cuda() for im in o.images], [m.cuda() for m in o.img_masks], o.lang_tokens.cuda(), o.lang_masks.cuda(),
            o.state.cuda(), o.noise.cuda())
    a1 = SampleActions(TINY, dw, use_cuda_graph=False)(*args)
    a2 = SampleActions(TINY, dw2, use_cuda_graph=False)(*args)
    assert torch.equal(a1.cpu(), a2.cpu())
