"""Parity of the benchmarked workloads (single text layer, prefix encode, batch-64 call), at their own shapes, with the oracle.

* one SmolVLM2 text decoder layer at prefix length 177 (hidden N(0,1) with 8 outlier channels x30, random
  N(0, 0.02) weights, SmoothQuant scales calibrated on that distribution), through the runner's own launch
  list: every int8 activation (q/k/v, o, gate/up) and every int32 accumulator bit-exact given the same bf16
  input, each bf16 stage within its rounding bound, the layer output at cosine >= 0.9999 against the oracle's
  layer run from the same hidden state;
* the full prefix encode (SigLIP 12x768 on two 512 px images, connector, 16 text layers) at batch 1 and
  batch 64 (split-K, the tile widths the batch-64 call picks): the prefix KV cache of every layer and the
  final prefix hidden states against the oracle on sampled observations;
* the batch-64 sample_actions call the benchmark times (split-K on, per-layer expert launches, GPU-calibrated
  scales from four observations) against the oracle on observations {0, 21, 42, 63}: cosine >= 0.999 and
  max-abs <= 2e-2 on the action chunk;
* the reference's debug core outputs (prefix_embs, prefix_out, suffix_out / v_t / x_t per step) and its
  embeds mode (image embeddings in place of images) against the oracle.
Intermediate names follow deploy/diagnose_3_4_numeric_baseline.py:55-70, :148-206.
"""

import pytest
import torch
import torch.nn.functional as F

from oracle import quant as Q
from oracle.model import OracleSmolVLA, apply_rope, eager_attention, make_att_2d_masks, rms_norm
from oracle.model import calibrate as oracle_calibrate
from smolvla_mujoco_libero_b200 import _lib as L
from smolvla_mujoco_libero_b200 import ops, synthetic
from smolvla_mujoco_libero_b200.calibrate import calibrate as gpu_calibrate, load_scale_json
from smolvla_mujoco_libero_b200.config import BENCH, CONNECTOR, TEXT, TINY
from smolvla_mujoco_libero_b200.model import DeviceWeights, SmolVLARunner
from smolvla_mujoco_libero_b200.policy import DebugCore, PrefixFeatures, SampleActions, debug_output_names
from smolvla_mujoco_libero_b200.weights import random_weights

pytestmark = pytest.mark.gpu
DEV = "cuda"
ROWS_B64 = (0, 21, 42, 63)


def cosine(a, b):
    return float(F.cosine_similarity(a.float().flatten().cpu(), b.float().flatten().cpu(), dim=0))


def max_abs(a, b):
    return float((a.float().cpu() - b.float().cpu()).abs().max())


def ulp_close(got, ref, ulps=1.0, max_mismatch=None):
    """|got - ref| <= ulps bf16 ulps of |ref| (+ 1e-5 max|ref|); optionally also a cap on the fraction of
    elements that differ at all (a summation order can flip a rare rounding)."""
    got, ref = got.float().cpu(), ref.float().cpu()
    tol = ref.abs() * (ulps * 2.0 ** -7) + 1e-5 * float(ref.abs().max()) + 1e-6
    assert not bool(((got - ref).abs() > tol).any()), float(((got - ref).abs() > tol).float().mean())
    if max_mismatch is not None:
        assert float((got != ref).float().mean()) <= max_mismatch


def _obs(cfg, b, seed, **kw):
    return synthetic.observations(b, seed=seed, image_size=cfg.image_size, n_tokens=cfg.n_lang, **kw)


def _rows(o, idx):
    idx = list(idx)
    return synthetic.Observation(images=[im[idx] for im in o.images], img_masks=[m[idx] for m in o.img_masks],
                                 lang_tokens=o.lang_tokens[idx], lang_masks=o.lang_masks[idx], state=o.state[idx],
                                 noise=o.noise[idx])


def _dev(o):
    return ([im.to(DEV) for im in o.images], [m.to(DEV) for m in o.img_masks], o.lang_tokens.to(DEV),
            o.lang_masks.to(DEV), o.state.to(DEV), o.noise.to(DEV))


# ----------------------------------------------------------------------------- one text decoder layer (L = 177)

def _layer_case(wavelength):
    """The single-layer workload: weights of one text layer (the rest of the model is present but unused),
    SmoothQuant scales calibrated on 8 hidden-state batches of the same distribution as the input."""
    cfg = BENCH.with_(vis_layers=0, text_layers=1, expert_layers=1, rope_wavelength=wavelength)
    w = random_weights(cfg, 3)
    g = synthetic.generator(1177)
    ch = synthetic.outlier_channels(cfg.hidden, 8, g)
    L_ = cfg.prefix_len
    assert L_ == 177
    h_in = synthetic.outlier_activations(L_, cfg.hidden, ch, 30.0, g)[None]
    calib = [synthetic.outlier_activations(L_, cfg.hidden, ch, 30.0, g)[None] for _ in range(8)]
    n_valid_lang = 42  # the last 6 language tokens are padding
    pad = torch.ones(1, L_, dtype=torch.bool)
    n_img = cfg.n_cams * cfg.n_img_tokens
    pad[:, n_img + n_valid_lang:n_img + cfg.n_lang] = False
    att = torch.tensor([0] * (L_ - 1) + [1], dtype=torch.bool)[None]
    mask = make_att_2d_masks(pad, att)
    pos = torch.cumsum(pad.to(torch.int64), dim=1) - 1
    # calibration of the layer's six W8A8 linears (the reference collector + build_entry on the bf16 layer)
    bf = OracleSmolVLA(cfg, w, mode="bf16")
    col = Q.PerChannelCollector(cfg.percentile)
    layer_mods = {f"{TEXT}.layers.0.{n}" for n in ("self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                                                    "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj")}
    bf.collector = lambda name, x: col.observe(name, x) if name in layer_mods else None
    for h in calib:
        bf.text_layer(0, h, mask, pos)
    entries = [Q.build_smoothquant_entry(r, w[f"{r['module']}.weight"], cfg.alpha) for r in col.rows()]
    assert {e["module"] for e in entries} == layer_mods
    # the connector is never run here (image embeddings are given); it still needs an entry to be packed
    k_conn = cfg.vis_hidden * cfg.scale_factor ** 2
    entries.append({"module": CONNECTOR, "scale": 0.05, "smooth_scale": [1.0] * k_conn,
                    "quantization": "smoothquant_symmetric_static_per_tensor", "smoothquant_alpha": cfg.alpha})
    js = {"smoothquant_alpha": cfg.alpha, "linear_call_scales": entries}
    return cfg, w, js, h_in, pad, mask, pos, n_valid_lang


@pytest.mark.parametrize("wavelength", [10_000.0, 100_000.0])
def test_text_decoder_layer_at_prefix_length_177(wavelength):
    cfg, w, js, h_in, pad, mask, pos, n_valid_lang = _layer_case(wavelength)
    p = f"{TEXT}.layers.0"
    dw = DeviceWeights(cfg, w, load_scale_json(js))
    r = SmolVLARunner(dw, 1, debug_taps=True, prefix_only=True, image_embeds=True)
    taps = {}

    def observe(names, buf):
        if names == ["prefix_embs"]:
            buf.copy_(h_in[0].to(DEV))  # the layer's input replaces the prefix embeddings
        for n in names:
            taps[n] = buf.clone()

    n_img = cfg.n_img_tokens
    embs = [torch.zeros(1, n_img, cfg.hidden, dtype=torch.bfloat16, device=DEV) for _ in range(cfg.n_cams)]
    lang_masks = torch.zeros(1, cfg.n_lang, dtype=torch.bool)
    lang_masks[:, :n_valid_lang] = True
    toks = torch.randint(0, cfg.vocab, (1, cfg.n_lang), generator=synthetic.generator(5))
    r.load_inputs(embs, [torch.ones(1, dtype=torch.bool, device=DEV)] * cfg.n_cams, toks.to(DEV),
                  lang_masks.to(DEV), torch.zeros(1, cfg.max_state_dim, device=DEV), None)
    r.run(observer=observe)
    torch.cuda.synchronize()
    assert L.device_error() == 0
    assert torch.equal(r.key_pad[0, :cfg.prefix_len].bool().cpu(), pad[0])
    orc = OracleSmolVLA(cfg, w, Q.load_activation_scales_by_module(js))
    lin = orc.lin
    h = h_in[0]

    def t(name):
        return taps[name].cpu()

    def int_dequant(mod, q8):
        m = lin[mod]
        return Q.w8a8_int_dequant(Q.int_gemm(q8, m.qweight), m.act_scale, m.weight_scale, m.bias)

    # RMSNorm + q/k/v quantisation: bf16 rows within one ulp of the oracle's, int8 bit-exact given them
    q_mod, k_mod, v_mod = (f"{p}.self_attn.{n}" for n in ("q_proj", "k_proj", "v_proj"))
    # RMSNorm rounds twice (x * rsqrt to bf16, then * weight): a flipped first rounding can leave two ulps
    y = t(q_mod)[:177]
    ulp_close(y, rms_norm(h, w[f"{p}.input_layernorm.weight"], cfg.rms_eps), ulps=2.0, max_mismatch=1e-3)
    q8 = {}
    for mod in (q_mod, k_mod, v_mod):
        q8[mod] = t(f"{mod}#int8")[:177]
        assert torch.equal(q8[mod], lin[mod].quantize_input(y)), mod
        # the packed weights and their int32 accumulators, bit-exact
        acc = ops.gemm_i8_i32(q8[mod].to(DEV), dw.lin[mod].weight)
        assert torch.equal(dw.lin[mod].weight.cpu(), lin[mod].qweight)
        assert torch.equal(dw.lin[mod].wscale.cpu(), lin[mod].weight_scale)
        assert torch.equal(acc.cpu(), Q.int_gemm(q8[mod], lin[mod].qweight)), mod
    # projections + RoPE (the KV cache): v bit-exact with bf16 of the integer-dequant form, q / k within one
    # ulp of the rotated pair
    v_ref = int_dequant(v_mod, q8[v_mod]).to(torch.bfloat16)
    assert torch.equal(t(f"{p}.self_attn.v")[:177], v_ref)
    assert torch.equal(r.vcache[0].cpu()[:177], v_ref)
    for mod, name, heads in ((q_mod, "q_rope", cfg.heads), (k_mod, "k_rope", cfg.kv_heads)):
        pre = int_dequant(mod, q8[mod]).to(torch.bfloat16)
        ref = apply_rope(pre.view(1, 177, heads, 64), pos, wavelength).reshape(177, -1)
        got = t(f"{p}.self_attn.{name}")[:177].float()
        pair = pre.float().view(177, heads, 2, 32)
        norm = (pair[:, :, 0] ** 2 + pair[:, :, 1] ** 2).sqrt()
        bound = (ref.float().abs() + torch.stack([norm, norm], 2).reshape(177, -1)) * 2.0 ** -7 + 1e-5
        assert bool(((got - ref.float()).abs() <= bound).all()), name
    # masked GQA attention: bf16 context against the oracle on the kernel's own q / k / v, int8 bit-exact
    qg, kg, vg = (t(f"{p}.self_attn.{n}")[:177][None] for n in ("q_rope", "k_rope", "v"))
    ctx = t(f"{p}.self_attn.o_proj")[:177]
    ctx_ref = eager_attention(qg, kg, vg, mask, cfg.heads, cfg.kv_heads)[0]
    assert cosine(ctx, ctx_ref) >= 0.9999 and max_abs(ctx, ctx_ref) <= 2e-2
    o_mod = f"{p}.self_attn.o_proj"
    ctx8 = t(f"{o_mod}#int8")[:177]
    assert torch.equal(ctx8, lin[o_mod].quantize_input(ctx))
    # o_proj + residual, bit-exact: bf16(bf16((acc * a) * w_s) + h)
    h1 = t(f"{p}.attn_residual")[:177]
    assert torch.equal(h1, (int_dequant(o_mod, ctx8).to(torch.bfloat16).float() + h.float()).to(torch.bfloat16))
    # post-attention RMSNorm + gate / up quantisation
    g_mod, u_mod, d_mod = (f"{p}.mlp.{n}" for n in ("gate_proj", "up_proj", "down_proj"))
    y2 = t(g_mod)[:177]
    ulp_close(y2, rms_norm(h1, w[f"{p}.post_attention_layernorm.weight"], cfg.rms_eps), ulps=2.0, max_mismatch=1e-3)
    for mod in (g_mod, u_mod):
        assert torch.equal(t(f"{mod}#int8")[:177], lin[mod].quantize_input(y2)), mod
    # SiLU gate (three bf16 roundings) and the W8A16 down projection + residual
    gate = int_dequant(g_mod, t(f"{g_mod}#int8")[:177]).to(torch.bfloat16)
    up = int_dequant(u_mod, t(f"{u_mod}#int8")[:177]).to(torch.bfloat16)
    act = t(d_mod)[:177]
    ulp_close(act, (F.silu(gate) * up), ulps=2.0)
    out = t(f"{p}.output")[:177]
    down = (act.float() @ lin[d_mod].weight.float().t()).to(torch.bfloat16)
    out_ref = (down.float() + h1.float()).to(torch.bfloat16).float()
    # one ulp of the projection (fp32 summation order) plus one of the sum, whatever the sum cancels
    bound = (down.float().abs() + out_ref.abs()) * 2.0 ** -7 + 1e-5
    assert bool(((out.float() - out_ref).abs() <= bound).all())
    # the whole layer against the oracle's layer from the same hidden state
    ref_taps = {}
    ref_out, (k_ref, v_ref2) = orc.text_layer(0, h_in, mask, pos, taps=ref_taps)
    assert cosine(out, ref_out[0]) >= 0.9999
    assert cosine(out.float() - h.float(), ref_out[0].float() - h.float()) >= 0.999
    assert cosine(r.kcache[0].cpu()[:177], k_ref[0]) >= 0.999
    assert cosine(r.vcache[0].cpu()[:177], v_ref2[0]) >= 0.999
    # the final RMSNorm (prefix_out)
    ulp_close(r.prefix_out.cpu()[:177], rms_norm(out, w[f"{TEXT}.norm.weight"], cfg.rms_eps), ulps=2.0,
              max_mismatch=1e-3)


# ----------------------------------------------------------------------------- benchmark architecture

@pytest.fixture(scope="module")
def bench():
    """BENCH weights with scales from the GPU calibration tool on four observations, as bench.py makes them."""
    torch.set_num_threads(max(8, torch.get_num_threads()))
    w = random_weights(BENCH, 0)
    js = gpu_calibrate(BENCH, w, [_obs(BENCH, 1, 100 + i) for i in range(4)])
    dw = DeviceWeights(BENCH, w, load_scale_json(js))
    orc = OracleSmolVLA(BENCH, w, Q.load_activation_scales_by_module(js))
    return w, js, dw, orc


def _prefix_check(feats, taps, row, ref_row=0):
    """16 quantized layers deep the two paths (exact int32 GEMMs on the GPU, bf16 fake-dequant GEMMs in the
    oracle) round differently and some int8 activations flip, so the bar is relative: cosine >= 0.999 and
    relative L2 <= 5% on the final prefix hidden states and on every layer's K and V."""
    z = feats["z"][row].cpu()
    ref = taps["prefix_out"][ref_row].float()
    rel = float((z - ref).norm() / ref.norm())
    assert cosine(z, ref) >= 0.999 and rel <= 0.05, (row, cosine(z, ref), rel, max_abs(z, ref))
    for layer, ((k, v), (rk, rv)) in enumerate(zip(feats["kv_cache"], taps["kv"])):
        for got, want in ((k[row], rk[ref_row]), (v[row], rv[ref_row])):
            got, want = got.float().cpu(), want.float()
            rel = float((got - want).norm() / want.norm())
            assert cosine(got, want) >= 0.999 and rel <= 0.05, (row, layer, cosine(got, want), rel)


def test_prefix_kv_cache_bench_architecture_batch1_and_batch64(bench):
    """Full prefix encode at batch 1 and at batch 64 (split-K), KV cache of all 16 layers + prefix_out."""
    w, js, dw, orc = bench
    pf = PrefixFeatures(BENCH, dw)
    o64 = _obs(BENCH, 64, 5000)
    images, img_masks, toks, lmask, state, _ = _dev(o64)
    f64 = pf.extract(images, img_masks, toks, lmask, state)
    f1 = pf.extract(*_dev(_rows(o64, [21]))[:5])
    torch.cuda.synchronize()
    assert L.device_error() == 0
    sub = _rows(o64, ROWS_B64)
    prefix, pad, att = orc.embed_prefix(sub.images, sub.img_masks, sub.lang_tokens, sub.lang_masks, sub.state)
    cache, prefix_out, _, _ = orc.prefix_forward(prefix, pad, att)
    taps = {"prefix_out": prefix_out, "kv": cache}
    for j, row in enumerate(ROWS_B64):
        _prefix_check(f64, taps, row, j)
    _prefix_check(f1, taps, 0, ROWS_B64.index(21))


def test_bench_batch64_sample_actions_matches_oracle(bench):
    """The call bench.py times: SmolVLARunner(weights, 64) with split-K, replayed as a CUDA graph."""
    w, js, dw, orc = bench
    runner = SmolVLARunner(dw, 64)
    assert runner.split_k and not runner.flow
    o = _obs(BENCH, 64, 1_000_000)
    runner.load_inputs(*_dev(o))
    runner.capture()
    runner.run()
    got = runner.actions().cpu()
    assert L.device_error() == 0
    assert torch.isfinite(got).all()
    sub = _rows(o, ROWS_B64)
    ref = orc.sample_actions(sub.images, sub.img_masks, sub.lang_tokens, sub.lang_masks, sub.state, sub.noise)
    A = BENCH.action_dim
    for j, row in enumerate(ROWS_B64):
        c, m = cosine(got[row, :, :A], ref[j, :, :A]), max_abs(got[row, :, :A], ref[j, :, :A])
        assert c >= 0.999 and m <= 2e-2, (row, c, m)
        # the padded action dimensions follow the same computation
        assert cosine(got[row], ref[j]) >= 0.999, row


# ----------------------------------------------------------------------------- debug core and embeds mode

@pytest.fixture(scope="module")
def tiny():
    w = random_weights(TINY, 0)
    js = oracle_calibrate(TINY, w, [_obs(TINY, 1, 100 + i) for i in range(2)])
    return w, js


def test_debug_outputs_match_oracle_and_the_deployed_call(tiny):
    w, js = tiny
    sa = SampleActions(TINY, DeviceWeights(TINY, w, load_scale_json(js)))
    o = _obs(TINY, 2, 77, n_valid_tokens=10)
    outs = sa.debug_outputs(*_dev(o))
    assert list(outs) == debug_output_names(TINY)
    # the debug launches compute the deployed call's arithmetic (same kernels and tile choices at this batch)
    assert torch.equal(outs["action_chunk"], sa(*_dev(o)))
    taps = {}
    ref = OracleSmolVLA(TINY, w, Q.load_activation_scales_by_module(js)).sample_actions(
        o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise, taps=taps)
    assert cosine(outs["action_chunk"], ref[:, :, :TINY.action_dim]) >= 0.999
    for name in debug_output_names(TINY)[1:]:
        got, want = outs[name], taps[name]
        assert got.shape == want.shape, name
        assert cosine(got, want) >= 0.999, name
        assert max_abs(got, want) <= 2e-2 * float(want.abs().max()) + 2e-2, name
    # x_t_step_NN is the Euler state after each step: the last one is the chunk
    last = f"x_t_step_{TINY.num_steps - 1:02d}"
    assert torch.equal(outs[last][:, :, :TINY.action_dim], outs["action_chunk"])
    # x_{k+1} = x_k + dt * v_k in fp32
    dt = -1.0 / TINY.num_steps
    x1 = o.noise.to(DEV) + dt * outs["v_t_step_00"]
    assert torch.allclose(outs["x_t_step_00"], x1, rtol=0, atol=1e-6)


def test_embeds_mode_matches_oracle(tiny):
    """Image embeddings (the connector's output, here the oracle's embed_image) in place of the images."""
    w, js = tiny
    sa = SampleActions(TINY, DeviceWeights(TINY, w, load_scale_json(js)))
    orc = OracleSmolVLA(TINY, w, Q.load_activation_scales_by_module(js))
    o = _obs(TINY, 3, 91)
    embs = [orc.embed_image(im) for im in o.images]
    got = sa.from_image_embeds([e.to(DEV) for e in embs], [m.to(DEV) for m in o.img_masks], o.lang_tokens.to(DEV),
                               o.lang_masks.to(DEV), o.state.to(DEV), o.noise.to(DEV)).cpu()
    ref = orc.sample_actions(None, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise,
                             image_embs=embs)[:, :, :TINY.action_dim]
    assert cosine(got, ref) >= 0.999 and max_abs(got, ref) <= 2e-2
    # the debug core in embeds mode: prefix_embs rows of the images are bf16(emb * bf16(sqrt(hidden)))
    core = DebugCore(sa)
    outs = core(embs[0].to(DEV), embs[1].to(DEV), o.img_masks[0].to(DEV), o.img_masks[1].to(DEV), o.state.to(DEV),
                o.lang_tokens.to(DEV), o.lang_masks.to(DEV), o.noise.to(DEV))
    assert len(outs) == len(core.output_names)
    prefix = outs[core.output_names.index("prefix_embs")].cpu()
    scale = torch.tensor(TINY.hidden ** 0.5, dtype=torch.bfloat16)
    n = TINY.n_img_tokens
    assert torch.equal(prefix[:, :n], embs[0] * scale)
    assert torch.equal(prefix[:, n:2 * n], embs[1] * scale)
    assert torch.equal(outs[0], got.to(DEV))
