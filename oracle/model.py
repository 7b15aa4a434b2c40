"""CPU restatement of the SmolVLA sample_actions core with SmoothQuant fake-dequant linears (oracle).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

The model code (VLAFlowMatching, SmolVLMWithExpertModel) lives in lerobot 0.5.1, which the reference does
not ship; everything here that lerobot computes is restated from the reference's call sites and
restatements and is therefore UNPINNED:
  * prefix embed, masks, positions, denoise loop: deploy/diagnose_3_4_numeric_baseline.py:42-206
  * attention: deploy/export_6f_layer0_attention_tensors.py:100-119, expand_kv
    deploy/diagnose_5i_attention_error_propagation.py:205-226
  * RoPE: deploy/validate_fused_rope_layout_math.py:28-42 (the only part pinned: tests/golden/rope_kat.npz)
  * SigLIP encoder, pixel-shuffle connector, Llama RMSNorm / MLP: transformers SmolVLM / Llama semantics
  * action expert, embed_suffix, cross-attention: lerobot 0.5.1 semantics (expert layers interleave
    self-attention over [prefix KV ; suffix] with cross-attention whose K/V are the expert's k_proj / v_proj
    applied to the cached prefix K (post-RoPE) and V; cross-attention queries use positions 0..49).
Linears follow deploy/linear_only_quant.py through oracle.quant (pinned by the golden fixtures).
"""

from __future__ import annotations

import math

import torch
import torch.nn.functional as F

MASKED = torch.finfo(torch.float32).min


# ----------------------------------------------------------------------------- primitives

def apply_rope(x: torch.Tensor, positions: torch.Tensor, max_wavelength: float = 10_000.0) -> torch.Tensor:
    """Rotate-half RoPE on x [B, L, H, D] (deploy/validate_fused_rope_layout_math.py:28-42)."""
    d_half = x.shape[-1] // 2
    dtype = x.dtype
    xf = x.to(torch.float32)
    freq_exponents = (2.0 / x.shape[-1]) * torch.arange(d_half, dtype=torch.float32)
    timescale = max_wavelength ** freq_exponents
    radians = positions[..., None].to(torch.float32) / timescale[None, None, :]
    radians = radians[..., None, :]
    sin, cos = torch.sin(radians), torch.cos(radians)
    x1, x2 = xf.split(d_half, dim=-1)
    out = torch.empty_like(xf)
    out[..., :d_half] = x1 * cos - x2 * sin
    out[..., d_half:] = x2 * cos + x1 * sin
    return out.to(dtype)


def rms_norm(x: torch.Tensor, weight: torch.Tensor, eps: float) -> torch.Tensor:
    """transformers LlamaRMSNorm: weight * bf16(x * rsqrt(mean(x^2) + eps))."""
    dtype = x.dtype
    h = x.to(torch.float32)
    var = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(var + eps)
    return weight * h.to(dtype)


def layer_norm(x: torch.Tensor, weight: torch.Tensor, bias: torch.Tensor, eps: float) -> torch.Tensor:
    return F.layer_norm(x, (x.shape[-1],), weight, bias, eps)


def pixel_shuffle(x: torch.Tensor, scale: int) -> torch.Tensor:
    """SmolVLM connector pixel shuffle: [B, S, D] -> [B, S / scale^2, D * scale^2]."""
    bsz, seq, dim = x.shape
    side = int(seq ** 0.5)
    x = x.view(bsz, side, side, dim)
    x = x.view(bsz, side, side // scale, dim * scale)
    x = x.permute(0, 2, 1, 3)
    x = x.reshape(bsz, side // scale, side // scale, dim * scale * scale)
    x = x.permute(0, 2, 1, 3)
    return x.reshape(bsz, seq // (scale * scale), dim * scale * scale)


def eager_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, mask: torch.Tensor | None, hq: int,
                    hkv: int) -> torch.Tensor:
    """q [B, Lq, hq*64], k/v [B, Lk, hkv*64] (bf16, post-RoPE), mask bool [B, Lq, Lk] -> bf16 [B, Lq, hq*64].

    deploy/export_6f_layer0_attention_tensors.py:100-119 with the GQA expansion of
    deploy/diagnose_5i_attention_error_propagation.py:205-226."""
    b, lq, _ = q.shape
    lk = k.shape[1]
    d = 64
    groups = hq // hkv
    qh = q.view(b, lq, hq, d)
    kh = k.view(b, lk, hkv, 1, d).expand(b, lk, hkv, groups, d).reshape(b, lk, hq, d)
    vh = v.view(b, lk, hkv, 1, d).expand(b, lk, hkv, groups, d).reshape(b, lk, hq, d)
    qt = qh.to(torch.float32).transpose(1, 2)
    kt = kh.to(torch.float32).transpose(1, 2)
    scores = torch.matmul(qt, kt.transpose(2, 3)) * (d ** -0.5)
    if mask is not None:
        scores = torch.where(mask[:, None, :, :], scores, MASKED)
    probs = torch.softmax(scores, dim=-1)
    ctx = torch.matmul(probs.to(vh.dtype), vh.permute(0, 2, 1, 3))
    return ctx.permute(0, 2, 1, 3).reshape(b, lq, hq * d)


def fused_rope_attention(q_raw: torch.Tensor, k_raw: torch.Tensor, v_raw: torch.Tensor, positions: torch.Tensor,
                         mask: torch.Tensor, hq: int, hkv: int, head_dim: int = 64,
                         max_wavelength: float = 10_000.0) -> torch.Tensor:
    """The SmolVLAFusedRopeAttention plugin's arithmetic (deploy/cuda/fused_rope_layout.cu:271-431), all fp32:
    raw q [B, L, hq*D], k / v [B, L, hkv*D] (any float dtype, read as fp32), positions [B, L], keep-mask bool
    [B, L, L] -> context fp32 [B, hq, L, D].  RoPE on the fp32 values (no rounding back to the input dtype),
    masked scores at finfo.min (a query with no kept key gets the mean of V), fp32 softmax and P.V."""
    b, L, _ = q_raw.shape
    g = hq // hkv
    q = apply_rope(q_raw.float().view(b, L, hq, head_dim), positions, max_wavelength)
    k = apply_rope(k_raw.float().view(b, L, hkv, head_dim), positions, max_wavelength).repeat_interleave(g, dim=2)
    v = v_raw.float().view(b, L, hkv, head_dim).repeat_interleave(g, dim=2)
    scores = torch.einsum("bqhd,bkhd->bhqk", q, k) * (head_dim ** -0.5)
    scores = torch.where(mask.bool()[:, None], scores, MASKED)
    return torch.einsum("bhqk,bkhd->bhqd", torch.softmax(scores, dim=-1), v)


def make_att_2d_masks(pad_masks: torch.Tensor, att_masks: torch.Tensor) -> torch.Tensor:
    """deploy/diagnose_3_4_numeric_baseline.py:42-46."""
    cumsum = torch.cumsum(att_masks.to(torch.int64), dim=1)
    att_2d = cumsum[:, None, :] <= cumsum[:, :, None]
    pad_2d = pad_masks[:, None, :] & pad_masks[:, :, None]
    return att_2d & pad_2d


def sinusoidal_time_embedding(t: torch.Tensor, dim: int, min_period: float, max_period: float) -> torch.Tensor:
    """lerobot create_sinusoidal_pos_embedding (float64 internally)."""
    fraction = torch.linspace(0.0, 1.0, dim // 2, dtype=torch.float64)
    period = min_period * (max_period / min_period) ** fraction
    scaling = 1.0 / period * 2 * math.pi
    sin_input = scaling[None, :] * t.to(torch.float64)[:, None]
    return torch.cat([torch.sin(sin_input), torch.cos(sin_input)], dim=1)


# ----------------------------------------------------------------------------- full core

class OracleSmolVLA:
    """sample_actions of SmolVLA on the CPU.

    mode = "quant": the deployed recipe -- SmoothQuant W8A8 (oracle.quant.W8A8Linear) on the vision tower,
                    connector and text q/k/v/o/gate/up; W8A16 on text down_proj and every expert linear;
                    bf16 state / action / time projections.
    mode = "bf16":  every linear in bf16 (the unquantised model, used for calibration).
    ``collector(module, x)`` (optional) sees the input of every W8A8-recipe linear, which is what the
    reference's PerChannelLinearInputCollector hooks (calibrate_smolvla_activation_channel_scales.py:62-84).
    """

    def __init__(self, cfg, weights: dict[str, torch.Tensor], scales: dict | None = None, mode: str = "quant"):
        from smolvla_mujoco_libero_b200.weights import linear_specs
        from . import quant as Q

        self.cfg, self.w, self.mode = cfg, weights, mode
        self.lin = {}
        for name, _n, k, has_bias, q in linear_specs(cfg):
            wt, b = weights[f"{name}.weight"], weights.get(f"{name}.bias") if has_bias else None
            if mode == "bf16" or q == "bf16":
                self.lin[name] = Q.Bf16Linear(wt, b)
            elif q == "w8a16":
                self.lin[name] = Q.W8A16Linear(wt, b)
            else:
                if scales is None or name not in scales:
                    raise KeyError(f"missing calibrated activation scale for quantized module: {name}")
                entry = Q.select_activation_scale_for_linear(scales[name], k)
                self.lin[name] = Q.W8A8Linear(wt, b, entry["scale"], torch.tensor(entry["smooth_scale"]))
        self.collector = None

    # -- helpers
    def _linear(self, name: str, x: torch.Tensor) -> torch.Tensor:
        if self.collector is not None and self.mode == "bf16":
            from smolvla_mujoco_libero_b200.weights import w8a8_modules
            if not hasattr(self, "_w8a8"):
                self._w8a8 = set(w8a8_modules(self.cfg))
            if name in self._w8a8:
                self.collector(name, x)
        return self.lin[name](x)

    # -- vision
    def vision_embeddings(self, image: torch.Tensor) -> torch.Tensor:
        """Patch-16 conv (bf16) + learned position embedding: fp32 [B,3,S,S] -> bf16 [B, n_patches, vis_hidden]
        (SmolVLMVisionEmbeddings with every patch valid, so the position ids are 0..n_patches-1)."""
        from smolvla_mujoco_libero_b200.config import VISION
        c, w = self.cfg, self.w
        pe = f"{VISION}.embeddings"
        x = F.conv2d(image.to(torch.bfloat16), w[f"{pe}.patch_embedding.weight"], w[f"{pe}.patch_embedding.bias"],
                     stride=c.patch)
        return x.flatten(2).transpose(1, 2) + w[f"{pe}.position_embedding.weight"][None]

    def vision_attention(self, i: int, y: torch.Tensor) -> torch.Tensor:
        """q/k/v projections, unmasked attention (scores and softmax in fp32, export_6f's restatement), out_proj."""
        from smolvla_mujoco_libero_b200.config import VISION
        c = self.cfg
        p = f"{VISION}.encoder.layers.{i}"
        q = self._linear(f"{p}.self_attn.q_proj", y)
        k = self._linear(f"{p}.self_attn.k_proj", y)
        v = self._linear(f"{p}.self_attn.v_proj", y)
        ctx = eager_attention(q, k, v, None, c.vis_heads, c.vis_heads)
        return self._linear(f"{p}.self_attn.out_proj", ctx)

    def vision_mlp(self, i: int, y: torch.Tensor) -> torch.Tensor:
        """fc1 -> GELU(tanh) -> fc2 (SmolVLMVisionMLP with gelu_pytorch_tanh)."""
        from smolvla_mujoco_libero_b200.config import VISION
        p = f"{VISION}.encoder.layers.{i}"
        return self._linear(f"{p}.mlp.fc2", F.gelu(self._linear(f"{p}.mlp.fc1", y), approximate="tanh"))

    def vision_layer(self, i: int, h: torch.Tensor) -> torch.Tensor:
        """Pre-LN encoder layer (SmolVLMEncoderLayer): h + attn(LN1(h)), then + mlp(LN2(.))."""
        from smolvla_mujoco_libero_b200.config import VISION
        c, w = self.cfg, self.w
        p = f"{VISION}.encoder.layers.{i}"
        h = h + self.vision_attention(i, layer_norm(h, w[f"{p}.layer_norm1.weight"], w[f"{p}.layer_norm1.bias"],
                                                    c.vis_eps))
        return h + self.vision_mlp(i, layer_norm(h, w[f"{p}.layer_norm2.weight"], w[f"{p}.layer_norm2.bias"],
                                                 c.vis_eps))

    def connector(self, h: torch.Tensor) -> torch.Tensor:
        """Post-LayerNorm output -> pixel shuffle -> modality projection (SmolVLMConnector)."""
        from smolvla_mujoco_libero_b200.config import CONNECTOR
        return self._linear(CONNECTOR, pixel_shuffle(h, self.cfg.scale_factor))

    def embed_image(self, image: torch.Tensor) -> torch.Tensor:
        """SigLIP + pixel-shuffle connector: fp32 [B,3,S,S] -> bf16 [B, n_img_tokens, hidden]."""
        from smolvla_mujoco_libero_b200.config import VISION
        c, w = self.cfg, self.w
        h = self.vision_embeddings(image)
        for i in range(c.vis_layers):
            h = self.vision_layer(i, h)
        h = layer_norm(h, w[f"{VISION}.post_layernorm.weight"], w[f"{VISION}.post_layernorm.bias"], c.vis_eps)
        return self.connector(h)

    # -- prefix
    def embed_prefix(self, images, img_masks, lang_tokens, lang_masks, state, image_embs=None):
        """deploy/diagnose_3_4_numeric_baseline.py:72-115.  The image embeddings come from embed_image, or, in
        the embeds mode of the exported core (deploy/export_smolvla_sample_actions_onnx.py:64-115), are given
        as ``image_embs`` (one bf16 [B, n_img_tokens, hidden] per camera) and ``images`` is ignored."""
        from smolvla_mujoco_libero_b200.config import TEXT
        c = self.cfg
        embs, pads, att = [], [], []
        sources = image_embs if image_embs is not None else [self.embed_image(img) for img in images]
        for e, m in zip(sources, img_masks):
            e = e.to(torch.bfloat16)
            e = e * torch.tensor(e.shape[-1] ** 0.5, dtype=e.dtype)
            embs.append(e)
            pads.append(m[:, None].expand(e.shape[0], e.shape[1]))
            att += [0] * e.shape[1]
        lang = F.embedding(lang_tokens, self.w[f"{TEXT}.embed_tokens.weight"])
        lang = lang * math.sqrt(lang.shape[-1])
        embs.append(lang)
        pads.append(lang_masks)
        att += [0] * lang.shape[1]
        st = self.lin["model.state_proj"](state.to(torch.bfloat16))[:, None, :]
        embs.append(st)
        pads.append(torch.ones(st.shape[0], 1, dtype=torch.bool))
        att += [1]
        prefix = torch.cat(embs, dim=1)
        pad = torch.cat(pads, dim=1)
        att_t = torch.tensor(att, dtype=torch.bool)[None].expand(prefix.shape[0], -1)
        return prefix, pad, att_t

    def _mlp(self, p: str, y: torch.Tensor) -> torch.Tensor:
        return self._linear(f"{p}.mlp.down_proj",
                            F.silu(self._linear(f"{p}.mlp.gate_proj", y)) * self._linear(f"{p}.mlp.up_proj", y))

    def text_layer(self, i: int, h: torch.Tensor, mask: torch.Tensor, pos: torch.Tensor, taps: dict | None = None):
        """One SmolVLM2 text decoder layer with KV fill (lerobot forward_attn_layer, fill_kv_cache=True):
        RMSNorm -> q/k/v (W8A8) -> RoPE -> masked GQA attention -> o_proj (W8A8) + residual -> RMSNorm ->
        SiLU(gate) * up (W8A8) -> down (W8A16) + residual.  Returns (h, (k post-RoPE, v)); ``taps`` (optional)
        receives the layer's intermediate bf16 tensors by name."""
        from smolvla_mujoco_libero_b200.config import TEXT
        c, w = self.cfg, self.w
        b, L, _ = h.shape
        p = f"{TEXT}.layers.{i}"
        y = rms_norm(h, w[f"{p}.input_layernorm.weight"], c.rms_eps)
        q = self._linear(f"{p}.self_attn.q_proj", y).view(b, L, c.heads, c.head_dim)
        k = self._linear(f"{p}.self_attn.k_proj", y).view(b, L, c.kv_heads, c.head_dim)
        v = self._linear(f"{p}.self_attn.v_proj", y)
        q = apply_rope(q, pos, c.rope_wavelength).reshape(b, L, -1)
        k = apply_rope(k, pos, c.rope_wavelength).reshape(b, L, -1)
        ctx = eager_attention(q, k, v, mask, c.heads, c.kv_heads)
        h1 = h + self._linear(f"{p}.self_attn.o_proj", ctx)
        y2 = rms_norm(h1, w[f"{p}.post_attention_layernorm.weight"], c.rms_eps)
        act = F.silu(self._linear(f"{p}.mlp.gate_proj", y2)) * self._linear(f"{p}.mlp.up_proj", y2)
        out = h1 + self._linear(f"{p}.mlp.down_proj", act)
        if taps is not None:
            taps.update(input_norm=y, q=q, k=k, v=v, ctx=ctx, attn_out=h1, post_norm=y2, mlp_act=act, out=out)
        return out, (k, v)

    def prefix_forward(self, prefix, pad, att):
        """VLM layers with KV fill (lerobot forward_attn_layer, fill_kv_cache=True)."""
        from smolvla_mujoco_libero_b200.config import TEXT
        c, w = self.cfg, self.w
        mask = make_att_2d_masks(pad, att)
        pos = torch.cumsum(pad.to(torch.int64), dim=1) - 1
        h = prefix
        cache = []
        for i in range(c.text_layers):
            h, kv = self.text_layer(i, h, mask, pos)
            cache.append(kv)
        prefix_out = rms_norm(h, w[f"{TEXT}.norm.weight"], c.rms_eps)
        return cache, prefix_out, mask, pos

    # -- suffix / expert
    def embed_suffix(self, x_t: torch.Tensor, t: float) -> torch.Tensor:
        c = self.cfg
        a = self.lin["model.action_in_proj"](x_t.to(torch.bfloat16))
        tt = torch.tensor([t], dtype=torch.float32).expand(x_t.shape[0])
        te = sinusoidal_time_embedding(tt, c.expert_hidden, c.min_period, c.max_period).to(a.dtype)
        at = torch.cat([a, te[:, None, :].expand_as(a)], dim=2)
        at = F.silu(self.lin["model.action_time_mlp_in"](at))
        return self.lin["model.action_time_mlp_out"](at)

    def denoise_step(self, cache, pad, x_t: torch.Tensor, t: float) -> torch.Tensor:
        from smolvla_mujoco_libero_b200.config import EXPERT
        c, w = self.cfg, self.w
        h = self.embed_suffix(x_t, t)
        b, S, _ = h.shape
        Lp = pad.shape[1]
        n_valid = pad.to(torch.int64).sum(-1, keepdim=True)
        spos = n_valid + torch.arange(S)[None]
        cpos = torch.arange(S)[None].expand(b, S)
        self_mask = torch.cat([pad[:, None, :].expand(b, S, Lp), torch.tril(torch.ones(S, S, dtype=torch.bool))[None].expand(b, S, S)], dim=2)
        cross_mask = pad[:, None, :].expand(b, S, Lp)
        for i in range(c.expert_layers):
            p = f"{EXPERT}.layers.{i}"
            y = rms_norm(h, w[f"{p}.input_layernorm.weight"], c.rms_eps)
            q = self._linear(f"{p}.self_attn.q_proj", y).view(b, S, c.heads, c.head_dim)
            kp, vp = cache[i]
            if c.is_cross_layer(i):
                q = apply_rope(q, cpos, c.rope_wavelength).reshape(b, S, -1)
                k = self._linear(f"{p}.self_attn.k_proj", kp)
                v = self._linear(f"{p}.self_attn.v_proj", vp)
                ctx = eager_attention(q, k, v, cross_mask, c.heads, c.kv_heads)
            else:
                q = apply_rope(q, spos, c.rope_wavelength).reshape(b, S, -1)
                k = self._linear(f"{p}.self_attn.k_proj", y).view(b, S, c.kv_heads, c.head_dim)
                k = apply_rope(k, spos, c.rope_wavelength).reshape(b, S, -1)
                v = self._linear(f"{p}.self_attn.v_proj", y)
                ctx = eager_attention(q, torch.cat([kp, k], 1), torch.cat([vp, v], 1), self_mask, c.heads, c.kv_heads)
            h = h + self._linear(f"{p}.self_attn.o_proj", ctx)
            y = rms_norm(h, w[f"{p}.post_attention_layernorm.weight"], c.rms_eps)
            h = h + self._mlp(p, y)
        out = rms_norm(h, w[f"{EXPERT}.norm.weight"], c.rms_eps)
        wo = self.lin["model.action_out_proj"]
        self.last_suffix_out = out
        return out.float() @ wo.weight.float().t() + wo.bias.float()

    @torch.no_grad()
    def sample_actions(self, images, img_masks, lang_tokens, lang_masks, state, noise, taps: dict | None = None,
                       image_embs=None):
        """Returns the fp32 chunk [B, chunk, max_action_dim] (callers slice the first action_dim).

        ``taps`` (optional) receives the debug outputs of deploy/diagnose_3_4_numeric_baseline.py:55-70 by the
        same names -- prefix_embs, prefix_out, suffix_out_step_NN (the expert's final-norm output that
        action_out_proj reads), v_t_step_NN, x_t_step_NN -- plus the prefix KV cache as ``kv``."""
        c = self.cfg
        prefix, pad, att = self.embed_prefix(images, img_masks, lang_tokens, lang_masks, state, image_embs)
        cache, prefix_out, _, _ = self.prefix_forward(prefix, pad, att)
        if taps is not None:
            taps["prefix_embs"] = prefix
            taps["prefix_out"] = prefix_out
            taps["kv"] = cache
        dt = -1.0 / c.num_steps
        x_t = noise.to(torch.float32)
        for step in range(c.num_steps):
            t = float(torch.tensor(1.0 + step * dt, dtype=torch.float32))
            v_t = self.denoise_step(cache, pad, x_t, t)
            x_t = x_t + dt * v_t
            if taps is not None:
                taps[f"suffix_out_step_{step:02d}"] = self.last_suffix_out
                taps[f"v_t_step_{step:02d}"] = v_t
                taps[f"x_t_step_{step:02d}"] = x_t
        return x_t


def calibrate(cfg, weights, observations, percentile: float | None = None, alpha: float | None = None):
    """Reference calibration semantics on the bf16 model: per-call per-channel percentile of every W8A8-recipe
    linear input, elementwise max over calls, then SmoothQuant build_entry -> scale JSON dict."""
    from . import quant as Q
    percentile = cfg.percentile if percentile is None else percentile
    alpha = cfg.alpha if alpha is None else alpha
    m = OracleSmolVLA(cfg, weights, mode="bf16")
    col = Q.PerChannelCollector(percentile)
    m.collector = lambda name, x: [col.observe(name, x[i:i + 1]) for i in range(x.shape[0])]
    for obs in observations:
        m.sample_actions(obs.images, obs.img_masks, obs.lang_tokens, obs.lang_masks, obs.state, obs.noise)
    rows = col.rows()
    entries = [Q.build_smoothquant_entry(r, weights[f"{r['module']}.weight"], alpha) for r in rows]
    return {"smoothquant_alpha": alpha, "linear_call_scales": entries}
