"""The quantized SmolVLA sample_actions runner on sm_100a.

``SmolVLARunner`` owns the device weights (int8 SmoothQuant / W8A16 packs made by libsvla's own packing
kernel, bf16 norms / embeddings / small projections), static activation buffers for one batch size, and the
ordered list of C-ABI launches of one ``sample_actions`` call.  Every launch descriptor is built once, so a
call is a flat sequence of ctypes calls; ``capture()`` records that sequence as one CUDA graph, the way the
reference's TensorRTCoreRunner replays a captured engine (deploy/trt_sample_actions_core_deploy.py:108-237).

Call structure (deploy/diagnose_3_4_numeric_baseline.py:148-206 and lerobot 0.5.1 semantics):
  masks / positions -> SigLIP (patch GEMM + 12 x [LN+quant, QKV, attention+quant, out_proj+residual,
  LN+quant, fc1+GELU+quant, fc2+residual]) -> post-LN + pixel shuffle + quant -> connector (x sqrt(960) in
  bf16, rows written into the prefix) | token embedding x sqrt(960) | state_proj -> 16 text layers
  (RMSNorm+quant(q,k,v), QKV GEMM with RoPE writing the KV cache, attention+quant, o_proj+residual,
  RMSNorm+quant(gate,up), gate/up GEMM with SiLU gate, W8A16 down+residual) -> cross-layer K/V projections of
  the cached prefix (step-invariant, computed once) -> 10 x [action_in, time MLP (per-step constant folded
  into the bias), 16 expert layers, final norm, action_out_proj + Euler update].
The last text layer's o_proj and MLP only feed the prefix output that sample_actions never returns, so
they are not launched unless ``debug_taps`` is on (the reference's action-only TensorRT engine drops them too).

mode = "quant": the deployed recipe.  mode = "bf16": every linear in bf16 with the original weights (the
unquantised model) -- used by ``calibrate`` to observe the inputs of every W8A8 linear.
"""

from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch

from . import _lib as L
from . import ops
from .config import CONNECTOR, EXPERT, TEXT, VISION, SmolVLAConfig
from .weights import linear_specs


def _bf(x):
    return x.to(torch.bfloat16)


@dataclass
class PackedLinear:
    n: int
    k: int
    kind: str                           # "w8a8" | "w8a16" | "bf16"
    weight: torch.Tensor                # int8 [n, k] (w8a8 / w8a16) or bf16 [n, k]
    wscale: torch.Tensor | None = None  # fp32 [n]
    bias: torch.Tensor | None = None    # bf16 [n]
    smooth: torch.Tensor | None = None  # fp32 [k] (w8a8)
    rsmooth: torch.Tensor | None = None  # fp32 [k] = 1 / smooth (w8a8), lets the quantisers multiply
    act_scale: float = 1.0              # w8a8
    weight_bf16: torch.Tensor | None = None  # original bf16 weight (bf16 / calibration mode)
    weight_deq: torch.Tensor | None = None   # w8a16: bf16(q * wscale), the weight W8A16Linear multiplies by
    flow_frag: torch.Tensor | None = None    # the fragment-order copy the persistent flow kernel reads (lazy)


def time_embedding_bf16(cfg: SmolVLAConfig) -> torch.Tensor:
    """bf16(sin/cos(2 pi t / period)) for the fixed step times t_k = fp32(1 - k / num_steps), computed in
    float64 as lerobot's create_sinusoidal_pos_embedding does.  A constant of the configuration."""
    dt = -1.0 / cfg.num_steps
    t = torch.tensor([1.0 + k * dt for k in range(cfg.num_steps)], dtype=torch.float32).to(torch.float64)
    frac = torch.linspace(0.0, 1.0, cfg.expert_hidden // 2, dtype=torch.float64)
    period = cfg.min_period * (cfg.max_period / cfg.min_period) ** frac
    sin_in = (1.0 / period * 2 * math.pi)[None, :] * t[:, None]
    return torch.cat([torch.sin(sin_in), torch.cos(sin_in)], dim=1).to(torch.bfloat16)


def _select(entry, in_features):
    if isinstance(entry, list) and entry and isinstance(entry[0], dict):
        for cand in entry:
            sm = cand.get("smooth_scale")
            if isinstance(sm, list) and len(sm) == in_features:
                return cand
        return entry[0]
    return entry


class DeviceWeights:
    """Device weights of the whole path, packed once with libsvla's packing kernel.

    ``scales`` is the module -> entry mapping that load_scale_json returns (the reference's
    load_activation_scales_by_module contract, deploy/linear_only_quant.py:208-246).  A W8A8 module without
    an entry raises, as replace_linear_modules does (deploy/linear_only_quant.py:277-279)."""

    def __init__(self, cfg: SmolVLAConfig, state: dict[str, torch.Tensor], scales: dict | None,
                 device="cuda", keep_bf16: bool = False):
        self.cfg = cfg
        self.device = torch.device(device)
        dev = self.device
        self.lin: dict[str, PackedLinear] = {}
        for name, n, k, has_bias, kind in linear_specs(cfg):
            w = _bf(state[f"{name}.weight"]).to(dev).contiguous()
            b = _bf(state[f"{name}.bias"]).to(dev) if has_bias else None
            if kind == "w8a8" and scales is not None:
                if name not in scales:
                    raise KeyError(f"missing calibrated activation scale for quantized module: {name}")
                e = _select(scales[name], k)
                if not isinstance(e, dict) or "smooth_scale" not in e:
                    raise ValueError(f"{name}: expected a SmoothQuant entry with smooth_scale")
                smooth = torch.tensor(e["smooth_scale"], dtype=torch.float32).clamp_min(1e-8).to(dev)
                if smooth.numel() != k:
                    raise ValueError(f"{name}: smooth_scale has {smooth.numel()} channels, expected {k}")
                q, ws = ops.pack_weight_i8(w, smooth)
                self.lin[name] = PackedLinear(n, k, "w8a8", q, ws, b, smooth, ops.reciprocal(smooth),
                                              max(float(e["scale"]), 1e-8), w if keep_bf16 else None)
            elif kind == "w8a16":
                q, ws = ops.pack_weight_i8(w)
                self.lin[name] = PackedLinear(n, k, "w8a16", q, ws, b, weight_bf16=w if keep_bf16 else None,
                                              weight_deq=ops.dequant_weight_bf16(q, ws))
            else:
                self.lin[name] = PackedLinear(n, k, "bf16", w, None, b, weight_bf16=w)
        self.t: dict[str, torch.Tensor] = {}
        for key, val in state.items():
            if key.rsplit(".", 1)[0] in self.lin:
                continue
            self.t[key] = _bf(val).to(dev).contiguous()
        pw = self.t[f"{VISION}.embeddings.patch_embedding.weight"]
        self.t["patch_w2d"] = pw.reshape(pw.shape[0], -1).contiguous()
        self.quantized = scales is not None
        torch.cuda.synchronize(dev)

    def nbytes(self) -> int:
        tot = 0
        for p in self.lin.values():
            for t in (p.weight, p.wscale, p.bias, p.smooth, p.weight_deq, p.flow_frag):
                if t is not None:
                    tot += t.numel() * t.element_size()
        return tot + sum(t.numel() * t.element_size() for t in self.t.values())


class SmolVLARunner:
    """Static buffers + launch list for one batch size."""

    W8A16_BF16_ROWS = 1  # M from which W8A16 linears run as bf16 GEMMs on the dequantized weight (all M:
    # measured faster than converting the int8 weight inside every tile, at M = 50 as at M = 3200)
    SPLITK_BYTES = 32 << 20  # split-K workspace shared by the runner's GEMMs (stream-ordered)

    def __init__(self, weights: DeviceWeights, batch: int, mode: str = "quant", debug_taps: bool = False,
                 split_k: bool = True, prefix_only: bool = False, flow: bool | None = None,
                 image_embeds: bool = False):
        if weights.cfg.expert_layers != weights.cfg.text_layers:
            raise ValueError("the expert must have one layer per text layer (each expert layer reads that layer's KV)")
        if mode == "quant" and not weights.quantized:
            raise ValueError("quant mode needs weights packed with a scale table")
        if mode == "bf16":
            for p in weights.lin.values():
                if p.weight_bf16 is None:
                    raise ValueError("bf16 mode needs DeviceWeights(..., keep_bf16=True)")
        self.w, self.cfg, self.B, self.mode, self.debug = weights, weights.cfg, batch, mode, debug_taps
        # prefix_only: stop after the prefix prefill, with the final-layer prefix hidden states in prefix_out
        # (the RL-token features, smollvla_rltoken/rlt/rl_token.py:50-88) and the KV cache filled
        self.prefix_only = prefix_only
        # image_embeds: the embeds mode of the exported core (deploy/export_smolvla_sample_actions_onnx.py:64-164):
        # the call takes one bf16 [B, n_img_tokens, hidden] image embedding per camera instead of the images,
        # and the vision tower and connector are not run
        self.image_embeds = image_embeds
        # split-K changes the fp32 summation order of the small-M bf16 GEMMs with the batch size; without it
        # every batch row's result is bit-identical at any batch size
        self.split_k = split_k
        # flow: the flow-matching loop as one persistent kernel (svla_flow) instead of ~117 launches per step;
        # None = when it applies (quant mode, batch * chunk <= 64 rows, no taps)
        can_flow = self._flow_supported(weights.cfg, batch, mode, debug_taps)
        if flow and not can_flow:
            raise ValueError("the persistent flow kernel needs quant mode, batch * chunk <= 64, no taps and "
                             "W8A16 expert linears")
        self.flow = can_flow if flow is None else bool(flow)
        self.dev = weights.device
        self.graph: torch.cuda.CUDAGraph | None = None
        self.taps: dict[str, list] = {}
        self._alloc()
        self._constants()
        self.launches: list = []
        self._build()

    def _flow_supported(self, c: SmolVLAConfig, batch: int, mode: str, debug: bool) -> bool:
        if mode != "quant" or debug or batch * c.chunk > L.FLOW_MAX_ROWS or c.expert_layers > L.FLOW_MAX_LAYERS:
            return False
        if c.expert_hidden % 16 or c.expert_hidden > 1024 or c.max_action_dim % 16 or c.expert_mlp % 16:
            return False
        expert = [p for n, p in self.w.lin.items() if n.startswith(EXPERT + ".")]
        return all(p.kind == "w8a16" for p in expert)

    # ------------------------------------------------------------------ buffers
    def _alloc(self):
        c, B, d = self.cfg, self.B, self.dev
        bf, i8, f32 = torch.bfloat16, torch.int8, torch.float32
        Lp, S = c.prefix_len, c.chunk
        NI = B * c.n_cams
        NV = 0 if self.image_embeds else NI * c.n_patches  # the vision tower's rows (none in embeds mode)
        z = lambda *s, dt=bf: torch.zeros(*s, dtype=dt, device=d)  # noqa: E731
        self.splitk_ws = ops.splitk_workspace(self.SPLITK_BYTES, d)
        if self.image_embeds:
            n_emb = c.n_cams * c.n_img_tokens
            self.in_emb = z(B, n_emb, c.hidden)
            # row b * n_emb + j of in_emb, viewed as a table, is image token j of sample b
            self.emb_rows = torch.arange(B * n_emb, dtype=torch.int64, device=d).view(B, n_emb)
            self.in_img = z(1, dt=f32)
        else:
            self.in_img = z(B, c.n_cams, c.channels, c.image_size, c.image_size, dt=f32)
        self.in_img_mask = z(c.n_cams, B, dt=torch.uint8)
        self.in_tokens = torch.zeros(B, c.n_lang, dtype=torch.int64, device=d)
        self.in_lang_mask = z(B, c.n_lang, dt=torch.uint8)
        self.in_state = z(B, c.max_state_dim, dt=f32)
        self.in_noise = z(B, S, c.max_action_dim, dt=f32)
        self.state_bf = z(B, c.max_state_dim)
        # mask rows are stored at 16-byte strides (the layout svla_build_masks writes); the views cover L keys
        ld = lambda n: (n + 15) // 16 * 16  # noqa: E731
        self.prefix_mask = z(B, Lp, ld(Lp), dt=torch.uint8)[:, :, :Lp]
        self.self_mask = z(B, S, ld(Lp + S), dt=torch.uint8)[:, :, :Lp + S]
        self.cross_mask = z(B, S, ld(Lp), dt=torch.uint8)[:, :, :Lp]
        # the prefix key padding (a row of the cross mask): the expert's self and cross attention use it in
        # the structured form (key padding over the prefix, causal over the chunk), the same masks as
        # self_mask / cross_mask with one row of flags per sample instead of one per query
        self.key_pad = self.cross_mask[:, 0, :]
        self.prefix_pos = z(B * Lp, dt=torch.int32)
        self.suffix_pos = z(B * S, dt=torch.int32)
        self.cross_pos = z(B * S, dt=torch.int32)
        H, Hv = c.hidden, c.vis_hidden
        q = self.mode == "quant"
        if not self.image_embeds:
            self.patches = z(NV, c.channels * c.patch * c.patch)
            self.vh = z(NV, Hv)
            self.v_in = [z(NV, Hv, dt=i8 if q else bf) for _ in range(3)]   # LN1 -> q/k/v inputs
            self.v_qkv = [z(NV, Hv) for _ in range(3)]
            self.v_ctx = z(NV, Hv, dt=i8 if q else bf)
            self.v_fc1_in = z(NV, Hv, dt=i8 if q else bf)
            self.v_fc2_in = z(NV, c.vis_mlp, dt=i8 if q else bf)
            self.conn_in = z(NI * c.n_img_tokens, Hv * c.scale_factor ** 2, dt=i8 if q else bf)
        self.h = z(B * Lp, H)
        self.t_in = [z(B * Lp, H, dt=i8 if q else bf) for _ in range(3)]
        self.t_q = z(B * Lp, c.q_dim)
        self.kcache = [z(B * Lp, c.kv_dim) for _ in range(c.text_layers)]
        self.vcache = [z(B * Lp, c.kv_dim) for _ in range(c.text_layers)]
        self.t_ctx = z(B * Lp, c.q_dim, dt=i8 if q else bf)
        self.t_mlp_in = [z(B * Lp, H, dt=i8 if q else bf) for _ in range(2)]
        self.t_mlp = z(B * Lp, c.mlp)
        E = c.expert_hidden
        self.ck = {i: z(B * Lp, c.kv_dim) for i in range(c.expert_layers) if c.is_cross_layer(i)}
        self.cv = {i: z(B * Lp, c.kv_dim) for i in range(c.expert_layers) if c.is_cross_layer(i)}
        self.xt = z(B * S, c.max_action_dim, dt=f32)
        self.xt_bf = z(B * S, c.max_action_dim)
        self.a_emb = z(B * S, E)
        self.a_t = z(B * S, E)
        self.eh = z(B * S, E)
        self.ey = z(B * S, E)
        self.eq = z(B * S, c.q_dim)
        self.ek = z(B * S, c.kv_dim)
        self.ev = z(B * S, c.kv_dim)
        self.ectx = z(B * S, c.q_dim)
        self.emlp = z(B * S, c.expert_mlp)
        if self.debug or self.prefix_only:
            self.prefix_out = z(B * Lp, H)
        if self.debug:
            # debug-only outputs that the deployed launches fuse away: the normalised rows in front of the
            # quantisers, the bf16 attention context beside its int8 copy, and v_t before the Euler update
            self.dbg_norm = z(max(NV, B * Lp, B * S), max(Hv, H, E))
            self.dbg_ctx = z(max(NV, B * Lp), max(Hv, c.q_dim))
            self.dbg_fc2 = z(NV, c.vis_mlp) if NV else None
            self.v_t = z(B * S, c.max_action_dim, dt=f32)

    def _constants(self):
        c = self.cfg
        self.max_pos = c.prefix_len + c.chunk
        self.rope_cs = ops.rope_table(self.max_pos, c.rope_wavelength, self.dev)
        # per-step constant of action_time_mlp_in: W[:, E:] . bf16(time_emb(t_k)) + b   (fp32)
        E = c.expert_hidden
        te = time_embedding_bf16(c).to(self.dev)
        mi = self.w.lin["model.action_time_mlp_in"]
        self.c_step = torch.empty(c.num_steps, E, dtype=torch.float32, device=self.dev)
        wt = mi.weight[:, E:]
        d = ops.gemm_desc(L.KIND_BF16, L.EPI_F32, c.num_steps, E,
                          [ops.Seg(a=te, b=wt, out=self.c_step, n=E, bias=mi.bias, ldb=mi.weight.stride(0))])
        ops.gemm(d)

    # ------------------------------------------------------------------ launch helpers
    def _add(self, fn, *args):
        self.launches.append((fn, args))

    def _tap(self, mods, buf):
        """A point in the launch list where ``buf`` holds the input of ``mods`` (bf16 mode / debug taps);
        the observer passed to run() sees it in stream order, before later launches reuse the buffer."""
        self.launches.append((_TAP, (list(mods), buf)))

    def _gemm(self, kind, epi, m, k, segs, **kw):
        # every B operand here is a packed weight, written when the model was built; GEMMs with few output
        # tiles split K over the SMs through the runner's split-K workspace
        ws = dict(workspace=self.splitk_ws, workspace_bytes=self.splitk_ws.numel()) if self.split_k else {}
        d = ops.gemm_desc(kind, epi, m, k, segs, weights_resident=1, **ws, **kw)
        self._keep.append(segs)
        self._add(L.lib().svla_gemm, d)

    def _deq_rows(self, p: PackedLinear, m: int) -> bool:
        """W8A16 linears with at least W8A16_BF16_ROWS rows multiply by the stored bf16(q * wscale) weight
        (a plain bf16 GEMM; the reference's W8A16Linear keeps exactly that buffer) instead of converting
        the int8 weight inside every output tile: the same operands, so the same results, and the per-tile
        conversion costs more than the weight bytes it saves."""
        return p.kind == "w8a16" and m >= self.W8A16_BF16_ROWS

    def _linear_seg(self, name: str, a: torch.Tensor, out, rope=0, n=None):
        p = self.w.lin[name]
        if self.mode == "bf16" or p.kind == "bf16":
            return ops.Seg(a=a, b=p.weight_bf16, out=out, n=p.n if n is None else n, bias=p.bias, rope=rope)
        if self._deq_rows(p, a.shape[0]):
            return ops.Seg(a=a, b=p.weight_deq, out=out, n=p.n, bias=p.bias, rope=rope)
        if p.kind == "w8a16":
            return ops.Seg(a=a, b=p.weight, out=out, n=p.n, wscale=p.wscale, bias=p.bias, rope=rope)
        return ops.Seg(a=a, b=p.weight, out=out, n=p.n, wscale=p.wscale, bias=p.bias, act_scale=p.act_scale, rope=rope)

    def _kind(self, name: str, m: int) -> int:
        p = self.w.lin[name]
        if self.mode == "bf16" or p.kind == "bf16" or self._deq_rows(p, m):
            return L.KIND_BF16
        return L.KIND_I8 if p.kind == "w8a8" else L.KIND_W8A16

    def _norm(self, x, weight, eps, bias=None, quant_mods=(), outs=None, y=None, pixel_shuffle=0, ps_grid=0,
              tap=None):
        """RMSNorm/LayerNorm + per-projection quantisation (quant mode) or bf16 output (bf16 mode)."""
        d = L.NormDesc()
        m, k = x.shape
        d.x, d.ldx, d.weight, d.bias, d.eps = x.data_ptr(), x.stride(0), weight.data_ptr(), \
            (bias.data_ptr() if bias is not None else None), float(eps)
        d.layernorm, d.m, d.k = int(bias is not None), m, k
        d.pixel_shuffle, d.ps_grid = pixel_shuffle, ps_grid
        quant = self.mode == "quant" and bool(quant_mods)
        if quant:
            for i, (mod, q) in enumerate(zip(quant_mods, outs)):
                p = self.w.lin[mod]
                d.q[i], d.smooth[i], d.act[i] = q.data_ptr(), p.smooth.data_ptr(), p.act_scale
                d.rsmooth[i] = p.rsmooth.data_ptr()
            d.nq, d.ldq = len(quant_mods), outs[0].stride(0)
            if y is None and self.debug and not pixel_shuffle:
                y = self.dbg_norm[:m, :k]  # debug: keep the bf16 rows the quantisers read
            if y is not None:
                d.y, d.ldy = y.data_ptr(), y.stride(0)
            target = y
        else:
            target = y if y is not None else outs[0]
            d.y, d.ldy = target.data_ptr(), target.stride(0)
        self._add(L.lib().svla_norm_quant, d)
        if tap is not None and target is not None and (not quant or self.debug):
            self._tap(tap, target)
        if quant and self.debug:
            for mod, q in zip(quant_mods, outs):
                self._tap([f"{mod}#int8"], q)

    def _attn(self, q, k1, v1, lq, hq, hkv, mask=None, k2=None, v2=None, out_mod=None, out=None, tap=None,
              key_mask=None, mask_keys=0):
        """attention; in quant mode with out_mod the context is quantised for that W8A8 linear.
        The batch is the number of sequences in q (images for the vision tower, samples otherwise)."""
        B = q.shape[0] // lq
        qv = q.view(B, lq, -1)
        l1 = k1.shape[0] // B
        k1v, v1v = k1.view(B, l1, -1), v1.view(B, l1, -1)
        k2v = v2v = None
        if k2 is not None:
            l2 = k2.shape[0] // B
            k2v, v2v = k2.view(B, l2, -1), v2.view(B, l2, -1)
        ov = out.view(B, lq, -1)
        quant = self.mode == "quant" and out_mod is not None
        if quant:
            p = self.w.lin[out_mod]
            # debug: the bf16 context beside the int8 one the next linear reads
            dbg = self.dbg_ctx[:q.shape[0], :q.shape[1]] if self.debug else None
            d = ops.attention_desc(qv, k1v, v1v, B, lq, hq, hkv, mask=mask, k2=k2v, v2=v2v, qo=ov,
                                   o=None if dbg is None else dbg.view(B, lq, -1),
                                   qo_smooth=p.smooth, qo_act=p.act_scale, qo_rsmooth=p.rsmooth,
                                   key_mask=key_mask, mask_keys=mask_keys)
        else:
            d = ops.attention_desc(qv, k1v, v1v, B, lq, hq, hkv, mask=mask, k2=k2v, v2=v2v, o=ov,
                                   key_mask=key_mask, mask_keys=mask_keys)
        self._add(L.lib().svla_attention, d)
        if tap is not None and not quant:
            self._tap(tap, out)
        elif tap is not None and self.debug:
            self._tap(tap, dbg)
            self._tap([f"{out_mod}#int8"], out)

    # ------------------------------------------------------------------ the call
    def _build(self):
        c, B, w = self.cfg, self.B, self.w
        lib = L.lib()
        self._keep = []
        Lp, S, H = c.prefix_len, c.chunk, c.hidden
        # masks and positions
        self._add(lib.svla_build_masks, self.in_img_mask[0].data_ptr(), self.in_img_mask[1].data_ptr()
                  if c.n_cams > 1 else self.in_img_mask[0].data_ptr(), self.in_lang_mask.data_ptr(), B,
                  c.n_img_tokens, c.n_lang, S, self.prefix_mask.data_ptr(), self.prefix_pos.data_ptr(),
                  self.self_mask.data_ptr(), self.cross_mask.data_ptr(), self.suffix_pos.data_ptr(),
                  self.cross_pos.data_ptr())
        if self.image_embeds:
            self._build_embeds_prefix()
        else:
            self._build_vision()
        # language tokens x sqrt(H) and the state token
        self._add(lib.svla_embed_tokens, self.in_tokens.data_ptr(), B, c.n_lang, w.t[f"{TEXT}.embed_tokens.weight"].data_ptr(),
                  c.vocab, H, float(math.sqrt(H)), self.h.data_ptr(), Lp, c.n_cams * c.n_img_tokens)
        self._add(lib.svla_f32_to_bf16, self.in_state.data_ptr(), self.state_bf.data_ptr(), self.in_state.numel())
        self._gemm(L.KIND_BF16, L.EPI_BF16, B, c.max_state_dim,
                   [self._linear_seg("model.state_proj", self.state_bf, self.h)], rows_per_group=1,
                   group_stride=Lp, row_offset=Lp - 1)
        if self.debug:
            self._tap(["prefix_embs"], self.h)
        self._build_text_and_expert()

    def _build_embeds_prefix(self):
        """Embeds mode: image token rows (b, cam, t) of the prefix = bf16(emb * bf16(sqrt(H))), the scaling of
        embed_prefix_from_image_embeds (deploy/export_smolvla_sample_actions_onnx.py:87-94)."""
        c, B = self.cfg, self.B
        n_emb = c.n_cams * c.n_img_tokens
        img_scale = float(torch.tensor(c.hidden ** 0.5, dtype=torch.bfloat16))
        self._add(L.lib().svla_embed_tokens, self.emb_rows.data_ptr(), B, n_emb, self.in_emb.data_ptr(), B * n_emb,
                  c.hidden, img_scale, self.h.data_ptr(), c.prefix_len, 0)

    def _build_vision(self):
        """SigLIP + post-LN + pixel shuffle + connector, writing the image token rows of the prefix."""
        c, B, w = self.cfg, self.B, self.w
        lib = L.lib()
        q_mode = self.mode == "quant"
        Lp, H = c.prefix_len, c.hidden
        NI = B * c.n_cams
        NV = NI * c.n_patches
        # ---------------- vision tower
        self._add(lib.svla_im2col, self.in_img.data_ptr(), NI, c.channels, c.image_size, c.patch,
                  self.patches.data_ptr())
        pe = f"{VISION}.embeddings"
        self._gemm(L.KIND_BF16, L.EPI_RESID, NV, self.patches.shape[1],
                   [ops.Seg(a=self.patches, b=w.t["patch_w2d"], out=self.vh, n=c.vis_hidden,
                            bias=w.t[f"{pe}.patch_embedding.bias"])],
                   resid=w.t[f"{pe}.position_embedding.weight"], ldr=c.vis_hidden, resid_rows=c.n_patches)
        for i in range(c.vis_layers):
            p = f"{VISION}.encoder.layers.{i}"
            mods = [f"{p}.self_attn.{n}" for n in ("q_proj", "k_proj", "v_proj")]
            self._norm(self.vh, w.t[f"{p}.layer_norm1.weight"], c.vis_eps, bias=w.t[f"{p}.layer_norm1.bias"],
                       quant_mods=mods, outs=self.v_in, tap=mods)
            a_in = self.v_in if q_mode else [self.v_in[0]] * 3
            self._gemm(self._kind(mods[0], NV), L.EPI_BF16, NV, c.vis_hidden,
                       [self._linear_seg(m, a, o) for m, a, o in zip(mods, a_in, self.v_qkv)])
            self._attn(self.v_qkv[0], self.v_qkv[1], self.v_qkv[2], c.n_patches, c.vis_heads, c.vis_heads,
                       out_mod=f"{p}.self_attn.out_proj", out=self.v_ctx, tap=[f"{p}.self_attn.out_proj"])
            self._gemm(self._kind(f"{p}.self_attn.out_proj", NV), L.EPI_RESID, NV, c.vis_hidden,
                       [self._linear_seg(f"{p}.self_attn.out_proj", self.v_ctx, self.vh)], resid=self.vh,
                       ldr=c.vis_hidden)
            self._norm(self.vh, w.t[f"{p}.layer_norm2.weight"], c.vis_eps, bias=w.t[f"{p}.layer_norm2.bias"],
                       quant_mods=[f"{p}.mlp.fc1"], outs=[self.v_fc1_in], tap=[f"{p}.mlp.fc1"])
            fc2 = w.lin[f"{p}.mlp.fc2"]
            if q_mode:
                gelu_bf16 = self.dbg_fc2 if self.debug else None  # debug: the bf16 GELU output beside the int8 one
                self._gemm(L.KIND_I8, L.EPI_GELU_QUANT, NV, c.vis_hidden,
                           [self._linear_seg(f"{p}.mlp.fc1", self.v_fc1_in, gelu_bf16)],
                           q_smooth=fc2.smooth, q_rsmooth=fc2.rsmooth, q_act=fc2.act_scale, qout=self.v_fc2_in,
                           ldq=c.vis_mlp)
                if self.debug:
                    self._tap([f"{p}.mlp.fc2"], gelu_bf16)
                    self._tap([f"{p}.mlp.fc2#int8"], self.v_fc2_in)
            else:
                self._gemm(L.KIND_BF16, L.EPI_GELU_QUANT, NV, c.vis_hidden,
                           [self._linear_seg(f"{p}.mlp.fc1", self.v_fc1_in, self.v_fc2_in)])
                self._tap([f"{p}.mlp.fc2"], self.v_fc2_in)
            self._gemm(self._kind(f"{p}.mlp.fc2", NV), L.EPI_RESID, NV, c.vis_mlp,
                       [self._linear_seg(f"{p}.mlp.fc2", self.v_fc2_in, self.vh)], resid=self.vh, ldr=c.vis_hidden)
        # post LayerNorm + pixel shuffle + connector quantisation
        self._norm(self.vh, w.t[f"{VISION}.post_layernorm.weight"], c.vis_eps, bias=w.t[f"{VISION}.post_layernorm.bias"],
                   quant_mods=[CONNECTOR], outs=[self.conn_in], pixel_shuffle=c.scale_factor, ps_grid=c.grid,
                   tap=[CONNECTOR])
        # connector -> prefix rows (b, cam, token) -> b*Lp + cam*n_img + token, x bf16(sqrt(H)) in bf16
        img_scale = float(torch.tensor(H ** 0.5, dtype=torch.bfloat16))
        self._gemm(self._kind(CONNECTOR, NI * c.n_img_tokens), L.EPI_BF16, NI * c.n_img_tokens, self.conn_in.shape[1],
                   [self._linear_seg(CONNECTOR, self.conn_in, self.h)], post_scale=img_scale,
                   rows_per_group=c.n_cams * c.n_img_tokens, group_stride=Lp)

    def _build_text_and_expert(self):
        c, B, w = self.cfg, self.B, self.w
        lib = L.lib()
        q_mode = self.mode == "quant"
        Lp, S, H, E = c.prefix_len, c.chunk, c.hidden, c.expert_hidden
        # ---------------- text layers (KV fill)
        for i in range(c.text_layers):
            p = f"{TEXT}.layers.{i}"
            mods = [f"{p}.self_attn.{n}" for n in ("q_proj", "k_proj", "v_proj")]
            self._norm(self.h, w.t[f"{p}.input_layernorm.weight"], c.rms_eps, quant_mods=mods, outs=self.t_in, tap=mods)
            a_in = self.t_in if q_mode else [self.t_in[0]] * 3
            outs = [self.t_q, self.kcache[i], self.vcache[i]]
            self._gemm(self._kind(mods[0], B * Lp), L.EPI_ROPE, B * Lp, H,
                       [self._linear_seg(m, a, o, rope=r) for m, a, o, r in zip(mods, a_in, outs, (1, 1, 0))],
                       rope_cs=self.rope_cs, pos=self.prefix_pos, max_pos=self.max_pos)
            if self.debug:  # post-RoPE q / k and v: k and v are also this layer's KV cache
                for name, buf in zip(("q_rope", "k_rope", "v"), outs):
                    self._tap([f"{p}.self_attn.{name}"], buf)
            last = i == c.text_layers - 1
            if last and not (self.debug or self.prefix_only) and self.mode == "quant":
                break
            self._attn(self.t_q, self.kcache[i], self.vcache[i], Lp, c.heads, c.kv_heads, mask=self.prefix_mask,
                       out_mod=f"{p}.self_attn.o_proj", out=self.t_ctx, tap=[f"{p}.self_attn.o_proj"])
            self._gemm(self._kind(f"{p}.self_attn.o_proj", B * Lp), L.EPI_RESID, B * Lp, c.q_dim,
                       [self._linear_seg(f"{p}.self_attn.o_proj", self.t_ctx, self.h)], resid=self.h, ldr=H)
            if self.debug:
                self._tap([f"{p}.attn_residual"], self.h)
            mods = [f"{p}.mlp.gate_proj", f"{p}.mlp.up_proj"]
            self._norm(self.h, w.t[f"{p}.post_attention_layernorm.weight"], c.rms_eps, quant_mods=mods,
                       outs=self.t_mlp_in, tap=mods)
            a_in = self.t_mlp_in if q_mode else [self.t_mlp_in[0]] * 2
            self._gemm(self._kind(mods[0], B * Lp), L.EPI_SILU_MUL, B * Lp, H,
                       [self._linear_seg(m, a, self.t_mlp) for m, a in zip(mods, a_in)], pair=True)
            if self.debug:
                self._tap([f"{p}.mlp.down_proj"], self.t_mlp)
            self._gemm(self._kind(f"{p}.mlp.down_proj", B * Lp), L.EPI_RESID, B * Lp, c.mlp,
                       [self._linear_seg(f"{p}.mlp.down_proj", self.t_mlp, self.h)], resid=self.h, ldr=H)
            if self.debug:
                self._tap([f"{p}.output"], self.h)
        if self.debug or self.prefix_only:
            self._norm(self.h, w.t[f"{TEXT}.norm.weight"], c.rms_eps, y=self.prefix_out)
            if self.debug:
                self._tap(["prefix_out"], self.prefix_out)
        if self.prefix_only:
            return
        # ---------------- cross-attention K/V of the cached prefix (step-invariant)
        for i in self.ck:
            p = f"{EXPERT}.layers.{i}.self_attn"
            self._gemm(self._kind(f"{p}.k_proj", B * Lp), L.EPI_BF16, B * Lp, c.kv_dim,
                       [self._linear_seg(f"{p}.k_proj", self.kcache[i], self.ck[i]),
                        self._linear_seg(f"{p}.v_proj", self.vcache[i], self.cv[i])])
        # ---------------- flow matching
        if self.flow:
            self._add(lib.svla_flow, self._flow_desc())
            return
        self._add(lib.svla_euler_init, self.in_noise.data_ptr(), self.xt.data_ptr(), self.xt_bf.data_ptr(),
                  self.xt.numel())
        dt = -1.0 / c.num_steps
        mi, mo = w.lin["model.action_time_mlp_in"], w.lin["model.action_time_mlp_out"]
        for step in range(c.num_steps):
            self._gemm(L.KIND_BF16, L.EPI_BF16, B * S, c.max_action_dim,
                       [self._linear_seg("model.action_in_proj", self.xt_bf, self.a_emb)])
            self._gemm(L.KIND_BF16, L.EPI_SILU, B * S, E,
                       [ops.Seg(a=self.a_emb, b=mi.weight[:, :E], ldb=mi.weight.stride(0), out=self.a_t, n=E,
                                bias_f32=self.c_step[step])])
            self._gemm(L.KIND_BF16, L.EPI_BF16, B * S, E, [self._linear_seg("model.action_time_mlp_out", self.a_t, self.eh)])
            for i in range(c.expert_layers):
                p = f"{EXPERT}.layers.{i}"
                self._norm(self.eh, w.t[f"{p}.input_layernorm.weight"], c.rms_eps, y=self.ey)
                kq = self._kind(f"{p}.self_attn.q_proj", B * S)
                if c.is_cross_layer(i):
                    self._gemm(kq, L.EPI_ROPE, B * S, E, [self._linear_seg(f"{p}.self_attn.q_proj", self.ey, self.eq, rope=1)],
                               rope_cs=self.rope_cs, pos=self.cross_pos, max_pos=self.max_pos)
                    self._attn(self.eq, self.ck[i], self.cv[i], S, c.heads, c.kv_heads, out=self.ectx,
                               key_mask=self.key_pad, mask_keys=Lp)
                else:
                    segs = [self._linear_seg(f"{p}.self_attn.q_proj", self.ey, self.eq, rope=1),
                            self._linear_seg(f"{p}.self_attn.k_proj", self.ey, self.ek, rope=1),
                            self._linear_seg(f"{p}.self_attn.v_proj", self.ey, self.ev, rope=0)]
                    self._gemm(kq, L.EPI_ROPE, B * S, E, segs, rope_cs=self.rope_cs, pos=self.suffix_pos,
                               max_pos=self.max_pos)
                    self._attn(self.eq, self.kcache[i], self.vcache[i], S, c.heads, c.kv_heads, key_mask=self.key_pad, mask_keys=Lp,
                               k2=self.ek, v2=self.ev, out=self.ectx)
                self._gemm(self._kind(f"{p}.self_attn.o_proj", B * S), L.EPI_RESID, B * S, c.q_dim,
                           [self._linear_seg(f"{p}.self_attn.o_proj", self.ectx, self.eh)], resid=self.eh, ldr=E)
                self._norm(self.eh, w.t[f"{p}.post_attention_layernorm.weight"], c.rms_eps, y=self.ey)
                self._gemm(self._kind(f"{p}.mlp.gate_proj", B * S), L.EPI_SILU_MUL, B * S, E,
                           [self._linear_seg(f"{p}.mlp.gate_proj", self.ey, self.emlp),
                            self._linear_seg(f"{p}.mlp.up_proj", self.ey, self.emlp)], pair=True)
                self._gemm(self._kind(f"{p}.mlp.down_proj", B * S), L.EPI_RESID, B * S, c.expert_mlp,
                           [self._linear_seg(f"{p}.mlp.down_proj", self.emlp, self.eh)], resid=self.eh, ldr=E)
            self._norm(self.eh, w.t[f"{EXPERT}.norm.weight"], c.rms_eps, y=self.ey)
            if self.debug:
                # the reference's debug outputs (deploy/diagnose_3_4_numeric_baseline.py:55-70): suffix_out
                # (what action_out_proj reads), v_t from the same GEMM in fp32, x_t after the Euler update
                self._tap([f"suffix_out_step_{step:02d}"], self.ey)
                self._gemm(L.KIND_BF16, L.EPI_F32, B * S, E,
                           [self._linear_seg("model.action_out_proj", self.ey, self.v_t)])
                self._tap([f"v_t_step_{step:02d}"], self.v_t)
            self._gemm(L.KIND_BF16, L.EPI_EULER, B * S, E,
                       [self._linear_seg("model.action_out_proj", self.ey, None)], dt=dt, xt=self.xt,
                       xt_bf16=self.xt_bf)
            if self.debug:
                self._tap([f"x_t_step_{step:02d}"], self.xt)

    def _flow_desc(self) -> L.FlowDesc:
        """Descriptor of the persistent flow kernel over this runner's buffers."""
        c, B, w = self.cfg, self.B, self.w
        E = c.expert_hidden

        def wt(name, cols=None):  # fragment-order copy of the weight (int8 for W8A16, else bf16), made once
            p = w.lin[name]
            if p.flow_frag is None:
                p.flow_frag = ops.flow_pack_weight(p.weight if cols is None else p.weight[:, :cols])
            return p.flow_frag.data_ptr()

        def ws(name):
            return w.lin[name].wscale.data_ptr()

        d = L.FlowDesc()
        d.batch, d.chunk, d.prefix_len, d.hidden, d.action_dim = B, c.chunk, c.prefix_len, E, c.max_action_dim
        d.heads, d.kv_heads, d.mlp, d.n_layers, d.num_steps = c.heads, c.kv_heads, c.expert_mlp, c.expert_layers, c.num_steps
        d.eps = float(c.rms_eps)
        d.noise, d.xt, d.xt_bf16 = self.in_noise.data_ptr(), self.xt.data_ptr(), self.xt_bf.data_ptr()
        d.w_action_in, d.b_action_in = wt("model.action_in_proj"), w.lin["model.action_in_proj"].bias.data_ptr()
        mi = w.lin["model.action_time_mlp_in"]
        d.w_time_in, d.time_in_const = wt("model.action_time_mlp_in", cols=E), self.c_step.data_ptr()
        d.w_time_out, d.b_time_out = wt("model.action_time_mlp_out"), w.lin["model.action_time_mlp_out"].bias.data_ptr()
        d.final_norm = w.t[f"{EXPERT}.norm.weight"].data_ptr()
        d.w_action_out, d.b_action_out = wt("model.action_out_proj"), w.lin["model.action_out_proj"].bias.data_ptr()
        d.key_mask, d.key_mask_bs = self.key_pad.data_ptr(), self.key_pad.stride(0)
        d.suffix_pos, d.cross_pos = self.suffix_pos.data_ptr(), self.cross_pos.data_ptr()
        d.rope_cs, d.max_pos = self.rope_cs.data_ptr(), self.max_pos
        d.a_emb, d.a_t, d.eh, d.eq = self.a_emb.data_ptr(), self.a_t.data_ptr(), self.eh.data_ptr(), self.eq.data_ptr()
        d.ek, d.ev, d.ectx, d.emlp = self.ek.data_ptr(), self.ev.data_ptr(), self.ectx.data_ptr(), self.emlp.data_ptr()
        self.flow_norm = torch.zeros(64 * 64, dtype=torch.float32, device=self.dev)
        d.norm_part = self.flow_norm.data_ptr()
        self.flow_sync = torch.zeros(2, dtype=torch.int32, device=self.dev)
        d.sync = self.flow_sync.data_ptr()
        for i in range(c.expert_layers):
            p = f"{EXPERT}.layers.{i}"
            ly = d.layer[i]
            ly.input_norm = w.t[f"{p}.input_layernorm.weight"].data_ptr()
            ly.post_norm = w.t[f"{p}.post_attention_layernorm.weight"].data_ptr()
            ly.wq, ly.sq = wt(f"{p}.self_attn.q_proj"), ws(f"{p}.self_attn.q_proj")
            ly.wo, ly.so = wt(f"{p}.self_attn.o_proj"), ws(f"{p}.self_attn.o_proj")
            ly.wg, ly.sg = wt(f"{p}.mlp.gate_proj"), ws(f"{p}.mlp.gate_proj")
            ly.wu, ly.su = wt(f"{p}.mlp.up_proj"), ws(f"{p}.mlp.up_proj")
            ly.wd, ly.sd = wt(f"{p}.mlp.down_proj"), ws(f"{p}.mlp.down_proj")
            ly.cross = int(c.is_cross_layer(i))
            if ly.cross:
                ly.keys, ly.values = self.ck[i].data_ptr(), self.cv[i].data_ptr()
            else:
                ly.wk, ly.sk = wt(f"{p}.self_attn.k_proj"), ws(f"{p}.self_attn.k_proj")
                ly.wv, ly.sv = wt(f"{p}.self_attn.v_proj"), ws(f"{p}.self_attn.v_proj")
                ly.keys, ly.values = self.kcache[i].data_ptr(), self.vcache[i].data_ptr()
        return d

    # ------------------------------------------------------------------ execution
    @property
    def n_launches(self) -> int:
        """Kernel launches per call (taps are not launches)."""
        return sum(1 for fn, _ in self.launches if fn is not _TAP)

    def _run_launches(self, observer=None):
        stream = torch.cuda.current_stream(self.dev).cuda_stream
        for fn, args in self.launches:
            if fn is _TAP:
                if observer is not None:
                    observer(*args)
                continue
            if isinstance(args[0], ctypes_structs):
                rc = fn(ctypes_byref(args[0]), stream)
            else:
                rc = fn(*args, stream)
            if rc != 0:
                L.check(rc, getattr(fn, "__name__", "svla"))

    def load_inputs(self, images, img_masks, lang_tokens, lang_masks, state, noise):
        """Copy one call's inputs into the static buffers (stream-ordered, no host sync).  In embeds mode
        ``images`` holds one bf16 [B, n_img_tokens, hidden] image embedding per camera."""
        c, B = self.cfg, self.B
        if state.shape[0] != B:
            raise ValueError(f"runner built for batch {B}, got {state.shape[0]}")
        if len(images) != c.n_cams or len(img_masks) != c.n_cams:
            raise ValueError(f"expected {c.n_cams} cameras")
        for cam in range(c.n_cams):
            if self.image_embeds:
                if tuple(images[cam].shape) != (B, c.n_img_tokens, c.hidden):
                    raise ValueError(f"image embedding {cam} must be [{B}, {c.n_img_tokens}, {c.hidden}]")
                n = c.n_img_tokens
                self.in_emb[:, cam * n:(cam + 1) * n].copy_(images[cam], non_blocking=True)
            else:
                self.in_img[:, cam].copy_(images[cam], non_blocking=True)
            self.in_img_mask[cam].copy_(img_masks[cam].to(torch.uint8), non_blocking=True)
        toks = lang_tokens
        if toks.shape[1] != c.n_lang:  # pad / truncate like match_static_shape (trt_sample_actions_core_deploy.py:276-286)
            t = torch.zeros(B, c.n_lang, dtype=toks.dtype, device=toks.device)
            m = torch.zeros(B, c.n_lang, dtype=torch.bool, device=toks.device)
            n = min(c.n_lang, toks.shape[1])
            t[:, :n] = toks[:, :n]
            m[:, :n] = lang_masks[:, :n]
            toks, lang_masks = t, m
        self.in_tokens.copy_(toks, non_blocking=True)
        self.in_lang_mask.copy_(lang_masks.to(torch.uint8), non_blocking=True)
        st = state
        if st.shape[1] != c.max_state_dim:
            st = torch.nn.functional.pad(st, (0, c.max_state_dim - st.shape[1]))
        self.in_state.copy_(st, non_blocking=True)
        if noise is not None:  # the prefix-only runner has no flow loop
            self.in_noise.copy_(noise.reshape(B, c.chunk, c.max_action_dim), non_blocking=True)

    def run(self, observer=None):
        """Launch the call on the current stream (graph replay when captured).  ``observer(mods, buf)`` is
        called at every tap point (direct launches only)."""
        if self.graph is not None and observer is None:
            self.graph.replay()
        else:
            self._run_launches(observer)

    def capture(self, warmup: int = 1):
        """Record the launch list as one CUDA graph (inputs and outputs are the static buffers)."""
        s = torch.cuda.Stream(self.dev)
        s.wait_stream(torch.cuda.current_stream(self.dev))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                self._run_launches()
        torch.cuda.current_stream(self.dev).wait_stream(s)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            self._run_launches()
        self.graph = g
        return g

    def actions(self) -> torch.Tensor:
        return self.xt.view(self.B, self.cfg.chunk, self.cfg.max_action_dim)

    def __call__(self, images, img_masks, lang_tokens, lang_masks, state, noise, observer=None) -> torch.Tensor:
        self.load_inputs(images, img_masks, lang_tokens, lang_masks, state, noise)
        self.run(observer)
        return self.actions()


import ctypes as _ct  # noqa: E402

ctypes_structs = (L.GemmDesc, L.NormDesc, L.AttnDesc, L.FlowDesc)
_TAP = object()  # marker of a tap entry in the launch list
ctypes_byref = _ct.byref
