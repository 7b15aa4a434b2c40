"""torch-facing wrappers of the libsvla.so C ABI.

Each function checks devices / dtypes / contiguity, allocates its outputs with torch (the only allocation in
this layer), and launches on torch's current CUDA stream through ctypes.  The most used ops are also
registered as ``torch.ops.svla.*`` custom ops.  Nothing here computes on the CPU: a missing library or a
CPU tensor raises.
"""

from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch

from . import _lib as L
from ._lib import check, lib


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _p(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _need(t: torch.Tensor, dtype: torch.dtype, name: str, contiguous: bool = True) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (there is no CPU path)")
    if t.dtype != dtype:
        raise ValueError(f"{name} must be {dtype}, got {t.dtype}")
    if contiguous and not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


# ----------------------------------------------------------------------------- SmoothQuant primitives

def pack_weight_i8(weight: torch.Tensor, smooth: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """int8 per-output-channel weights with an optional SmoothQuant fold (deploy/linear_only_quant.py:43-54)."""
    _need(weight, torch.bfloat16, "weight")
    n, k = weight.shape
    if smooth is not None:
        _need(smooth, torch.float32, "smooth")
    q = torch.empty(n, k, dtype=torch.int8, device=weight.device)
    ws = torch.empty(n, dtype=torch.float32, device=weight.device)
    check(lib().svla_pack_weight_i8(_p(weight), _p(smooth), n, k, _p(q), _p(ws), _stream()), "pack_weight_i8")
    return q, ws


def dequant_weight_bf16(q: torch.Tensor, ws: torch.Tensor) -> torch.Tensor:
    """bf16(q * ws[:, None]): the weight W8A16Linear multiplies by (deploy/linear_only_quant.py:122-124)."""
    _need(q, torch.int8, "q")
    _need(ws, torch.float32, "ws")
    n, k = q.shape
    out = torch.empty(n, k, dtype=torch.bfloat16, device=q.device)
    check(lib().svla_dequant_weight_bf16(_p(q), _p(ws), n, k, _p(out), _stream()), "dequant_weight_bf16")
    return out


def reciprocal(x: torch.Tensor) -> torch.Tensor:
    """Correctly rounded 1 / x (fp32) on the device -- the reciprocal smooth vectors the quantisers accept."""
    _need(x, torch.float32, "x")
    y = torch.empty_like(x)
    check(lib().svla_reciprocal(_p(x), _p(y), x.numel(), _stream()), "reciprocal")
    return y


def quantize_smooth(x: torch.Tensor, smooth: torch.Tensor | None, act_scale: float) -> torch.Tensor:
    _need(x, torch.bfloat16, "x")
    m, k = x.shape
    q = torch.empty(m, k, dtype=torch.int8, device=x.device)
    check(lib().svla_quantize_smooth(_p(x), k, _p(smooth), float(act_scale), _p(q), k, m, k, _stream()),
          "quantize_smooth")
    return q


def channel_percentile(x: torch.Tensor, rows: int, q: float, amax: torch.Tensor, pamax: torch.Tensor) -> None:
    """Max-accumulate per-channel max(|x|) and torch.quantile(|x|, q) of each `rows`-token call of x (bf16
    [calls * rows, K], unit stride along K) into amax / pamax (fp32 [K], zero-filled before the first call)."""
    _need(x, torch.bfloat16, "x", contiguous=False)
    if x.dim() != 2 or x.stride(1) != 1:
        raise ValueError("channel_percentile: x must be 2-D with unit stride along channels")
    m, k = x.shape
    if rows <= 0 or m % rows:
        raise ValueError(f"channel_percentile: {m} rows are not a whole number of {rows}-token calls")
    for t, n in ((amax, "amax"), (pamax, "pamax")):
        _need(t, torch.float32, n)
        if t.numel() != k or t.device != x.device:
            raise ValueError(f"channel_percentile: {n} must be fp32 [{k}] on {x.device}")
    check(lib().svla_channel_percentile(_p(x), x.stride(0), m // rows, rows, k, float(q), _p(amax), _p(pamax),
                                        _stream()), "channel_percentile")


def flow_pack_weight(w: torch.Tensor) -> torch.Tensor:
    """The fragment-order copy of an int8 or bf16 weight [n, k] (any row stride, unit column stride) that the
    persistent flow kernel reads (svla_flow_pack_weight)."""
    if w.dtype not in (torch.int8, torch.bfloat16):
        raise ValueError(f"flow_pack_weight: int8 or bf16 weight expected, got {w.dtype}")
    _need(w, w.dtype, "w", contiguous=False)
    if w.dim() != 2 or w.stride(1) != 1:
        raise ValueError("flow_pack_weight: w must be 2-D with unit column stride")
    n, k = w.shape
    eb = w.element_size()
    nbytes = lib().svla_flow_packed_bytes(n, k, eb)
    if nbytes == 0:
        raise ValueError(f"flow_pack_weight: [{n}, {k}] is not a multiple of 16 in both dimensions")
    out = torch.empty(nbytes, dtype=torch.uint8, device=w.device)
    check(lib().svla_flow_pack_weight(_p(w), eb, w.stride(0), n, k, _p(out), _stream()), "flow_pack_weight")
    return out


def gemm_i8_i32(qx: torch.Tensor, qw: torch.Tensor) -> torch.Tensor:
    _need(qx, torch.int8, "qx")
    _need(qw, torch.int8, "qw")
    m, k = qx.shape
    n = qw.shape[0]
    acc = torch.empty(m, n, dtype=torch.int32, device=qx.device)
    check(lib().svla_gemm_i8_i32(_p(qx), _p(qw), m, n, k, _p(acc), _stream()), "gemm_i8_i32")
    return acc


def sq_linear_w8a8(x: torch.Tensor, smooth: torch.Tensor | None, act_scale: float, qweight: torch.Tensor,
                   wscale: torch.Tensor, bias: torch.Tensor | None = None,
                   workspace: torch.Tensor | None = None) -> torch.Tensor:
    _need(x, torch.bfloat16, "x")
    m, k = x.shape
    n = qweight.shape[0]
    y = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    need = int(lib().svla_sq_linear_w8a8_workspace_size(m, k))
    if workspace is None:
        workspace = torch.empty(need, dtype=torch.uint8, device=x.device)
    check(lib().svla_sq_linear_w8a8(_p(x), _p(smooth), float(act_scale), _p(qweight), _p(wscale), _p(bias), m, n, k,
                                    _p(y), _p(workspace), workspace.numel(), _stream()), "sq_linear_w8a8")
    return y


def w8a16_linear(x: torch.Tensor, qweight: torch.Tensor, wscale: torch.Tensor,
                 bias: torch.Tensor | None = None) -> torch.Tensor:
    _need(x, torch.bfloat16, "x")
    m, k = x.shape
    n = qweight.shape[0]
    y = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    check(lib().svla_w8a16_linear(_p(x), _p(qweight), _p(wscale), _p(bias), m, n, k, _p(y), _stream()),
          "w8a16_linear")
    return y


# ----------------------------------------------------------------------------- general GEMM

@dataclass
class Seg:
    a: torch.Tensor              # [M, lda]
    b: torch.Tensor              # [n, ldb]
    out: torch.Tensor | None     # [M', ldo]
    n: int
    wscale: torch.Tensor | None = None
    bias: torch.Tensor | None = None
    bias_f32: torch.Tensor | None = None
    act_scale: float = 1.0
    rope: int = 0
    lda: int | None = None
    ldb: int | None = None
    ldo: int | None = None


def gemm_desc(kind: int, epi: int, m: int, k: int, segs: list[Seg], pair: bool = False, block_n: int = 0,
              **extra) -> L.GemmDesc:
    d = L.GemmDesc()
    d.kind, d.epi, d.m, d.k, d.nseg, d.pair, d.block_n = kind, epi, m, k, len(segs), int(pair), block_n
    for i, s in enumerate(segs):
        g = d.seg[i]
        g.a, g.b = s.a.data_ptr(), s.b.data_ptr()
        g.lda = s.lda if s.lda is not None else s.a.stride(0)
        g.ldb = s.ldb if s.ldb is not None else s.b.stride(0)
        g.wscale, g.bias, g.bias_f32 = _p(s.wscale), _p(s.bias), _p(s.bias_f32)
        g.out = _p(s.out)
        g.ldo = s.ldo if s.ldo is not None else (s.out.stride(0) if s.out is not None else s.n)
        g.n, g.act_scale, g.rope = s.n, float(s.act_scale), int(s.rope)
    for key, val in extra.items():
        if isinstance(val, torch.Tensor):
            val = val.data_ptr()
        setattr(d, key, val)
    return d


def splitk_workspace(nbytes: int, device) -> torch.Tensor:
    """A zeroed split-K workspace for svla_gemm (its leading tile counters must start at zero)."""
    return torch.zeros(max(int(nbytes), L.SPLITK_COUNTER_BYTES + 4096), dtype=torch.uint8, device=device)


def gemm(desc: L.GemmDesc) -> None:
    check(lib().svla_gemm(ctypes.byref(desc), _stream()), "svla_gemm")


# ----------------------------------------------------------------------------- norm + quant

def norm_quant(x: torch.Tensor, weight: torch.Tensor, eps: float, bias: torch.Tensor | None = None,
               quants: list[tuple[torch.Tensor, float]] = (), want_y: bool = True, pixel_shuffle: int = 0,
               ps_grid: int = 0, y: torch.Tensor | None = None, q_out: list[torch.Tensor] | None = None,
               rsmooth: list[torch.Tensor | None] | None = None):
    _need(x, torch.bfloat16, "x", contiguous=False)
    m, k = x.shape
    d = L.NormDesc()
    d.x, d.ldx, d.weight, d.bias, d.eps = x.data_ptr(), x.stride(0), weight.data_ptr(), _p(bias), float(eps)
    d.layernorm, d.m, d.k = int(bias is not None), m, k
    # with a pixel shuffle every output (bf16 and int8) is in the shuffled [m / s^2, k * s^2] layout
    qm, qk = (m // (pixel_shuffle ** 2), k * pixel_shuffle ** 2) if pixel_shuffle else (m, k)
    if want_y and y is None:
        y = torch.empty(qm, qk, dtype=torch.bfloat16, device=x.device)
    if y is not None and (y.shape[0] < qm or y.stride(0) < qk):
        raise ValueError(f"y must hold [{qm}, {qk}]")
    d.y, d.ldy = _p(y), (y.stride(0) if y is not None else 0)
    outs = []
    for i, (smooth, act) in enumerate(quants):
        q = q_out[i] if q_out is not None else torch.empty(qm, qk, dtype=torch.int8, device=x.device)
        if q.shape[0] < qm or q.stride(0) < qk:
            raise ValueError(f"int8 output {i} must hold [{qm}, {qk}]")
        outs.append(q)
        d.q[i], d.smooth[i], d.act[i] = q.data_ptr(), smooth.data_ptr(), float(act)
        if rsmooth is not None and rsmooth[i] is not None:
            d.rsmooth[i] = rsmooth[i].data_ptr()
    d.nq, d.ldq = len(quants), (outs[0].stride(0) if outs else 0)
    d.pixel_shuffle, d.ps_grid = pixel_shuffle, ps_grid
    check(lib().svla_norm_quant(ctypes.byref(d), _stream()), "svla_norm_quant")
    return y, outs


# ----------------------------------------------------------------------------- attention / RoPE

def attention_desc(q: torch.Tensor, k1: torch.Tensor, v1: torch.Tensor, batch: int, lq: int, hq: int, hkv: int,
                   mask: torch.Tensor | None = None, k2: torch.Tensor | None = None, v2: torch.Tensor | None = None,
                   o: torch.Tensor | None = None, qo: torch.Tensor | None = None,
                   qo_smooth: torch.Tensor | None = None, qo_act: float = 0.0, scale: float = 0.0,
                   qo_rsmooth: torch.Tensor | None = None, impl: int = L.ATTN_AUTO,
                   key_mask: torch.Tensor | None = None, mask_keys: int = 0) -> L.AttnDesc:
    """q [B, Lq, >=hq*64] (row stride = stride(1)), k/v [B, L, >=hkv*64], mask [B, Lq, L1+L2] (uint8/bool)."""
    d = L.AttnDesc()
    d.q, d.q_bs, d.q_rs = q.data_ptr(), q.stride(0), q.stride(1)
    d.k1, d.v1, d.kv1_bs, d.kv1_rs, d.l1 = k1.data_ptr(), v1.data_ptr(), k1.stride(0), k1.stride(1), k1.shape[1]
    assert v1.stride() == k1.stride()
    if k2 is not None:
        assert v2 is not None and v2.stride() == k2.stride()
        d.k2, d.v2, d.kv2_bs, d.kv2_rs, d.l2 = k2.data_ptr(), v2.data_ptr(), k2.stride(0), k2.stride(1), k2.shape[1]
    if mask is not None:
        d.mask, d.mask_bs, d.mask_rs = mask.data_ptr(), mask.stride(0), mask.stride(1)
    if key_mask is not None:  # [B, >= mask_keys] key flags; keys from mask_keys on are causal
        d.key_mask, d.key_mask_bs, d.mask_keys = key_mask.data_ptr(), key_mask.stride(0), int(mask_keys)
    if o is not None:
        d.o, d.o_bs, d.o_rs = o.data_ptr(), o.stride(0), o.stride(1)
    if qo is not None:
        d.qo, d.qo_bs, d.qo_rs = qo.data_ptr(), qo.stride(0), qo.stride(1)
        d.qo_smooth, d.qo_act = qo_smooth.data_ptr(), float(qo_act)
        d.qo_rsmooth = _p(qo_rsmooth)
    d.batch, d.lq, d.hq, d.hkv, d.scale, d.impl = batch, lq, hq, hkv, float(scale), impl
    return d


def attention_run(desc: L.AttnDesc) -> None:
    check(lib().svla_attention(ctypes.byref(desc), _stream()), "svla_attention")


def attention(q, k1, v1, hq: int, hkv: int, mask=None, k2=None, v2=None, qo_smooth=None, qo_act=0.0,
              qo_rsmooth=None, impl: int = L.ATTN_AUTO, key_mask=None, mask_keys: int = 0):
    """bf16 context [B, Lq, hq*64] (and the int8 context when qo_smooth is given)."""
    b, lq = q.shape[0], q.shape[1]
    o = torch.empty(b, lq, hq * 64, dtype=torch.bfloat16, device=q.device)
    qo = torch.empty(b, lq, hq * 64, dtype=torch.int8, device=q.device) if qo_smooth is not None else None
    if mask is not None and mask.dtype == torch.bool:
        mask = mask.view(torch.uint8)
    attention_run(attention_desc(q, k1, v1, b, lq, hq, hkv, mask=mask, k2=k2, v2=v2, o=o, qo=qo,
                                 qo_smooth=qo_smooth, qo_act=qo_act, qo_rsmooth=qo_rsmooth, impl=impl,
                                 key_mask=key_mask, mask_keys=mask_keys))
    return (o, qo) if qo is not None else o


_DT = {torch.float32: L.DT_FLOAT, torch.float16: L.DT_HALF, torch.bfloat16: L.DT_BF16, torch.int32: L.DT_INT32,
       torch.int64: L.DT_INT64}


def _dtype_code(t: torch.Tensor, allowed: tuple, name: str) -> int:
    code = _DT.get(t.dtype)
    if code is None or code not in allowed:
        raise ValueError(f"{name}: unsupported dtype {t.dtype}")
    return code


def rope_layout(q_raw: torch.Tensor, k_raw: torch.Tensor, pos: torch.Tensor, q_heads: int, kv_heads: int,
                max_wavelength: float = 10000.0, head_dim: int = 64):
    """Plugin semantics of SmolVLAFusedRopeLayout (deploy/cuda/fused_rope_layout.h:24-34): fp32 / fp16 / bf16
    q_raw [B, L, Hq*D] and k_raw [B, L, Hkv*D], int32 / int64 positions [B, L] -> q [B, Hq, L, D] and
    k [B, Hq, D, L] in the input dtype."""
    for t, n in ((q_raw, "q_raw"), (k_raw, "k_raw"), (pos, "pos")):
        _need(t, t.dtype, n)
    if k_raw.dtype != q_raw.dtype:
        raise ValueError("q_raw and k_raw must share a dtype")
    dt = _dtype_code(q_raw, (L.DT_FLOAT, L.DT_HALF, L.DT_BF16), "q_raw")
    pt = _dtype_code(pos, (L.DT_INT32, L.DT_INT64), "pos")
    b, l, _ = q_raw.shape
    q_out = torch.empty(b, q_heads, l, head_dim, dtype=q_raw.dtype, device=q_raw.device)
    k_out = torch.empty(b, q_heads, head_dim, l, dtype=q_raw.dtype, device=q_raw.device)
    params = L.RopeParams(q_heads, kv_heads, head_dim, float(max_wavelength))
    check(lib().svla_fused_rope_layout(_p(q_raw), _p(k_raw), _p(pos), _p(q_out), _p(k_out), b, l, ctypes.byref(params),
                                       dt, pt, _stream()), "fused_rope_layout")
    return q_out, k_out


def rope_attention(q_raw: torch.Tensor, k_raw: torch.Tensor, v_raw: torch.Tensor, pos: torch.Tensor | None,
                   mask: torch.Tensor, q_heads: int, kv_heads: int, max_wavelength: float = 10000.0,
                   head_dim: int = 64) -> torch.Tensor:
    """Plugin semantics of SmolVLAFusedRopeAttention (deploy/cuda/fused_rope_layout.h:44-50): raw q / k / v,
    positions [B, L] (int32 / int64; None with an fp32 mask = the implicit-position fp32 variant), keep-mask
    [B, L, L] (bool, or fp32 > 0.5) -> fp32 context [B, Hq, L, D]."""
    for t, n in ((q_raw, "q_raw"), (k_raw, "k_raw"), (v_raw, "v_raw"), (mask, "mask")):
        _need(t, t.dtype, n)
    if not (k_raw.dtype == v_raw.dtype == q_raw.dtype):
        raise ValueError("q_raw, k_raw and v_raw must share a dtype")
    b, l, _ = q_raw.shape
    ctx = torch.empty(b, q_heads, l, head_dim, dtype=torch.float32, device=q_raw.device)
    params = L.RopeParams(q_heads, kv_heads, head_dim, float(max_wavelength))
    if pos is None:
        _need(q_raw, torch.float32, "q_raw")
        _need(mask, torch.float32, "mask")
        check(lib().svla_fused_rope_attention_f32_mask_implicit_pos(_p(q_raw), _p(k_raw), _p(v_raw), _p(mask), _p(ctx),
                                                                    b, l, ctypes.byref(params), _stream()),
              "fused_rope_attention_f32_mask_implicit_pos")
        return ctx
    _need(pos, pos.dtype, "pos")
    dt = _dtype_code(q_raw, (L.DT_FLOAT, L.DT_HALF, L.DT_BF16), "q_raw")
    pt = _dtype_code(pos, (L.DT_INT32, L.DT_INT64), "pos")
    if mask.dtype not in (torch.bool, torch.uint8):
        raise ValueError("mask must be bool / uint8 (use pos=None for the fp32-mask variant)")
    check(lib().svla_fused_rope_attention(_p(q_raw), _p(k_raw), _p(v_raw), _p(pos), _p(mask), _p(ctx), b, l,
                                          ctypes.byref(params), dt, pt, _stream()), "fused_rope_attention")
    return ctx


def rope_table(max_pos: int, max_wavelength: float, device) -> torch.Tensor:
    cs = torch.empty(max_pos, 32, 2, dtype=torch.float32, device=device)
    check(lib().svla_rope_table(_p(cs), max_pos, float(max_wavelength), _stream()), "rope_table")
    return cs


# ----------------------------------------------------------------------------- torch custom ops

@torch.library.custom_op("svla::sq_linear_w8a8", mutates_args=())
def _sq_linear_op(x: torch.Tensor, smooth: torch.Tensor, act_scale: float, qweight: torch.Tensor,
                  wscale: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    return sq_linear_w8a8(x, smooth, act_scale, qweight, wscale, bias)


@_sq_linear_op.register_fake
def _(x, smooth, act_scale, qweight, wscale, bias):
    return x.new_empty(x.shape[0], qweight.shape[0])


@torch.library.custom_op("svla::w8a16_linear", mutates_args=())
def _w8a16_op(x: torch.Tensor, qweight: torch.Tensor, wscale: torch.Tensor, bias: torch.Tensor | None) -> torch.Tensor:
    return w8a16_linear(x, qweight, wscale, bias)


@_w8a16_op.register_fake
def _(x, qweight, wscale, bias):
    return x.new_empty(x.shape[0], qweight.shape[0])


@torch.library.custom_op("svla::rope_layout", mutates_args=())
def _rope_layout_op(q_raw: torch.Tensor, k_raw: torch.Tensor, pos: torch.Tensor, q_heads: int, kv_heads: int,
                    max_wavelength: float) -> tuple[torch.Tensor, torch.Tensor]:
    return rope_layout(q_raw, k_raw, pos, q_heads, kv_heads, max_wavelength)


@_rope_layout_op.register_fake
def _(q_raw, k_raw, pos, q_heads, kv_heads, max_wavelength):
    b, l, w = q_raw.shape
    d = w // q_heads
    return q_raw.new_empty(b, q_heads, l, d), q_raw.new_empty(b, q_heads, d, l)


@torch.library.custom_op("svla::rope_attention", mutates_args=())
def _rope_attention_op(q_raw: torch.Tensor, k_raw: torch.Tensor, v_raw: torch.Tensor, pos: torch.Tensor,
                       mask: torch.Tensor, q_heads: int, kv_heads: int, max_wavelength: float) -> torch.Tensor:
    return rope_attention(q_raw, k_raw, v_raw, pos, mask, q_heads, kv_heads, max_wavelength,
                          head_dim=q_raw.shape[-1] // q_heads)


@_rope_attention_op.register_fake
def _(q_raw, k_raw, v_raw, pos, mask, q_heads, kv_heads, max_wavelength):
    b, l, w = q_raw.shape
    return q_raw.new_empty(b, q_heads, l, w // q_heads, dtype=torch.float32)
