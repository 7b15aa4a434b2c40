"""Parity of the sm_100a kernels (through the C ABI) with the CPU oracle.

Bars (stated per test):
  * int8 activations, int8 weights, weight scales and int32 accumulators: bit-exact.
  * W8A8 output: bit-exact with bf16 of the fp32 integer-dequant form (acc*a)*w_s + b that the kernel
    computes; against the reference's bf16 fake-dequant output (which rounds qx*a and qw*w_s to bf16 before
    a bf16 GEMM): cosine >= 0.9999, relative L2 <= 1e-2, max-abs <= 1e-2 * max|y_ref|.
  * bf16 GEMMs / W8A16: against an fp32 torch reference of the same bf16 operands rounded to bf16,
    |diff| <= 1 bf16 ulp (2^-7 |ref|) + 1e-5 * max|ref| (fp32 summation order differs).
  * composite epilogues (SiLU gate: three bf16 roundings) within 2 bf16 ulps; residual adds within one ulp
    of the pre-residual value plus one ulp of the sum.
  * norms / attention: stated in each test.
"""

import math

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from oracle import quant as Q
from smolvla_mujoco_libero_b200 import _lib as L
from smolvla_mujoco_libero_b200 import ops, synthetic

pytestmark = pytest.mark.gpu
DEV = "cuda"


def bf16_ulp_close(got: torch.Tensor, ref: torch.Tensor, ulps: float = 1.0, atol: float = 1e-6) -> tuple[bool, float]:
    got = got.float().cpu()
    ref = ref.float().cpu()
    tol = ref.abs() * (ulps * 2.0 ** -7) + atol + 1e-5 * float(ref.abs().max())
    bad = (got - ref).abs() > tol
    return (not bool(bad.any())), float(bad.float().mean())


def rope_close(got: torch.Tensor, ref: torch.Tensor, y: torch.Tensor, rope: int) -> None:
    """RoPE outputs: within one bf16 ulp of the result plus one of the rotated pair's norm sqrt(x1^2 + x2^2)
    (a rotation keeps the norm; a near-zero output of a large pair inherits the pair's rounding)."""
    got, ref, y = got.float().cpu(), ref.float().cpu(), y.float().cpu()
    r = y.abs()
    if rope:
        h = y.view(y.shape[0], -1, 2, 32)
        norm = (h[:, :, 0] ** 2 + h[:, :, 1] ** 2).sqrt()
        r = torch.stack([norm, norm], dim=2).reshape(y.shape)
    tol = (ref.abs() + r) * 2.0 ** -7 + 1e-5 * float(ref.abs().max())
    bad = (got - ref).abs() > tol
    assert not bool(bad.any()), float(bad.float().mean())


def fake_dequant_close(y: torch.Tensor, ref: torch.Tensor) -> None:
    y, ref = y.float().cpu(), ref.float().cpu()
    d = (y - ref).abs()
    assert cosine(y, ref) >= 0.9999
    assert float(d.norm() / ref.norm()) <= 1e-2
    assert float(d.max()) <= 1e-2 * float(ref.abs().max())


def cosine(a, b):
    return float(F.cosine_similarity(a.float().flatten().cpu(), b.float().flatten().cpu(), dim=0))


def _bf16(a):
    return torch.from_numpy(np.asarray(a)).view(torch.bfloat16)


@pytest.fixture(autouse=True)
def _no_device_error():
    L.device_error(reset=True)
    yield
    torch.cuda.synchronize()
    assert L.device_error(reset=True) == 0


# ----------------------------------------------------------------------------- SmoothQuant primitives

def test_pack_weight_bit_exact_with_smoothing():
    case = synthetic.smoothquant_linear_case()
    smooth = torch.rand(960, generator=synthetic.generator(5)) * 4 + 0.1
    q_ref, ws_ref = Q.pack_w8a8_weight(case.weight, smooth)
    q, ws = ops.pack_weight_i8(case.weight.to(DEV), smooth.to(DEV))
    assert torch.equal(q.cpu(), q_ref)
    assert torch.equal(ws.cpu(), ws_ref)
    q2, ws2 = ops.pack_weight_i8(case.weight.to(DEV))
    q2_ref, ws2_ref = Q.quantize_weight_per_out_channel(case.weight)
    assert torch.equal(q2.cpu(), q2_ref) and torch.equal(ws2.cpu(), ws2_ref)


def test_fast_quantiser_matches_two_divides_on_boundaries():
    """The reciprocal fast path must give exactly round((y / s) / a).clamp(-128, 127).  RMSNorm of a row of
    ones returns the norm weight w itself, so per-channel smooth scales s = w / (t * a) put y / s / a on
    chosen targets t: on .5 rounding boundaries, 1e-7 .. 1e-3 beside them, and beyond the clamp."""
    g = synthetic.generator(17)
    halves = torch.arange(-131, 131, dtype=torch.float32) + 0.5
    jitter = torch.tensor([0.0, 1e-6, -1e-6, 9e-4, -9e-4, 1.1e-3, -1.1e-3, 0.3])
    targets = (halves[:, None] + jitter[None, :]).flatten()
    targets = torch.cat([targets, torch.tensor([300.0, -300.0, 255.9, -256.1, 127.4, -128.4, 0.0, 1e-3])])
    k = ((targets.numel() + 7) // 8) * 8
    t = torch.zeros(k)
    t[: targets.numel()] = targets
    t[targets.numel():] = 0.25
    w = ((torch.rand(k, generator=g) + 0.5) * torch.where(torch.rand(k, generator=g) > 0.5, 1.0, -1.0)).to(torch.bfloat16)
    a = 0.0173
    s = (w.float() / (t * a)).abs().clamp_min(1e-6)
    x = torch.ones(4, k, dtype=torch.bfloat16)
    y, (q_exact,) = ops.norm_quant(x.to(DEV), w.to(DEV), 1e-5, quants=[(s.to(DEV), a)])
    _, (q_fast,) = ops.norm_quant(x.to(DEV), w.to(DEV), 1e-5, quants=[(s.to(DEV), a)], rsmooth=[ops.reciprocal(s.to(DEV))])
    assert torch.equal(y.cpu()[0], w)
    ref = Q.smooth_quantize_activation(y.cpu(), s, a)
    assert torch.equal(q_exact.cpu(), ref)
    assert torch.equal(q_fast.cpu(), ref)


def test_quantize_smooth_bit_exact(golden):
    g = golden["linear_full"]
    case = synthetic.smoothquant_linear_case()
    smooth = torch.tensor(g["smooth_scale"], dtype=torch.float32)
    q = ops.quantize_smooth(case.x.to(DEV), smooth.to(DEV), g["act_scale"])
    assert torch.equal(q.cpu(), Q.smooth_quantize_activation(case.x, smooth, g["act_scale"]))


@pytest.mark.parametrize("m,k,n", [(177, 960, 2560), (177, 960, 320), (1, 128, 64), (3, 960, 960),
                                   (50, 720, 960), (300, 2560, 960), (129, 12288, 960), (1024, 768, 3072)])
def test_gemm_i8_i32_bit_exact(m, k, n):
    g = synthetic.generator(m * 7 + k + n)
    qx = torch.randint(-128, 128, (m, k), generator=g, dtype=torch.int8)
    qw = torch.randint(-127, 128, (n, k), generator=g, dtype=torch.int8)
    acc = ops.gemm_i8_i32(qx.to(DEV), qw.to(DEV))
    assert torch.equal(acc.cpu(), Q.int_gemm(qx, qw))


def test_sq_linear_single_linear_workload(golden):
    """The single-linear workload (X [177,960] with outliers, W [2560,960], alpha 0.85, p99.99 over 32 batches)."""
    g = golden["linear_full"]
    case = synthetic.smoothquant_linear_case()
    smooth = torch.tensor(g["smooth_scale"], dtype=torch.float32)
    lin = Q.W8A8Linear(case.weight, None, g["act_scale"], smooth)
    qw, ws = ops.pack_weight_i8(case.weight.to(DEV), smooth.to(DEV))
    y = ops.sq_linear_w8a8(case.x.to(DEV), smooth.to(DEV), g["act_scale"], qw, ws)
    qx = lin.quantize_input(case.x)
    y_int = Q.w8a8_int_dequant(Q.int_gemm(qx, lin.qweight), g["act_scale"], lin.weight_scale, None)
    assert torch.equal(y.cpu(), y_int.to(torch.bfloat16))          # kernel == fp32 int-dequant form, rounded
    fake_dequant_close(y, lin(case.x))                               # reference bf16 fake-dequant


def test_sq_linear_golden_small_with_bias(golden_dir):
    d = np.load(golden_dir / "linear_small.npz")
    x, w, b = _bf16(d["x_bf16"]), _bf16(d["weight_bf16"]), _bf16(d["bias_bf16"])
    a = float(d["act_scale"][0])
    smooth = torch.from_numpy(d["smooth_scale"])
    qw, ws = ops.pack_weight_i8(w.to(DEV), smooth.to(DEV))
    assert torch.equal(qw.cpu(), torch.from_numpy(d["qweight"]))
    assert torch.equal(ws.cpu(), torch.from_numpy(d["weight_scale"]))
    qx = ops.quantize_smooth(x.to(DEV), smooth.to(DEV), a)
    assert torch.equal(qx.cpu().float() * torch.tensor(a, dtype=torch.float32), torch.from_numpy(d["x_deq"]))
    y = ops.sq_linear_w8a8(x.to(DEV), smooth.to(DEV), a, qw, ws, b.to(DEV))
    fake_dequant_close(y, torch.from_numpy(d["y_bf16"]).view(torch.bfloat16))


# ----------------------------------------------------------------------------- W8A16 / bf16

def test_w8a16_golden(golden_dir):
    d = np.load(golden_dir / "w8a16_small.npz")
    x, w, b = _bf16(d["x_bf16"]), _bf16(d["weight_bf16"]), _bf16(d["bias_bf16"])
    qw, ws = ops.pack_weight_i8(w.to(DEV))
    y = ops.w8a16_linear(x.to(DEV), qw, ws, b.to(DEV))
    w_deq = _bf16(d["weight_deq_bf16"]).float()
    ref = (x.float() @ w_deq.t() + b.float()).to(torch.bfloat16)
    ok, frac = bf16_ulp_close(y, ref, ulps=1.0)
    assert ok, frac
    assert cosine(y, _bf16(d["y_bf16"])) >= 0.99999


@pytest.mark.parametrize("m,k,n", [(50, 720, 960), (50, 720, 320), (50, 2048, 720), (177, 2560, 960),
                                   (177, 320, 320), (3, 64, 16), (600, 720, 4096)])
def test_w8a16_shapes(m, k, n):
    g = synthetic.generator(m + 3 * k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.02).to(torch.bfloat16)
    lin = Q.W8A16Linear(w, b)
    qw, ws = ops.pack_weight_i8(w.to(DEV))
    assert torch.equal(qw.cpu(), lin.qweight)
    y = ops.w8a16_linear(x.to(DEV), qw, ws, b.to(DEV))
    ref = (x.float() @ lin.weight.float().t() + b.float()).to(torch.bfloat16)
    ok, frac = bf16_ulp_close(y, ref, ulps=1.0)
    assert ok, frac


@pytest.mark.parametrize("m,k,n", [(50, 32, 720), (50, 1440, 720), (1, 32, 960), (2048, 768, 768)])
def test_bf16_gemm(m, k, n):
    g = synthetic.generator(m + k + n)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16)
    b = (torch.randn(n, generator=g) * 0.05).to(torch.bfloat16)
    xd, wd, bd = x.to(DEV), w.to(DEV), b.to(DEV)
    out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_BF16, L.EPI_BF16, m, k, [ops.Seg(a=xd, b=wd, out=out, n=n, bias=bd)]))
    ref = (x.float() @ w.float().t() + b.float()).to(torch.bfloat16)
    ok, frac = bf16_ulp_close(out, ref, ulps=1.0)
    assert ok, frac


# ----------------------------------------------------------------------------- epilogues

def _rand_i8(shape, g):
    return torch.randint(-128, 128, shape, generator=g, dtype=torch.int8)


def test_epilogue_rope_qkv_segments():
    """q/k/v as three segments with their own int8 A, weights and scales; RoPE on q and k."""
    g = synthetic.generator(11)
    m, k = 177, 960
    pos = torch.arange(m, dtype=torch.int32)
    cs = ops.rope_table(256, 10000.0, DEV)
    segs, refs = [], []
    for n, rope in ((960, 1), (320, 1), (320, 0)):
        qx, qw = _rand_i8((m, k), g), _rand_i8((n, k), g)
        ws = torch.rand(n, generator=g) * 1e-3
        a = 0.01 + torch.rand(1, generator=g).item() * 0.01
        out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
        segs.append(ops.Seg(a=qx.to(DEV), b=qw.to(DEV), out=out, n=n, wscale=ws.to(DEV), act_scale=a, rope=rope))
        y = Q.w8a8_int_dequant(Q.int_gemm(qx, qw), a, ws, None).to(torch.bfloat16)
        yr = y
        if rope:
            from oracle.model import apply_rope
            yr = apply_rope(y.view(1, m, n // 64, 64), pos.long()[None]).reshape(m, n)
        refs.append((yr, y, rope))
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_ROPE, m, k, segs, rope_cs=cs, pos=pos.to(DEV), max_pos=256))
    for s, (ref, y, rope) in zip(segs, refs):
        rope_close(s.out, ref, y, rope)


def test_epilogue_resid_silu_mul_gelu_quant_euler_f32():
    g = synthetic.generator(12)
    m, k, n = 177, 960, 320
    qx, qw = _rand_i8((m, k), g), _rand_i8((n, k), g)
    ws = torch.rand(n, generator=g) * 1e-3
    a = 0.02
    y_int = Q.w8a8_int_dequant(Q.int_gemm(qx, qw), a, ws, None)
    yb = y_int.to(torch.bfloat16)
    qxd, qwd, wsd = qx.to(DEV), qw.to(DEV), ws.to(DEV)
    # residual (in place)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    out = res.to(DEV).clone()
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_RESID, m, k, [ops.Seg(a=qxd, b=qwd, out=out, n=n, wscale=wsd, act_scale=a)],
                           resid=out, ldr=n))
    ok, _ = bf16_ulp_close(out, (yb.float() + res.float()).to(torch.bfloat16), ulps=1.0)
    assert ok
    # SiLU-gate pair
    qx2, qw2 = _rand_i8((m, k), g), _rand_i8((n, k), g)
    ws2 = torch.rand(n, generator=g) * 1e-3
    u = Q.w8a8_int_dequant(Q.int_gemm(qx2, qw2), 0.03, ws2, None).to(torch.bfloat16)
    h = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_SILU_MUL, m, k,
                           [ops.Seg(a=qxd, b=qwd, out=h, n=n, wscale=wsd, act_scale=a),
                            ops.Seg(a=qx2.to(DEV), b=qw2.to(DEV), out=h, n=n, wscale=ws2.to(DEV), act_scale=0.03)],
                           pair=True))
    ref = (F.silu(yb) * u)
    ok, frac = bf16_ulp_close(h, ref, ulps=2.0, atol=1e-5)  # three bf16 roundings, as above
    assert ok, frac
    # GELU(tanh) + quantise for the next linear
    smooth = torch.rand(n, generator=g) + 0.5
    qout = torch.empty(m, n, dtype=torch.int8, device=DEV)
    ybf = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_GELU_QUANT, m, k, [ops.Seg(a=qxd, b=qwd, out=ybf, n=n, wscale=wsd, act_scale=a)],
                           q_smooth=smooth.to(DEV), q_act=0.01, qout=qout, ldq=n))
    qout_fast = torch.empty_like(qout)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_GELU_QUANT, m, k, [ops.Seg(a=qxd, b=qwd, out=None, n=n, wscale=wsd, act_scale=a)],
                           q_smooth=smooth.to(DEV), q_rsmooth=ops.reciprocal(smooth.to(DEV)), q_act=0.01, qout=qout_fast,
                           ldq=n))
    assert torch.equal(qout_fast, qout)
    gref = F.gelu(yb, approximate="tanh")
    ok, frac = bf16_ulp_close(ybf, gref, ulps=1.0, atol=1e-5)
    assert ok, frac
    q_from_got = Q.smooth_quantize_activation(ybf.cpu(), smooth, 0.01)
    assert torch.equal(qout.cpu(), q_from_got)   # quantiser bit-exact given the bf16 value
    # fp32 output and the Euler update
    xb = torch.randn(50, 720, generator=g).to(torch.bfloat16)
    wb = (torch.randn(32, 720, generator=g) * 0.05).to(torch.bfloat16)
    bb = (torch.randn(32, generator=g) * 0.05).to(torch.bfloat16)
    v_ref = xb.float() @ wb.float().t() + bb.float()
    f32 = torch.empty(50, 32, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_BF16, L.EPI_F32, 50, 720, [ops.Seg(a=xb.to(DEV), b=wb.to(DEV), out=f32, n=32, bias=bb.to(DEV))]))
    assert torch.allclose(f32.cpu(), v_ref, rtol=1e-5, atol=1e-5)
    xt0 = torch.randn(50, 32, generator=g)
    xt = xt0.to(DEV).clone()
    xtb = torch.empty(50, 32, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_BF16, L.EPI_EULER, 50, 720, [ops.Seg(a=xb.to(DEV), b=wb.to(DEV), out=None, n=32, bias=bb.to(DEV), ldo=32)],
                           dt=-0.1, xt=xt, xt_bf16=xtb))
    x_ref = xt0 + (-0.1) * v_ref
    assert torch.allclose(xt.cpu(), x_ref, rtol=1e-5, atol=1e-5)
    assert torch.equal(xtb.cpu(), xt.cpu().to(torch.bfloat16))


def test_row_remap_and_post_scale():
    """Connector-style output: rows scattered into the prefix buffer, then bf16(y) * 31 rounded again."""
    g = synthetic.generator(13)
    m, k, n = 256, 256, 64
    qx, qw = _rand_i8((m, k), g), _rand_i8((n, k), g)
    ws = torch.rand(n, generator=g) * 1e-3
    y = Q.w8a8_int_dequant(Q.int_gemm(qx, qw), 0.01, ws, None).to(torch.bfloat16)
    ref = (y.float() * 31.0).to(torch.bfloat16)
    buf = torch.zeros(2 * 177, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_BF16, m, k, [ops.Seg(a=qx.to(DEV), b=qw.to(DEV), out=buf, n=n, wscale=ws.to(DEV), act_scale=0.01)],
                           rows_per_group=128, group_stride=177, post_scale=31.0))
    buf = buf.cpu()
    assert torch.equal(buf[0:128], ref[0:128])
    assert torch.equal(buf[177:177 + 128], ref[128:256])
    assert buf[128:177].abs().sum() == 0


@pytest.mark.parametrize("layout", ["offset", "padded_rows"])
def test_epilogues_on_16_byte_aligned_rows_equal_32_byte_aligned(layout):
    """The bf16 output stores and residual loads use 256-bit accesses when every row starts on a 32-byte
    boundary and 128-bit ones otherwise.  Outputs / residuals 16 bytes off (a +8 element slice, or rows of
    n + 8 elements) take the 128-bit path; the results must equal the 32-byte aligned call bit for bit."""
    g = synthetic.generator(31)
    m, k, n = 300, 256, 320
    qx, qw = _rand_i8((m, k), g).to(DEV), _rand_i8((n, k), g).to(DEV)
    ws = (torch.rand(n, generator=g) * 1e-3).to(DEV)
    bias = (torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).to(DEV)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16).to(DEV)

    def seg(out, ldo=None):
        return ops.Seg(a=qx, b=qw, out=out, n=n, wscale=ws, bias=bias, act_scale=0.02, ldo=ldo)

    def buf():
        if layout == "offset":  # base 16 bytes past a 32-byte boundary, rows of n elements
            raw = torch.zeros(m * n + 16, dtype=torch.bfloat16, device=DEV)
            return raw[8:8 + m * n].view(m, n), None
        raw = torch.zeros(m, n + 8, dtype=torch.bfloat16, device=DEV)  # 656-byte rows
        return raw[:, :n], n + 8

    y_ref = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_BF16, m, k, [seg(y_ref)]))
    y, ldo = buf()
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_BF16, m, k, [seg(y, ldo)]))
    assert torch.equal(y, y_ref)
    r_ref = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_RESID, m, k, [seg(r_ref)], resid=res, ldr=n))
    r_in, ldr = buf()
    r_in.copy_(res)
    r_out, ldo = buf()
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_RESID, m, k, [seg(r_out, ldo)], resid=r_in, ldr=ldr or n))
    assert torch.equal(r_out, r_ref)
    assert torch.equal(r_ref.cpu(), (y_ref.float() + res.float()).to(torch.bfloat16).cpu())


# ----------------------------------------------------------------------------- CTA pairs

def _pair_case(kind, epi, m, n, k, g, nseg=1, pair=False):
    """Operands and a descriptor builder for one GEMM; build(cta_pair) returns (descriptor, outputs)."""
    if kind == L.KIND_I8:
        a = [_rand_i8((m, k), g).to(DEV) for _ in range(nseg)]
        b = [_rand_i8((n, k), g).to(DEV) for _ in range(nseg)]
    else:
        a = [torch.randn(m, k, generator=g).to(torch.bfloat16).to(DEV) for _ in range(nseg)]
        b = [(torch.randn(n, k, generator=g) * 0.05).to(torch.bfloat16).to(DEV) for _ in range(nseg)]
    ws = [(torch.rand(n, generator=g) * 1e-3).to(DEV) for _ in range(nseg)]
    bias = [(torch.randn(n, generator=g) * 0.1).to(torch.bfloat16).to(DEV) for _ in range(nseg)]
    res = torch.randn(m, n, generator=g).to(torch.bfloat16).to(DEV)
    smooth = (torch.rand(n, generator=g) + 0.5).to(DEV)
    pos = torch.randint(0, 227, (m,), generator=g, dtype=torch.int32).to(DEV)
    cs = ops.rope_table(227, 10000.0, DEV)
    odt = torch.int32 if epi == L.EPI_I32 else torch.bfloat16

    def build(cta_pair):
        outs = [torch.zeros(m, n, dtype=odt, device=DEV) for _ in range(1 if pair else nseg)]
        if epi == L.EPI_RESID:
            outs[0].copy_(res)
        segs = [ops.Seg(a=a[i], b=b[i], out=outs[0 if pair else i], n=n, wscale=ws[i], act_scale=0.01 + 0.01 * i,
                        bias=None if epi == L.EPI_I32 else bias[i], rope=1 if (epi == L.EPI_ROPE and i < 2) else 0)
                for i in range(nseg)]
        extra = {}
        if epi == L.EPI_RESID:
            extra = dict(resid=outs[0], ldr=n)
        if epi == L.EPI_ROPE:
            extra = dict(rope_cs=cs, pos=pos, max_pos=227)
        qout = None
        if epi == L.EPI_GELU_QUANT:
            qout = torch.zeros(m, n, dtype=torch.int8, device=DEV)
            extra = dict(q_smooth=smooth, q_rsmooth=ops.reciprocal(smooth), q_act=0.02, qout=qout, ldq=n)
        d = ops.gemm_desc(kind, epi, m, k, segs, pair=pair, cta_pair=cta_pair, block_n=128, **extra)
        return d, outs + ([qout] if qout is not None else [])
    return build


@pytest.mark.parametrize("kind,m,n,k,block_n", [
    (L.KIND_BF16, 3200, 2048, 720, 128),   # expert gate / up at batch 64
    (L.KIND_BF16, 50, 2048, 720, 64),      # batch 1, 64-column tiles
    (L.KIND_I8, 300, 1024, 960, 128),      # W8A8 pair over one activation tensor
])
def test_pair_over_one_a_operand_equals_two_mmas(kind, m, n, k, block_n):
    """A gate / up pair whose two linears read the same A tensor runs one MMA of N = 2 * block_n per k-step;
    the same pair with A passed as two copies runs two MMAs of N = block_n.  Outputs must match bit for bit
    (each output element sees the same products in the same K order)."""
    g = synthetic.generator(m + n + k + block_n)
    if kind == L.KIND_I8:
        x = _rand_i8((m, k), g).to(DEV)
        ws = [(_rand_i8((n, k), g).to(DEV), (torch.rand(n, generator=g) * 1e-3).to(DEV)) for _ in range(2)]
        segs = lambda a0, a1, out: [ops.Seg(a=a, b=w, out=out, n=n, wscale=s, act_scale=0.02)
                                    for a, (w, s) in zip((a0, a1), ws)]
    else:
        x = (torch.randn(m, k, generator=g) * 0.5).to(DEV, torch.bfloat16)
        ws = [((torch.randn(n, k, generator=g) * 0.02).to(DEV, torch.bfloat16), None) for _ in range(2)]
        segs = lambda a0, a1, out: [ops.Seg(a=a, b=w, out=out, n=n) for a, (w, _) in zip((a0, a1), ws)]
    outs = []
    for a1 in (x, x.clone()):
        out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
        ops.gemm(ops.gemm_desc(kind, L.EPI_SILU_MUL, m, k, segs(x, a1, out), pair=True, block_n=block_n))
        outs.append(out)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    assert bool(torch.isfinite(outs[0].float()).all())


@pytest.mark.parametrize("kind,epi,m,n,k,nseg,pair", [
    (L.KIND_I8, L.EPI_I32, 1000, 512, 768, 1, False),        # 8 row tiles: 4 pairs, the last partly past M
    (L.KIND_I8, L.EPI_BF16, 2048, 768, 768, 3, False),       # SigLIP q/k/v segments
    (L.KIND_I8, L.EPI_GELU_QUANT, 1280, 3072, 768, 1, False),
    (L.KIND_I8, L.EPI_RESID, 768, 768, 3072, 1, False),
    (L.KIND_I8, L.EPI_ROPE, 1416, 320, 960, 3, False),       # text q/k/v with RoPE, 8 x 177 rows
    (L.KIND_BF16, L.EPI_RESID, 3200, 720, 2048, 1, False),   # expert down_proj
    (L.KIND_BF16, L.EPI_SILU_MUL, 3200, 2048, 720, 2, True),  # expert gate / up pair
    (L.KIND_BF16, L.EPI_ROPE, 3200, 320, 720, 3, False),     # expert q/k/v
])
def test_cta_pairs_equal_single_ctas(kind, epi, m, n, k, nseg, pair):
    """tcgen05 cta_group::2 (256-row tiles over two SMs, each loading half of B) against one CTA per 128-row
    tile: every output bit-identical (the same MMA K order per output element)."""
    g = synthetic.generator(m + n + k + epi)
    build = _pair_case(kind, epi, m, n, k, g, nseg, pair)
    d1, o1 = build(1)
    ops.gemm(d1)
    d2, o2 = build(2)
    ops.gemm(d2)
    torch.cuda.synchronize()
    for x, y in zip(o1, o2):
        assert torch.equal(x, y)


def test_cta_pair_int32_matches_oracle():
    g = synthetic.generator(77)
    m, n, k = 1000, 512, 768
    qx, qw = _rand_i8((m, k), g), _rand_i8((n, k), g)
    acc = torch.zeros(m, n, dtype=torch.int32, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_I32, m, k, [ops.Seg(a=qx.to(DEV), b=qw.to(DEV), out=acc, n=n)],
                           cta_pair=2, block_n=256))
    assert torch.equal(acc.cpu(), Q.int_gemm(qx, qw))


# ----------------------------------------------------------------------------- norms

def test_rmsnorm_quant_three_outputs():
    from oracle.model import rms_norm
    g = synthetic.generator(21)
    ch = synthetic.outlier_channels(960, 8, g)
    x = synthetic.outlier_activations(177, 960, ch, 30.0, g)
    w = (1.0 + 0.1 * torch.randn(960, generator=g)).to(torch.bfloat16)
    smooths = [torch.rand(960, generator=g) * 3 + 0.2 for _ in range(3)]
    acts = [0.02, 0.03, 0.05]
    y, qs = ops.norm_quant(x.to(DEV), w.to(DEV), 1e-5, quants=[(s.to(DEV), a) for s, a in zip(smooths, acts)])
    # the reciprocal fast path gives the same int8 values
    _, qf = ops.norm_quant(x.to(DEV), w.to(DEV), 1e-5, quants=[(s.to(DEV), a) for s, a in zip(smooths, acts)],
                           rsmooth=[ops.reciprocal(s.to(DEV)) for s in smooths])
    for a_, b_ in zip(qs, qf):
        assert torch.equal(a_, b_)
    ref = rms_norm(x, w, 1e-5)
    ok, frac = bf16_ulp_close(y, ref, ulps=1.0)
    assert ok, frac
    assert float((y.cpu() != ref).float().mean()) < 1e-3   # sum order may flip a rare rounding
    for q, s, a in zip(qs, smooths, acts):
        assert torch.equal(q.cpu(), Q.smooth_quantize_activation(y.cpu(), s, a))


def test_layernorm_and_pixel_shuffle_quant():
    from oracle.model import pixel_shuffle
    g = synthetic.generator(22)
    x = torch.randn(2 * 1024, 768, generator=g).to(torch.bfloat16)
    w = (1.0 + 0.1 * torch.randn(768, generator=g)).to(torch.bfloat16)
    b = (0.1 * torch.randn(768, generator=g)).to(torch.bfloat16)
    smooth = torch.rand(768 * 16, generator=g) + 0.5
    y, (q,) = ops.norm_quant(x.to(DEV), w.to(DEV), 1e-6, bias=b.to(DEV), quants=[(smooth.to(DEV), 0.02)],
                             pixel_shuffle=4, ps_grid=32)
    ref = F.layer_norm(x.float(), (768,), w.float(), b.float(), 1e-6).to(torch.bfloat16)
    ref_shuffled = pixel_shuffle(ref.view(2, 1024, 768), 4).reshape(128, 768 * 16)
    assert y.shape == (128, 768 * 16)          # the bf16 output is written in the shuffled layout too
    ok, frac = bf16_ulp_close(y, ref_shuffled, ulps=1.0, atol=1e-5)
    assert ok, frac
    assert torch.equal(q.cpu(), Q.smooth_quantize_activation(y.cpu(), smooth, 0.02))


# ----------------------------------------------------------------------------- attention

def _attn_ref(q, k, v, mask, hq, hkv):
    from oracle.model import eager_attention
    return eager_attention(q, k, v, mask, hq, hkv)


@pytest.mark.parametrize("b,lq,lk,hq,hkv,masked", [(1, 177, 177, 15, 5, True), (2, 50, 177, 15, 5, True),
                                                  (1, 1024, 1024, 12, 12, False), (3, 5, 9, 15, 5, True)])
def test_attention_single_source(b, lq, lk, hq, hkv, masked):
    g = synthetic.generator(b * 1000 + lq + lk)
    q = torch.randn(b, lq, hq * 64, generator=g).to(torch.bfloat16)
    k = torch.randn(b, lk, hkv * 64, generator=g).to(torch.bfloat16)
    v = torch.randn(b, lk, hkv * 64, generator=g).to(torch.bfloat16)
    mask = (torch.rand(b, lq, lk, generator=g) > 0.3) if masked else None
    if masked:
        mask[:, 0, :] = False   # a fully masked row: uniform over all keys, as the reference
    o = ops.attention(q.to(DEV), k.to(DEV), v.to(DEV), hq, hkv, mask=None if mask is None else mask.to(DEV))
    ref = _attn_ref(q, k, v, mask, hq, hkv)
    assert cosine(o, ref) >= 0.9999
    assert float((o.cpu().float() - ref.float()).abs().max()) <= 2e-2


@pytest.mark.parametrize("b,lq,lk,hq,hkv", [(2, 1024, 1024, 12, 12), (1, 300, 200, 4, 4), (2, 130, 77, 15, 5),
                                             (1, 256, 128, 2, 1), (1, 129, 1, 2, 2)])
def test_attention_tcgen05_kernel(b, lq, lk, hq, hkv):
    """The tcgen05 kernel (unmasked, single source) against the reference and the mma.sync kernel, with
    query tails (a second query tile partly or wholly empty) and key tails (a last key tile of 1..127)."""
    g = synthetic.generator(b * 7 + lq * 3 + lk)
    q = torch.randn(b, lq, hq * 64, generator=g).to(torch.bfloat16)
    k = torch.randn(b, lk, hkv * 64, generator=g).to(torch.bfloat16)
    v = torch.randn(b, lk, hkv * 64, generator=g).to(torch.bfloat16)
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    o_tc = ops.attention(qd, kd, vd, hq, hkv, impl=L.ATTN_TCGEN05)
    o_ms = ops.attention(qd, kd, vd, hq, hkv, impl=L.ATTN_MMA_SYNC)
    ref = _attn_ref(q, k, v, None, hq, hkv)
    assert cosine(o_tc, ref) >= 0.9999
    assert float((o_tc.cpu().float() - ref.float()).abs().max()) <= 2e-2
    assert float((o_tc.cpu().float() - o_ms.cpu().float()).abs().max()) <= 2e-2
    # fused int8 output (the out_proj input): the quantisation of the kernel's own bf16 context
    smooth = torch.rand(hq * 64, generator=g) + 0.5
    o2, qo = ops.attention(qd, kd, vd, hq, hkv, qo_smooth=smooth.to(DEV), qo_act=0.01,
                           qo_rsmooth=ops.reciprocal(smooth.to(DEV)), impl=L.ATTN_TCGEN05)
    assert torch.equal(o2.cpu(), o_tc.cpu())
    qo_ref = Q.smooth_quantize_activation(o2.cpu().reshape(-1, hq * 64), smooth, 0.01).reshape(b, lq, -1)
    assert torch.equal(qo.cpu(), qo_ref)


def test_attention_tcgen05_rejects_what_it_cannot_take():
    """The tcgen05 kernel reads byte masks as aligned 16-key runs of rows padded to 16 keys, from one key source:
    an unpadded mask row or a byte mask over two sources is refused (the automatic choice then takes the
    mma.sync kernel)."""
    q = torch.zeros(1, 128, 64, dtype=torch.bfloat16, device=DEV)
    k = torch.zeros(1, 100, 64, dtype=torch.bfloat16, device=DEV)
    mask = torch.ones(1, 128, 100, dtype=torch.bool, device=DEV)  # row stride 100: not padded
    with pytest.raises(L.SvlaError):
        ops.attention(q, k, k, 1, 1, mask=mask, impl=L.ATTN_TCGEN05)
    padded = torch.ones(1, 128, 256, dtype=torch.bool, device=DEV)[:, :, :228]
    with pytest.raises(L.SvlaError):
        ops.attention(q, k, k, 1, 1, mask=padded, k2=k[:, :, :], v2=k[:, :, :], impl=L.ATTN_TCGEN05)
    o = ops.attention(q, k, k, 1, 1, mask=mask)  # automatic: the mma.sync kernel takes it
    assert torch.isfinite(o.float()).all()


def _masked_case(seed, b, lq, l1, l2, hq, hkv):
    g = synthetic.generator(seed)
    q = torch.randn(b, lq, hq * 64, generator=g).to(torch.bfloat16)
    k1 = torch.randn(b, l1, hkv * 64, generator=g).to(torch.bfloat16)
    v1 = torch.randn(b, l1, hkv * 64, generator=g).to(torch.bfloat16)
    k2 = torch.randn(b, max(l2, 1), hkv * 64, generator=g).to(torch.bfloat16)[:, :l2]
    v2 = torch.randn(b, max(l2, 1), hkv * 64, generator=g).to(torch.bfloat16)[:, :l2]
    pad = torch.rand(b, l1, generator=g) > 0.25
    pad[:, -1] = True
    return g, q, k1, v1, k2, v2, pad


@pytest.mark.parametrize("b,lq,l1,l2,hq,hkv", [(3, 50, 177, 50, 15, 5), (2, 50, 177, 0, 15, 5),
                                               (2, 7, 70, 9, 4, 2), (1, 130, 200, 30, 6, 6)])
def test_attention_tcgen05_structured_mask(b, lq, l1, l2, hq, hkv):
    """The action expert's structured mask on tcgen05 (GQA rows packed query-major, the prefix keys and the
    chunk's own keys as two sources): against the reference attention on the equivalent byte mask and against
    the mma.sync kernel; a sample whose prefix keys are all padding gives its queries only the causal keys."""
    g, q, k1, v1, k2, v2, pad = _masked_case(b * 31 + lq + l1 + l2, b, lq, l1, l2, hq, hkv)
    # sample 0's prefix keys are all padding: with one key source every key is masked (uniform weights over
    # all keys, as the reference), with two its queries see only the causal chunk keys
    pad[0, :] = False
    full = torch.zeros(b, lq, l1 + l2, dtype=torch.bool)
    full[:, :, :l1] = pad[:, None, :]
    if l2:
        full[:, :, l1:] = torch.tril(torch.ones(lq, l2, dtype=torch.bool))
    key_rows = torch.zeros(b, (l1 + 15) // 16 * 16 + 16, dtype=torch.uint8)
    key_rows[:, :l1] = pad.to(torch.uint8)
    dev = lambda t: t.to(DEV)  # noqa: E731
    srcs = dict(k2=dev(k2), v2=dev(v2)) if l2 else {}
    kw = dict(key_mask=dev(key_rows)[:, :l1], mask_keys=l1, **srcs)
    o_tc = ops.attention(dev(q), dev(k1), dev(v1), hq, hkv, impl=L.ATTN_TCGEN05, **kw)
    o_ms = ops.attention(dev(q), dev(k1), dev(v1), hq, hkv, impl=L.ATTN_MMA_SYNC, **kw)
    kk, vv = (torch.cat([k1, k2], 1), torch.cat([v1, v2], 1)) if l2 else (k1, v1)
    ref = _attn_ref(q, kk, vv, full, hq, hkv)
    assert cosine(o_tc, ref) >= 0.9999
    assert float((o_tc.cpu().float() - ref.float()).abs().max()) <= 2e-2
    assert float((o_tc.cpu().float() - o_ms.cpu().float()).abs().max()) <= 2e-2
    assert _lib_device_error() == 0


def _lib_device_error():
    return L.device_error()


@pytest.mark.parametrize("b,lq,lk,hq,hkv", [(2, 177, 177, 15, 5), (1, 40, 100, 3, 1), (2, 129, 64, 2, 2)])
def test_attention_tcgen05_byte_mask(b, lq, lk, hq, hkv):
    """The VLM prefix's byte mask on tcgen05 (rows padded to 16 keys), with a fully masked query row and the
    fused int8 output: against the reference, the mma.sync kernel, and the same keys given as key flags."""
    g = synthetic.generator(b * 17 + lq + lk)
    q = torch.randn(b, lq, hq * 64, generator=g).to(torch.bfloat16)
    k = torch.randn(b, lk, hkv * 64, generator=g).to(torch.bfloat16)
    v = torch.randn(b, lk, hkv * 64, generator=g).to(torch.bfloat16)
    mask = torch.rand(b, lq, lk, generator=g) > 0.3
    mask[:, 0, :] = False
    ld = (lk + 15) // 16 * 16
    store = torch.zeros(b, lq, ld, dtype=torch.bool)
    store[:, :, :lk] = mask
    md = store.to(DEV)[:, :, :lk]
    qd, kd, vd = q.to(DEV), k.to(DEV), v.to(DEV)
    o_tc = ops.attention(qd, kd, vd, hq, hkv, mask=md, impl=L.ATTN_TCGEN05)
    o_ms = ops.attention(qd, kd, vd, hq, hkv, mask=md, impl=L.ATTN_MMA_SYNC)
    ref = _attn_ref(q, k, v, mask, hq, hkv)
    assert cosine(o_tc, ref) >= 0.9999
    assert float((o_tc.cpu().float() - ref.float()).abs().max()) <= 2e-2
    assert float((o_tc.cpu().float() - o_ms.cpu().float()).abs().max()) <= 2e-2
    smooth = torch.rand(hq * 64, generator=g) + 0.5
    o2, qo = ops.attention(qd, kd, vd, hq, hkv, mask=md, qo_smooth=smooth.to(DEV), qo_act=0.01,
                           qo_rsmooth=ops.reciprocal(smooth.to(DEV)), impl=L.ATTN_TCGEN05)
    assert torch.equal(o2.cpu(), o_tc.cpu())
    qo_ref = Q.smooth_quantize_activation(o2.cpu().reshape(-1, hq * 64), smooth, 0.01).reshape(b, lq, -1)
    assert torch.equal(qo.cpu(), qo_ref)
    # the same visibility as key flags for a mask that has the key-padding form
    pad = torch.rand(b, lk, generator=g) > 0.25
    fm = torch.zeros(b, lq, ld, dtype=torch.bool)
    fm[:, :, :lk] = pad[:, None, :]
    kr = torch.zeros(b, ld, dtype=torch.uint8)
    kr[:, :lk] = pad.to(torch.uint8)
    o_b = ops.attention(qd, kd, vd, hq, hkv, mask=fm.to(DEV)[:, :, :lk], impl=L.ATTN_TCGEN05)
    o_k = ops.attention(qd, kd, vd, hq, hkv, key_mask=kr.to(DEV)[:, :lk], mask_keys=lk, impl=L.ATTN_TCGEN05)
    assert torch.equal(o_b.cpu(), o_k.cpu())


def test_attention_two_sources_and_quant_out():
    g = synthetic.generator(31)
    b, lq, l1, l2, hq, hkv = 2, 50, 177, 50, 15, 5
    q = torch.randn(b, lq, hq * 64, generator=g).to(torch.bfloat16)
    k1 = torch.randn(b, l1, hkv * 64, generator=g).to(torch.bfloat16)
    v1 = torch.randn(b, l1, hkv * 64, generator=g).to(torch.bfloat16)
    k2 = torch.randn(b, l2, hkv * 64, generator=g).to(torch.bfloat16)
    v2 = torch.randn(b, l2, hkv * 64, generator=g).to(torch.bfloat16)
    mask = torch.ones(b, lq, l1 + l2, dtype=torch.bool)
    mask[:, :, l1:] = torch.tril(torch.ones(lq, l2, dtype=torch.bool))
    smooth = torch.rand(hq * 64, generator=g) + 0.5
    o, qo = ops.attention(q.to(DEV), k1.to(DEV), v1.to(DEV), hq, hkv, mask=mask.to(DEV), k2=k2.to(DEV), v2=v2.to(DEV),
                          qo_smooth=smooth.to(DEV), qo_act=0.01)
    _, qo_fast = ops.attention(q.to(DEV), k1.to(DEV), v1.to(DEV), hq, hkv, mask=mask.to(DEV), k2=k2.to(DEV),
                               v2=v2.to(DEV), qo_smooth=smooth.to(DEV), qo_act=0.01,
                               qo_rsmooth=ops.reciprocal(smooth.to(DEV)))
    assert torch.equal(qo, qo_fast)
    ref = _attn_ref(q, torch.cat([k1, k2], 1), torch.cat([v1, v2], 1), mask, hq, hkv)
    assert cosine(o, ref) >= 0.9999
    qo_ref = Q.smooth_quantize_activation(o.cpu().reshape(-1, hq * 64), smooth, 0.01).reshape(b, lq, -1)
    assert torch.equal(qo.cpu(), qo_ref)


# ----------------------------------------------------------------------------- RoPE / layout

def _ulp(dtype) -> float:
    return {torch.float32: 2.0 ** -23, torch.float16: 2.0 ** -10, torch.bfloat16: 2.0 ** -7}[dtype]


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("pos_dtype", [torch.int32, torch.int64])
def test_rope_layout_against_reference_kat(golden_dir, dtype, pos_dtype):
    """validate_fused_rope_layout_math.py inputs (seed 1000, L = 177) through the plugin-semantics kernel, in
    each data / position type the plugin takes (deploy/cuda/fused_rope_layout.cu:545-571).  fp32: within 1e-5
    of the KAT's own values; fp16 / bf16: within one ulp of the output type of the fp32 rotation of the
    same (rounded) inputs."""
    from oracle.model import apply_rope
    torch.manual_seed(1000)
    q_raw = torch.randn(1, 177, 15 * 64)
    k_raw = torch.randn(1, 177, 5 * 64)
    d = np.load(golden_dir / "rope_kat.npz")
    rows = torch.from_numpy(d["rows"])
    qx, kx = q_raw.to(dtype), k_raw.to(dtype)
    pos = torch.arange(177, dtype=pos_dtype)[None]
    q_out, k_out = ops.rope_layout(qx.to(DEV), kx.to(DEV), pos.to(DEV), 15, 5, 10000.0)
    assert q_out.dtype == dtype and q_out.shape == (1, 15, 177, 64) and k_out.shape == (1, 15, 64, 177)
    q_rot = q_out.cpu().float().transpose(1, 2)[0]                 # [177, 15, 64]
    k_rot = k_out.cpu().float().permute(0, 3, 1, 2)[0][:, ::3]     # [177, 5, 64] (undo the GQA expansion)
    if dtype == torch.float32:
        assert float((q_rot[rows] - torch.from_numpy(d["q_rot"])).abs().max()) <= 1e-5
        assert float((k_rot[rows] - torch.from_numpy(d["k_rot"])).abs().max()) <= 1e-5
    ref_q = apply_rope(qx.float().view(1, 177, 15, 64), pos, 10000.0)[0]
    ref_k = apply_rope(kx.float().view(1, 177, 5, 64), pos, 10000.0)[0]
    for got, ref in ((q_rot, ref_q), (k_rot, ref_k)):
        tol = ref.abs() * _ulp(dtype) + 2e-6
        assert bool(((got - ref).abs() <= tol + 1e-6 + (ref.abs() * 2e-6)).all())
    kk = k_out.cpu()
    for j in range(5):
        assert torch.equal(kk[0, 3 * j], kk[0, 3 * j + 1]) and torch.equal(kk[0, 3 * j], kk[0, 3 * j + 2])


def test_rope_layout_batched_positions_and_head_width():
    """Two samples with padded (repeated) positions and a 32-wide head."""
    from oracle.model import apply_rope
    g = synthetic.generator(44)
    b, l, hq, hkv, dh = 2, 50, 4, 2, 32
    q = torch.randn(b, l, hq * dh, generator=g)
    k = torch.randn(b, l, hkv * dh, generator=g)
    pad = torch.ones(b, l, dtype=torch.bool)
    pad[1, 30:40] = False
    pos = (torch.cumsum(pad.to(torch.int64), 1) - 1)
    q_out, k_out = ops.rope_layout(q.to(DEV), k.to(DEV), pos.to(DEV), hq, hkv, 100000.0, head_dim=dh)
    ref_q = apply_rope(q.view(b, l, hq, dh), pos, 100000.0).transpose(1, 2)
    ref_k = apply_rope(k.view(b, l, hkv, dh), pos, 100000.0).repeat_interleave(hq // hkv, 2).permute(0, 2, 3, 1)
    assert float((q_out.cpu() - ref_q).abs().max()) <= 1e-5
    assert float((k_out.cpu() - ref_k).abs().max()) <= 1e-5


def _rope_attention_case(b, l, hq, hkv, seed):
    from oracle.model import make_att_2d_masks
    g = synthetic.generator(seed)
    q = torch.randn(b, l, hq * 64, generator=g)
    k = torch.randn(b, l, hkv * 64, generator=g)
    v = torch.randn(b, l, hkv * 64, generator=g)
    pad = torch.ones(b, l, dtype=torch.bool)
    if b > 1:
        pad[1, l - 21:l - 1] = False   # padded language tokens: their rows are fully masked
    att = torch.zeros(b, l, dtype=torch.bool)
    att[:, -1] = True                  # the state token
    mask = make_att_2d_masks(pad, att)
    pos = torch.cumsum(pad.to(torch.int64), 1) - 1
    return q, k, v, pos, mask, pad


@pytest.mark.parametrize("dtype", [torch.float32, torch.float16, torch.bfloat16])
@pytest.mark.parametrize("pos_dtype", [torch.int32, torch.int64])
def test_fused_rope_attention_plugin_semantics(dtype, pos_dtype):
    """raw q / k / v + position ids + bool mask -> fp32 context [B, 15, L, 64]
    (deploy/cuda/fused_rope_layout.h:44-46; the v3 plugin, deploy/cuda/fused_attention_v3_real.cpp:104-116).
    Bar: max-abs <= 2e-5 against the fp32 restatement on the same (rounded) inputs -- fp32 summation order and
    the sin / cos / exp last bits differ; fully masked query rows are the mean of V."""
    from oracle.model import fused_rope_attention
    q, k, v, pos, mask, pad = _rope_attention_case(2, 177, 15, 5, 61)
    qx, kx, vx = q.to(dtype), k.to(dtype), v.to(dtype)
    ctx = ops.rope_attention(qx.to(DEV), kx.to(DEV), vx.to(DEV), pos.to(pos_dtype).to(DEV), mask.to(DEV), 15, 5)
    assert ctx.dtype == torch.float32 and ctx.shape == (2, 15, 177, 64)
    ref = fused_rope_attention(qx, kx, vx, pos, mask, 15, 5)
    assert float((ctx.cpu() - ref).abs().max()) <= 2e-5
    mean_v = vx.float().view(2, 177, 5, 64).mean(1).repeat_interleave(3, 1)    # [B, 15, 64]
    dead = (~pad[1]).nonzero().flatten()
    assert float((ctx.cpu()[1][:, dead] - mean_v[1][:, None]).abs().max()) <= 2e-5


def test_fused_rope_attention_fp32_mask_implicit_positions():
    """launchFusedRopeAttentionFp32MaskImplicitPos (deploy/cuda/fused_rope_layout.cu:433-543, :790-800):
    positions 0..L-1, fp32 mask with keep = value > 0.5."""
    from oracle.model import fused_rope_attention
    q, k, v, _, mask, _ = _rope_attention_case(1, 130, 15, 5, 62)
    pos = torch.arange(130)[None]
    mf = mask.float() * 0.75 + torch.rand(mask.shape, generator=synthetic.generator(2)) * 0.2
    ctx = ops.rope_attention(q.to(DEV), k.to(DEV), v.to(DEV), None, mf.to(DEV), 15, 5)
    ref = fused_rope_attention(q, k, v, pos, mf > 0.5, 15, 5)
    assert float((ctx.cpu() - ref).abs().max()) <= 2e-5


def test_rope_entry_points_reject_what_the_plugin_rejects():
    x = torch.zeros(1, 4, 64, device=DEV)
    pos = torch.zeros(1, 4, dtype=torch.int16, device=DEV)
    with pytest.raises(ValueError):
        ops.rope_layout(x, x, pos, 1, 1)            # int16 positions
    with pytest.raises(L.SvlaError):
        ops.rope_layout(x, x, pos.int(), 3, 2)      # 3 query heads over 2 kv heads
    with pytest.raises(L.SvlaError):
        ops.rope_attention(x, x, x, pos.int(), torch.ones(1, 4, 4, dtype=torch.bool, device=DEV), 1, 1,
                           head_dim=48)           # head_dim not a multiple of 32


# ----------------------------------------------------------------------------- W8A16 epilogues (the expert's)

def _w8a16_ref(x, w):
    """fp32 product of bf16 x with the reference's bf16(q * w_s) weights (deploy/linear_only_quant.py:119-137)."""
    lin = Q.W8A16Linear(w, None)
    return x.float() @ lin.weight.float().t()


@pytest.mark.parametrize("m,n,k", [(50, 720, 2048), (100, 720, 960), (3200, 720, 2048)])
def test_w8a16_resid(m, n, k):
    g = synthetic.generator(m + n + k + 1)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    res = torch.randn(m, n, generator=g).to(torch.bfloat16)
    qw, ws = ops.pack_weight_i8(w.to(DEV))
    out = res.to(DEV).clone()
    ops.gemm(ops.gemm_desc(L.KIND_W8A16, L.EPI_RESID, m, k, [ops.Seg(a=x.to(DEV), b=qw, out=out, n=n, wscale=ws)],
                           resid=out, ldr=n))
    y = _w8a16_ref(x, w)
    ref = (y.to(torch.bfloat16).float() + res.float()).to(torch.bfloat16)
    # one bf16 ulp of y (its rounding may differ after a different fp32 summation order and survives
    # cancellation against the residual) plus one ulp of the sum
    d = (out.cpu().float() - ref.float()).abs()
    tol = (y.abs() + ref.float().abs()) * 2.0 ** -7 + 1e-5 * float(ref.float().abs().max())
    assert bool((d <= tol).all()), float((d > tol).float().mean())


@pytest.mark.parametrize("m,n,k", [(50, 2048, 720), (100, 2048, 720), (3200, 2048, 720)])
def test_w8a16_silu_mul_pair(m, n, k):
    g = synthetic.generator(m + n + k + 2)
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    wg = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    wu = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
    qg, sg_ = ops.pack_weight_i8(wg.to(DEV))
    qu, su = ops.pack_weight_i8(wu.to(DEV))
    xd = x.to(DEV)
    h = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
    ops.gemm(ops.gemm_desc(L.KIND_W8A16, L.EPI_SILU_MUL, m, k,
                           [ops.Seg(a=xd, b=qg, out=h, n=n, wscale=sg_), ops.Seg(a=xd, b=qu, out=h, n=n, wscale=su)],
                           pair=True))
    gate = _w8a16_ref(x, wg).to(torch.bfloat16)
    up = _w8a16_ref(x, wu).to(torch.bfloat16)
    ref = F.silu(gate) * up
    # three bf16 roundings (gate, silu(gate), product): a one-ulp flip upstream can leave two at the end
    ok, frac = bf16_ulp_close(h, ref, ulps=2.0, atol=1e-5)
    assert ok, frac


@pytest.mark.parametrize("m", [50, 100, 3200])
def test_w8a16_rope_qkv(m):
    from oracle.model import apply_rope
    g = synthetic.generator(m + 3)
    k = 720
    x = torch.randn(m, k, generator=g).to(torch.bfloat16)
    pos = (177 + torch.arange(m) % 50).to(torch.int32)
    cs = ops.rope_table(256, 10000.0, DEV)
    segs, refs = [], []
    xd = x.to(DEV)
    for n, rope in ((960, 1), (320, 1), (320, 0)):
        w = (torch.randn(n, k, generator=g) * 0.02).to(torch.bfloat16)
        qw, ws = ops.pack_weight_i8(w.to(DEV))
        out = torch.empty(m, n, dtype=torch.bfloat16, device=DEV)
        segs.append(ops.Seg(a=xd, b=qw, out=out, n=n, wscale=ws, rope=rope))
        y = _w8a16_ref(x, w).to(torch.bfloat16)
        yr = apply_rope(y.view(1, m, n // 64, 64), pos.long()[None]).reshape(m, n) if rope else y
        refs.append((yr, y, rope))
    ops.gemm(ops.gemm_desc(L.KIND_W8A16, L.EPI_ROPE, m, k, segs, rope_cs=cs, pos=pos.to(DEV), max_pos=256))
    for s_, (ref, y, rope) in zip(segs, refs):
        rope_close(s_.out, ref, y, rope)


# ----------------------------------------------------------------------------- W8A16 as a bf16 GEMM

@pytest.mark.parametrize("n,k", [(720, 2048), (960, 720), (16, 8)])
def test_dequant_weight_bit_exact(n, k):
    g = synthetic.generator(n + k + 7)
    w = (torch.randn(n, k, generator=g) * 0.03).to(torch.bfloat16)
    lin = Q.W8A16Linear(w, None)
    qw, ws = ops.pack_weight_i8(w.to(DEV))
    assert torch.equal(ops.dequant_weight_bf16(qw, ws).cpu(), lin.weight)


@pytest.mark.parametrize("epi,m,n,k", [("resid", 640, 720, 2048), ("silu_mul", 640, 2048, 720),
                                       ("rope", 640, 960, 720), ("bf16", 700, 320, 960)])
def test_w8a16_equals_bf16_gemm_on_dequantized_weight(epi, m, n, k):
    """The large-M form of a W8A16 linear (a bf16 GEMM on bf16(q * wscale)) gives the same bits as the
    int8-operand kernel: both feed identical bf16 operands to the same MMA sequence."""
    g = synthetic.generator(m + n + k + 11)
    x = torch.randn(m, k, generator=g).to(DEV, torch.bfloat16)
    ws_, bs_ = [], []
    for _ in range(2 if epi == "silu_mul" else 1):
        qw, sc = ops.pack_weight_i8((torch.randn(n, k, generator=g) * 0.02).to(DEV, torch.bfloat16))
        ws_.append((qw, sc, ops.dequant_weight_bf16(qw, sc)))
        bs_.append((torch.randn(n, generator=g) * 0.02).to(DEV, torch.bfloat16))
    res = torch.randn(m, n, generator=g).to(DEV, torch.bfloat16)
    pos = (177 + torch.arange(m) % 50).to(DEV, torch.int32)
    cs = ops.rope_table(256, 10000.0, DEV)
    e = {"resid": L.EPI_RESID, "silu_mul": L.EPI_SILU_MUL, "rope": L.EPI_ROPE, "bf16": L.EPI_BF16}[epi]
    outs = []
    for kind in (L.KIND_W8A16, L.KIND_BF16):
        out = res.clone()
        segs = [ops.Seg(a=x, b=qw if kind == L.KIND_W8A16 else deq, out=out, n=n,
                        wscale=sc if kind == L.KIND_W8A16 else None, bias=b, rope=1 if epi == "rope" else 0)
                for (qw, sc, deq), b in zip(ws_, bs_)]
        extra = {"resid": dict(resid=out, ldr=n), "silu_mul": dict(pair=True),
                 "rope": dict(rope_cs=cs, pos=pos, max_pos=256), "bf16": {}}[epi]
        ops.gemm(ops.gemm_desc(kind, e, m, k, segs, **extra))
        outs.append(out.cpu())
    assert torch.equal(outs[0], outs[1])


# ----------------------------------------------------------------------------- split-K

@pytest.mark.parametrize("m,n,k,splits", [(50, 720, 2048, 0), (50, 960, 768, 3), (177, 320, 1024, 4), (7, 64, 384, 2)])
def test_split_k_i8_is_bit_exact(m, n, k, splits):
    """int32 partial sums are exact: split-K int8 GEMMs equal the single-pass kernel bit for bit, and the
    workspace counters are back at zero after every launch."""
    g = synthetic.generator(m * 3 + n + k + splits)
    a, w = _rand_i8((m, k), g).to(DEV), _rand_i8((n, k), g).to(DEV)
    ws = ops.splitk_workspace(8 << 20, DEV)
    outs = []
    for sk, wsp in ((1, None), (splits, ws)):
        acc = torch.empty(m, n, dtype=torch.int32, device=DEV)
        extra = dict(split_k=sk) if wsp is None else dict(split_k=sk, workspace=wsp, workspace_bytes=wsp.numel())
        ops.gemm(ops.gemm_desc(L.KIND_I8, L.EPI_I32, m, k, [ops.Seg(a=a, b=w, out=acc, n=n)], **extra))
        outs.append(acc.cpu())
    assert torch.equal(outs[0], outs[1])
    assert torch.equal(outs[0], Q.int_gemm(a.cpu(), w.cpu()))
    assert int(ws[:L.SPLITK_COUNTER_BYTES].count_nonzero()) == 0


@pytest.mark.parametrize("kind,epi,m,n,k", [(L.KIND_W8A16, "resid", 50, 720, 2048), (L.KIND_BF16, "silu_mul", 50, 2048, 720),
                                            (L.KIND_BF16, "rope", 50, 960, 720), (L.KIND_BF16, "resid", 100, 720, 960),
                                            (L.KIND_I8, "gelu_quant", 64, 1024, 2048)])
def test_split_k_epilogues_match_single_pass(kind, epi, m, n, k):
    """Split-K sums the fp32 partials in another order than one K loop: the bf16 outputs agree with the
    single-pass kernel to bf16 rounding (bounded by |y| where a residual or a rotation cancels); int8
    accumulators are exact, so I8 results agree bit for bit."""
    g = synthetic.generator(m + n + k + kind)
    if kind == L.KIND_I8:
        x = _rand_i8((m, k), g).to(DEV)
    else:
        x = torch.randn(m, k, generator=g).to(DEV, torch.bfloat16)
    wts = []
    for _ in range(2 if epi == "silu_mul" else 1):
        w = (torch.randn(n, k, generator=g) * 0.02).to(DEV, torch.bfloat16)
        wts.append((w, None) if kind == L.KIND_BF16 else ops.pack_weight_i8(w))
    res = torch.randn(m, n, generator=g).to(DEV, torch.bfloat16)
    pos = (177 + torch.arange(m) % 50).to(DEV, torch.int32)
    cs = ops.rope_table(256, 10000.0, DEV)
    smooth = (torch.rand(n, generator=g) + 0.5).to(DEV)
    ws = ops.splitk_workspace(16 << 20, DEV)
    e = {"resid": L.EPI_RESID, "silu_mul": L.EPI_SILU_MUL, "rope": L.EPI_ROPE, "gelu_quant": L.EPI_GELU_QUANT}[epi]
    outs = []
    for split in (1, 0):
        out = res.clone()
        qout = torch.zeros(m, n, dtype=torch.int8, device=DEV)
        segs = [ops.Seg(a=x, b=b, out=None if epi == "gelu_quant" else out, n=n, wscale=sc, act_scale=0.02,
                        rope=1 if epi == "rope" else 0) for b, sc in wts]
        extra = {"resid": dict(resid=out, ldr=n), "silu_mul": dict(pair=True),
                 "rope": dict(rope_cs=cs, pos=pos, max_pos=256),
                 "gelu_quant": dict(q_smooth=smooth, q_rsmooth=ops.reciprocal(smooth), q_act=0.05, qout=qout, ldq=n)}[epi]
        ops.gemm(ops.gemm_desc(kind, e, m, k, segs, split_k=split, workspace=ws, workspace_bytes=ws.numel(), **extra))
        outs.append((out.cpu(), qout.cpu()))
    assert int(ws[:L.SPLITK_COUNTER_BYTES].count_nonzero()) == 0
    a0, a1 = outs[0][0].float(), outs[1][0].float()
    if kind == L.KIND_I8:
        assert torch.equal(outs[0][1], outs[1][1])
    elif epi == "resid":
        # a one-ulp flip of bf16(y) survives cancellation against the residual: bound it by |y|
        r = res.cpu().float()
        tol = ((a0 - r).abs() + a0.abs()) * 2.0 ** -7 + 1e-5 * float(a0.abs().max())
        assert bool(((a1 - a0).abs() <= tol).all()), float(((a1 - a0).abs() > tol).float().mean())
    elif epi == "rope":
        # x1 cos - x2 sin cancels: bound the difference by the (rotation-invariant) norm of each pair
        a0v, a1v = a0.view(m, n // 64, 2, 32), a1.view(m, n // 64, 2, 32)
        pn = (a0v[:, :, 0] ** 2 + a0v[:, :, 1] ** 2).sqrt().unsqueeze(2)
        tol = pn * 2.0 ** -7 + 1e-5 * float(a0.abs().max())
        assert bool(((a1v - a0v).abs() <= tol).all()), float(((a1v - a0v).abs() > tol).float().mean())
    else:
        ok, frac = bf16_ulp_close(outs[1][0], outs[0][0], ulps=2.0, atol=1e-5)
        assert ok, frac


@pytest.mark.parametrize("two_sources", [True, False])
def test_structured_mask_equals_byte_mask(two_sources):
    """Key padding over the prefix keys plus causal order over the chunk keys, given as one row of key flags
    per sample, gives the same bits as the equivalent [B, Lq, Lk] byte mask (the action expert's masks)."""
    g = synthetic.generator(77 + int(two_sources))
    b, lq, l1, hq, hkv = 3, 50, 177, 15, 5
    l2 = lq if two_sources else 0
    q = torch.randn(b, lq, hq * 64, generator=g).to(DEV, torch.bfloat16)
    k1 = torch.randn(b, l1, hkv * 64, generator=g).to(DEV, torch.bfloat16)
    v1 = torch.randn(b, l1, hkv * 64, generator=g).to(DEV, torch.bfloat16)
    k2 = torch.randn(b, max(l2, 1), hkv * 64, generator=g).to(DEV, torch.bfloat16)[:, :l2]
    v2 = torch.randn(b, max(l2, 1), hkv * 64, generator=g).to(DEV, torch.bfloat16)[:, :l2]
    pad = torch.rand(b, l1, generator=g) > 0.25
    pad[:, -1] = True
    full = torch.zeros(b, lq, l1 + l2, dtype=torch.bool)
    full[:, :, :l1] = pad[:, None, :]
    if two_sources:
        full[:, :, l1:] = torch.tril(torch.ones(lq, l2, dtype=torch.bool))
    srcs = dict(k2=k2, v2=v2) if two_sources else {}
    mma = L.ATTN_MMA_SYNC  # the same kernel on both forms (the byte mask here has unpadded rows)
    o_byte = ops.attention(q, k1, v1, hq, hkv, mask=full.to(DEV), impl=mma, **srcs)
    key_rows = torch.zeros(b, 192, dtype=torch.uint8)
    key_rows[:, :l1] = pad.to(torch.uint8)
    o_key = ops.attention(q, k1, v1, hq, hkv, key_mask=key_rows.to(DEV)[:, :l1], mask_keys=l1, impl=mma, **srcs)
    assert torch.equal(o_byte.cpu(), o_key.cpu())


@pytest.mark.parametrize("rows,k,calls", [(1, 8, 3), (2, 13, 2), (177, 960, 4), (1024, 768, 2), (4096, 40, 1)])
@pytest.mark.parametrize("q", [0.9999, 0.5, 0.0, 1.0, 0.37])
def test_channel_percentile_bit_exact_with_torch_quantile(rows, k, calls, q):
    """svla_channel_percentile: per call, amax and torch.quantile(|x|, q) (the oracle's collector statistic),
    max-accumulated over calls -- bit-exact in fp32.  Inputs carry ties (bf16 rounding of a narrow range),
    exact zeros and a ragged channel count."""
    g = torch.Generator().manual_seed(rows * 7 + k)
    x = (torch.randn(calls * rows, k, generator=g) * torch.linspace(0.01, 40.0, k)).to(torch.bfloat16)
    x[::5, ::3] = 0
    x[1::7] = x[1::7].float().clamp(-0.5, 0.5).to(torch.bfloat16)  # many equal values
    amax = torch.zeros(k, device=DEV)
    pamax = torch.zeros(k, device=DEV)
    ops.channel_percentile(x.to(DEV), rows, q, amax, pamax)
    ref_a = torch.zeros(k)
    ref_p = torch.zeros(k)
    for c in range(calls):
        a, p = Q.per_channel_percentile_amax(x[c * rows:(c + 1) * rows], q * 100.0)
        ref_a = torch.maximum(ref_a, a)
        ref_p = torch.maximum(ref_p, p)
    assert torch.equal(amax.cpu(), ref_a)
    assert torch.equal(pamax.cpu(), ref_p)


def test_channel_percentile_strided_rows_and_rejects():
    """A row-strided view (a column slice of a wider buffer) reads only its own channels; bad shapes are
    refused by the C ABI before any launch."""
    x = torch.randn(354, 1000, dtype=torch.bfloat16)
    v = x[:, 16:976]
    amax = torch.zeros(960, device=DEV)
    pamax = torch.zeros(960, device=DEV)
    xd = x.to(DEV)
    ops.channel_percentile(xd[:, 16:976], 177, 0.9999, amax, pamax)
    ra, rp = [torch.maximum(*t) for t in zip(Q.per_channel_percentile_amax(v[:177], 99.99),
                                              Q.per_channel_percentile_amax(v[177:], 99.99))]
    assert torch.equal(amax.cpu(), ra) and torch.equal(pamax.cpu(), rp)
    lib = L.lib()
    assert lib.svla_channel_percentile(ops._p(xd), 1000, 1, 4097, 8, 0.5, ops._p(amax), ops._p(pamax), 0) != 0
    assert lib.svla_channel_percentile(ops._p(xd), 4, 1, 8, 8, 0.5, ops._p(amax), ops._p(pamax), 0) != 0
    assert lib.svla_channel_percentile(ops._p(xd), 1000, 1, 8, 8, 1.5, ops._p(amax), ops._p(pamax), 0) != 0


@pytest.mark.parametrize("batch,n_img,n_lang,chunk", [(1, 64, 48, 50), (3, 64, 48, 50), (2, 5, 7, 3)])
def test_build_masks_match_the_reference_mask_formulas(batch, n_img, n_lang, chunk):
    """svla_build_masks against make_att_2d_masks / cumsum(pad) - 1 (deploy/diagnose_3_4_numeric_baseline.py:42-46)
    and the suffix rules; padding bytes of every 16-byte row stay 0."""
    from oracle.model import make_att_2d_masks
    g = torch.Generator().manual_seed(batch * 100 + n_img)
    m0 = torch.randint(0, 2, (batch,), generator=g, dtype=torch.uint8)
    m1 = torch.ones(batch, dtype=torch.uint8)
    lang = (torch.rand(batch, n_lang, generator=g) > 0.3).to(torch.uint8)
    Lp, Ls = 2 * n_img + n_lang + 1, chunk
    ld = lambda n: (n + 15) // 16 * 16  # noqa: E731
    pm = torch.full((batch, Lp, ld(Lp)), 7, dtype=torch.uint8, device=DEV)
    sm = torch.full((batch, Ls, ld(Lp + Ls)), 7, dtype=torch.uint8, device=DEV)
    cm = torch.full((batch, Ls, ld(Lp)), 7, dtype=torch.uint8, device=DEV)
    pp = torch.empty(batch, Lp, dtype=torch.int32, device=DEV)
    sp = torch.empty(batch, Ls, dtype=torch.int32, device=DEV)
    cp = torch.empty(batch, Ls, dtype=torch.int32, device=DEV)
    d = [t.to(DEV) for t in (m0, m1, lang)]
    rc = L.lib().svla_build_masks(d[0].data_ptr(), d[1].data_ptr(), d[2].data_ptr(), batch, n_img, n_lang, chunk,
                                  pm.data_ptr(), pp.data_ptr(), sm.data_ptr(), cm.data_ptr(), sp.data_ptr(),
                                  cp.data_ptr(), ops._stream())
    assert rc == 0, L.lib().svla_last_error()
    pad = torch.cat([m0[:, None].expand(batch, n_img), m1[:, None].expand(batch, n_img), lang,
                     torch.ones(batch, 1, dtype=torch.uint8)], dim=1).bool()
    att = torch.zeros(batch, Lp, dtype=torch.bool)
    att[:, -1] = True
    pm, sm, cm = pm.cpu(), sm.cpu(), cm.cpu()
    assert torch.equal(pm[:, :, :Lp].bool(), make_att_2d_masks(pad, att))
    assert torch.equal(pp.cpu().long(), torch.cumsum(pad.long(), dim=1) - 1)
    causal = torch.arange(Ls)[None, :] <= torch.arange(Ls)[:, None]
    want_self = torch.cat([pad[:, None, :].expand(batch, Ls, Lp), causal[None].expand(batch, Ls, Ls)], dim=2)
    assert torch.equal(sm[:, :, :Lp + Ls].bool(), want_self)
    assert torch.equal(cm[:, :, :Lp].bool(), pad[:, None, :].expand(batch, Ls, Lp))
    assert torch.equal(sp.cpu().long(), pad.long().sum(1, keepdim=True) + torch.arange(Ls)[None])
    assert torch.equal(cp.cpu().long(), torch.arange(Ls)[None].expand(batch, Ls))
    for t, n in ((pm, Lp), (sm, Lp + Ls), (cm, Lp)):
        assert int(t[:, :, n:].sum()) == 0 and int(t.max()) <= 1
