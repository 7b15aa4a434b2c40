"""Profiling driver: build the benchmark model and run sample_actions calls inside an NVTX range, or
time one operator on random inputs.

    python -m smolvla_mujoco_libero_b200.profile --batch 1 --iters 3 [--graph]
    python -m smolvla_mujoco_libero_b200.profile --op gemm --kind i8 --epi gelu_quant --m 16384 --n 3072 --k 768
    python -m smolvla_mujoco_libero_b200.profile --op attn --batch 16 --lq 1024 --lk 1024 --heads 12 --kv-heads 12
    python -m smolvla_mujoco_libero_b200.profile --op attn --batch 64 --lq 50 --lk 227 --heads 15 --kv-heads 5 --mask --mask-ld 240

Each call is wrapped in the NVTX range "sample_actions", so a profiler can capture exactly those launches
(e.g. ``ncu --nvtx --nvtx-include "sample_actions/" --metrics gpu__time_duration.sum ...``).  Prints the
per-call device time (CUDA events) and the number of kernel launches per call.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import _lib as L
from . import ops, synthetic
from .calibrate import calibrate, load_scale_json
from .config import BENCH
from .model import DeviceWeights, SmolVLARunner
from .weights import random_weights


EPIS = {"bf16": 0, "resid": 3, "gelu_quant": 5, "rope": 2, "silu_mul": 4}
KINDS = {"i8": 0, "bf16": 1, "w8a16": 2}


def time_op(fn, iters: int, reps: int = 20) -> list[float]:
    """Per-launch device time: `reps` back-to-back launches between two events (so host launch latency
    overlaps device work), repeated `iters` times."""
    fn()
    torch.cuda.synchronize()
    out = []
    for _ in range(iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("op")
        s.record()
        for _ in range(reps):
            fn()
        e.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        out.append(s.elapsed_time(e) / reps)
    return out


def op_gemm(a) -> dict:
    from . import _lib as L
    from . import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(0)
    kind, epi = KINDS[a.kind], EPIS[a.epi]
    adt = torch.int8 if kind == 0 else torch.bfloat16
    mk = lambda r, c, dt: (torch.randint(-100, 100, (r, c), generator=g, dtype=torch.int8) if dt == torch.int8  # noqa: E731
                           else torch.randn(r, c, generator=g).to(dt)).to(dev)
    A = mk(a.m, a.k, adt)
    B = mk(a.n, a.k, torch.bfloat16 if kind == 1 else torch.int8)
    ws = torch.rand(a.n, generator=g).to(dev) * 1e-3
    out = torch.empty(a.m, a.n, dtype=torch.bfloat16, device=dev)
    segs = [ops.Seg(a=A, b=B, out=out, n=a.n, wscale=ws, act_scale=0.01)]
    extra = {}
    if epi == 5:
        smooth = torch.rand(a.n, generator=g).to(dev) + 0.5
        qout = torch.empty(a.m, a.n, dtype=torch.int8, device=dev)
        segs[0].out = None
        extra = dict(q_smooth=smooth, q_rsmooth=ops.reciprocal(smooth), q_act=0.02, qout=qout, ldq=a.n)
    elif epi == 3:
        extra = dict(resid=out, ldr=a.n)
    elif epi == 4:
        segs.append(ops.Seg(a=A, b=B, out=out, n=a.n, wscale=ws, act_scale=0.01))
        extra = dict(pair=True)
    elif epi == 2:
        # q (n columns) and k, v (kv_n columns each) of one input, RoPE on q and k: the QKV projection
        segs[0].rope = 1
        for rope in (1, 0):
            Bk = mk(a.kv_n, a.k, torch.bfloat16 if kind == 1 else torch.int8)
            wk = torch.rand(a.kv_n, generator=g).to(dev) * 1e-3
            ok = torch.empty(a.m, a.kv_n, dtype=torch.bfloat16, device=dev)
            segs.append(ops.Seg(a=A, b=Bk, out=ok, n=a.kv_n, wscale=wk, act_scale=0.01, rope=rope))
        max_pos = 256
        pos = torch.randint(0, max_pos, (a.m,), generator=g, dtype=torch.int32).to(dev)
        extra = dict(rope_cs=ops.rope_table(max_pos, 100000.0, dev), pos=pos, max_pos=max_pos)
    if a.split_k != 1:
        ws = ops.splitk_workspace(64 << 20, dev)
        extra.update(split_k=a.split_k, workspace=ws, workspace_bytes=ws.numel())
    d = ops.gemm_desc(kind, epi, a.m, a.k, segs, block_n=a.block_n, cta_pair=a.cta_pair, **extra)
    ms = time_op(lambda: ops.gemm(d), a.iters)
    # phase clock stamps of CTA 0 from one more launch
    dbg = torch.zeros(32, dtype=torch.int64, device=dev)
    d.debug_clock = dbg.data_ptr()
    ops.gemm(d)
    torch.cuda.synchronize()
    c = dbg.cpu().tolist()
    d.debug_clock = None
    names = ["entry", "setup", "tma0", "full0", "conv0", "commit0", "epi_consts", "epi_acc", "epi_done", "sync_end", "dealloc",
             "sk_stored", "sk_bar", "sk_counted", "sk_last", "sk_notlast"]
    # MMA warp, accumulator buffer of tile i: wait begins / ends (a long wait = the epilogue sets the pace)
    names += [f"acc{i}_{w}" for i in range(8) for w in ("wait", "free")]
    phases = {names[i]: (c[i] - c[0]) if c[i] else None for i in range(len(names))}
    ops_count = 2.0 * a.m * a.k * (a.n * (2 if epi == 4 else 1) + (2 * a.kv_n if epi == 2 else 0))
    best = min(ms)
    return {"op": "gemm", "kind": a.kind, "epi": a.epi, "m": a.m, "n": a.n, "k": a.k, "split_k": a.split_k,
            "cta_pair": a.cta_pair, "ms": ms,
            "tflops_best": ops_count / (best / 1e3) / 1e12, "cta0_cycles": phases}


def op_norm(a) -> dict:
    """LayerNorm (or RMSNorm with --rms) fused with three SmoothQuant int8 outputs: the SigLIP q/k/v input."""
    from . import _lib as L
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(0)
    x = torch.randn(a.m, a.k, generator=g).to(dev, torch.bfloat16)
    w = (torch.rand(a.k, generator=g) + 0.5).to(dev, torch.bfloat16)
    b = None if a.rms else (torch.randn(a.k, generator=g) * 0.1).to(dev, torch.bfloat16)
    qs = [torch.empty(a.m, a.k, dtype=torch.int8, device=dev) for _ in range(3)]
    sm = [(torch.rand(a.k, generator=g) + 0.5).to(dev) for _ in range(3)]
    rs = [ops.reciprocal(t) for t in sm]
    d = L.NormDesc()
    d.x, d.ldx, d.weight, d.bias, d.eps = x.data_ptr(), a.k, w.data_ptr(), (b.data_ptr() if b is not None else None), 1e-6
    d.layernorm, d.m, d.k, d.nq, d.ldq = int(b is not None), a.m, a.k, 3, a.k
    for i in range(3):
        d.q[i], d.smooth[i], d.rsmooth[i], d.act[i] = qs[i].data_ptr(), sm[i].data_ptr(), rs[i].data_ptr(), 0.05
    ms = time_op(lambda: L.check(L.lib().svla_norm_quant(d, ops._stream()), "norm"), a.iters)
    nbytes = a.m * a.k * (2 + 3)
    return {"op": "norm", "m": a.m, "k": a.k, "ms": ms, "GBps_best": nbytes / (min(ms) / 1e3) / 1e9}


def op_attn(a) -> dict:
    from . import _lib as L
    from . import ops
    dev = torch.device("cuda", 0)
    g = torch.Generator(device="cpu").manual_seed(0)
    q = torch.randn(a.batch, a.lq, a.heads * 64, generator=g).to(torch.bfloat16).to(dev)
    k = torch.randn(a.batch, a.lk, a.kv_heads * 64, generator=g).to(torch.bfloat16).to(dev)
    v = torch.randn(a.batch, a.lk, a.kv_heads * 64, generator=g).to(torch.bfloat16).to(dev)
    mask = None
    if a.mask:
        # key padding (last 10% of keys masked) with the mask rows stored at a stride of `mask_ld` bytes
        ld = max(a.mask_ld, a.lk)
        full = torch.zeros(a.batch, a.lq, ld, dtype=torch.uint8)
        full[:, :, : a.lk - a.lk // 10] = 1
        mask = full.to(dev)[:, :, : a.lk]
    key_mask = None
    if a.prefix > 0:
        # the action expert's structured mask: padding flags over the first `prefix` keys (last 10% off),
        # causal order over the rest
        kf = torch.zeros(a.batch, (a.prefix + 15) // 16 * 16, dtype=torch.uint8)
        kf[:, : a.prefix - a.prefix // 10] = 1
        key_mask = kf.to(dev)
    impl = {"auto": L.ATTN_AUTO, "mma": L.ATTN_MMA_SYNC, "tc": L.ATTN_TCGEN05}[a.impl]
    ms = time_op(lambda: ops.attention(q, k, v, a.heads, a.kv_heads, mask=mask, key_mask=key_mask,
                                       mask_keys=a.prefix, impl=impl), a.iters)
    flops = 4.0 * a.batch * a.heads * a.lq * a.lk * 64
    # phase clock stamps of one CTA of the tcgen05 kernel (when that kernel runs)
    from . import _lib as L
    dbg = torch.zeros(96, dtype=torch.int64, device=dev)
    o = torch.empty(a.batch, a.lq, a.heads * 64, dtype=torch.bfloat16, device=dev)
    d = ops.attention_desc(q, k, v, a.batch, a.lq, a.heads, a.kv_heads, mask=mask, o=o)
    d.debug_clock = dbg.data_ptr()
    ops.attention_run(d)
    torch.cuda.synchronize()
    c = dbg.cpu().tolist()
    phases = {i: c[i] - c[0] for i in range(96) if c[i]} if c[0] else {}
    return {"op": "attn", "batch": a.batch, "lq": a.lq, "lk": a.lk, "heads": a.heads, "kv_heads": a.kv_heads,
            "mask": a.mask, "mask_ld": a.mask_ld, "prefix": a.prefix, "ms": ms, "tflops_best": flops / (min(ms) / 1e3) / 1e12,
            "cta_cycles": phases}


def summarize_launches(csv_path: str, top: int = 30) -> str:
    """Per-kernel launches, total device time and share from an ncu launch list
    (``--metrics gpu__time_duration.sum --csv``): the summary format of the committed profiles."""
    import csv
    import re
    rows = list(csv.reader(open(csv_path)))
    hi = next(i for i, r in enumerate(rows) if "Kernel Name" in r)
    h = rows[hi]
    ki, vi, ui = h.index("Kernel Name"), h.index("Metric Value"), h.index("Metric Unit")
    tot: dict[str, list] = {}
    for r in rows[hi + 1:]:
        if len(r) <= vi or r[vi] == "":
            continue
        v = float(r[vi].replace(",", ""))
        v = v / 1e3 if r[ui] in ("nsecond", "ns") else (v * 1e3 if r[ui] in ("msecond", "ms") else v)  # -> us
        name = re.sub(r"\(svla::[A-Za-z]+\)", "", r[ki]).replace("svla::", "")
        name = re.sub(r"\(GemmArgs\)|\(AttnTcArgs\)|\(AttnArgs\)|\(NormQuantArgs\)|\(MaskArgs\)", "", name)
        name = re.sub(r"\(.*\)$", "", name.replace("void ", ""))
        e = tot.setdefault(name, [0, 0.0])
        e[0] += 1
        e[1] += v
    total = sum(e[1] for e in tot.values())
    n = sum(e[0] for e in tot.values())
    out = [f"launches {n} total {total / 1e3:.3f} ms"]
    for name, (cnt, us) in sorted(tot.items(), key=lambda kv: -kv[1][1])[:top]:
        out.append(f"{name[:52]:52s} launches {cnt:5d} total {us / 1e3:9.3f} ms share {100 * us / total:5.1f}% "
                   f"avg {us / cnt:9.2f} us")
    return "\n".join(out)


_BYTE_UNITS = {"byte": 1.0, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9, "KB": 1e3, "MB": 1e6, "GB": 1e9}


def ncu_traffic(csv_path: str, kernel: str) -> tuple[float, int]:
    """Mean dram__bytes_read.sum + dram__bytes_write.sum per launch of the kernels whose name contains `kernel`
    in an `ncu -i <rep> --page raw --csv` export, and the number of launches."""
    import csv
    with open(csv_path, newline="") as f:
        rows = list(csv.DictReader(f))
    units = rows[0] if rows and not rows[0].get("ID", "").strip().isdigit() else {}
    tot, n = 0.0, 0
    for r in rows:
        if not r.get("ID", "").strip().isdigit() or kernel not in r.get("Kernel Name", ""):
            continue
        b = 0.0
        for m in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            b += float(r[m].replace(",", "")) * _BYTE_UNITS.get(units.get(m, "byte").strip(), 1.0)
        tot += b
        n += 1
    if n == 0:
        raise ValueError(f"no launch of {kernel!r} in {csv_path}")
    return tot / n, n


def update_traffic(json_path: str, key: str, csv_path: str, kernel: str, scale: float, note: str) -> dict:
    """Writes traffic[key] = {dram_bytes_per_launch: mean bytes x scale, ...} into the machine-readable traffic
    table that bench.py reads (the DRAM bytes of one full-size launch, from a capture of a smaller case scaled by
    the units processed when scale != 1)."""
    from pathlib import Path
    b, n = ncu_traffic(csv_path, kernel)
    path = Path(json_path)
    table = json.loads(path.read_text()) if path.exists() else {}
    table[key] = {"dram_bytes_per_launch": b * scale, "captured_bytes_per_launch": b, "scale": scale,
                  "launches": n, "kernel": kernel, "note": note}
    path.write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")
    return table[key]


FLOW_EVENTS = {1: "barrier_in", 2: "barrier_out", 3: "staged", 4: "mma", 5: "epilogue", 6: "attn", 7: "copied",
               8: "keys", 9: "attn_done"}


def flow_phase_names(cfg) -> list[str]:
    """Phase names of one flow step in kernel order (the kernel puts one grid barrier after each)."""
    names = ["action_in", "time_in", "time_out"]
    for _ in range(cfg.expert_layers):
        names += ["qkv", "attention", "o_proj", "gate_up", "down"]
    return names + ["action_out"]


def flow_events(r, cta: int = 0) -> dict:
    """Per-phase breakdown of one persistent flow kernel launch from its own globaltimer events (CTA 0 or the last
    CTA): for each phase kind, the mean microseconds from the barrier exit to each event, the barrier wait and
    the whole phase (barrier exit to next barrier exit)."""
    fd = next(args[0] for fn, args in r.launches if fn is L.lib().svla_flow)
    dbg = torch.zeros(2 * 1024 * 2, dtype=torch.int64, device=r.dev)
    fd.debug_clock = dbg.data_ptr()
    r._run_launches()
    torch.cuda.synchronize()
    fd.debug_clock = None
    ev = dbg.view(2, 1024, 2)[cta].cpu().tolist()
    ev = [(c, t) for c, t in ev if c]
    names = flow_phase_names(r.cfg)
    # phases start at each barrier exit (the first barrier, after x_t = noise, opens phase 0)
    starts = [i for i, (c, _) in enumerate(ev) if c == 2]
    acc: dict[str, dict[str, list[float]]] = {}
    for pi in range(len(starts) - 1):
        i0, i1 = starts[pi], starts[pi + 1]
        t0 = ev[i0][1]
        kind = names[pi % len(names)]
        d = acc.setdefault(kind, {})
        seen = set()
        for c, t in ev[i0 + 1:i1 + 1]:
            key = FLOW_EVENTS.get(c, str(c))
            if key in seen:
                continue
            seen.add(key)
            d.setdefault(key, []).append((t - t0) / 1e3)
        d.setdefault("phase", []).append((ev[i1][1] - t0) / 1e3)
    out = {k: {e: round(sum(v) / len(v), 3) for e, v in d.items()} | {"n": len(d["phase"])} for k, d in acc.items()}
    return {"cta": cta, "events": len(ev), "phases": len(starts) - 1, "mean_us_from_barrier_exit": out}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--op", default="sample_actions", choices=["sample_actions", "gemm", "attn", "norm"])
    ap.add_argument("--rms", action="store_true", help="--op norm: RMSNorm instead of LayerNorm")
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--calib-samples", type=int, default=1)
    ap.add_argument("--kind", default="i8", choices=list(KINDS))
    ap.add_argument("--epi", default="bf16", choices=list(EPIS))
    ap.add_argument("--m", type=int, default=16384)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=768)
    ap.add_argument("--kv-n", type=int, default=320, help="--epi rope: columns of the k and v segments")
    ap.add_argument("--block-n", type=int, default=0)
    ap.add_argument("--split-k", type=int, default=1, help="GEMM split-K: 1 off, 0 automatic, n splits")
    ap.add_argument("--cta-pair", type=int, default=0, help="GEMM CTA pairs: 0 automatic, 1 off, 2 on")
    ap.add_argument("--lq", type=int, default=1024)
    ap.add_argument("--lk", type=int, default=1024)
    ap.add_argument("--heads", type=int, default=12)
    ap.add_argument("--kv-heads", type=int, default=12)
    ap.add_argument("--mask", action="store_true")
    ap.add_argument("--mask-ld", type=int, default=0)
    ap.add_argument("--impl", default="auto", choices=["auto", "mma", "tc"], help="--op attn: kernel choice")
    ap.add_argument("--prefix", type=int, default=0, help="--op attn: structured mask, key padding over this many "
                    "prefix keys and causal order over the rest")
    ap.add_argument("--summarize", default=None, help="print the per-kernel summary of an ncu launch-list CSV")
    ap.add_argument("--ncu-traffic", nargs=3, metavar=("CSV", "KERNEL", "KEY"), default=None,
                    help="update the traffic table (--traffic-json) entry KEY from an ncu raw CSV export")
    ap.add_argument("--traffic-json", default="profiles/traffic.json")
    ap.add_argument("--scale", type=float, default=1.0, help="--ncu-traffic: full-size units / captured units")
    ap.add_argument("--note", default="", help="--ncu-traffic: the capture (case, command)")
    ap.add_argument("--flow-events", action="store_true", help="sample_actions at batch 1: per-phase breakdown of "
                    "the persistent flow kernel from its own globaltimer events")
    a = ap.parse_args()
    if a.summarize:
        print(summarize_launches(a.summarize))
        return
    if a.ncu_traffic:
        csv_path, kernel, key = a.ncu_traffic
        print(json.dumps(update_traffic(a.traffic_json, key, csv_path, kernel, a.scale, a.note)))
        return
    if a.op == "gemm":
        print(json.dumps(op_gemm(a)))
        return
    if a.op == "norm":
        print(json.dumps(op_norm(a)))
        return
    if a.op == "attn":
        print(json.dumps(op_attn(a)))
        return
    cfg = BENCH
    dev = torch.device("cuda", 0)
    obs = lambda b, s: synthetic.observations(b, seed=s, image_size=cfg.image_size, n_tokens=cfg.n_lang)  # noqa: E731
    state = random_weights(cfg, 0)
    js = calibrate(cfg, state, [obs(1, 100 + i) for i in range(a.calib_samples)], device=dev)
    r = SmolVLARunner(DeviceWeights(cfg, state, load_scale_json(js), device=dev), a.batch)
    o = obs(a.batch, 5)
    r.load_inputs([im.to(dev) for im in o.images], [m.to(dev) for m in o.img_masks], o.lang_tokens.to(dev),
                  o.lang_masks.to(dev), o.state.to(dev), o.noise.to(dev))
    if a.graph:
        r.capture()
    r.run()
    torch.cuda.synchronize()
    times = []
    for _ in range(a.iters):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.nvtx.range_push("sample_actions")
        s.record()
        r.run()
        e.record()
        torch.cuda.nvtx.range_pop()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    print(json.dumps({"batch": a.batch, "launches_per_call": r.n_launches, "ms_per_call": times, "graph": a.graph}))
    if a.flow_events and r.flow:
        for cta in (0, 1):
            print(json.dumps(flow_events(r, cta)))


if __name__ == "__main__":
    main()
