#!/usr/bin/env python3
"""Benchmark of the quantized SmolVLA sample_actions path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--batch 64] [--impl svla|reference]
    torchrun --nproc-per-node N bench.py --gpus N ...          (one process per GPU)

Metric: action chunks/s at batch 64 independent synthetic observations per GPU (whole job, weak scaling,
no collective on the data path), with batch-1 sample_actions p50 latency reported beside it.  A "step" is
one sample_actions call at batch 64 (SigLIP on 128 images, 16 text layers, 10 flow steps x 16 expert
layers) replayed as one CUDA graph; inputs and activations (> 2 GB) exceed L2, so no flush is needed.

--impl reference times the CPU oracle (restatement of the reference's fake-quant path) on the host cores
on rank 0 only: each step is one observation of the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time
from datetime import timedelta
from pathlib import Path

import torch
import torch.distributed as dist

REPO = Path(__file__).resolve().parent
sys.path.insert(0, str(REPO))

METRIC = "action chunks/s at bs64 per GPU (sample_actions, SmolVLA SmoothQuant W8A8/W8A16)"
UNIT = "chunks/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--impl", default="svla", choices=["svla", "reference"])
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--calib-samples", type=int, default=4)
    ap.add_argument("--b1-iters", type=int, default=30)
    ap.add_argument("--cpu-iters", type=int, default=30)
    ap.add_argument("--cpu-warmup", type=int, default=3)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


def dist_env():
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return rank, world, local


PG_TIMEOUT_S = 120  # ranks that wait for a missing peer end with an error instead of hanging


def init_ranks(world: int, backend: str, device=None, timeout_s: float = PG_TIMEOUT_S) -> None:
    """One process per GPU (nccl) or per CPU rank (gloo, tests); rendezvous from the torchrun environment.  A
    collective that waits for a rank which has died or hangs ends with an error after `timeout_s`."""
    if world > 1:
        kw = {"device_id": device} if device is not None else {}
        dist.init_process_group(backend, timeout=timedelta(seconds=timeout_s), **kw)


def max_over_ranks(value: float, world: int, device="cpu") -> float:
    """The slowest rank's time: every rank takes this step (same collective, same order) after its timed
    region."""
    if world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(units_per_rank: int, world: int, steps: int, ms: float) -> float:
    """Units per second of the whole job: every rank's units over the slowest rank's time."""
    return units_per_rank * world * steps / (ms / 1e3)


def arm_config(cfg, batch: int, world: int) -> dict:
    """The `config` of the bench line, shared by both arms."""
    return {"workload": f"sample_actions bs{batch} per GPU: SigLIP {cfg.vis_layers}x{cfg.vis_hidden} on "
                        f"{batch * cfg.n_cams} images {cfg.image_size}px + connector, text {cfg.text_layers}x"
                        f"{cfg.hidden} (L={cfg.prefix_len}), expert {cfg.expert_layers}x{cfg.expert_hidden} x "
                        f"{cfg.num_steps} flow steps",
            "global_batch": batch * world, "seq_len": cfg.prefix_len, "parallelism": f"dp{world} (replicas, no collectives)",
            "l2": "inputs+activations > L2 (no flush needed)", "cuda_graph": True}


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms during the timed region."""

    FIELDS = "index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active," \
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown," \
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"

    def __init__(self, local_index: int):
        vis = os.environ.get("CUDA_VISIBLE_DEVICES", "")
        ids = [v.strip() for v in vis.split(",") if v.strip()]
        self.idx = ids[local_index] if local_index < len(ids) else str(local_index)
        self.proc = None
        self.lines: list[str] = []

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower() == "active":
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(smax) if smax else None,
                "reasons": sorted(reasons), "samples": len(sm)}


def make_observations(cfg, batch, seed):
    from smolvla_mujoco_libero_b200 import synthetic
    return synthetic.observations(batch, seed=seed, image_size=cfg.image_size, n_tokens=cfg.n_lang)


def cpu_baseline(cfg, state, scales_json, iters: int, warmup: int):
    """The oracle (CPU restatement of the reference fake-quant path) on the host cores, batch 1: `warmup`
    untimed calls, then `iters` timed calls (value from the median; p50 / p95 reported)."""
    from oracle import quant as Q
    from oracle.model import OracleSmolVLA
    torch.set_num_threads(os.cpu_count() or 1)
    m = OracleSmolVLA(cfg, state, Q.load_activation_scales_by_module(scales_json))
    o = make_observations(cfg, 1, 10_000)
    times = []
    for i in range(warmup + iters):
        t0 = time.perf_counter()
        m.sample_actions(o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)
        if i >= warmup:
            times.append(time.perf_counter() - t0)
    times.sort()
    p50 = statistics.median(times)
    p95 = times[min(len(times) - 1, int(round(0.95 * (len(times) - 1))))]
    return {"value": 1.0 / p50, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
            "p50_s_per_chunk": p50, "p95_s_per_chunk": p95, "iters": iters, "warmup": warmup,
            "sample": f"{iters} timed batch-1 sample_actions calls after {warmup} warm-up calls (the bs64 workload "
                      f"per observation): p50 {p50:.3f} s/chunk, p95 {p95:.3f} s/chunk, fp32/bf16 torch CPU oracle"}


def run_reference(args, rank, world):
    if rank != 0:
        return 0
    from smolvla_mujoco_libero_b200.calibrate import calibrate
    from smolvla_mujoco_libero_b200.config import BENCH
    from smolvla_mujoco_libero_b200.weights import random_weights
    from oracle import quant as Q
    from oracle.model import OracleSmolVLA, calibrate as oracle_calibrate
    torch.set_num_threads(os.cpu_count() or 1)
    cfg = BENCH
    state = random_weights(cfg, args.seed)
    js = oracle_calibrate(cfg, state, [make_observations(cfg, 1, 100 + i) for i in range(2)])
    m = OracleSmolVLA(cfg, state, Q.load_activation_scales_by_module(js))
    o = make_observations(cfg, 1, 10_000)
    for _ in range(args.warmup):
        m.sample_actions(o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        m.sample_actions(o.images, o.img_masks, o.lang_tokens, o.lang_masks, o.state, o.noise)
    el = time.perf_counter() - t0
    value = args.steps / el
    line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": el * 1e3 / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8/bf16", "data": "synthetic",
            "impl": "reference",
            "config": arm_config(cfg, args.batch, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": torch.get_num_threads(), "kind": "port",
                             "sample": "one batch-1 observation per step (bounded sample of the bs64 workload)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def time_kernel(fn, iters=20, warm=3):
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main():
    args = parse()
    rank, world, local = dist_env()
    if args.impl == "reference":
        return run_reference(args, rank, world)

    from smolvla_mujoco_libero_b200 import _lib as L
    from smolvla_mujoco_libero_b200.calibrate import calibrate, load_scale_json
    from smolvla_mujoco_libero_b200.config import BENCH
    from smolvla_mujoco_libero_b200.model import DeviceWeights, SmolVLARunner
    from smolvla_mujoco_libero_b200.weights import random_weights

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    init_ranks(world, "nccl", dev)
    cfg = BENCH
    B = args.batch
    peaks = json.loads((REPO / "MEASURED_PEAKS.json").read_text()) if (REPO / "MEASURED_PEAKS.json").exists() else {}

    state = random_weights(cfg, args.seed)
    js = calibrate(cfg, state, [make_observations(cfg, 1, 100 + i) for i in range(args.calib_samples)], device=dev)
    weights = DeviceWeights(cfg, state, load_scale_json(js), device=dev)

    # ---------------- batch-64 throughput (inputs resident in HBM)
    runner = SmolVLARunner(weights, B)
    obs = make_observations(cfg, B, 1_000_000 + rank * B)
    dev_in = ([im.to(dev) for im in obs.images], [m.to(dev) for m in obs.img_masks], obs.lang_tokens.to(dev),
              obs.lang_masks.to(dev), obs.state.to(dev), obs.noise.to(dev))
    runner.load_inputs(*dev_in)
    runner.capture()
    for _ in range(args.warmup):
        runner.run()
    torch.cuda.synchronize()
    clocks = ClockSampler(local)
    clocks.start()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ev0.record()
    for _ in range(args.steps):
        runner.run()
    ev1.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clk = clocks.stop()
    ms = max_over_ranks(ev0.elapsed_time(ev1), world, dev)
    assert torch.isfinite(runner.actions()).all(), "non-finite actions"
    assert L.device_error() == 0, "device error word set"
    value = whole_job_rate(B, world, args.steps, ms)
    launches = runner.n_launches * args.steps

    # ---------------- end to end through the C ABI (svla_engine_sample_actions on the packed weights) with host
    # (pinned) buffers: every step copies its observations in and its actions out inside the timed region
    import tempfile

    from smolvla_mujoco_libero_b200.checkpoint import save_packed
    from smolvla_mujoco_libero_b200.engine import NativeSampleActions
    with tempfile.TemporaryDirectory() as tmp:
        packed = Path(tmp) / f"packed_rank{rank}.safetensors"
        save_packed(weights, packed)
        engine = NativeSampleActions(packed, max_batch=B, device=dev)
    host = ([im.pin_memory() for im in obs.images], [m.pin_memory() for m in obs.img_masks],
            obs.lang_tokens.pin_memory(), obs.lang_masks.pin_memory(), obs.state.pin_memory(), obs.noise.pin_memory())
    out_host = torch.empty(B, cfg.chunk, cfg.max_action_dim, dtype=torch.float32).pin_memory()
    h2d = sum(t.numel() * t.element_size() for t in (*host[0], *host[1], *host[2:]))
    d2h = out_host.numel() * out_host.element_size()

    def e2e_step():
        engine.sample_actions(*host, out=out_host)

    for _ in range(max(2, args.warmup)):
        e2e_step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        e2e_step()
    e1.record()
    torch.cuda.synchronize()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1), world, dev)
    e2e_value = whole_job_rate(B, world, args.steps, e2e_ms)
    assert torch.equal(out_host, runner.actions().cpu()), "engine and runner disagree"

    # batch-1 end to end through the same call (one observation in from pinned host memory, its chunk out)
    o1 = make_observations(cfg, 1, 2_000_000 + rank)
    host1 = ([im.pin_memory() for im in o1.images], [m.pin_memory() for m in o1.img_masks],
             o1.lang_tokens.pin_memory(), o1.lang_masks.pin_memory(), o1.state.pin_memory(), o1.noise.pin_memory())
    out1 = torch.empty(1, cfg.chunk, cfg.max_action_dim, dtype=torch.float32).pin_memory()
    lat_e2e = []
    for i in range(args.b1_iters + 5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        engine.sample_actions(*host1, out=out1)
        b.record()
        torch.cuda.synchronize()
        if i >= 5:
            lat_e2e.append(a.elapsed_time(b))
    lat_e2e.sort()
    engine.close()

    # ---------------- batch-1 latency (p50 over individually timed calls, inputs resident)
    r1 = SmolVLARunner(weights, 1)
    r1.load_inputs([im.to(dev) for im in o1.images], [m.to(dev) for m in o1.img_masks], o1.lang_tokens.to(dev),
                   o1.lang_masks.to(dev), o1.state.to(dev), o1.noise.to(dev))
    r1.capture()
    lat = []
    for i in range(args.b1_iters + 5):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        r1.run()
        b.record()
        torch.cuda.synchronize()
        if i >= 5:
            lat.append(a.elapsed_time(b))
    lat.sort()
    p50 = lat[len(lat) // 2]
    p95 = lat[min(len(lat) - 1, int(round(0.95 * (len(lat) - 1))))]

    # ---------------- roofline of the dominant kernel (the SigLIP attention: the largest share of the batch-64
    # launch list) and of the largest GEMM, each timed live on its own with the step's own arguments
    roof = attention_roofline(runner, peaks)
    roof_b1 = flow_roofline(r1, peaks)
    roof_gemm = dominant_kernel_roofline(runner, peaks)

    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "int8/bf16", "data": "synthetic (seeded observations, random-init weights, GPU-calibrated SmoothQuant scales)",
        "config": arm_config(cfg, B, world),
        "batch1_p50_ms": p50, "batch1_p95_ms": p95, "batch1_e2e_p50_ms": lat_e2e[len(lat_e2e) // 2],
        "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                "call": "svla_engine_sample_actions (C ABI, pinned host buffers)"},
        "gpu_launches": launches,
        "roofline": roof,
        "roofline_gemm": roof_gemm,
        "roofline_batch1": roof_b1,
        "clocks": clk,
    }
    # the CPU baseline runs on rank 0 at N = 1 only: under torchrun the other ranks would wait for it at the
    # closing barrier for longer than the process-group timeout
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(cfg, state, js, args.cpu_iters, args.cpu_warmup)
    if rank == 0:
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


def measure_int8_peak(dev) -> float | None:
    """Dense int8 tensor throughput of the library GEMM (torch._int_mm, cuBLASLt) on 8192^3: a measurement
    reference for the roofline only, never on the product path."""
    try:
        a = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
        b = torch.randint(-128, 127, (8192, 8192), dtype=torch.int8, device=dev)
        ms = time_kernel(lambda: torch._int_mm(a, b), iters=10)
        return 2 * 8192 ** 3 / (ms / 1e3) / 1e12
    except Exception:  # noqa: BLE001 - any failure just means "no measured int8 peak"
        return None


def profile_traffic(name: str) -> float | None:
    """DRAM bytes (read + write) of one full-size launch of kernel `name` from the committed traffic table
    (profiles/traffic.json, written by `python -m smolvla_mujoco_libero_b200.profile --ncu-traffic` from an ncu
    capture), or None when the table has no entry."""
    f = REPO / "profiles" / "traffic.json"
    if not f.exists():
        return None
    entry = json.loads(f.read_text()).get(name)
    return None if entry is None else float(entry["dram_bytes_per_launch"])


def attention_roofline(runner, peaks):
    """The largest attention launch of the step (SigLIP self-attention, tcgen05 kernel) timed on its own with
    CUDA events.  Algorithmic work: 4 * B * Hq * Lq * Lk * 64 flops (Q.K^T and P.V)."""
    from smolvla_mujoco_libero_b200 import _lib as L
    best = None
    for fn, a in runner.launches:
        if fn is L.lib().svla_attention:
            d = a[0]
            lk = d.l1 + max(d.l2, 0)
            flops = 4.0 * d.batch * d.hq * d.lq * lk * 64
            if best is None or flops > best[0]:
                best = (flops, d)
    flops, d = best
    stream = torch.cuda.current_stream().cuda_stream
    import ctypes
    fn = L.lib().svla_attention
    ms = time_kernel(lambda: fn(ctypes.byref(d), stream), iters=20)
    achieved = flops / (ms / 1e3) / 1e12
    peak = float(peaks.get("bf16_tflops", 1590.0))
    src = "MEASURED_PEAKS.json bf16_tflops (burst: the kernel is timed alone)" if "bf16_tflops" in peaks \
        else "fallback 1.59 PFLOP/s"
    traffic = profile_traffic("attention_tc_siglip_b128")
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": traffic, "kernel": f"attention_tc B={d.batch} Hq={d.hq} Lq={d.lq} Lk={d.l1} d=64",
            "ms_per_launch": ms, "flops_per_launch": flops, "peak_source": src}


def flow_roofline(runner, peaks):
    """The batch-1 call's dominant kernel (svla_flow: the whole flow-matching loop, about two thirds of the batch-1
    launch list) timed on its own with CUDA events on the launch stream.  Algorithmic bytes: per flow step the
    expert layers' int8 weights (fragment order) with their fp32 scales, and the bf16 action / time projections,
    each read once; the prefix K/V once per call."""
    import ctypes

    from smolvla_mujoco_libero_b200 import _lib as L
    from smolvla_mujoco_libero_b200.config import EXPERT
    flows = [a[0] for fn, a in runner.launches if fn is L.lib().svla_flow]
    if not flows:
        return None
    d, c, w = flows[0], runner.cfg, runner.w
    E = c.expert_hidden
    per_step = 0
    for name, p in w.lin.items():
        if name.startswith(EXPERT + ".layers."):
            if c.is_cross_layer(int(name.split(".layers.")[1].split(".")[0])) and (".k_proj" in name or ".v_proj" in name):
                continue  # cross layers read the precomputed K/V projections, not these weights
            per_step += p.n * p.k + p.n * 4  # int8 weight + fp32 per-channel scale
    per_step += (E * c.max_action_dim * 2) * 2 + E * E * 2 * 2  # action in / out, time MLP (in: first E columns)
    kv = c.expert_layers * c.prefix_len * c.kv_dim * 2 * 2
    nbytes = per_step * c.num_steps + kv
    stream = torch.cuda.current_stream().cuda_stream
    fn = L.lib().svla_flow
    ms = time_kernel(lambda: fn(ctypes.byref(d), stream), iters=5)
    achieved = nbytes / (ms / 1e3) / 1e9
    peak = float(peaks.get("hbm_gbs", 6650.0))
    src = "MEASURED_PEAKS.json hbm_gbs" if "hbm_gbs" in peaks else "fallback 6.65 TB/s"
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": profile_traffic("flow_kernel_b1"), "kernel": f"flow_kernel batch {d.batch} x {c.num_steps} steps",
            "ms_per_launch": ms, "bytes_per_launch": nbytes, "peak_source": src}


def dominant_kernel_roofline(runner, peaks):
    """The largest W8A8 GEMM launch of the step (SigLIP fc1, GELU + int8 quant epilogue) timed on its own with
    CUDA events.  Algorithmic work: 2 * M * N * K int8 ops."""
    from smolvla_mujoco_libero_b200 import _lib as L
    best = None
    for fn, a in runner.launches:
        if fn is L.lib().svla_gemm:
            d = a[0]
            n = sum(d.seg[i].n for i in range(d.nseg))
            flops = 2.0 * d.m * n * d.k * (2 if d.pair else 1)
            if best is None or flops > best[0]:
                best = (flops, d)
    flops, d = best
    stream = torch.cuda.current_stream().cuda_stream
    import ctypes
    fn = L.lib().svla_gemm
    ms = time_kernel(lambda: fn(ctypes.byref(d), stream), iters=20)
    achieved = flops / (ms / 1e3) / 1e12
    int8 = d.kind == L.KIND_I8
    bf16 = float(peaks.get("bf16_tflops", 1590.0))
    extra = {}
    if int8:
        # the stated int8 peak: twice the measured dense bf16 GEMM rate (the tensor cores' int8 : bf16 ratio);
        # a library's int8 GEMM rate is reported beside it as a reference point, not used as the peak
        peak, src = 2 * bf16, "2 x MEASURED_PEAKS.json bf16_tflops (burst; int8 runs at twice the bf16 rate)"
        lib_int8 = measure_int8_peak(torch.device("cuda", torch.cuda.current_device()))
        if lib_int8 is not None:
            extra = {"cublaslt_int8_tops_in_run": lib_int8, "frac_of_cublaslt_int8": achieved / lib_int8}
    else:
        peak, src = bf16, "MEASURED_PEAKS.json bf16_tflops (burst)"
    return {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
            "traffic": profile_traffic("gemm_i8_gelu_quant_fc1_b64"),
            "kernel": f"gemm_sm100 kind={'i8' if int8 else d.kind} M={d.m} N={sum(d.seg[i].n for i in range(d.nseg))} K={d.k}",
            "ms_per_launch": ms, "peak_source": src, **extra}


if __name__ == "__main__":
    sys.exit(main())
