"""Profiling driver: build the benchmark model and run sample_actions calls inside an NVTX range.

    python -m smolvla_mujoco_libero_b200.profile --batch 1 --iters 3 [--graph]

Each call is wrapped in the NVTX range "sample_actions", so a profiler can capture exactly those launches
(e.g. ``ncu --nvtx --nvtx-include "sample_actions/" --metrics gpu__time_duration.sum ...``).  Prints the
per-call device time (CUDA events) and the number of kernel launches per call.
"""

from __future__ import annotations

import argparse
import json

import torch

from . import synthetic
from .calibrate import calibrate, load_scale_json
from .config import BENCH
from .model import DeviceWeights, SmolVLARunner
from .weights import random_weights


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--graph", action="store_true")
    ap.add_argument("--calib-samples", type=int, default=1)
    a = ap.parse_args()
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


if __name__ == "__main__":
    main()
