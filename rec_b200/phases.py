"""Phase timeline of the persistent decode kernel.

Every CTA stamps the GPU global timer when it arrives at and leaves each grid
barrier (rec_set_profile).  From the stamps, per phase type:
  work_med / work_max : time from leaving the previous barrier to arriving at
                        this one (median / slowest CTA) — the phase's own work
  skew                : last arrival minus first arrival (load imbalance)
  release             : first release minus last arrival (barrier latency)
  wall                : median release-to-release time (what the step pays)
"""
from __future__ import annotations

import ctypes as C

import numpy as np
import torch

from ._lib import check, lib

PHASES = ["Q", "A", "O", "R", "G", "D"]


def capture(session, token: int, position: int, steps: int = 1) -> np.ndarray:
    """Runs `steps` greedy steps with the timeline enabled; returns stamps
    [steps * barriers, ctas, 2] in ns."""
    cfg = session.cfg
    grid = torch.cuda.get_device_properties(session.workspace.device).multi_processor_count
    per_step = 6 * cfg.n_layers + 1
    n = steps * per_step * grid * 2
    buf = torch.zeros(n, dtype=torch.int64, device=session.workspace.device)
    check(lib().rec_set_profile(session.ctx, C.c_void_p(buf.data_ptr()), n), "rec_set_profile")
    try:
        session.greedy(token, position, steps)
    finally:
        check(lib().rec_set_profile(session.ctx, None, 0), "rec_set_profile")
    return buf.view(steps * per_step, grid, 2).cpu().numpy().astype(np.int64)


def summarize(stamps: np.ndarray, n_layers: int) -> dict:
    per_step = 6 * n_layers + 1
    arrive, release = stamps[..., 0], stamps[..., 1]
    out = {p: {"work_med": [], "work_max": [], "skew": [], "release": [], "wall": []} for p in PHASES + ["H"]}
    for i in range(1, stamps.shape[0]):
        k = i % per_step
        name = "H" if k == per_step - 1 else PHASES[k % 6]
        if k == 0:  # Q of a step follows E of the previous one; skip the step boundary
            continue
        work = arrive[i] - release[i - 1]
        d = out[name]
        d["work_med"].append(np.median(work))
        d["work_max"].append(work.max())
        d["skew"].append(arrive[i].max() - arrive[i].min())
        d["release"].append(release[i].min() - arrive[i].max())
        d["wall"].append(np.median(release[i]) - np.median(release[i - 1]))
    res = {}
    for name, d in out.items():
        if d["wall"]:
            res[name] = {k: round(float(np.mean(v)) / 1e3, 3) for k, v in d.items()}  # us
    step_ns = float(np.median(release[-1]) - np.median(release[0]))
    res["step_us_between_first_and_last_barrier"] = round(step_ns / 1e3, 1)
    return res
