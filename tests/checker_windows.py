"""Checker runs of env windows for the long GPU parity tests.

A window is the env range [offset, offset + n) of a benchmark configuration,
run on the CPU checker with its global env indices (env_offset), so its
states equal those rows of a full-size GPU batch.  `run_window` is a plain
function so that a spawned process pool can run several windows while the
GPU batch steps (spawned workers do not inherit the parent's CUDA context).
"""
from __future__ import annotations

import concurrent.futures as cf
import multiprocessing as mp

import numpy as np

from harness import STATE_FIELDS


def workload(cfg: str, done_args=None):
    from nesle_b200 import workloads as w

    wl = w.CONFIGS[cfg]()
    if done_args is not None:
        wl.done_args = tuple(done_args)
    return wl


def checkpoints(steps: int, every: int) -> list[int]:
    """Steps (0-based) after which states are compared: every `every`-th and the last."""
    return [s for s in range(steps) if (s + 1) % every == 0 or s == steps - 1]


def run_window(cfg: str, done_args, offset: int, n: int, steps: int, every: int, gray84: bool = False,
               fields=STATE_FIELDS) -> dict:
    """{step: {field: array}} of the checker at every checkpoint step, plus the
    number of auto-resets the window saw under key "dones"."""
    from oracle import Oracle

    wl = workload(cfg, done_args)
    env = np.arange(offset, offset + n)
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    o = Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=e2l, done_mode=wl.done_mode,
               done_args=wl.done_args, seed=wl.seed, env_offset=offset)
    marks = set(checkpoints(steps, every))
    out: dict = {"dones": 0}
    for s in range(steps):
        o.step(wl.actions(env, s))
        out["dones"] += int(o.get("last_done").sum())
        if s in marks:
            snap = {f: o.get(f) for f in fields}
            if gray84:
                snap["gray84"] = o.render()["gray84"]
            out[s] = snap
    return out


def pool(workers: int) -> cf.ProcessPoolExecutor:
    return cf.ProcessPoolExecutor(max_workers=workers, mp_context=mp.get_context("spawn"))
