#!/usr/bin/env python
"""Env-step throughput of the B200 batched NES core (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (BASELINE.json metric "env-steps/s (frameskip 4, 65,536 envs/GPU)"):
configuration 4 -- 65,536 envs per GPU, RAM observation mode, frameskip 4,
joypad-driven divergent synthetic ROM, 8 seeded snapshots (global env i starts
from snapshot i mod 8), uniform u8 actions, done at a per-episode frame limit
U[500, 5000] with fused auto-reset.  Envs shard across GPUs with no data-path
collective (weak scaling); under torchrun each rank runs its own 65,536 envs.

value  : device-resident loop -- actions for every step already in HBM, one
         step_device (C-ABI nesle_step, fused auto-reset) per step, timed with
         CUDA events on the launching stream, max over ranks.
e2e    : the public host API CudaBatch.step(actions) per step -- pinned host
         actions copied in, kernel, rewards and dones read back -- wall clock,
         max over ranks.
--impl reference : the reference's own CPU core (nesle::Console compiled
         unchanged from the reference sources into oracle/_ref/) on all host
         threads, on a bounded sample of the same workload per step.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "env-steps/s (frameskip 4, 65,536 envs/GPU) at 1/2/4/8 B200"
UNIT = "env-steps/s"
# Algorithmic HBM bytes of one env-step in RAM mode: one compulsory round trip
# of the mutable per-env state (2 KB RAM read + write, OAM 256 written, CPU and
# PPU scalars 88, controller/DMA/reward baselines 30, action 1, reward 4 +
# done 1).
BYTES_PER_ENV_STEP = 4476


def parse_args(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference", "reference-cuda"], default="ours",
                    help="reference: the reference CPU core on the host cores; reference-cuda: the reference's "
                         "own CUDA kernel (oracle/_ref/cuda, built by `make -C oracle ref-cuda`) on this GPU")
    ap.add_argument("--done", choices=["workload", "smb"], default="workload",
                    help="smb: the reference's SMB done predicate instead of the workload's (the only one the "
                         "reference CUDA kernel has)")
    ap.add_argument("--envs", type=int, default=None, help="envs per GPU (65,536; 2,048 for config5)")
    ap.add_argument("--workload", default="config4", choices=["config4", "config3", "config2", "config1", "config5"])
    ap.add_argument("--obs", default="gray84", choices=["gray84", "rgb", "index"],
                    help="pixel mode (config3): the observation rendered every env-step")
    ap.add_argument("--burn-in", type=int, default=None,
                    help="untimed env-steps before the warm-up, so the timed region sees steady-state auto-resets "
                         "(default 150 for config4, whose first frame-limit dones come at env-step 125; else 0)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-vecenv", action="store_true", help="skip the host VecEnv end-to-end figure")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args(argv)


def dist_env():
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    return rank, world, local


def make_workload(name: str):
    from nesle_b200 import workloads as w

    # config 5's environment is config 2's (ROM, snapshot, 7-mask table, RAM-byte done)
    return {"config4": w.config4, "config3": w.config3, "config2": w.config2, "config1": w.config1,
            "config5": w.config2}[name]()


def apply_done_option(wl, args):
    if args.done == "smb":
        from nesle_b200 import workloads as w

        wl.done_mode, wl.done_args = w.DONE_SMB, (0, 0)
    return wl


def is_pixel(wl) -> bool:
    return wl.name.startswith("config3")


OBS_DESC = {"gray84": "gray 84x84 (7056 B/env) rendered every env-step from the palette-index frame",
            "rgb": "RGB 240x256x3 (184,320 B/env) rendered every env-step (the reference render())",
            "index": "palette-index frame 240x256 (61,440 B/env) rendered every env-step"}
# Pixel-mode bytes per env-step of the observation pass: snapshot NT 2048 + palette 32 + OAM 256 read,
# the observation written.
OBS_WRITE = {"gray84": 7056, "rgb": 184320, "index": 61440}


def workload_config(wl, envs: int, world: int, obs: str = "gray84") -> dict:
    return {
        "workload": f"{wl.name}: benchmark config {wl.name[6]}" if wl.name.startswith("config") else wl.name,
        "envs_per_gpu": envs,
        "total_envs": envs * world,
        "frameskip": wl.frameskip,
        "observation": (OBS_DESC[obs] if is_pixel(wl) else "ram (2048 B/env, zero-copy view)"),
        "snapshots": len(wl.snapshots),
        "done": {0: "smb (reference predicate)", 1: "RAM[$FF]==$FF", 2: "frame limit U[500,5000]"}[wl.done_mode],
        "auto_reset": "fused",
        "actions": "uniform u8 joypad bytes (counter RNG)" if wl.name.startswith("config4") else "counter RNG",
        "l2": "state larger than L2 (RAM 128 MiB + records/OAM/PRG-RAM per 65,536 envs); no flush",
        "parallelism": f"env-sharded dp{world}",
    }


# ---------------------------------------------------------------------------
# Clock sampling during the timed region.
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.lines: list[str] = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.device}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except (FileNotFoundError, OSError):
            self.proc = None
            return self
        # nvidia-smi's start-up can delay kernel launches; time only once it reports.
        t0 = time.perf_counter()
        while not self.lines and self.proc.poll() is None and time.perf_counter() - t0 < 10.0:
            time.sleep(0.05)
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        sm, mx, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx.append(float(parts[2]))
            except ValueError:
                continue
            for name, val in zip(names, parts[5:9]):
                if val.lower().startswith("active"):
                    reasons.add(name)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": max(mx), "reasons": sorted(reasons),
                "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU baselines (reference CPU core).
# ---------------------------------------------------------------------------
def host_threads() -> int:
    return max(1, len(os.sched_getaffinity(0)))


def reference_cpu_rate(wl, envs_total: int, steps: int, warmup: int, budget_s: float = 15.0) -> dict:
    """Reference CPU core on a bounded sample of the workload: env-steps/s."""
    from oracle import Reference, reference_available, Oracle

    threads = host_threads()
    kind = "reference" if reference_available() else "port"

    def make(n, offset):
        env = np.arange(offset, offset + n)
        kw = dict(env_to_level=wl.env_to_level(env) if wl.env_to_level else None, done_mode=wl.done_mode,
                  done_args=wl.done_args, seed=wl.seed, env_offset=offset)
        if kind == "reference":
            return Reference("A", n, wl.frameskip, wl.rom.image, wl.snapshots, threads=threads, **kw), env
        return Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, **kw), env

    # calibrate: grow the sample until one warm step fills its share of the budget
    # (small samples are dominated by per-step thread start-up)
    per_step_budget = budget_s / max(1, steps)
    sample_envs = min(envs_total, threads * 8)
    while True:
        sim, env = make(sample_envs, 0)
        sim.step(wl.actions(env, 0))
        t0 = time.perf_counter()
        sim.step(wl.actions(env, 1))
        dt = time.perf_counter() - t0
        if sample_envs >= envs_total or dt >= 0.7 * per_step_budget:
            break
        grow = max(2.0, min(16.0, per_step_budget / max(dt, 1e-6)))
        sample_envs = min(envs_total, max(threads, int(sample_envs * grow) // threads * threads))
    sim, env = make(sample_envs, 0)
    for s in range(warmup):
        sim.step(wl.actions(env, s))
    times = []
    for s in range(warmup, warmup + steps):
        t0 = time.perf_counter()
        sim.step(wl.actions(env, s))
        times.append(time.perf_counter() - t0)
    total = sum(times)
    rate = sample_envs * steps / total
    cores = threads if kind == "reference" else 1
    return {"value": rate, "unit": UNIT, "cores": cores, "kind": kind,
            "sample": f"{sample_envs} envs x {steps} env-steps (after {warmup} warm-up) of {wl.name}, "
                      f"{threads} host threads, nesle::Console stepped as NativeConsole.step",
            "seconds": total}


# ---------------------------------------------------------------------------
# Our arm.
# ---------------------------------------------------------------------------
def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "_fallback": True}


def profile_traffic(summary: str = "step_kernel_config4.txt") -> float | None:
    """DRAM bytes per launch of a kernel from its committed ncu summary."""
    p = ROOT / "profiles" / summary
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        line = line.strip()
        if line.startswith("dram_bytes_per_launch_full_size:"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def profile_figure(summary: str, key: str) -> float | None:
    """A `key: value` line of a committed ncu summary (e.g. warp instructions per launch)."""
    p = ROOT / "profiles" / summary
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        line = line.strip()
        if line.startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except ValueError:
                return None
    return None


def issue_roofline(instr: int, envs: int, kernel_ms: float, sm_mhz: float, summary: str | None) -> dict:
    """Secondary roofline of the step kernel: warp-instruction issue.  The warp
    instructions per launch come from the committed ncu summary of the same
    workload (a count of the code, not a time); the rate uses the live kernel time."""
    peak = 148 * 4 * sm_mhz * 1e6
    out = {"emulated_instructions_per_s": instr / (kernel_ms / 1e3) if instr else None,
           "emulated_instructions_per_env_step": instr / envs if instr else None,
           "peak_warp_issue_per_s": peak, "unit": "warp instructions/s"}
    warp = profile_figure(summary, "warp_instructions_per_launch") if summary else None
    if warp:
        out["warp_instructions_per_launch"] = warp
        out["achieved"] = warp / (kernel_ms / 1e3)
        out["issue_frac"] = out["achieved"] / peak
        if instr:
            out["warp_instructions_per_32_emulated_instructions"] = warp * 32 / instr
    return out


def shard(rank: int, envs_per_rank: int) -> tuple[int, np.ndarray]:
    """Global env range of one rank: [rank * n, (rank + 1) * n)."""
    offset = rank * envs_per_rank
    return offset, np.arange(offset, offset + envs_per_rank)


def combine_over_ranks(elapsed_ms: float, e2e_s: float | None, instr: int, device, world: int):
    """Max over ranks of the device and end-to-end times, sum of emulated instructions."""
    import torch
    import torch.distributed as dist

    if world <= 1:
        return elapsed_ms, e2e_s, instr
    vals = torch.tensor([elapsed_ms, e2e_s or 0.0, float(instr)], dtype=torch.float64, device=device)
    mx = vals.clone()
    dist.all_reduce(mx, op=dist.ReduceOp.MAX)
    sm = vals.clone()
    dist.all_reduce(sm, op=dist.ReduceOp.SUM)
    return float(mx[0]), (float(mx[1]) if e2e_s is not None else None), int(sm[2])


def run_ours(args, rank, world, local) -> dict | None:
    import torch
    import torch.distributed as dist

    from nesle_b200 import build as nb
    from nesle_b200._cuda_core import CudaBatch

    nb.build()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    wl = apply_done_option(make_workload(args.workload), args)
    n = args.envs
    offset, env = shard(rank, n)
    from nesle_b200.native_ppo import batch_snapshot_args

    batch = CudaBatch(n, wl.frameskip, wl.rom.image, *batch_snapshot_args(wl, env), device=local,
                      done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed, env_offset=offset)
    burn = args.burn_in
    total_steps = burn + args.warmup + args.steps
    acts = torch.from_numpy(np.stack([wl.actions(env, s) for s in range(total_steps)])).to(dev)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    pixel = is_pixel(wl)

    def device_step(s):
        batch.step_device(acts[s], auto_reset=True, synchronize=False)

    def render_obs():
        if args.obs == "gray84":
            batch.obs_gray84_device(render=True)
        elif args.obs == "index":
            batch.frames_index_device(render=True)
        else:
            batch.render_device()

    for s in range(burn):  # untimed: brings the frame-limit episodes to their first resets
        device_step(s)
    for s in range(burn, burn + args.warmup):
        device_step(s)
        if pixel:
            render_obs()
    torch.cuda.synchronize(dev)
    episodes_before = int(batch.get_field("episode").astype(np.int64).sum())
    barrier()
    torch.cuda.synchronize(dev)
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    mids = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    instr = 0
    with ClockSampler(local) as clocks:
        time.sleep(0.3)  # let the sampler attach
        for i, s in enumerate(range(burn + args.warmup, total_steps)):
            starts[i].record(stream)
            device_step(s)
            mids[i].record(stream)
            if pixel:
                render_obs()  # the observation of this env-step
            ends[i].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    per_step_ms = [a.elapsed_time(b) for a, b in zip(starts, mids)]
    per_obs_ms = [a.elapsed_time(b) for a, b in zip(mids, ends)]
    elapsed_ms = starts[0].elapsed_time(ends[-1])
    instr = int(batch.get_field("stat_instructions").astype(np.int64).sum())  # last step only
    resets = int(batch.get_field("episode").astype(np.int64).sum()) - episodes_before
    batch.synchronize()  # raises on illegal-opcode faults

    # e2e through the public host API with pinned host buffers
    e2e_s = None
    if not args.no_e2e:
        host_acts = torch.empty((total_steps, n), dtype=torch.uint8, pin_memory=True)
        host_acts.copy_(acts.cpu())
        host_np = host_acts.numpy()
        obs_kw = dict(render_frame=False, copy_obs=True, obs_mode=args.obs) if pixel else \
            dict(render_frame=False, copy_obs=False)
        out = None
        for s in range(burn, burn + args.warmup):  # held like the timed loop holds it: host buffers at steady state
            out = batch.step(host_np[s], **obs_kw)
        barrier()
        t0 = time.perf_counter()
        for s in range(burn + args.warmup, total_steps):
            out = batch.step(host_np[s], **obs_kw)
        e2e_s = time.perf_counter() - t0
        assert out["rewards"].shape == (n,)
        barrier()

    # e2e through the host VecEnv (SB3 contract): RAM observations copied to the host every step
    vec_s = None
    if not args.no_e2e and not args.no_vecenv and not pixel:
        from nesle_b200.vec_env import NesleVecEnv

        vec = NesleVecEnv(None, n, wl.frameskip, action_masks=np.arange(256), observation_mode="ram", batch=batch)
        host_idx = acts.cpu().numpy().astype(np.int64)
        for s in range(burn, burn + args.warmup):
            vec.step(host_idx[s])
        barrier()
        t0 = time.perf_counter()
        for s in range(burn + args.warmup, total_steps):
            obs, rew, dones, infos = vec.step(host_idx[s])
        vec_s = time.perf_counter() - t0
        assert obs.shape == (n, 2048) and len(infos) == n
        barrier()
        del vec

    elapsed_ms, e2e_s, instr = combine_over_ranks(elapsed_ms, e2e_s, instr, dev, world)
    vec_s, _, resets = combine_over_ranks(vec_s or 0.0, None, resets, dev, world)
    clock_summary = clocks.summary()

    result = None
    if rank == 0:
        total_env_steps = n * world * args.steps
        value = total_env_steps / (elapsed_ms / 1e3)
        kernel_ms = statistics.mean(per_step_ms)
        obs_ms = statistics.mean(per_obs_ms) if pixel else 0.0
        peaks = measured_peaks()
        peak = float(peaks.get("hbm_gbs", 6650.0))
        sm_mhz = clock_summary.get("sm_mhz") or float(peaks.get("sm_max_mhz", 1965.0))
        step_roof = {"kernel": f"step kernel ({batch.step_kernel_placement} RAM placement)", "bound": "hbm",
                     "achieved": BYTES_PER_ENV_STEP * n / (kernel_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                     "traffic": profile_traffic() if args.workload == "config4" else None, "ms": kernel_ms,
                     "note": "of measured HBM copy bandwidth; the kernel is latency/issue-bound (see issue)"}
        step_roof["frac"] = step_roof["achieved"] / peak
        result = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
            "config": workload_config(wl, n, world, args.obs),
            "roofline": step_roof,
            "issue": issue_roofline(instr, n * world, kernel_ms, sm_mhz,
                                    "step_kernel_config4.txt" if args.workload == "config4" else None),
            "resets_in_timed_region": resets,
            "burn_in_steps": burn,
            "kernel_ms": kernel_ms,
            "gpu_launches": args.steps * (2 if pixel else 1),
            "clocks": clock_summary,
        }
        if pixel:
            obs_bytes = 2048 + 32 + 256 + OBS_WRITE[args.obs]
            obs_roof = {"kernel": "gray84_kernel" if args.obs == "gray84" else "render_kernel", "bound": "hbm",
                        "achieved": obs_bytes * n / (obs_ms / 1e3) / 1e9, "peak": peak, "unit": "GB/s",
                        "traffic": profile_traffic("gray84_kernel_config3.txt" if args.obs == "gray84"
                                                   else f"render_kernel_{args.obs}_config3.txt"), "ms": obs_ms}
            obs_roof["frac"] = obs_roof["achieved"] / peak
            # `roofline` describes the dominant kernel, `second_kernel` the other one
            result["second_kernel"] = obs_roof
            if obs_ms > kernel_ms:
                result["roofline"], result["second_kernel"] = obs_roof, step_roof
        if e2e_s:
            d2h = (5 + (OBS_WRITE[args.obs] if pixel else 0)) * n * world
            result["e2e"] = {"value": total_env_steps / e2e_s, "unit": UNIT, "h2d_bytes_per_step": n * world,
                             "d2h_bytes_per_step": d2h,
                             "path": (f"CudaBatch.step(pinned u8 actions, obs_mode='{args.obs}') -> obs, rewards, "
                                      "dones as numpy" if pixel else
                                      "CudaBatch.step(pinned u8 actions) -> rewards, dones as numpy")}
        if vec_s:
            result["e2e_host_obs"] = {
                "value": total_env_steps / vec_s, "unit": UNIT, "h2d_bytes_per_step": 8 * n * world,
                "d2h_bytes_per_step": (2048 + 5) * n * world,
                "path": "NesleVecEnv(observation_mode='ram').step(action indices) -> RAM observations, rewards, "
                        "dones and infos on the host (SB3 auto-reset contract)"}
        if world == 1 and not args.no_cpu_baseline:
            result["cpu_baseline"] = reference_cpu_rate(wl, n, steps=2, warmup=1)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


def run_reference(args, rank, world, local) -> dict | None:
    """The reference's CPU implementation of the path on this box's host cores."""
    if rank != 0:
        return None
    wl = apply_done_option(make_workload(args.workload), args)
    base = reference_cpu_rate(wl, args.envs * world, steps=args.steps, warmup=args.warmup,
                              budget_s=min(120.0, 6.0 * (args.steps + args.warmup)))
    return {
        "metric": METRIC, "value": base["value"], "unit": UNIT, "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": 1e3 * base["seconds"] / args.steps, "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None, "dtype": "u8", "data": "synthetic", "impl": "reference",
        "config": workload_config(wl, args.envs, world),
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }


def load_reference_cuda():
    """The reference's own pybind11 CUDA module, compiled unchanged for sm_100a."""
    import importlib.util

    found = sorted((ROOT / "oracle" / "_ref" / "cuda").glob("_cuda_core*.so"))
    if not found:
        return None
    spec = importlib.util.spec_from_file_location("_cuda_core", found[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def run_reference_cuda(args, rank, world, local) -> dict | None:
    """The reference CUDA kernel (console_step_kernel through CudaBatch.step_device) on this GPU."""
    if rank != 0:
        return None
    import torch

    from nesle_b200 import build as nb
    from nesle_b200 import workloads as w
    from nesle_b200._cuda_core import CudaBatch
    from nesle_b200.native_ppo import batch_snapshot_args

    ref = load_reference_cuda()
    if ref is None:
        return {"impl": "reference-cuda", "unavailable": "reference CUDA binding not built (make -C oracle ref-cuda)"}
    nb.build()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    wl = make_workload(args.workload)
    wl.done_mode, wl.done_args = w.DONE_SMB, (0, 0)  # the reference kernel's only done predicate
    n = args.envs
    env = np.arange(n)
    snap, e2l = batch_snapshot_args(wl, env)
    total = args.warmup + args.steps
    acts = torch.from_numpy(np.stack([wl.actions(env, s) for s in range(total)])).to(dev)
    # Gate: the reference kernel executes `trap` on an illegal opcode.  Run this
    # library's kernel (same semantics, but it records the opcode instead) on
    # the identical inputs first; the reference runs only if none occurred.
    ours = CudaBatch(n, wl.frameskip, wl.rom.image, snap, e2l, device=local, done_mode=w.DONE_SMB)
    try:
        for s in range(total):
            ours.step_device(acts[s], auto_reset=True, synchronize=True)
    except RuntimeError as exc:
        return {"impl": "reference-cuda", "unavailable": f"illegal opcode on these inputs ({exc}); not run"}
    del ours
    if snap is None:
        batch = ref.CudaBatch(n, wl.frameskip, wl.rom.image)
    elif e2l is None:
        batch = ref.CudaBatch(n, wl.frameskip, wl.rom.image, snap)
    else:
        batch = ref.CudaBatch(n, wl.frameskip, wl.rom.image, list(snap), e2l)
    stream = torch.cuda.current_stream(dev)
    for s in range(args.warmup):
        batch.step_device(acts[s], auto_reset=True, synchronize=True)
    torch.cuda.synchronize(dev)
    t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        t0.record(stream)
        for s in range(args.warmup, total):
            batch.step_device(acts[s], auto_reset=True, synchronize=True)
        t1.record(stream)
        torch.cuda.synchronize(dev)
    elapsed_ms = t0.elapsed_time(t1)
    return {
        "metric": METRIC, "value": n * args.steps / (elapsed_ms / 1e3), "unit": UNIT, "n_gpus": 1,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8", "data": "synthetic",
        "impl": "reference-cuda",
        "config": dict(workload_config(wl, n, 1), reference="cpp/bindings/cuda_module.cu + "
                       "cpp/src/cuda/kernels.cu compiled unchanged for sm_100a; step_device(auto_reset=True)"),
        "clocks": clocks.summary(),
    }


def run_ppo(args, rank, world, local) -> dict | None:
    """Config 5: GPU-resident rollout + PPO update; one step = one PPO iteration."""
    import torch
    import torch.distributed as dist

    from nesle_b200 import build as nb
    from nesle_b200.native_ppo import NativePPOConfig, PPOTrainer

    nb.build()
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    cfg = NativePPOConfig(num_envs=args.envs)
    tr = PPOTrainer(cfg, device=local, rank=rank, world=world)
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        tr.iteration()
    torch.cuda.synchronize(dev)
    barrier()
    ev = [[torch.cuda.Event(enable_timing=True) for _ in range(3)] for _ in range(args.steps)]
    with ClockSampler(local) as clocks:
        for i in range(args.steps):
            ev[i][0].record(stream)
            tr.rollout()
            ev[i][1].record(stream)
            tr.update()
            ev[i][2].record(stream)
        torch.cuda.synchronize(dev)
    barrier()
    elapsed_ms = ev[0][0].elapsed_time(ev[-1][2])
    rollout_ms = statistics.mean(e[0].elapsed_time(e[1]) for e in ev)
    update_ms = statistics.mean(e[1].elapsed_time(e[2]) for e in ev)
    tr.batch.synchronize()

    # the step kernel alone at this size (the rollout's dominant kernel)
    acts = torch.zeros(cfg.num_envs, dtype=torch.uint8, device=dev)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    k0.record(stream)
    for _ in range(10):
        tr.batch.step_device(acts, auto_reset=True, synchronize=False)
    k1.record(stream)
    torch.cuda.synchronize(dev)
    kernel_ms = k0.elapsed_time(k1) / 10

    # e2e: the public training call with the loss read back each iteration
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        loss = float(tr.iteration()["loss"])
    e2e_s = time.perf_counter() - t0
    assert math.isfinite(loss)
    elapsed_ms, e2e_s, _ = combine_over_ranks(elapsed_ms, e2e_s, 0, dev, world)
    clock_summary = clocks.summary()
    result = None
    if rank == 0:
        samples = cfg.num_envs * cfg.n_steps * world * args.steps
        peaks = measured_peaks()
        hbm = float(peaks.get("hbm_gbs", 6650.0))
        params = sum(p.numel() for p in tr.model.parameters())
        # forward + backward of every minibatch sample in every epoch: 6 flops per parameter
        update_flops = 6.0 * params * cfg.num_envs * cfg.n_steps * cfg.update_epochs
        tflops = update_flops / (update_ms / 1e3) / 1e12
        bf16_peak = float(peaks.get("bf16_tflops", 1590.0))
        step_roof = {"kernel": f"step kernel ({tr.batch.step_kernel_placement} RAM placement)", "bound": "hbm",
                     "achieved": BYTES_PER_ENV_STEP * cfg.num_envs / (kernel_ms / 1e3) / 1e9, "peak": hbm,
                     "unit": "GB/s", "traffic": None, "ms": kernel_ms,
                     "note": "of measured HBM copy bandwidth; at 2,048 envs the kernel is bound by the latency "
                             "of one env's instruction chain (see issue)"}
        step_roof["frac"] = step_roof["achieved"] / hbm
        result = {
            "metric": METRIC, "value": samples / (elapsed_ms / 1e3), "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "u8 env / bf16 policy",
            "data": "synthetic",
            "config": {"workload": "config5-ppo: benchmark config 5 (GPU-resident rollout + PPO)",
                       "envs_per_gpu": cfg.num_envs, "total_envs": cfg.num_envs * world, "frameskip": cfg.frameskip,
                       "n_steps": cfg.n_steps, "batch_size": cfg.batch_size, "update_epochs": cfg.update_epochs,
                       "gamma": cfg.gamma, "gae_lambda": cfg.gae_lambda,
                       "policy": "bf16 MLP 2048->512->256 ReLU, 7 logits + value, random init",
                       "env": "config2 ROM and snapshot, 7-mask action table, RAM[$FF]==$FF done, fused auto-reset",
                       "observation": "RAM via DLPack, no copy",
                       "l2": "no flush: each iteration writes 537 MB of rollout observations (> L2)",
                       "parallelism": f"env-sharded dp{world}, NCCL gradient all-reduce"},
            "roofline": step_roof,
            "update": {"ms": update_ms, "bound": "tensor", "achieved": tflops, "peak": bf16_peak,
                       "unit": "TFLOP/s", "frac": tflops / bf16_peak, "params": params,
                       "note": "of measured cuBLAS bf16 burst; minibatches of 8,192 are launch-bound"},
            "rollout_ms": rollout_ms,
            "kernel_ms": kernel_ms,
            "gpu_launches": args.steps * cfg.n_steps,
            "clocks": clock_summary,
            "e2e": {"value": samples / e2e_s, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 4,
                    "path": "PPOTrainer.iteration() with the loss read on the host every iteration"},
        }
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()
    return result


def main(argv=None) -> int:
    args = parse_args(argv)
    if args.envs is None:
        args.envs = 2048 if args.workload == "config5" else 65536
    if args.burn_in is None:
        args.burn_in = 150 if args.workload == "config4" else 0
    rank, world, local = dist_env()
    # Libraries (NCCL announces its version) may write to stdout; the result must
    # be the only line there, so fd 1 points at stderr until it is printed.
    result_out = os.fdopen(os.dup(1), "w")
    sys.stdout.flush()
    os.dup2(2, 1)
    if args.impl == "reference":
        res = run_reference(args, rank, world, local)
    elif args.impl == "reference-cuda":
        res = run_reference_cuda(args, rank, world, local)
    elif args.workload == "config5":
        res = run_ppo(args, rank, world, local)
    else:
        res = run_ours(args, rank, world, local)
    if res is not None:
        print(json.dumps(res), file=result_out, flush=True)
    return 0


if __name__ == "__main__":
    sys.exit(main())
