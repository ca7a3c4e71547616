"""Generate the golden fixtures in this folder from the reference itself.

Runs the reference's own sources, compiled unchanged into ``oracle/_ref``
(``make -C oracle``), on the seeded benchmark workloads at small sizes and
records what they produce:

* kind "B" -- the reference's batched CUDA-kernel semantics on the host
  (``cpp/src/cuda/kernels.cu:19-104`` over the ``batch_*.cuh`` headers) with
  the ``step_device`` auto-reset order (``cpp/bindings/cuda_module.cu:635-656``);
* kind "A" -- the reference CPU core (``nesle::Console``, ``cpp/include/nesle/console.hpp``),
  for configuration 1 (power-on boot, no snapshot).

Per env-step it stores the CPU registers, cycle and frame counters, rewards
and dones, and a SHA-256 of every env's RAM; after the last step the full
RAM, OAM, nametable and palette arrays, and a SHA-256 per env of the RGB frame
rendered by the reference renderer (``batch_render.cuh``).

Usage (needs the reference tree and a built ``oracle/_ref``)::

    python tests/golden/make_golden.py
"""
from __future__ import annotations

import hashlib
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))

from nesle_b200 import workloads as w  # noqa: E402
from oracle import Reference, build  # noqa: E402

OUT = Path(__file__).with_name("reference_configs.npz")

# (name, workload factory, kind, envs, env-steps, auto_reset)
CASES = [
    ("config1_B", w.config1, "B", 8, 6, False),
    ("config1_A", w.config1, "A", 8, 6, False),
    ("config2_B", w.config2, "B", 8, 6, True),
    ("config3_B", w.config3, "B", 8, 6, True),
    ("config4_B", w.config4, "B", 8, 6, True),
    ("config4_short_B", None, "B", 8, 12, True),  # frame limit [6, 20]: many auto-resets
]
PER_STEP = ("pc", "a", "x", "y", "sp", "p", "cycles", "frame", "last_reward", "last_done")
PER_STEP_A = ("pc", "a", "x", "y", "sp", "p", "cycles", "frame")
FINAL_B = ("ram", "oam", "nt", "pal", "prg_ram", "ppu_ctrl", "ppu_mask", "ppu_status", "v", "t", "fine_x", "w",
           "scroll_x", "scroll_y", "episode", "prev_x", "prev_time")
FINAL_A = ("ram", "oam", "ppu_ctrl", "ppu_mask", "ppu_status")

def short_config4() -> w.Workload:
    wl = w.config4()
    wl.done_args = (6, 20)
    return wl


def sha(rows: np.ndarray) -> np.ndarray:
    flat = rows.reshape(rows.shape[0], -1)
    return np.array([np.frombuffer(hashlib.sha256(r.tobytes()).digest(), np.uint8) for r in flat])


def main() -> None:
    build()
    arrays: dict[str, np.ndarray] = {}
    for name, make, kind, n, steps, auto_reset in CASES:
        wl = (make or short_config4)()
        env = np.arange(n)
        e2l = wl.env_to_level(env) if wl.env_to_level else None
        ref = Reference(kind, n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=e2l,
                        done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
        fields = PER_STEP if kind == "B" else PER_STEP_A
        per = {f: [] for f in fields}
        ram_sha = []
        for s in range(steps):
            ref.step(wl.actions(env, s), auto_reset=auto_reset)
            for f in fields:
                per[f].append(ref.get(f))
            ram_sha.append(sha(ref.get("ram")))
        for f in fields:
            arrays[f"{name}/step/{f}"] = np.stack(per[f])
        arrays[f"{name}/step/ram_sha256"] = np.stack(ram_sha)
        for f in (FINAL_B if kind == "B" else FINAL_A):
            arrays[f"{name}/final/{f}"] = ref.get(f)
        if kind == "B":
            arrays[f"{name}/final/rgb_sha256"] = sha(ref.render_rgb())
        arrays[f"{name}/meta"] = np.array([n, steps, int(auto_reset), wl.frameskip], np.int64)
        print(f"{name}: {n} envs x {steps} env-steps, kind {kind}")
    np.savez_compressed(OUT, **arrays)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
