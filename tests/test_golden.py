"""Golden fixtures recorded from the reference itself (tests/golden/make_golden.py).

The checker (CPU) and the CUDA path (through the C ABI, GPU) are both held to
the committed outputs of the reference's own sources -- the batched-kernel
semantics ("B") and, for the power-on configuration, the reference CPU core
("A") -- on the seeded benchmark workloads.  Needs neither the reference tree
nor its build.
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import pytest

from nesle_b200 import workloads as w

GOLDEN = Path(__file__).with_name("golden") / "reference_configs.npz"


def _short_config4() -> w.Workload:
    wl = w.config4()
    wl.done_args = (6, 20)
    return wl


MAKERS = {"config1": w.config1, "config2": w.config2, "config3": w.config3, "config4": w.config4,
          "config4_short": _short_config4}


def _cases() -> list[str]:
    z = np.load(GOLDEN)
    return sorted({k.split("/")[0] for k in z.files})


def _sha(rows: np.ndarray) -> np.ndarray:
    flat = rows.reshape(rows.shape[0], -1)
    return np.array([np.frombuffer(hashlib.sha256(r.tobytes()).digest(), np.uint8) for r in flat])


def _replay(case: str, make_sim) -> None:
    z = np.load(GOLDEN)
    n, steps, auto_reset, frameskip = (int(v) for v in z[f"{case}/meta"])
    wl = MAKERS[case.rsplit("_", 1)[0]]()
    assert wl.frameskip == frameskip
    env = np.arange(n)
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    sim = make_sim(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=e2l, done_mode=wl.done_mode,
                   done_args=wl.done_args, seed=wl.seed)
    step_fields = [k.split("/")[2] for k in z.files if k.startswith(f"{case}/step/") and not k.endswith("sha256")]
    for s in range(steps):
        sim.step(wl.actions(env, s), auto_reset=bool(auto_reset))
        for f in step_fields:
            np.testing.assert_array_equal(sim.get(f), z[f"{case}/step/{f}"][s], err_msg=f"{case} step {s} {f}")
        np.testing.assert_array_equal(_sha(sim.get("ram")), z[f"{case}/step/ram_sha256"][s],
                                      err_msg=f"{case} step {s} ram")
    for k in z.files:
        if k.startswith(f"{case}/final/") and not k.endswith("sha256"):
            f = k.split("/")[2]
            np.testing.assert_array_equal(sim.get(f), z[k], err_msg=f"{case} final {f}")
    if f"{case}/final/rgb_sha256" in z.files:
        np.testing.assert_array_equal(_sha(sim.render()["rgb"]), z[f"{case}/final/rgb_sha256"],
                                      err_msg=f"{case} rgb frames")


def test_fixture_covers_every_benchmark_config():
    assert {c.rsplit("_", 1)[0] for c in _cases()} >= {"config1", "config2", "config3", "config4"}
    assert "config1_A" in _cases()  # the reference CPU core, not only the batched semantics


@pytest.mark.parametrize("case", _cases())
def test_checker_matches_golden(case):
    from oracle import Oracle

    _replay(case, Oracle)


@pytest.mark.gpu
@pytest.mark.parametrize("case", _cases())
def test_cuda_path_matches_golden(case):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from harness import GpuCore

    _replay(case, GpuCore)
