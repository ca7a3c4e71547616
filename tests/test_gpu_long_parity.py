"""GPU parity at the benchmark configurations' stated sizes and lengths.

The short lockstep tests compare every env every step at sizes the checker
runs in seconds.  These run the GPU batch at the configuration's own size and
length and re-run env windows (global env indices) on the CPU checker in
spawned worker processes while the GPU steps; every state field of every
window env is compared at regular checkpoints and after the last step:

* config 4 as specified: 65,536 envs, 8 snapshots, uniform joypad bytes and
  the real U[500, 5000] frame limit, for 1,300 env-steps, so that every env
  passes at least one done and fused auto-reset (5,000 frames = 1,250 steps);
* config 2 as specified: 4,096 envs x 10,000 env-steps, RAM[$FF] == $FF done;
* config 3 at 65,536 envs for 24 env-steps, 84x84 observations included.
"""
from __future__ import annotations

import numpy as np
import pytest

from checker_windows import checkpoints, pool, run_window, workload
from harness import STATE_FIELDS, GpuCore, assert_same_window

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()


def _run(cfg: str, n: int, steps: int, every: int, windows: list[tuple[int, int]], gray84: bool = False,
         done_args=None, store_all=()):
    """Steps a GpuCore of n envs while the checker runs `windows` (offset, size)
    in worker processes; compares at every checkpoint.  Returns (gpu core, dones
    over the whole batch per env, stored per-checkpoint fields of all envs)."""
    wl = workload(cfg, done_args)
    env = np.arange(n)
    marks = checkpoints(steps, every)
    with pool(len(windows)) as ex:
        futures = [ex.submit(run_window, cfg, done_args, off, size, steps, every, gray84) for off, size in windows]
        g = GpuCore(n, wl.frameskip, wl.rom.image, wl.snapshots,
                    env_to_level=wl.env_to_level(env) if wl.env_to_level else None, done_mode=wl.done_mode,
                    done_args=wl.done_args, seed=wl.seed)
        got = {off: {} for off, _ in windows}
        stored = {}
        dones = np.zeros(n, np.int64)
        for s in range(steps):
            g.step(wl.actions(env, s))
            dones += g.get("last_done")
            if s in marks:
                for off, size in windows:
                    got[off][s] = g.window(np.arange(off, off + size))
                if gray84:
                    obs = g.gray84()
                    for off, size in windows:
                        got[off][s]["gray84"] = obs[off:off + size].copy()
                if store_all:
                    stored[s] = {f: g.get(f) for f in store_all}
        want = [f.result() for f in futures]
    fields = STATE_FIELDS + (("gray84",) if gray84 else ())
    for (off, size), w_ in zip(windows, want):
        for s in marks:
            assert_same_window(w_[s], got[off][s], fields, f"{cfg} envs {off}..{off + size - 1} step {s}")
    window_dones = sum(w_["dones"] for w_ in want)
    return g, dones, stored, window_dones


def test_config4_as_specified_real_frame_limit():
    """65,536 envs x 1,300 env-steps with the real frame limit: every env is
    reset at least once; three 32-env windows compared every 50 steps."""
    n, steps = 65536, 1300
    windows = [(0, 32), (32768 - 16, 32), (n - 32, 32)]
    g, dones, _, window_dones = _run("config4", n, steps, 50, windows)
    episodes = g.get("episode")
    assert (episodes >= 1).all(), "some env never reached its frame limit"
    assert int(dones.sum()) == int(episodes.sum())
    assert window_dones >= 96
    assert (g.get("status") == 0).all()


def test_config2_as_specified():
    """4,096 envs x 10,000 env-steps (RAM mode, 7-mask actions, RAM[$FF] == $FF
    done with fused auto-reset); four 8-env windows compared every 500 steps, and
    a window around the first env the GPU saw done re-run afterwards."""
    n, steps, every = 4096, 10_000, 500
    windows = [(0, 8), (1365, 8), (2730, 8), (n - 8, 8)]
    light = ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "frame", "episode", "last_reward", "last_done")
    g, dones, stored, _ = _run("config2", n, steps, every, windows, store_all=light)
    assert (g.get("status") == 0).all()
    done_envs = np.nonzero(dones)[0]
    if len(done_envs):
        off = int(min(done_envs[0], n - 8))
        want = run_window("config2", None, off, 8, steps, every, fields=light)
        for s in checkpoints(steps, every):
            got = {f: stored[s][f][off:off + 8] for f in light}
            assert_same_window(want[s], got, light, f"config2 envs {off}.. step {s}")
        assert want["dones"] >= 1
    print(f"config2: {int(dones.sum())} dones over {n} envs x {steps} steps")


def test_config3_full_size_pixel_mode():
    """65,536 envs x 24 env-steps in pixel mode; three 32-env windows compared
    (state and 84x84 observations) every 6 steps."""
    n, steps = 65536, 24
    windows = [(0, 32), (32768 - 16, 32), (n - 32, 32)]
    g, _, _, _ = _run("config3", n, steps, 6, windows, gray84=True)
    assert (g.get("status") == 0).all()
