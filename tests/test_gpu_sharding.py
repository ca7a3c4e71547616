"""Env sharding on the CUDA path: two shards equal one batch, bit for bit.

A multi-GPU run gives rank r the global env range [r k, (r + 1) k) through
env_offset.  The product keys snapshot levels (env_to_level of the global
index), the frame-limit RNG and the action stream by the global index, so two
batches of k envs with env_offset 0 and k must reproduce one batch of 2 k
envs exactly.  Both shards run on one device here; that is the same code path
a rank takes on its own GPU.
"""
from __future__ import annotations

import numpy as np
import pytest

from harness import STATE_FIELDS, GpuCore, assert_same_window

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()


def _make(wl, n, offset):
    env = np.arange(offset, offset + n)
    return GpuCore(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=wl.env_to_level(env),
                   done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed, env_offset=offset)


def _compare(whole, shards, k, sample, label):
    """Every state field of `sample` envs of the whole batch against the shard rows."""
    want = whole.window(sample)
    got0 = shards[0].window(sample[sample < k])
    got1 = shards[1].window(sample[sample >= k] - k)
    got = {f: np.concatenate([got0[f], got1[f]]) for f in want}
    assert_same_window(want, got, STATE_FIELDS, label)


@pytest.mark.parametrize("k,steps,done_args,every", [
    (1000, 60, (6, 20), 10),          # short episodes: many auto-resets per shard
    (32768, 150, (500, 5000), 50),    # config 4 as specified at full size (first dones from step 125)
])
def test_two_shards_equal_one_batch(k, steps, done_args, every):
    from nesle_b200 import workloads as w

    wl = w.config4()
    wl.done_args = done_args
    whole = _make(wl, 2 * k, 0)
    shards = [_make(wl, k, 0), _make(wl, k, k)]
    rng = np.random.default_rng(k)
    sample = np.unique(np.concatenate([np.arange(16), np.arange(k - 16, k + 16), np.arange(2 * k - 16, 2 * k),
                                       rng.choice(2 * k, 256, replace=False)]))
    dones = 0
    for s in range(steps):
        whole.step(wl.actions(np.arange(2 * k), s))
        shards[0].step(wl.actions(np.arange(k), s))
        shards[1].step(wl.actions(np.arange(k, 2 * k), s))
        dones += int(whole.get("last_done").sum())
        if (s + 1) % every == 0 or s == steps - 1:
            _compare(whole, shards, k, sample, f"k={k} step {s}")
    for f in ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "oam", "episode", "last_reward", "last_done"):
        np.testing.assert_array_equal(whole.get(f), np.concatenate([shards[0].get(f), shards[1].get(f)]),
                                      err_msg=f"{f} over all envs")
    assert dones > 0
