"""nesle_render_gray84_noalloc: the 84x84 observation without device allocation.

Compared byte for byte with the allocating path (nesle_render(GRAY84) +
nesle_copy_field("obs_gray84")) on two calls in a row with a step between,
and checked to reject batches beyond its static scratch.  Kept in its own
file, collected last, and independent of every other test's state.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

from nesle_b200 import _lib
from nesle_b200 import workloads as w

pytestmark = pytest.mark.gpu

SCRATCH_ENVS = 1024


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()


def _noalloc(core, out: np.ndarray) -> int:
    return core.lib.nesle_render_gray84_noalloc(core._h, out.ctypes.data, out.nbytes, None)


@pytest.mark.parametrize("n", [200, SCRATCH_ENVS])
def test_matches_allocating_render_on_two_calls_in_a_row(n):
    from harness import GpuCore

    wl = w.config3()
    env = np.arange(n)
    g = GpuCore(n, wl.frameskip, wl.rom.image, [], done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    for s in range(2):
        g.step(wl.actions(env, s))
        _lib.check(g.lib.nesle_render(g._h, _lib.RENDER_GRAY84, None))
        ref = g.get("obs_gray84")
        out = np.full((n, 84, 84), 0xA5, np.uint8)
        _lib.check(_noalloc(g, out))
        np.testing.assert_array_equal(out, ref, err_msg=f"call {s}")
    assert len(np.unique(ref)) > 8  # real frames, not a constant


def test_first_call_on_a_fresh_batch_leaves_no_frame_buffer():
    """On a batch that has never rendered, the no-allocation call works first
    and leaves no observation buffer behind; the allocating render made
    afterwards gives the same bytes."""
    from harness import GpuCore

    wl = w.config3()
    n = 96
    g = GpuCore(n, wl.frameskip, wl.rom.image, [], done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    g.step(wl.actions(np.arange(n), 0))
    out = np.full((n, 84, 84), 0x5A, np.uint8)
    _lib.check(_noalloc(g, out))
    probe = np.zeros((n, 84, 84), np.uint8)
    rc = g.lib.nesle_copy_field(g._h, b"obs_gray84", probe.ctypes.data, probe.nbytes)
    assert rc == _lib.NESLE_ERR_RUNTIME and b"not been rendered" in g.lib.nesle_last_error()
    _lib.check(g.lib.nesle_render(g._h, _lib.RENDER_GRAY84, None))
    np.testing.assert_array_equal(out, g.get("obs_gray84"))


def test_rejects_batches_beyond_the_scratch_and_wrong_sizes():
    from harness import GpuCore

    wl = w.config1()
    big = GpuCore(SCRATCH_ENVS + 1, wl.frameskip, wl.rom.image)
    out = np.zeros((SCRATCH_ENVS + 1, 84, 84), np.uint8)
    assert _noalloc(big, out) == _lib.NESLE_ERR_INVALID
    assert b"at most 1024 envs" in big.lib.nesle_last_error()
    small = GpuCore(8, wl.frameskip, wl.rom.image)
    short = np.zeros((7, 84, 84), np.uint8)
    assert _noalloc(small, short) == _lib.NESLE_ERR_INVALID
    assert small.lib.nesle_render_gray84_noalloc(small._h, None, 8 * 84 * 84, None) == _lib.NESLE_ERR_INVALID
    ok = np.zeros((8, 84, 84), np.uint8)
    assert _noalloc(small, ok) == _lib.NESLE_OK
    assert ctypes.c_int(_noalloc(small, ok)).value == _lib.NESLE_OK  # repeatable
