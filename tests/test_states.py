"""Env state save / restore (nesle_save_states / nesle_load_states) and the
FCS writer: the device-side capture and restore of the reference
(device_reset.cuh:72-263) over index lists, and snapshots written from live
states.
"""
from __future__ import annotations

import numpy as np
import pytest

from nesle_b200 import workloads as w

pytestmark = pytest.mark.gpu

FIELDS = ("pc", "a", "x", "y", "sp", "p", "cycles", "frame", "ram", "oam", "nametable", "palette", "prg_ram",
          "last_rewards", "last_done", "status", "stat_instructions")


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()
    return t


def _batch(n, wl):
    from nesle_b200._cuda_core import CudaBatch
    from nesle_b200.native_ppo import batch_snapshot_args

    return CudaBatch(n, wl.frameskip, wl.rom.image, *batch_snapshot_args(wl, np.arange(n)), device=0,
                     done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)


def _snapshot(b):
    return {f: b.get_field(f) for f in FIELDS}


def _step(torch, b, wl, s, n):
    b.step_device(torch.from_numpy(wl.actions(np.arange(n), s)).cuda(), auto_reset=True)


@pytest.mark.parametrize("device", [False, True])
def test_restore_replays_the_same_continuation(torch, device):
    wl = w.config4()
    wl.done_args = (8, 24)  # resets inside the window
    n = 96
    b = _batch(n, wl)
    for s in range(3):
        _step(torch, b, wl, s, n)
    saved = b.save_states(np.arange(n), device=device)
    for s in range(3, 7):
        _step(torch, b, wl, s, n)
    first = _snapshot(b)
    b.load_states(np.arange(n), saved)
    for s in range(3, 7):
        _step(torch, b, wl, s, n)
    again = _snapshot(b)
    for f in FIELDS:
        np.testing.assert_array_equal(again[f], first[f], err_msg=f)
    assert int(first["stat_instructions"].sum()) > 0


def test_one_state_loaded_into_many_envs(torch):
    wl = w.config1()
    n = 40
    b = _batch(n, wl)
    for s in range(2):
        _step(torch, b, wl, s, n)
    src = b.save_states([7])
    b.load_states(np.arange(n), np.repeat(src, n, axis=0))
    same = np.full(n, 0x81, np.uint8)
    for _ in range(3):
        b.step_device(torch.from_numpy(same).cuda(), auto_reset=False)
    st = _snapshot(b)
    for f in ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "oam"):
        assert (st[f] == st[f][7]).all(), f


def test_fcs_written_from_a_live_state(torch):
    from nesle_b200._cuda_core import CudaBatch, parse_fcs_state

    wl = w.config4()
    n = 16
    b = _batch(n, wl)
    for s in range(3):
        _step(torch, b, wl, s, n)
    fcs = b.save_fcs(5)
    d = parse_fcs_state(fcs)
    assert (d["pc"], d["a"], d["x"], d["y"], d["sp"], d["p"]) == tuple(
        int(b.get_field(f)[5]) for f in ("pc", "a", "x", "y", "sp", "p"))
    assert d["cpu_ram"] == b.get_field("ram")[5].tobytes()
    assert d["oam"] == b.get_field("oam")[5].tobytes()
    assert d["nametable_ram"] == b.get_field("nametable")[5].tobytes()
    # the written state seeds a new batch like any FCS snapshot
    c = CudaBatch(2, wl.frameskip, wl.rom.image, fcs, device=0)
    np.testing.assert_array_equal(c.get_field("ram"), np.repeat(b.get_field("ram")[5:6], 2, axis=0))
    assert (c.get_field("pc") == d["pc"]).all()


def test_bad_indices_and_shapes_are_rejected(torch):
    wl = w.config1()
    b = _batch(8, wl)
    with pytest.raises(ValueError):
        b.save_states([8])
    good = b.save_states([0, 1])
    with pytest.raises(ValueError):
        b.load_states([0], good)
    with pytest.raises(ValueError):
        b.load_states([0, 9], good)
