"""The Python mirror of the reference binding (nesle_b200._cuda_core).

Modelled on the reference's own tests of ``nesle._cuda_core.CudaBatch``
(tests/test_device_frames.py, tests/test_env.py, tests/test_fcs_parser.py):
constructors and their validation errors, host and device steps against the
checker, u8 / int64 / __cuda_array_interface__ actions, the DLPack and CAI
views, masked resets, poke_ram, step_stats, render shapes, the properties, and
the loud failure on an illegal opcode.
"""
from __future__ import annotations

import numpy as np
import pytest

import kat_roms as kat
from nesle_b200 import workloads as w


def test_parse_fcs_state_round_trip():
    """Host-only entry point: the FCS parser needs no GPU."""
    from nesle_b200._cuda_core import parse_fcs_state

    s = w.random_snapshot(5, 0x8123, nmi_and_rendering=True)
    s.ppu_v, s.ppu_t, s.ppu_x, s.ppu_w = 0x2345, 0x1234, 5, 1
    d = parse_fcs_state(w.write_fcs(s))
    assert (d["pc"], d["a"], d["x"], d["y"], d["sp"], d["p"]) == (s.pc, s.a, s.x, s.y, s.sp, s.p)
    assert (d["ppu_ctrl"], d["ppu_mask"], d["ppu_v"], d["ppu_t"], d["ppu_x"], d["ppu_w"]) == (0x80, 0x1E, 0x2345,
                                                                                           0x1234, 5, 1)
    assert d["cpu_ram"] == s.cpu_ram
    with pytest.raises(ValueError):
        parse_fcs_state(b"not an FCS file")


@pytest.fixture(scope="module")
def torch():
    t = pytest.importorskip("torch")
    if not t.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build

    build.build()
    return t


def _batch(n=32, wl=None, **kw):
    from nesle_b200._cuda_core import CudaBatch

    wl = wl or w.config4()
    env = np.arange(n)
    return CudaBatch(n, wl.frameskip, wl.rom.image, wl.snapshots, wl.env_to_level(env), device=0,
                     done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed, **kw), wl, env


def _oracle(n, wl):
    from oracle import Oracle

    env = np.arange(n)
    return Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=wl.env_to_level(env),
                  done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)


@pytest.mark.gpu
def test_constructor_validation(torch):
    from nesle_b200._cuda_core import CudaBatch

    wl = w.config4()
    with pytest.raises(ValueError):
        CudaBatch(0, 4, wl.rom.image)
    with pytest.raises(ValueError):
        CudaBatch(4, 0, wl.rom.image)
    with pytest.raises(ValueError):
        CudaBatch(4, 4)  # ROM-less synthetic mode
    with pytest.raises(ValueError):
        CudaBatch(4, 4, wl.rom.image, wl.snapshots, np.zeros(3, np.uint8))  # wrong env_to_level shape
    with pytest.raises(ValueError):
        CudaBatch(4, 4, wl.rom.image, wl.snapshots, np.full(4, 8, np.uint8))  # level out of range
    with pytest.raises(ValueError):
        CudaBatch(4, 4, wl.rom.image, [wl.snapshots[0]] * 256, np.zeros(4, np.uint8))  # > 255 levels
    with pytest.raises(ValueError):
        CudaBatch(4, 4, b"NES\x1a" + bytes(12))  # truncated image
    mapper1 = bytearray(wl.rom.image)
    mapper1[6] |= 0x10
    with pytest.raises(ValueError):
        CudaBatch(4, 4, bytes(mapper1))
    four = bytearray(wl.rom.image)
    four[6] |= 0x08
    with pytest.raises(ValueError):
        CudaBatch(4, 4, bytes(four))


@pytest.mark.gpu
def test_properties(torch):
    from nesle_b200._cuda_core import CudaBatch

    b, _, _ = _batch(8)
    assert b.name == "cuda-console" and b.has_snapshot and b.num_levels == 8
    wl1 = w.config1()
    c = CudaBatch(4, 4, wl1.rom.image, device=0)
    assert not c.has_snapshot and c.num_levels == 0
    assert hasattr(b, "step_device") and hasattr(b, "ram_device")  # native_ppo's bridge check
    assert b.step_kernel_placement == "shared"  # small batches stage RAM in shared memory
    big = CudaBatch(40000, 4, wl1.rom.image, device=0)
    assert big.step_kernel_placement == "interleaved"  # large batches: every env resident, RAM interleaved


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", ["u8", "i64", "cai"])
def test_step_device_action_kinds_match_checker(torch, dtype):
    n = 48
    b, wl, env = _batch(n)
    o = _oracle(n, wl)
    for s in range(3):
        a = wl.actions(env, s)
        t = torch.from_numpy(a).cuda()
        if dtype == "i64":
            t = t.to(torch.int64)
        if dtype == "cai":
            class CAI:  # a foreign producer exposing only __cuda_array_interface__
                def __init__(self, x):
                    self.x = x
                    self.__cuda_array_interface__ = x.__cuda_array_interface__
            t = CAI(t)
        out = b.step_device(t, auto_reset=True)
        o.step(a)
        np.testing.assert_array_equal(torch.as_tensor(out["ram"], device="cuda").cpu().numpy(), o.get("ram"))
        np.testing.assert_array_equal(torch.utils.dlpack.from_dlpack(out["rewards"]).cpu().numpy(),
                                      o.get("last_reward"))
        np.testing.assert_array_equal(torch.utils.dlpack.from_dlpack(out["dones"]).cpu().numpy(),
                                      o.get("last_done"))


@pytest.mark.gpu
def test_step_device_rejects_bad_actions(torch):
    b, _, _ = _batch(8)
    with pytest.raises(ValueError):
        b.step_device(torch.zeros(8, dtype=torch.uint8))  # host tensor
    with pytest.raises(ValueError):
        b.step_device(torch.zeros(7, dtype=torch.uint8, device="cuda"))
    with pytest.raises(ValueError):
        b.step_device(torch.zeros(8, dtype=torch.float32, device="cuda"))
    with pytest.raises(ValueError):
        b.step_device(torch.zeros(16, dtype=torch.uint8, device="cuda")[::2])
    with pytest.raises(ValueError):
        b.step(np.zeros(7, np.uint8))


@pytest.mark.gpu
def test_host_step_obs_modes_and_stats(torch):
    n = 16
    b, wl, env = _batch(n)
    o = _oracle(n, wl)
    a = wl.actions(env, 0)
    out = b.step(a)  # reference default: RGB obs
    o.step(a, device_api=False, auto_reset=False)
    assert out["obs"].shape == (n, 240, 256, 3) and out["obs"].dtype == np.uint8
    np.testing.assert_array_equal(out["obs"], o.render()["rgb"])
    np.testing.assert_array_equal(out["rewards"], o.get("reward"))
    np.testing.assert_array_equal(out["dones"], o.get("done"))
    a = wl.actions(env, 1)
    g = b.step(a, obs_mode="gray84")
    o.step(a, device_api=False, auto_reset=False)
    np.testing.assert_array_equal(g["obs"], o.render()["gray84"])
    st = b.step_stats(wl.actions(env, 2))
    o.step(wl.actions(env, 2), device_api=False, auto_reset=False)
    np.testing.assert_array_equal(st["instructions"], o.get("stat_instructions"))
    np.testing.assert_array_equal(st["frames_completed"], o.get("stat_frames"))
    assert "obs" not in st
    with pytest.raises(ValueError):
        b.step(a, obs_mode="hsv")


@pytest.mark.gpu
def test_views_dlpack_cai_and_copies_agree(torch):
    b, wl, env = _batch(16)
    b.step_device(torch.from_numpy(wl.actions(env, 0)).cuda())
    ram_view = b.ram_device()
    assert ram_view.__dlpack_device__() == (2, 0)
    cai = ram_view.__cuda_array_interface__
    assert cai["shape"] == (16, 2048) and cai["typestr"] == "|u1" and cai["version"] == 3
    t = torch.utils.dlpack.from_dlpack(ram_view)
    np.testing.assert_array_equal(t.cpu().numpy(), b.ram())
    side = torch.cuda.Stream()
    with torch.cuda.stream(side):
        t2 = torch.utils.dlpack.from_dlpack(ram_view.__dlpack__(stream=side.cuda_stream))
        s = t2.sum()
    torch.cuda.synchronize()
    assert int(s) == int(b.ram().astype(np.int64).sum())
    fr = b.render()
    assert fr.shape == (16, 240, 256, 3)
    np.testing.assert_array_equal(torch.as_tensor(b.frames_device(), device="cuda").cpu().numpy(), fr)
    assert b.oam().shape == (16, 256)


@pytest.mark.gpu
def test_reset_envs_poke_ram_reset_device(torch):
    n = 24
    b, wl, env = _batch(n)
    o = _oracle(n, wl)
    for s in range(2):
        b.step_device(torch.from_numpy(wl.actions(env, s)).cuda())
        o.step(wl.actions(env, s))
    mask = (np.arange(n) % 4 == 1).astype(np.uint8)
    b.reset_envs(mask)
    o.reset_envs(mask)
    b.poke_ram(0x7F3, 0x5A)
    o.poke_ram(0x7F3, 0x5A)
    np.testing.assert_array_equal(b.ram(), o.get("ram"))
    with pytest.raises(ValueError):
        b.reset_envs(np.zeros(n - 1, np.uint8))
    view = b.reset_device()
    o.reset()
    np.testing.assert_array_equal(torch.as_tensor(view, device="cuda").cpu().numpy(), o.get("ram"))


@pytest.mark.gpu
def test_illegal_opcode_raises_runtime_error(torch):
    from nesle_b200._cuda_core import CudaBatch

    rom = kat.rom_with({0x8000: bytes([0xA9, 0x05, 0x02])})
    b = CudaBatch(4, 2, rom, device=0)
    with pytest.raises(RuntimeError, match="illegal 6502 opcode 0x02"):
        b.step(np.zeros(4, np.uint8), render_frame=False, copy_obs=False)


@pytest.mark.gpu
@pytest.mark.parametrize("make", [w.config1, w.config3, w.config4])
def test_step_profile_histograms_match_checker(torch, make):
    """step_profile: stats and the opcode / fetch-address histograms, exact (200 envs: several
    warps, lanes of one warp at the same and at different addresses)."""
    from nesle_b200._cuda_core import CudaBatch
    from oracle import Oracle

    wl = make()
    n = 200
    env = np.arange(n)
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    kw = dict(done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    snaps = wl.snapshots if wl.snapshots else None
    b = CudaBatch(n, wl.frameskip, wl.rom.image, snaps, e2l if snaps and len(snaps) > 1 else None, device=0, **kw)
    o = Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=e2l, **kw)
    for s in range(2):
        a = wl.actions(env, s)
        out = b.step_profile(a)
        ops, pcs = o.step_profile(a)
        np.testing.assert_array_equal(out["opcode_counts"], ops)
        np.testing.assert_array_equal(out["pc_counts"], pcs)
        np.testing.assert_array_equal(out["instructions"], o.get("stat_instructions"))
        np.testing.assert_array_equal(out["rewards"], o.get("reward"))
        assert int(out["opcode_counts"].sum()) == int(out["instructions"].sum())
        b.step_device(torch.from_numpy(wl.actions(env, 10 + s)).cuda())  # unprofiled steps in between
        o.step(wl.actions(env, 10 + s))



@pytest.mark.gpu
def test_views_keep_the_batch_alive(torch):
    """The lifetime contract of the reference views (cuda_module.cu keep_alive<0, 1>,
    tests/test_env_reset_state.py): a view -- and a tensor made from it -- keeps its
    CudaBatch alive.  Checked by weak reference; freed memory is never touched."""
    import gc
    import weakref

    b, wl, env = _batch(8)
    ref = weakref.ref(b)
    view = b.ram_device()
    t = torch.utils.dlpack.from_dlpack(b.rewards_device())
    del b
    gc.collect()
    assert ref() is not None  # held by `view` and by `t`
    del view
    gc.collect()
    assert ref() is not None  # still held through the DLPack tensor
    assert t.shape == (8,)
    del t
    gc.collect()
    assert ref() is None


@pytest.mark.gpu
def test_render_after_step_matches_inline_render(torch):
    """tests/test_render_freshness.py: step(render_frame=False) + render() and
    step(render_frame=True) give the same, fresh frame."""
    wl = w.config3()
    n = 4
    from nesle_b200._cuda_core import CudaBatch

    a = CudaBatch(n, 4, wl.rom.image, device=0)
    c = CudaBatch(n, 4, wl.rom.image, device=0)
    first = a.render()
    acts = np.full(n, 0x80, np.uint8)
    for _ in range(6):
        a.step(acts, render_frame=False, copy_obs=False)
        out = c.step(acts, render_frame=True, copy_obs=True)
    fa = a.render()
    np.testing.assert_array_equal(fa, out["obs"])
    assert int((fa != first).sum()) > 100  # the frame moved on


@pytest.mark.gpu
def test_observation_arrays_are_fresh_and_their_buffers_recycled(torch):
    """Host observations come from pooled page-locked buffers: every step hands
    out a new array (a kept one is never overwritten), and a buffer is reused
    only after the array made from it is dropped."""
    import gc

    from nesle_b200 import _cuda_core

    n = 16
    b, wl, env = _batch(n)
    o = _oracle(n, wl)
    kept = []
    for s in range(3):
        a = wl.actions(env, s)
        out = b.step(a, obs_mode="gray84")
        o.step(a, device_api=False, auto_reset=False)
        want = o.render()["gray84"]
        np.testing.assert_array_equal(out["obs"], want)
        kept.append((out["obs"], want))
    assert len({k[0].ctypes.data for k in kept}) == 3
    for got, want in kept:  # later steps did not write into earlier arrays
        np.testing.assert_array_equal(got, want)
    used = {k[0].ctypes.data for k in kept}
    kept.clear()
    out = got = want = None
    gc.collect()
    assert used <= set(_cuda_core._HOST_BUFFERS._free.get(n * 84 * 84, []))
    out = b.step(wl.actions(env, 3), obs_mode="gray84")
    assert out["obs"].ctypes.data in used  # a dropped buffer, not a new allocation
    o.step(wl.actions(env, 3), device_api=False, auto_reset=False)
    np.testing.assert_array_equal(out["obs"], o.render()["gray84"])
    out = None
    _cuda_core.release_host_buffers()
    assert not _cuda_core._HOST_BUFFERS._free.get(n * 84 * 84)


def test_host_buffer_pool_recycles_only_dropped_arrays():
    """The page-locked pool (with a fake allocator, no GPU): arrays are fresh,
    a buffer comes back only when its last array or view is gone, and
    release() frees what the pool holds."""
    import ctypes
    import gc

    from nesle_b200._cuda_core import _HostBuffers

    keep, freed = [], []

    class FakeLib:
        def nesle_host_alloc(self, nbytes, out):
            buf = ctypes.create_string_buffer(int(nbytes))
            keep.append(buf)
            out._obj.value = ctypes.addressof(buf)
            return 0

        def nesle_host_free(self, ptr):
            freed.append(ptr.value)
            return 0

    pool, lib = _HostBuffers(), FakeLib()
    a = pool.array(lib, (4, 8), np.uint8)
    b = pool.array(lib, (4, 8), np.uint8)
    assert a.ctypes.data != b.ctypes.data and len(keep) == 2
    a[:] = 1
    b[:] = 2
    pa = a.ctypes.data
    view = b[1:]
    del a, b
    gc.collect()
    assert pool._free[32] == [pa]  # b's buffer is still held by `view`
    c = pool.array(lib, (4, 8), np.uint8)
    assert c.ctypes.data == pa and len(keep) == 2  # reused, not allocated
    assert (view == 2).all()
    del view, c
    gc.collect()
    assert sorted(pool._free[32]) == sorted([pa, ctypes.addressof(keep[1])])
    pool.release(lib)
    assert not pool._free[32] and sorted(freed) == sorted([pa, ctypes.addressof(keep[1])])
