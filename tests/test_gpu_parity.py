"""GPU parity: libnesle_b200.so through its C ABI against the CPU checker.

Bit-exact per-env RAM, CPU registers, cycles, PPU state, done/reward and
palette-index frames after every step, on every benchmark configuration at
sizes the checker runs in seconds, plus size-independent properties at the
full 65,536-env configuration.
"""
from __future__ import annotations

import ctypes

import numpy as np
import pytest

import kat_roms as kat
from harness import STATE_FIELDS, GpuCore, assert_same, run_lockstep
from nesle_b200 import _lib
from nesle_b200 import workloads as w
from oracle import Oracle

pytestmark = pytest.mark.gpu

# Every RAM placement of the step kernel (NESLE_STEP_KERNEL).
PLACEMENTS = ["shared", "global", "hybrid", "hybrid-stack", "global-async", "hybrid-async", "interleaved",
              "interleaved-async", "global-preload", "hybrid-preload", "interleaved-preload"]


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from nesle_b200 import build
    build.build()


@pytest.mark.parametrize("make,auto_reset,n", [(w.config1, False, 64), (w.config2, True, 200),
                                               (w.config3, True, 200), (w.config4, True, 200)])
@pytest.mark.parametrize("variant", PLACEMENTS)
def test_configs_lockstep(make, auto_reset, n, variant, monkeypatch):
    """Every step, every field, against the checker (200 envs = 2 full CTAs + a partial one),
    for both placements of env RAM in the step kernel."""
    monkeypatch.setenv("NESLE_STEP_KERNEL", variant)
    run_lockstep(make, n, 6, auto_reset, [GpuCore])


def test_config1_full_length():
    """Config 1 as specified: 64 envs, 600 frames (150 env-steps), from power-on."""
    run_lockstep(w.config1, 64, 150, False, [GpuCore], check_every=10)


def test_frame_limit_auto_reset_many_episodes():
    def short():
        wl = w.config4()
        wl.done_args = (5, 17)
        return wl
    _, _, dones = run_lockstep(short, 97, 24, True, [GpuCore])
    assert dones > 50


@pytest.mark.parametrize("rom,snaps", [
    (kat.LDA_TAX_INX_STA, []), (kat.JSR_RTS, []), (kat.BNE_PAGE_CROSS, []), (kat.SEC_SBC, []),
    (kat.NMI_ROM, []), (kat.DMA_ROM, [kat.dma_snapshot()]), (kat.DMA_ZP_ROM, [kat.dma_zp_snapshot()]),
    (kat.IDLE_ROM, [])])
@pytest.mark.parametrize("variant", PLACEMENTS)
def test_known_answer_roms(rom, snaps, variant, monkeypatch):
    monkeypatch.setenv("NESLE_STEP_KERNEL", variant)
    o = Oracle(3, 2, rom, snaps)
    g = GpuCore(3, 2, rom, snaps)
    for _ in range(3):
        a = np.array([0x81, 0x00, 0xFF], np.uint8)
        o.step(a, auto_reset=False)
        g.step(a, auto_reset=False)
        assert_same(o, g)


@pytest.mark.parametrize("case", kat.REWARD_CASES)
def test_reward_known_answers(case):
    (pp, ps, pt), (cp, cs, ct, state), reward, done = case
    g = GpuCore(1, 1, kat.IDLE_ROM, [kat.mario_snapshot(pp, ps, pt)])
    for addr, val in ((0x6D, cp), (0x86, cs), (0x0E, state), (0x7F8, ct // 100), (0x7F9, (ct // 10) % 10),
                      (0x7FA, ct % 10)):
        g.poke_ram(addr, val)
    g.step(np.zeros(1, np.uint8), auto_reset=False)
    assert g.get("last_reward")[0] == reward and g.get("last_done")[0] == done


def test_every_official_opcode():
    from test_core_host import _single_instruction_cases

    for opc, rom, snap in _single_instruction_cases(3, 1):
        o = Oracle(1, 1, rom, [snap])
        g = GpuCore(1, 1, rom, [snap])
        o.step(np.zeros(1, np.uint8), auto_reset=False)
        g.step(np.zeros(1, np.uint8), auto_reset=False)
        try:
            assert_same(o, g, ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "prg_ram", "status"))
        except AssertionError as e:
            raise AssertionError(f"opcode {opc:#04x}: {e}") from None


def test_render_index_rgb_gray_match_checker():
    from test_core_host import render_snapshots

    wl = w.config4()
    n = 8
    snaps = render_snapshots(11, 4, wl.rom.loop_head)
    kw = dict(env_to_level=np.arange(n) % 4, done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, snaps, **kw)
    g = GpuCore(n, 4, wl.rom.image, snaps, **kw)
    for s in range(3):
        a = wl.actions(np.arange(n), s)
        o.step(a)
        g.step(a)
    ro, rg = o.render(), g.render()
    for k in ("index", "rgb", "gray84"):
        np.testing.assert_array_equal(ro[k], rg[k], err_msg=k)
    assert len(np.unique(ro["index"])) > 8


def test_config3_frames_every_step():
    """Pixel mode on the GPU: index, RGB and 84x84 gray frames after every env-step."""
    wl = w.config3()
    n = 64
    env = np.arange(n)
    kw = dict(done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, [], **kw)
    g = GpuCore(n, 4, wl.rom.image, [], **kw)
    for s in range(4):
        a = wl.actions(env, s)
        o.step(a)
        g.step(a)
        assert_same(o, g)
        ro, rg = o.render(), g.render()
        for k in ("index", "rgb", "gray84"):
            np.testing.assert_array_equal(ro[k], rg[k], err_msg=f"step {s} {k}")


def test_reset_envs_poke_and_host_step():
    wl = w.config4()
    n = 100
    kw = dict(env_to_level=wl.env_to_level(np.arange(n)), done_mode=wl.done_mode, done_args=wl.done_args,
              seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, wl.snapshots, **kw)
    g = GpuCore(n, 4, wl.rom.image, wl.snapshots, **kw)
    a = wl.actions(np.arange(n), 0)
    o.step(a, device_api=False)
    g.step(a, device_api=False)
    assert_same(o, g)
    mask = (np.arange(n) % 3 == 0).astype(np.uint8)
    o.reset_envs(mask)
    g.reset_envs(mask)
    o.poke_ram(0x7F0, 0x99)
    g.poke_ram(0x7F0, 0x99)
    assert_same(o, g)
    for s in range(1, 3):
        a = wl.actions(np.arange(n), s)
        o.step(a)
        g.step(a)
        assert_same(o, g)
    o.reset()
    g.reset()
    assert_same(o, g)


def test_illegal_opcode_sets_status_without_fault():
    rom = kat.rom_with({0x8000: bytes([0xA9, 0x05, 0x02])})
    o = Oracle(4, 2, rom)
    g = GpuCore(4, 2, rom)
    for _ in range(2):
        o.step(np.zeros(4, np.uint8), auto_reset=False)
        g.step(np.zeros(4, np.uint8), auto_reset=False)
        assert_same(o, g)
    assert (g.get("status") == (0x80000000 | 0x020000 | 0x8002)).all()


@pytest.mark.parametrize("offset", [0, 32768 - 48, 65536 - 96])
def test_full_size_config4_windows_match_checker(offset):
    """65,536 envs on the GPU; three windows of 96 envs re-run on the checker."""
    full = _full_size_run(steps=3)
    wl = w.config4()
    n = 96
    env = np.arange(offset, offset + n)
    o = Oracle(n, 4, wl.rom.image, wl.snapshots, env_to_level=wl.env_to_level(env), done_mode=wl.done_mode,
               done_args=wl.done_args, seed=wl.seed, env_offset=offset)
    for s in range(3):
        o.step(wl.actions(env, s))
    for f in ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "oam", "frame", "last_reward", "last_done"):
        np.testing.assert_array_equal(o.get(f), full[f][offset:offset + n], err_msg=f)


_FULL_CACHE: dict = {}


def _full_size_run(steps: int) -> dict:
    if steps not in _FULL_CACHE:
        wl = w.config4()
        n = 65536
        env = np.arange(n)
        g = GpuCore(n, 4, wl.rom.image, wl.snapshots, env_to_level=wl.env_to_level(env), done_mode=wl.done_mode,
                    done_args=wl.done_args, seed=wl.seed)
        for s in range(steps):
            g.step(wl.actions(env, s))
        _FULL_CACHE[steps] = {f: g.get(f) for f in ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "oam", "frame",
                                                    "last_reward", "last_done", "status")}
        del g
    return _FULL_CACHE[steps]


def test_full_size_properties():
    """Size-independent checks at full size: healthy, deterministic, envs diverged."""
    a = _full_size_run(steps=3)
    assert (a["status"] == 0).all()
    assert (a["frame"] == 12).all()  # 3 env-steps x frameskip 4
    assert len(np.unique(a["pc"])) > 100  # joypad-driven divergence
    wl = w.config4()
    g = GpuCore(65536, 4, wl.rom.image, wl.snapshots, env_to_level=wl.env_to_level(np.arange(65536)),
                done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    for s in range(3):
        g.step(wl.actions(np.arange(65536), s))
    np.testing.assert_array_equal(g.get("ram"), a["ram"])
    np.testing.assert_array_equal(g.get("cycles"), a["cycles"])


def _windows_match(wl, full, offsets, n, steps, fields, render=False):
    """Re-run envs [off, off+n) on the checker and compare with rows of a full-size GPU run."""
    for off in offsets:
        env = np.arange(off, off + n)
        e2l = wl.env_to_level(env) if wl.env_to_level else None
        o = Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=e2l, done_mode=wl.done_mode,
                   done_args=wl.done_args, seed=wl.seed, env_offset=off)
        for s in range(steps):
            o.step(wl.actions(env, s))
        for f in fields:
            np.testing.assert_array_equal(o.get(f), full[f][off:off + n], err_msg=f"{f} at envs {off}+")
        if render:
            np.testing.assert_array_equal(o.render()["gray84"], full["gray84"][off:off + n],
                                          err_msg=f"gray84 at envs {off}+")


def _full_run(wl, n, steps):
    env = np.arange(n)
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    g = GpuCore(n, wl.frameskip, wl.rom.image, wl.snapshots, env_to_level=e2l, done_mode=wl.done_mode,
                done_args=wl.done_args, seed=wl.seed)
    for s in range(steps):
        g.step(wl.actions(env, s))
    return g


def test_ragged_multiwave_batch_matches_checker():
    """150,001 envs (hybrid placement, several waves of CTAs, a partial last CTA):
    windows at the start, the middle and the end re-run on the checker."""
    wl = w.config4()
    n = 150_001
    g = _full_run(wl, n, 2)
    fields = ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "last_reward", "last_done")
    full = {f: g.get(f) for f in fields + ("status",)}
    assert (full["status"] == 0).all()
    _windows_match(wl, full, [0, 75_000 - 40, n - 64], 64, 2, fields)


def test_full_size_pixel_mode_matches_checker():
    """Config 3 at 65,536 envs: state and 84x84 observations of three windows."""
    wl = w.config3()
    n = 65536
    g = _full_run(wl, n, 2)
    fields = ("pc", "ram", "oam", "scroll_x", "last_done")
    full = {f: g.get(f) for f in fields}
    _lib.check(g.lib.nesle_render(g._h, _lib.RENDER_GRAY84, None))
    full["gray84"] = g.get("obs_gray84")
    _windows_match(wl, full, [0, 32_768 - 16, n - 32], 32, 2, fields, render=True)


@pytest.mark.parametrize("seed", [5, 6])
def test_render_scroll_split_matches_checker(seed):
    """The render kernels under random control, mask and mid-frame scroll (split
    row moving with sprite 0), random CHR / nametables / palette / OAM: all three
    observation formats after every step, 64 envs over 8 snapshots."""
    n = 64
    snaps = kat.render_scroll_snapshots(seed, 8)
    kw = dict(env_to_level=np.arange(n) % 8)
    o = Oracle(n, 4, kat.RENDER_SCROLL_ROM, snaps, **kw)
    g = GpuCore(n, 4, kat.RENDER_SCROLL_ROM, snaps, **kw)
    for _ in range(4):
        o.step(np.zeros(n, np.uint8), auto_reset=False)
        g.step(np.zeros(n, np.uint8), auto_reset=False)
        assert_same(o, g, label="render-scroll")
        ro, rg = o.render(), g.render()
        for k in ("index", "rgb", "gray84"):
            np.testing.assert_array_equal(ro[k], rg[k], err_msg=k)


@pytest.mark.parametrize("n", [3, 37])
def test_render_copy_matches_render_then_copy(n):
    """nesle_render_copy (8 env ranges, each copied while the next renders) gives
    the bytes of nesle_render + nesle_copy_field, also for batches whose ranges
    are ragged (37 envs) or fewer than 8 (3 envs)."""
    from test_core_host import render_snapshots

    wl = w.config4()
    snaps = render_snapshots(11, 4, wl.rom.loop_head)
    g = GpuCore(n, 4, wl.rom.image, snaps, env_to_level=np.arange(n) % 4, done_mode=wl.done_mode,
                done_args=wl.done_args, seed=wl.seed)
    g.step(wl.actions(np.arange(n), 0))
    want = g.render()
    for mode, key, field in ((_lib.RENDER_RGB, "rgb", "frames_rgb"), (_lib.RENDER_INDEX, "index", "frames_index"),
                             (_lib.RENDER_GRAY84, "gray84", "obs_gray84")):
        dtype, shape = _lib.FIELDS[field]
        out = np.full((n, *shape), 0xAB, dtype)
        _lib.check(g.lib.nesle_render_copy(g._h, mode, out.ctypes.data, out.nbytes, None))
        np.testing.assert_array_equal(out, want[key], err_msg=key)
        assert g.lib.nesle_render_copy(g._h, mode, out.ctypes.data, out.nbytes - 1, None) == _lib.NESLE_ERR_INVALID


@pytest.mark.parametrize("variant", PLACEMENTS)
def test_controller_protocol_matches_checker(variant, monkeypatch):
    """The controller known-answer ROM on every RAM placement: strobe-high reads,
    reads past the 8 latched bits, $4017, step boundaries all through the reads."""
    monkeypatch.setenv("NESLE_STEP_KERNEL", variant)
    n = 64
    o = Oracle(n, 1, kat.CONTROLLER_ROM, [])
    g = GpuCore(n, 1, kat.CONTROLLER_ROM, [])
    rng = np.random.default_rng(0)
    for _ in range(12):
        a = rng.integers(0, 256, n, dtype=np.uint8)
        o.step(a, auto_reset=False)
        g.step(a, auto_reset=False)
        assert_same(o, g, label=f"controller {variant}")


BOARD_FIELDS = STATE_FIELDS + ("prg_bank", "chr_bank", "snap_chr_bank")


@pytest.mark.parametrize("rom", ["UXROM_ROM", "CNROM_ROM"])
@pytest.mark.parametrize("variant", ["shared", "global", "hybrid"])
def test_boards_match_checker(rom, variant, monkeypatch):
    """UxROM and CNROM cartridges (no counterpart in the reference): every field
    every step against the checker, env resets through the mask, a saved state
    loaded into another env, and all three frame formats."""
    monkeypatch.setenv("NESLE_STEP_KERNEL", variant)
    image = getattr(kat, rom)
    n = 100
    o = Oracle(n, 2, image)
    g = GpuCore(n, 2, image)
    rng = np.random.default_rng(11)
    for s in range(8):
        a = rng.integers(0, 256, n, dtype=np.uint8)
        o.step(a, auto_reset=False)
        g.step(a, auto_reset=False)
        assert_same(o, g, BOARD_FIELDS, f"{rom} {variant} step {s}")
        if s == 4:
            mask = (np.arange(n) % 5 == 0).astype(np.uint8)
            o.reset_envs(mask)
            g.reset_envs(mask)
            assert_same(o, g, BOARD_FIELDS, f"{rom} {variant} after reset_envs")
    ro, rg = o.render(), g.render()
    for k in ("index", "rgb", "gray84"):
        np.testing.assert_array_equal(ro[k], rg[k], err_msg=k)
    w_ = g.window(np.arange(n))
    blob = np.zeros((1, _lib.STATE_BYTES), np.uint8)
    idx = np.array([7], np.uint32)
    _lib.check(g.lib.nesle_save_states(g._h, idx.ctypes.data, 1, 0, blob.ctypes.data, 0, None))
    dst = np.array([8], np.uint32)
    _lib.check(g.lib.nesle_load_states(g._h, dst.ctypes.data, 1, 0, blob.ctypes.data, 0, None))
    for f in ("prg_bank", "chr_bank", "snap_chr_bank", "pc", "ram"):
        got = g.get(f)
        np.testing.assert_array_equal(got[8], got[7], err_msg=f"{f} after loading env 7's state into env 8")
    assert w_["pc"].shape == (n,)


def test_unsupported_boards_are_rejected():
    bad = kat.board_image(1, bytes(32768), bytes(8192))  # MMC1
    with pytest.raises(ValueError, match="supported cartridges"):
        GpuCore(4, 1, bad)


def test_unknown_placement_is_rejected(monkeypatch):
    monkeypatch.setenv("NESLE_STEP_KERNEL", "registers")
    with pytest.raises(ValueError, match="unknown placement 'registers'"):
        GpuCore(4, 1, kat.board_image(0, bytes(32768), bytes(8192)))


@pytest.mark.parametrize("variant", ["interleaved", "global-async", "hybrid-preload"])
def test_boards_fall_back_to_the_hybrid_placement(variant, monkeypatch):
    """Placements without a board instantiation run UxROM / CNROM batches on
    the hybrid kernel (shared and global are kept as asked)."""
    monkeypatch.setenv("NESLE_STEP_KERNEL", variant)
    g = GpuCore(8, 2, kat.UXROM_ROM)
    info = _lib.Info()
    _lib.check(g.lib.nesle_get_info(g._h, ctypes.byref(info)))
    assert _lib.PLACEMENTS[info.step_placement] == "hybrid"
