"""Pin the CPU checker (oracle/nes_oracle.c) before trusting it.

1. Known answers restated from the reference's own C++ tests.
2. Entry-by-entry equality with the reference decode table.
3. Bit-exact equality with the reference sources compiled unchanged
   (oracle/_ref): kind B (batched-kernel headers) on every config, and kind A
   (the nesle::Console CPU core) where no documented A/B divergence applies.
4. FCS parsing equality with the reference parser.
"""
from __future__ import annotations

import gzip
import os
from pathlib import Path

import numpy as np
import pytest

import kat_roms as kat
from nesle_b200 import workloads as w
from oracle import Oracle, Reference, reference_available

needs_ref = pytest.mark.skipif(not reference_available(), reason="oracle/_ref not built")


def _one(rom: bytes, snaps=(), **kw) -> Oracle:
    return Oracle(1, kw.pop("frameskip", 1), rom, list(snaps), **kw)


# --- 1. known answers (reference tests/cpp/*) --------------------------------

def test_kat_lda_tax_inx_sta_cycles():
    o = _one(kat.LDA_TAX_INX_STA)
    tr = o.step_traced(np.zeros(1, np.uint8), 0, auto_reset=False)
    assert list(tr["op"][:4]) == [0xA9, 0xAA, 0xE8, 0x8D]
    assert list(np.diff(np.r_[7, tr["cycles"][:4]])) == [2, 2, 2, 4]  # test_cpu.cpp:50-57
    assert tr["a"][3] == 0x41 and tr["x"][3] == 0x42
    assert o.get("ram")[0, 0x200] == 0x41


def test_kat_jsr_rts():
    o = _one(kat.JSR_RTS)
    tr = o.step_traced(np.zeros(1, np.uint8), 0, auto_reset=False)
    assert tr["pc"][1] == 0x9000 and tr["sp"][0] == 0xFB  # after JSR (test_cpu.cpp:70-71)
    assert tr["pc"][3] == 0x8003                           # after RTS (:74)
    assert o.get("ram")[0, 0x10] == 0x77                   # (:76)


def test_kat_branch_page_cross():
    o = _one(kat.BNE_PAGE_CROSS)
    tr = o.step_traced(np.zeros(1, np.uint8), 0, auto_reset=False)
    assert tr["op"][0] == 0xD0 and tr["cycles"][0] - 7 == 4 and tr["pc"][1] == 0x8100


def test_kat_sbc():
    o = _one(kat.SEC_SBC)
    tr = o.step_traced(np.zeros(1, np.uint8), 0, auto_reset=False)
    assert tr["a"][2] == 0x0F and tr["p"][2] & 1


def test_kat_nmi_first_frame():
    o = _one(kat.NMI_ROM)
    o.step(np.zeros(1, np.uint8), auto_reset=False)  # test_console.cpp:334-342
    assert o.get("ram")[0, 0] == 1
    assert o.get("nmi_pending")[0] == 0 and o.get("ppu_status")[0] & 0x80 == 0
    assert o.get("frame")[0] == 1


def test_kat_dma_cycles():
    o = _one(kat.DMA_ROM, [kat.dma_snapshot()])
    tr = o.step_traced(np.zeros(1, np.uint8), 0, auto_reset=False)
    assert tr["cycles"][0] == 2 and tr["cycles"][1] == 2 + 517  # test_console.cpp:356-359
    oam = o.get("oam")[0]
    assert oam[0] == 0xFF and oam[1] == 0xFE


@pytest.mark.parametrize("case", kat.REWARD_CASES)
def test_kat_reward(case):
    (pp, ps, pt), (cp, cs, ct, state), reward, done = case
    o = _one(kat.IDLE_ROM, [kat.mario_snapshot(pp, ps, pt)])
    o.poke_ram(0x6D, cp)
    o.poke_ram(0x86, cs)
    o.poke_ram(0x0E, state)
    for i, d in enumerate((ct // 100, (ct // 10) % 10, ct % 10)):
        o.poke_ram(0x7F8 + i, d)
    o.step(np.zeros(1, np.uint8), auto_reset=False)  # test_cuda_batch.cpp:82-87
    assert o.get("last_reward")[0] == reward
    assert o.get("last_done")[0] == done


def test_illegal_opcode_sets_status_and_freezes():
    rom = kat.rom_with({0x8000: bytes([0xA9, 0x05, 0x02])})  # LDA #5 ; JAM
    o = _one(rom)
    o.step(np.zeros(1, np.uint8), auto_reset=False)
    st = int(o.get("status")[0])
    assert st == 0x80000000 | (0x02 << 16) | 0x8002
    assert o.get("pc")[0] == 0x8002 and o.get("a")[0] == 5


def test_counter_rand_matches_python():
    for args in [(0, 1, 0, 0), (4, 2, 7, 3), (2**63 + 5, 1, 65535, 10**6)]:
        assert Oracle.counter_rand(*args) == int(w.counter_rand(*args))


# --- 2. decode table -----------------------------------------------------------

@needs_ref
def test_decode_table_matches_reference():
    om, oc, of = Oracle.decode_table()
    rm, rc, rf = Reference.decode_table()
    np.testing.assert_array_equal(om, rm)
    np.testing.assert_array_equal(oc, rc)
    np.testing.assert_array_equal(of, rf)


# --- 3. whole-path equality with the reference sources ------------------------

FIELDS_B = ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "prg_ram", "frame", "frame_dot",
            "ppu_status", "ppu_ctrl", "ppu_mask", "nmi_pending", "oam", "oam_addr", "v", "t", "w",
            "open_bus", "scroll_x", "scroll_y", "snap_oam", "snap_nt", "snap_sx_start", "snap_sx_end",
            "ctrl_shift", "ctrl_count", "ctrl_strobe", "reward", "last_reward", "done", "last_done",
            "prev_x", "prev_time", "stat_instructions", "stat_frames", "episode")
FIELDS_A = ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "frame", "ppu_status", "oam",
            "last_reward", "last_done", "prev_x", "prev_time")


def _run_pair(make, kind: str, n: int, steps: int, auto_reset: bool, fields) -> int:
    wl = make()
    env = np.arange(n)
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    kw = dict(env_to_level=e2l, done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, wl.frameskip, wl.rom.image, wl.snapshots, **kw)
    r = Reference(kind, n, wl.frameskip, wl.rom.image, wl.snapshots, **kw)
    dones = 0
    for s in range(steps):
        act = wl.actions(env, s)
        o.step(act, auto_reset=auto_reset)
        r.step(act, auto_reset=auto_reset)
        for f in fields:
            np.testing.assert_array_equal(o.get(f), r.get(f), err_msg=f"{wl.name} step {s} field {f}")
        dones += int(o.get("last_done").sum())
        assert (o.get("status") == 0).all()
    return dones


@needs_ref
@pytest.mark.parametrize("make,auto_reset", [(w.config1, False), (w.config2, True), (w.config3, True),
                                             (w.config4, True)])
def test_checker_matches_reference_batched(make, auto_reset):
    _run_pair(make, "B", 8, 10, auto_reset, FIELDS_B)


@needs_ref
@pytest.mark.parametrize("make,auto_reset", [(w.config1, False), (w.config2, True), (w.config4, True)])
def test_checker_matches_reference_cpu_core(make, auto_reset):
    _run_pair(make, "A", 8, 10, auto_reset, FIELDS_A)


@needs_ref
def test_checker_matches_reference_through_resets():
    """config 4 with a short frame limit so auto-reset fires many times."""
    def short():
        wl = w.config4()
        wl.done_args = (6, 20)
        return wl
    assert _run_pair(short, "B", 8, 12, True, FIELDS_B) > 0


@needs_ref
def test_checker_render_matches_reference_rgb():
    wl = w.config1()
    n = 4
    o = Oracle(n, 4, wl.rom.image)
    r = Reference("B", n, 4, wl.rom.image)
    for s in range(3):
        act = wl.actions(np.arange(n), s)
        o.step(act, auto_reset=False)
        r.step(act, auto_reset=False)
    ours = o.render()
    np.testing.assert_array_equal(ours["rgb"], r.render_rgb())


@needs_ref
def test_checker_config3_frames_match_reference_rgb():
    """Pixel configuration: sprites, per-frame scroll and the sprite-0 split, RGB byte-equal
    to the reference renderer after every env-step.  (Compared with the batched semantics
    only: the reference CPU core renders live state with one scroll and times sprite-0 hits
    per dot, both documented divergences.)"""
    wl = w.config3()
    n = 4
    env = np.arange(n)
    kw = dict(done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, [], **kw)
    r = Reference("B", n, 4, wl.rom.image, [], **kw)
    for s in range(4):
        a = wl.actions(env, s)
        o.step(a)
        r.step(a)
        np.testing.assert_array_equal(o.render()["rgb"], r.render_rgb(), err_msg=f"step {s}")
    assert (o.get("snap_sx_start") != o.get("snap_sx_end")).any()  # the split happened


@needs_ref
@pytest.mark.parametrize("make", [w.config1, w.config3, w.config4])
def test_checker_profile_histograms_match_reference(make):
    """step_profile: opcode and fetch-address histograms as console_step_kernel counts them."""
    wl = make()
    n = 6
    env = np.arange(n)
    e2l = wl.env_to_level(env) if wl.env_to_level else None
    kw = dict(env_to_level=e2l, done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, wl.snapshots, **kw)
    r = Reference("B", n, 4, wl.rom.image, wl.snapshots, **kw)
    for s in range(3):
        a = wl.actions(env, s)
        (oo, op), (ro, rp) = o.step_profile(a), r.step_profile(a)
        np.testing.assert_array_equal(oo, ro)
        np.testing.assert_array_equal(op, rp)
        assert int(oo.sum()) == int(o.get("stat_instructions").sum()) > 0
        o.step(a), r.step(a)  # and an ordinary step between profiles


# --- 4. FCS parsing -------------------------------------------------------------

@needs_ref
def test_fcs_writer_round_trips_through_reference_parser():
    s = w.random_snapshot(77, 0x8123, nmi_and_rendering=True)
    s.ppu_v, s.ppu_t, s.ppu_x, s.ppu_w, s.ppu_open_bus, s.ppu_read_buffer = 0x2345, 0x1234, 5, 1, 0x90, 0xFF
    d = Reference.parse_fcs(w.write_fcs(s))
    assert (d["pc"], d["a"], d["x"], d["y"], d["sp"], d["p"]) == (s.pc, s.a, s.x, s.y, s.sp, s.p)
    assert (d["ctrl"], d["mask"], d["v"], d["t"], d["fine_x"], d["w"]) == (0x80, 0x1E, 0x2345, 0x1234, 5, 1)
    assert (d["open_bus"], d["read_buffer"]) == (0x90, 0xFF)
    assert d["ram"] == s.cpu_ram


def _reference_state_files():
    root = Path(os.environ.get("NESLE_REFERENCE", Path(__file__).resolve().parents[2] / "reference"))
    return sorted((root / "docs" / "data").glob("smb_level*_1.state"))


@needs_ref
@pytest.mark.skipif(not _reference_state_files(), reason="reference FCS fixtures not present")
def test_reference_fcs_known_values():
    """Known values of smb_level1_1.state (reference tests/test_fcs_parser.py:30-96)."""
    data = gzip.decompress(_reference_state_files()[0].read_bytes())
    d = Reference.parse_fcs(data)
    assert (d["pc"], d["a"], d["x"], d["y"], d["sp"], d["p"]) == (0x8057, 0x90, 0x00, 0x01, 0xFF, 0xA5)
    assert (d["ctrl"], d["mask"], d["status"], d["v"], d["t"]) == (0x90, 0x1E, 0x40, 0x0800, 0)
    assert (d["read_buffer"], d["open_bus"], d["pal"][0]) == (0xFF, 0x90, 0x22)


def test_touched_ram_fraction_of_the_benchmark_workload():
    """Config 4 (the metric's workload) touches >= 95% of each env's RAM sectors per
    env-step, so its HBM bound is the full 4,476-B round trip; config 3 touches fewer."""
    def fraction(make, steps=8, n=16):
        wl = make()
        env = np.arange(n)
        e2l = wl.env_to_level(env) if wl.env_to_level else None
        o = Oracle(n, 4, wl.rom.image, wl.snapshots, env_to_level=e2l, done_mode=wl.done_mode,
                   done_args=wl.done_args, seed=wl.seed)
        out = []
        for s in range(steps):
            o.step(wl.actions(env, s))
            if s >= 2:
                out += [bin(int(t)).count("1") / 64 for t in o.get("ram_touch")]
        return float(np.mean(out))

    assert fraction(w.config4) >= 0.95
    assert fraction(w.config3) < 0.95

