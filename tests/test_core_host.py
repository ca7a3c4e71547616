"""The product kernel core (nesle_b200/csrc/nes_core.cuh), compiled for the
CPU, against the checker.  Same inputs, bit-exact state after every step."""
from __future__ import annotations

import numpy as np
import pytest

import kat_roms as kat
from harness import (STATE_FIELDS, HostCore, HostCoreEarly1, HostCoreGlobal, HostCoreGlobalAsync, HostCoreHybrid,
                     HostCoreHybridAsync, HostCoreHybridEarly1, HostCoreHybridEarly2, HostCoreHybridStack,
                     HostCoreHybridV1, HostCoreV1, assert_same, run_lockstep)
from nesle_b200 import workloads as w
from oracle import Oracle

# Every RAM placement of the step kernel, each compiled for the CPU.
ALL_CORES = [HostCore, HostCoreGlobal, HostCoreHybrid, HostCoreHybridStack, HostCoreGlobalAsync, HostCoreHybridAsync,
             HostCoreEarly1, HostCoreHybridEarly1, HostCoreHybridEarly2, HostCoreV1, HostCoreHybridV1]


@pytest.mark.parametrize("make,auto_reset", [(w.config1, False), (w.config2, True), (w.config3, True),
                                             (w.config4, True)])
def test_configs_lockstep(make, auto_reset):
    run_lockstep(make, 8, 8, auto_reset, ALL_CORES)


def test_config3_frames_match_checker_every_step():
    """Pixel mode: index, RGB and 84x84 gray frames after every env-step."""
    wl = w.config3()
    n = 4
    env = np.arange(n)
    kw = dict(done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, [], **kw)
    h = HostCoreGlobal(n, 4, wl.rom.image, [], **kw)
    for s in range(4):
        a = wl.actions(env, s)
        o.step(a)
        h.step(a)
        ro, rh = o.render(), h.render()
        for k in ("index", "rgb", "gray84"):
            np.testing.assert_array_equal(ro[k], rh[k], err_msg=f"step {s} {k}")
    assert all(len(np.unique(ro["index"][e])) > 4 for e in range(n))


def test_frame_limit_auto_reset_lockstep():
    def short():
        wl = w.config4()
        wl.done_args = (5, 17)
        return wl
    _, _, dones = run_lockstep(short, 12, 20, True, ALL_CORES)
    assert dones > 10


def test_smb_done_auto_reset_every_step():
    """config 1 under the SMB predicate is done almost every step: cold auto-resets."""
    _, _, dones = run_lockstep(w.config1, 6, 6, True, [HostCore])
    assert dones > 0


@pytest.mark.parametrize("rom,snaps", [
    (kat.LDA_TAX_INX_STA, []), (kat.JSR_RTS, []), (kat.BNE_PAGE_CROSS, []), (kat.SEC_SBC, []),
    (kat.NMI_ROM, []), (kat.DMA_ROM, [kat.dma_snapshot()]), (kat.DMA_ZP_ROM, [kat.dma_zp_snapshot()]),
    (kat.IDLE_ROM, [])])
@pytest.mark.parametrize("core", ALL_CORES)
def test_known_answer_roms(rom, snaps, core):
    o = Oracle(2, 2, rom, snaps)
    h = core(2, 2, rom, snaps)
    for _ in range(3):
        a = np.array([0x81, 0x00], np.uint8)
        o.step(a, auto_reset=False)
        h.step(a, auto_reset=False)
        assert_same(o, h)


def _single_instruction_cases(seed: int, per_opcode: int):
    """(rom, snapshot) pairs: one opcode with random operands, then JMP-to-self."""
    rng = np.random.default_rng(seed)
    for opc in sorted(w.OPCODES):
        mn, mode = w.OPCODES[opc]
        for k in range(per_opcode):
            ops = rng.integers(0, 256, size=2)
            if mode in (w.ABS, w.ABSX, w.ABSY) and mn not in ("JMP", "JSR"):
                # mix RAM, PRG and PRG-RAM targets
                ops[1] = rng.choice([0x00, 0x03, 0x07, 0x80, 0x9F, 0xFF, 0x60, 0x7F])
            code = bytes([opc, *ops[: w.MODE_LEN[mode] - 1]])
            after = 0x8000 + len(code)
            body = {0x8000: code, after: bytes([0x4C, after & 0xFF, after >> 8])}
            if mn in ("JMP", "JSR"):
                tgt = 0x9000 + k
                body[0x8000] = bytes([opc, tgt & 0xFF, tgt >> 8])
                body[tgt] = bytes([0x4C, tgt & 0xFF, tgt >> 8])
                if mode == w.IND:  # pointer in RAM, target in PRG
                    body[0x8000] = bytes([opc, 0x10 + k, 0x03])
            rom = kat.rom_with(body, nmi=0xC000, irq=0xC100)
            ram = bytearray(rng.integers(0, 256, size=2048, dtype=np.uint8).tobytes())
            if mode == w.IND:
                ram[0x310 + k] = 0x00
                ram[0x311 + k] = 0xC2
            s = w.Snapshot(pc=0x8000, a=int(rng.integers(256)), x=int(rng.integers(256)), y=int(rng.integers(256)),
                           sp=int(rng.integers(256)), p=int(rng.integers(256)) & 0xEF, cpu_ram=bytes(ram))
            yield opc, rom, w.write_fcs(s)


@pytest.mark.parametrize("seed", [1, 2])
def test_every_official_opcode_from_random_state(seed):
    """Each official opcode once from a random register/flag/RAM state (P bit 5 may be clear)."""
    for opc, rom, snap in _single_instruction_cases(seed, 1):
        o = Oracle(1, 1, rom, [snap])
        sims = [cls(1, 1, rom, [snap]) for cls in ALL_CORES]
        a = np.zeros(1, np.uint8)
        o.step(a, auto_reset=False)
        for h in sims:
            h.step(a, auto_reset=False)
            try:
                assert_same(o, h, ("pc", "a", "x", "y", "sp", "p", "cycles", "ram", "prg_ram", "status"))
            except AssertionError as e:
                raise AssertionError(f"opcode {opc:#04x} ({type(h).__name__}): {e}") from None


def render_snapshots(seed: int, k: int, pc: int) -> list[bytes]:
    """Snapshots with random nametables, palette and OAM and rendering on, so
    rendered frames exercise background, attributes, sprites and both views."""
    rng = np.random.default_rng(seed)
    out = []
    for i in range(k):
        s = w.random_snapshot(seed + i, pc, nmi_and_rendering=True)
        s.nametable_ram = rng.integers(0, 256, 2048, dtype=np.uint8).tobytes()
        s.palette_ram = rng.integers(0, 64, 32, dtype=np.uint8).tobytes()
        s.oam = rng.integers(0, 256, 256, dtype=np.uint8).tobytes()
        s.ppu_ctrl = 0x80 | int(rng.integers(0, 64)) & 0x3B
        s.ppu_mask = 0x1E | int(rng.integers(0, 2))
        out.append(w.write_fcs(s))
    return out


def test_render_matches_checker():
    wl = w.config4()
    n = 4
    snaps = render_snapshots(5, 4, wl.rom.loop_head)
    kw = dict(env_to_level=np.arange(n) % 4, done_mode=wl.done_mode, done_args=wl.done_args, seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, snaps, **kw)
    h = HostCore(n, 4, wl.rom.image, snaps, **kw)
    for s in range(3):
        a = wl.actions(np.arange(n), s)
        o.step(a)
        h.step(a)
    ro, rh = o.render(), h.render()
    for k in ("index", "rgb", "gray84"):
        np.testing.assert_array_equal(ro[k], rh[k], err_msg=k)
    assert len(np.unique(ro["index"])) > 8  # the frames have content


def test_reset_envs_poke_and_host_step():
    wl = w.config4()
    n = 6
    kw = dict(env_to_level=wl.env_to_level(np.arange(n)), done_mode=wl.done_mode, done_args=wl.done_args,
              seed=wl.seed)
    o = Oracle(n, 4, wl.rom.image, wl.snapshots, **kw)
    h = HostCore(n, 4, wl.rom.image, wl.snapshots, **kw)
    a = wl.actions(np.arange(n), 0)
    o.step(a, device_api=False)
    h.step(a, device_api=False)
    assert_same(o, h)
    mask = np.array([1, 0, 1, 0, 0, 1], np.uint8)
    o.reset_envs(mask)
    h.reset_envs(mask)
    o.poke_ram(0x123, 0x45)
    h.poke_ram(0x123, 0x45)
    assert_same(o, h)
    o.step(a)
    h.step(a)
    assert_same(o, h)
    o.reset()
    h.reset()
    assert_same(o, h)


def test_illegal_opcode_freezes_env():
    rom = kat.rom_with({0x8000: bytes([0xA9, 0x05, 0x02])})
    o = Oracle(2, 2, rom)
    h = HostCore(2, 2, rom)
    for _ in range(2):
        o.step(np.zeros(2, np.uint8), auto_reset=False)
        h.step(np.zeros(2, np.uint8), auto_reset=False)
        assert_same(o, h)
    assert (h.get("status") == (0x80000000 | 0x020000 | 0x8002)).all()


def test_render_scroll_split_matches_checker():
    """Random control, mask and mid-frame scroll (two-region split with a moving
    sprite 0), random CHR, nametables, palette and OAM: frames in all three
    formats after every step."""
    n = 16
    snaps = kat.render_scroll_snapshots(5, 8)
    kw = dict(env_to_level=np.arange(n) % 8)
    o = Oracle(n, 4, kat.RENDER_SCROLL_ROM, snaps, **kw)
    h = HostCore(n, 4, kat.RENDER_SCROLL_ROM, snaps, **kw)
    for _ in range(3):
        o.step(np.zeros(n, np.uint8), auto_reset=False)
        h.step(np.zeros(n, np.uint8), auto_reset=False)
        assert_same(o, h, label="render-scroll")
        ro, rh = o.render(), h.render()
        for k in ("index", "rgb", "gray84"):
            np.testing.assert_array_equal(ro[k], rh[k], err_msg=k)
    assert (o.get("snap_sx_start") != o.get("snap_sx_end")).any()


@pytest.mark.parametrize("cls", ALL_CORES)
def test_controller_protocol_matches_checker(cls):
    """Strobe-high reads, reads past the 8 latched bits and $4017, with step
    boundaries at every point of the read sequence (the controller shift
    register is one marker word inside a step, shift/count in the record)."""
    n = 16
    o = Oracle(n, 1, kat.CONTROLLER_ROM, [])
    h = cls(n, 1, kat.CONTROLLER_ROM, [])
    rng = np.random.default_rng(0)
    for _ in range(12):
        a = rng.integers(0, 256, n, dtype=np.uint8)
        o.step(a, auto_reset=False)
        h.step(a, auto_reset=False)
        assert_same(o, h, label="controller")


BOARD_FIELDS = STATE_FIELDS + ("prg_bank", "chr_bank", "snap_chr_bank")


@pytest.mark.parametrize("rom", ["UXROM_ROM", "CNROM_ROM"])
@pytest.mark.parametrize("core", [HostCore, HostCoreGlobal, HostCoreHybrid, HostCoreV1, HostCoreHybridV1])
def test_boards_match_checker(rom, core):
    """UxROM and CNROM (bank writes with bus conflicts, code and data in the
    switchable PRG bank, banked CHR read through $2007 and rendered from the
    bank latched at vblank): every field every step, frames at the end."""
    image = getattr(kat, rom)
    n = 12
    o = Oracle(n, 2, image)
    h = core(n, 2, image)
    rng = np.random.default_rng(3)
    for s in range(8):
        a = rng.integers(0, 256, n, dtype=np.uint8)
        o.step(a, auto_reset=False)
        h.step(a, auto_reset=False)
        assert_same(o, h, BOARD_FIELDS, f"{rom} step {s}")
    ro, rh = o.render(), h.render()
    for k in ("index", "rgb", "gray84"):
        np.testing.assert_array_equal(ro[k], rh[k], err_msg=k)
    assert len(np.unique(o.get("prg_bank" if rom == "UXROM_ROM" else "chr_bank"))) > 1
