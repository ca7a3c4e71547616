"""Tiny known-answer ROMs and snapshots, restating the fixtures the reference's
own C++ tests build in code (tests/cpp/test_cpu.cpp, test_console.cpp,
test_cuda_batch.cpp, test_cuda_batch_console.cpp).  Shared by the checker
pin tests (CPU) and the GPU parity tests, so both sides run the same inputs.
"""
from __future__ import annotations

import struct

from nesle_b200 import workloads as w


def rom_with(code: dict[int, bytes], reset: int = 0x8000, nmi: int = 0x9000,
             irq: int = 0x9000, chr_rom: bytes | None = None, flags6: int = 0x01) -> bytes:
    """32 KB NROM image filled with NOP ($EA), code placed at CPU addresses."""
    prg = bytearray([0xEA]) * 32768
    for addr, data in code.items():
        prg[addr - 0x8000: addr - 0x8000 + len(data)] = data
    prg[0x7FFA:0x7FFC] = struct.pack("<H", nmi)
    prg[0x7FFC:0x7FFE] = struct.pack("<H", reset)
    prg[0x7FFE:0x8000] = struct.pack("<H", irq)
    return w.ines_image(bytes(prg), chr_rom if chr_rom is not None else bytes(8192), flags6)


def asm(base: int, *lines) -> bytes:
    a = w.Asm(base)
    for ln in lines:
        if isinstance(ln, bytes):
            a.raw(ln)
        else:
            a.emit(*ln)
    return a.assemble()[0]


# test_cpu.cpp:34-56  LDA #$41 / TAX / INX / STA $0200 -> cycles 2,2,2,4
LDA_TAX_INX_STA = rom_with({0x8000: asm(0x8000, ("LDA", w.IMM, 0x41), ("TAX",), ("INX",),
                                        ("STA", w.ABS, 0x0200), ("JMP", w.ABS, 0x800A))})

# test_cpu.cpp:58-76  JSR $9000 / (LDA #$77 / RTS) / STA $10
JSR_RTS = rom_with({0x8000: asm(0x8000, ("JSR", w.ABS, 0x9000), ("STA", w.ZP, 0x10),
                                ("JMP", w.ABS, 0x8005)),
                    0x9000: asm(0x9000, ("LDA", w.IMM, 0x77), ("RTS",))}, nmi=0xA000)

# test_cpu.cpp:78-86  BNE +1 at $80FD, taken across a page: 4 cycles, pc=$8100
BNE_PAGE_CROSS = rom_with({0x80FD: bytes([0xD0, 0x01]), 0x8100: asm(0x8100, ("JMP", w.ABS, 0x8100))},
                          reset=0x80FD)

# test_cpu.cpp:88-101  SEC / LDA #$10 / SBC #$01 -> A=$0F, C=1
SEC_SBC = rom_with({0x8000: asm(0x8000, ("SEC",), ("LDA", w.IMM, 0x10), ("SBC", w.IMM, 0x01),
                                ("JMP", w.ABS, 0x8005))})

# test_console.cpp:72-92 / test_cuda_batch_console.cpp  NMI: INC $00 / RTI at $9000
NMI_ROM = rom_with({0x8000: asm(0x8000, ("LDA", w.IMM, 0x80), ("STA", w.ABS, 0x2000),
                                ("JMP", w.ABS, 0x8005)),
                    0x9000: asm(0x9000, ("INC", w.ZP, 0x00), ("RTI",))})

# test_console.cpp:94-110  LDA #$02 / STA $4014 -> 2 then 517 CPU cycles
DMA_ROM = rom_with({0x8000: asm(0x8000, ("LDA", w.IMM, 0x02), ("STA", w.ABS, 0x4014),
                                ("JMP", w.ABS, 0x8005))})

# OAM DMA from page $00 and from its mirror $08 ((page << 8) & $7FF = $000):
# the source is the zero page.
DMA_ZP_ROM = rom_with({0x8000: asm(0x8000, ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x4014), ("INC", w.ZP, 0x10),
                                   ("LDA", w.IMM, 0x08), ("STA", w.ABS, 0x4014), ("JMP", w.ABS, 0x800C))})

IDLE_ROM = rom_with({0x8000: asm(0x8000, ("JMP", w.ABS, 0x8000))})


def dma_zp_snapshot() -> bytes:
    """PC at $8000 with RAM $0000+i = 3 i + 1 (mod 256)."""
    ram = bytearray(2048)
    for i in range(256):
        ram[i] = (3 * i + 1) & 0xFF
    return w.write_fcs(w.Snapshot(pc=0x8000, cpu_ram=bytes(ram)))


def dma_snapshot() -> bytes:
    """PC at $8000 with RAM $0200+i = $FF-i (test_console.cpp:99-101)."""
    ram = bytearray(2048)
    for i in range(256):
        ram[0x200 + i] = 0xFF - i
    return w.write_fcs(w.Snapshot(pc=0x8000, cpu_ram=bytes(ram)))


def mario_snapshot(x_page: int, x_screen: int, timer: int, player_state: int = 8,
                   y_viewport: int = 1) -> bytes:
    """RAM laid out like test_cuda_batch.cpp:21-33, PC parked on an idle JMP."""
    ram = bytearray(2048)
    ram[0x6D] = x_page
    ram[0x86] = x_screen
    ram[0xB5] = y_viewport
    ram[0x0E] = player_state
    ram[0x75A] = 2
    ram[0x7F8:0x7FB] = bytes([timer // 100, (timer // 10) % 10, timer % 10])
    return w.write_fcs(w.Snapshot(pc=0x8000, cpu_ram=bytes(ram)))


# Reward cases of test_cuda_batch.cpp:45-87: (previous x, previous timer) come
# from the snapshot, the current values are poked into RAM before the step.
REWARD_CASES = [
    # prev (page, screen, timer), current (page, screen, timer, player_state), reward, done
    ((0, 40, 400), (0, 43, 399, 8), 2.0, 0),
    ((0, 80, 399), (0, 90, 398, 8), -1.0, 0),
    ((0, 48, 400), (0, 50, 399, 0x0B), -24.0, 1),
]


# Render coverage beyond what snapshots alone reach (a warm reset zeroes the
# scroll): PPUCTRL/PPUMASK from RAM $10/$11 (NMI and both layers forced on),
# then $2005 rewritten in the main loop from RAM $12/$13, which also change
# every pass, so the scroll latched at the frame's start and the one captured
# at vblank differ (the two-region split).  The NMI handler DMAs OAM from page
# $02 and moves sprite 0, so the split row changes from frame to frame.
_RS_INIT = asm(0x8000, ("LDA", w.ZP, 0x10), ("ORA", w.IMM, 0x80), ("STA", w.ABS, 0x2000),
               ("LDA", w.ZP, 0x11), ("ORA", w.IMM, 0x18), ("STA", w.ABS, 0x2001))
_RS_LOOP = 0x8000 + len(_RS_INIT)
RENDER_SCROLL_ROM = rom_with(
    {0x8000: _RS_INIT + asm(_RS_LOOP, ("LDA", w.ZP, 0x12), ("STA", w.ABS, 0x2005), ("LDA", w.ZP, 0x13),
                            ("STA", w.ABS, 0x2005), ("INC", w.ZP, 0x12), ("DEC", w.ZP, 0x13),
                            ("JMP", w.ABS, _RS_LOOP)),
     0x9000: asm(0x9000, ("PHA",), ("LDA", w.IMM, 0x02), ("STA", w.ABS, 0x4014), ("INC", w.ABS, 0x0203),
                 ("INC", w.ABS, 0x0200), ("PLA",), ("RTI",))},
    chr_rom=bytes(__import__("numpy").random.default_rng(77).integers(0, 256, 8192, dtype="uint8")))


def render_scroll_snapshots(seed: int, k: int) -> list[bytes]:
    """k snapshots at the ROM's reset code with random RAM (so random control,
    mask and scroll bytes), nametables, palette and OAM."""
    import numpy as np

    rng = np.random.default_rng(seed)
    out = []
    for i in range(k):
        s = w.random_snapshot(seed + i, 0x8000, nmi_and_rendering=True)
        s.nametable_ram = rng.integers(0, 256, 2048, dtype=np.uint8).tobytes()
        s.palette_ram = rng.integers(0, 64, 32, dtype=np.uint8).tobytes()
        s.oam = rng.integers(0, 256, 256, dtype=np.uint8).tobytes()
        out.append(w.write_fcs(s))
    return out


# Controller protocol (batch_bus.cuh:105-133): reads with the strobe held high
# (the live A bit, no shifting), then 12 reads after it drops (8 latched bits,
# then 1s), and $4017 (constant $41 in the batched bus).  The loop is short and
# its length depends on the A bit, so step boundaries land everywhere in it,
# strobe high and mid-sequence included, at different points in different envs.
def _controller_rom() -> bytes:
    a = w.Asm(0x8000)
    a.emit("LDA", w.IMM, 0x01)
    a.emit("STA", w.ABS, 0x4016)
    a.emit("LDA", w.ABS, 0x4016)
    a.emit("STA", w.ZP, 0x10)
    a.emit("LDA", w.ABS, 0x4016)
    a.emit("STA", w.ZP, 0x11)
    a.emit("AND", w.IMM, 0x01)
    a.branch("BEQ", "even")
    for _ in range(4):
        a.emit("NOP")
    a.label("even")
    a.emit("LDA", w.IMM, 0x00)
    a.emit("STA", w.ABS, 0x4016)
    a.emit("LDX", w.IMM, 0x00)
    a.label("rd")
    a.emit("LDA", w.ABS, 0x4016)
    a.emit("STA", w.ZPX, 0x20)
    a.emit("INX")
    a.emit("CPX", w.IMM, 0x0C)
    a.branch("BNE", "rd")
    a.emit("LDA", w.ABS, 0x4017)
    a.emit("STA", w.ZP, 0x30)
    a.emit("INC", w.ZP, 0x40)
    a.emit("JMP", w.ABS, 0x8000)
    return rom_with({0x8000: a.assemble()[0]})


CONTROLLER_ROM = _controller_rom()


# The reference VecEnv trace (tests/golden/make_ref_callers.py,
# tests/test_ref_callers.py): dones that depend on the action, so auto-reset
# masks are partial.  The NMI handler strobes the controller and reads A; while
# A is held, $B5 counts up (the SMB predicate's "dying": $B5 > 1), so an env
# whose action holds A for a whole env-step (4 frames) is done at its end.  It
# also advances $86 (SMB x) every frame, so rewards are +4 per env-step.  The
# main loop does indexed RAM work and draws nothing in particular.
_TRACE_LOOP = 0x8000 + 12  # after the reset code and LDX #0
ENV_TRACE_ROM = rom_with({
    0x8000: asm(0x8000, ("LDA", w.IMM, 0x80), ("STA", w.ABS, 0x2000), ("LDA", w.IMM, 0x1E), ("STA", w.ABS, 0x2001),
                ("LDX", w.IMM, 0x00),
                ("INC", w.ABS, 0x0300), ("LDA", w.ABS, 0x0300), ("STA", w.ABSX, 0x0400), ("INX",),
                ("ADC", w.ZP, 0x40), ("STA", w.ZP, 0x40), ("JMP", w.ABS, _TRACE_LOOP)),
    0x9000: asm(0x9000, ("PHA",), ("LDA", w.IMM, 0x01), ("STA", w.ABS, 0x4016), ("LDA", w.IMM, 0x00),
                ("STA", w.ABS, 0x4016), ("LDA", w.ABS, 0x4016), ("AND", w.IMM, 0x01), ("BEQ", w.REL, 0x02),
                ("INC", w.ZP, 0xB5), ("INC", w.ZP, 0x86), ("PLA",), ("RTI",)),
})


def env_trace_snapshots(k: int = 8) -> list[bytes]:
    """k levels parked at the trace ROM's loop, alive ($0E = 8, $B5 = 0), with
    different x positions and loop counters, NMI and rendering on."""
    snaps = []
    for lvl in range(k):
        ram = bytearray(2048)
        ram[0x0E], ram[0xB5], ram[0x75A], ram[0x770] = 8, 0, 2, 1
        ram[0x86], ram[0x6D] = 16 * lvl, lvl & 1
        ram[0x300], ram[0x40] = 7 * lvl, lvl
        ram[0x7F8:0x7FB] = bytes([3, 0, 0])
        snaps.append(w.write_fcs(w.Snapshot(pc=_TRACE_LOOP, a=lvl, x=3 * lvl, cpu_ram=bytes(ram), ppu_ctrl=0x80,
                                            ppu_mask=0x1E)))
    return snaps


# Cartridge boards beyond NROM (no counterpart in the reference, which is
# NROM-only): UxROM (mapper 2) and CNROM (mapper 3).  Both select a bank by a
# write to $8000-$FFFF whose value is ANDed with the ROM byte at that address
# (bus conflict), so the programs write through a table of bank numbers.
def board_image(mapper: int, prg: bytes, chr_rom: bytes, flags6: int = 0x01) -> bytes:
    assert len(prg) % 16384 == 0 and len(chr_rom) % 8192 == 0
    header = b"NES\x1a" + bytes([len(prg) // 16384, len(chr_rom) // 8192, flags6 | ((mapper & 0xF) << 4),
                                 mapper & 0xF0]) + bytes(8)
    return header + prg + chr_rom


def _joypad_bits(n: int) -> list:
    """Strobe the controller, then read n buttons into X: X = b0 | b1 << 1 | ..."""
    lines = [("LDA", w.IMM, 1), ("STA", w.ABS, 0x4016), ("LDA", w.IMM, 0), ("STA", w.ABS, 0x4016),
             ("LDX", w.IMM, 0), ("STX", w.ZP, 0x20)]
    for k in range(n):
        lines += [("LDA", w.ABS, 0x4016), ("AND", w.IMM, 1)]
        lines += [("ASL", w.ACC)] * k
        lines += [("ORA", w.ZP, 0x20), ("STA", w.ZP, 0x20)]
    lines += [("LDX", w.ZP, 0x20)]
    return lines


def _uxrom_rom() -> bytes:
    """64 KB UxROM: 4 switchable banks, each with a routine at $8000 that
    stores its bank's signature (read from $8010) and counts its calls; the
    fixed bank picks a bank from two joypad bits each pass (no conflict), then
    writes $FF over a table byte holding 1 (conflict: bank 1), calling each."""
    banks = []
    for b in range(4):
        bank = bytearray([0xEA]) * 16384
        code = asm(0x8000, ("LDA", w.ABS, 0x8010), ("STA", w.ABS, 0x0310 + b), ("INC", w.ABS, 0x0320 + b),
                   ("LDA", w.ABSY, 0x8011), ("STA", w.ZP, 0x30), ("RTS",))
        bank[:len(code)] = code
        bank[0x10] = 0xA0 + b
        bank[0x11:0x15] = bytes([(0x11 * (b + 1) + 4 * j) & 0xFF for j in range(4)])
        banks.append(bank)
    fixed = banks[3]
    table = 0xC100
    main = asm(0xC000, ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2000), ("LDY", w.IMM, 0x00),
               *_joypad_bits(2), ("LDA", w.ABSX, table), ("STA", w.ABSX, table), ("JSR", w.ABS, 0x8000),
               ("LDA", w.IMM, 0xFF), ("STA", w.ABS, table + 1), ("JSR", w.ABS, 0x8000),
               ("INY",), ("TYA",), ("AND", w.IMM, 3), ("TAY",), ("INC", w.ABS, 0x0300), ("JMP", w.ABS, 0xC004))
    fixed[0x4000 - 0x4000:len(main)] = main
    fixed[0x100:0x104] = bytes([0, 1, 2, 3])
    fixed[0x3FFA:0x3FFC] = struct.pack("<H", 0xC000)  # NMI (off)
    fixed[0x3FFC:0x3FFE] = struct.pack("<H", 0xC000)
    fixed[0x3FFE:0x4000] = struct.pack("<H", 0xC000)
    return board_image(2, b"".join(bytes(x) for x in banks), bytes((i * 7) & 0xFF for i in range(8192)))


def _cnrom_rom() -> bytes:
    """32 KB PRG, 4 CHR banks of distinct patterns (CNROM).  Reset fills the
    first nametable with a tile ramp and the palette, turns rendering and NMI
    on; the main loop selects a CHR bank from two joypad bits, reads a
    pattern byte back through $2006/$2007 into RAM and waits for vblank."""
    prg = bytearray([0xEA]) * 32768
    table = 0xE000
    init = [("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2000), ("STA", w.ABS, 0x2001),
            ("LDA", w.IMM, 0x3F), ("STA", w.ABS, 0x2006), ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2006),
            ("LDX", w.IMM, 0x00)]
    pal = asm(0x8000, *init)
    fill_pal = asm(0x8000 + len(pal), ("TXA",), ("ASL", w.ACC), ("ADC", w.IMM, 0x05), ("STA", w.ABS, 0x2007),
                   ("INX",), ("CPX", w.IMM, 0x20), ("BNE", w.REL, 0xF5))
    nt_start = asm(0x8000 + len(pal) + len(fill_pal), ("LDA", w.IMM, 0x20), ("STA", w.ABS, 0x2006),
                   ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2006), ("LDY", w.IMM, 0x04), ("LDX", w.IMM, 0x00))
    base = 0x8000 + len(pal) + len(fill_pal) + len(nt_start)
    fill_nt = asm(base, ("TXA",), ("STA", w.ABS, 0x2007), ("INX",), ("BNE", w.REL, 0xF9), ("DEY",),
                  ("BNE", w.REL, 0xF6))
    on = asm(base + len(fill_nt), ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2005), ("STA", w.ABS, 0x2005),
             ("LDA", w.IMM, 0x80), ("STA", w.ABS, 0x2000), ("LDA", w.IMM, 0x1E), ("STA", w.ABS, 0x2001))
    head = base + len(fill_nt) + len(on)
    loop = asm(head, *_joypad_bits(2), ("LDA", w.ABSX, table), ("STA", w.ABSX, table),
               ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2006), ("LDA", w.IMM, 0x10), ("STA", w.ABS, 0x2006),
               ("LDA", w.ABS, 0x2007), ("LDA", w.ABS, 0x2007), ("STA", w.ABS, 0x0340), ("STX", w.ABS, 0x0341),
               ("INC", w.ABS, 0x0342), ("LDA", w.IMM, 0x00), ("STA", w.ABS, 0x2005), ("STA", w.ABS, 0x2005),
               ("JMP", w.ABS, head))
    code = pal + fill_pal + nt_start + fill_nt + on + loop
    prg[:len(code)] = code
    prg[table - 0x8000:table - 0x8000 + 4] = bytes([0, 1, 2, 3])
    prg[0x7000:0x7002] = bytes([0x40, 0x40])  # NMI: RTI
    prg[0x7FFA:0x7FFC] = struct.pack("<H", 0xF000)
    prg[0x7FFC:0x7FFE] = struct.pack("<H", 0x8000)
    prg[0x7FFE:0x8000] = struct.pack("<H", 0xF000)
    chr_rom = bytes(((i * (k + 3)) ^ (k * 0x55) ^ (i >> 4)) & 0xFF for k in range(4) for i in range(8192))
    return board_image(3, bytes(prg), chr_rom)


UXROM_ROM = _uxrom_rom()
CNROM_ROM = _cnrom_rom()
