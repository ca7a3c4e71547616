"""Seeded synthetic workloads for the batched NES core.

The reference measures its env-step kernel on the commercial Super Mario Bros.
ROM, which is not available here.  These generators build the stand-in inputs
the benchmark configurations describe: mapper-0 iNES images whose main loop is
random official 6502 code, FCEUX ``FCS`` save states used as reset snapshots,
and per-env action streams drawn from a counter-based RNG so that the CPU
checker and the GPU kernel see identical inputs without sharing any state.

Design constraints on the generated code (all enforced here, checked by the
tests through the CPU checker):

* Data accesses of the random code stay inside CPU RAM ($0000-$08FE) or read
  PRG ROM (immediates).  Zero-page and absolute operands are drawn from $00-$FF
  and $0300-$07FF; indexed absolute accesses reach at most $08FE (a RAM mirror).
* Indirect modes read their pointer from zero page, which random stores can
  overwrite.  Every ``(zp,X)`` / ``(zp),Y`` instruction is therefore preceded by
  a transparent guard ``PHP PHA LDA #lo STA p LDA #hi STA p+1 PLA PLP`` that
  writes a pointer into $0300-$06FF and restores A, P and SP.  This keeps the
  reference CPU core (``nesle::Console``) and the reference batched bus on the
  same side of every documented divergence (open-bus reads of write-only PPU
  registers, $4000-$4017 reads, OAM-DMA sources above $1FFF).
* Branch targets are forward, inside the block, on drawn-instruction
  boundaries (never inside a guard).
* Illegal opcode $02 fills unreachable PRG space, so any control-flow escape is
  caught by the checker's illegal-opcode status instead of running silently.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass, field
from typing import Callable, Sequence

import numpy as np

from .fcs import Snapshot, write_fcs  # noqa: F401  (FCS writer; snapshots are a workload input)

# ---------------------------------------------------------------------------
# Counter-based RNG (SplitMix64 finaliser, Steele/Lea/Flood 2014).  The same
# function is restated in C (oracle/nes_oracle.c) and CUDA (csrc/nes_core.cuh).
# ---------------------------------------------------------------------------

_M64 = np.uint64(0xFFFFFFFFFFFFFFFF)
STREAM_ACTION = 1
STREAM_FRAME_LIMIT = 2


def splitmix64(x: np.ndarray | int) -> np.ndarray:
    z = np.asarray(x, dtype=np.uint64) + np.uint64(0x9E3779B97F4A7C15)
    with np.errstate(over="ignore"):
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
    return z ^ (z >> np.uint64(31))


def counter_rand(seed: int, stream: int, a: np.ndarray | int, b: np.ndarray | int) -> np.ndarray:
    """64-bit value for counter (seed, stream, a, b): mix(mix(mix(seed ^ stream<<56) ^ a) ^ b)."""
    k = splitmix64(np.uint64(seed & 0xFFFFFFFFFFFFFFFF) ^ (np.uint64(stream) << np.uint64(56)))
    k = splitmix64(k ^ np.asarray(a, dtype=np.uint64))
    return splitmix64(k ^ np.asarray(b, dtype=np.uint64))


def frame_limit(seed: int, env: np.ndarray | int, episode: np.ndarray | int,
                lo: int = 500, hi: int = 5000) -> np.ndarray:
    """Per-episode frame limit, uniform in [lo, hi], keyed by the global env id."""
    r = counter_rand(seed, STREAM_FRAME_LIMIT, env, episode)
    return (np.uint64(lo) + r % np.uint64(hi - lo + 1)).astype(np.uint32)


# SIMPLE_MOVEMENT of the reference action table (src/nesle/actions.py:56-64):
# NOOP, right, right+A, right+B, right+A+B, A, left as controller bit masks
# (bit 0 = A, bit 1 = B, bit 6 = left, bit 7 = right).
SIMPLE_MOVEMENT_MASKS = (0x00, 0x80, 0x81, 0x82, 0x83, 0x01, 0x40)


def uniform_actions(seed: int, env_ids: np.ndarray, step: int) -> np.ndarray:
    return (counter_rand(seed, STREAM_ACTION, env_ids, step) & np.uint64(0xFF)).astype(np.uint8)


def table_actions(seed: int, env_ids: np.ndarray, step: int,
                  table: Sequence[int] = SIMPLE_MOVEMENT_MASKS) -> np.ndarray:
    idx = counter_rand(seed, STREAM_ACTION, env_ids, step) % np.uint64(len(table))
    return np.asarray(table, dtype=np.uint8)[idx.astype(np.int64)]


# ---------------------------------------------------------------------------
# Official 6502 opcode map (standard NMOS 6502 opcode matrix).
# ---------------------------------------------------------------------------

IMP, ACC, IMM, ZP, ZPX, ZPY, ABS, ABSX, ABSY, INDX, INDY, IND, REL = range(13)
MODE_LEN = {IMP: 1, ACC: 1, IMM: 2, ZP: 2, ZPX: 2, ZPY: 2, ABS: 3, ABSX: 3, ABSY: 3,
            INDX: 2, INDY: 2, IND: 3, REL: 2}

_GROUP = {  # mnemonic -> {mode: opcode}
    "ADC": {IMM: 0x69, ZP: 0x65, ZPX: 0x75, ABS: 0x6D, ABSX: 0x7D, ABSY: 0x79, INDX: 0x61, INDY: 0x71},
    "AND": {IMM: 0x29, ZP: 0x25, ZPX: 0x35, ABS: 0x2D, ABSX: 0x3D, ABSY: 0x39, INDX: 0x21, INDY: 0x31},
    "CMP": {IMM: 0xC9, ZP: 0xC5, ZPX: 0xD5, ABS: 0xCD, ABSX: 0xDD, ABSY: 0xD9, INDX: 0xC1, INDY: 0xD1},
    "EOR": {IMM: 0x49, ZP: 0x45, ZPX: 0x55, ABS: 0x4D, ABSX: 0x5D, ABSY: 0x59, INDX: 0x41, INDY: 0x51},
    "LDA": {IMM: 0xA9, ZP: 0xA5, ZPX: 0xB5, ABS: 0xAD, ABSX: 0xBD, ABSY: 0xB9, INDX: 0xA1, INDY: 0xB1},
    "ORA": {IMM: 0x09, ZP: 0x05, ZPX: 0x15, ABS: 0x0D, ABSX: 0x1D, ABSY: 0x19, INDX: 0x01, INDY: 0x11},
    "SBC": {IMM: 0xE9, ZP: 0xE5, ZPX: 0xF5, ABS: 0xED, ABSX: 0xFD, ABSY: 0xF9, INDX: 0xE1, INDY: 0xF1},
    "STA": {ZP: 0x85, ZPX: 0x95, ABS: 0x8D, ABSX: 0x9D, ABSY: 0x99, INDX: 0x81, INDY: 0x91},
    "ASL": {ACC: 0x0A, ZP: 0x06, ZPX: 0x16, ABS: 0x0E, ABSX: 0x1E},
    "LSR": {ACC: 0x4A, ZP: 0x46, ZPX: 0x56, ABS: 0x4E, ABSX: 0x5E},
    "ROL": {ACC: 0x2A, ZP: 0x26, ZPX: 0x36, ABS: 0x2E, ABSX: 0x3E},
    "ROR": {ACC: 0x6A, ZP: 0x66, ZPX: 0x76, ABS: 0x6E, ABSX: 0x7E},
    "INC": {ZP: 0xE6, ZPX: 0xF6, ABS: 0xEE, ABSX: 0xFE},
    "DEC": {ZP: 0xC6, ZPX: 0xD6, ABS: 0xCE, ABSX: 0xDE},
    "LDX": {IMM: 0xA2, ZP: 0xA6, ZPY: 0xB6, ABS: 0xAE, ABSY: 0xBE},
    "LDY": {IMM: 0xA0, ZP: 0xA4, ZPX: 0xB4, ABS: 0xAC, ABSX: 0xBC},
    "STX": {ZP: 0x86, ZPY: 0x96, ABS: 0x8E},
    "STY": {ZP: 0x84, ZPX: 0x94, ABS: 0x8C},
    "CPX": {IMM: 0xE0, ZP: 0xE4, ABS: 0xEC},
    "CPY": {IMM: 0xC0, ZP: 0xC4, ABS: 0xCC},
    "BIT": {ZP: 0x24, ABS: 0x2C},
    "JMP": {ABS: 0x4C, IND: 0x6C},
    "JSR": {ABS: 0x20},
    "BPL": {REL: 0x10}, "BMI": {REL: 0x30}, "BVC": {REL: 0x50}, "BVS": {REL: 0x70},
    "BCC": {REL: 0x90}, "BCS": {REL: 0xB0}, "BNE": {REL: 0xD0}, "BEQ": {REL: 0xF0},
}
_IMPLIED = {
    "BRK": 0x00, "RTI": 0x40, "RTS": 0x60, "PHP": 0x08, "PLP": 0x28, "PHA": 0x48, "PLA": 0x68,
    "CLC": 0x18, "SEC": 0x38, "CLI": 0x58, "SEI": 0x78, "CLV": 0xB8, "CLD": 0xD8, "SED": 0xF8,
    "DEY": 0x88, "DEX": 0xCA, "INY": 0xC8, "INX": 0xE8, "TXA": 0x8A, "TYA": 0x98, "TXS": 0x9A,
    "TAY": 0xA8, "TAX": 0xAA, "TSX": 0xBA, "NOP": 0xEA,
}

OPCODES: dict[int, tuple[str, int]] = {}
for _mn, _modes in _GROUP.items():
    for _mode, _op in _modes.items():
        OPCODES[_op] = (_mn, _mode)
for _mn, _op in _IMPLIED.items():
    OPCODES[_op] = (_mn, IMP)
assert len(OPCODES) == 151

# Opcodes the random blocks may draw: every official opcode except BRK, RTI,
# JMP (ind) (excluded by the benchmark text) and JSR, RTS, JMP abs (they would
# send control to random addresses).
EXCLUDED = {0x00, 0x40, 0x6C, 0x20, 0x60, 0x4C}
POOL = tuple(sorted(op for op in OPCODES if op not in EXCLUDED))
assert len(POOL) == 145


def op(mn: str, mode: int = IMP) -> int:
    return _IMPLIED[mn] if mode == IMP and mn in _IMPLIED else _GROUP[mn][mode]


# ---------------------------------------------------------------------------
# Tiny assembler: a list of items, each either raw bytes or a forward branch
# to a named label, laid out from a base address.
# ---------------------------------------------------------------------------


@dataclass
class _Branch:
    opcode: int
    target: str


@dataclass
class Asm:
    base: int
    items: list = field(default_factory=list)
    labels: dict = field(default_factory=dict)

    def label(self, name: str) -> None:
        self.items.append(("label", name))

    def emit(self, mn: str, mode: int = IMP, operand: int | None = None) -> None:
        opc = op(mn, mode)
        n = MODE_LEN[mode]
        data = [opc]
        if n == 2:
            data.append(operand & 0xFF)
        elif n == 3:
            data += [operand & 0xFF, (operand >> 8) & 0xFF]
        self.items.append(bytes(data))

    def raw(self, data: bytes) -> None:
        self.items.append(bytes(data))

    def branch(self, mn: str, target: str) -> None:
        self.items.append(_Branch(op(mn, REL), target))

    def assemble(self) -> tuple[bytes, dict]:
        addr = self.base
        labels = {}
        for it in self.items:
            if isinstance(it, tuple):
                labels[it[1]] = addr
            elif isinstance(it, _Branch):
                addr += 2
            else:
                addr += len(it)
        out = bytearray()
        addr = self.base
        for it in self.items:
            if isinstance(it, tuple):
                continue
            if isinstance(it, _Branch):
                off = labels[it.target] - (addr + 2)
                if not -128 <= off <= 127:
                    raise ValueError(f"branch to {it.target} out of range ({off})")
                out += bytes([it.opcode, off & 0xFF])
                addr += 2
            else:
                out += it
                addr += len(it)
        return bytes(out), labels


# ---------------------------------------------------------------------------
# Random code blocks.
# ---------------------------------------------------------------------------


def _random_instruction(rng: np.random.Generator) -> tuple[int, int | None]:
    opc = int(rng.choice(POOL))
    mode = OPCODES[opc][1]
    if mode in (IMP, ACC):
        return opc, None
    if mode in (IMM, ZP, ZPX, ZPY, INDX, INDY):
        return opc, int(rng.integers(0, 256))
    if mode in (ABS, ABSX, ABSY):
        return opc, int(rng.integers(0x0300, 0x0800))
    if mode == REL:
        return opc, None  # target chosen at layout time
    raise AssertionError(mode)


def _guard(a: Asm, opc: int, zp: int, pointer: int) -> None:
    """Transparent pointer guard: leaves A, X, Y, P and SP unchanged."""
    mode = OPCODES[opc][1]
    store = ZPX if mode == INDX else ZP
    a.emit("PHP")
    a.emit("PHA")
    a.emit("LDA", IMM, pointer & 0xFF)
    a.emit("STA", store, zp)
    a.emit("LDA", IMM, pointer >> 8)
    a.emit("STA", store, (zp + 1) & 0xFF)
    a.emit("PLA")
    a.emit("PLP")


def _instr_bytes(opc: int, operand: int | None) -> int:
    n = MODE_LEN[OPCODES[opc][1]]
    if OPCODES[opc][1] in (INDX, INDY):
        n += 12  # guard
    return n


def emit_random_block(a: Asm, rng: np.random.Generator, name: str, count: int = 16,
                      skip_label: str | None = None, skip_index: int = 0) -> None:
    """``count`` random instructions with forward in-block branches.

    If ``skip_label`` is given, that label is placed in front of drawn
    instruction ``skip_index`` (used as a branch target by a block preamble).
    """
    instrs = [_random_instruction(rng) for _ in range(count)]
    sizes = [_instr_bytes(o, v) for o, v in instrs]
    starts = np.concatenate([[0], np.cumsum(sizes)])  # byte offset of each boundary
    for i, (opc, operand) in enumerate(instrs):
        if skip_label is not None and i == skip_index:
            a.label(skip_label)
        a.label(f"{name}_{i}")
        mode = OPCODES[opc][1]
        if mode == REL:
            here = starts[i] + 2
            choices = [j for j in range(i + 1, count + 1) if starts[j] - here <= 127]
            j = int(rng.choice(choices))
            a.branch(OPCODES[opc][0], f"{name}_{j}")
        elif mode in (INDX, INDY):
            _guard(a, opc, operand, int(rng.integers(0x0300, 0x0700)))
            a.raw(bytes([opc, operand]))
        else:
            n = MODE_LEN[mode]
            data = [opc]
            if n >= 2:
                data.append(operand & 0xFF)
            if n == 3:
                data.append(operand >> 8)
            a.raw(bytes(data))
    a.label(f"{name}_{count}")


# ---------------------------------------------------------------------------
# iNES images.
# ---------------------------------------------------------------------------

PRG_BASE = 0x8000
LOOP_HEAD = 0x8010
NMI_HANDLER = 0xF000
IRQ_STUB = 0xF800
FILL_BYTE = 0x02  # JAM: illegal, so escapes are detected


def ines_image(prg: bytes, chr_rom: bytes, flags6: int = 0x01) -> bytes:
    assert len(prg) in (16384, 32768) and len(chr_rom) == 8192
    header = b"NES\x1a" + bytes([len(prg) // 16384, 1, flags6, 0]) + bytes(8)
    return header + prg + chr_rom


def _place(prg: bytearray, addr: int, code: bytes) -> None:
    off = addr - PRG_BASE
    if any(b != FILL_BYTE for b in prg[off:off + len(code)]):
        raise ValueError(f"overlapping code at ${addr:04X}")
    prg[off:off + len(code)] = code


def _vectors(prg: bytearray, nmi: int, reset: int, irq: int) -> None:
    prg[0x7FFA:0x7FFC] = struct.pack("<H", nmi)
    prg[0x7FFC:0x7FFE] = struct.pack("<H", reset)
    prg[0x7FFE:0x8000] = struct.pack("<H", irq)


@dataclass(frozen=True)
class RomInfo:
    image: bytes
    loop_head: int
    nmi_handler: int
    code_bytes: int


def random_loop_rom(seed: int, *, blocks: int = 256, per_block: int = 16,
                    joypad_branches: bool = False) -> RomInfo:
    """Mapper-0 image: reset code, ``blocks`` random blocks, JMP to loop head, NMI handler.

    Reset writes $2000=$80 (NMI on) and $2001=$1E (background + sprites on).
    The NMI handler does OAM DMA from page $02, writes $2005 X and Y scroll from
    two seeded zero-page bytes, and returns with RTI.  It saves and restores A
    (PHA/PLA; RTI restores P), so it is transparent to the interrupted code --
    without that an NMI landing inside a pointer guard would store the
    handler's A as the pointer's high byte.

    With ``joypad_branches`` each block opens with a controller strobe, reads
    $4016 (1 + block mod 8) times so a different button bit is sampled per
    block, and branches with ``AND #1 / BNE`` over a seeded number of the
    block's random instructions.
    """
    rng = np.random.default_rng(seed)
    prg = bytearray([FILL_BYTE]) * 32768

    reset = Asm(PRG_BASE)
    reset.emit("LDA", IMM, 0x80)
    reset.emit("STA", ABS, 0x2000)
    reset.emit("LDA", IMM, 0x1E)
    reset.emit("STA", ABS, 0x2001)
    reset.emit("JMP", ABS, LOOP_HEAD)
    code, _ = reset.assemble()
    _place(prg, PRG_BASE, code)

    loop = Asm(LOOP_HEAD)
    for b in range(blocks):
        name = f"b{b}"
        if joypad_branches:
            loop.emit("LDA", IMM, 0x01)
            loop.emit("STA", ABS, 0x4016)
            loop.emit("LSR", ACC)
            loop.emit("STA", ABS, 0x4016)
            for _ in range(1 + (b & 7)):
                loop.emit("LDA", ABS, 0x4016)
            loop.emit("AND", IMM, 0x01)
            loop.branch("BNE", f"{name}_skip")
            # At most 8 skipped instructions of at most 14 bytes (guarded
            # indirect) each: always inside the +127 branch range.
            skip = int(rng.integers(1, min(per_block, 8) + 1))
            emit_random_block(loop, rng, name, per_block, f"{name}_skip", skip)
        else:
            emit_random_block(loop, rng, name, per_block)
    loop.emit("JMP", ABS, LOOP_HEAD)
    code, _ = loop.assemble()
    loop_bytes = len(code)
    if LOOP_HEAD + len(code) > NMI_HANDLER:
        raise ValueError("random loop does not fit below the NMI handler")
    _place(prg, LOOP_HEAD, code)

    zp_a, zp_b = (int(v) for v in rng.integers(0, 256, size=2))
    nmi = Asm(NMI_HANDLER)
    nmi.emit("PHA")  # the handler preserves A, so an NMI inside a pointer guard is harmless
    nmi.emit("LDA", IMM, 0x02)
    nmi.emit("STA", ABS, 0x4014)
    nmi.emit("LDA", ZP, zp_a)
    nmi.emit("STA", ABS, 0x2005)
    nmi.emit("LDA", ZP, zp_b)
    nmi.emit("STA", ABS, 0x2005)
    nmi.emit("PLA")
    nmi.emit("RTI")
    code, _ = nmi.assemble()
    _place(prg, NMI_HANDLER, code)
    _place(prg, IRQ_STUB, bytes([op("RTI")]))
    _vectors(prg, NMI_HANDLER, PRG_BASE, IRQ_STUB)

    chr_rom = rng.integers(0, 256, size=8192, dtype=np.uint8).tobytes()
    return RomInfo(ines_image(bytes(prg), chr_rom), LOOP_HEAD, NMI_HANDLER, loop_bytes)


# Zero-page cells of the sprite/scroll ROM.  Random stores may overwrite them;
# that only perturbs the RNG, the scroll or the frame handshake, never control flow.
ZP_RNG, ZP_JOY, ZP_SCROLL, ZP_NMI_FLAG, ZP_PTR = 0xF0, 0xF1, 0xF2, 0xF3, 0xF4
NT_IMAGE = 0xE000       # 2 KB nametable image (both physical nametables) copied at reset
PALETTE_IMAGE = 0xE800  # 32 palette bytes
OPAQUE_TILE = 0xFF      # all-opaque tile in both pattern tables
SPRITE0_Y = 30
SPRITE_LOOP_HEAD = 0x8100  # the reset code is longer than the 16 bytes below LOOP_HEAD


def _lcg_byte(a: Asm) -> None:
    """A = rng = rng * 5 + $1B (mod 256): full period, no fixed point."""
    a.emit("LDA", ZP, ZP_RNG)
    a.emit("ASL", ACC)
    a.emit("ASL", ACC)
    a.emit("CLC")
    a.emit("ADC", ZP, ZP_RNG)
    a.emit("CLC")
    a.emit("ADC", IMM, 0x1B)
    a.emit("STA", ZP, ZP_RNG)


def sprite_scroll_rom(seed: int, *, blocks: int = 8, per_block: int = 16) -> RomInfo:
    """Sprite- and scroll-heavy mapper-0 image (the pixel-mode configuration).

    Reset copies a 2 KB nametable image (random tiles and attributes, rows 3-4
    of both nametables the all-opaque tile $FF) and a random palette through
    $2006/$2007, then enables rendering and NMI ($2001=$1E, $2000=$80).

    Main loop, once per frame: strobe the controller and fold its 8 bits into
    an 8-bit LCG; fill sprites 1-63 of the OAM buffer at $0200 with LCG bytes
    (uniform X, Y, tile, attribute); put sprite 0 at Y=30 on tile $FF (opaque,
    over the opaque band, so the hit is certain); run ``blocks`` random blocks;
    wait for the NMI handler's flag.

    NMI handler (saves A, X, Y): OAM DMA from page $02; horizontal scroll +=
    (joypad & 3) + 1 written to $2005 for the next frame; wait for the
    sprite-0 flag to clear (pre-render line) and then to set (line 30); write
    $2005 again with an LCG byte (the mid-frame split); set the flag.
    """
    rng = np.random.default_rng(seed)
    prg = bytearray([FILL_BYTE]) * 32768

    reset = Asm(PRG_BASE)
    reset.emit("SEI")
    reset.emit("CLD")
    reset.emit("LDX", IMM, 0xFF)
    reset.emit("TXS")
    reset.emit("LDA", IMM, 0x00)
    reset.emit("STA", ABS, 0x2000)
    reset.emit("STA", ABS, 0x2001)
    reset.emit("LDA", ABS, 0x2002)          # reset the $2005/$2006 latch
    reset.emit("LDA", IMM, 0x3F)
    reset.emit("STA", ABS, 0x2006)
    reset.emit("LDA", IMM, 0x00)
    reset.emit("STA", ABS, 0x2006)
    reset.emit("LDX", IMM, 0x00)
    reset.label("pal")
    reset.emit("LDA", ABSX, PALETTE_IMAGE)
    reset.emit("STA", ABS, 0x2007)
    reset.emit("INX")
    reset.emit("CPX", IMM, 32)
    reset.branch("BNE", "pal")
    reset.emit("LDA", IMM, 0x20)
    reset.emit("STA", ABS, 0x2006)
    reset.emit("LDA", IMM, 0x00)
    reset.emit("STA", ABS, 0x2006)
    reset.emit("LDA", IMM, NT_IMAGE & 0xFF)
    reset.emit("STA", ZP, ZP_PTR)
    reset.emit("LDA", IMM, NT_IMAGE >> 8)
    reset.emit("STA", ZP, ZP_PTR + 1)
    reset.emit("LDX", IMM, 8)               # 8 pages of 256 bytes
    reset.emit("LDY", IMM, 0)
    reset.label("nt")
    reset.emit("LDA", INDY, ZP_PTR)
    reset.emit("STA", ABS, 0x2007)
    reset.emit("INY")
    reset.branch("BNE", "nt")
    reset.emit("INC", ZP, ZP_PTR + 1)
    reset.emit("DEX")
    reset.branch("BNE", "nt")
    reset.emit("LDA", IMM, int(rng.integers(1, 256)))
    reset.emit("STA", ZP, ZP_RNG)
    reset.emit("LDA", IMM, 0x00)
    reset.emit("STA", ZP, ZP_SCROLL)
    reset.emit("STA", ZP, ZP_NMI_FLAG)
    reset.emit("STA", ABS, 0x2005)
    reset.emit("STA", ABS, 0x2005)
    # Rendering first: enabling NMI inside vblank raises the NMI at once, and
    # the handler's sprite-0 wait needs rendering on.
    reset.emit("LDA", IMM, 0x1E)
    reset.emit("STA", ABS, 0x2001)
    reset.emit("LDA", IMM, 0x80)
    reset.emit("STA", ABS, 0x2000)
    reset.emit("JMP", ABS, SPRITE_LOOP_HEAD)
    code, _ = reset.assemble()
    if PRG_BASE + len(code) > SPRITE_LOOP_HEAD:
        raise ValueError("reset code overlaps the main loop")
    _place(prg, PRG_BASE, code)

    loop = Asm(SPRITE_LOOP_HEAD)
    # controller -> joy, rng ^= joy
    loop.emit("LDA", IMM, 0x01)
    loop.emit("STA", ABS, 0x4016)
    loop.emit("LSR", ACC)
    loop.emit("STA", ABS, 0x4016)
    loop.emit("LDX", IMM, 8)
    loop.label("joy")
    loop.emit("LDA", ABS, 0x4016)
    loop.emit("LSR", ACC)
    loop.emit("ROL", ZP, ZP_JOY)
    loop.emit("DEX")
    loop.branch("BNE", "joy")
    loop.emit("LDA", ZP, ZP_JOY)
    loop.emit("EOR", ZP, ZP_RNG)
    loop.emit("STA", ZP, ZP_RNG)
    # sprites 1..63
    loop.emit("LDX", IMM, 4)
    loop.label("fill")
    _lcg_byte(loop)
    loop.emit("STA", ABSX, 0x0200)
    loop.emit("INX")
    loop.branch("BNE", "fill")
    # sprite 0: Y=30, opaque tile, front priority, X in [$40, $BF]
    loop.emit("LDA", IMM, SPRITE0_Y)
    loop.emit("STA", ABS, 0x0200)
    loop.emit("LDA", IMM, OPAQUE_TILE)
    loop.emit("STA", ABS, 0x0201)
    loop.emit("LDA", IMM, 0x00)
    loop.emit("STA", ABS, 0x0202)
    _lcg_byte(loop)
    loop.emit("AND", IMM, 0x7F)
    loop.emit("CLC")
    loop.emit("ADC", IMM, 0x40)
    loop.emit("STA", ABS, 0x0203)
    for b in range(blocks):
        emit_random_block(loop, rng, f"s{b}", per_block)
    loop.label("wait")
    loop.emit("LDA", ZP, ZP_NMI_FLAG)
    loop.branch("BEQ", "wait")
    loop.emit("LDA", IMM, 0x00)
    loop.emit("STA", ZP, ZP_NMI_FLAG)
    loop.emit("JMP", ABS, SPRITE_LOOP_HEAD)
    code, _ = loop.assemble()
    loop_bytes = len(code)
    if SPRITE_LOOP_HEAD + len(code) > NT_IMAGE:
        raise ValueError("main loop does not fit below the nametable image")
    _place(prg, SPRITE_LOOP_HEAD, code)

    nt = rng.integers(0, 256, size=2048, dtype=np.uint8)
    for base in (0, 1024):  # both physical nametables: rows 3-4 opaque band
        nt[base + 3 * 32: base + 5 * 32] = OPAQUE_TILE
    _place(prg, NT_IMAGE, nt.tobytes())
    pal = (rng.integers(0, 64, size=32, dtype=np.uint8)).tobytes()
    _place(prg, PALETTE_IMAGE, pal)

    nmi = Asm(NMI_HANDLER)
    nmi.emit("PHA")
    nmi.emit("TXA")
    nmi.emit("PHA")
    nmi.emit("TYA")
    nmi.emit("PHA")
    nmi.emit("LDA", IMM, 0x02)
    nmi.emit("STA", ABS, 0x4014)
    nmi.emit("LDA", ZP, ZP_JOY)
    nmi.emit("AND", IMM, 0x03)
    nmi.emit("SEC")
    nmi.emit("ADC", ZP, ZP_SCROLL)
    nmi.emit("STA", ZP, ZP_SCROLL)
    nmi.emit("STA", ABS, 0x2005)
    nmi.emit("LDA", IMM, 0x00)
    nmi.emit("STA", ABS, 0x2005)
    nmi.label("clear")
    nmi.emit("BIT", ABS, 0x2002)
    nmi.branch("BVS", "clear")
    nmi.label("hit")
    nmi.emit("BIT", ABS, 0x2002)
    nmi.branch("BVC", "hit")
    _lcg_byte(nmi)
    nmi.emit("STA", ABS, 0x2005)
    nmi.emit("LDA", IMM, 0x00)
    nmi.emit("STA", ABS, 0x2005)
    nmi.emit("LDA", IMM, 0x01)
    nmi.emit("STA", ZP, ZP_NMI_FLAG)
    nmi.emit("PLA")
    nmi.emit("TAY")
    nmi.emit("PLA")
    nmi.emit("TAX")
    nmi.emit("PLA")
    nmi.emit("RTI")
    code, _ = nmi.assemble()
    _place(prg, NMI_HANDLER, code)
    _place(prg, IRQ_STUB, bytes([op("RTI")]))
    _vectors(prg, NMI_HANDLER, PRG_BASE, IRQ_STUB)

    chr_rom = bytearray(rng.integers(0, 256, size=8192, dtype=np.uint8).tobytes())
    for table in (0x0000, 0x1000):
        off = table + OPAQUE_TILE * 16
        chr_rom[off:off + 16] = b"\xff" * 16
    return RomInfo(ines_image(bytes(prg), bytes(chr_rom)), SPRITE_LOOP_HEAD, NMI_HANDLER, loop_bytes)


def random_snapshot(seed: int, pc: int, *, nmi_and_rendering: bool = False) -> Snapshot:
    """Random 2 KB RAM and A/X/Y/SP; P = $24 plus random N/V/Z/C; PC at ``pc``.

    PPU registers are at power-on values, or with ``nmi_and_rendering`` as if
    the reset code had run ($2000=$80, $2001=$1E).
    """
    rng = np.random.default_rng(seed)
    a, x, y, sp = (int(v) for v in rng.integers(0, 256, size=4))
    p = 0x24 | (int(rng.integers(0, 256)) & 0xC3)
    ram = rng.integers(0, 256, size=2048, dtype=np.uint8).tobytes()
    s = Snapshot(pc=pc, a=a, x=x, y=y, sp=sp, p=p, cpu_ram=ram)
    if nmi_and_rendering:
        s.ppu_ctrl, s.ppu_mask = 0x80, 0x1E
    return s


# ---------------------------------------------------------------------------
# Benchmark configurations (BASELINE.json "configs").
# ---------------------------------------------------------------------------

DONE_SMB = 0          # reference predicate: SMB flag/death/game over
DONE_RAM_EQ = 1       # RAM[addr] == value   (config 2)
DONE_FRAME_LIMIT = 2  # frames since reset >= per-episode U[lo, hi]  (config 4)


@dataclass
class Workload:
    name: str
    rom: RomInfo
    snapshots: list[bytes]
    env_to_level: Callable[[np.ndarray], np.ndarray] | None
    actions: Callable[[np.ndarray, int], np.ndarray]
    done_mode: int
    done_args: tuple[int, int]
    frameskip: int = 4
    seed: int = 0


def config1(seed: int = 1) -> Workload:
    """64 envs x 600 frames from power-on; random joypad bytes (the ROM ignores them)."""
    rom = random_loop_rom(seed)
    return Workload("config1-boot", rom, [], None,
                    lambda env, step: uniform_actions(seed, env, step), DONE_SMB, (0, 0), 4, seed)


def config2(seed: int = 2) -> Workload:
    """RAM mode, 7-mask action table, 1 synthetic snapshot, done when RAM[$FF] == $FF."""
    rom = random_loop_rom(seed)
    snap = write_fcs(random_snapshot(seed + 1000, rom.loop_head))
    return Workload("config2-ram", rom, [snap], None,
                    lambda env, step: table_actions(seed, env, step), DONE_RAM_EQ, (0x00FF, 0xFF),
                    4, seed)


def config4(seed: int = 4) -> Workload:
    """Divergent RAM mode: joypad-driven branches in every block, 8 snapshots,
    env i starts from snapshot i mod 8, done at a per-episode frame limit in [500, 5000]."""
    rom = random_loop_rom(seed, joypad_branches=True)
    snaps = [write_fcs(random_snapshot(seed * 100 + k, rom.loop_head, nmi_and_rendering=True))
             for k in range(8)]
    return Workload("config4-divergent", rom, snaps,
                    lambda env: (np.asarray(env) % 8).astype(np.uint8),
                    lambda env, step: uniform_actions(seed, env, step),
                    DONE_FRAME_LIMIT, (500, 5000), 4, seed)


def config3(seed: int = 3) -> Workload:
    """Pixel mode: sprite/scroll ROM from power-on, uniform joypad bytes (they drive
    the scroll and the sprite RNG), done at a per-episode frame limit in [500, 5000];
    the observation is the 84x84 gray downsample of the palette-index frame."""
    rom = sprite_scroll_rom(seed)
    return Workload("config3-pixel", rom, [], None,
                    lambda env, step: uniform_actions(seed, env, step),
                    DONE_FRAME_LIMIT, (500, 5000), 4, seed)


CONFIGS = {"config1": config1, "config2": config2, "config3": config3, "config4": config4}
