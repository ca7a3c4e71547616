"""FCEUX FCS save states: the snapshot format of the reference binding.

``write_fcs`` serialises a console state; the layout is the one the
reference parser reads (cpp/include/nesle/fcs.hpp:187-226): a 16-byte header
"FCS\xff", then chunks tag:u8 size:u32le payload, each payload a run of
sub-chunks name[4] size:u32le data.  The CPU chunk (tag 1) carries PC, A, X,
Y, S, P and the 2 KB RAM; the PPU chunk (tag 3) the nametables, palette, OAM
and registers; the cartridge chunk (tag 16) the 8 KB PRG-RAM.  Parsing is
``nesle_parse_fcs`` / ``parse_fcs_state`` in the C library.
"""
from __future__ import annotations

import struct
from dataclasses import dataclass


@dataclass
class Snapshot:
    pc: int = 0
    a: int = 0
    x: int = 0
    y: int = 0
    sp: int = 0xFD
    p: int = 0x24
    cpu_ram: bytes = bytes(2048)
    prg_ram: bytes = bytes(8192)
    ppu_ctrl: int = 0
    ppu_mask: int = 0
    ppu_status: int = 0
    ppu_oam_addr: int = 0
    ppu_open_bus: int = 0
    ppu_read_buffer: int = 0
    ppu_x: int = 0
    ppu_w: int = 0
    ppu_v: int = 0
    ppu_t: int = 0
    nametable_ram: bytes = bytes(2048)
    palette_ram: bytes = bytes(32)
    oam: bytes = bytes(256)


def _sub(name: str, payload: bytes) -> bytes:
    return name.encode().ljust(4, b"\0") + struct.pack("<I", len(payload)) + payload


def write_fcs(s: Snapshot) -> bytes:
    cpu = b"".join([
        _sub("PC", struct.pack("<H", s.pc)), _sub("A", bytes([s.a])), _sub("X", bytes([s.x])),
        _sub("Y", bytes([s.y])), _sub("S", bytes([s.sp])), _sub("P", bytes([s.p])),
        _sub("DB", b"\0"), _sub("RAM", s.cpu_ram),
    ])
    ppu = b"".join([
        _sub("NTAR", s.nametable_ram), _sub("PRAM", s.palette_ram), _sub("SPRA", s.oam),
        _sub("PPUR", bytes([s.ppu_ctrl, s.ppu_mask, s.ppu_status, 0])),
        _sub("PSPL", bytes([s.ppu_oam_addr])), _sub("XOFF", bytes([s.ppu_x])),
        _sub("VTGL", bytes([s.ppu_w])), _sub("RADD", struct.pack("<H", s.ppu_v)),
        _sub("TADD", struct.pack("<H", s.ppu_t)), _sub("VBUF", bytes([s.ppu_read_buffer])),
        _sub("PGEN", bytes([s.ppu_open_bus])),
    ])
    cart = _sub("WRAM", s.prg_ram)
    header = b"FCS\xff" + bytes(12)

    def chunk(tag: int, payload: bytes) -> bytes:
        return bytes([tag]) + struct.pack("<I", len(payload)) + payload

    return header + chunk(1, cpu) + chunk(3, ppu) + chunk(16, cart)
