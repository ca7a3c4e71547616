// formats.h -- iNES cartridge images and FCEUX FCS save states (host side).
#pragma once
#include <stddef.h>
#include <stdint.h>

#include <string>
#include <vector>

namespace nesle {

struct Cartridge {
    std::vector<uint8_t> prg;  // 16 or 32 KB (NROM, CNROM) or 32-256 KB (UxROM) as stored in the image
    std::vector<uint8_t> chr;  // 0 or N * 8 KB
    uint16_t mapper = 0;
    uint8_t prg_banks = 0, chr_banks = 0;
    bool horizontal = false;   // nametable arrangement (flags6 bit 0 clear)
    bool four_screen = false;
};

// Parses an iNES/NES 2.0 image and applies the reference binding's checks for
// the console path (cpp/src/rom.cpp:65-121, cpp/bindings/cuda_module.cu:381-398),
// widened to the UxROM and CNROM boards.  Returns false with `err` set on failure.
bool parse_ines(const uint8_t* data, size_t len, Cartridge& out, std::string& err);

// One FCS save state (cpp/include/nesle/fcs.hpp:19-45).
struct FcsState {
    uint16_t pc = 0;
    uint8_t a = 0, x = 0, y = 0, sp = 0xFD, p = 0x24;
    uint64_t cycles = 0;
    uint8_t ppu_ctrl = 0, ppu_mask = 0, ppu_status = 0, ppu_oam_addr = 0, ppu_open_bus = 0,
            ppu_read_buffer = 0, ppu_x = 0, ppu_w = 0;
    uint16_t ppu_v = 0, ppu_t = 0;
    uint8_t cpu_ram[2048] = {};
    uint8_t prg_ram[8192] = {};
    uint8_t nametable_ram[2048] = {};
    uint8_t palette_ram[32] = {};
    uint8_t oam[256] = {};
};

// Parses an uncompressed FCS file (fcs.hpp:187-226).  Returns false with
// `err` set on malformed input.
bool parse_fcs(const uint8_t* data, size_t len, FcsState& out, std::string& err);

}  // namespace nesle
