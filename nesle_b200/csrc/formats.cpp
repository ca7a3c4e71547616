// formats.cpp -- iNES and FCS parsing for the B200 batch (host side).
#include "formats.h"

#include <string.h>

namespace nesle {

bool parse_ines(const uint8_t* b, size_t len, Cartridge& out, std::string& err) {
    // cpp/src/rom.cpp:65-121
    if (len < 16) { err = "iNES data is shorter than the 16-byte header"; return false; }
    if (b[0] != 'N' || b[1] != 'E' || b[2] != 'S' || b[3] != 0x1A) {
        err = "iNES header magic must be NES<EOF>";
        return false;
    }
    const uint8_t prg_banks = b[4], chr_banks = b[5], f6 = b[6], f7 = b[7];
    const bool nes2 = (f7 & 0x0C) == 0x08;
    if (nes2 && b[9] != 0) { err = "NES 2.0 extended PRG/CHR ROM sizes are not supported yet"; return false; }
    uint16_t mapper = static_cast<uint16_t>((f6 >> 4) | (f7 & 0xF0));
    if (nes2) mapper = static_cast<uint16_t>(mapper | ((b[8] & 0x0F) << 8));
    size_t off = 16 + ((f6 & 0x04) ? 512 : 0);
    const size_t prg = static_cast<size_t>(prg_banks) * 16384, chr = static_cast<size_t>(chr_banks) * 8192;
    if (len < off + prg + chr) { err = "iNES data is truncated for declared PRG/CHR sizes"; return false; }
    // cuda_module.cu:381-398 accepts NROM only (mapper 0, PRG 16/32 KB).  This
    // core also runs the two discrete-logic boards (no counterpart in the
    // reference): UxROM (mapper 2: 2-16 PRG banks of 16 KB, a power of two,
    // switchable at $8000, the last one fixed at $C000) and CNROM (mapper 3:
    // 16/32 KB PRG, 1-4 CHR banks of 8 KB, a power of two).
    const auto pow2 = [](unsigned n) { return n != 0 && (n & (n - 1)) == 0; };
    const bool nrom = mapper == 0 && (prg_banks == 1 || prg_banks == 2);
    const bool uxrom = mapper == 2 && prg_banks >= 2 && prg_banks <= 16 && pow2(prg_banks) && chr_banks <= 1;
    const bool cnrom = mapper == 3 && (prg_banks == 1 || prg_banks == 2) && chr_banks <= 4 && pow2(chr_banks);
    if (!nrom && !uxrom && !cnrom) {
        err = "supported cartridges: mapper 0/NROM (16/32 KB PRG), 2/UxROM (32-256 KB PRG, power-of-two banks, "
              "8 KB CHR) and 3/CNROM (16/32 KB PRG, 8-32 KB CHR, power-of-two banks)";
        return false;
    }
    if (f6 & 0x08) {
        // The reference batch sizes nametable RAM at 2 KB per env but indexes
        // four-screen layouts up to 4 KB; this build rejects the layout.
        err = "four-screen nametable layouts are not supported by the batched core";
        return false;
    }
    out.prg.assign(b + off, b + off + prg);
    out.chr.assign(b + off + prg, b + off + prg + chr);
    out.mapper = mapper;
    out.prg_banks = prg_banks;
    out.chr_banks = chr_banks;
    out.horizontal = (f6 & 0x01) == 0;
    out.four_screen = false;
    return true;
}

namespace {

uint32_t le32(const uint8_t* p) {
    return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8) | (static_cast<uint32_t>(p[2]) << 16) |
           (static_cast<uint32_t>(p[3]) << 24);
}

template <size_t N>
bool fixed(uint8_t (&dst)[N], const uint8_t* src, uint32_t n, const char* label, std::string& err) {
    if (n != N) {
        err = std::string("FCS: ") + label + " expected " + std::to_string(N) + " bytes, got " + std::to_string(n);
        return false;
    }
    memcpy(dst, src, N);
    return true;
}

// fcs.hpp:91-160
bool apply(FcsState& s, int tag, const std::string& name, const uint8_t* p, uint32_t n, std::string& err) {
    if (tag == 1) {
        if (name == "PC") {
            if (n != 2) { err = "FCS: CPU.PC must be 2 bytes"; return false; }
            s.pc = static_cast<uint16_t>(p[0] | (p[1] << 8));
        } else if (name == "A" && n == 1) s.a = p[0];
        else if (name == "X" && n == 1) s.x = p[0];
        else if (name == "Y" && n == 1) s.y = p[0];
        else if (name == "S" && n == 1) s.sp = p[0];
        else if (name == "P" && n == 1) s.p = p[0];
        else if (name == "RAM") return fixed(s.cpu_ram, p, n, "CPU.RAM", err);
    } else if (tag == 3) {
        if (name == "NTAR") return fixed(s.nametable_ram, p, n, "PPU.NTAR", err);
        if (name == "PRAM") return fixed(s.palette_ram, p, n, "PPU.PRAM", err);
        if (name == "SPRA") return fixed(s.oam, p, n, "PPU.SPRA", err);
        if (name == "PPUR") {
            if (n < 3) { err = "FCS: PPU.PPUR too short"; return false; }
            s.ppu_ctrl = p[0]; s.ppu_mask = p[1]; s.ppu_status = p[2];
        } else if (name == "PSPL" && n == 1) s.ppu_oam_addr = p[0];
        else if (name == "XOFF" && n == 1) s.ppu_x = p[0] & 7;
        else if (name == "VTGL" && n == 1) s.ppu_w = p[0] & 1;
        else if (name == "RADD" && n == 2) s.ppu_v = static_cast<uint16_t>(p[0] | (p[1] << 8));
        else if (name == "TADD" && n == 2) s.ppu_t = static_cast<uint16_t>(p[0] | (p[1] << 8));
        else if (name == "VBUF" && n == 1) s.ppu_read_buffer = p[0];
        else if (name == "PGEN" && n == 1) s.ppu_open_bus = p[0];
    } else if (tag == 16) {
        if (name == "WRAM") return fixed(s.prg_ram, p, n, "CART.WRAM", err);
    }
    return true;
}

}  // namespace

bool parse_fcs(const uint8_t* d, size_t len, FcsState& s, std::string& err) {
    // fcs.hpp:187-226
    s = FcsState{};
    if (len < 16) { err = "FCS: header too short"; return false; }
    if (d[0] != 'F' || d[1] != 'C' || d[2] != 'S' || d[3] != 0xFF) {
        err = "FCS: bad magic (expected 'FCS\\xff')";
        return false;
    }
    size_t off = 16;
    while (off + 5 <= len) {
        const int tag = d[off];
        const uint32_t size = le32(d + off + 1);
        off += 5;
        if (off + size > len) { err = "FCS: top-level chunk extends past file"; return false; }
        if (tag == 1 || tag == 3 || tag == 16) {
            size_t so = 0;
            while (so + 8 <= size) {
                std::string name(reinterpret_cast<const char*>(d + off + so), 4);
                while (!name.empty() && name.back() == '\0') name.pop_back();
                const uint32_t ss = le32(d + off + so + 4);
                so += 8;
                if (so + ss > size) { err = "FCS: sub-chunk \"" + name + "\" extends past parent payload"; return false; }
                if (!apply(s, tag, name, d + off + so, ss, err)) return false;
                so += ss;
            }
            if (so != size) { err = "FCS: trailing bytes in sub-chunk stream"; return false; }
        }
        off += size;
    }
    if (off != len) { err = "FCS: trailing bytes after last top-level chunk"; return false; }
    return true;
}

}  // namespace nesle
