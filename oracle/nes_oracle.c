/*
 * nes_oracle.c -- CPU checker for the batched NES env-step path.
 *
 * TEST INFRASTRUCTURE ONLY (see nes_oracle.h).  A deliberately plain,
 * per-opcode-switch restatement of what the reference CUDA kernel computes, so
 * that it shares no code or structure with the product kernel it checks.
 * Every function names the reference lines (paths inside hbofz/NeSLE) whose
 * behaviour it restates.  Extensions that the reference does not have (the
 * RAM-byte and frame-limit done predicates, the illegal-opcode status word,
 * the palette-index and 84x84 grey outputs) are marked "EXTENSION".
 */
#include "nes_oracle.h"

#include <stdlib.h>
#include <string.h>

enum { IMP, ACC, IMM, ZP, ZPX, ZPY, ABS, ABSX, ABSY, INDX, INDY, IND, REL };

enum {
    I_ILL, I_LDA, I_LDX, I_LDY, I_STA, I_STX, I_STY, I_TAX, I_TAY, I_TXA, I_TYA, I_TSX, I_TXS,
    I_PHA, I_PHP, I_PLA, I_PLP, I_ORA, I_AND, I_EOR, I_ADC, I_SBC, I_CMP, I_CPX, I_CPY, I_BIT,
    I_INC, I_DEC, I_INX, I_INY, I_DEX, I_DEY, I_ASL, I_LSR, I_ROL, I_ROR, I_JMP, I_JSR, I_RTS,
    I_RTI, I_BRK, I_BRANCH, I_CLC, I_SEC, I_CLI, I_SEI, I_CLV, I_CLD, I_SED, I_NOP
};

#define F_PAGE 1
#define F_RMW 2
#define F_STORE 4
#define F_ILLEGAL 8

typedef struct { uint8_t ins, mode, cycles, flags; } decode_t;
static decode_t g_decode[256];

/* Official opcode matrix with base cycles; restates the 151 entries of
 * cpp/include/nesle/cpu.hpp:200-350 (pinned entry-by-entry against the
 * compiled reference table by tests/test_oracle_pin.py). */
static void build_decode(void) {
    static int built = 0;
    if (built) return;
    for (int i = 0; i < 256; ++i) g_decode[i] = (decode_t){I_ILL, IMP, 0, F_ILLEGAL};
#define D(opc, ins, mode, cyc, fl) g_decode[opc] = (decode_t){ins, mode, cyc, fl}
    /* group-1 ALU ops: imm zp zpx abs absx absy indx indy */
#define G1(ins, b)                                                                  \
    D(b + 0x09, ins, IMM, 2, 0); D(b + 0x05, ins, ZP, 3, 0); D(b + 0x15, ins, ZPX, 4, 0); \
    D(b + 0x0D, ins, ABS, 4, 0); D(b + 0x1D, ins, ABSX, 4, F_PAGE);                    \
    D(b + 0x19, ins, ABSY, 4, F_PAGE); D(b + 0x01, ins, INDX, 6, 0);                   \
    D(b + 0x11, ins, INDY, 5, F_PAGE)
    G1(I_ORA, 0x00); G1(I_AND, 0x20); G1(I_EOR, 0x40); G1(I_ADC, 0x60);
    G1(I_LDA, 0xA0); G1(I_CMP, 0xC0); G1(I_SBC, 0xE0);
#undef G1
    D(0x85, I_STA, ZP, 3, F_STORE); D(0x95, I_STA, ZPX, 4, F_STORE); D(0x8D, I_STA, ABS, 4, F_STORE);
    D(0x9D, I_STA, ABSX, 5, F_STORE); D(0x99, I_STA, ABSY, 5, F_STORE);
    D(0x81, I_STA, INDX, 6, F_STORE); D(0x91, I_STA, INDY, 6, F_STORE);
    /* shifts and inc/dec: acc/zp/zpx/abs/absx */
#define SH(ins, b)                                                                      \
    D(b + 0x0A, ins, ACC, 2, 0); D(b + 0x06, ins, ZP, 5, F_RMW); D(b + 0x16, ins, ZPX, 6, F_RMW); \
    D(b + 0x0E, ins, ABS, 6, F_RMW); D(b + 0x1E, ins, ABSX, 7, F_RMW)
    SH(I_ASL, 0x00); SH(I_ROL, 0x20); SH(I_LSR, 0x40); SH(I_ROR, 0x60);
#undef SH
    D(0xE6, I_INC, ZP, 5, F_RMW); D(0xF6, I_INC, ZPX, 6, F_RMW); D(0xEE, I_INC, ABS, 6, F_RMW);
    D(0xFE, I_INC, ABSX, 7, F_RMW);
    D(0xC6, I_DEC, ZP, 5, F_RMW); D(0xD6, I_DEC, ZPX, 6, F_RMW); D(0xCE, I_DEC, ABS, 6, F_RMW);
    D(0xDE, I_DEC, ABSX, 7, F_RMW);
    D(0xA2, I_LDX, IMM, 2, 0); D(0xA6, I_LDX, ZP, 3, 0); D(0xB6, I_LDX, ZPY, 4, 0);
    D(0xAE, I_LDX, ABS, 4, 0); D(0xBE, I_LDX, ABSY, 4, F_PAGE);
    D(0xA0, I_LDY, IMM, 2, 0); D(0xA4, I_LDY, ZP, 3, 0); D(0xB4, I_LDY, ZPX, 4, 0);
    D(0xAC, I_LDY, ABS, 4, 0); D(0xBC, I_LDY, ABSX, 4, F_PAGE);
    D(0x86, I_STX, ZP, 3, F_STORE); D(0x96, I_STX, ZPY, 4, F_STORE); D(0x8E, I_STX, ABS, 4, F_STORE);
    D(0x84, I_STY, ZP, 3, F_STORE); D(0x94, I_STY, ZPX, 4, F_STORE); D(0x8C, I_STY, ABS, 4, F_STORE);
    D(0xE0, I_CPX, IMM, 2, 0); D(0xE4, I_CPX, ZP, 3, 0); D(0xEC, I_CPX, ABS, 4, 0);
    D(0xC0, I_CPY, IMM, 2, 0); D(0xC4, I_CPY, ZP, 3, 0); D(0xCC, I_CPY, ABS, 4, 0);
    D(0x24, I_BIT, ZP, 3, 0); D(0x2C, I_BIT, ABS, 4, 0);
    D(0x4C, I_JMP, ABS, 3, 0); D(0x6C, I_JMP, IND, 5, 0); D(0x20, I_JSR, ABS, 6, 0);
    D(0x60, I_RTS, IMP, 6, 0); D(0x40, I_RTI, IMP, 6, 0); D(0x00, I_BRK, IMP, 7, 0);
    for (int b = 0x10; b <= 0xF0; b += 0x20) D(b, I_BRANCH, REL, 2, 0);
    D(0x08, I_PHP, IMP, 3, 0); D(0x28, I_PLP, IMP, 4, 0); D(0x48, I_PHA, IMP, 3, 0);
    D(0x68, I_PLA, IMP, 4, 0);
    D(0x18, I_CLC, IMP, 2, 0); D(0x38, I_SEC, IMP, 2, 0); D(0x58, I_CLI, IMP, 2, 0);
    D(0x78, I_SEI, IMP, 2, 0); D(0xB8, I_CLV, IMP, 2, 0); D(0xD8, I_CLD, IMP, 2, 0);
    D(0xF8, I_SED, IMP, 2, 0);
    D(0x88, I_DEY, IMP, 2, 0); D(0xCA, I_DEX, IMP, 2, 0); D(0xC8, I_INY, IMP, 2, 0);
    D(0xE8, I_INX, IMP, 2, 0); D(0x8A, I_TXA, IMP, 2, 0); D(0x98, I_TYA, IMP, 2, 0);
    D(0x9A, I_TXS, IMP, 2, 0); D(0xA8, I_TAY, IMP, 2, 0); D(0xAA, I_TAX, IMP, 2, 0);
    D(0xBA, I_TSX, IMP, 2, 0); D(0xEA, I_NOP, IMP, 2, 0);
#undef D
    built = 1;
}

void oracle_decode_table(uint8_t *mode, uint8_t *base_cycles, uint8_t *flags) {
    build_decode();
    for (int i = 0; i < 256; ++i) {
        mode[i] = g_decode[i].mode;
        base_cycles[i] = g_decode[i].cycles;
        flags[i] = g_decode[i].flags;
    }
}

/* ------------------------------------------------------------------------ */
/* Per-env state: every field of the reference BatchBuffers SoA
 * (cpp/include/nesle/cuda/state.cuh:103-203) plus this build's extensions.   */
/* ------------------------------------------------------------------------ */
typedef struct {
    uint16_t pc;
    uint8_t a, x, y, sp, p;
    uint64_t cycles;
    uint8_t cpu_nmi_pending, irq_pending;
    uint8_t ctrl_shift, ctrl_count, ctrl_strobe;
    uint32_t pending_dma;
    uint8_t ppu_ctrl, ppu_mask, ppu_status, oam_addr, nmi_pending;
    uint32_t frame_dot;
    uint64_t frame;
    uint16_t v, t;
    uint8_t fine_x, w, open_bus, read_buffer, scroll_x, scroll_y;
    uint8_t lat_sx, lat_sy, lat_ctrl;
    uint8_t snap_sx_start, snap_sy_start, snap_ctrl_start;
    uint8_t snap_sx_end, snap_sy_end, snap_ctrl_end, snap_mask;
    int32_t prev_x, prev_time;
    float reward, last_reward;
    uint8_t done, last_done, action;
    uint32_t episode, status;               /* EXTENSION */
    uint64_t stat_instructions;
    uint32_t stat_frames, stat_budget_hits;
    uint8_t ram[2048], prg_ram[8192], nt[2048], pal[32], oam[256];
    uint8_t snap_oam[256], snap_nt[2048], snap_pal[32];
    uint8_t prg_bank, chr_bank, snap_chr_bank; /* EXTENSION: UxROM / CNROM bank registers */
    uint64_t ram_touch; /* MEASUREMENT: 32-byte RAM sectors read or written during the last env-step */
} env_t;

#define TOUCH(e, a) ((e)->ram_touch |= 1ull << (((a) & 0x7FFu) >> 5))

typedef struct {
    uint16_t pc;
    uint8_t a, x, y, sp, p;
    uint64_t cycles;
    uint8_t ctrl, mask, status, oam_addr, open_bus, read_buffer, fine_x, w;
    uint16_t v, t;
    uint8_t ram[2048], prg_ram[8192], nt[2048], pal[32], oam[256];
} snap_t;

struct nes_oracle {
    uint32_t n, frameskip;
    uint64_t max_instr;
    uint8_t *prg;
    uint32_t prg_size;
    uint8_t *chr;
    uint32_t chr_size;
    uint8_t horizontal; /* nametable arrangement: 0 vertical, 1 horizontal */
    uint32_t mapper, prg_banks, chr_banks; /* EXTENSION: 0 NROM, 2 UxROM, 3 CNROM */
    uint8_t *prg_rom;                      /* the whole PRG ROM (UxROM banks) */
    snap_t *snaps;
    uint32_t nsnap;
    uint8_t *env_to_level;
    uint32_t done_mode, done_a, done_b;
    uint64_t seed;
    uint32_t env_offset;
    env_t *env;
    uint32_t trace_env, trace_cap, trace_n;
    uint8_t *trace_buf;
    uint64_t *prof_opcode, *prof_pc; /* step_profile histograms (256, 65536) or NULL */
};

static __thread char g_err[256];
const char *oracle_last_error(void) { return g_err; }

/* ------------------------------------------------------------------------ */
/* Counter RNG: SplitMix64 finaliser (Steele, Lea, Flood, OOPSLA 2014).       */
/* ------------------------------------------------------------------------ */
static uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
uint64_t oracle_counter_rand(uint64_t seed, uint32_t stream, uint64_t a, uint64_t b) {
    uint64_t k = splitmix64(seed ^ ((uint64_t)stream << 56));
    k = splitmix64(k ^ a);
    return splitmix64(k ^ b);
}
static uint32_t frame_limit(const nes_oracle *o, uint32_t env, uint32_t episode) {
    uint64_t r = oracle_counter_rand(o->seed, 2, (uint64_t)o->env_offset + env, episode);
    return o->done_a + (uint32_t)(r % (uint64_t)(o->done_b - o->done_a + 1));
}

/* ------------------------------------------------------------------------ */
/* iNES and FCS parsing.                                                      */
/* ------------------------------------------------------------------------ */

/* cpp/src/rom.cpp:65-121 plus the NROM checks of cuda_module.cu:381-398. */
static int parse_ines(nes_oracle *o, const uint8_t *b, size_t len) {
    if (len < 16) { strcpy(g_err, "iNES data is shorter than the 16-byte header"); return -1; }
    if (b[0] != 'N' || b[1] != 'E' || b[2] != 'S' || b[3] != 0x1A) {
        strcpy(g_err, "iNES header magic must be NES<EOF>"); return -1;
    }
    uint8_t prg_banks = b[4], chr_banks = b[5], f6 = b[6], f7 = b[7];
    int nes2 = (f7 & 0x0C) == 0x08;
    if (nes2 && b[9] != 0) { strcpy(g_err, "NES 2.0 extended sizes are not supported"); return -1; }
    unsigned mapper = (f6 >> 4) | (f7 & 0xF0);
    if (nes2) mapper |= (unsigned)(b[8] & 0x0F) << 8;
    size_t off = 16 + ((f6 & 0x04) ? 512 : 0);
    size_t prg = (size_t)prg_banks * 16384, chr = (size_t)chr_banks * 8192;
    if (len < off + prg + chr) { strcpy(g_err, "iNES data is truncated for declared PRG/CHR sizes"); return -1; }
    /* EXTENSION: the reference accepts NROM only; this checker also restates
     * UxROM (mapper 2, power-of-two 16 KB PRG banks, the last one fixed at
     * $C000) and CNROM (mapper 3, 16/32 KB PRG, power-of-two 8 KB CHR banks). */
    int pow2_prg = prg_banks && !(prg_banks & (prg_banks - 1)), pow2_chr = chr_banks && !(chr_banks & (chr_banks - 1));
    int nrom = mapper == 0 && (prg_banks == 1 || prg_banks == 2);
    int uxrom = mapper == 2 && prg_banks >= 2 && prg_banks <= 16 && pow2_prg && chr_banks <= 1;
    int cnrom = mapper == 3 && (prg_banks == 1 || prg_banks == 2) && chr_banks <= 4 && pow2_chr;
    if (!nrom && !uxrom && !cnrom) {
        strcpy(g_err, "supported cartridges: mapper 0/NROM, 2/UxROM and 3/CNROM"); return -1;
    }
    if (f6 & 0x08) { strcpy(g_err, "four-screen nametables are not supported"); return -1; }
    o->mapper = mapper;
    o->prg_banks = prg_banks;
    o->chr_banks = chr_banks;
    o->prg_rom = malloc(prg);
    memcpy(o->prg_rom, b + off, prg);
    if (uxrom) { /* the fixed window: bank 0 at $8000, the last bank at $C000 */
        o->prg_size = 32768;
        o->prg = malloc(32768);
        memcpy(o->prg, b + off, 16384);
        memcpy(o->prg + 16384, b + off + prg - 16384, 16384);
    } else {
        o->prg_size = (uint32_t)prg;
        o->prg = malloc(prg);
        memcpy(o->prg, b + off, prg);
    }
    o->chr_size = (uint32_t)chr;
    o->chr = chr ? malloc(chr) : NULL;
    if (chr) memcpy(o->chr, b + off + prg, chr);
    o->horizontal = (f6 & 0x01) ? 0 : 1;
    return 0;
}

static uint32_t le32(const uint8_t *p) { return p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24); }

/* cpp/include/nesle/fcs.hpp:91-160 (sub-chunk fields) and :187-226 (walk). */
static int fcs_apply(snap_t *s, int tag, const char *name, const uint8_t *p, uint32_t n) {
#define IS(str) (strcmp(name, str) == 0)
#define FIXED(dst, str)                                                          \
    do {                                                                         \
        if (n != sizeof(dst)) { strcpy(g_err, "FCS: " str " has the wrong size"); return -1; } \
        memcpy(dst, p, n);                                                       \
    } while (0)
    if (tag == 1) {
        if (IS("PC")) { if (n != 2) { strcpy(g_err, "FCS: CPU.PC must be 2 bytes"); return -1; } s->pc = (uint16_t)(p[0] | (p[1] << 8)); }
        else if (IS("A") && n == 1) s->a = p[0];
        else if (IS("X") && n == 1) s->x = p[0];
        else if (IS("Y") && n == 1) s->y = p[0];
        else if (IS("S") && n == 1) s->sp = p[0];
        else if (IS("P") && n == 1) s->p = p[0];
        else if (IS("RAM")) FIXED(s->ram, "CPU.RAM");
    } else if (tag == 3) {
        if (IS("NTAR")) FIXED(s->nt, "PPU.NTAR");
        else if (IS("PRAM")) FIXED(s->pal, "PPU.PRAM");
        else if (IS("SPRA")) FIXED(s->oam, "PPU.SPRA");
        else if (IS("PPUR")) {
            if (n < 3) { strcpy(g_err, "FCS: PPU.PPUR too short"); return -1; }
            s->ctrl = p[0]; s->mask = p[1]; s->status = p[2];
        } else if (IS("PSPL") && n == 1) s->oam_addr = p[0];
        else if (IS("XOFF") && n == 1) s->fine_x = p[0] & 7;
        else if (IS("VTGL") && n == 1) s->w = p[0] & 1;
        else if (IS("RADD") && n == 2) s->v = (uint16_t)(p[0] | (p[1] << 8));
        else if (IS("TADD") && n == 2) s->t = (uint16_t)(p[0] | (p[1] << 8));
        else if (IS("VBUF") && n == 1) s->read_buffer = p[0];
        else if (IS("PGEN") && n == 1) s->open_bus = p[0];
    } else if (tag == 16) {
        if (IS("WRAM")) FIXED(s->prg_ram, "CART.WRAM");
    }
    return 0;
#undef IS
#undef FIXED
}

static int parse_fcs(snap_t *s, const uint8_t *d, size_t len) {
    memset(s, 0, sizeof(*s));
    s->sp = 0xFD;
    s->p = 0x24;
    if (len < 16) { strcpy(g_err, "FCS: header too short"); return -1; }
    if (d[0] != 'F' || d[1] != 'C' || d[2] != 'S' || d[3] != 0xFF) { strcpy(g_err, "FCS: bad magic"); return -1; }
    size_t off = 16;
    while (off + 5 <= len) {
        int tag = d[off];
        uint32_t size = le32(d + off + 1);
        off += 5;
        if (off + size > len) { strcpy(g_err, "FCS: top-level chunk extends past file"); return -1; }
        if (tag == 1 || tag == 3 || tag == 16) {
            size_t so = 0;
            while (so + 8 <= size) {
                char name[5];
                memcpy(name, d + off + so, 4);
                name[4] = 0;
                uint32_t ss = le32(d + off + so + 4);
                so += 8;
                if (so + ss > size) { strcpy(g_err, "FCS: sub-chunk extends past parent payload"); return -1; }
                if (fcs_apply(s, tag, name, d + off + so, ss)) return -1;
                so += ss;
            }
            if (so != size) { strcpy(g_err, "FCS: trailing bytes in sub-chunk stream"); return -1; }
        }
        off += size;
    }
    if (off != len) { strcpy(g_err, "FCS: trailing bytes after last top-level chunk"); return -1; }
    return 0;
}

/* ------------------------------------------------------------------------ */
/* Bus: cpp/include/nesle/cuda/batch_bus.cuh.                                  */
/* ------------------------------------------------------------------------ */

/* batch_bus.cuh:35-53 */
static uint16_t mirror_pal(uint16_t a) {
    uint16_t i = a & 0x1F;
    if (i == 0x10 || i == 0x14 || i == 0x18 || i == 0x1C) i -= 0x10;
    return i;
}
static uint16_t mirror_nt(const nes_oracle *o, uint16_t a) {
    uint16_t i = (uint16_t)((a - 0x2000) & 0x0FFF);
    if (o->horizontal) return (uint16_t)((i & 0x03FF) | ((i & 0x0800) >> 1));
    return i & 0x07FF;
}
/* batch_bus.cuh:55-95 (live state) and batch_render.cuh:104-121 (any view). */
static uint8_t ppu_mem_read(const nes_oracle *o, uint8_t chr_bank, const uint8_t *nt, const uint8_t *pal,
                            uint16_t a) {
    a &= 0x3FFF;
    if (a < 0x2000) {
        /* EXTENSION: CNROM selects an 8 KB CHR bank */
        uint32_t off = o->mapper == 3 ? (uint32_t)chr_bank * 8192u : 0u;
        return (o->chr && o->chr_size) ? o->chr[(off + a) % o->chr_size] : 0;
    }
    if (a < 0x3F00) {
        if (a >= 0x3000) a -= 0x1000;
        return nt[mirror_nt(o, a)];
    }
    return pal[mirror_pal(a)];
}
static void ppu_mem_write(const nes_oracle *o, env_t *e, uint16_t a, uint8_t v) {
    a &= 0x3FFF;
    if (a < 0x2000) return;
    if (a < 0x3F00) {
        if (a >= 0x3000) a -= 0x1000;
        e->nt[mirror_nt(o, a)] = v;
        return;
    }
    e->pal[mirror_pal(a)] = v;
}

/* batch_bus.cuh:105-133 */
static void latch_controller(env_t *e) { e->ctrl_shift = e->action; e->ctrl_count = 0; }
static uint8_t read_controller(env_t *e) {
    if (e->ctrl_strobe) return (uint8_t)(0x40 | (e->action & 1));
    uint8_t bit = 1;
    if (e->ctrl_count < 8) {
        bit = e->ctrl_shift & 1;
        e->ctrl_shift >>= 1;
        e->ctrl_count++;
    }
    return (uint8_t)(0x40 | bit);
}

/* batch_bus.cuh:135-154 */
static void oam_dma(env_t *e, uint8_t page) {
    uint16_t base = (uint16_t)(page << 8);
    for (int i = 0; i < 256; ++i) {
        TOUCH(e, base + i);
        e->oam[(uint8_t)(e->oam_addr + i)] = e->ram[(base + i) & 0x7FF];
    }
    e->pending_dma += 513;
}

/* PRG ROM at $8000-$FFFF (batch_bus.cuh:24-33); EXTENSION: UxROM maps the
 * env's bank at $8000-$BFFF. */
static uint8_t prg_read(const nes_oracle *o, const env_t *e, uint16_t a) {
    if (o->mapper == 2 && a < 0xC000) return o->prg_rom[(uint32_t)e->prg_bank * 0x4000u + (a & 0x3FFF)];
    uint32_t i = (uint32_t)(a - 0x8000);
    i &= (o->prg_size == 16384) ? 0x3FFF : 0x7FFF;
    return o->prg[i];
}

/* batch_bus.cuh:156-213 */
static uint8_t bus_read(const nes_oracle *o, env_t *e, uint16_t a) {
    if (a < 0x2000) { TOUCH(e, a); return e->ram[a & 0x7FF]; }
    if (a < 0x4000) {
        int reg = (a - 0x2000) & 7;
        if (reg == 2) {
            uint8_t v = (uint8_t)((e->ppu_status & 0xE0) | (e->open_bus & 0x1F));
            e->ppu_status &= 0x7F;
            e->nmi_pending = 0;
            e->w = 0;
            e->open_bus = v;
            return v;
        }
        if (reg == 4) return e->oam[e->oam_addr];
        if (reg == 7) {
            uint16_t pa = e->v & 0x3FFF;
            uint8_t v;
            if (pa >= 0x3F00) {
                v = ppu_mem_read(o, e->chr_bank, e->nt, e->pal, pa);
                e->read_buffer = ppu_mem_read(o, e->chr_bank, e->nt, e->pal, (uint16_t)(pa - 0x1000));
            } else {
                v = e->read_buffer;
                e->read_buffer = ppu_mem_read(o, e->chr_bank, e->nt, e->pal, pa);
            }
            e->v = (uint16_t)(e->v + ((e->ppu_ctrl & 0x04) ? 32 : 1));
            e->open_bus = v;
            return v;
        }
        return 0;
    }
    if (a == 0x4016) return read_controller(e);
    if (a == 0x4017) return 0x41;
    if (a >= 0x6000 && a < 0x8000) return e->prg_ram[a - 0x6000];
    if (a >= 0x8000) return prg_read(o, e, a);
    return 0;
}

/* batch_bus.cuh:215-304 */
static void bus_write(const nes_oracle *o, env_t *e, uint16_t a, uint8_t v) {
    if (a < 0x2000) { TOUCH(e, a); e->ram[a & 0x7FF] = v; return; }
    if (a < 0x4000) {
        int reg = (a - 0x2000) & 7;
        if (reg == 0) {
            if ((v & 0x80) && !(e->ppu_ctrl & 0x80) && (e->ppu_status & 0x80)) e->nmi_pending = 1;
            e->ppu_ctrl = v;
            e->t = (uint16_t)((e->t & 0xF3FF) | ((v & 3) << 10));
        } else if (reg == 1) {
            e->ppu_mask = v;
        } else if (reg == 3) {
            e->oam_addr = v;
        } else if (reg == 4) {
            e->oam[e->oam_addr] = v;
            e->oam_addr++;
        } else if (reg == 5) {
            if (e->w == 0) {
                e->fine_x = v & 7;
                e->scroll_x = v;
                e->t = (uint16_t)((e->t & 0xFFE0) | (v >> 3));
                e->w = 1;
            } else {
                e->scroll_y = v;
                e->t = (uint16_t)((e->t & 0x8FFF) | ((v & 7) << 12));
                e->t = (uint16_t)((e->t & 0xFC1F) | ((v & 0xF8) << 2));
                e->w = 0;
            }
        } else if (reg == 6) {
            if (e->w == 0) {
                e->t = (uint16_t)((e->t & 0x00FF) | ((v & 0x3F) << 8));
                e->w = 1;
            } else {
                e->t = (uint16_t)((e->t & 0x7F00) | v);
                e->v = e->t;
                e->w = 0;
            }
        } else if (reg == 7) {
            ppu_mem_write(o, e, e->v, v);
            e->v = (uint16_t)(e->v + ((e->ppu_ctrl & 0x04) ? 32 : 1));
        }
        e->open_bus = v;
        return;
    }
    if (a == 0x4014) { oam_dma(e, v); return; }
    if (a == 0x4016) {
        uint8_t next = v & 1;
        if (next || e->ctrl_strobe) latch_controller(e);
        e->ctrl_strobe = next;
        return;
    }
    if (a >= 0x6000 && a < 0x8000) e->prg_ram[a - 0x6000] = v;
    if (a >= 0x8000 && o->mapper) { /* EXTENSION: board register, with the bus conflict of the ROM byte */
        v &= prg_read(o, e, a);
        if (o->mapper == 2) e->prg_bank = (uint8_t)(v & (o->prg_banks - 1));
        else e->chr_bank = (uint8_t)(v & (o->chr_banks - 1));
    }
}

/* ------------------------------------------------------------------------ */
/* 6502 (2A03: no decimal mode): cpp/include/nesle/cpu.hpp:84-123,378-730.     */
/* ------------------------------------------------------------------------ */
#define FC 0x01
#define FZ 0x02
#define FI 0x04
#define FD 0x08
#define FB 0x10
#define FU 0x20
#define FV 0x40
#define FN 0x80

static void setf(env_t *e, uint8_t f, int on) {
    if (on) e->p |= f; else e->p &= (uint8_t)~f;
    e->p |= FU;
}
static void setzn(env_t *e, uint8_t v) { setf(e, FZ, v == 0); setf(e, FN, v & 0x80); }
static void push(const nes_oracle *o, env_t *e, uint8_t v) { bus_write(o, e, (uint16_t)(0x100 | e->sp), v); e->sp--; }
static uint8_t pull(const nes_oracle *o, env_t *e) { e->sp++; return bus_read(o, e, (uint16_t)(0x100 | e->sp)); }

/* cpu.hpp:112-123 */
static void cpu_nmi(const nes_oracle *o, env_t *e) {
    push(o, e, (uint8_t)(e->pc >> 8));
    push(o, e, (uint8_t)e->pc);
    push(o, e, (uint8_t)((e->p & ~FB) | FU));
    setf(e, FI, 1);
    uint8_t lo = bus_read(o, e, 0xFFFA), hi = bus_read(o, e, 0xFFFB);
    e->pc = (uint16_t)(lo | (hi << 8));
    e->cycles += 7;
}

static void adc(env_t *e, uint8_t m) {
    unsigned sum = e->a + m + (e->p & FC);
    uint8_t r = (uint8_t)sum;
    setf(e, FV, (~(e->a ^ m) & (e->a ^ r)) & 0x80);
    setf(e, FC, sum > 0xFF);
    e->a = r;
    setzn(e, r);
}
static void cmp(env_t *e, uint8_t reg, uint8_t m) {
    setf(e, FC, reg >= m);
    setzn(e, (uint8_t)(reg - m));
}

/* One cpu::step.  Returns the opcode; *op_pc receives the instruction address.
 * Returns -1 (and leaves pc/cycles untouched) on an illegal opcode: the
 * reference executes `trap` there (cpu.hpp:716-720); this build records a
 * status word instead (EXTENSION). */
static int cpu_step(const nes_oracle *o, env_t *e, uint16_t *op_pc) {
    uint16_t start = e->pc;
    *op_pc = start;
    uint8_t opc = bus_read(o, e, e->pc);
    decode_t d = g_decode[opc];
    if (d.flags & F_ILLEGAL) {
        e->status = ORACLE_STATUS_ILLEGAL | ((uint32_t)opc << 16) | start;
        return -1;
    }
    e->pc++;
    unsigned extra = 0;
    uint16_t addr = 0;
#define FETCH() (bus_read(o, e, e->pc++))
    switch (d.mode) {
    case IMP: case ACC: case REL: break;
    case IMM: addr = e->pc++; break;
    case ZP: addr = FETCH(); break;
    case ZPX: addr = (uint8_t)(FETCH() + e->x); break;
    case ZPY: addr = (uint8_t)(FETCH() + e->y); break;
    case ABS: { uint8_t lo = FETCH(); uint8_t hi = FETCH(); addr = (uint16_t)(lo | (hi << 8)); break; }
    case ABSX: case ABSY: {
        uint8_t lo = FETCH(); uint8_t hi = FETCH();
        uint16_t base = (uint16_t)(lo | (hi << 8));
        addr = (uint16_t)(base + (d.mode == ABSX ? e->x : e->y));
        if ((d.flags & F_PAGE) && ((base ^ addr) & 0xFF00)) extra++;
        break;
    }
    case INDX: {
        uint8_t ptr = (uint8_t)(FETCH() + e->x);
        uint8_t lo = bus_read(o, e, ptr), hi = bus_read(o, e, (uint8_t)(ptr + 1));
        addr = (uint16_t)(lo | (hi << 8));
        break;
    }
    case INDY: {
        uint8_t ptr = FETCH();
        uint8_t lo = bus_read(o, e, ptr), hi = bus_read(o, e, (uint8_t)(ptr + 1));
        uint16_t base = (uint16_t)(lo | (hi << 8));
        addr = (uint16_t)(base + e->y);
        if ((d.flags & F_PAGE) && ((base ^ addr) & 0xFF00)) extra++;
        break;
    }
    case IND: {
        uint8_t lo = FETCH(); uint8_t hi = FETCH();
        uint16_t ptr = (uint16_t)(lo | (hi << 8));
        uint8_t tl = bus_read(o, e, ptr);
        uint8_t th = bus_read(o, e, (uint16_t)((ptr & 0xFF00) | ((ptr + 1) & 0x00FF)));
        addr = (uint16_t)(tl | (th << 8));
        break;
    }
    }
    uint8_t m, r;
    switch (d.ins) {
    case I_LDA: e->a = bus_read(o, e, addr); setzn(e, e->a); break;
    case I_LDX: e->x = bus_read(o, e, addr); setzn(e, e->x); break;
    case I_LDY: e->y = bus_read(o, e, addr); setzn(e, e->y); break;
    case I_STA: bus_write(o, e, addr, e->a); break;
    case I_STX: bus_write(o, e, addr, e->x); break;
    case I_STY: bus_write(o, e, addr, e->y); break;
    case I_TAX: e->x = e->a; setzn(e, e->x); break;
    case I_TAY: e->y = e->a; setzn(e, e->y); break;
    case I_TXA: e->a = e->x; setzn(e, e->a); break;
    case I_TYA: e->a = e->y; setzn(e, e->a); break;
    case I_TSX: e->x = e->sp; setzn(e, e->x); break;
    case I_TXS: e->sp = e->x; break;
    case I_PHA: push(o, e, e->a); break;
    case I_PHP: push(o, e, (uint8_t)(e->p | FB | FU)); break;
    case I_PLA: e->a = pull(o, e); setzn(e, e->a); break;
    case I_PLP: e->p = (uint8_t)((pull(o, e) | FU) & ~FB); break;
    case I_ORA: e->a |= bus_read(o, e, addr); setzn(e, e->a); break;
    case I_AND: e->a &= bus_read(o, e, addr); setzn(e, e->a); break;
    case I_EOR: e->a ^= bus_read(o, e, addr); setzn(e, e->a); break;
    case I_ADC: adc(e, bus_read(o, e, addr)); break;
    case I_SBC: adc(e, (uint8_t)(bus_read(o, e, addr) ^ 0xFF)); break;
    case I_CMP: cmp(e, e->a, bus_read(o, e, addr)); break;
    case I_CPX: cmp(e, e->x, bus_read(o, e, addr)); break;
    case I_CPY: cmp(e, e->y, bus_read(o, e, addr)); break;
    case I_BIT:
        m = bus_read(o, e, addr);
        setf(e, FZ, (e->a & m) == 0); setf(e, FN, m & 0x80); setf(e, FV, m & 0x40);
        break;
    case I_INC: r = (uint8_t)(bus_read(o, e, addr) + 1); bus_write(o, e, addr, r); setzn(e, r); break;
    case I_DEC: r = (uint8_t)(bus_read(o, e, addr) - 1); bus_write(o, e, addr, r); setzn(e, r); break;
    case I_INX: e->x++; setzn(e, e->x); break;
    case I_INY: e->y++; setzn(e, e->y); break;
    case I_DEX: e->x--; setzn(e, e->x); break;
    case I_DEY: e->y--; setzn(e, e->y); break;
    case I_ASL: case I_LSR: case I_ROL: case I_ROR: {
        m = (d.mode == ACC) ? e->a : bus_read(o, e, addr);
        int c = e->p & FC;
        if (d.ins == I_ASL || d.ins == I_ROL) {
            setf(e, FC, m & 0x80);
            r = (uint8_t)((m << 1) | (d.ins == I_ROL ? c : 0));
        } else {
            setf(e, FC, m & 1);
            r = (uint8_t)((m >> 1) | (d.ins == I_ROR && c ? 0x80 : 0));
        }
        setzn(e, r);
        if (d.mode == ACC) e->a = r; else bus_write(o, e, addr, r);
        break;
    }
    case I_JMP: e->pc = addr; break;
    case I_JSR: {
        uint16_t ret = (uint16_t)(e->pc - 1);
        push(o, e, (uint8_t)(ret >> 8)); push(o, e, (uint8_t)ret);
        e->pc = addr;
        break;
    }
    case I_RTS: { uint8_t lo = pull(o, e); uint8_t hi = pull(o, e); e->pc = (uint16_t)((lo | (hi << 8)) + 1); break; }
    case I_RTI: {
        e->p = (uint8_t)((pull(o, e) | FU) & ~FB);
        uint8_t lo = pull(o, e); uint8_t hi = pull(o, e);
        e->pc = (uint16_t)(lo | (hi << 8));
        break;
    }
    case I_BRK: {
        e->pc++;
        push(o, e, (uint8_t)(e->pc >> 8)); push(o, e, (uint8_t)e->pc);
        push(o, e, (uint8_t)(e->p | FB | FU));
        setf(e, FI, 1);
        uint8_t lo = bus_read(o, e, 0xFFFE), hi = bus_read(o, e, 0xFFFF);
        e->pc = (uint16_t)(lo | (hi << 8));
        break;
    }
    case I_BRANCH: {
        static const uint8_t sel[4] = {FN, FV, FC, FZ};
        int flag = (e->p & sel[opc >> 6]) != 0;
        int8_t off = (int8_t)FETCH();
        if (flag == ((opc & 0x20) != 0)) {
            uint16_t old = e->pc;
            e->pc = (uint16_t)(e->pc + off);
            extra++;
            if ((old ^ e->pc) & 0xFF00) extra++;
        }
        break;
    }
    case I_CLC: setf(e, FC, 0); break;
    case I_SEC: setf(e, FC, 1); break;
    case I_CLI: setf(e, FI, 0); break;
    case I_SEI: setf(e, FI, 1); break;
    case I_CLV: setf(e, FV, 0); break;
    case I_CLD: setf(e, FD, 0); break;
    case I_SED: setf(e, FD, 1); break;
    case I_NOP: break;
    }
#undef FETCH
    e->cycles += (uint8_t)(extra + d.cycles);
    return opc;
}

/* ------------------------------------------------------------------------ */
/* Lazy PPU timing: cpp/include/nesle/cuda/batch_ppu.cuh:15-21,62-73,138-269. */
/* ------------------------------------------------------------------------ */
#define FRAME_DOTS (341u * 262u)
#define SPRITE0_DOT (30u * 341u + 1u)
#define VBLANK_DOT (241u * 341u + 1u)
#define PRERENDER_DOT (261u * 341u + 1u)

static uint32_t dist_to(uint32_t cur, uint32_t ev) { return ev > cur ? ev - cur : FRAME_DOTS - cur + ev; }

/* batch_ppu.cuh:138-177 */
static uint32_t dots_to_next_event(const env_t *e) {
    uint32_t next = FRAME_DOTS - e->frame_dot;
    uint32_t d = dist_to(e->frame_dot, VBLANK_DOT);
    if (d < next) next = d;
    d = dist_to(e->frame_dot, PRERENDER_DOT);
    if (d < next) next = d;
    if (e->ppu_mask & 0x18) {
        d = dist_to(e->frame_dot, SPRITE0_DOT);
        if (d < next) next = d;
    }
    return next;
}

/* batch_ppu.cuh:62-73 */
static void set_vblank(env_t *e, int on) {
    uint8_t was = e->ppu_status & 0x80;
    if (on) {
        e->ppu_status |= 0x80;
        if (!was && (e->ppu_ctrl & 0x80)) e->nmi_pending = 1;
        return;
    }
    e->ppu_status &= 0x7F;
    e->nmi_pending = 0;
}

/* batch_ppu.cuh:183-269.  Returns frames completed. */
static uint32_t ppu_settle(env_t *e, uint32_t ppu_cycles) {
    uint32_t start = e->frame_dot, end = start + ppu_cycles;
    uint32_t frames = end / FRAME_DOTS;
    for (uint32_t f = 0; f <= frames; ++f) {
#define CROSSED(ev) ((f * FRAME_DOTS + (ev)) > start && (f * FRAME_DOTS + (ev)) <= end)
        if (CROSSED(SPRITE0_DOT) && (e->ppu_mask & 0x18)) e->ppu_status |= 0x40;
        if (CROSSED(VBLANK_DOT)) {
            set_vblank(e, 1);
            e->snap_sx_start = e->lat_sx;
            e->snap_sy_start = e->lat_sy;
            e->snap_ctrl_start = e->lat_ctrl;
            e->snap_sx_end = e->scroll_x;
            e->snap_sy_end = e->scroll_y;
            e->snap_ctrl_end = e->ppu_ctrl;
            e->snap_mask = e->ppu_mask;
            memcpy(e->snap_oam, e->oam, 256);
            memcpy(e->snap_nt, e->nt, 2048);
            memcpy(e->snap_pal, e->pal, 32);
            e->snap_chr_bank = e->chr_bank;
        }
        if (CROSSED(PRERENDER_DOT)) {
            set_vblank(e, 0);
            e->ppu_status &= 0x1F;
            e->lat_sx = e->scroll_x;
            e->lat_sy = e->scroll_y;
            e->lat_ctrl = e->ppu_ctrl;
        }
#undef CROSSED
    }
    e->frame_dot = end % FRAME_DOTS;
    e->frame += frames;
    return frames;
}

/* ------------------------------------------------------------------------ */
/* Reward, done and resets: cpp/include/nesle/cuda/batch_step.cuh.            */
/* ------------------------------------------------------------------------ */
static int bcd3(const uint8_t *ram, int a) {
    return (ram[a] & 0xF) * 100 + (ram[a + 1] & 0xF) * 10 + (ram[a + 2] & 0xF);
}

/* batch_step.cuh:51-106, plus the EXTENSION done predicates. */
static void apply_reward(const nes_oracle *o, env_t *e, uint32_t env) {
    const uint8_t *ram = e->ram;
    static const uint16_t kRead[] = {0x6D, 0x86, 0x7F8, 0x7F9, 0x7FA, 0x0E, 0xB5, 0x75A, 0x16, 0x1D, 0x770};
    for (size_t i = 0; i < sizeof(kRead) / sizeof(kRead[0]); ++i) TOUCH(e, kRead[i]);
    if (o->done_mode == ORACLE_DONE_RAM_EQ) TOUCH(e, o->done_a);
    int x = ram[0x6D] * 0x100 + ram[0x86];
    int time = bcd3(ram, 0x7F8);
    int dying = ram[0x0E] == 0x0B || ram[0xB5] > 1;
    int dead = ram[0x0E] == 0x06;
    int over = ram[0x75A] == 0xFF;
    int stage_over = 0;
    for (int i = 0; i < 5; ++i) {
        uint8_t en = ram[0x16 + i];
        if ((en == 0x2D || en == 0x31) && ram[0x1D] == 3) stage_over = 1;
    }
    int flag = ram[0x770] == 2 || stage_over;
    int rx = x - e->prev_x;
    if (rx < -5 || rx > 5) rx = 0;
    int rt = time - e->prev_time;
    if (rt > 0) rt = 0;
    int death = (dying || dead) ? -25 : 0;
    e->reward = (float)(rx + rt + death);
    uint8_t done = (flag || dying || dead || over) ? 1 : 0;
    if (o->done_mode == ORACLE_DONE_RAM_EQ) done = ram[o->done_a & 0x7FF] == (uint8_t)o->done_b;
    else if (o->done_mode == ORACLE_DONE_FRAME_LIMIT) done = e->frame >= frame_limit(o, env, e->episode);
    e->done = done;
    e->prev_x = x;
    e->prev_time = time;
}

/* batch_step.cuh:109-172 */
static void cold_reset(const nes_oracle *o, env_t *e) {
    uint32_t base = o->prg_size == 16384 ? 0x3FFC : 0x7FFC;
    e->pc = (uint16_t)(o->prg[base] | (o->prg[base + 1] << 8));
    e->a = e->x = e->y = 0;
    e->sp = 0xFD;
    e->p = 0x24;
    e->cycles = 7;
    e->cpu_nmi_pending = e->irq_pending = 0;
    e->ctrl_shift = 0; e->ctrl_count = 8; e->ctrl_strobe = 0;
    e->pending_dma = 0;
    memset(e->ram, 0, 2048);
    memset(e->prg_ram, 0, 8192);
    e->ppu_ctrl = e->ppu_mask = e->ppu_status = e->oam_addr = e->nmi_pending = 0;
    e->frame_dot = 0; e->frame = 0;
    e->v = e->t = 0;
    e->fine_x = e->w = e->open_bus = e->read_buffer = e->scroll_x = e->scroll_y = 0;
    memset(e->nt, 0, 2048); memset(e->pal, 0, 32); memset(e->oam, 0, 256);
    e->prev_x = 0; e->prev_time = 0;
    e->reward = 0.0f; e->done = 0;
    e->status = 0;
}

/* batch_step.cuh:174-242 */
static void warm_reset(const nes_oracle *o, env_t *e, uint32_t env) {
    const snap_t *s = &o->snaps[o->env_to_level[env]];
    e->pc = s->pc; e->a = s->a; e->x = s->x; e->y = s->y; e->sp = s->sp; e->p = s->p;
    e->cycles = s->cycles;
    e->cpu_nmi_pending = e->irq_pending = 0;
    e->ctrl_shift = 0; e->ctrl_count = 8; e->ctrl_strobe = 0;
    e->pending_dma = 0;
    memcpy(e->ram, s->ram, 2048);
    memcpy(e->prg_ram, s->prg_ram, 8192);
    e->ppu_ctrl = s->ctrl; e->ppu_mask = s->mask; e->ppu_status = s->status;
    e->oam_addr = s->oam_addr; e->nmi_pending = 0;
    e->frame_dot = 0; e->frame = 0;
    e->v = s->v; e->t = s->t; e->fine_x = s->fine_x; e->w = s->w;
    e->open_bus = s->open_bus; e->read_buffer = s->read_buffer;
    e->scroll_x = e->scroll_y = 0;
    memcpy(e->nt, s->nt, 2048); memcpy(e->pal, s->pal, 32); memcpy(e->oam, s->oam, 256);
    e->prev_x = s->ram[0x6D] * 0x100 + s->ram[0x86];
    e->prev_time = bcd3(s->ram, 0x7F8);
    e->reward = 0.0f; e->done = 0;
    e->status = 0;
}

static void reset_env(const nes_oracle *o, env_t *e, uint32_t env) {
    if (o->nsnap) warm_reset(o, e, env); else cold_reset(o, e);
    e->prg_bank = e->chr_bank = 0; /* EXTENSION: board registers; the snapshot's CHR bank survives */
}

/* cuda_module.cu:1443-1463 */
static void seed_presentation(env_t *e) {
    e->snap_chr_bank = e->chr_bank;
    memcpy(e->snap_nt, e->nt, 2048);
    memcpy(e->snap_pal, e->pal, 32);
    memcpy(e->snap_oam, e->oam, 256);
    e->snap_mask = e->ppu_mask;
    e->lat_sx = e->snap_sx_start = e->snap_sx_end = e->scroll_x;
    e->lat_sy = e->snap_sy_start = e->snap_sy_end = e->scroll_y;
    e->lat_ctrl = e->snap_ctrl_start = e->snap_ctrl_end = e->ppu_ctrl;
}

/* ------------------------------------------------------------------------ */
/* The env-step kernel body: cpp/src/cuda/kernels.cu:19-104, with
 * step_batch_console_instruction_lazy (batch_console.hpp:77-109) and the idle
 * fast-forward (batch_console.hpp:129-152) inlined.                            */
/* ------------------------------------------------------------------------ */
static void env_step(const nes_oracle *o, env_t *e, uint32_t env) {
    e->ram_touch = 0;
    uint32_t pending = 0;
    uint32_t horizon = dots_to_next_event(e);
    uint64_t total_instr = 0;
    uint32_t total_frames = 0, budget = 0;
    for (uint32_t frame = 0; frame < o->frameskip; ++frame) {
        uint64_t instr = 0;
        uint32_t done_frames = 0;
        while (instr < o->max_instr && done_frames == 0 && e->status == 0) {
            if (pending >= horizon) {
                done_frames += ppu_settle(e, pending);
                pending = 0;
                horizon = dots_to_next_event(e);
                if (done_frames) break;
            }
            uint64_t before = e->cycles;
            if (e->nmi_pending) {
                e->nmi_pending = 0;
                cpu_nmi(o, e);
            }
            uint16_t op_pc;
            int opc = cpu_step(o, e, &op_pc);
            if (opc < 0) break; /* EXTENSION: illegal opcode freezes the env */
            if (e->pending_dma) {
                e->cycles += e->pending_dma;
                e->pending_dma = 0;
            }
            pending += (uint32_t)(e->cycles - before) * 3u;
            ++instr;
            /* kernels.cu:59-64: one count per executed instruction, by opcode
             * and by the address it was fetched from (after any NMI entry). */
            if (o->prof_opcode) o->prof_opcode[opc]++;
            if (o->prof_pc) o->prof_pc[op_pc]++;
            if (o->trace_buf && env == o->trace_env && o->trace_n < o->trace_cap) {
                uint8_t *r = ((nes_oracle *)o)->trace_buf + (size_t)o->trace_n * 16;
                r[0] = (uint8_t)op_pc; r[1] = (uint8_t)(op_pc >> 8); r[2] = (uint8_t)opc;
                r[3] = e->a; r[4] = e->x; r[5] = e->y; r[6] = e->p; r[7] = e->sp;
                memcpy(r + 8, &e->cycles, 8);
                ((nes_oracle *)o)->trace_n++;
            }
            if (opc == 0x4C && e->pc == op_pc && done_frames == 0) {
                done_frames += ppu_settle(e, pending);
                pending = 0;
                uint32_t jumps = (dots_to_next_event(e) + 8u) / 9u;
                if (jumps) {
                    e->cycles += (uint64_t)jumps * 3u;
                    done_frames += ppu_settle(e, jumps * 9u);
                }
                horizon = dots_to_next_event(e);
            }
        }
        if (pending) {
            done_frames += ppu_settle(e, pending);
            pending = 0;
            horizon = dots_to_next_event(e);
        }
        total_instr += instr;
        total_frames += done_frames;
        if (done_frames == 0 && instr >= o->max_instr) ++budget;
        if (e->status) break;
    }
    e->stat_instructions = total_instr;
    e->stat_frames = total_frames;
    e->stat_budget_hits = budget;
    apply_reward(o, e, env);
}

/* ------------------------------------------------------------------------ */
/* Host API.                                                                   */
/* ------------------------------------------------------------------------ */
nes_oracle *oracle_create(uint32_t num_envs, uint32_t frameskip, const uint8_t *rom,
                          size_t rom_len, const uint8_t *const *snapshots,
                          const size_t *snapshot_lens, uint32_t num_snapshots,
                          const uint8_t *env_to_level, uint32_t done_mode, uint32_t done_a,
                          uint32_t done_b, uint64_t seed, uint32_t env_offset) {
    build_decode();
    g_err[0] = 0;
    if (num_envs == 0) { strcpy(g_err, "num_envs must be positive"); return NULL; }
    if (frameskip == 0) { strcpy(g_err, "frameskip must be positive"); return NULL; }
    if (num_snapshots > 255) { strcpy(g_err, "at most 255 snapshot levels supported per CudaBatch"); return NULL; }
    if (done_mode == ORACLE_DONE_FRAME_LIMIT && done_b < done_a) { strcpy(g_err, "bad frame-limit range"); return NULL; }
    nes_oracle *o = calloc(1, sizeof(*o));
    o->n = num_envs;
    o->frameskip = frameskip;
    o->max_instr = 200000;
    if (parse_ines(o, rom, rom_len)) { oracle_destroy(o); return NULL; }
    o->nsnap = num_snapshots;
    o->snaps = calloc(num_snapshots ? num_snapshots : 1, sizeof(snap_t));
    for (uint32_t i = 0; i < num_snapshots; ++i) {
        if (parse_fcs(&o->snaps[i], snapshots[i], snapshot_lens[i])) { oracle_destroy(o); return NULL; }
    }
    o->env_to_level = calloc(num_envs, 1);
    if (env_to_level) {
        for (uint32_t i = 0; i < num_envs; ++i) {
            if (num_snapshots && env_to_level[i] >= num_snapshots) {
                strcpy(g_err, "env_to_level out of range");
                oracle_destroy(o);
                return NULL;
            }
            o->env_to_level[i] = env_to_level[i];
        }
    }
    o->done_mode = done_mode; o->done_a = done_a; o->done_b = done_b;
    o->seed = seed;
    o->env_offset = env_offset;
    o->env = calloc(num_envs, sizeof(env_t));
    oracle_reset(o);
    return o;
}

void oracle_destroy(nes_oracle *o) {
    if (!o) return;
    free(o->prg); free(o->prg_rom); free(o->chr); free(o->snaps); free(o->env_to_level); free(o->env);
    free(o);
}

uint32_t oracle_num_envs(const nes_oracle *o) { return o->n; }

void oracle_set_trace(nes_oracle *o, uint32_t env, uint8_t *buf, uint32_t cap) {
    o->trace_env = env; o->trace_buf = buf; o->trace_cap = cap; o->trace_n = 0;
}
uint32_t oracle_trace_count(const nes_oracle *o) { return o->trace_n; }

void oracle_set_profile(nes_oracle *o, uint64_t *opcode_counts, uint64_t *pc_counts) {
    o->prof_opcode = opcode_counts;
    o->prof_pc = pc_counts;
}

void oracle_reset(nes_oracle *o) {
    for (uint32_t i = 0; i < o->n; ++i) {
        env_t *e = &o->env[i];
        e->action = 0;
        e->episode = 0;
        reset_env(o, e, i);
        seed_presentation(e);
    }
}

void oracle_reset_envs(nes_oracle *o, const uint8_t *mask) {
    for (uint32_t i = 0; i < o->n; ++i) {
        if (mask[i]) {
            o->env[i].episode++;
            reset_env(o, &o->env[i], i);
        }
    }
}

void oracle_step(nes_oracle *o, const uint8_t *actions, int device_api, int auto_reset) {
    for (uint32_t i = 0; i < o->n; ++i) {
        env_t *e = &o->env[i];
        e->action = actions[i];
        env_step(o, e, i);
        if (device_api) {
            e->last_reward = e->reward;
            e->last_done = e->done;
            if (auto_reset && e->last_done) {
                e->episode++;
                reset_env(o, e, i);
            }
        }
    }
}

void oracle_poke_ram(nes_oracle *o, uint16_t address, uint8_t value) {
    for (uint32_t i = 0; i < o->n; ++i) o->env[i].ram[address & 0x7FF] = value;
}

/* ------------------------------------------------------------------------ */
/* Renderer: cpp/include/nesle/cuda/batch_render.cuh:123-434 over the
 * presentation-snapshot views resolved as in :333-370.                       */
/* ------------------------------------------------------------------------ */
typedef struct { const uint8_t *nt, *pal, *oam; uint8_t sx, sy, ctrl, mask, chr_bank; } view_t;

/* NES master palette (2C02), 64 RGB triples, as in batch_render.cuh:23-40. */
static const uint8_t kRgb[64][3] = {
    {0x54,0x54,0x54},{0x00,0x1e,0x74},{0x08,0x10,0x90},{0x30,0x00,0x88},{0x44,0x00,0x64},{0x5c,0x00,0x30},{0x54,0x04,0x00},{0x3c,0x18,0x00},
    {0x20,0x2a,0x00},{0x08,0x3a,0x00},{0x00,0x40,0x00},{0x00,0x3c,0x00},{0x00,0x32,0x3c},{0x00,0x00,0x00},{0x00,0x00,0x00},{0x00,0x00,0x00},
    {0x98,0x96,0x98},{0x08,0x4c,0xc4},{0x30,0x32,0xec},{0x5c,0x1e,0xe4},{0x88,0x14,0xb0},{0xa0,0x14,0x64},{0x98,0x22,0x20},{0x78,0x3c,0x00},
    {0x54,0x5a,0x00},{0x28,0x72,0x00},{0x08,0x7c,0x00},{0x00,0x76,0x28},{0x00,0x66,0x78},{0x00,0x00,0x00},{0x00,0x00,0x00},{0x00,0x00,0x00},
    {0xec,0xee,0xec},{0x4c,0x9a,0xec},{0x78,0x7c,0xec},{0xb0,0x62,0xec},{0xe4,0x54,0xec},{0xec,0x58,0xb4},{0xec,0x6a,0x64},{0xd4,0x88,0x20},
    {0xa0,0xaa,0x00},{0x74,0xc4,0x00},{0x4c,0xd0,0x20},{0x38,0xcc,0x6c},{0x38,0xb4,0xcc},{0x3c,0x3c,0x3c},{0x00,0x00,0x00},{0x00,0x00,0x00},
    {0xec,0xee,0xec},{0xa8,0xcc,0xec},{0xbc,0xbc,0xec},{0xd4,0xb2,0xec},{0xec,0xae,0xec},{0xec,0xae,0xd4},{0xec,0xb4,0xb0},{0xe4,0xc4,0x90},
    {0xcc,0xd2,0x78},{0xb4,0xde,0x78},{0xa8,0xe2,0x90},{0x98,0xe2,0xb4},{0xa0,0xd6,0xe4},{0xa0,0xa2,0xa0},{0x00,0x00,0x00},{0x00,0x00,0x00},
};

/* batch_render.cuh:123-131 */
static uint8_t pal_entry(const nes_oracle *o, const view_t *v, uint16_t idx) {
    uint8_t c = ppu_mem_read(o, v->chr_bank, v->nt, v->pal, (uint16_t)(0x3F00 + idx));
    if (v->mask & 1) c &= 0x30;
    return c & 0x3F;
}
/* batch_render.cuh:148-159 */
static uint8_t pattern_px(const nes_oracle *o, const view_t *v, uint16_t tile_base, int fx, int fy) {
    uint8_t lo = ppu_mem_read(o, v->chr_bank, v->nt, v->pal, (uint16_t)(tile_base + fy));
    uint8_t hi = ppu_mem_read(o, v->chr_bank, v->nt, v->pal, (uint16_t)(tile_base + fy + 8));
    int bit = 7 - fx;
    return (uint8_t)(((lo >> bit) & 1) | (((hi >> bit) & 1) << 1));
}
/* batch_render.cuh:161-204 */
static uint8_t bg_color(const nes_oracle *o, const view_t *v, int x, int y) {
    if (!(v->mask & 0x08) || (!(v->mask & 0x02) && x < 8)) return 0;
    unsigned wy = (unsigned)v->sy + (unsigned)y;
    unsigned cy = (wy % 240) / 8, fy = wy & 7;
    unsigned base = v->ctrl & 3;
    unsigned nty = ((base >> 1) + wy / 240) & 1;
    unsigned wx = (unsigned)v->sx + (unsigned)x;
    unsigned cx = (wx & 0xFF) / 8, fx = wx & 7;
    unsigned ntx = ((base & 1) + wx / 256) & 1;
    uint16_t ntb = (uint16_t)(0x2000 + (ntx | (nty << 1)) * 0x400);
    uint16_t pb = (v->ctrl & 0x10) ? 0x1000 : 0;
    uint8_t tile = ppu_mem_read(o, v->chr_bank, v->nt, v->pal, (uint16_t)(ntb + cy * 32 + cx));
    uint8_t c = pattern_px(o, v, (uint16_t)(pb + tile * 16), (int)fx, (int)fy);
    if (c == 0) return 0;
    uint8_t at = ppu_mem_read(o, v->chr_bank, v->nt, v->pal, (uint16_t)(ntb + 0x3C0 + (cy / 4) * 8 + cx / 4));
    int shift = ((cy & 2) << 1) | (cx & 2);
    return pal_entry(o, v, (uint16_t)(((at >> shift) & 3) * 4 + c));
}
/* batch_render.cuh:206-240 */
static uint8_t sprite_px(const nes_oracle *o, const view_t *v, uint8_t tile, uint8_t attr, int px, int py) {
    if (attr & 0x40) px = 7 - px;
    if (v->ctrl & 0x20) {
        if (attr & 0x80) py = 15 - py;
        uint16_t pb = (tile & 1) ? 0x1000 : 0;
        uint8_t tn = (uint8_t)((tile & 0xFE) + py / 8);
        return pattern_px(o, v, (uint16_t)(pb + tn * 16), px, py & 7);
    }
    if (attr & 0x80) py = 7 - py;
    uint16_t pb = (v->ctrl & 0x08) ? 0x1000 : 0;
    return pattern_px(o, v, (uint16_t)(pb + tile * 16), px, py);
}

static const int kGrayW = 84;

/* EXTENSION: BT.601 integer luma of each NES colour. */
static uint8_t luma(int c) {
    return (uint8_t)((299 * kRgb[c][0] + 587 * kRgb[c][1] + 114 * kRgb[c][2] + 500) / 1000);
}

void oracle_render(const nes_oracle *o, uint8_t *index, uint8_t *rgb, uint8_t *gray84) {
    uint8_t *fb = malloc(240 * 256);
    for (uint32_t env = 0; env < o->n; ++env) {
        const env_t *e = &o->env[env];
        /* batch_render.cuh:333-370 */
        view_t play = {e->snap_nt, e->snap_pal, e->snap_oam, e->snap_sx_end, e->snap_sy_end,
                       e->snap_ctrl_end, e->snap_mask, e->snap_chr_bank};
        view_t hud = play;
        hud.sx = e->snap_sx_start; hud.sy = e->snap_sy_start; hud.ctrl = e->snap_ctrl_start;
        /* Rows above `split` use the frame-start view; the rest, the backdrop,
         * sprites and the behind-background test use the second view.  With
         * sprite 0 off screen (split >= 240) both are the frame-start view. */
        int split = e->snap_oam[0] + 1 + ((play.ctrl & 0x20) ? 16 : 8);
        view_t lower = play;
        if (split >= 240) { lower = hud; split = 0; }
        const view_t *spr = &lower;
        for (int y = 0; y < 240; ++y) {
            const view_t *bgv = (y < split) ? &hud : &lower;
            for (int x = 0; x < 256; ++x) {
                /* batch_render.cuh:378-434 */
                uint8_t c = bg_color(o, bgv, x, y);
                if (c == 0) c = pal_entry(o, spr, 0);
                int show_left = (spr->mask & 0x04) != 0;
                if ((spr->mask & 0x10) && (show_left || x >= 8)) {
                    int h = (spr->ctrl & 0x20) ? 16 : 8;
                    for (int s = 0; s < 64; ++s) {
                        const uint8_t *so = spr->oam + s * 4;
                        int sy = y - (so[0] + 1);
                        if (sy < 0 || sy >= h) continue;
                        int sx = x - so[3];
                        if (sx < 0 || sx >= 8) continue;
                        uint8_t attr = so[2];
                        if ((attr & 0x20) && bg_color(o, spr, x, y) != 0) continue;
                        uint8_t sc = sprite_px(o, spr, so[1], attr, sx, sy);
                        if (sc == 0) continue;
                        c = pal_entry(o, spr, (uint16_t)(0x10 + (attr & 3) * 4 + sc));
                        break;
                    }
                }
                fb[y * 256 + x] = c;
            }
        }
        if (index) memcpy(index + (size_t)env * 61440, fb, 61440);
        if (rgb) {
            uint8_t *dst = rgb + (size_t)env * 61440 * 3;
            for (int i = 0; i < 61440; ++i) {
                dst[i * 3] = kRgb[fb[i] & 0x3F][0];
                dst[i * 3 + 1] = kRgb[fb[i] & 0x3F][1];
                dst[i * 3 + 2] = kRgb[fb[i] & 0x3F][2];
            }
        }
        if (gray84) {
            /* EXTENSION: exact area resample 256x240 -> 84x84 in integers.
             * x: source column sx covers [21*sx, 21*sx+21), output column ox
             * covers [64*ox, 64*ox+64) (units of 1/21 px); y: source row sy
             * covers [7*sy, 7*sy+7), output row oy covers [20*oy, 20*oy+20).
             * Output = round(sum(luma * overlap_x * overlap_y) / (64*20)). */
            uint8_t *dst = gray84 + (size_t)env * kGrayW * kGrayW;
            for (int oy = 0; oy < 84; ++oy) {
                for (int ox = 0; ox < 84; ++ox) {
                    uint32_t acc = 0;
                    int y0 = (20 * oy) / 7, y1 = (20 * oy + 19) / 7;
                    int x0 = (64 * ox) / 21, x1 = (64 * ox + 63) / 21;
                    for (int sy = y0; sy <= y1; ++sy) {
                        int wy = (7 * sy + 7 < 20 * oy + 20 ? 7 * sy + 7 : 20 * oy + 20) -
                                 (7 * sy > 20 * oy ? 7 * sy : 20 * oy);
                        for (int sx = x0; sx <= x1; ++sx) {
                            int wx = (21 * sx + 21 < 64 * ox + 64 ? 21 * sx + 21 : 64 * ox + 64) -
                                     (21 * sx > 64 * ox ? 21 * sx : 64 * ox);
                            acc += (uint32_t)luma(fb[sy * 256 + sx] & 0x3F) * (uint32_t)(wx * wy);
                        }
                    }
                    dst[oy * 84 + ox] = (uint8_t)((acc + 640) / 1280);
                }
            }
        }
    }
    free(fb);
}

/* ------------------------------------------------------------------------ */
/* Field export.                                                               */
/* ------------------------------------------------------------------------ */
typedef struct { const char *name; int width; size_t off; } field_t;
#define FLD(n, w) {#n, w, offsetof(env_t, n)}
static const field_t kFields[] = {
    FLD(pc, 2), FLD(a, 1), FLD(x, 1), FLD(y, 1), FLD(sp, 1), FLD(p, 1), FLD(cycles, 8),
    FLD(ctrl_shift, 1), FLD(ctrl_count, 1), FLD(ctrl_strobe, 1), FLD(pending_dma, 4),
    FLD(ppu_ctrl, 1), FLD(ppu_mask, 1), FLD(ppu_status, 1), FLD(oam_addr, 1), FLD(nmi_pending, 1),
    FLD(frame_dot, 4), FLD(frame, 8), FLD(v, 2), FLD(t, 2), FLD(fine_x, 1), FLD(w, 1),
    FLD(open_bus, 1), FLD(read_buffer, 1), FLD(scroll_x, 1), FLD(scroll_y, 1),
    FLD(lat_sx, 1), FLD(lat_sy, 1), FLD(lat_ctrl, 1), FLD(snap_sx_start, 1), FLD(snap_sy_start, 1),
    FLD(snap_ctrl_start, 1), FLD(snap_sx_end, 1), FLD(snap_sy_end, 1), FLD(snap_ctrl_end, 1),
    FLD(snap_mask, 1), FLD(prev_x, 4), FLD(prev_time, 4), FLD(reward, 4), FLD(last_reward, 4),
    FLD(done, 1), FLD(last_done, 1), FLD(action, 1), FLD(episode, 4), FLD(status, 4),
    FLD(stat_instructions, 8), FLD(stat_frames, 4), FLD(stat_budget_hits, 4),
    FLD(ram, 2048), FLD(prg_ram, 8192), FLD(nt, 2048), FLD(pal, 32), FLD(oam, 256),
    FLD(snap_oam, 256), FLD(snap_nt, 2048), FLD(snap_pal, 32), FLD(ram_touch, 8),
    FLD(prg_bank, 1), FLD(chr_bank, 1), FLD(snap_chr_bank, 1),
};
#undef FLD

static const field_t *find_field(const char *name) {
    for (size_t i = 0; i < sizeof(kFields) / sizeof(kFields[0]); ++i)
        if (strcmp(kFields[i].name, name) == 0) return &kFields[i];
    return NULL;
}
int oracle_field_width(const char *field) {
    const field_t *f = find_field(field);
    return f ? f->width : -1;
}
int oracle_get_field(const nes_oracle *o, const char *field, void *out) {
    const field_t *f = find_field(field);
    if (!f) return -1;
    uint8_t *dst = out;
    for (uint32_t i = 0; i < o->n; ++i) memcpy(dst + (size_t)i * f->width, (const uint8_t *)&o->env[i] + f->off, f->width);
    return 0;
}
