// nes_core.cuh -- the per-env NES core of the B200 env-step kernel.
//
// One CUDA thread runs one console.  The hot loop is a *uniform datapath*
// 6502: every opcode executes the same instruction stream (fetch, table
// decode, effective address, one memory read, a combined adder/logic/shifter,
// one memory write, register/flag write-back), with the differences between
// opcodes carried as data in a decode table (this file's 32-byte entries for
// the first datapath and the profiled kernel; nes_v2.cuh's 64-byte entries for
// the production kernels).  Lanes of a warp that sit at
// different PCs therefore stay converged through the common path; only I/O
// accesses, NMI entry, PPU event settlement, OAM DMA and the stack-transfer
// instructions (JSR/RTS/RTI/BRK/JMP-indirect) take divergent side paths.
//
// Semantics restate the reference batched kernel (hbofz/NeSLE
// cpp/src/cuda/kernels.cu:19-104 and cpp/include/nesle/cpu.hpp,
// cuda/batch_bus.cuh, cuda/batch_ppu.cuh, cuda/batch_console.hpp,
// cuda/batch_step.cuh); each function names the lines it follows.
//
// Memory: a Ctx says where the env's 2 KB RAM is for the launch.  Either the
// whole row is staged in shared memory in a bank-interleaved layout -- byte
// `a` of the env in slot `s` of a CTA with `S` slots is at
// ((a & 0x7FC) * S + s * 4 + (a & 3)), so slot s always hits bank s % 32 and
// no RAM access of a warp bank-conflicts (small batches) -- or one page (the
// zero page by default) is staged in an interleaved shared-memory slot and the
// rest is used in place: in the env's row, or (the default for large batches,
// e.g. 65,536 envs) in a working copy in global memory interleaved the same
// way, so a warp's accesses to one address are one 128-byte line.  PRG ROM
// (32 KB) and the execution entries are staged once per CTA into shared
// memory in every placement.
//
// The header also compiles as plain C++ (NESLE_HD expands to nothing) so the
// same code can be unit-tested on the CPU against the checker.
#pragma once
#include <stdint.h>
#include <string.h>

#include <initializer_list>

#include "nesle_state.h"

#ifdef __CUDACC__
#define NESLE_HD __host__ __device__ __forceinline__
#else
#define NESLE_HD inline
#endif

namespace nesle {

// ---------------------------------------------------------------------------
// Decode word.
// ---------------------------------------------------------------------------
enum Mode : uint32_t { IMP, ACC, IMM, ZP, ZPX, ZPY, ABS, ABSX, ABSY, INDX, INDY, IND, REL, PUSH, PULL };

// bit positions
enum : uint32_t {
    D_LEN = 4,       // 2 bits: length - 1
    D_IDX = 6,       // 2 bits: 0 none, 1 X, 2 Y
    D_BASE = 8,      // 2 bits: 0 b1 (zero page), 1 b1|b2<<8, 2 indirect, 3 stack
    D_ZPW = 10,      // zero-page wrap
    D_INDX = 11,     // (zp,X): add X to the pointer
    D_IMM = 12,      // operand value is the immediate byte
    D_PULL = 13,     // stack address pre-increments
    D_CYC = 14,      // 3 bits: base cycles
    D_PAGE = 17,     // +1 cycle on page cross
    D_RD = 18,       // reads the memory operand
    D_WM = 19,       // writes the result to memory
    D_OPA = 20,      // 3 bits: 0 A, 1 X, 2 Y, 3 SP, 4 M, 5 zero, 6 P|$30
    D_BM = 23,       // adder B input uses M
    D_BX = 24,       // adder B input xor $FF
    D_CINC = 25,     // adder carry-in = C
    D_CIN1 = 26,     // adder carry-in = 1
    D_UNIT = 27,     // 3 bits: 0 add, 1 and, 2 or, 3 xor, 4 shl, 5 shr
    D_ROT = 30,      // shift rotates through C
    D_WA = 31,       // write A
    D_WX = 32,
    D_WY = 33,
    D_WSP = 34,
    D_WP = 35,       // PLP: P <- (r | $20) & ~$10
    D_SPD = 36,      // 2 bits: 0 none, 1 SP-1, 2 SP+1
    D_FLG = 38,      // 2 bits: 0 none, 1 NZ, 2 NZC, 3 NZCV
    D_BIT = 40,      // BIT: N,V from M, Z from r
    D_FCM = 41,      // 8 bits: constant flag mask (CLC/SEC/...)
    D_FCV = 49,      // constant flag value (set when 1)
    D_BR = 50,       // branch
    D_BRF = 51,      // 3 bits: flag bit position tested
    D_BRP = 54,      // branch taken when flag == this
    D_JMP = 55,      // JMP absolute
    D_SPECIAL = 56,  // JSR RTS RTI BRK JMP(ind): side path
    D_ILLEGAL = 57,
};

enum : uint32_t { U_ADD, U_AND, U_OR, U_XOR, U_SHL, U_SHR };
enum : uint32_t { A_A, A_X, A_Y, A_SP, A_M, A_ZERO, A_PHP };
enum : uint32_t { F_NONE, F_NZ, F_NZC, F_NZCV };

struct DecodeTable {
    uint64_t e[256];
};

namespace dt {
constexpr uint64_t B(uint32_t pos, uint64_t v = 1) { return v << pos; }

constexpr uint64_t mode_bits(Mode m) {
    uint64_t len = 0, idx = 0, base = 0, zpw = 0, indx = 0, imm = 0, pull = 0;
    switch (m) {
        case IMP: case ACC: len = 0; break;
        case IMM: len = 1; imm = 1; break;
        case ZP: len = 1; base = 0; zpw = 1; break;
        case ZPX: len = 1; base = 0; zpw = 1; idx = 1; break;
        case ZPY: len = 1; base = 0; zpw = 1; idx = 2; break;
        case ABS: len = 2; base = 1; break;
        case ABSX: len = 2; base = 1; idx = 1; break;
        case ABSY: len = 2; base = 1; idx = 2; break;
        case INDX: len = 1; base = 2; indx = 1; break;
        case INDY: len = 1; base = 2; idx = 2; break;
        case IND: len = 2; base = 1; break;
        case REL: len = 1; break;
        case PUSH: len = 0; base = 3; break;
        case PULL: len = 0; base = 3; pull = 1; break;
    }
    return uint64_t(m) | B(D_LEN, len) | B(D_IDX, idx) | B(D_BASE, base) | B(D_ZPW, zpw) |
           B(D_INDX, indx) | B(D_IMM, imm) | B(D_PULL, pull);
}

struct Op {
    uint32_t opa = A_ZERO, unit = U_ADD;
    bool bm = false, bx = false, cinc = false, cin1 = false, rot = false;
    bool rd = false, wm = false, wa = false, wx = false, wy = false, wsp = false, wp = false;
    uint32_t spd = 0, flg = F_NONE;
    bool bit = false;
    uint32_t fcm = 0;
    bool fcv = false, br = false, jmp = false, special = false;
    uint32_t brf = 0;
    bool brp = false;
};

constexpr uint64_t pack(Mode m, uint32_t cycles, bool page, const Op& o) {
    uint64_t w = mode_bits(m) | B(D_CYC, cycles) | B(D_PAGE, page ? 1 : 0);
    w |= B(D_RD, o.rd) | B(D_WM, o.wm) | B(D_OPA, o.opa) | B(D_BM, o.bm) | B(D_BX, o.bx);
    w |= B(D_CINC, o.cinc) | B(D_CIN1, o.cin1) | B(D_UNIT, o.unit) | B(D_ROT, o.rot);
    w |= B(D_WA, o.wa) | B(D_WX, o.wx) | B(D_WY, o.wy) | B(D_WSP, o.wsp) | B(D_WP, o.wp);
    w |= B(D_SPD, o.spd) | B(D_FLG, o.flg) | B(D_BIT, o.bit) | B(D_FCM, o.fcm) | B(D_FCV, o.fcv);
    w |= B(D_BR, o.br) | B(D_BRF, o.brf) | B(D_BRP, o.brp) | B(D_JMP, o.jmp) | B(D_SPECIAL, o.special);
    return w;
}

// Operation templates.
constexpr Op load(uint32_t dst) {  // LDA/LDX/LDY: r = M
    Op o; o.rd = true; o.opa = A_ZERO; o.bm = true; o.flg = F_NZ;
    o.wa = dst == 0; o.wx = dst == 1; o.wy = dst == 2; return o;
}
constexpr Op store(uint32_t src) {  // STA/STX/STY: mem <- reg
    Op o; o.wm = true; o.opa = src; return o;
}
constexpr Op logic(uint32_t unit) { Op o; o.rd = true; o.opa = A_A; o.unit = unit; o.wa = true; o.flg = F_NZ; return o; }
constexpr Op adc(bool sub) {
    Op o; o.rd = true; o.opa = A_A; o.bm = true; o.bx = sub; o.cinc = true; o.wa = true; o.flg = F_NZCV; return o;
}
constexpr Op cmp(uint32_t reg) { Op o; o.rd = true; o.opa = reg; o.bm = true; o.bx = true; o.cin1 = true; o.flg = F_NZC; return o; }
constexpr Op bit() { Op o; o.rd = true; o.opa = A_A; o.unit = U_AND; o.bit = true; return o; }
constexpr Op incdec_mem(bool dec) {
    Op o; o.rd = true; o.wm = true; o.opa = A_M; o.bx = dec; o.cin1 = !dec; o.flg = F_NZ; return o;
}
constexpr Op incdec_reg(uint32_t reg, bool dec) {
    Op o; o.opa = reg; o.bx = dec; o.cin1 = !dec; o.flg = F_NZ; o.wx = reg == A_X; o.wy = reg == A_Y; return o;
}
constexpr Op shift(bool right, bool rot, bool acc) {
    Op o; o.unit = right ? U_SHR : U_SHL; o.rot = rot; o.flg = F_NZC;
    if (acc) { o.opa = A_A; o.wa = true; } else { o.opa = A_M; o.rd = true; o.wm = true; }
    return o;
}
constexpr Op transfer(uint32_t src, uint32_t dst, bool flags) {
    Op o; o.opa = src; o.flg = flags ? F_NZ : F_NONE;
    o.wa = dst == A_A; o.wx = dst == A_X; o.wy = dst == A_Y; o.wsp = dst == A_SP; return o;
}
constexpr Op flagop(uint32_t mask, bool set) { Op o; o.fcm = mask; o.fcv = set; return o; }
constexpr Op branch(uint32_t flagpos, bool pol) { Op o; o.br = true; o.brf = flagpos; o.brp = pol; return o; }

constexpr DecodeTable build() {
    DecodeTable t{};
    for (auto& e : t.e) e = B(D_ILLEGAL);
    // group-1 ALU ops: opcode base + {imm 09, zp 05, zpx 15, abs 0D, absx 1D, absy 19, indx 01, indy 11}
    struct G1 { uint32_t base; Op op; };
    const G1 g1[] = {{0x00, logic(U_OR)}, {0x20, logic(U_AND)}, {0x40, logic(U_XOR)}, {0x60, adc(false)},
                     {0xA0, load(0)}, {0xC0, cmp(A_A)}, {0xE0, adc(true)}};
    for (const auto& g : g1) {
        t.e[g.base + 0x09] = pack(IMM, 2, false, g.op);
        t.e[g.base + 0x05] = pack(ZP, 3, false, g.op);
        t.e[g.base + 0x15] = pack(ZPX, 4, false, g.op);
        t.e[g.base + 0x0D] = pack(ABS, 4, false, g.op);
        t.e[g.base + 0x1D] = pack(ABSX, 4, true, g.op);
        t.e[g.base + 0x19] = pack(ABSY, 4, true, g.op);
        t.e[g.base + 0x01] = pack(INDX, 6, false, g.op);
        t.e[g.base + 0x11] = pack(INDY, 5, true, g.op);
    }
    // The immediate forms of the logic ops read b1 (D_IMM); clear D_RD there.
    for (uint32_t b : {0x09u, 0x29u, 0x49u, 0x69u, 0xA9u, 0xC9u, 0xE9u}) t.e[b] &= ~B(D_RD);
    const Op sta = store(A_A);
    t.e[0x85] = pack(ZP, 3, false, sta); t.e[0x95] = pack(ZPX, 4, false, sta);
    t.e[0x8D] = pack(ABS, 4, false, sta); t.e[0x9D] = pack(ABSX, 5, false, sta);
    t.e[0x99] = pack(ABSY, 5, false, sta); t.e[0x81] = pack(INDX, 6, false, sta);
    t.e[0x91] = pack(INDY, 6, false, sta);
    // shifts: acc 0A, zp 06, zpx 16, abs 0E, absx 1E
    struct SH { uint32_t base; bool right, rot; };
    const SH sh[] = {{0x00, false, false}, {0x20, false, true}, {0x40, true, false}, {0x60, true, true}};
    for (const auto& s : sh) {
        t.e[s.base + 0x0A] = pack(ACC, 2, false, shift(s.right, s.rot, true));
        t.e[s.base + 0x06] = pack(ZP, 5, false, shift(s.right, s.rot, false));
        t.e[s.base + 0x16] = pack(ZPX, 6, false, shift(s.right, s.rot, false));
        t.e[s.base + 0x0E] = pack(ABS, 6, false, shift(s.right, s.rot, false));
        t.e[s.base + 0x1E] = pack(ABSX, 7, false, shift(s.right, s.rot, false));
    }
    const Op inc = incdec_mem(false), dec = incdec_mem(true);
    t.e[0xE6] = pack(ZP, 5, false, inc); t.e[0xF6] = pack(ZPX, 6, false, inc);
    t.e[0xEE] = pack(ABS, 6, false, inc); t.e[0xFE] = pack(ABSX, 7, false, inc);
    t.e[0xC6] = pack(ZP, 5, false, dec); t.e[0xD6] = pack(ZPX, 6, false, dec);
    t.e[0xCE] = pack(ABS, 6, false, dec); t.e[0xDE] = pack(ABSX, 7, false, dec);
    const Op ldx = load(1), ldy = load(2);
    t.e[0xA2] = pack(IMM, 2, false, ldx) & ~B(D_RD); t.e[0xA6] = pack(ZP, 3, false, ldx);
    t.e[0xB6] = pack(ZPY, 4, false, ldx); t.e[0xAE] = pack(ABS, 4, false, ldx);
    t.e[0xBE] = pack(ABSY, 4, true, ldx);
    t.e[0xA0] = pack(IMM, 2, false, ldy) & ~B(D_RD); t.e[0xA4] = pack(ZP, 3, false, ldy);
    t.e[0xB4] = pack(ZPX, 4, false, ldy); t.e[0xAC] = pack(ABS, 4, false, ldy);
    t.e[0xBC] = pack(ABSX, 4, true, ldy);
    const Op stx = store(A_X), sty = store(A_Y);
    t.e[0x86] = pack(ZP, 3, false, stx); t.e[0x96] = pack(ZPY, 4, false, stx); t.e[0x8E] = pack(ABS, 4, false, stx);
    t.e[0x84] = pack(ZP, 3, false, sty); t.e[0x94] = pack(ZPX, 4, false, sty); t.e[0x8C] = pack(ABS, 4, false, sty);
    const Op cpx = cmp(A_X), cpy = cmp(A_Y);
    t.e[0xE0] = pack(IMM, 2, false, cpx) & ~B(D_RD); t.e[0xE4] = pack(ZP, 3, false, cpx);
    t.e[0xEC] = pack(ABS, 4, false, cpx);
    t.e[0xC0] = pack(IMM, 2, false, cpy) & ~B(D_RD); t.e[0xC4] = pack(ZP, 3, false, cpy);
    t.e[0xCC] = pack(ABS, 4, false, cpy);
    t.e[0x24] = pack(ZP, 3, false, bit()); t.e[0x2C] = pack(ABS, 4, false, bit());
    Op jmp; jmp.jmp = true;
    t.e[0x4C] = pack(ABS, 3, false, jmp);
    Op special; special.special = true;
    t.e[0x6C] = pack(IND, 5, false, special);
    t.e[0x20] = pack(ABS, 6, false, special);
    t.e[0x60] = pack(IMP, 6, false, special);
    t.e[0x40] = pack(IMP, 6, false, special);
    t.e[0x00] = pack(IMP, 7, false, special);
    // branches: xxy10000, bits 7-6 select N V C Z, bit 5 the value that branches
    const uint32_t flagpos[4] = {7, 6, 0, 1};
    for (uint32_t op = 0x10; op <= 0xF0; op += 0x20)
        t.e[op] = pack(REL, 2, false, branch(flagpos[op >> 6], (op & 0x20) != 0));
    // stack
    Op pha = store(A_A); pha.spd = 1;
    Op php = store(A_PHP); php.spd = 1;
    Op pla = load(0); pla.spd = 2;
    Op plp; plp.rd = true; plp.opa = A_ZERO; plp.bm = true; plp.wp = true; plp.spd = 2;
    t.e[0x48] = pack(PUSH, 3, false, pha); t.e[0x08] = pack(PUSH, 3, false, php);
    t.e[0x68] = pack(PULL, 4, false, pla); t.e[0x28] = pack(PULL, 4, false, plp);
    // flags: C=01 I=04 D=08 V=40
    t.e[0x18] = pack(IMP, 2, false, flagop(0x01, false)); t.e[0x38] = pack(IMP, 2, false, flagop(0x01, true));
    t.e[0x58] = pack(IMP, 2, false, flagop(0x04, false)); t.e[0x78] = pack(IMP, 2, false, flagop(0x04, true));
    t.e[0xB8] = pack(IMP, 2, false, flagop(0x40, false)); t.e[0xD8] = pack(IMP, 2, false, flagop(0x08, false));
    t.e[0xF8] = pack(IMP, 2, false, flagop(0x08, true));
    // register ops
    t.e[0xE8] = pack(IMP, 2, false, incdec_reg(A_X, false)); t.e[0xCA] = pack(IMP, 2, false, incdec_reg(A_X, true));
    t.e[0xC8] = pack(IMP, 2, false, incdec_reg(A_Y, false)); t.e[0x88] = pack(IMP, 2, false, incdec_reg(A_Y, true));
    t.e[0xAA] = pack(IMP, 2, false, transfer(A_A, A_X, true)); t.e[0xA8] = pack(IMP, 2, false, transfer(A_A, A_Y, true));
    t.e[0x8A] = pack(IMP, 2, false, transfer(A_X, A_A, true)); t.e[0x98] = pack(IMP, 2, false, transfer(A_Y, A_A, true));
    t.e[0xBA] = pack(IMP, 2, false, transfer(A_SP, A_X, true)); t.e[0x9A] = pack(IMP, 2, false, transfer(A_X, A_SP, false));
    t.e[0xEA] = pack(IMP, 2, false, Op{});
    return t;
}
}  // namespace dt

constexpr DecodeTable kDecodeHost = dt::build();

// ---------------------------------------------------------------------------
// Execution entry: the 64-bit specification word of each opcode expanded into
// 32 bytes of byte-aligned, ready-to-use masks, so the datapath combines
// operands with AND/OR instead of extracting fields and chaining selects.
//   w0: b0 flags0 (E0_*), b1 flags1 (E1_*), b2 length, b3 base cycles
//   w1: b0 index shift, b1 index mask, b2 (zp,X) add mask, b3 operand-A shift
//   w2: b0 A-from-register mask, b1 A-from-M mask, b2 A-from-P mask, b3 B-from-M mask
//   w3: b0 B xor, b1 carry-in (bit0: from C, bit1: one), b2 adder mask, b3 AND mask
//   w4: b0 XOR mask, b1 shifter mask, b2 P keep mask, b3 P computed mask
//   w5: b0 P set bits, b1 P-from-result mask, b2 branch flag mask, b3 branch value
//   w6: register write mask over R = A | X<<8 | Y<<16 | SP<<24
//   w7: stack-pointer delta added to R (+-1 in the top byte)
// ---------------------------------------------------------------------------
enum : uint32_t {
    E0_RD = 1u << 0, E0_WM = 1u << 1, E0_IMM = 1u << 2, E0_BR = 1u << 3, E0_JMP = 1u << 4,
    E0_SPECIAL = 1u << 5, E0_ILLEGAL = 1u << 6, E0_PAGE = 1u << 7,
    E1_STACK = 1u << 8, E1_PULL = 1u << 9, E1_IND = 1u << 10, E1_ZP = 1u << 11, E1_BIT = 1u << 12,
    E1_SHL = 1u << 13, E1_ROT = 1u << 14,
};

struct Entry {
    uint32_t w[8];
};
struct EntryTable {
    Entry e[256];
};

namespace dt {
constexpr uint32_t F(uint64_t w, uint32_t pos, uint32_t bits) { return (uint32_t)(w >> pos) & ((1u << bits) - 1u); }

constexpr Entry expand(uint64_t w) {
    Entry e{};
    const uint32_t idx = F(w, D_IDX, 2), base = F(w, D_BASE, 2), opa = F(w, D_OPA, 3), unit = F(w, D_UNIT, 3);
    const uint32_t flg = F(w, D_FLG, 2), fcm = F(w, D_FCM, 8);
    const bool bit = F(w, D_BIT, 1), wp = F(w, D_WP, 1), br = F(w, D_BR, 1);
    uint32_t f0 = 0, f1 = 0;
    f0 |= F(w, D_RD, 1) ? E0_RD : 0u;
    f0 |= F(w, D_WM, 1) ? E0_WM : 0u;
    f0 |= F(w, D_IMM, 1) ? E0_IMM : 0u;
    f0 |= br ? E0_BR : 0u;
    f0 |= F(w, D_JMP, 1) ? E0_JMP : 0u;
    f0 |= F(w, D_SPECIAL, 1) ? E0_SPECIAL : 0u;
    f0 |= F(w, D_ILLEGAL, 1) ? E0_ILLEGAL : 0u;
    f0 |= F(w, D_PAGE, 1) ? E0_PAGE : 0u;
    f1 |= base == 3 ? E1_STACK : 0u;
    f1 |= F(w, D_PULL, 1) ? E1_PULL : 0u;
    f1 |= base == 2 ? E1_IND : 0u;
    f1 |= F(w, D_ZPW, 1) ? E1_ZP : 0u;
    f1 |= bit ? E1_BIT : 0u;
    f1 |= unit == U_SHL ? E1_SHL : 0u;
    f1 |= F(w, D_ROT, 1) ? E1_ROT : 0u;
    const uint32_t len = F(w, D_ILLEGAL, 1) ? 1u : F(w, D_LEN, 2) + 1u;
    e.w[0] = f0 | f1 | (len << 16) | (F(w, D_CYC, 3) << 24);
    const uint32_t idx_sh = idx == 1 ? 8u : (idx == 2 ? 16u : 0u);
    const uint32_t opa_sh = opa == A_X ? 8u : opa == A_Y ? 16u : opa == A_SP ? 24u : 0u;
    e.w[1] = idx_sh | ((idx ? 0xFFu : 0u) << 8) | ((F(w, D_INDX, 1) ? 0xFFu : 0u) << 16) | (opa_sh << 24);
    const bool reg = opa <= A_SP;
    e.w[2] = (reg ? 0xFFu : 0u) | ((opa == A_M ? 0xFFu : 0u) << 8) | ((opa == A_PHP ? 0xFFu : 0u) << 16) |
             ((F(w, D_BM, 1) ? 0xFFu : 0u) << 24);
    const uint32_t cin = (F(w, D_CINC, 1) ? 1u : 0u) | (F(w, D_CIN1, 1) ? 2u : 0u);
    const bool logic_and = unit == U_AND || unit == U_OR, logic_xor = unit == U_XOR || unit == U_OR;
    e.w[3] = (F(w, D_BX, 1) ? 0xFFu : 0u) | (cin << 8) | ((unit == U_ADD ? 0xFFu : 0u) << 16) |
             ((logic_and ? 0xFFu : 0u) << 24);
    uint32_t comp = flg == F_NZ ? 0x82u : flg == F_NZC ? 0x83u : flg == F_NZCV ? 0xC3u : 0u;
    if (bit) comp = 0xC2u;
    uint32_t keep = 0xFFu & ~comp & ~fcm;
    uint32_t set = F(w, D_FCV, 1) ? fcm : 0u;
    uint32_t from_r = 0;
    if (flg || bit || fcm) set |= 0x20u;  // set_flag forces the unused bit (cpu.hpp:52-59)
    if (wp) { keep = 0; comp = 0; from_r = 0xEFu; set |= 0x20u; }  // PLP: (pulled | $20) & ~$10
    const bool shifter = unit == U_SHL || unit == U_SHR;
    e.w[4] = (logic_xor ? 0xFFu : 0u) | ((shifter ? 0xFFu : 0u) << 8) | (keep << 16) | (comp << 24);
    const uint32_t brmask = br ? (1u << F(w, D_BRF, 3)) : 0u;
    const uint32_t brval = br ? (F(w, D_BRP, 1) ? brmask : 0u) : 0xFFu;  // 0xFF never matches: not a branch
    e.w[5] = set | (from_r << 8) | (brmask << 16) | (brval << 24);
    e.w[6] = (F(w, D_WA, 1) ? 0xFFu : 0u) | (F(w, D_WX, 1) ? 0xFF00u : 0u) | (F(w, D_WY, 1) ? 0xFF0000u : 0u) |
             (F(w, D_WSP, 1) ? 0xFF000000u : 0u);
    const uint32_t spd = F(w, D_SPD, 2);
    e.w[7] = spd == 1 ? 0xFF000000u : (spd == 2 ? 0x01000000u : 0u);
    return e;
}

constexpr EntryTable build_entries() {
    EntryTable t{};
    const DecodeTable d = build();
    for (int i = 0; i < 256; ++i) t.e[i] = expand(d.e[i]);
    return t;
}
}  // namespace dt

constexpr EntryTable kEntriesHost = dt::build_entries();

NESLE_HD uint32_t byte_of(uint32_t w, uint32_t k) { return (w >> (8 * k)) & 0xFFu; }

NESLE_HD uint32_t dfield(uint64_t d, uint32_t pos, uint32_t bits) {
    return static_cast<uint32_t>(d >> pos) & ((1u << bits) - 1u);
}

// ---------------------------------------------------------------------------
// Counter RNG (SplitMix64 finaliser, Steele/Lea/Flood 2014), keyed exactly as
// nesle_b200.workloads.counter_rand.
// ---------------------------------------------------------------------------
NESLE_HD uint64_t splitmix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
NESLE_HD uint32_t frame_limit(const BatchView& v, uint32_t env, uint32_t episode) {
    uint64_t k = splitmix64(v.seed ^ (2ull << 56));
    k = splitmix64(k ^ (uint64_t)(v.env_offset + env));
    k = splitmix64(k ^ (uint64_t)episode);
    return v.done_a + (uint32_t)(k % (uint64_t)(v.done_b - v.done_a + 1));
}

// Index of the highest set bit (v != 0).
NESLE_HD uint32_t msb_index(uint32_t v) {
#if defined(__CUDA_ARCH__)
    return 31u - (uint32_t)__clz(v);
#else
    return 31u - (uint32_t)__builtin_clz(v);
#endif
}

// ---------------------------------------------------------------------------
// Lane state: every scalar of the env, register-resident during a launch.
// ---------------------------------------------------------------------------
struct Lane {
    uint32_t pc, R, p;  // R = A | X<<8 | Y<<16 | SP<<24
    uint64_t cycles;
    uint64_t frame;
    uint32_t frame_dot, ctrl, mask, status, nmi;
    uint32_t oam_addr, v, t, fine_x, w, open_bus, read_buffer, scroll_x, scroll_y;
    uint32_t lat_sx, lat_sy, lat_ctrl, ssx0, ssy0, sc0, ssx1, ssy1, sc1, smask;
    uint32_t csr, cstrobe, action, flags;  // csr: controller shift register, marker form (load_lane)
    int32_t prev_x, prev_time;
    uint32_t episode, status_word, cpu_nmi, irq;
    uint32_t dma;  // pending OAM-DMA cycles of the current instruction
    // per-launch loop state
    uint32_t pending, horizon, instr, fcomp, fidx;
    uint64_t tot_instr;
    uint32_t tot_frames, budget;
};

NESLE_HD void load_lane(Lane& L, const EnvRecord& r, uint8_t action) {
    L.pc = r.pc; L.p = r.p;
    L.R = (uint32_t)r.a | ((uint32_t)r.x << 8) | ((uint32_t)r.y << 16) | ((uint32_t)r.sp << 24);
    L.cycles = r.cycles; L.frame = r.frame; L.frame_dot = r.frame_dot;
    L.ctrl = r.ppu_ctrl; L.mask = r.ppu_mask; L.status = r.ppu_status; L.nmi = r.nmi_pending;
    L.oam_addr = r.oam_addr; L.v = r.v; L.t = r.t; L.fine_x = r.fine_x; L.w = r.w;
    L.open_bus = r.open_bus; L.read_buffer = r.read_buffer; L.scroll_x = r.scroll_x; L.scroll_y = r.scroll_y;
    L.lat_sx = r.lat_sx; L.lat_sy = r.lat_sy; L.lat_ctrl = r.lat_ctrl;
    L.ssx0 = r.snap_sx_start; L.ssy0 = r.snap_sy_start; L.sc0 = r.snap_ctrl_start;
    L.ssx1 = r.snap_sx_end; L.ssy1 = r.snap_sy_end; L.sc1 = r.snap_ctrl_end; L.smask = r.snap_mask;
    // Controller shift register as one value: the unread bits under a marker
    // bit, so a read is `csr & 1` then `csr >>= 1` while csr > 1, and csr == 1
    // means all 8 bits are read (further reads return 1).  Exact for every state
    // the bus can reach (count <= 8, shift < 2^(8 - count)).  `action` carries
    // the marker for a latch.
    const uint32_t cnt = r.ctrl_count < 8 ? r.ctrl_count : 8u;
    L.csr = (r.ctrl_shift & ((0x100u >> cnt) - 1u)) | (0x100u >> cnt);
    L.cstrobe = r.ctrl_strobe; L.flags = r.flags;
    L.action = (uint32_t)action | 0x100u;
    L.prev_x = r.prev_x; L.prev_time = r.prev_time; L.episode = r.episode; L.status_word = r.status;
    L.cpu_nmi = r.cpu_nmi_pending; L.irq = r.irq_pending; L.dma = r.pending_dma;
}

NESLE_HD void store_lane(const Lane& L, EnvRecord& r) {
    r.pc = (uint16_t)L.pc; r.a = (uint8_t)L.R; r.x = (uint8_t)(L.R >> 8); r.y = (uint8_t)(L.R >> 16);
    r.sp = (uint8_t)(L.R >> 24); r.p = (uint8_t)L.p; r.nmi_pending = (uint8_t)L.nmi;
    r.cycles = L.cycles; r.frame = L.frame; r.frame_dot = L.frame_dot;
    r.ppu_ctrl = (uint8_t)L.ctrl; r.ppu_mask = (uint8_t)L.mask; r.ppu_status = (uint8_t)L.status;
    r.oam_addr = (uint8_t)L.oam_addr; r.v = (uint16_t)L.v; r.t = (uint16_t)L.t;
    r.fine_x = (uint8_t)L.fine_x; r.w = (uint8_t)L.w; r.open_bus = (uint8_t)L.open_bus;
    r.read_buffer = (uint8_t)L.read_buffer; r.scroll_x = (uint8_t)L.scroll_x; r.scroll_y = (uint8_t)L.scroll_y;
    r.lat_sx = (uint8_t)L.lat_sx; r.lat_sy = (uint8_t)L.lat_sy; r.lat_ctrl = (uint8_t)L.lat_ctrl;
    r.snap_sx_start = (uint8_t)L.ssx0; r.snap_sy_start = (uint8_t)L.ssy0; r.snap_ctrl_start = (uint8_t)L.sc0;
    r.snap_sx_end = (uint8_t)L.ssx1; r.snap_sy_end = (uint8_t)L.ssy1; r.snap_ctrl_end = (uint8_t)L.sc1;
    r.snap_mask = (uint8_t)L.smask;
    const uint32_t top = msb_index(L.csr);
    r.ctrl_shift = (uint8_t)(L.csr ^ (1u << top)); r.ctrl_count = (uint8_t)(8u - top);
    r.ctrl_strobe = (uint8_t)L.cstrobe;
    r.flags = (uint8_t)L.flags; r.prev_x = L.prev_x; r.prev_time = L.prev_time;
    r.pending_dma = L.dma; r.episode = L.episode; r.status = L.status_word;
    r.cpu_nmi_pending = (uint8_t)L.cpu_nmi; r.irq_pending = (uint8_t)L.irq;
    r.stat_instructions = L.tot_instr; r.stat_frames = L.tot_frames; r.stat_budget_hits = L.budget;
}

// ---------------------------------------------------------------------------
// Memory context of one lane: RAM slot in the interleaved shared array, the
// shared PRG/decode copies, and the env's rows of the global byte arrays.
// ---------------------------------------------------------------------------
struct EntryQuad;  // nes_v2.cuh

struct Ctx {
    uint8_t* ram;         // &smem_ram[slot * 4]; byte a at ram[(a & 0x7FC) * slots + (a & 3)]
    uint32_t slots;       // RAM slots per CTA (interleave stride / 4)
    uint8_t* zp;          // hybrid placement: the env's page slot in shared memory, else null
    uint32_t zslots;      // lanes per slot row (interleave stride / 4)
    uint32_t zpage;       // RAM page held in the slot: 0x000 (zero page) or 0x100 (stack)
    const uint8_t* prg;   // 32 KB (shared)
    const Entry* dec;     // execution entries (shared)
    const EntryQuad* dec2;  // v2 execution entries, quad-major (shared), when the kernel runs the v2 datapath
    const BatchView* view;
    uint32_t env;
    uint32_t frameskip;   // copies of view fields read on every iteration
    uint32_t max_instr;
    uint8_t* prg_ram;     // env rows in global memory
    uint8_t* nt;
    uint8_t* pal;
    uint8_t* oam;
    // Cartridge board: the PRG addresses the shared 32 KB copy serves
    // ([prg_lo, $FFFF]: $8000 for NROM and CNROM, $C000 for UxROM, whose
    // $8000-$BFFF bank is per env) and whether writes to $8000-$FFFF reach the
    // bus (board registers).  NROM kernels set both as constants.
    uint32_t prg_lo;
    bool prg_writes;
};

NESLE_HD uint32_t ram_off(const Ctx& c, uint32_t a) { return (a & 0x7FCu) * c.slots + (a & 3u); }
// Byte `a` of the env's RAM.  With a page slot (c.zp, hybrid placement) the
// page c.zpage and its mirrors live there, interleaved 4 bytes per lane with a
// row of c.zslots lanes; everything else is at c.ram.
NESLE_HD uint8_t* zp_slot(const Ctx& c, uint32_t a) { return c.zp + (a & 0xFCu) * c.zslots + (a & 3u); }
NESLE_HD bool in_zp_slot(const Ctx& c, uint32_t a) { return c.zp && (a & 0x700u) == c.zpage; }
NESLE_HD uint8_t* ram_ptr(const Ctx& c, uint32_t a) {
    return in_zp_slot(c, a) ? zp_slot(c, a) : c.ram + ram_off(c, a);
}
NESLE_HD uint32_t ram_rd(const Ctx& c, uint32_t a) { return *ram_ptr(c, a); }
NESLE_HD void ram_wr(const Ctx& c, uint32_t a, uint32_t v) { *ram_ptr(c, a) = (uint8_t)v; }

// 16-byte-aligned row copies (every row base is a multiple of 16).
NESLE_HD void copy16(uint8_t* dst, const uint8_t* src) {
#if defined(__CUDA_ARCH__)
    *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
#else
    memcpy(dst, src, 16);
#endif
}
NESLE_HD void store16(uint8_t* dst, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
#if defined(__CUDA_ARCH__)
    *reinterpret_cast<uint4*>(dst) = make_uint4(a, b, c, d);
#else
    const uint32_t w[4] = {a, b, c, d};
    memcpy(dst, w, 16);
#endif
}
NESLE_HD void zero_row(uint8_t* dst, uint32_t n) {
    for (uint32_t i = 0; i < n; i += 16) store16(dst + i, 0, 0, 0, 0);
}
NESLE_HD void copy_row(uint8_t* dst, const uint8_t* src, uint32_t n) {
    for (uint32_t i = 0; i < n; i += 16) copy16(dst + i, src + i);
}

// ---------------------------------------------------------------------------
// PPU memory and registers: batch_bus.cuh:35-103, 156-292.
// ---------------------------------------------------------------------------
NESLE_HD uint32_t mirror_pal(uint32_t a) {
    uint32_t i = a & 0x1F;
    return ((i & 0x13) == 0x10) ? i - 0x10 : i;  // $10/$14/$18/$1C alias $00/$04/$08/$0C
}
NESLE_HD uint32_t mirror_nt(uint32_t horizontal, uint32_t a) {
    uint32_t i = (a - 0x2000u) & 0x0FFFu;
    return horizontal ? ((i & 0x03FFu) | ((i & 0x0800u) >> 1)) : (i & 0x07FFu);
}
// The env's board registers (UxROM, CNROM).
NESLE_HD MapperState& mapper_state(const Ctx& c) { return c.view->mstate[c.env]; }

// CHR byte `a` ($0000-$1FFF) through the board: CNROM selects an 8 KB bank.
NESLE_HD uint32_t chr_rd(const Ctx& c, uint32_t a) {
    const BatchView& v = *c.view;
    if (!v.chr_size) return 0u;
    const uint32_t off = v.mapper == kMapperCnrom ? (uint32_t)mapper_state(c).chr_bank * 8192u : 0u;
    return v.chr[(off + a) % v.chr_size];
}

// PRG byte `a` ($8000-$FFFF) through the board: UxROM's $8000-$BFFF is the
// env's bank of the whole PRG ROM; everything else is in the 32 KB copy.
NESLE_HD uint32_t prg_rd(const Ctx& c, uint32_t a) {
    if (a < c.prg_lo) return c.view->prg_rom[(uint32_t)mapper_state(c).prg_bank * 0x4000u + (a & 0x3FFFu)];
    return c.prg[a & 0x7FFF];
}

// Write to the board register at $8000-$FFFF (bus conflict: the ROM drives the
// data bus too, so the value is ANDed with the PRG byte at that address).
NESLE_HD void board_wr(const Ctx& c, uint32_t a, uint32_t val) {
    const BatchView& v = *c.view;
    if (v.mapper == kMapperNrom) return;
    val &= prg_rd(c, a);
    MapperState& ms = mapper_state(c);
    if (v.mapper == kMapperUxrom) ms.prg_bank = (uint8_t)(val & (v.prg_banks - 1u));
    else ms.chr_bank = (uint8_t)(val & (v.chr_banks - 1u));
}

NESLE_HD uint32_t ppu_mem_rd(const Ctx& c, uint32_t a) {
    a &= 0x3FFF;
    if (a < 0x2000) return chr_rd(c, a);
    if (a < 0x3F00) {
        if (a >= 0x3000) a -= 0x1000;
        return c.nt[mirror_nt(c.view->horizontal, a)];
    }
    return c.pal[mirror_pal(a)];
}
NESLE_HD void ppu_mem_wr(const Ctx& c, Lane& L, uint32_t a, uint32_t v) {
    a &= 0x3FFF;
    if (a < 0x2000) return;
    if (a < 0x3F00) {
        if (a >= 0x3000) a -= 0x1000;
        c.nt[mirror_nt(c.view->horizontal, a)] = (uint8_t)v;
        L.flags |= kFlagNtDirty;
        return;
    }
    c.pal[mirror_pal(a)] = (uint8_t)v;
    L.flags |= kFlagPalDirty;
}

// batch_bus.cuh:135-154: OAM DMA from RAM page & 0x7FF, +513 cycles.
NESLE_HD void oam_dma(const Ctx& c, Lane& L, uint32_t page) {
    const uint32_t base = (page << 8) & 0x7FF;
    if ((L.oam_addr & 0xFF) == 0 && !(c.zp && (base & 0x700u) == c.zpage)) {
        // Aligned destination: assemble 4 RAM bytes (one interleaved smem word
        // each) and store 16 bytes at a time.
        for (uint32_t i = 0; i < 256; i += 16) {
            uint32_t wds[4];
            for (uint32_t k = 0; k < 4; ++k) {
                const uint32_t a = base + i + 4 * k;
                const uint8_t* src = c.ram + (a & 0x7FCu) * c.slots;
                wds[k] = (uint32_t)src[0] | ((uint32_t)src[1] << 8) | ((uint32_t)src[2] << 16) |
                         ((uint32_t)src[3] << 24);
            }
            store16(c.oam + i, wds[0], wds[1], wds[2], wds[3]);
        }
    } else {
        for (uint32_t i = 0; i < 256; ++i) c.oam[(L.oam_addr + i) & 0xFF] = (uint8_t)ram_rd(c, base + i);
    }
    L.flags |= kFlagOamDirty;
    L.dma += 513;
}

// Side-effecting or non-RAM/PRG read: batch_bus.cuh:156-213.
NESLE_HD uint32_t io_rd(const Ctx& c, Lane& L, uint32_t a) {
    if (a < 0x2000) return ram_rd(c, a);
    if (a < 0x4000) {
        const uint32_t reg = a & 7;
        if (reg == 2) {
            const uint32_t val = (L.status & 0xE0) | (L.open_bus & 0x1F);
            L.status &= 0x7F;
            L.nmi = 0;
            L.w = 0;
            L.open_bus = val;
            return val;
        }
        if (reg == 4) return c.oam[L.oam_addr & 0xFF];
        if (reg == 7) {
            const uint32_t pa = L.v & 0x3FFF;
            uint32_t val;
            if (pa >= 0x3F00) {
                val = ppu_mem_rd(c, pa);
                L.read_buffer = ppu_mem_rd(c, pa - 0x1000);
            } else {
                val = L.read_buffer;
                L.read_buffer = ppu_mem_rd(c, pa);
            }
            L.v = (L.v + ((L.ctrl & 0x04) ? 32u : 1u)) & 0xFFFF;
            L.open_bus = val;
            return val;
        }
        return 0;
    }
    if (a == 0x4016) {  // batch_bus.cuh:110-123
        if (L.cstrobe) return 0x40 | (L.action & 1);
        const uint32_t bit = L.csr & 1;
        if (L.csr > 1) L.csr >>= 1;
        return 0x40 | bit;
    }
    if (a == 0x4017) return 0x41;
    if (a >= 0x6000 && a < 0x8000) return c.prg_ram[a - 0x6000];
    if (a >= 0x8000) return prg_rd(c, a);
    return 0;
}

// batch_bus.cuh:215-304.
NESLE_HD void io_wr(const Ctx& c, Lane& L, uint32_t a, uint32_t val) {
    val &= 0xFF;
    if (a < 0x2000) { ram_wr(c, a, val); return; }
    if (a < 0x4000) {
        const uint32_t reg = a & 7;
        if (reg == 0) {
            if ((val & 0x80) && !(L.ctrl & 0x80) && (L.status & 0x80)) L.nmi = 1;
            L.ctrl = val;
            L.t = (L.t & 0xF3FF) | ((val & 3) << 10);
        } else if (reg == 1) {
            L.mask = val;
        } else if (reg == 3) {
            L.oam_addr = val;
        } else if (reg == 4) {
            c.oam[L.oam_addr & 0xFF] = (uint8_t)val;
            L.oam_addr = (L.oam_addr + 1) & 0xFF;
            L.flags |= kFlagOamDirty;
        } else if (reg == 5) {
            if (L.w == 0) {
                L.fine_x = val & 7;
                L.scroll_x = val;
                L.t = (L.t & 0xFFE0) | (val >> 3);
                L.w = 1;
            } else {
                L.scroll_y = val;
                L.t = (L.t & 0x8FFF) | ((val & 7) << 12);
                L.t = (L.t & 0xFC1F) | ((val & 0xF8) << 2);
                L.w = 0;
            }
        } else if (reg == 6) {
            if (L.w == 0) {
                L.t = (L.t & 0x00FF) | ((val & 0x3F) << 8);
                L.w = 1;
            } else {
                L.t = (L.t & 0x7F00) | val;
                L.v = L.t;
                L.w = 0;
            }
        } else if (reg == 7) {
            ppu_mem_wr(c, L, L.v, val);
            L.v = (L.v + ((L.ctrl & 0x04) ? 32u : 1u)) & 0xFFFF;
        }
        L.open_bus = val;
        return;
    }
    if (a == 0x4014) { oam_dma(c, L, val); return; }
    if (a == 0x4016) {  // batch_bus.cuh:125-133
        const uint32_t next = val & 1;
        if (next || L.cstrobe) L.csr = L.action;
        L.cstrobe = next;
        return;
    }
    if (a >= 0x6000 && a < 0x8000) c.prg_ram[a - 0x6000] = (uint8_t)val;
    if (a >= 0x8000) board_wr(c, a, val);
}

// Fast-path predicates: RAM and PRG reads have no side effects; writes to
// RAM are plain stores and writes to $4000-$5FFF except $4014/$4016, and to
// PRG, are ignored by the reference bus.
NESLE_HD bool fast_read(uint32_t a) { return a < 0x2000 || a >= 0x8000; }
NESLE_HD bool fast_write(uint32_t a) { return a < 0x2000; }

NESLE_HD void push8(const Ctx& c, Lane& L, uint32_t v) {
    ram_wr(c, 0x100 | (L.R >> 24), v);
    L.R -= 0x01000000u;
}
NESLE_HD uint32_t pull8(const Ctx& c, Lane& L) {
    L.R += 0x01000000u;
    return ram_rd(c, 0x100 | (L.R >> 24));
}

// cpu.hpp:112-123
NESLE_HD void nmi_entry(const Ctx& c, Lane& L) {
    push8(c, L, L.pc >> 8);
    push8(c, L, L.pc & 0xFF);
    push8(c, L, (L.p & ~0x10u) | 0x20u);
    L.p |= 0x24;
    L.pc = c.prg[0x7FFA] | (c.prg[0x7FFB] << 8);
}

// ---------------------------------------------------------------------------
// Lazy PPU timing: batch_ppu.cuh:15-21,62-73,138-269.
// ---------------------------------------------------------------------------
enum : uint32_t {
    kFrameDots = 341u * 262u,
    kSprite0Dot = 30u * 341u + 1u,
    kVblankDot = 241u * 341u + 1u,
    kPreRenderDot = 261u * 341u + 1u,
};

NESLE_HD uint32_t dist_to(uint32_t cur, uint32_t ev) { return ev > cur ? ev - cur : kFrameDots - cur + ev; }

NESLE_HD uint32_t next_event(const Lane& L) {  // batch_ppu.cuh:138-177
    uint32_t n = kFrameDots - L.frame_dot;
    uint32_t d = dist_to(L.frame_dot, kVblankDot);
    n = d < n ? d : n;
    d = dist_to(L.frame_dot, kPreRenderDot);
    n = d < n ? d : n;
    if (L.mask & 0x18) {
        d = dist_to(L.frame_dot, kSprite0Dot);
        n = d < n ? d : n;
    }
    return n;
}



// Vblank presentation snapshot (batch_ppu.cuh:223-249).  Byte arrays are
// copied only when written since the last snapshot (the copy would otherwise
// reproduce identical bytes).
NESLE_HD void presentation_snapshot(const Ctx& c, Lane& L) {
    L.ssx0 = L.lat_sx; L.ssy0 = L.lat_sy; L.sc0 = L.lat_ctrl;
    L.ssx1 = L.scroll_x; L.ssy1 = L.scroll_y; L.sc1 = L.ctrl; L.smask = L.mask;
    const BatchView& v = *c.view;
    const size_t e = c.env;
    if (L.flags & kFlagOamDirty) copy_row(v.snap_oam + e * kOamBytes, c.oam, kOamBytes);
    if (L.flags & kFlagNtDirty) copy_row(v.snap_nt + e * kNtBytes, c.nt, kNtBytes);
    if (L.flags & kFlagPalDirty) copy_row(v.snap_pal + e * kPalBytes, c.pal, kPalBytes);
    L.flags &= ~(uint32_t)(kFlagOamDirty | kFlagNtDirty | kFlagPalDirty);
    if (v.mapper == kMapperCnrom) {
        MapperState& ms = mapper_state(c);
        ms.snap_chr_bank = ms.chr_bank;
    }
}

// batch_ppu.cuh:183-269; returns frames completed.
NESLE_HD uint32_t settle(const Ctx& c, Lane& L, uint32_t dots) {
    const uint32_t start = L.frame_dot, end = start + dots;
    const uint32_t frames = end / kFrameDots;
    for (uint32_t f = 0; f <= frames; ++f) {
        const uint32_t o = f * kFrameDots;
        if (o + kSprite0Dot > start && o + kSprite0Dot <= end && (L.mask & 0x18)) L.status |= 0x40;
        if (o + kVblankDot > start && o + kVblankDot <= end) {
            const bool was = (L.status & 0x80) != 0;
            L.status |= 0x80;
            if (!was && (L.ctrl & 0x80)) L.nmi = 1;
            presentation_snapshot(c, L);
        }
        if (o + kPreRenderDot > start && o + kPreRenderDot <= end) {
            L.status &= 0x1F;  // vblank, sprite-0 and overflow cleared
            L.nmi = 0;
            L.lat_sx = L.scroll_x; L.lat_sy = L.scroll_y; L.lat_ctrl = L.ctrl;
        }
    }
    L.frame_dot = end % kFrameDots;
    L.frame += frames;
    return frames;
}

// ---------------------------------------------------------------------------
// Side path: instructions with several stack/bus transfers (cpu.hpp:586,
// 666-694): JMP (ind), JSR, RTS, RTI, BRK.  `b1`,`b2` are the operand bytes.
// ---------------------------------------------------------------------------
NESLE_HD void exec_special(const Ctx& c, Lane& L, uint32_t op, uint32_t b1, uint32_t b2) {
    const uint32_t b16 = b1 | (b2 << 8);
    switch (op) {
        case 0x6C: {  // JMP (ind) with the page-wrap fetch bug
            const uint32_t lo = io_rd(c, L, b16);
            const uint32_t hi = io_rd(c, L, (b16 & 0xFF00) | ((b16 + 1) & 0xFF));
            L.pc = lo | (hi << 8);
            break;
        }
        case 0x20: {  // JSR
            const uint32_t ret = (L.pc + 2) & 0xFFFF;
            push8(c, L, ret >> 8);
            push8(c, L, ret & 0xFF);
            L.pc = b16;
            break;
        }
        case 0x60: {  // RTS
            const uint32_t lo = pull8(c, L), hi = pull8(c, L);
            L.pc = ((lo | (hi << 8)) + 1) & 0xFFFF;
            break;
        }
        case 0x40: {  // RTI
            L.p = (pull8(c, L) | 0x20) & ~0x10u;
            const uint32_t lo = pull8(c, L), hi = pull8(c, L);
            L.pc = lo | (hi << 8);
            break;
        }
        default: {  // BRK
            const uint32_t ret = (L.pc + 2) & 0xFFFF;
            push8(c, L, ret >> 8);
            push8(c, L, ret & 0xFF);
            push8(c, L, L.p | 0x30);
            L.p |= 0x24;
            L.pc = io_rd(c, L, 0xFFFE) | (io_rd(c, L, 0xFFFF) << 8);
            break;
        }
    }
}



#if defined(__CUDA_ARCH__)
#define NESLE_FUNNEL(lo, hi, s) __funnelshift_r((lo), (hi), (s))
#else
#define NESLE_FUNNEL(lo, hi, s) ((uint32_t)((((uint64_t)(hi) << 32) | (lo)) >> ((s) & 31)))
#endif

// ---------------------------------------------------------------------------
// Instruction fetch.  The instruction at the next PC is fetched and decoded
// while the current one executes (its PC is known before its data path runs:
// flags for branches come from the previous instruction).  PRG ROM cannot be
// written, so a fetch from the shared PRG window is exact whenever it happens;
// every other fetch goes through the bus when the instruction starts.
// ---------------------------------------------------------------------------
struct Fetched {
    uint32_t op, b1, b2;
    Entry e;
};

// pc is in the shared PRG copy with two bytes after it ($FFFE-$FFFF start
// instructions through the bus).
NESLE_HD bool in_prg_window(const Ctx& c, uint32_t pc) { return pc - c.prg_lo <= 0xFFFDu - c.prg_lo; }

NESLE_HD void load_entry(const Ctx& c, uint32_t op, Entry& e) {
#if defined(__CUDA_ARCH__)
    const uint4* src = reinterpret_cast<const uint4*>(&c.dec[op]);
    const uint4 a = src[0], b = src[1];
    e.w[0] = a.x; e.w[1] = a.y; e.w[2] = a.z; e.w[3] = a.w;
    e.w[4] = b.x; e.w[5] = b.y; e.w[6] = b.z; e.w[7] = b.w;
#else
    e = c.dec[op];
#endif
}

// Memory-safe for any pc (the shared PRG copy carries one padding word);
// meaningful only when in_prg_window(pc).
NESLE_HD void fetch_prg(const Ctx& c, uint32_t pc, Fetched& f) {
    const uint32_t wi = (pc & 0x7FFF) >> 2;
    const uint32_t* p32 = reinterpret_cast<const uint32_t*>(c.prg);
    const uint32_t bytes = NESLE_FUNNEL(p32[wi], p32[wi + 1], (pc & 3) * 8);
    f.op = bytes & 0xFF;
    f.b1 = (bytes >> 8) & 0xFF;
    f.b2 = (bytes >> 16) & 0xFF;
    load_entry(c, f.op, f.e);
}

// Fetch through the bus, only the bytes the opcode uses, in order
// (cpu.hpp:382-392, 566-587): code in RAM, PRG-RAM or I/O space.
NESLE_HD void fetch_bus(const Ctx& c, Lane& L, Fetched& f) {
    f.op = io_rd(c, L, L.pc);
    load_entry(c, f.op, f.e);
    const uint32_t len = byte_of(f.e.w[0], 2);  // 1 for illegal opcodes
    f.b1 = len >= 2 ? io_rd(c, L, (L.pc + 1) & 0xFFFF) : 0u;
    f.b2 = len >= 3 ? io_rd(c, L, (L.pc + 2) & 0xFFFF) : 0u;
}

// ---------------------------------------------------------------------------
// One instruction on the uniform datapath: cpu.hpp:378-730 restated as data
// flow over the opcode's execution entry.  Straight-line except for the rare
// I/O side paths; shared-memory loads are unconditional where cheap and
// results are merged with table masks, so lanes at different opcodes stay
// converged.  Returns the instruction's cycles; on return `f` holds the next
// instruction and `fresh` says whether it is valid.
// kSharedRam: the env's RAM sits in the interleaved shared-memory slot;
// otherwise it is the env's row in global memory and loads are predicated.
// ---------------------------------------------------------------------------
// Effective address of instruction `f` with the lane's current registers
// (cpu.hpp:378-587 addressing modes); `page` gets the page-cross cycle.
// Indirect pointers are read from RAM here (the zero-page slot in the hybrid
// placement).
template <bool kSharedRam>
NESLE_HD uint32_t effective_address(const Ctx& c, const Lane& L, const Fetched& f, uint32_t& page) {
    const uint32_t R = L.R, w0 = f.e.w[0], w1 = f.e.w[1];
    const uint32_t b16 = f.b1 | (f.b2 << 8);
    const uint32_t idx = (R >> byte_of(w1, 0)) & byte_of(w1, 1);
    const uint32_t zp = (f.b1 + ((R >> 8) & byte_of(w1, 2))) & 0xFF;
    const bool ind = (w0 & E1_IND) != 0;
    uint32_t ptr = 0;
    if (kSharedRam || ind) ptr = ram_rd(c, zp) | (ram_rd(c, (zp + 1) & 0xFF) << 8);
    const uint32_t wrap = (w0 & E1_ZP) ? 0xFFu : 0xFFFFu;
    const uint32_t base = ind ? ptr : (b16 & wrap);
    const uint32_t addr = (base + idx) & wrap;
    page = ((w0 & E0_PAGE) && ((base ^ addr) & 0xFF00u)) ? 1u : 0u;
    return (w0 & E1_STACK) ? (0x100u | (((R >> 24) + ((w0 >> 9) & 1u)) & 0xFFu)) : addr;
}

// The instruction at effective address `addr` (page-cross cycle `page`).
// kAsync: a RAM operand outside the zero-page slot was loaded ahead into
// `ahead_byte` when `ahead`.
template <bool kSharedRam, bool kAsync>
NESLE_HD uint32_t exec_at(const Ctx& c, Lane& L, Fetched& f, bool& fresh, uint32_t addr, uint32_t page,
                          bool ahead, uint32_t ahead_byte) {
    const uint32_t pc = L.pc, b1 = f.b1, b2 = f.b2, R = L.R, P = L.p;
    const uint32_t w0 = f.e.w[0], w1 = f.e.w[1], w2 = f.e.w[2], w3 = f.e.w[3], w4 = f.e.w[4], w5 = f.e.w[5];
    const uint32_t wmask = f.e.w[6], spd = f.e.w[7];
    const uint32_t b16 = b1 | (b2 << 8);
    (void)w1;

    // ---- next PC (flags from the previous instruction), then prefetch it ----
    const uint32_t seq = (pc + byte_of(w0, 2)) & 0xFFFF;
    const uint32_t target = (seq + (uint32_t)(int32_t)(int8_t)b1) & 0xFFFF;
    const bool taken = (P & byte_of(w5, 2)) == byte_of(w5, 3);
    uint32_t npc = taken ? target : seq;
    npc = (w0 & E0_JMP) ? b16 : npc;
    uint32_t cyc = byte_of(w0, 3) + (taken ? 1u + (((seq ^ target) & 0xFF00u) ? 1u : 0u) : 0u) + page;
    Fetched nf;
    fetch_prg(c, npc, nf);

    // ---- operand read: RAM/PRG from fast memory, $4016/$4017 and the
    //      unmapped $4000-$5FFF reads inline, PPU registers and PRG-RAM aside ----
    const bool rd = (w0 & E0_RD) != 0, wm = (w0 & E0_WM) != 0;
    const bool is_ram = addr < 0x2000u, is_prg = addr >= c.prg_lo, is_ctrl = addr == 0x4016u;
    const bool banked = addr >= 0x8000u && !is_prg;  // UxROM's switchable bank: through the bus
    // Hybrid placement: ram_ptr points into the zero-page slot or the row, and
    // the operand is one (generic) access either way.
    uint8_t* ram_byte = ram_ptr(c, addr);
    uint32_t mem;
    if (kSharedRam) {
        const uint8_t* src = is_ram ? ram_byte : c.prg + (addr & 0x7FFF);
        mem = *src;
    } else if (kAsync) {
        mem = c.prg[addr & 0x7FFF];
        if (rd && is_ram) mem = ahead ? ahead_byte : (uint32_t)*ram_byte;
    } else {
        mem = c.prg[addr & 0x7FFF];
        if (rd && is_ram) mem = *ram_byte;
    }
    const uint32_t cbit = (L.cstrobe ? L.action : L.csr) & 1u;
    uint32_t m = (is_ram || is_prg) ? mem : (is_ctrl ? (0x40u | cbit) : (addr == 0x4017u ? 0x41u : 0u));
    m = (w0 & E0_IMM) ? b1 : m;
    const bool io_space = (addr - 0x2000u < 0x2000u) || (addr - 0x6000u < 0x2000u);
    if (rd && (io_space || banked)) m = io_rd(c, L, addr);
    const bool shift_now = rd && is_ctrl && !L.cstrobe && L.csr > 1u;  // batch_bus.cuh:115-121
    L.csr = shift_now ? (L.csr >> 1) : L.csr;

    // ---- ALU: operands and units merged through the entry's masks ----
    const uint32_t opa = ((R >> byte_of(w1, 3)) & byte_of(w2, 0)) | (m & byte_of(w2, 1)) |
                         ((P | 0x30u) & byte_of(w2, 2));
    const uint32_t opb = (m & byte_of(w2, 3)) ^ byte_of(w3, 0);
    const uint32_t cinb = byte_of(w3, 1);
    const uint32_t sum = opa + opb + ((P & cinb & 1u) | (cinb >> 1));
    const uint32_t rotc = (w0 & E1_ROT) ? (P & 1u) : 0u;
    const bool shl = (w0 & E1_SHL) != 0;
    const uint32_t rsh = shl ? (((opa << 1) | rotc) & 0xFFu) : ((opa >> 1) | (rotc << 7));
    const uint32_t csh = shl ? (opa >> 7) : (opa & 1u);
    const uint32_t kadd = byte_of(w3, 2), kand = byte_of(w3, 3), kxor = byte_of(w4, 0), ksh = byte_of(w4, 1);
    const uint32_t r = (sum & kadd) | (opa & m & kand) | ((opa ^ m) & kxor) | (rsh & ksh);
    const uint32_t cout = (((sum >> 8) & kadd) | (csh & ksh)) & 1u;

    // ---- flags: P = (P & keep) | (computed & comp) | set | (r & from_r) ----
    const uint32_t zbit = r == 0 ? 0x02u : 0u;
    const uint32_t vbit = ((~(opa ^ opb) & (opa ^ r)) >> 1) & 0x40u;
    const uint32_t nv = (w0 & E1_BIT) ? (m & 0xC0u) : ((r & 0x80u) | vbit);
    const uint32_t p = (P & byte_of(w4, 2)) | ((nv | zbit | cout) & byte_of(w4, 3)) | byte_of(w5, 0) |
                       (r & byte_of(w5, 1));

    // ---- memory write ----
    if (wm && is_ram) *ram_byte = (uint8_t)r;
    const bool cw = wm && is_ctrl;  // $4016 strobe (batch_bus.cuh:125-133)
    const bool latch = cw && ((r & 1u) || L.cstrobe);
    L.csr = latch ? L.action : L.csr;
    L.cstrobe = cw ? (r & 1u) : L.cstrobe;
    if (wm && (io_space || addr == 0x4014u || (c.prg_writes && addr >= 0x8000u))) io_wr(c, L, addr, r);

    // ---- register write-back ----
    L.R = ((R & ~wmask) | ((r * 0x01010101u) & wmask)) + spd;
    L.p = p;
    L.pc = npc;
    f = nf;
    // The prefetch stays valid after I/O side effects (PRG ROM cannot change);
    // only a pending NMI, which a $2000 write can raise, needs the loop top.
    fresh = in_prg_window(c, npc) && !L.nmi;
    return cyc;
}

template <bool kSharedRam>
NESLE_HD uint32_t exec_uniform(const Ctx& c, Lane& L, Fetched& f, bool& fresh) {
    uint32_t page;
    const uint32_t addr = effective_address<kSharedRam>(c, L, f, page);
    return exec_at<kSharedRam, false>(c, L, f, fresh, addr, page, false, 0u);
}

// ---------------------------------------------------------------------------
// Per-launch loop: kernels.cu:19-104 as a per-lane state machine so a warp can
// keep executing instructions for lanes whose frames end at different times.
// ---------------------------------------------------------------------------
NESLE_HD void frame_end(const Ctx& c, Lane& L) {
    if (L.pending) {
        L.fcomp += settle(c, L, L.pending);
        L.pending = 0;
        L.horizon = next_event(L);
    }
    L.tot_instr += L.instr;
    L.tot_frames += L.fcomp;
    if (L.fcomp == 0 && L.instr >= c.max_instr) L.budget++;
    L.fidx++;
    if (L.status_word) L.fidx = c.frameskip;  // frozen env: no further frames
    L.instr = 0;
    L.fcomp = 0;
}

// Loop-top bookkeeping (kernels.cu:46-56).  Returns false when the lane has
// finished all frames of this step.
NESLE_HD bool loop_top(const Ctx& c, Lane& L) {
    for (;;) {
        if (L.fidx >= c.frameskip) return false;
        if (L.status_word || L.instr >= c.max_instr || L.fcomp != 0) {
            frame_end(c, L);
            continue;
        }
        if (L.pending >= L.horizon) {
            L.fcomp += settle(c, L, L.pending);
            L.pending = 0;
            L.horizon = next_event(L);
            if (L.fcomp) { frame_end(c, L); continue; }
        }
        return true;
    }
}

// JMP-to-self fast-forward (kernels.cu:66-76, batch_console.hpp:129-152).
NESLE_HD void idle_fast_forward(const Ctx& c, Lane& L) {
    L.fcomp += settle(c, L, L.pending);
    L.pending = 0;
    const uint32_t jumps = (next_event(L) + 8u) / 9u;
    if (jumps) {
        L.cycles += (uint64_t)jumps * 3u;
        L.fcomp += settle(c, L, jumps * 9u);
    }
    L.horizon = next_event(L);
}

NESLE_HD void begin_step(Lane& L) {
    L.pending = 0;
    L.horizon = next_event(L);
    L.instr = 0;
    L.fcomp = 0;
    L.fidx = 0;
    L.tot_instr = 0;
    L.tot_frames = 0;
    L.budget = 0;
}

// All frames of one env-step: step_batch_console_instruction_lazy
// (batch_console.hpp:77-109) per iteration, with the loop-top bookkeeping,
// NMI entry and bus fetches on the rare path.
// Instruction histograms (step_profile): a profiler's count(opcode, pc) is
// called once per executed instruction with its opcode and the address it was
// fetched from (kernels.cu:59-64).  NoProfile compiles to nothing.
struct NoProfile {
    NESLE_HD void count(uint32_t, uint32_t) const {}
};

template <bool kSharedRam, class Prof = NoProfile>
NESLE_HD void run_frames(const Ctx& c, Lane& L, const Prof& prof = Prof()) {
    Fetched f{};
    bool fresh = false;
    for (;;) {
        uint32_t it_cyc = 0;
        if (!fresh || L.pending >= L.horizon || L.instr >= c.max_instr) {
            if (!loop_top(c, L)) break;
            if (L.nmi) {
                L.nmi = 0;
                nmi_entry(c, L);
                it_cyc = 7;
                fresh = false;
            }
            if (!fresh) {
                if (in_prg_window(c, L.pc)) fetch_prg(c, L.pc, f);
                else fetch_bus(c, L, f);
                fresh = true;
            }
        }
        const uint32_t pc = L.pc, op = f.op;
        if (f.e.w[0] & (E0_SPECIAL | E0_ILLEGAL)) {
            if (f.e.w[0] & E0_ILLEGAL) {
                // The reference executes `trap` (cpu.hpp:716-720); the env stops instead.
                L.status_word = NESLE_STATUS_ILLEGAL | (op << 16) | pc;
                L.cycles += it_cyc;
                fresh = false;
                continue;
            }
            exec_special(c, L, op, f.b1, f.b2);
            it_cyc += byte_of(f.e.w[0], 3);
            fresh = in_prg_window(c, L.pc) && !L.nmi;
            if (fresh) fetch_prg(c, L.pc, f);
        } else {
            it_cyc += exec_uniform<kSharedRam>(c, L, f, fresh);
        }
        prof.count(op, pc);
        it_cyc += L.dma;
        L.dma = 0;
        L.cycles += it_cyc;
        L.pending += it_cyc * 3u;
        L.instr++;
        // JMP to itself.  The reference also requires that no frame completed
        // in this iteration; that always holds here, because a completed frame
        // sends the next iteration through loop_top before any instruction runs.
        if (op == 0x4C && L.pc == pc) {
            idle_fast_forward(c, L);
            fresh = false;
        }
    }
}

// ---------------------------------------------------------------------------
// Decoupled operand loads (in-place RAM placements).
//
// With RAM rows in global memory a warp's operand load waits for its slowest
// lane, and a lane's RAM line is usually in L2 or DRAM, so every iteration of
// the synchronous loop pays the worst latency of 32 lanes.  Here each lane
// loads the operand of its *next* instruction as soon as its effective address
// is known (at the end of the current instruction) with an asynchronous copy
// into its own shared-memory word that completes on its own barrier.  At the
// top of the next iteration the lane tests that barrier without waiting: a
// lane whose operand has arrived executes, one whose operand is still in
// flight sits the iteration out while the other lanes run.  The lanes of a warp
// therefore no longer wait for each other's memory.
//
// Exactness: the load is issued after every store of the lane's earlier
// instructions (program order), and between the issue and the use the lane
// executes nothing.  Operands in the zero-page slot, PRG ROM, I/O space and
// immediates are read when the instruction executes, as in run_frames.
//
// `Async` provides issue(byte address) / ready(parity) / byte() / drain().
// Two device implementations (kernels.cu): cp.async into a shared-memory word
// with a per-lane mbarrier (lanes idle until their own operand arrives), and a
// plain load into a register issued one iteration ahead (ready() is always
// true: the warp waits at the first use, after the independent start of the
// next iteration).  The host build copies at issue time and reports "not
// ready" on a pseudo-random quarter of tests to exercise the idle path.
// ---------------------------------------------------------------------------
constexpr uint32_t kAsyncSpinLimit = 1u << 22;  // idle iterations one operand may take before the lane stops

// Effective address of `f`; issues its operand load when that operand is a
// RAM byte outside the zero-page slot.  Returns whether a load was issued.
template <class Async>
NESLE_HD bool prepare_operand(const Ctx& c, const Lane& L, const Fetched& f, uint32_t& addr, uint32_t& page,
                              Async& A) {
    addr = effective_address<false>(c, L, f, page);
    const uint32_t w0 = f.e.w[0];
    const bool need = (w0 & E0_RD) && !(w0 & (E0_SPECIAL | E0_ILLEGAL)) && addr < 0x2000u && !in_zp_slot(c, addr);
    if (need) A.issue(c.ram + ram_off(c, addr));
    return need;
}

template <class Async>
NESLE_HD void run_frames_async(const Ctx& c, Lane& L, Async& A) {
    Fetched f{};
    bool fresh = false;
    bool pend = false;      // the current instruction's operand load is issued and not yet consumed
    uint32_t parity = 0;    // phase of the lane's barrier that the pending load completes
    uint32_t addr = 0, page = 0, pre_cyc = 0, spins = 0;
    for (;;) {
        if (!fresh || L.pending >= L.horizon || L.instr >= c.max_instr) {
            if (!loop_top(c, L)) break;
            if (L.nmi) {
                L.nmi = 0;
                nmi_entry(c, L);
                pre_cyc = 7;
                fresh = false;
            }
            if (!fresh) {
                if (in_prg_window(c, L.pc)) fetch_prg(c, L.pc, f);
                else fetch_bus(c, L, f);
                fresh = true;
            }
            pend = prepare_operand(c, L, f, addr, page, A);
        }
        if (pend && !A.ready(parity)) {
            if (++spins >= kAsyncSpinLimit) {  // stop the lane; the step reports it as faulted
                L.status_word = NESLE_STATUS_STALL | addr;
                fresh = false;
            }
            continue;
        }
        uint32_t ahead = 0;
        if (pend) {
            ahead = A.byte();
            parity ^= 1u;
            spins = 0;
        }
        const uint32_t pc = L.pc, op = f.op;
        uint32_t it_cyc = pre_cyc;
        pre_cyc = 0;
        if (f.e.w[0] & (E0_SPECIAL | E0_ILLEGAL)) {
            if (f.e.w[0] & E0_ILLEGAL) {
                // The reference executes `trap` (cpu.hpp:716-720); the env stops instead.
                L.status_word = NESLE_STATUS_ILLEGAL | (op << 16) | pc;
                L.cycles += it_cyc;
                fresh = false;
                pend = false;
                continue;
            }
            exec_special(c, L, op, f.b1, f.b2);
            it_cyc += byte_of(f.e.w[0], 3);
            fresh = in_prg_window(c, L.pc) && !L.nmi;
            if (fresh) fetch_prg(c, L.pc, f);
        } else {
            it_cyc += exec_at<false, true>(c, L, f, fresh, addr, page, pend, ahead);
        }
        pend = false;
        it_cyc += L.dma;
        L.dma = 0;
        L.cycles += it_cyc;
        L.pending += it_cyc * 3u;
        L.instr++;
        if (op == 0x4C && L.pc == pc) {  // JMP to itself (see run_frames)
            idle_fast_forward(c, L);
            fresh = false;
        }
        // The next instruction's operand, unless the next iteration starts at the loop top.
        if (fresh && L.pending < L.horizon && L.instr < c.max_instr) pend = prepare_operand(c, L, f, addr, page, A);
    }
    if (pend) A.drain(parity);
}

// Host stand-in for the asynchronous operand load: the copy happens at issue
// and a deterministic third of the readiness tests say "not yet".
struct HostAsync {
    uint32_t v = 0, state = 0x9E3779B9u;
    NESLE_HD void issue(const uint8_t* src) { v = *src; }
    NESLE_HD bool ready(uint32_t) {
        state = state * 1664525u + 1013904223u;
        return (state >> 30) != 0u;
    }
    NESLE_HD uint32_t byte() const { return v; }
    NESLE_HD void drain(uint32_t) {}
};

// ---------------------------------------------------------------------------
// Reward and done: batch_step.cuh:41-106 plus the configuration predicates.
// ---------------------------------------------------------------------------
NESLE_HD void reward_done(const Ctx& c, Lane& L, float& reward, uint8_t& done) {
    const BatchView& v = *c.view;
    const int x = (int)ram_rd(c, 0x6D) * 0x100 + (int)ram_rd(c, 0x86);
    const int time = (int)(ram_rd(c, 0x7F8) & 0xF) * 100 + (int)(ram_rd(c, 0x7F9) & 0xF) * 10 +
                     (int)(ram_rd(c, 0x7FA) & 0xF);
    const uint32_t ps = ram_rd(c, 0x0E);
    const bool dying = ps == 0x0B || ram_rd(c, 0xB5) > 1;
    const bool dead = ps == 0x06;
    const bool over = ram_rd(c, 0x75A) == 0xFF;
    bool stage_over = false;
    const uint32_t fl = ram_rd(c, 0x1D);
    for (uint32_t i = 0; i < 5; ++i) {
        const uint32_t e = ram_rd(c, 0x16 + i);
        stage_over |= (e == 0x2D || e == 0x31) && fl == 3;
    }
    const bool flag = ram_rd(c, 0x770) == 2 || stage_over;
    int rx = x - L.prev_x;
    if (rx < -5 || rx > 5) rx = 0;
    int rt = time - L.prev_time;
    if (rt > 0) rt = 0;
    reward = (float)(rx + rt + ((dying || dead) ? -25 : 0));
    bool dn = flag || dying || dead || over;
    if (v.done_mode == kDoneRamEq) dn = ram_rd(c, v.done_a & 0x7FF) == (v.done_b & 0xFF);
    else if (v.done_mode == kDoneFrameLimit) dn = L.frame >= frame_limit(v, c.env, L.episode);
    done = dn ? 1 : 0;
    L.prev_x = x;
    L.prev_time = time;
}

// ---------------------------------------------------------------------------
// Resets on global memory: batch_step.cuh:109-242.
// ---------------------------------------------------------------------------
// Byte rows of resets, split over `lanes` cooperating threads (lane `lane`
// takes every lanes-th 16-byte chunk); one thread passes (0, 1).
NESLE_HD void zero_part(uint8_t* dst, uint32_t n, uint32_t lane, uint32_t lanes) {
    for (uint32_t i = lane * 16; i < n; i += lanes * 16) store16(dst + i, 0, 0, 0, 0);
}
NESLE_HD void copy_part(uint8_t* dst, const uint8_t* src, uint32_t n, uint32_t lane, uint32_t lanes) {
    for (uint32_t i = lane * 16; i < n; i += lanes * 16) copy16(dst + i, src + i);
}

// Record part of the power-on reset (batch_step.cuh:109-172).
NESLE_HD void cold_reset_record(const BatchView& v, EnvRecord& r) {
    const uint32_t episode = r.episode;
    memset(&r, 0, sizeof(r));
    r.episode = episode;
    r.pc = v.reset_vector;
    r.sp = 0xFD;
    r.p = 0x24;
    r.cycles = 7;
    r.ctrl_count = 8;
    r.flags = kFlagNtDirty | kFlagPalDirty | kFlagOamDirty;
}

// Record part of the snapshot reset from bank slot env_to_level[env]
// (batch_step.cuh:174-242).
NESLE_HD void warm_reset_record(const BatchView& v, uint32_t env, EnvRecord& r) {
    const BankRecord& s = v.bank[v.env_to_level[env]];
    const uint32_t episode = r.episode;
    memset(&r, 0, sizeof(r));
    r.episode = episode;
    r.pc = s.pc; r.a = s.a; r.x = s.x; r.y = s.y; r.sp = s.sp; r.p = s.p; r.cycles = s.cycles;
    r.ctrl_count = 8;
    r.ppu_ctrl = s.ctrl; r.ppu_mask = s.mask; r.ppu_status = s.status; r.oam_addr = s.oam_addr;
    r.v = s.v; r.t = s.t; r.fine_x = s.fine_x; r.w = s.w; r.open_bus = s.open_bus; r.read_buffer = s.read_buffer;
    r.prev_x = s.prev_x; r.prev_time = s.prev_time;
    r.flags = kFlagNtDirty | kFlagPalDirty | kFlagOamDirty;
}

// Byte rows of the reset: zeroed (power-on) or copied from the bank slot.
NESLE_HD void reset_rows(const BatchView& v, uint32_t env, uint32_t lane, uint32_t lanes) {
    const size_t e = env;
    if (v.num_levels) {
        const size_t lvl = v.env_to_level[env];
        copy_part(v.ram + e * kRamBytes, v.bank_ram + lvl * kRamBytes, kRamBytes, lane, lanes);
        copy_part(v.prg_ram + e * kPrgRamBytes, v.bank_prg_ram + lvl * kPrgRamBytes, kPrgRamBytes, lane, lanes);
        copy_part(v.nt + e * kNtBytes, v.bank_nt + lvl * kNtBytes, kNtBytes, lane, lanes);
        copy_part(v.pal + e * kPalBytes, v.bank_pal + lvl * kPalBytes, kPalBytes, lane, lanes);
        copy_part(v.oam + e * kOamBytes, v.bank_oam + lvl * kOamBytes, kOamBytes, lane, lanes);
    } else {
        zero_part(v.ram + e * kRamBytes, kRamBytes, lane, lanes);
        zero_part(v.prg_ram + e * kPrgRamBytes, kPrgRamBytes, lane, lanes);
        zero_part(v.nt + e * kNtBytes, kNtBytes, lane, lanes);
        zero_part(v.pal + e * kPalBytes, kPalBytes, lane, lanes);
        zero_part(v.oam + e * kOamBytes, kOamBytes, lane, lanes);
    }
}

// The reset kernels of the reference rewrite the console state only: the
// presentation-snapshot scalars and the per-step statistics of the step that
// triggered the reset survive.
NESLE_HD void reset_record(const BatchView& v, uint32_t env, EnvRecord& r) {
    if (v.mstate) {  // board registers reset to bank 0; the CHR bank of the presentation snapshot survives
        v.mstate[env].prg_bank = 0;
        v.mstate[env].chr_bank = 0;
    }
    const EnvRecord keep = r;
    if (v.num_levels) warm_reset_record(v, env, r);
    else cold_reset_record(v, r);
    r.lat_sx = keep.lat_sx; r.lat_sy = keep.lat_sy; r.lat_ctrl = keep.lat_ctrl;
    r.snap_sx_start = keep.snap_sx_start; r.snap_sy_start = keep.snap_sy_start;
    r.snap_ctrl_start = keep.snap_ctrl_start; r.snap_sx_end = keep.snap_sx_end;
    r.snap_sy_end = keep.snap_sy_end; r.snap_ctrl_end = keep.snap_ctrl_end; r.snap_mask = keep.snap_mask;
    r.stat_instructions = keep.stat_instructions;
    r.stat_frames = keep.stat_frames;
    r.stat_budget_hits = keep.stat_budget_hits;
}

// Snapshot (warm) or power-on (cold) reset of one env by one thread.
NESLE_HD void reset_env(const BatchView& v, uint32_t env, EnvRecord& r) {
    reset_record(v, env, r);
    reset_rows(v, env, 0, 1);
}

// cuda_module.cu:1443-1463: presentation snapshot from live state -- the
// record part, then the rows (after the live rows are final).
NESLE_HD void seed_presentation_record(EnvRecord& r) {
    r.snap_mask = r.ppu_mask;
    r.lat_sx = r.snap_sx_start = r.snap_sx_end = r.scroll_x;
    r.lat_sy = r.snap_sy_start = r.snap_sy_end = r.scroll_y;
    r.lat_ctrl = r.snap_ctrl_start = r.snap_ctrl_end = r.ppu_ctrl;
    r.flags &= ~(uint8_t)(kFlagNtDirty | kFlagPalDirty | kFlagOamDirty);
}
NESLE_HD void seed_presentation_rows(const BatchView& v, uint32_t env, uint32_t lane, uint32_t lanes) {
    const size_t e = env;
    copy_part(v.snap_nt + e * kNtBytes, v.nt + e * kNtBytes, kNtBytes, lane, lanes);
    copy_part(v.snap_pal + e * kPalBytes, v.pal + e * kPalBytes, kPalBytes, lane, lanes);
    copy_part(v.snap_oam + e * kOamBytes, v.oam + e * kOamBytes, kOamBytes, lane, lanes);
}
NESLE_HD void seed_presentation_board(const BatchView& v, uint32_t env) {
    if (v.mstate) v.mstate[env].snap_chr_bank = v.mstate[env].chr_bank;
}
NESLE_HD void seed_presentation(const BatchView& v, uint32_t env, EnvRecord& r) {
    seed_presentation_rows(v, env, 0, 1);
    seed_presentation_record(r);
    seed_presentation_board(v, env);
}

// ---------------------------------------------------------------------------
// Whole-step helpers shared by the CUDA kernel and the host unit-test build.
// ---------------------------------------------------------------------------

// Runs env `c.env` for one env-step (frameskip frames).  Its RAM must be
// staged at `c.ram`; `rec` is updated in place.
template <bool kSharedRam = true, class Prof = NoProfile>
NESLE_HD void run_env_step(const Ctx& c, EnvRecord& rec, uint8_t action, float& reward, uint8_t& done,
                           const Prof& prof = Prof()) {
    Lane L;
    load_lane(L, rec, action);
    begin_step(L);
    run_frames<kSharedRam>(c, L, prof);
    reward_done(c, L, reward, done);
    store_lane(L, rec);
}

// The same with the RAM row in place and operands loaded ahead (run_frames_async).
template <class Async>
NESLE_HD void run_env_step_async(const Ctx& c, EnvRecord& rec, uint8_t action, float& reward, uint8_t& done,
                                 Async& A) {
    Lane L;
    load_lane(L, rec, action);
    begin_step(L);
    run_frames_async(c, L, A);
    reward_done(c, L, reward, done);
    store_lane(L, rec);
}

// Outputs and the fused auto-reset of step_device (cuda_module.cu:635-656):
// last_* hold the pre-reset values; the reset clears rewards/done.
// The env's RAM must already be back in global memory.  Returns true when
// the env's status word became non-zero during this step.
NESLE_HD bool finish_env(const BatchView& v, uint32_t env, EnvRecord& rec, uint32_t status_before,
                         float reward, uint8_t done, bool device_api, bool auto_reset) {
    v.rewards[env] = reward;
    v.done[env] = done;
    const bool faulted = rec.status != 0 && status_before == 0;
    if (device_api) {
        v.last_rewards[env] = reward;
        v.last_done[env] = done;
        if (auto_reset && done) {
            rec.episode++;
            reset_env(v, env, rec);
            v.rewards[env] = 0.0f;
            v.done[env] = 0;
        }
    }
    return faulted;
}

}  // namespace nesle
