// nes_v2.cuh -- the 6502 datapath with operand-ready execution entries.
//
// Same semantics as exec_uniform / run_frames in nes_core.cuh (cpu.hpp:378-730,
// kernels.cu:19-104), fewer integer-pipe instructions per emulated
// instruction.  The first datapath kept the ALU pipe busy two thirds of the
// time at the occupancy a 65,536-env batch allows (ncu: 169 ALU-pipe warp
// instructions per warp iteration), much of it unpacking table fields; this
// one spends the pipe on the computation:
//
//  * a 64-byte execution entry per opcode (Entry2) holds every field as an
//    operand the datapath uses directly: byte-permute selectors (PRMT) that
//    pick an index or operand register out of the packed register word,
//    full-word masks, and multipliers for the operand-B and carry-in terms;
//  * masks ANDed with values known to be below 256 share their word with other
//    fields above bit 8 ("dirty" upper bits cost nothing there);
//  * operand B, the carry-in and the shifter are multiply-adds (the FMA pipe,
//    which the integer datapath otherwise leaves idle); the shifter yields a
//    9-bit value with the shifted-out bit at bit 8, like the adder's carry, so
//    one carry extraction serves both units;
//  * the next instruction's three bytes are prefetched one iteration ahead,
//    and with them, per kernel, none, one or two 16-byte quarters of its
//    entry (the fields the next-PC and address stages read first); the rest
//    (ALU, flags, write-back) is loaded at the top of its own iteration, where
//    the address stage hides its latency;
//  * the table is stored quad-major (four 16-byte quarters, each an array over
//    the 256 opcodes), so lanes of one warp loading different opcodes spread
//    over all 32 banks instead of colliding on a 64-byte stride;
//  * the (zp,X) / (zp),Y pointer is two word loads and a funnel shift, so the
//    indirect modes add a handful of instructions, not two routed byte reads.
//
// The header compiles as plain C++ too (the host unit-test build), like
// nes_core.cuh.
#pragma once
#include "nes_core.cuh"

namespace nesle {

// PRMT (byte permute, default mode): result byte n is byte s[4n+2:4n] of the
// eight bytes {x, y}; if bit 4n+3 of s is set, the sign of that byte is
// replicated instead.
NESLE_HD uint32_t prmt(uint32_t x, uint32_t y, uint32_t s) {
#if defined(__CUDA_ARCH__)
    uint32_t d;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(d) : "r"(x), "r"(y), "r"(s));
    return d;
#else
    const uint64_t v = ((uint64_t)y << 32) | x;
    uint32_t r = 0;
    for (uint32_t n = 0; n < 4; ++n) {
        const uint32_t k = (s >> (4 * n)) & 0xFu;
        uint32_t b = (uint32_t)(v >> ((k & 7u) * 8u)) & 0xFFu;
        if (k & 8u) b = (b & 0x80u) ? 0xFFu : 0u;
        r |= b << (8 * n);
    }
    return r;
#endif
}

// ---------------------------------------------------------------------------
// Execution entry v2 (word index: contents).  Words 0-7 are the early half.
//   E_FLAGS  flags (X_*), length at bits 16-17, base cycles at bits 24-27
//   E_SELIDX PRMT selector of the index byte of R (X, Y, SP or zero) | of the
//            (zp,X) pointer offset (X or zero) << 16
//   E_BRVAL  branch value (bit 8 set for non-branches: never taken)
//   E_BRMASK branch flag mask (with bit 8) | SP delta byte << 24 (0x01, 0xFF)
//   E_BASEM  base mask applied to the operand word (0xFF zero page, 0xFFFF absolute)
//   E_ADDK   base increment (1 for stack pulls)
//   E_WRAP   address wrap (0xFF zero page and stack, 0xFFFF otherwise)
//   E_ORV    address OR (0x100 for the stack)
//   E_SELA   PRMT selector of operand A over {R, m | (P|$30) << 8}
//   E_BMUL   operand B multiplier (0, 1, -1): B = m * E_BMUL + E_BADD
//   E_BADD   operand B addend (0, 0xFF; plus 1 where the carry-in is a constant 1)
//   E_CINM   carry-in multiplier (carry-in = C * E_CINM)
//   E_SUMM   adder result mask (0x1FF: the sum with its carry at bit 8)
//   E_LOGIC  AND mask | XOR mask << 8 | shifter mask << 16 (0x1FF, carry at bit 8)
//   E_PMASK  P keep mask | computed mask << 8 | set bits << 16 | from-result mask << 24
//   E_WMASK  register write mask over R = A | X<<8 | Y<<16 | SP<<24
// ---------------------------------------------------------------------------
enum : uint32_t {
    E_FLAGS = 0, E_SELIDX, E_BRVAL, E_BRMASK, E_BASEM, E_ADDK, E_WRAP, E_ORV,
    E_SELA, E_BMUL, E_BADD, E_CINM, E_SUMM, E_LOGIC, E_PMASK, E_WMASK,
};

enum : uint32_t {
    X_ROT = 1u << 0,      // shift rotates through C (bit 0: C & flags & 1 is the rotate-in bit)
    X_SHL = 1u << 1,
    X_RD = 1u << 2,
    X_WM = 1u << 3,
    X_IMM = 1u << 4,
    X_JMP = 1u << 5,
    X_SIDE = 1u << 6,     // JSR RTS RTI BRK JMP(ind) or illegal: the side path
    X_ILLEGAL = 1u << 7,
    X_PAGE = 1u << 8,     // bit 8: ANDed with (base ^ addr) it is the page-cross bit
    X_IND = 1u << 9,
    X_BIT = 1u << 10,
};

struct Entry2 {
    uint32_t w[16];
};
// Quad-major table: q[k][op] holds words 4k..4k+3 of opcode op's entry.
struct alignas(16) EntryQuad {
    uint32_t w[4];
};
struct EntryTable2 {
    EntryQuad q[4][256];
};

namespace dt {
constexpr Entry2 expand2(uint64_t w) {
    Entry2 e{};
    const uint32_t idx = F(w, D_IDX, 2), base = F(w, D_BASE, 2), opa = F(w, D_OPA, 3), unit = F(w, D_UNIT, 3);
    const uint32_t flg = F(w, D_FLG, 2), fcm = F(w, D_FCM, 8);
    const bool bit = F(w, D_BIT, 1), wp = F(w, D_WP, 1), br = F(w, D_BR, 1), illegal = F(w, D_ILLEGAL, 1);
    const bool stack = base == 3;
    uint32_t f = 0;
    f |= F(w, D_ROT, 1) ? X_ROT : 0u;
    f |= unit == U_SHL ? X_SHL : 0u;
    f |= F(w, D_RD, 1) ? X_RD : 0u;
    f |= F(w, D_WM, 1) ? X_WM : 0u;
    f |= F(w, D_IMM, 1) ? X_IMM : 0u;
    f |= F(w, D_JMP, 1) ? X_JMP : 0u;
    f |= (F(w, D_SPECIAL, 1) || illegal) ? X_SIDE : 0u;
    f |= illegal ? X_ILLEGAL : 0u;
    f |= F(w, D_PAGE, 1) ? X_PAGE : 0u;
    f |= base == 2 ? X_IND : 0u;
    f |= bit ? X_BIT : 0u;
    const uint32_t len = illegal ? 1u : F(w, D_LEN, 2) + 1u;
    e.w[E_FLAGS] = f | (len << 16) | (F(w, D_CYC, 3) << 24);
    const uint32_t idx_byte = stack ? 3u : idx == 1 ? 1u : idx == 2 ? 2u : 4u;
    const uint32_t xind_byte = F(w, D_INDX, 1) ? 1u : 4u;
    e.w[E_SELIDX] = (0x4440u | idx_byte) | ((0x4440u | xind_byte) << 16);
    e.w[E_BASEM] = stack || base == 2 ? 0u : base == 0 ? 0xFFu : 0xFFFFu;
    e.w[E_ADDK] = stack && F(w, D_PULL, 1) ? 1u : 0u;
    e.w[E_WRAP] = (stack || F(w, D_ZPW, 1)) ? 0xFFu : 0xFFFFu;
    e.w[E_ORV] = stack ? 0x100u : 0u;
    const uint32_t opa_byte = opa == A_A ? 0u : opa == A_X ? 1u : opa == A_Y ? 2u : opa == A_SP ? 3u
                              : opa == A_M ? 4u : opa == A_PHP ? 5u : 6u;
    e.w[E_SELA] = 0x6660u | opa_byte;
    const bool bm = F(w, D_BM, 1), bx = F(w, D_BX, 1);
    e.w[E_BMUL] = bm ? (bx ? 0xFFFFFFFFu : 1u) : 0u;
    e.w[E_BADD] = (bx ? 0xFFu : 0u) + (F(w, D_CIN1, 1) ? 1u : 0u);
    e.w[E_CINM] = F(w, D_CINC, 1) ? 1u : 0u;
    e.w[E_SUMM] = unit == U_ADD ? 0x1FFu : 0u;
    const bool logic_and = unit == U_AND || unit == U_OR, logic_xor = unit == U_XOR || unit == U_OR;
    const bool shifter = unit == U_SHL || unit == U_SHR;
    e.w[E_LOGIC] = (logic_and ? 0xFFu : 0u) | ((logic_xor ? 0xFFu : 0u) << 8) | ((shifter ? 0x1FFu : 0u) << 16);
    uint32_t comp = flg == F_NZ ? 0x82u : flg == F_NZC ? 0x83u : flg == F_NZCV ? 0xC3u : 0u;
    if (bit) comp = 0xC2u;
    uint32_t keep = 0xFFu & ~comp & ~fcm;
    uint32_t set = F(w, D_FCV, 1) ? fcm : 0u;
    uint32_t from_r = 0;
    if (flg || bit || fcm) set |= 0x20u;  // set_flag forces the unused bit (cpu.hpp:52-59)
    if (wp) { keep = 0; comp = 0; from_r = 0xEFu; set |= 0x20u; }  // PLP: (pulled | $20) & ~$10
    e.w[E_PMASK] = keep | (comp << 8) | (set << 16) | (from_r << 24);
    const uint32_t brmask = br ? (1u << F(w, D_BRF, 3)) : 0u;
    e.w[E_BRVAL] = br ? (F(w, D_BRP, 1) ? brmask : 0u) : 0x100u;
    const uint32_t spd = F(w, D_SPD, 2);
    e.w[E_BRMASK] = (brmask | 0x100u) | ((spd == 1 ? 0xFFu : spd == 2 ? 0x01u : 0u) << 24);
    e.w[E_WMASK] = (F(w, D_WA, 1) ? 0xFFu : 0u) | (F(w, D_WX, 1) ? 0xFF00u : 0u) | (F(w, D_WY, 1) ? 0xFF0000u : 0u) |
              (F(w, D_WSP, 1) ? 0xFF000000u : 0u);
    return e;
}

constexpr EntryTable2 build_entries2() {
    EntryTable2 t{};
    const DecodeTable d = build();
    for (int i = 0; i < 256; ++i) {
        const Entry2 e = expand2(d.e[i]);
        for (int k = 0; k < 4; ++k)
            for (int j = 0; j < 4; ++j) t.q[k][i].w[j] = e.w[4 * k + j];
    }
    return t;
}
}  // namespace dt

constexpr EntryTable2 kEntries2Host = dt::build_entries2();

// Quarters [q0, q1) of opcode op's entry into w[4 * q0 ...].
template <uint32_t q0, uint32_t q1>
NESLE_HD void load_quads(const EntryQuad* table, uint32_t op, uint32_t* w) {
    if constexpr (q1 > q0) {
#pragma unroll
        for (uint32_t q = q0; q < q1; ++q) {
#if defined(__CUDA_ARCH__)
            const uint4 v = reinterpret_cast<const uint4*>(table)[q * 256u + op];
            w[4 * q + 0] = v.x;
            w[4 * q + 1] = v.y;
            w[4 * q + 2] = v.z;
            w[4 * q + 3] = v.w;
#else
            for (uint32_t j = 0; j < 4; ++j) w[4 * q + j] = table[q * 256u + op].w[j];
#endif
        }
    }
}

// Bytes op | b1 << 8 | b2 << 16 (| junk << 24) at `pc` in the shared PRG copy;
// memory-safe for any pc, meaningful when in_prg_window(pc).
NESLE_HD uint32_t fetch_bytes(const Ctx& c, uint32_t pc) {
    const uint32_t* p32 = reinterpret_cast<const uint32_t*>(c.prg);
    const uint32_t wi = (pc & 0x7FFFu) >> 2;
    return NESLE_FUNNEL(p32[wi], p32[wi + 1], pc * 8u);
}

// The same through the bus, only the bytes the opcode uses, in order
// (cpu.hpp:382-392, 566-587): code in RAM, PRG-RAM or I/O space.
NESLE_HD uint32_t fetch_bytes_bus(const Ctx& c, Lane& L) {
    L.pc &= 0xFFFFu;
    const uint32_t op = io_rd(c, L, L.pc);
    const uint32_t len = (c.dec2[op].w[E_FLAGS] >> 16) & 3u;  // quarter 0 holds E_FLAGS
    const uint32_t b1 = len >= 2 ? io_rd(c, L, (L.pc + 1) & 0xFFFF) : 0u;
    const uint32_t b2 = len >= 3 ? io_rd(c, L, (L.pc + 2) & 0xFFFF) : 0u;
    return op | (b1 << 8) | (b2 << 16);
}

// One instruction (bytes `nb`, entry `E`) on the uniform datapath; returns its
// cycles.  On return `nb` holds the next instruction's bytes, `early` the
// first kEarlyQuads quarters of their entry, and `fresh` says whether they are
// valid (prefetched from the PRG window, no NMI due).
// The program counter may exceed $FFFF transiently (pc + length, branch
// targets): such a value is never in the PRG window, so it always goes
// through the loop top, which masks it.
template <bool kSharedRam, uint32_t kEarlyQuads, bool kSameStride = false>
NESLE_HD uint32_t exec_v2(const Ctx& c, Lane& L, uint32_t& nb, uint32_t* early, const Entry2& E, bool& fresh) {
    const uint32_t pc = L.pc, R = L.R, P = L.p, f = E.w[E_FLAGS], bytes = nb;
    const uint32_t b16 = prmt(bytes, 0u, 0x4421u);

    // ---- next PC (flags from the previous instruction), prefetch ----
    const uint32_t seq = pc + ((f >> 16) & 3u);
    const uint32_t target = seq + prmt(bytes, 0u, 0x9991u);  // + sign-extended b1
    const bool taken = ((P ^ E.w[E_BRVAL]) & E.w[E_BRMASK]) == 0u;  // P ^ E_BRVAL < $200: the SP byte drops out
    uint32_t npc = taken ? target : seq;
    npc = (f & X_JMP) ? b16 : npc;
    const uint32_t branch_cyc = taken ? 1u + (((seq ^ target) >> 8) & 1u) : 0u;
    nb = fetch_bytes(c, npc);
    load_quads<0, kEarlyQuads>(c.dec2, nb & 0xFFu, early);

    // ---- effective address ----
    const uint32_t idx = prmt(R, 0u, E.w[E_SELIDX]);
    uint32_t base = b16 & E.w[E_BASEM];
    if (f & X_IND) {
        // The two pointer bytes at zp and zp + 1 (wrapping in the zero page) as
        // two word loads and a funnel shift, from wherever page 0 lives: the
        // slot, or c.ram (interleaved shared row, or the row in place, stride 1).
        const uint32_t zp = ((bytes >> 8) + prmt(R, 0u, E.w[E_SELIDX] >> 16)) & 0xFFu;
        const bool zs = c.zp && c.zpage == 0u;
        const uint32_t* zw = reinterpret_cast<const uint32_t*>(zs ? c.zp : c.ram);
        const uint32_t st = zs ? c.zslots : c.slots;
        const uint32_t w0 = zw[(zp >> 2) * st], w1 = zw[(((zp >> 2) + 1u) & 63u) * st];
        base = NESLE_FUNNEL(w0, w1, zp * 8u) & 0xFFFFu;
    }
    const uint32_t addr = ((base + idx + E.w[E_ADDK]) & E.w[E_WRAP]) | E.w[E_ORV];
    const uint32_t page = (((base ^ addr) & f) >> 8) & 1u;  // X_PAGE is bit 8
    const uint32_t cyc = (f >> 24) + branch_cyc + page;

    // ---- operand ----
    const bool rd = (f & X_RD) != 0, wm = (f & X_WM) != 0;
    const bool is_ram = addr < 0x2000u, is_prg = addr >= c.prg_lo, is_ctrl = addr == 0x4016u;
    // kSameStride (interleaved placement): the zero-page slot and the working
    // copy share the lane stride, so one offset serves both and only the base
    // is selected.
    uint8_t* ram_byte = kSameStride ? ((addr & 0x700u) == 0u ? c.zp : c.ram) + ram_off(c, addr) : ram_ptr(c, addr);
    uint32_t mem;
    if (kSharedRam) {
        const uint8_t* src = is_ram ? ram_byte : c.prg + (addr & 0x7FFF);
        mem = *src;
    } else {
        mem = c.prg[addr & 0x7FFF];
        if (rd && is_ram) mem = *ram_byte;
    }
    // $4016: the marker-form shift register (load_lane); while the strobe is
    // high a read returns the current action's A bit (batch_bus.cuh:110-123).
    uint32_t m = is_ctrl ? (0x40u | ((L.cstrobe ? L.action : L.csr) & 1u)) : mem;
    m = (f & X_IMM) ? ((bytes >> 8) & 0xFFu) : m;
    if (rd && !(is_ram || is_prg || is_ctrl)) m = io_rd(c, L, addr);  // PPU, $4017, PRG-RAM, banked PRG, unmapped
    const uint32_t shifted = L.csr > 1u ? L.csr >> 1 : L.csr;         // batch_bus.cuh:115-121
    L.csr = (rd && is_ctrl && !L.cstrobe) ? shifted : L.csr;

    // ---- ALU ----
    const uint32_t pool = (P | 0x30u) * 256u + m;                 // {m, P|$30, 0, 0}
    const uint32_t opa = prmt(R, pool, E.w[E_SELA]);
    const uint32_t opb = m * E.w[E_BMUL] + E.w[E_BADD];
    const uint32_t sum = opa + opb + (P & 1u) * E.w[E_CINM];
    const uint32_t rotc = f & P & 1u;                              // X_ROT is bit 0
    const uint32_t shl9 = opa * 2u + rotc;                         // result, out bit at 8
    const uint32_t t9 = rotc * 256u + opa;
    const uint32_t shr9 = (t9 * 513u) >> 1;                        // (t9 >> 1) | (t9 & 1) << 8
    const uint32_t sh9 = (f & X_SHL) ? shl9 : shr9;
    const uint32_t lg = E.w[E_LOGIC];
    const uint32_t r9 = (sum & E.w[E_SUMM]) | (opa & m & lg) | ((opa ^ m) & (lg >> 8) & 0xFFu) | (sh9 & (lg >> 16));
    const uint32_t r = r9 & 0xFFu;

    // ---- flags: P = (P & keep) | (computed & comp) | set | (r & from_r) ----
    const uint32_t vbit = ((~(opa ^ opb) & (opa ^ r)) >> 1) & 0x40u;
    const uint32_t nv = (f & X_BIT) ? (m & 0xC0u) : ((r & 0x80u) | vbit);
    const uint32_t computed = nv | (r == 0u ? 0x02u : 0u) | (r9 >> 8);
    const uint32_t pm = E.w[E_PMASK];
    const uint32_t p = (P & pm) | (computed & (pm >> 8) & 0xFFu) | ((pm >> 16) & 0xFFu) | (r & (pm >> 24));

    // ---- memory write ----
    if (wm && is_ram) *ram_byte = (uint8_t)r;
    const bool cw = wm && is_ctrl;  // $4016 strobe (batch_bus.cuh:125-133)
    const bool latch = cw && ((r | L.cstrobe) & 1u);
    L.csr = latch ? L.action : L.csr;
    L.cstrobe = cw ? (r & 1u) : L.cstrobe;
    // The NMI line is clear on entry (the loop top consumes it), and an I/O
    // write ($2000) is the only way this path can raise it.
    bool nmi_clear = true;
    if (wm && !(is_ram || (is_prg && !c.prg_writes) || is_ctrl)) {
        io_wr(c, L, addr, r);
        nmi_clear = !L.nmi;
    }

    // ---- register write-back ----
    L.R = ((R & ~E.w[E_WMASK]) | (prmt(r, 0u, 0u) & E.w[E_WMASK])) + (E.w[E_BRMASK] & 0xFF000000u);
    L.p = p;
    L.pc = npc;
    fresh = in_prg_window(c, npc) && nmi_clear;
    return cyc;
}

// All frames of one env-step on the v2 datapath (run_frames' structure: the
// loop top, NMI entry and bus fetches on the rare path).  kEarlyQuads (0, 1
// or 2) quarters of the next entry are prefetched one iteration ahead, the
// rest loaded at the top of the iteration: prefetching hides a shared-memory
// load behind the current instruction but keeps 4 registers per quarter live
// across the loop, so the best depth depends on the kernel's other register
// pressure and on how much memory latency it already waits for.
template <bool kSharedRam, uint32_t kEarlyQuads, bool kSameStride = false>
NESLE_HD void run_frames_v2(const Ctx& c, Lane& L) {
    uint32_t nb = 0;
    bool fresh = false;
    Entry2 E;  // quarters below kEarlyQuads: prefetched with nb (valid with fresh); the rest per iteration
    for (;;) {
        uint32_t it_cyc = 0;
        if (!fresh || L.pending >= L.horizon || L.instr >= c.max_instr) {
            L.pc &= 0xFFFFu;
            if (!loop_top(c, L)) break;
            if (L.nmi) {
                L.nmi = 0;
                nmi_entry(c, L);
                it_cyc = 7;
                fresh = false;
            }
            if (!fresh) {
                nb = in_prg_window(c, L.pc) ? fetch_bytes(c, L.pc) : fetch_bytes_bus(c, L);
                load_quads<0, kEarlyQuads>(c.dec2, nb & 0xFFu, E.w);
                fresh = true;
            }
        }
        const uint32_t pc = L.pc, op = nb & 0xFFu;
        load_quads<kEarlyQuads, 4>(c.dec2, op, E.w);
        if (E.w[E_FLAGS] & X_SIDE) {
            if (E.w[E_FLAGS] & X_ILLEGAL) {
                // The reference executes `trap` (cpu.hpp:716-720); the env stops instead.
                L.status_word = NESLE_STATUS_ILLEGAL | (op << 16) | pc;
                L.cycles += it_cyc;
                fresh = false;
                continue;
            }
            exec_special(c, L, op, (nb >> 8) & 0xFFu, (nb >> 16) & 0xFFu);
            it_cyc += (E.w[E_FLAGS] >> 24) & 0xFu;
            fresh = in_prg_window(c, L.pc) && !L.nmi;
            if (fresh) {
                nb = fetch_bytes(c, L.pc);
                load_quads<0, kEarlyQuads>(c.dec2, nb & 0xFFu, E.w);
            }
        } else {
            uint32_t next[8];
            it_cyc += exec_v2<kSharedRam, kEarlyQuads, kSameStride>(c, L, nb, next, E, fresh);
            if constexpr (kEarlyQuads > 0) {
#pragma unroll
                for (uint32_t j = 0; j < 4 * kEarlyQuads; ++j) E.w[j] = next[j];
            }
        }
        it_cyc += L.dma;
        L.dma = 0;
        L.cycles += it_cyc;
        L.pending += it_cyc * 3u;
        L.instr++;
        if (op == 0x4C && L.pc == pc) {  // JMP to itself (see run_frames)
            idle_fast_forward(c, L);
            fresh = false;
        }
    }
}

template <bool kSharedRam, uint32_t kEarlyQuads, bool kSameStride = false>
NESLE_HD void run_env_step_v2(const Ctx& c, EnvRecord& rec, uint8_t action, float& reward, uint8_t& done) {
    Lane L;
    load_lane(L, rec, action);
    begin_step(L);
    run_frames_v2<kSharedRam, kEarlyQuads, kSameStride>(c, L);
    reward_done(c, L, reward, done);
    store_lane(L, rec);
}

}  // namespace nesle
