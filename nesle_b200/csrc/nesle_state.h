// nesle_state.h -- device-memory layout of one batch (shared by host and device code).
//
// Per-env scalar state is one 128-byte record (AoS): a lane loads it with eight
// 16-byte vector loads at kernel start and stores it back at exit, so no
// scalar lives in global memory during emulation.  Byte arrays (RAM, PRG-RAM,
// nametables, palette, OAM and their presentation-snapshot copies) are
// env-major [num_envs][bytes] arrays; RAM is exposed unchanged as the
// (N, 2048) observation view.
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
namespace nesle {
#endif

enum {
    kRamBytes = 2048,
    kPrgRamBytes = 8192,
    kNtBytes = 2048,
    kPalBytes = 32,
    kOamBytes = 256,
    kFrameW = 256,
    kFrameH = 240,
    kGray = 84,
};

// Record flags (EnvRecord::flags).
enum {
    kFlagNtDirty = 1,   // nametable written since the last presentation snapshot
    kFlagPalDirty = 2,  // palette written since the last presentation snapshot
    kFlagOamDirty = 4,  // OAM written since the last presentation snapshot
};

// Status word (EnvRecord::status): 0 = healthy.
#define NESLE_STATUS_ILLEGAL 0x80000000u   // bits 16-23 opcode, 0-15 address
#define NESLE_STATUS_STALL 0x40000000u     // an operand load did not complete in time; bits 0-15 address

typedef struct __attribute__((aligned(16))) EnvRecord {
    // CPU (cpp/include/nesle/cpu.hpp:31-40)
    uint16_t pc;
    uint8_t a, x, y, sp, p;
    uint8_t nmi_pending;  // PPU NMI line (hot PPU state)
    uint64_t cycles;      // 8
    // PPU timing (batch_ppu.cuh, PpuHotState)
    uint64_t frame;       // 16
    uint32_t frame_dot;   // 24
    uint8_t ppu_ctrl, ppu_mask, ppu_status, oam_addr;  // 28
    uint16_t v, t;        // 32
    uint8_t fine_x, w, open_bus, read_buffer;          // 36
    uint8_t scroll_x, scroll_y, lat_sx, lat_sy;        // 40
    uint8_t lat_ctrl, snap_sx_start, snap_sy_start, snap_ctrl_start;  // 44
    uint8_t snap_sx_end, snap_sy_end, snap_ctrl_end, snap_mask;       // 48
    uint8_t ctrl_shift, ctrl_count, ctrl_strobe, flags;               // 52
    int32_t prev_x, prev_time;   // 56, 60
    uint32_t pending_dma;        // 64
    uint32_t episode;            // 68
    uint32_t status;             // 72
    uint8_t cpu_nmi_pending, irq_pending, pad0, pad1;  // 76
    uint64_t stat_instructions;  // 80
    uint32_t stat_frames, stat_budget_hits;  // 88, 92
    uint8_t reserved[32];        // 96..127
} EnvRecord;

#ifdef __cplusplus
static_assert(sizeof(EnvRecord) == 128, "EnvRecord must stay 128 bytes");
static_assert(offsetof(EnvRecord, cycles) == 8 && offsetof(EnvRecord, frame) == 16, "layout");
static_assert(offsetof(EnvRecord, prev_x) == 56 && offsetof(EnvRecord, stat_instructions) == 80, "layout");
#endif

// Snapshot bank slot: the scalar part of one FCS save state
// (cpp/include/nesle/fcs.hpp:19-45); byte arrays live in BankArrays.
typedef struct __attribute__((aligned(16))) BankRecord {
    uint16_t pc;
    uint8_t a, x, y, sp, p, ctrl;
    uint64_t cycles;
    uint8_t mask, status, oam_addr, open_bus, read_buffer, fine_x, w, pad;
    uint16_t v, t;
    int32_t prev_x, prev_time;  // reward baselines seeded from the slot's RAM
    uint32_t pad2;
} BankRecord;

#ifdef __cplusplus
static_assert(sizeof(BankRecord) == 48, "BankRecord layout");
#endif

// Saved env state (nesle_save_states / nesle_load_states): one flat blob per
// env, every part 16-byte aligned.
enum {
    kStateRec = 0,                               // EnvRecord
    kStateRam = kStateRec + 128,                 // 2048
    kStatePrgRam = kStateRam + kRamBytes,        // 8192
    kStateNt = kStatePrgRam + kPrgRamBytes,      // 2048
    kStatePal = kStateNt + kNtBytes,             // 32
    kStateOam = kStatePal + kPalBytes,           // 256
    kStateSnapNt = kStateOam + kOamBytes,        // 2048
    kStateSnapPal = kStateSnapNt + kNtBytes,     // 32
    kStateSnapOam = kStateSnapPal + kPalBytes,   // 256
    kStateOut = kStateSnapOam + kOamBytes,       // reward f32, last reward f32, done u8, last done u8,
                                                 // MapperState (4 bytes at +12)
    kStateBytes = kStateOut + 16,                // 15,056
};

// Cartridge boards (iNES mapper numbers).
enum {
    kMapperNrom = 0,   // the reference's only board
    kMapperUxrom = 2,  // 16 KB PRG bank at $8000 selected by writes to $8000-$FFFF; last bank fixed at $C000
    kMapperCnrom = 3,  // 8 KB CHR bank selected by writes to $8000-$FFFF
};

// Bank registers of one env (UxROM, CNROM); zero on every reset.  Writes have
// bus conflicts: the value written is ANDed with the PRG byte at the address.
typedef struct MapperState {
    uint8_t prg_bank;       // UxROM: 16 KB bank at $8000-$BFFF
    uint8_t chr_bank;       // CNROM: 8 KB CHR bank
    uint8_t snap_chr_bank;  // CNROM: chr_bank latched at vblank (the presentation snapshot renders with it)
    uint8_t pad;
} MapperState;

// Done predicates.
enum {
    kDoneSmb = 0,         // reference predicate (cpp/include/nesle/cuda/batch_step.cuh:100-103)
    kDoneRamEq = 1,       // RAM[a] == b
    kDoneFrameLimit = 2,  // frames since reset >= per-episode U[a, b]
};

// Everything a kernel needs, passed by value.
typedef struct BatchView {
    EnvRecord* rec;
    uint8_t* ram;
    uint8_t* prg_ram;
    uint8_t* nt;
    uint8_t* pal;
    uint8_t* oam;
    uint8_t* snap_nt;
    uint8_t* snap_pal;
    uint8_t* snap_oam;
    const uint8_t* actions;
    float* rewards;
    uint8_t* done;
    float* last_rewards;
    uint8_t* last_done;
    uint32_t* fault_count;
    // cartridge
    const uint8_t* prg;  // 32 KB (16 KB images mirrored at upload)
    const uint8_t* chr;  // chr_size bytes or NULL
    uint32_t chr_size;
    uint32_t horizontal;  // nametable arrangement: 0 vertical, 1 horizontal
    uint16_t reset_vector;
    uint16_t pad;
    // snapshot bank
    const BankRecord* bank;
    const uint8_t* bank_ram;
    const uint8_t* bank_prg_ram;
    const uint8_t* bank_nt;
    const uint8_t* bank_pal;
    const uint8_t* bank_oam;
    const uint8_t* env_to_level;
    uint32_t num_levels;
    // sizes and policy
    uint32_t num_envs;
    uint32_t frameskip;
    uint32_t max_instructions;
    uint32_t done_mode, done_a, done_b;
    uint32_t env_offset;
    uint64_t seed;
    // interleaved placements: the step kernel's working copy of RAM, per CTA
    // [512 words][lanes][4 bytes] (NULL otherwise)
    uint8_t* ram_work;
    // cartridge board (kMapper*): bank registers per env, the whole PRG ROM
    // (prg above is the 32 KB window at $8000 at power-on: for UxROM bank 0 and
    // the fixed last bank), bank counts
    MapperState* mstate;
    const uint8_t* prg_rom;
    uint32_t mapper, prg_banks, chr_banks, pad3;
} BatchView;

#ifdef __cplusplus
}  // namespace nesle
#endif
