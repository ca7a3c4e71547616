// core_host.cpp -- host build of the product kernel core, for CPU unit tests.
//
// TEST INFRASTRUCTURE ONLY.  Compiles nesle_b200/csrc/nes_core.cuh and
// nes_render.cuh as plain C++ and drives them exactly as the CUDA kernels do
// (RAM staged in the bank-interleaved slot layout, run_env_step, write-back,
// finish_env), so the core's logic can be compared with the CPU checker
// without a GPU.  The product library never loads this file.
#include <stdlib.h>
#include <string.h>

#include <string>
#include <vector>

#include "../../include/nesle_b200.h"
#include "../../nesle_b200/csrc/formats.h"
#include "../../nesle_b200/csrc/nes_core.cuh"
#include "../../nesle_b200/csrc/nes_render.cuh"
#include "../../nesle_b200/csrc/nes_v2.cuh"

using namespace nesle;

namespace {
thread_local std::string g_err;
constexpr uint32_t kSlots = 4;  // interleave width used by the host harness
const uint8_t kRgb[192] = NESLE_PALETTE_RGB;

struct HostBatch {
    BatchView v{};
    std::vector<EnvRecord> rec;
    std::vector<uint8_t> ram, prg_ram, nt, pal, oam, snap_nt, snap_pal, snap_oam, done, last_done, prg, chr;
    std::vector<float> rewards, last_rewards;
    std::vector<BankRecord> bank;
    std::vector<uint8_t> bram, bprg, bnt, bpal, boam, e2l, prg_rom;
    std::vector<MapperState> mstate;
    uint32_t fault = 0;
    bool global_ram = false;  // run the in-place (global-RAM) variant of the core
    bool hybrid = false;      // ... with one page in a separate slot (hybrid placement)
    bool async = false;       // ... with operands loaded ahead (run_frames_async, HostAsync)
    bool v2 = true;           // the v2 datapath (nes_v2.cuh), as the product's unprofiled kernels
    uint32_t early = 0;       // v2: entry quarters prefetched one iteration ahead (0-2)
    uint32_t slot_page = 0;   // the slot's page: 0x000 or 0x100
    std::vector<uint8_t> smem_ram = std::vector<uint8_t>(kSlots * kRamBytes);
};

int bcd3(const uint8_t* r, int a) { return (r[a] & 0xF) * 100 + (r[a + 1] & 0xF) * 10 + (r[a + 2] & 0xF); }

void stage(HostBatch& h, uint32_t env, uint32_t slot) {
    for (uint32_t a = 0; a < kRamBytes; ++a)
        h.smem_ram[(a & 0x7FC) * kSlots + slot * 4 + (a & 3)] = h.ram[(size_t)env * kRamBytes + a];
}
void unstage(HostBatch& h, uint32_t env, uint32_t slot) {
    for (uint32_t a = 0; a < kRamBytes; ++a)
        h.ram[(size_t)env * kRamBytes + a] = h.smem_ram[(a & 0x7FC) * kSlots + slot * 4 + (a & 3)];
}
}  // namespace

template <bool kSharedRam>
static void step_v2(uint32_t early, const Ctx& c, EnvRecord& rec, uint8_t action, float& reward, uint8_t& done) {
    if (early == 2) run_env_step_v2<kSharedRam, 2>(c, rec, action, reward, done);
    else if (early == 1) run_env_step_v2<kSharedRam, 1>(c, rec, action, reward, done);
    else run_env_step_v2<kSharedRam, 0>(c, rec, action, reward, done);
}

extern "C" {

const char* host_last_error() { return g_err.c_str(); }

int host_create(const nesle_create_args* a, void** out) {
    Cartridge cart;
    std::string err;
    if (!parse_ines(a->rom, a->rom_len, cart, err)) { g_err = err; return NESLE_ERR_INVALID; }
    auto* h = new HostBatch();
    const size_t n = a->num_envs, k = a->num_snapshots;
    h->rec.assign(n, EnvRecord{});
    h->ram.assign(n * kRamBytes, 0); h->prg_ram.assign(n * kPrgRamBytes, 0);
    h->nt.assign(n * kNtBytes, 0); h->pal.assign(n * kPalBytes, 0); h->oam.assign(n * kOamBytes, 0);
    h->snap_nt.assign(n * kNtBytes, 0); h->snap_pal.assign(n * kPalBytes, 0); h->snap_oam.assign(n * kOamBytes, 0);
    h->rewards.assign(n, 0.f); h->last_rewards.assign(n, 0.f); h->done.assign(n, 0); h->last_done.assign(n, 0);
    h->prg.resize(32768 + 16, 0);
    const size_t last = cart.prg.size() - 16384;  // the kernels' window: UxROM bank 0 + fixed last bank
    for (size_t i = 0; i < 32768; ++i)
        h->prg[i] = cart.mapper == kMapperUxrom ? cart.prg[i < 16384 ? i : last + i - 16384] : cart.prg[i % cart.prg.size()];
    h->prg_rom = cart.mapper == kMapperUxrom ? cart.prg : std::vector<uint8_t>(h->prg.begin(), h->prg.begin() + 32768);
    h->mstate.assign(n, MapperState{});
    h->chr = cart.chr;
    h->bank.resize(k ? k : 1);
    h->bram.resize(k * kRamBytes); h->bprg.resize(k * kPrgRamBytes); h->bnt.resize(k * kNtBytes);
    h->bpal.resize(k * kPalBytes); h->boam.resize(k * kOamBytes);
    for (size_t i = 0; i < k; ++i) {
        FcsState s;
        if (!parse_fcs(a->snapshots[i], a->snapshot_lens[i], s, err)) { g_err = err; delete h; return NESLE_ERR_INVALID; }
        BankRecord& r = h->bank[i];
        r = BankRecord{};
        r.pc = s.pc; r.a = s.a; r.x = s.x; r.y = s.y; r.sp = s.sp; r.p = s.p; r.cycles = s.cycles;
        r.ctrl = s.ppu_ctrl; r.mask = s.ppu_mask; r.status = s.ppu_status; r.oam_addr = s.ppu_oam_addr;
        r.open_bus = s.ppu_open_bus; r.read_buffer = s.ppu_read_buffer; r.fine_x = s.ppu_x; r.w = s.ppu_w;
        r.v = s.ppu_v; r.t = s.ppu_t;
        r.prev_x = s.cpu_ram[0x6D] * 0x100 + s.cpu_ram[0x86];
        r.prev_time = bcd3(s.cpu_ram, 0x7F8);
        memcpy(&h->bram[i * kRamBytes], s.cpu_ram, kRamBytes);
        memcpy(&h->bprg[i * kPrgRamBytes], s.prg_ram, kPrgRamBytes);
        memcpy(&h->bnt[i * kNtBytes], s.nametable_ram, kNtBytes);
        memcpy(&h->bpal[i * kPalBytes], s.palette_ram, kPalBytes);
        memcpy(&h->boam[i * kOamBytes], s.oam, kOamBytes);
    }
    h->e2l.assign(n, 0);
    if (a->env_to_level) memcpy(h->e2l.data(), a->env_to_level, n);
    BatchView& v = h->v;
    v.rec = h->rec.data(); v.ram = h->ram.data(); v.prg_ram = h->prg_ram.data(); v.nt = h->nt.data();
    v.pal = h->pal.data(); v.oam = h->oam.data(); v.snap_nt = h->snap_nt.data(); v.snap_pal = h->snap_pal.data();
    v.snap_oam = h->snap_oam.data(); v.rewards = h->rewards.data(); v.done = h->done.data();
    v.last_rewards = h->last_rewards.data(); v.last_done = h->last_done.data(); v.fault_count = &h->fault;
    v.prg = h->prg.data(); v.chr = h->chr.empty() ? nullptr : h->chr.data(); v.chr_size = (uint32_t)h->chr.size();
    v.horizontal = cart.horizontal; v.reset_vector = (uint16_t)(h->prg[0x7FFC] | (h->prg[0x7FFD] << 8));
    v.bank = h->bank.data(); v.bank_ram = h->bram.data(); v.bank_prg_ram = h->bprg.data(); v.bank_nt = h->bnt.data();
    v.bank_pal = h->bpal.data(); v.bank_oam = h->boam.data(); v.env_to_level = h->e2l.data();
    v.num_levels = (uint32_t)k; v.num_envs = (uint32_t)n; v.frameskip = a->frameskip;
    v.max_instructions = a->max_instructions_per_frame ? a->max_instructions_per_frame : 200000u;
    v.done_mode = a->done_mode; v.done_a = a->done_a; v.done_b = a->done_b; v.env_offset = a->env_offset;
    v.seed = a->seed;
    v.mapper = cart.mapper; v.prg_banks = cart.prg_banks; v.chr_banks = cart.chr_banks;
    v.mstate = h->mstate.data(); v.prg_rom = h->prg_rom.data();
    for (uint32_t e = 0; e < n; ++e) {
        EnvRecord& r = h->rec[e];
        r.episode = 0;
        reset_env(v, e, r);
        seed_presentation(v, e, r);
    }
    *out = h;
    return NESLE_OK;
}

void host_destroy(void* p) { delete static_cast<HostBatch*>(p); }

void host_set_global_ram(void* p, int on) {
    auto* h = static_cast<HostBatch*>(p);
    // 1 in place, 2 (3) in place with the zero page (stack page) in a separate slot,
    // 4 (5) in place (hybrid) with operands loaded ahead
    h->global_ram = on != 0;
    h->hybrid = on == 2 || on == 3 || on == 5;
    h->async = on == 4 || on == 5;
    h->slot_page = on == 3 ? 0x100u : 0u;
}

void host_set_v2(void* p, int on) { static_cast<HostBatch*>(p)->v2 = on != 0; }
void host_set_early(void* p, int quads) { static_cast<HostBatch*>(p)->early = (uint32_t)quads; }

void host_reset(void* p) {
    auto* h = static_cast<HostBatch*>(p);
    for (uint32_t e = 0; e < h->v.num_envs; ++e) {
        EnvRecord& r = h->rec[e];
        r.episode = 0;
        reset_env(h->v, e, r);
        h->rewards[e] = 0; h->done[e] = 0;
        seed_presentation(h->v, e, r);
    }
}

void host_reset_envs(void* p, const uint8_t* mask) {
    auto* h = static_cast<HostBatch*>(p);
    for (uint32_t e = 0; e < h->v.num_envs; ++e) {
        if (!mask[e]) continue;
        h->rec[e].episode++;
        reset_env(h->v, e, h->rec[e]);
        h->rewards[e] = 0; h->done[e] = 0;
    }
}

void host_poke_ram(void* p, uint16_t address, uint8_t value) {
    auto* h = static_cast<HostBatch*>(p);
    for (uint32_t e = 0; e < h->v.num_envs; ++e) h->ram[(size_t)e * kRamBytes + (address & 0x7FF)] = value;
}

void host_step(void* p, const uint8_t* actions, int device_api, int auto_reset) {
    auto* h = static_cast<HostBatch*>(p);
    static const EntryTable& dec_table = kEntriesHost;
    static const EntryTable2& dec_table2 = kEntries2Host;
    const Entry* dec = dec_table.e;
    for (uint32_t e = 0; e < h->v.num_envs; ++e) {
        const uint32_t slot = e % kSlots;
        if (!h->global_ram) stage(*h, e, slot);
        Ctx c;
        c.ram = h->global_ram ? h->ram.data() + (size_t)e * kRamBytes : h->smem_ram.data() + slot * 4;
        c.slots = h->global_ram ? 1 : kSlots;
        c.prg = h->prg.data();
        c.dec = dec;
        c.dec2 = &dec_table2.q[0][0];
        c.view = &h->v;
        c.env = e;
        c.frameskip = h->v.frameskip;
        c.max_instr = h->v.max_instructions;
        c.prg_ram = h->v.prg_ram + (size_t)e * kPrgRamBytes;
        c.nt = h->v.nt + (size_t)e * kNtBytes;
        c.pal = h->v.pal + (size_t)e * kPalBytes;
        c.oam = h->v.oam + (size_t)e * kOamBytes;
        c.zp = nullptr;
        c.zslots = 0;
        c.zpage = 0;
        c.prg_lo = h->v.mapper == kMapperUxrom ? 0xC000u : 0x8000u;
        c.prg_writes = h->v.mapper != kMapperNrom;
        uint32_t zp[64];  // hybrid placement: this env's slot page as one lane of words
        if (h->hybrid) {
            c.zpage = h->slot_page;
            memcpy(zp, h->ram.data() + (size_t)e * kRamBytes + c.zpage, 256);
            c.zp = reinterpret_cast<uint8_t*>(zp);
            c.zslots = 1;
        }
        EnvRecord rec = h->rec[e];
        const uint32_t before = rec.status;
        float reward;
        uint8_t done;
        if (h->global_ram) {
            if (h->async) {
                HostAsync A;
                A.state ^= e * 0x85EBCA6Bu;  // a different idle pattern per env
                run_env_step_async(c, rec, actions[e], reward, done, A);
            } else if (h->v2) {
                step_v2<false>(h->early, c, rec, actions[e], reward, done);
            } else {
                run_env_step<false>(c, rec, actions[e], reward, done);
            }
            if (h->hybrid) memcpy(h->ram.data() + (size_t)e * kRamBytes + c.zpage, zp, 256);
        } else {
            if (h->v2) step_v2<true>(h->early, c, rec, actions[e], reward, done);
            else run_env_step<true>(c, rec, actions[e], reward, done);
            unstage(*h, e, slot);
        }
        if (finish_env(h->v, e, rec, before, reward, done, device_api != 0, auto_reset != 0)) h->fault++;
        h->rec[e] = rec;
    }
}

// mode: 0 rgb (N*240*256*3), 1 index (N*240*256), 2 gray84 (N*84*84)
void host_render(void* p, int mode, uint8_t* out) {
    auto* h = static_cast<HostBatch*>(p);
    std::vector<uint8_t> fb(kFrameW * kFrameH), luma(kFrameW * kFrameH);
    for (uint32_t e = 0; e < h->v.num_envs; ++e) {
        const RenderEnv re = render_env(h->v, h->rec[e], e);
        uint8_t res[32];
        resolve_palette(re, res);
        uint16_t spat[64 * 16] = {};
        const uint32_t h = (re.lower.ctrl & 0x20) ? 16 : 8;
        for (uint32_t i = 0; i < 64 * 16; ++i)
            if (i % 16 < h) spat[i] = (uint16_t)sprite_pattern_row(re.lower, i / 16, i % 16);
        uint64_t cols[kFrameW / 8];
        for (uint32_t g = 0; g < kFrameW / 8; ++g) cols[g] = sprite_col_mask(re, g);
        for (uint32_t y = 0; y < kFrameH; ++y) {  // the kernels' path: row tiles, sprite tables, resolved palette
            const uint64_t rows = sprite_row_mask(re, y);
            const RenderView& v = bg_view(re, y);
            uint32_t tiles[kRowTiles];
            for (uint32_t j = 0; j < kRowTiles; ++j) tiles[j] = slot_entry(v, y, j);
            for (uint32_t x = 0; x < kFrameW; ++x) {
                const uint32_t bgc = bg_from_entry_tables(v, res, tiles[tile_slot(v, x)], x, v.sx + x);
                fb[y * kFrameW + x] = (uint8_t)compose_pixel_tables(re, res, x, y, bgc, rows & cols[x >> 3], spat);
            }
        }
        if (mode == 1) {
            memcpy(out + (size_t)e * fb.size(), fb.data(), fb.size());
        } else if (mode == 0) {
            for (size_t i = 0; i < fb.size(); ++i)
                for (int ch = 0; ch < 3; ++ch) out[((size_t)e * fb.size() + i) * 3 + ch] = kRgb[fb[i] * 3 + ch];
        } else {
            for (size_t i = 0; i < fb.size(); ++i)
                luma[i] = (uint8_t)luma_of_rgb(kRgb[fb[i] * 3], kRgb[fb[i] * 3 + 1], kRgb[fb[i] * 3 + 2]);
            for (uint32_t k = 0; k < kFrameH / kGrayStripRows; ++k)
                for (uint32_t oy = k * kGrayStripOut; oy < (k + 1) * kGrayStripOut; ++oy)
                    for (uint32_t ox = 0; ox < kGray; ++ox)
                        out[(size_t)e * kGray * kGray + oy * kGray + ox] =
                            (uint8_t)gray84_pixel(luma.data() + k * kGrayStripRows * kFrameW, k * kGrayStripRows, ox, oy);
        }
    }
}

// Same field names as nesle_copy_field().
int host_copy_field(void* p, const char* name, void* out, uint64_t bytes) {
    auto* h = static_cast<HostBatch*>(p);
    const std::string f = name;
    const uint64_t n = h->v.num_envs;
    struct Arr { const char* name; const void* ptr; uint64_t width; };
    const Arr arrays[] = {
        {"ram", h->ram.data(), kRamBytes}, {"prg_ram", h->prg_ram.data(), kPrgRamBytes},
        {"nametable", h->nt.data(), kNtBytes}, {"palette", h->pal.data(), kPalBytes}, {"oam", h->oam.data(), kOamBytes},
        {"snap_nametable", h->snap_nt.data(), kNtBytes}, {"snap_palette", h->snap_pal.data(), kPalBytes},
        {"snap_oam", h->snap_oam.data(), kOamBytes}, {"rewards", h->rewards.data(), 4}, {"done", h->done.data(), 1},
        {"last_rewards", h->last_rewards.data(), 4}, {"last_done", h->last_done.data(), 1},
    };
    for (const auto& a : arrays) {
        if (f == a.name) {
            if (bytes != n * a.width) { g_err = "wrong size"; return NESLE_ERR_INVALID; }
            memcpy(out, a.ptr, bytes);
            return NESLE_OK;
        }
    }
#define RF(nm, member)                                                                            \
    if (f == nm) {                                                                                \
        const size_t w = sizeof(((EnvRecord*)nullptr)->member);                                   \
        if (bytes != n * w) { g_err = "wrong size"; return NESLE_ERR_INVALID; }                   \
        for (uint64_t e = 0; e < n; ++e) memcpy((uint8_t*)out + e * w, &h->rec[e].member, w);    \
        return NESLE_OK;                                                                          \
    }
    RF("pc", pc) RF("a", a) RF("x", x) RF("y", y) RF("sp", sp) RF("p", p) RF("nmi_pending", nmi_pending)
    RF("cycles", cycles) RF("frame", frame) RF("frame_dot", frame_dot) RF("ppu_ctrl", ppu_ctrl)
    RF("ppu_mask", ppu_mask) RF("ppu_status", ppu_status) RF("oam_addr", oam_addr) RF("v", v) RF("t", t)
    RF("fine_x", fine_x) RF("w", w) RF("open_bus", open_bus) RF("read_buffer", read_buffer)
    RF("scroll_x", scroll_x) RF("scroll_y", scroll_y) RF("lat_sx", lat_sx) RF("lat_sy", lat_sy)
    RF("lat_ctrl", lat_ctrl) RF("snap_sx_start", snap_sx_start) RF("snap_sy_start", snap_sy_start)
    RF("snap_ctrl_start", snap_ctrl_start) RF("snap_sx_end", snap_sx_end) RF("snap_sy_end", snap_sy_end)
    RF("snap_ctrl_end", snap_ctrl_end) RF("snap_mask", snap_mask) RF("ctrl_shift", ctrl_shift)
    RF("ctrl_count", ctrl_count) RF("ctrl_strobe", ctrl_strobe) RF("prev_x", prev_x) RF("prev_time", prev_time)
    RF("pending_dma", pending_dma) RF("episode", episode) RF("status", status)
    RF("stat_instructions", stat_instructions) RF("stat_frames", stat_frames) RF("stat_budget_hits", stat_budget_hits)
#undef RF
    const char* board_fields[] = {"prg_bank", "chr_bank", "snap_chr_bank"};
    for (uint32_t k = 0; k < 3; ++k)
        if (f == board_fields[k]) {
            if (bytes != n) { g_err = "wrong size"; return NESLE_ERR_INVALID; }
            for (uint64_t e = 0; e < n; ++e) static_cast<uint8_t*>(out)[e] = reinterpret_cast<const uint8_t*>(&h->mstate[e])[k];
            return NESLE_OK;
        }
    g_err = "unknown field " + f;
    return NESLE_ERR_INVALID;
}

}  // extern "C"
