// ref_harness.cpp -- drives the UNMODIFIED reference sources on the CPU.
//
// TEST INFRASTRUCTURE ONLY.  Compiled by oracle/Makefile against the
// reference tree (hbofz/NeSLE cpp/include, cpp/src/rom.cpp, cpp/src/smb.cpp)
// into oracle/_ref/libnesle_ref.so.  It exposes two reference paths through a
// small C API so tests can pin the C checker (nes_oracle.c) and bench.py can
// time the reference's CPU path:
//
//  * kind 'B': the reference batched-kernel headers run on host vectors, as
//    the reference's own host tests do (tests/cpp/test_cuda_batch_console.cpp).
//    Only the __global__ loop body of console_step_kernel
//    (cpp/src/cuda/kernels.cu:19-104) and the step_device auto-reset glue
//    (cpp/bindings/cuda_module.cu:594-666) are restated here; every emulation
//    step calls the reference's own functions.
//  * kind 'A': N x nesle::Console, the reference CPU core, stepped the way
//    NativeConsole.step does (cpp/bindings/module.cpp:72-93), with the SMB
//    reward from cpp/src/smb.cpp.  Snapshot resets inject state through the
//    Console/Ppu public API.
//
// The benchmark-configuration done predicates (RAM byte, frame limit) are not
// in the reference; they are applied here after the reference reward exactly
// as the product does.
#include <cstdint>
#include <cstring>
#include <exception>
#include <memory>
#include <span>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "nesle/console.hpp"
#include "nesle/cpu.hpp"
#include "nesle/cuda/batch_console.hpp"
#include "nesle/cuda/batch_render.cuh"
#include "nesle/cuda/batch_step.cuh"
#include "nesle/fcs.hpp"
#include "nesle/rom.hpp"
#include "nesle/smb.hpp"

namespace {

thread_local std::string g_error;

std::uint64_t splitmix64(std::uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

std::uint32_t frame_limit(std::uint64_t seed, std::uint32_t lo, std::uint32_t hi,
                          std::uint64_t env, std::uint64_t episode) {
    std::uint64_t k = splitmix64(seed ^ (2ull << 56));
    k = splitmix64(k ^ env);
    k = splitmix64(k ^ episode);
    return lo + static_cast<std::uint32_t>(k % (hi - lo + 1));
}

struct Config {
    std::uint32_t n = 0, frameskip = 4, done_mode = 0, done_a = 0, done_b = 0, env_offset = 0;
    std::uint64_t seed = 0, max_instr = 200000;
};

// ---------------------------------------------------------------------------
// Kind B: reference batch headers over host vectors.
// ---------------------------------------------------------------------------
struct BatchB {
    Config cfg;
    nesle::RomImage rom;
    std::vector<nesle::fcs::StateSnapshot> snaps;
    template <class T> using V = std::vector<T>;
    V<std::uint16_t> pc, v, t;
    V<std::uint8_t> a, x, y, sp, p, cpu_nmi, irq, ram, prg_ram, shift, count, strobe;
    V<std::uint64_t> cycles, frame;
    V<std::uint32_t> dma, frame_dot;
    V<std::uint8_t> ctrl, mask, status, oam_addr, nmi, fx, w, open_bus, read_buf, sx, sy, nt, pal, oam;
    V<std::uint8_t> lat_sx, lat_sy, lat_ctrl, s_sx0, s_sy0, s_c0, s_sx1, s_sy1, s_c1, s_mask, s_oam, s_nt, s_pal;
    V<std::uint8_t> actions, done, last_done, frames;
    V<float> rewards, last_rewards;
    V<int> prev_x, prev_time;
    V<std::uint32_t> episode, stat_frames, stat_budget;
    V<std::uint64_t> stat_instr;
    // snapshot bank
    V<std::uint8_t> b_ram, b_prg, b_nt, b_pal, b_oam, b_a, b_x, b_y, b_sp, b_p, b_ctrl, b_mask, b_status,
        b_oam_addr, b_open, b_rbuf, b_fx, b_w, env_to_level;
    V<std::uint16_t> b_pc, b_v, b_t;
    V<std::uint64_t> b_cycles;
    nesle::cuda::BatchBuffers buf{};
    nesle::cuda::SnapshotTemplate bank{};
    std::uint64_t* prof_opcode = nullptr;  // kernels.cu:59-64 histograms, when set
    std::uint64_t* prof_pc = nullptr;

    void allocate() {
        const std::size_t n = cfg.n;
        for (auto* vec : {&a, &x, &y, &sp, &p, &cpu_nmi, &irq, &shift, &count, &strobe, &ctrl, &mask, &status,
                          &oam_addr, &nmi, &fx, &w, &open_bus, &read_buf, &sx, &sy, &lat_sx, &lat_sy, &lat_ctrl,
                          &s_sx0, &s_sy0, &s_c0, &s_sx1, &s_sy1, &s_c1, &s_mask, &actions, &done, &last_done})
            vec->assign(n, 0);
        pc.assign(n, 0); v.assign(n, 0); t.assign(n, 0);
        cycles.assign(n, 0); frame.assign(n, 0); dma.assign(n, 0); frame_dot.assign(n, 0);
        ram.assign(n * 2048, 0); prg_ram.assign(n * 8192, 0); nt.assign(n * 2048, 0); pal.assign(n * 32, 0);
        oam.assign(n * 256, 0); s_oam.assign(n * 256, 0); s_nt.assign(n * 2048, 0); s_pal.assign(n * 32, 0);
        frames.assign(n * 61440 * 3, 0);
        rewards.assign(n, 0.f); last_rewards.assign(n, 0.f); prev_x.assign(n, 0); prev_time.assign(n, 0);
        episode.assign(n, 0); stat_frames.assign(n, 0); stat_budget.assign(n, 0); stat_instr.assign(n, 0);
        auto& c = buf.cpu;
        c.pc = pc.data(); c.a = a.data(); c.x = x.data(); c.y = y.data(); c.sp = sp.data(); c.p = p.data();
        c.cycles = cycles.data(); c.nmi_pending = cpu_nmi.data(); c.irq_pending = irq.data(); c.ram = ram.data();
        c.prg_ram = prg_ram.data(); c.controller1_shift = shift.data(); c.controller1_shift_count = count.data();
        c.controller1_strobe = strobe.data(); c.pending_dma_cycles = dma.data();
        auto& q = buf.ppu;
        q.ctrl = ctrl.data(); q.mask = mask.data(); q.status = status.data(); q.oam_addr = oam_addr.data();
        q.nmi_pending = nmi.data(); q.frame_dot = frame_dot.data(); q.frame = frame.data(); q.v = v.data();
        q.t = t.data(); q.x = fx.data(); q.w = w.data(); q.open_bus = open_bus.data(); q.read_buffer = read_buf.data();
        q.scroll_x = sx.data(); q.scroll_y = sy.data(); q.nametable_ram = nt.data(); q.palette_ram = pal.data();
        q.oam = oam.data(); q.lat_scroll_x = lat_sx.data(); q.lat_scroll_y = lat_sy.data(); q.lat_ctrl = lat_ctrl.data();
        q.snap_scroll_x_start = s_sx0.data(); q.snap_scroll_y_start = s_sy0.data(); q.snap_ctrl_start = s_c0.data();
        q.snap_scroll_x_end = s_sx1.data(); q.snap_scroll_y_end = s_sy1.data(); q.snap_ctrl_end = s_c1.data();
        q.snap_mask = s_mask.data(); q.snap_oam = s_oam.data(); q.snap_nametable = s_nt.data();
        q.snap_palette = s_pal.data();
        buf.cart.prg_rom = rom.prg_rom.data();
        buf.cart.prg_rom_size = static_cast<std::uint32_t>(rom.prg_rom.size());
        buf.cart.chr_rom = rom.chr_rom.empty() ? nullptr : rom.chr_rom.data();
        buf.cart.chr_rom_size = static_cast<std::uint32_t>(rom.chr_rom.size());
        buf.cart.mapper = 0;
        // cuda_module.cu:212-222
        switch (rom.metadata.nametable_arrangement) {
            case nesle::NametableArrangement::Vertical: buf.cart.nametable_arrangement = nesle::cuda::kNametableVertical; break;
            case nesle::NametableArrangement::Horizontal: buf.cart.nametable_arrangement = nesle::cuda::kNametableHorizontal; break;
            default: buf.cart.nametable_arrangement = nesle::cuda::kNametableFourScreen; break;
        }
        buf.action_masks = actions.data(); buf.done = done.data(); buf.rewards = rewards.data();
        buf.previous_mario_x = prev_x.data(); buf.previous_mario_time = prev_time.data();
        buf.frames_rgb = frames.data();
    }

    // cuda_module.cu:1291-1415 (bank layout), host-side.
    void upload_bank(const std::uint8_t* e2l) {
        const std::size_t k = snaps.size();
        if (k == 0) return;
        b_ram.resize(k * 2048); b_prg.resize(k * 8192); b_nt.resize(k * 2048); b_pal.resize(k * 32); b_oam.resize(k * 256);
        for (auto* vec : {&b_a, &b_x, &b_y, &b_sp, &b_p, &b_ctrl, &b_mask, &b_status, &b_oam_addr, &b_open, &b_rbuf, &b_fx, &b_w})
            vec->resize(k);
        b_pc.resize(k); b_v.resize(k); b_t.resize(k); b_cycles.resize(k);
        for (std::size_t i = 0; i < k; ++i) {
            const auto& s = snaps[i];
            std::memcpy(&b_ram[i * 2048], s.cpu_ram.data(), 2048);
            std::memcpy(&b_prg[i * 8192], s.prg_ram.data(), 8192);
            std::memcpy(&b_nt[i * 2048], s.nametable_ram.data(), 2048);
            std::memcpy(&b_pal[i * 32], s.palette_ram.data(), 32);
            std::memcpy(&b_oam[i * 256], s.oam.data(), 256);
            b_pc[i] = s.pc; b_a[i] = s.a; b_x[i] = s.x; b_y[i] = s.y; b_sp[i] = s.sp; b_p[i] = s.p;
            b_cycles[i] = s.cycles; b_ctrl[i] = s.ppu_ctrl; b_mask[i] = s.ppu_mask; b_status[i] = s.ppu_status;
            b_oam_addr[i] = s.ppu_oam_addr; b_open[i] = s.ppu_open_bus; b_rbuf[i] = s.ppu_read_buffer;
            b_fx[i] = s.ppu_x; b_w[i] = s.ppu_w; b_v[i] = s.ppu_v; b_t[i] = s.ppu_t;
        }
        env_to_level.assign(cfg.n, 0);
        if (e2l) std::memcpy(env_to_level.data(), e2l, cfg.n);
        bank.cpu_ram = b_ram.data(); bank.prg_ram = b_prg.data(); bank.nametable_ram = b_nt.data();
        bank.palette_ram = b_pal.data(); bank.oam = b_oam.data(); bank.pc = b_pc.data(); bank.a = b_a.data();
        bank.x = b_x.data(); bank.y = b_y.data(); bank.sp = b_sp.data(); bank.p = b_p.data();
        bank.cycles = b_cycles.data(); bank.ppu_ctrl = b_ctrl.data(); bank.ppu_mask = b_mask.data();
        bank.ppu_status = b_status.data(); bank.ppu_oam_addr = b_oam_addr.data(); bank.ppu_open_bus = b_open.data();
        bank.ppu_read_buffer = b_rbuf.data(); bank.ppu_x = b_fx.data(); bank.ppu_w = b_w.data();
        bank.ppu_v = b_v.data(); bank.ppu_t = b_t.data(); bank.env_to_level = env_to_level.data();
        bank.num_levels = static_cast<std::uint32_t>(k);
    }

    void reset_env(std::uint32_t env) {
        if (!snaps.empty()) nesle::cuda::warm_reset_console_env(buf, env, bank);
        else nesle::cuda::cold_reset_console_env(buf, env);
    }

    // cuda_module.cu:469-480 + 1417-1463: reset every env, then seed the
    // presentation snapshot from live state.
    void reset_all() {
        for (std::uint32_t e = 0; e < cfg.n; ++e) {
            actions[e] = 0;
            episode[e] = 0;
            reset_env(e);
        }
        s_nt = nt; s_pal = pal; s_oam = oam; s_mask = mask;
        lat_sx = s_sx0 = s_sx1 = sx;
        lat_sy = s_sy0 = s_sy1 = sy;
        lat_ctrl = s_c0 = s_c1 = ctrl;
    }

    // kernels.cu:19-104, one env.
    void step_env(std::uint32_t env) {
        using namespace nesle::cuda;
        auto state = load_cpu_state(buf, env);
        auto hot = load_ppu_hot_state(buf, env);
        std::uint32_t pending = 0;
        std::uint32_t horizon = batch_ppu_cycles_until_next_timing_event_hot(hot);
        std::uint64_t total_instr = 0;
        std::uint32_t total_frames = 0, budget = 0;
        for (std::uint32_t f = 0; f < cfg.frameskip; ++f) {
            std::uint64_t instr = 0;
            std::uint32_t frames_done = 0;
            while (instr < cfg.max_instr && frames_done == 0) {
                if (pending >= horizon) {
                    frames_done += batch_ppu_step_env_hot(buf, env, pending, hot).frames_completed;
                    pending = 0;
                    horizon = batch_ppu_cycles_until_next_timing_event_hot(hot);
                    if (frames_done != 0) break;
                }
                const auto s = step_batch_console_instruction_lazy(buf, env, state, hot);
                pending += s.ppu_cycles;
                if (prof_opcode) ++prof_opcode[s.cpu.opcode];
                if (prof_pc) ++prof_pc[s.cpu.pc];
                ++instr;
                if (s.cpu.opcode == 0x4C && state.pc == s.cpu.pc && frames_done == 0) {
                    frames_done += batch_ppu_step_env_hot(buf, env, pending, hot).frames_completed;
                    pending = 0;
                    frames_done += fast_forward_batch_console_idle_loop_hot(buf, env, state, hot).frames_completed;
                    horizon = batch_ppu_cycles_until_next_timing_event_hot(hot);
                }
            }
            if (pending != 0) {
                frames_done += batch_ppu_step_env_hot(buf, env, pending, hot).frames_completed;
                pending = 0;
                horizon = batch_ppu_cycles_until_next_timing_event_hot(hot);
            }
            total_instr += instr;
            total_frames += frames_done;
            if (frames_done == 0 && instr >= cfg.max_instr) ++budget;
        }
        store_cpu_state(buf, env, state);
        store_ppu_hot_state(buf, env, hot);
        apply_batch_reward_env(buf, env);
        if (cfg.done_mode == 1) done[env] = ram[env * 2048 + (cfg.done_a & 0x7FF)] == cfg.done_b;
        if (cfg.done_mode == 2)
            done[env] = frame[env] >= frame_limit(cfg.seed, cfg.done_a, cfg.done_b, cfg.env_offset + env, episode[env]);
        stat_instr[env] = total_instr;
        stat_frames[env] = total_frames;
        stat_budget[env] = budget;
    }

    // cuda_module.cu:594-666 (device_api) or :533-592.
    void step(const std::uint8_t* act, int device_api, int auto_reset) {
        std::memcpy(actions.data(), act, cfg.n);
        for (std::uint32_t e = 0; e < cfg.n; ++e) step_env(e);
        if (!device_api) return;
        last_rewards = rewards;
        last_done = done;
        if (auto_reset)
            for (std::uint32_t e = 0; e < cfg.n; ++e)
                if (last_done[e]) { episode[e]++; reset_env(e); }
    }

    void render() {
        for (std::uint32_t e = 0; e < cfg.n; ++e) {
            auto views = nesle::cuda::resolve_render_env_views(buf, e);
            for (std::uint32_t px = 0; px < 61440; ++px)
                nesle::cuda::render_batch_rgb_pixel_env(buf, views.hud, views.play, e, views.split_y, px);
        }
    }
};

// ---------------------------------------------------------------------------
// Kind A: the reference CPU core, one nesle::Console per env.
// ---------------------------------------------------------------------------
struct ConsoleA {
    Config cfg;
    std::vector<std::uint8_t> rom_bytes;
    std::vector<nesle::fcs::StateSnapshot> snaps;
    std::vector<std::uint8_t> env_to_level;
    std::vector<std::unique_ptr<nesle::Console>> con;
    std::vector<nesle::cpu::CpuState> cpu;
    std::vector<int> prev_x, prev_time;
    std::vector<float> rewards, last_rewards;
    std::vector<std::uint8_t> done, last_done;
    std::vector<std::uint32_t> episode;
    std::vector<std::uint64_t> stat_instr;
    std::vector<std::uint32_t> stat_frames;

    void reset_env(std::uint32_t e) {
        con[e] = std::make_unique<nesle::Console>(nesle::parse_ines(rom_bytes));
        auto& c = *con[e];
        cpu[e] = nesle::cpu::CpuState{};
        if (snaps.empty()) {
            c.reset_cpu(cpu[e]);
            prev_x[e] = 0;
            prev_time[e] = 0;
        } else {
            const auto& s = snaps[env_to_level[e]];
            if (s.ppu_v || s.ppu_t || s.ppu_x || s.ppu_w || s.ppu_open_bus || s.ppu_read_buffer || s.ppu_oam_addr)
                throw std::invalid_argument("Console snapshot injection needs power-on v/t/x/w/open-bus/read-buffer/OAMADDR");
            auto& st = cpu[e];
            st.pc = s.pc; st.a = s.a; st.x = s.x; st.y = s.y; st.sp = s.sp; st.p = s.p; st.cycles = s.cycles;
            st.variant = nesle::cpu::CpuVariant::Ricoh2A03;
            c.cpu_ram() = s.cpu_ram;
            for (std::uint16_t i = 0; i < 8192; ++i) c.write(static_cast<std::uint16_t>(0x6000 + i), s.prg_ram[i]);
            nesle::Ppu::RenderState rs;
            rs.ctrl = s.ppu_ctrl; rs.mask = s.ppu_mask; rs.status = s.ppu_status;
            rs.palette_ram = s.palette_ram; rs.oam = s.oam; rs.nametable_ram = s.nametable_ram;
            c.ppu().load_render_state(rs);
            const auto snap = nesle::smb::read_ram(std::span<const std::uint8_t>(s.cpu_ram.data(), 2048));
            prev_x[e] = snap.x_pos;
            prev_time[e] = snap.time;
        }
        rewards[e] = 0.f;
        done[e] = 0;
    }

    void reset_all() {
        for (std::uint32_t e = 0; e < cfg.n; ++e) { episode[e] = 0; reset_env(e); }
    }

    void step_env(std::uint32_t e, std::uint8_t action) {
        auto& c = *con[e];
        c.controller1().set_buttons(action);
        std::uint64_t instr = 0;
        std::uint32_t frames = 0;
        for (std::uint32_t f = 0; f < cfg.frameskip; ++f) {
            const auto r = c.step_frame(cpu[e], cfg.max_instr);
            instr += r.instructions;
            frames += r.frames_completed;
        }
        stat_instr[e] = instr;
        stat_frames[e] = frames;
        const auto& ram = c.cpu_ram();
        const auto cur = nesle::smb::read_ram(std::span<const std::uint8_t>(ram.data(), 2048));
        nesle::smb::MarioRamState prev{};
        prev.x_pos = prev_x[e];
        prev.time = prev_time[e];
        rewards[e] = static_cast<float>(nesle::smb::compute_reward(prev, cur).total);
        std::uint8_t d = (cur.flag_get || cur.is_dying || cur.is_dead || cur.is_game_over) ? 1 : 0;
        if (cfg.done_mode == 1) d = ram[cfg.done_a & 0x7FF] == cfg.done_b;
        if (cfg.done_mode == 2)
            d = c.ppu().frame() >= frame_limit(cfg.seed, cfg.done_a, cfg.done_b, cfg.env_offset + e, episode[e]);
        done[e] = d;
        prev_x[e] = cur.x_pos;
        prev_time[e] = cur.time;
    }

    void step(const std::uint8_t* act, int device_api, int auto_reset, int threads) {
        auto work = [&](std::uint32_t lo, std::uint32_t hi) {
            for (std::uint32_t e = lo; e < hi; ++e) {
                step_env(e, act[e]);
                if (device_api) {
                    last_rewards[e] = rewards[e];
                    last_done[e] = done[e];
                    if (auto_reset && last_done[e]) { episode[e]++; reset_env(e); }
                }
            }
        };
        if (threads <= 1) { work(0, cfg.n); return; }
        std::vector<std::thread> pool;
        const std::uint32_t chunk = (cfg.n + threads - 1) / threads;
        for (int t = 0; t < threads; ++t) {
            const std::uint32_t lo = t * chunk, hi = std::min(cfg.n, lo + chunk);
            if (lo < hi) pool.emplace_back(work, lo, hi);
        }
        for (auto& th : pool) th.join();
    }
};

struct Handle {
    char kind;
    std::unique_ptr<BatchB> b;
    std::unique_ptr<ConsoleA> a;
};

template <class F>
int guarded(F&& f) {
    try {
        f();
        return 0;
    } catch (const std::exception& ex) {
        g_error = ex.what();
        return -1;
    }
}

}  // namespace

extern "C" {

const char* ref_last_error() { return g_error.c_str(); }

void* ref_create(char kind, std::uint32_t n, std::uint32_t frameskip, const std::uint8_t* rom, std::size_t rom_len,
                 const std::uint8_t* const* snaps, const std::size_t* lens, std::uint32_t nsnap,
                 const std::uint8_t* env_to_level, std::uint32_t done_mode, std::uint32_t done_a, std::uint32_t done_b,
                 std::uint64_t seed, std::uint32_t env_offset) {
    Handle* h = nullptr;
    const int rc = guarded([&] {
        Config cfg;
        cfg.n = n; cfg.frameskip = frameskip; cfg.done_mode = done_mode; cfg.done_a = done_a; cfg.done_b = done_b;
        cfg.seed = seed; cfg.env_offset = env_offset;
        std::vector<std::uint8_t> bytes(rom, rom + rom_len);
        std::vector<nesle::fcs::StateSnapshot> parsed;
        for (std::uint32_t i = 0; i < nsnap; ++i)
            parsed.push_back(nesle::fcs::parse(std::span<const std::uint8_t>(snaps[i], lens[i])));
        auto hh = std::make_unique<Handle>();
        hh->kind = kind;
        if (kind == 'B') {
            auto b = std::make_unique<BatchB>();
            b->cfg = cfg;
            b->rom = nesle::parse_ines(bytes);
            if (!b->rom.metadata.is_nrom()) throw std::invalid_argument("CUDA console mode currently supports mapper 0/NROM ROMs");
            b->snaps = std::move(parsed);
            b->allocate();
            b->upload_bank(env_to_level);
            b->reset_all();
            hh->b = std::move(b);
        } else {
            auto a = std::make_unique<ConsoleA>();
            a->cfg = cfg;
            a->rom_bytes = bytes;
            a->snaps = std::move(parsed);
            a->env_to_level.assign(n, 0);
            if (env_to_level) std::memcpy(a->env_to_level.data(), env_to_level, n);
            a->con.resize(n);
            a->cpu.resize(n);
            a->prev_x.assign(n, 0); a->prev_time.assign(n, 0); a->rewards.assign(n, 0.f);
            a->last_rewards.assign(n, 0.f); a->done.assign(n, 0); a->last_done.assign(n, 0);
            a->episode.assign(n, 0); a->stat_instr.assign(n, 0); a->stat_frames.assign(n, 0);
            a->reset_all();
            hh->a = std::move(a);
        }
        h = hh.release();
    });
    return rc == 0 ? h : nullptr;
}

void ref_destroy(void* h) { delete static_cast<Handle*>(h); }

int ref_reset(void* hv) {
    auto* h = static_cast<Handle*>(hv);
    return guarded([&] { if (h->b) h->b->reset_all(); else h->a->reset_all(); });
}

int ref_reset_envs(void* hv, const std::uint8_t* mask) {
    auto* h = static_cast<Handle*>(hv);
    return guarded([&] {
        const std::uint32_t n = h->b ? h->b->cfg.n : h->a->cfg.n;
        for (std::uint32_t e = 0; e < n; ++e) {
            if (!mask[e]) continue;
            if (h->b) { h->b->episode[e]++; h->b->reset_env(e); }
            else { h->a->episode[e]++; h->a->reset_env(e); }
        }
    });
}

int ref_step(void* hv, const std::uint8_t* actions, int device_api, int auto_reset, int threads) {
    auto* h = static_cast<Handle*>(hv);
    return guarded([&] {
        if (h->b) h->b->step(actions, device_api, auto_reset);
        else h->a->step(actions, device_api, auto_reset, threads);
    });
}

// Kind B only: opcode / fetch-address histograms of the following steps, as
// console_step_kernel counts them (kernels.cu:59-64).  NULL stops counting.
int ref_set_profile(void* hv, std::uint64_t* opcode_counts, std::uint64_t* pc_counts) {
    auto* h = static_cast<Handle*>(hv);
    return guarded([&] {
        if (!h->b) throw std::invalid_argument("profiling is only available for kind B");
        h->b->prof_opcode = opcode_counts;
        h->b->prof_pc = pc_counts;
    });
}

int ref_render_rgb(void* hv, std::uint8_t* out) {
    auto* h = static_cast<Handle*>(hv);
    return guarded([&] {
        if (!h->b) throw std::invalid_argument("render is only available for kind B");
        h->b->render();
        std::memcpy(out, h->b->frames.data(), h->b->frames.size());
    });
}

// Named per-env fields, same names as oracle_get_field().
int ref_get_field(void* hv, const char* name, void* out) {
    auto* h = static_cast<Handle*>(hv);
    const std::string f = name;
    return guarded([&] {
        auto put = [&](const auto& vec) { std::memcpy(out, vec.data(), vec.size() * sizeof(vec[0])); };
        if (h->b) {
            auto& b = *h->b;
            if (f == "pc") put(b.pc); else if (f == "a") put(b.a); else if (f == "x") put(b.x);
            else if (f == "y") put(b.y); else if (f == "sp") put(b.sp); else if (f == "p") put(b.p);
            else if (f == "cycles") put(b.cycles); else if (f == "ram") put(b.ram); else if (f == "prg_ram") put(b.prg_ram);
            else if (f == "ctrl_shift") put(b.shift); else if (f == "ctrl_count") put(b.count);
            else if (f == "ctrl_strobe") put(b.strobe); else if (f == "pending_dma") put(b.dma);
            else if (f == "ppu_ctrl") put(b.ctrl); else if (f == "ppu_mask") put(b.mask);
            else if (f == "ppu_status") put(b.status); else if (f == "oam_addr") put(b.oam_addr);
            else if (f == "nmi_pending") put(b.nmi); else if (f == "frame_dot") put(b.frame_dot);
            else if (f == "frame") put(b.frame); else if (f == "v") put(b.v); else if (f == "t") put(b.t);
            else if (f == "fine_x") put(b.fx); else if (f == "w") put(b.w); else if (f == "open_bus") put(b.open_bus);
            else if (f == "read_buffer") put(b.read_buf); else if (f == "scroll_x") put(b.sx);
            else if (f == "scroll_y") put(b.sy); else if (f == "lat_sx") put(b.lat_sx); else if (f == "lat_sy") put(b.lat_sy);
            else if (f == "lat_ctrl") put(b.lat_ctrl); else if (f == "snap_sx_start") put(b.s_sx0);
            else if (f == "snap_sy_start") put(b.s_sy0); else if (f == "snap_ctrl_start") put(b.s_c0);
            else if (f == "snap_sx_end") put(b.s_sx1); else if (f == "snap_sy_end") put(b.s_sy1);
            else if (f == "snap_ctrl_end") put(b.s_c1); else if (f == "snap_mask") put(b.s_mask);
            else if (f == "prev_x") put(b.prev_x); else if (f == "prev_time") put(b.prev_time);
            else if (f == "reward") put(b.rewards); else if (f == "last_reward") put(b.last_rewards);
            else if (f == "done") put(b.done); else if (f == "last_done") put(b.last_done);
            else if (f == "nt") put(b.nt); else if (f == "pal") put(b.pal); else if (f == "oam") put(b.oam);
            else if (f == "snap_oam") put(b.s_oam); else if (f == "snap_nt") put(b.s_nt); else if (f == "snap_pal") put(b.s_pal);
            else if (f == "episode") put(b.episode); else if (f == "stat_instructions") put(b.stat_instr);
            else if (f == "stat_frames") put(b.stat_frames); else if (f == "stat_budget_hits") put(b.stat_budget);
            else throw std::invalid_argument("unknown field " + f);
        } else {
            auto& a = *h->a;
            const std::uint32_t n = a.cfg.n;
            auto* o8 = static_cast<std::uint8_t*>(out);
            if (f == "ram") {
                for (std::uint32_t e = 0; e < n; ++e) std::memcpy(o8 + e * 2048, a.con[e]->cpu_ram().data(), 2048);
            } else if (f == "pc") {
                for (std::uint32_t e = 0; e < n; ++e) std::memcpy(o8 + e * 2, &a.cpu[e].pc, 2);
            } else if (f == "a" || f == "x" || f == "y" || f == "sp" || f == "p") {
                for (std::uint32_t e = 0; e < n; ++e) {
                    const auto& s = a.cpu[e];
                    o8[e] = f == "a" ? s.a : f == "x" ? s.x : f == "y" ? s.y : f == "sp" ? s.sp : s.p;
                }
            } else if (f == "cycles") {
                for (std::uint32_t e = 0; e < n; ++e) std::memcpy(o8 + e * 8, &a.cpu[e].cycles, 8);
            } else if (f == "frame") {
                for (std::uint32_t e = 0; e < n; ++e) { const std::uint64_t fr = a.con[e]->ppu().frame(); std::memcpy(o8 + e * 8, &fr, 8); }
            } else if (f == "ppu_status" || f == "ppu_ctrl" || f == "ppu_mask" || f == "oam_addr") {
                for (std::uint32_t e = 0; e < n; ++e) {
                    const auto& q = a.con[e]->ppu();
                    o8[e] = f == "ppu_status" ? q.status() : f == "ppu_ctrl" ? q.ctrl() : f == "ppu_mask" ? q.mask() : q.oam_addr();
                }
            } else if (f == "oam") {
                for (std::uint32_t e = 0; e < n; ++e) std::memcpy(o8 + e * 256, a.con[e]->ppu().oam().data(), 256);
            } else if (f == "reward") put(a.rewards); else if (f == "last_reward") put(a.last_rewards);
            else if (f == "done") put(a.done); else if (f == "last_done") put(a.last_done);
            else if (f == "prev_x") put(a.prev_x); else if (f == "prev_time") put(a.prev_time);
            else if (f == "episode") put(a.episode); else if (f == "stat_instructions") put(a.stat_instr);
            else if (f == "stat_frames") put(a.stat_frames);
            else throw std::invalid_argument("unknown field " + f);
        }
    });
}

// Kind A only: one env stepped instruction by instruction with the same
// 16-byte records as oracle_set_trace(); `frames` frames at the env's action.
int ref_trace_console(void* hv, std::uint32_t env, std::uint8_t action, std::uint32_t frames,
                      std::uint8_t* buf, std::uint32_t cap, std::uint32_t* count) {
    auto* h = static_cast<Handle*>(hv);
    return guarded([&] {
        if (!h->a) throw std::invalid_argument("trace is only available for kind A");
        auto& c = *h->a->con[env];
        auto& st = h->a->cpu[env];
        c.controller1().set_buttons(action);
        std::uint32_t n = 0;
        for (std::uint32_t f = 0; f < frames; ++f) {
            for (;;) {
                const auto r = c.step_cpu_instruction(st);
                if (n < cap) {
                    std::uint8_t* p = buf + static_cast<std::size_t>(n) * 16;
                    p[0] = static_cast<std::uint8_t>(r.cpu.pc); p[1] = static_cast<std::uint8_t>(r.cpu.pc >> 8);
                    p[2] = r.cpu.opcode; p[3] = st.a; p[4] = st.x; p[5] = st.y; p[6] = st.p; p[7] = st.sp;
                    std::memcpy(p + 8, &st.cycles, 8);
                    ++n;
                }
                if (r.frames_completed) break;
            }
        }
        *count = n;
    });
}

// The reference decode table (cpu.hpp:190-357), for pinning the checker's.
void ref_decode_table(std::uint8_t* mode, std::uint8_t* cycles, std::uint8_t* flags) {
    for (int i = 0; i < 256; ++i) {
        const auto e = nesle::cpu::detail::decode(static_cast<std::uint8_t>(i));
        mode[i] = static_cast<std::uint8_t>(e.mode);
        cycles[i] = e.base_cycles;
        flags[i] = e.flags;
    }
}

// nesle::fcs::parse (fcs.hpp:187-226) -> flat record for comparison.
struct RefFcs {
    std::uint16_t pc, v, t;
    std::uint8_t a, x, y, sp, p, ctrl, mask, status, oam_addr, open_bus, read_buffer, fine_x, w;
    std::uint8_t ram[2048], prg_ram[8192], nt[2048], pal[32], oam[256];
};

int ref_parse_fcs(const std::uint8_t* data, std::size_t len, RefFcs* out) {
    return guarded([&] {
        const auto s = nesle::fcs::parse(std::span<const std::uint8_t>(data, len));
        out->pc = s.pc; out->v = s.ppu_v; out->t = s.ppu_t; out->a = s.a; out->x = s.x; out->y = s.y;
        out->sp = s.sp; out->p = s.p; out->ctrl = s.ppu_ctrl; out->mask = s.ppu_mask; out->status = s.ppu_status;
        out->oam_addr = s.ppu_oam_addr; out->open_bus = s.ppu_open_bus; out->read_buffer = s.ppu_read_buffer;
        out->fine_x = s.ppu_x; out->w = s.ppu_w;
        std::memcpy(out->ram, s.cpu_ram.data(), 2048); std::memcpy(out->prg_ram, s.prg_ram.data(), 8192);
        std::memcpy(out->nt, s.nametable_ram.data(), 2048); std::memcpy(out->pal, s.palette_ram.data(), 32);
        std::memcpy(out->oam, s.oam.data(), 256);
    });
}

}  // extern "C"
