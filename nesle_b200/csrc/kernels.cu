// kernels.cu -- sm_100a kernels of the batched NES core.
//
//   step_kernel_global  one env-step per thread, every env resident; with kHybrid
//                   the zero page is staged in shared memory, with kInterleave
//                   the rest of RAM lives for the launch in an env-interleaved
//                   working copy (kHybrid + kInterleave: the default above two
//                   shared-memory waves, e.g. at 65,536 envs)
//   step_kernel     one env-step per thread, env RAM staged in shared memory
//                   (the default for small batches, e.g. 2,048 envs)
//   reset_kernel    masked or full snapshot/cold reset
//   poke_kernel     one RAM byte in every env
//   render_kernel   colour-index or RGB frame from the presentation snapshot
//   gray84_kernel   84x84 area-resampled luma observation
#include <cuda_runtime.h>
#include <stdlib.h>

#include "kernels.h"
#include "nes_core.cuh"
#include "nes_render.cuh"
#include "nes_v2.cuh"

// NESLE_V2: the shared-RAM and in-place step kernels run the v2 datapath
// (nes_v2.cuh); the profiled and ahead-loading variants keep the first one.
#ifndef NESLE_V2
#define NESLE_V2 1
#endif

namespace nesle {

__constant__ EntryTable kEntriesConst = dt::build_entries();
__constant__ EntryTable2 kEntries2Const = dt::build_entries2();
__constant__ uint8_t kPaletteRgb[192] = NESLE_PALETTE_RGB;

// --------------------------------------------------------------------------
// Env step with RAM staged in shared memory.  One CTA = kStepSlots envs =
// kStepSlots threads: 32 KB PRG + 8 KB execution entries + kStepSlots x 2 KB
// interleaved RAM.  The default for batches of up to two waves of these CTAs
// (NESLE_STEP_KERNEL=shared forces it); larger batches use the in-place kernel.
// --------------------------------------------------------------------------
constexpr uint32_t kPrgSmem = 32768 + 16;  // +16: the two-word fetch at $FFFC-$FFFD reads one word past the ROM
constexpr uint32_t kDecSmem = NESLE_V2 ? sizeof(EntryTable2) : 256 * sizeof(Entry);  // the table a kernel stages

// Execution-entry quarters the v2 datapath prefetches one iteration ahead, per
// placement.  B200, env-steps/s with 0 / 1 / 2 quarters: shared RAM, 2,048
// envs of config 2: 240 / 247 / 244 k; hybrid, 65,536 envs of config 4:
// 2.27 / 2.27 / 2.18 M (2 spills), config 2: 3.26 / 3.15 / 3.13 M.  For the
// interleaved kernel the best depth moved with the datapath: 2 quarters won
// config 4 before the word-load pointer read (2.36 M against 2.34 / 2.31 M
// with 1 / 0), 1 quarter wins after it (2.50 M against 2.47 M; config 2 3.42
// against 3.31 M).  Config 4 is the benchmark workload.
constexpr uint32_t kEarlyShared = 1;
constexpr uint32_t kEarlyInPlace = 0;
constexpr uint32_t kEarlyInterleaved = 1;

// Stages the execution entries of the datapath the kernel runs (v2 when
// kV2) into shared memory at `dst`.
template <bool kV2>
__device__ __forceinline__ void stage_entries(uint8_t* dst, uint32_t tid, uint32_t threads) {
    const uint4* src = kV2 ? reinterpret_cast<const uint4*>(&kEntries2Const) : reinterpret_cast<const uint4*>(&kEntriesConst);
    const uint32_t n = (kV2 ? sizeof(EntryTable2) : sizeof(EntryTable)) / 16;
    for (uint32_t i = tid; i < n; i += threads) reinterpret_cast<uint4*>(dst)[i] = src[i];
}

__device__ __forceinline__ uint32_t* ram_word(uint8_t* slot, uint32_t word) {
    return reinterpret_cast<uint32_t*>(slot + word * 4u * kStepSlots);
}

// kBoard: the cartridge may be UxROM or CNROM (Ctx::prg_lo / prg_writes at
// run time); NROM batches run the kBoard = false instantiations, where both
// are constants.
template <bool kBoard>
__global__ void __launch_bounds__(kStepSlots, 1)
step_kernel(const BatchView* __restrict__ vp, const uint8_t* __restrict__ act8,
            const long long* __restrict__ act64, uint32_t flags) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* s_prg = smem;
    Entry* s_dec = reinterpret_cast<Entry*>(smem + kPrgSmem);
    uint8_t* s_ram = smem + kPrgSmem + kDecSmem;
    const BatchView& v = *vp;
    const uint32_t tid = threadIdx.x;

    const uint4* prg_src = reinterpret_cast<const uint4*>(v.prg);
    for (uint32_t i = tid; i < 2048; i += blockDim.x) reinterpret_cast<uint4*>(s_prg)[i] = prg_src[i];
    if (tid == 0) reinterpret_cast<uint4*>(s_prg)[2048] = make_uint4(0, 0, 0, 0);
    stage_entries<NESLE_V2>(reinterpret_cast<uint8_t*>(s_dec), tid, blockDim.x);

    const uint32_t env = blockIdx.x * kStepSlots + tid;
    const bool active = env < v.num_envs;
    uint8_t* slot = s_ram + tid * 4;
    if (active) {
        // Each lane stages its own 2 KB row: conflict-free (its bank only).
        const uint4* src = reinterpret_cast<const uint4*>(v.ram + (size_t)env * kRamBytes);
#pragma unroll 4
        for (uint32_t q = 0; q < kRamBytes / 16; ++q) {
            const uint4 w = src[q];
            *ram_word(slot, 4 * q + 0) = w.x;
            *ram_word(slot, 4 * q + 1) = w.y;
            *ram_word(slot, 4 * q + 2) = w.z;
            *ram_word(slot, 4 * q + 3) = w.w;
        }
    }
    __syncthreads();
    if (!active) return;

    Ctx c;
    c.ram = slot;
    c.slots = kStepSlots;
    c.zp = nullptr;
    c.zslots = 0;
    c.zpage = 0;
    c.prg = s_prg;
    c.dec = s_dec;
    c.dec2 = reinterpret_cast<const EntryQuad*>(s_dec);
    c.view = vp;
    c.env = env;
    c.frameskip = v.frameskip;
    c.max_instr = v.max_instructions;
    c.prg_ram = v.prg_ram + (size_t)env * kPrgRamBytes;
    c.nt = v.nt + (size_t)env * kNtBytes;
    c.pal = v.pal + (size_t)env * kPalBytes;
    c.oam = v.oam + (size_t)env * kOamBytes;
    c.prg_lo = kBoard && v.mapper == kMapperUxrom ? 0xC000u : 0x8000u;
    c.prg_writes = kBoard;

    EnvRecord rec = v.rec[env];
    const uint32_t status_before = rec.status;
    const uint8_t action = act64 ? (uint8_t)(act64[env] & 0xFF) : act8[env];
    float reward;
    uint8_t done;
    if (NESLE_V2) run_env_step_v2<true, kEarlyShared>(c, rec, action, reward, done);
    else run_env_step(c, rec, action, reward, done);

    uint4* dst = reinterpret_cast<uint4*>(v.ram + (size_t)env * kRamBytes);
#pragma unroll 4
    for (uint32_t q = 0; q < kRamBytes / 16; ++q) {
        dst[q] = make_uint4(*ram_word(slot, 4 * q + 0), *ram_word(slot, 4 * q + 1), *ram_word(slot, 4 * q + 2),
                            *ram_word(slot, 4 * q + 3));
    }
    const bool faulted = finish_env(v, env, rec, status_before, reward, done, flags & kStepDeviceApi,
                                    flags & kStepAutoReset);
    v.rec[env] = rec;
    if (faulted) atomicAdd(v.fault_count, 1u);
}

// --------------------------------------------------------------------------
// Env step, RAM in place.  The env's RAM row stays in global memory and only
// PRG + execution entries are staged, so a CTA holds up to 448 envs and every
// env of a 65,536-env batch is resident at once (one CTA per SM): warp
// parallelism, not shared-memory capacity, hides the memory latency.
// kProfile adds the step_profile histograms: opcode counts gathered per CTA in
// shared memory, fetch-address counts with warp-aggregated global atomics.
// --------------------------------------------------------------------------
struct DeviceProfile {
    uint32_t* op_counts;             // shared, 256
    unsigned long long* pc_counts;   // global, 65536
    NESLE_HD void count(uint32_t op, uint32_t pc) const {
#if defined(__CUDA_ARCH__)
        const uint32_t active = __activemask(), lane = threadIdx.x & 31u;
        uint32_t peers = __match_any_sync(active, op);
        if (lane == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&op_counts[op], (uint32_t)__popc(peers));
        peers = __match_any_sync(active, pc);
        if (lane == (uint32_t)(__ffs(peers) - 1)) atomicAdd(&pc_counts[pc], (unsigned long long)__popc(peers));
#endif
    }
};

// Asynchronous operand load of one lane (run_frames_async): a 4-byte cp.async
// from the env's RAM row into the lane's shared-memory word, completing on the
// lane's own mbarrier (expected arrival count 1, so every load is one phase).
// Readiness is tested without waiting (mbarrier.test_wait.parity).
struct DeviceAsync {
    uint32_t word_addr, bar_addr;  // shared-window addresses
    uint32_t shift = 0;            // bit position of the operand in the loaded word
    __device__ __forceinline__ void init(uint32_t* word, unsigned long long* bar) {
        word_addr = static_cast<uint32_t>(__cvta_generic_to_shared(word));
        bar_addr = static_cast<uint32_t>(__cvta_generic_to_shared(bar));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bar_addr) : "memory");
    }
    __device__ __forceinline__ void issue(const uint8_t* byte_addr) {
        const uint8_t* src = reinterpret_cast<const uint8_t*>(reinterpret_cast<uintptr_t>(byte_addr) & ~(uintptr_t)3);
        shift = static_cast<uint32_t>(reinterpret_cast<uintptr_t>(byte_addr) & 3u) * 8u;
        asm volatile("cp.async.ca.shared::cta.global [%0], [%1], 4;" ::"r"(word_addr), "l"(src) : "memory");
        asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(bar_addr) : "memory");
    }
    __device__ __forceinline__ bool ready(uint32_t parity) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(ok)
            : "r"(bar_addr), "r"(parity)
            : "memory");
        return ok != 0;
    }
    __device__ __forceinline__ uint32_t byte() const {
        uint32_t w;
        asm volatile("ld.shared::cta.u32 %0, [%1];" : "=r"(w) : "r"(word_addr) : "memory");
        return (w >> shift) & 0xFFu;
    }
    // A load still in flight when the lane stops (only after a stall): wait for
    // it with the same bound, so nothing lands in shared memory after the CTA.
    __device__ __forceinline__ void drain(uint32_t parity) {
        for (uint32_t i = 0; i < kAsyncSpinLimit && !ready(parity); ++i) {
        }
    }
};

constexpr uint32_t kAsyncSmemPerLane = 12;  // mbarrier (8 B) + operand word (4 B)

// The operand of the next instruction as a plain global byte load into a
// register, issued at the end of the current iteration (run_frames_async with
// ready() always true).  The asm keeps the load where it is issued: the
// compiler would otherwise move it down to its first use, and its "memory"
// clobber keeps every earlier store of the lane ahead of it.
struct DevicePreload {
    uint32_t v = 0;
    __device__ __forceinline__ void issue(const uint8_t* byte_addr) {
        asm volatile("ld.global.u8 %0, [%1];" : "=r"(v) : "l"(byte_addr) : "memory");
    }
    __device__ __forceinline__ bool ready(uint32_t) const { return true; }
    __device__ __forceinline__ uint32_t byte() const { return v; }
    __device__ __forceinline__ void drain(uint32_t) const {}
};

// kHybrid: each env's zero page ($0000-$00FF) is staged into shared memory for
// the launch (interleaved 4 bytes per lane: every lane keeps to its own bank)
// and written back before the env's done/auto-reset; the rest of RAM stays in
// place.  Zero-page operands and indirect pointers then cost a shared-memory
// access instead of a global one.
// kOperand: 0 operands read when the instruction executes; 1 RAM operands
// outside the slot loaded ahead with cp.async and per-lane barriers (which
// follow the slots in shared memory); 2 loaded ahead into a register.
// kInterleave: for the launch, RAM outside the slot moves to an env-interleaved
// working copy in device memory (BatchView::ram_work: per CTA, word w of lane
// l at (w * lanes + l) * 4), so the same address of the 32 envs of a warp is
// one 128-byte line instead of 32 rows; copied in at the start and back at the
// end of the launch.
template <bool kProfile, bool kHybrid, int kOperand = 0, bool kInterleave = false, bool kBoard = false>
__global__ void __launch_bounds__(kGlobalMaxThreads, 1)
step_kernel_global(const BatchView* __restrict__ vp, const uint8_t* __restrict__ act8,
                   const long long* __restrict__ act64, uint32_t flags, unsigned long long* __restrict__ prof_op,
                   unsigned long long* __restrict__ prof_pc, uint32_t slot_page) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint32_t s_op[kProfile ? 256 : 1];
    uint8_t* s_prg = smem;
    Entry* s_dec = reinterpret_cast<Entry*>(smem + kPrgSmem);
    uint32_t* s_zp = reinterpret_cast<uint32_t*>(smem + kPrgSmem + kDecSmem);  // [64 words][blockDim lanes]
    uint8_t* s_async = smem + kPrgSmem + kDecSmem + (kHybrid ? (size_t)blockDim.x * 256 : 0);  // kOperand == 1
    const BatchView& v = *vp;
    const uint32_t tid = threadIdx.x;
    const uint4* prg_src = reinterpret_cast<const uint4*>(v.prg);
    for (uint32_t i = tid; i < 2048; i += blockDim.x) reinterpret_cast<uint4*>(s_prg)[i] = prg_src[i];
    if (tid == 0) reinterpret_cast<uint4*>(s_prg)[2048] = make_uint4(0, 0, 0, 0);
    constexpr bool kV2 = NESLE_V2 && !kProfile && kOperand == 0;  // the datapath this instantiation runs
    stage_entries<kV2>(reinterpret_cast<uint8_t*>(s_dec), tid, blockDim.x);
    if (kProfile)
        for (uint32_t i = tid; i < 256; i += blockDim.x) s_op[i] = 0;
    __syncthreads();
    const uint32_t env = blockIdx.x * blockDim.x + tid;
    if (env < v.num_envs) {
        Ctx c;
        c.ram = v.ram + (size_t)env * kRamBytes;
        c.slots = 1;
        c.zp = nullptr;
        c.zslots = 0;
        c.zpage = 0;
        if (kHybrid) {
            const uint4* src = reinterpret_cast<const uint4*>(c.ram + slot_page);
#pragma unroll 4
            for (uint32_t q = 0; q < 16; ++q) {
                const uint4 w = src[q];
                s_zp[(4 * q + 0) * blockDim.x + tid] = w.x;
                s_zp[(4 * q + 1) * blockDim.x + tid] = w.y;
                s_zp[(4 * q + 2) * blockDim.x + tid] = w.z;
                s_zp[(4 * q + 3) * blockDim.x + tid] = w.w;
            }
            c.zp = reinterpret_cast<uint8_t*>(s_zp + tid);
            c.zslots = blockDim.x;
            c.zpage = slot_page;
        }
        uint32_t* work = nullptr;
        if (kInterleave) {
            work = reinterpret_cast<uint32_t*>(v.ram_work + (size_t)blockIdx.x * blockDim.x * kRamBytes) + tid;
            const uint4* src = reinterpret_cast<const uint4*>(c.ram);
#pragma unroll 4
            for (uint32_t q = 0; q < kRamBytes / 16; ++q) {
                const uint4 w = src[q];
                work[(4 * q + 0) * blockDim.x] = w.x;
                work[(4 * q + 1) * blockDim.x] = w.y;
                work[(4 * q + 2) * blockDim.x] = w.z;
                work[(4 * q + 3) * blockDim.x] = w.w;
            }
            c.ram = reinterpret_cast<uint8_t*>(work);
            c.slots = blockDim.x;
        }
        c.prg = s_prg;
        c.dec = s_dec;
        c.dec2 = reinterpret_cast<const EntryQuad*>(s_dec);
        c.view = vp;
        c.env = env;
        c.frameskip = v.frameskip;
        c.max_instr = v.max_instructions;
        c.prg_ram = v.prg_ram + (size_t)env * kPrgRamBytes;
        c.nt = v.nt + (size_t)env * kNtBytes;
        c.pal = v.pal + (size_t)env * kPalBytes;
        c.oam = v.oam + (size_t)env * kOamBytes;
        c.prg_lo = kBoard && v.mapper == kMapperUxrom ? 0xC000u : 0x8000u;
        c.prg_writes = kBoard;

        EnvRecord rec = v.rec[env];
        const uint32_t status_before = rec.status;
        const uint8_t action = act64 ? (uint8_t)(act64[env] & 0xFF) : act8[env];
        float reward;
        uint8_t done;
        if (kProfile) {
            run_env_step<false>(c, rec, action, reward, done, DeviceProfile{s_op, prof_pc});
        } else if (kOperand == 1) {
            DeviceAsync A;
            A.init(reinterpret_cast<uint32_t*>(s_async + (size_t)blockDim.x * 8 + tid * 4),
                   reinterpret_cast<unsigned long long*>(s_async + tid * 8));
            run_env_step_async(c, rec, action, reward, done, A);
        } else if (kOperand == 2) {
            DevicePreload A;
            run_env_step_async(c, rec, action, reward, done, A);
        } else if (kV2) {
            run_env_step_v2<false, kInterleave ? kEarlyInterleaved : kEarlyInPlace, kInterleave>(c, rec, action, reward,
                                                                                                 done);
        } else {
            run_env_step<false>(c, rec, action, reward, done);
        }
        uint8_t* row = v.ram + (size_t)env * kRamBytes;
        if (kInterleave) {  // back in place first; the slot's page is written over it below
            uint4* dst = reinterpret_cast<uint4*>(row);
#pragma unroll 4
            for (uint32_t q = 0; q < kRamBytes / 16; ++q)
                dst[q] = make_uint4(work[(4 * q + 0) * blockDim.x], work[(4 * q + 1) * blockDim.x],
                                    work[(4 * q + 2) * blockDim.x], work[(4 * q + 3) * blockDim.x]);
        }
        if (kHybrid) {  // back in place before a possible auto-reset rewrites the row
            uint4* dst = reinterpret_cast<uint4*>(row + slot_page);
#pragma unroll 4
            for (uint32_t q = 0; q < 16; ++q)
                dst[q] = make_uint4(s_zp[(4 * q + 0) * blockDim.x + tid], s_zp[(4 * q + 1) * blockDim.x + tid],
                                    s_zp[(4 * q + 2) * blockDim.x + tid], s_zp[(4 * q + 3) * blockDim.x + tid]);
        }
        const bool faulted = finish_env(v, env, rec, status_before, reward, done, flags & kStepDeviceApi,
                                        flags & kStepAutoReset);
        v.rec[env] = rec;
        if (faulted) atomicAdd(v.fault_count, 1u);
    }
    if (kProfile) {
        __syncthreads();
        for (uint32_t i = tid; i < 256; i += blockDim.x)
            if (s_op[i]) atomicAdd(&prof_op[i], (unsigned long long)s_op[i]);
    }
}

// --------------------------------------------------------------------------
// Env state save / load: one CTA per listed env copies its rows to or from a
// kStateBytes blob with 16-byte accesses.  Indices past the batch are skipped.
// --------------------------------------------------------------------------
__device__ __forceinline__ void copy_part(uint8_t* blob, uint8_t* row, uint32_t bytes, bool save) {
    uint4* b = reinterpret_cast<uint4*>(blob);
    uint4* r = reinterpret_cast<uint4*>(row);
    for (uint32_t i = threadIdx.x; i < bytes / 16; i += blockDim.x) {
        if (save) b[i] = r[i];
        else r[i] = b[i];
    }
}

__global__ void __launch_bounds__(128)
state_kernel(const BatchView* __restrict__ vp, const uint32_t* __restrict__ envs, uint8_t* __restrict__ blobs,
             uint32_t save) {
    const BatchView& v = *vp;
    const uint32_t env = envs[blockIdx.x];
    if (env >= v.num_envs) return;
    uint8_t* blob = blobs + (size_t)blockIdx.x * kStateBytes;
    const bool s = save != 0;
    copy_part(blob + kStateRec, reinterpret_cast<uint8_t*>(v.rec + env), 128, s);
    copy_part(blob + kStateRam, v.ram + (size_t)env * kRamBytes, kRamBytes, s);
    copy_part(blob + kStatePrgRam, v.prg_ram + (size_t)env * kPrgRamBytes, kPrgRamBytes, s);
    copy_part(blob + kStateNt, v.nt + (size_t)env * kNtBytes, kNtBytes, s);
    copy_part(blob + kStatePal, v.pal + (size_t)env * kPalBytes, kPalBytes, s);
    copy_part(blob + kStateOam, v.oam + (size_t)env * kOamBytes, kOamBytes, s);
    copy_part(blob + kStateSnapNt, v.snap_nt + (size_t)env * kNtBytes, kNtBytes, s);
    copy_part(blob + kStateSnapPal, v.snap_pal + (size_t)env * kPalBytes, kPalBytes, s);
    copy_part(blob + kStateSnapOam, v.snap_oam + (size_t)env * kOamBytes, kOamBytes, s);
    if (threadIdx.x == 0) {
        float* f = reinterpret_cast<float*>(blob + kStateOut);
        uint8_t* u = blob + kStateOut + 8;
        MapperState* ms = reinterpret_cast<MapperState*>(blob + kStateOut + 12);
        if (s) {
            f[0] = v.rewards[env];
            f[1] = v.last_rewards[env];
            u[0] = v.done[env];
            u[1] = v.last_done[env];
            *ms = v.mstate[env];
        } else {
            v.rewards[env] = f[0];
            v.last_rewards[env] = f[1];
            v.done[env] = u[0];
            v.last_done[env] = u[1];
            v.mstate[env] = *ms;
        }
    }
}

// --------------------------------------------------------------------------
// Resets.
// --------------------------------------------------------------------------
// One warp per env: lane 0 rewrites the record, the 32 lanes copy the byte
// rows with contiguous 16-byte stores (512 bytes per warp store).
__global__ void __launch_bounds__(128)
reset_kernel(const BatchView* __restrict__ vp, const uint8_t* __restrict__ mask, uint32_t full) {
    const BatchView& v = *vp;
    const uint32_t lane = threadIdx.x & 31u;
    const uint32_t env = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    if (env >= v.num_envs) return;
    if (!full && !mask[env]) return;  // both uniform across the warp
    if (lane == 0) {
        EnvRecord rec = v.rec[env];
        if (full) rec.episode = 0;
        else rec.episode++;
        reset_record(v, env, rec);
        if (full) {
            seed_presentation_record(rec);
            seed_presentation_board(v, env);
        }
        v.rec[env] = rec;
        v.rewards[env] = 0.0f;
        v.done[env] = 0;
    }
    reset_rows(v, env, lane, 32);
    if (full) {
        __syncwarp();  // the live rows are final before they are copied to the snapshot
        seed_presentation_rows(v, env, lane, 32);
    }
}

__global__ void poke_kernel(const BatchView* __restrict__ vp, uint32_t address, uint32_t value) {
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x * blockDim.x + threadIdx.x;
    if (env < v.num_envs) v.ram[(size_t)env * kRamBytes + (address & 0x7FF)] = (uint8_t)value;
}

// --------------------------------------------------------------------------
// Rendering, one CTA of kRenderThreads per env.  The env's presentation
// snapshot (nametables, palette, OAM) and the CHR ROM are staged in shared
// memory and each scanline's sprites are found once (a 64-bit row mask), so a
// pixel reads only shared memory and visits only the sprites on its row.
// --------------------------------------------------------------------------
constexpr uint32_t kRenderThreads = 256;
constexpr uint32_t kChrMax = 8192;

struct SnapSmem {
    uint8_t chr[kChrMax];
    uint8_t nt[kNtBytes];
    uint8_t pal[kPalBytes];
    uint8_t oam[kOamBytes];
    uint8_t res[32];  // resolved palette
    uint64_t rows[kFrameH];
    uint64_t cols[kFrameW / 8];
    uint16_t spat[64 * 16];  // sprite pattern rows, flips applied
};
static_assert(offsetof(SnapSmem, res) % 4 == 0 && offsetof(SnapSmem, oam) % 4 == 0,
              "the resolved palette and the OAM entries are read as 4-byte words");

__device__ __forceinline__ RenderEnv stage_snapshot(const BatchView& v, uint32_t env, SnapSmem& sm) {
    const uint32_t tid = threadIdx.x;
    uint32_t chr_size;
    const uint8_t* chr = snapshot_chr(v, env, chr_size);  // CNROM: the bank latched at vblank
    if (chr_size > kChrMax) chr_size = 0u;
    for (uint32_t i = tid; i < chr_size / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sm.chr)[i] = reinterpret_cast<const uint4*>(chr)[i];
    const uint4* nt = reinterpret_cast<const uint4*>(v.snap_nt + (size_t)env * kNtBytes);
    for (uint32_t i = tid; i < kNtBytes / 16; i += blockDim.x) reinterpret_cast<uint4*>(sm.nt)[i] = nt[i];
    if (tid < kOamBytes / 16)
        reinterpret_cast<uint4*>(sm.oam)[tid] = reinterpret_cast<const uint4*>(v.snap_oam + (size_t)env * kOamBytes)[tid];
    if (tid < kPalBytes / 16)
        reinterpret_cast<uint4*>(sm.pal)[tid] = reinterpret_cast<const uint4*>(v.snap_pal + (size_t)env * kPalBytes)[tid];
    __syncthreads();
    const RenderEnv e = render_env_at(v.rec[env], sm.nt, sm.pal, sm.oam, sm.chr, chr_size, v.horizontal);
    for (uint32_t y = tid; y < kFrameH; y += blockDim.x) sm.rows[y] = sprite_row_mask(e, y);
    if (tid < kFrameW / 8) sm.cols[tid] = sprite_col_mask(e, tid);
    if (tid < 32) sm.res[tid] = (uint8_t)rv_palette(e.lower, tid);
    const uint32_t h = (e.lower.ctrl & 0x20) ? 16 : 8;
    for (uint32_t i = tid; i < 64 * 16; i += blockDim.x)
        if (i % 16 < h) sm.spat[i] = (uint16_t)sprite_pattern_row(e.lower, i / 16, i % 16);
    __syncthreads();
    return e;
}

// Resident CTAs per SM the render kernels are compiled for (register caps of
// 40 and 48): both are issue-bound with a barrier per phase, so occupancy
// pays; 6 and 5 measured best (gray84 is limited to 5 by shared memory).
constexpr int kRenderMinBlocks = 6, kGrayMinBlocks = 5;

// Bits 0-3 of x as the bytes of a word: bit k -> byte k = 0xFF.
__device__ __forceinline__ uint32_t byte_mask(uint32_t x) {
    return (((x & 0xFu) * 0x00204081u) & 0x01010101u) * 0xFFu;
}

// The 4 bytes of a byte-compare result (0xFF or 0 each) as bits 0-3.
__device__ __forceinline__ uint32_t byte_flags(uint32_t m) { return ((m & 0x08040201u) * 0x01010101u) >> 24; }

// Bit k of x (k < 8) moved to bit 4k: the 8 bits spread over the nibbles.
__device__ __forceinline__ uint32_t spread_nibbles(uint32_t x) {
    x = (x | (x << 12)) & 0x000F000Fu;
    x = (x | (x << 6)) & 0x03030303u;
    return (x | (x << 3)) & 0x11111111u;
}

// Sprite-free pixels of one 8-column segment: row y, columns 8 c8 .. 8 c8 + 7,
// packed one per byte (pixel p in byte p % 4 of out[p / 4]).  `tiles` are the
// row's tile entries (slot j = scrolled tile column (sx >> 3) + j); a pixel is
// the byte of its palette group's word `group` picked by its pattern value
// (colours or luma, see group_colors).  Returns the sprites that may cover the
// segment (0: the values are final).
__device__ __forceinline__ uint64_t segment_background(const RenderEnv& e, const SnapSmem& sm, const uint32_t* tiles,
                                                       const uint32_t* group, uint32_t y, uint32_t c8,
                                                       uint32_t out[2]) {
    const RenderView& bv = bg_view(e, y);
    const RenderView& s = e.lower;
    uint32_t lo8 = 0, hi8 = 0, grp0 = 0, grp1 = 0, keep = 8;  // pixels p < keep are in tile slot c8
    if ((bv.mask & 0x08) && ((bv.mask & 0x02) || c8 != 0)) {
        const uint32_t e0 = tiles[c8], e1 = tiles[c8 + 1], fine = bv.sx & 7u;
        lo8 = ((((e0 & 0xFFu) << 8) | (e1 & 0xFFu)) << fine >> 8) & 0xFFu;  // pixel p at bit 7 - p
        hi8 = (((e0 & 0xFF00u) | ((e1 >> 8) & 0xFFu)) << fine >> 8) & 0xFFu;
        grp0 = (e0 >> 16) & 3u;
        grp1 = (e1 >> 16) & 3u;
        keep = 8u - fine;
    }
    // All 8 pixels with two byte permutes: selector nibble p is pixel p's
    // pattern value (0-3), plus 4 (a byte of w1) from pixel `keep` on.
    const uint32_t sel = spread_nibbles(__brev(lo8) >> 24) | (spread_nibbles(__brev(hi8) >> 24) << 1) |
                         (uint32_t)(0x44444444ull << (4u * keep));
    const uint32_t w0 = group[grp0], w1 = group[grp1];
    out[0] = __byte_perm(w0, w1, sel & 0xFFFFu);
    out[1] = __byte_perm(w0, w1, sel >> 16);
    return ((s.mask & 0x10) && ((s.mask & 0x04) || c8 != 0)) ? (sm.rows[y] & sm.cols[c8]) : 0ull;
}

// What a sprite-free pixel of palette group g shows for pattern value 0..3, as
// bytes: the backdrop for 0, else colour 4g+c -- or the backdrop again when
// that colour is index 0, which the reference composes as transparent
// (compose_pixel_tables' `bgc ? bgc : res[0]`).
__device__ __forceinline__ uint32_t group_colors(const SnapSmem& sm, uint32_t grp) {
    uint32_t w = sm.res[0];
    for (uint32_t c = 1; c < 4; ++c) {
        const uint32_t col = sm.res[grp * 4 + c];
        w |= (col ? col : (uint32_t)sm.res[0]) << (8 * c);
    }
    return w;
}

// The 8 pixels of a segment that sprites may cover, as compose_pixel_tables
// gives them pixel by pixel, with each sprite applied to all 8 at once: in
// index order a sprite claims the pixels not yet claimed where it is opaque and
// eligible (in front, or behind a background of colour 0).  Colour indices
// packed one per byte (pixel p in byte p), or their luma with kLuma.
template <bool kLuma>
__device__ __forceinline__ uint64_t sprite_segment(const RenderEnv& e, const SnapSmem& sm, const uint32_t* tiles,
                                                   const uint8_t* lut, uint32_t y, uint32_t c8, uint64_t spr) {
    const RenderView& bv = bg_view(e, y);
    const RenderView& s = e.lower;
    const uint32_t x0 = 8u * c8;
    uint32_t lo8 = 0, hi8 = 0, grp0 = 0, grp1 = 0, keep = 8;
    if ((bv.mask & 0x08) && ((bv.mask & 0x02) || c8 != 0)) {
        const uint32_t e0 = tiles[c8], e1 = tiles[c8 + 1], fine = bv.sx & 7u;
        lo8 = ((((e0 & 0xFFu) << 8) | (e1 & 0xFFu)) << fine >> 8) & 0xFFu;  // pixel p at bit 7 - p
        hi8 = (((e0 & 0xFF00u) | ((e1 >> 8) & 0xFFu)) << fine >> 8) & 0xFFu;
        grp0 = (e0 >> 16) & 3u;
        grp1 = (e1 >> 16) & 3u;
        keep = 8u - fine;
    }
    // Background colour indices of the 8 pixels, pixel p in byte p (0:
    // transparent): two byte permutes over the groups' raw palette words
    // (byte 0 zero, bytes 1-3 the group's colours), as in segment_background.
    const uint32_t* res32 = reinterpret_cast<const uint32_t*>(sm.res);
    const uint32_t sel = spread_nibbles(__brev(lo8) >> 24) | (spread_nibbles(__brev(hi8) >> 24) << 1) |
                         (uint32_t)(0x44444444ull << (4u * keep));
    const uint32_t r0 = res32[grp0] & 0xFFFFFF00u, r1 = res32[grp1] & 0xFFFFFF00u;
    const uint32_t bg_lo = __byte_perm(r0, r1, sel & 0xFFFFu), bg_hi = __byte_perm(r0, r1, sel >> 16);
    // bit p: the background a behind-background sprite is tested against is non-zero
    uint32_t bgop = byte_flags(__vcmpne4(bg_lo, 0u)) | (byte_flags(__vcmpne4(bg_hi, 0u)) << 4);
    bool bgop_ready = (int)y >= e.split;  // above the split the reference tests the lower view's background
    uint32_t spc_lo = 0, spc_hi = 0;       // colour of the claiming sprite, byte p
    uint32_t claimed = 0;
    while (spr && claimed != 0xFFu) {
        const uint32_t i = lowest_set(spr);
        spr &= spr - 1;
        const uint32_t so = reinterpret_cast<const uint32_t*>(sm.oam)[i];  // Y, tile, attributes, X
        const int d = (int)(so >> 24) - (int)x0;  // segment pixel of the sprite's column 0 (-7..7)
        const uint32_t pat = sm.spat[i * 16 + (y - (so & 0xFFu) - 1)];
        uint32_t plo = pat & 0xFFu, phi = pat >> 8;  // sprite pixel sx at bit sx
        if (d >= 0) {
            plo = (plo << d) & 0xFFu;
            phi = (phi << d) & 0xFFu;
        } else {
            plo >>= -d;
            phi >>= -d;
        }
        uint32_t take = (plo | phi) & ~claimed;
        const uint32_t attr = (so >> 16) & 0xFFu;
        if (take && (attr & 0x20)) {
            if (!bgop_ready) {
                bgop = 0;
                for (uint32_t p = 0; p < 8; ++p) bgop |= (rv_background(s, x0 + p, y) != 0 ? 1u : 0u) << p;
                bgop_ready = true;
            }
            take &= ~bgop;
        }
        if (!take) continue;
        claimed |= take;
        // The sprite palette's colours of its 8 pixels (pixel p's pattern
        // value in selector nibble p), kept where the sprite takes the pixel.
        const uint32_t pw = res32[4u + (attr & 3u)];
        const uint32_t ssel = spread_nibbles(plo) | (spread_nibbles(phi) << 1);
        spc_lo |= __byte_perm(pw, 0u, ssel & 0xFFFFu) & byte_mask(take & 0xFu);
        spc_hi |= __byte_perm(pw, 0u, ssel >> 16) & byte_mask(take >> 4);
    }
    // Claimed pixels show the sprite; the others the background, or the
    // backdrop res[0] where the background is transparent.
    const uint32_t back = (uint32_t)sm.res[0] * 0x01010101u;
    const uint32_t c_lo = (spc_lo & byte_mask(claimed & 0xFu)) |
                          ((bg_lo | (back & ~__vcmpne4(bg_lo, 0u))) & ~byte_mask(claimed & 0xFu));
    const uint32_t c_hi = (spc_hi & byte_mask(claimed >> 4)) |
                          ((bg_hi | (back & ~__vcmpne4(bg_hi, 0u))) & ~byte_mask(claimed >> 4));
    if (!kLuma) return (uint64_t)c_lo | ((uint64_t)c_hi << 32);
    uint64_t out = 0;
#pragma unroll
    for (uint32_t p = 0; p < 8; ++p)
        out |= (uint64_t)lut[((p < 4 ? c_lo : c_hi) >> (8 * (p & 3))) & 0xFFu] << (8 * p);
    return out;
}

// One strip of `rows` rows into `buf` (row r at buf + r * 256): tile entries,
// then (A) every 8-column segment from the tile entries, listing the segments
// a sprite may cover, then (B) those segments again, one per thread, composed
// with the sprites (sprite_segment).  kLuma stores luma (lut[colour]) instead
// of colours.
// Ends with a barrier; `list` holds rows * 32 entries.
template <bool kLuma>
__device__ __forceinline__ void render_strip(const RenderEnv& e, const SnapSmem& sm, uint32_t* tiles, uint32_t row0,
                                             uint32_t rows, const uint32_t* group, const uint8_t* lut, uint8_t* buf,
                                             uint16_t* list, uint32_t& count) {
    const uint32_t tid = threadIdx.x, lane = tid & 31u;
    for (uint32_t i = tid; i < rows * kRowTiles; i += blockDim.x) {
        const uint32_t r = i / kRowTiles, j = i - r * kRowTiles, y = row0 + r;
        tiles[i] = slot_entry(bg_view(e, y), y, j);
    }
    if (tid == 0) count = 0;
    __syncthreads();
    for (uint32_t sg = tid; sg < rows * 32u; sg += blockDim.x) {  // whole warps: rows * 32 is a warp multiple
        const uint32_t r = sg >> 5, c8 = sg & 31u;
        uint32_t w[2];
        const uint64_t spr = segment_background(e, sm, tiles + r * kRowTiles, group, row0 + r, c8, w);
        *reinterpret_cast<uint2*>(buf + r * kFrameW + 8u * c8) = make_uint2(w[0], w[1]);
        const uint32_t want = __ballot_sync(__activemask(), spr != 0);
        if (want) {
            const uint32_t first = __ffs(want) - 1u;
            uint32_t base = 0;
            if (lane == first) base = atomicAdd(&count, (uint32_t)__popc(want));
            base = __shfl_sync(__activemask(), base, first);
            if (spr) list[base + __popc(want & ((1u << lane) - 1u))] = (uint16_t)sg;
        }
    }
    __syncthreads();
    const uint32_t tasks = count;
    for (uint32_t t = tid; t < tasks; t += blockDim.x) {
        const uint32_t sg = list[t], r = sg >> 5, c8 = sg & 31u, y = row0 + r;
        const uint64_t px = sprite_segment<kLuma>(e, sm, tiles + r * kRowTiles, lut, y, c8, sm.rows[y] & sm.cols[c8]);
        *reinterpret_cast<uint2*>(buf + r * kFrameW + 8u * c8) = make_uint2((uint32_t)px, (uint32_t)(px >> 32));
    }
    __syncthreads();
}

// Colour-index or RGB frame, one CTA per env, strips of 20 rows rendered into
// shared memory (render_strip), then written out as 8-byte (index) or 3 x
// 8-byte (RGB) stores, each warp covering a contiguous stretch of the frame.
constexpr uint32_t kRenderStripRows = 20;
__global__ void __launch_bounds__(kRenderThreads, kRenderMinBlocks)
render_kernel(const BatchView* __restrict__ vp, uint8_t* __restrict__ out, uint32_t rgb, uint32_t env0) {
    __shared__ __align__(16) SnapSmem sm;
    __shared__ uint32_t s_tiles[kRenderStripRows * kRowTiles];
    __shared__ __align__(16) uint8_t s_buf[kRenderStripRows * kFrameW];
    __shared__ uint16_t s_list[kRenderStripRows * 32];
    __shared__ uint32_t s_rgb[64];
    __shared__ uint32_t s_group[4];
    __shared__ uint32_t s_count;
    const BatchView& v = *vp;
    const uint32_t env = env0 + blockIdx.x, tid = threadIdx.x;
    if (tid < 64)
        s_rgb[tid] = kPaletteRgb[tid * 3] | ((uint32_t)kPaletteRgb[tid * 3 + 1] << 8) |
                     ((uint32_t)kPaletteRgb[tid * 3 + 2] << 16);
    const RenderEnv e = stage_snapshot(v, env, sm);
    if (tid < 4) s_group[tid] = group_colors(sm, tid);  // read after render_strip's first barrier
    uint8_t* dst = out + (size_t)env * (kFrameW * kFrameH) * (rgb ? 3u : 1u);
    for (uint32_t row0 = 0; row0 < kFrameH; row0 += kRenderStripRows) {
        render_strip<false>(e, sm, s_tiles, row0, kRenderStripRows, s_group, nullptr, s_buf, s_list, s_count);
        uint8_t* d = dst + (size_t)row0 * kFrameW * (rgb ? 3u : 1u);
        for (uint32_t q = tid; q < kRenderStripRows * kFrameW / 8u; q += kRenderThreads) {
            const uint2 w = *reinterpret_cast<const uint2*>(s_buf + 8u * q);
            if (rgb) {
                uint32_t b[6];  // 8 pixels x 3 bytes
#pragma unroll
                for (uint32_t p = 0; p < 8; ++p) {
                    const uint32_t c = s_rgb[(((p < 4) ? w.x : w.y) >> (8 * (p & 3))) & 0x3Fu];
#pragma unroll
                    for (uint32_t ch = 0; ch < 3; ++ch) {
                        const uint32_t o = 3 * p + ch;
                        if (o % 4 == 0) b[o / 4] = 0;
                        b[o / 4] |= ((c >> (8 * ch)) & 0xFFu) << (8 * (o % 4));
                    }
                }
                uint2* o = reinterpret_cast<uint2*>(d + 24u * q);
                o[0] = make_uint2(b[0], b[1]);
                o[1] = make_uint2(b[2], b[3]);
                o[2] = make_uint2(b[4], b[5]);
            } else {
                *reinterpret_cast<uint2*>(d + 8u * q) = w;
            }
        }
        __syncthreads();  // s_buf is rewritten by the next strip
    }
}

// 84x84 grey observation, one CTA per env, on the same staged snapshot, in 6
// strips of 40 source rows (exactly 14 output rows each), assembled in shared
// memory and written out with one bulk copy per two strips:
//   1. the strip as luma (render_strip with the palette groups in luma);
//   2. horizontal area sums: output column ox covers source columns
//      64 ox / 21 .. + 3 with weights in units of 1/21 px;
//   3. vertical area sums over 3-4 rows (1/7 px units), rounded: the integer
//      (sum(luma * wx * wy) + 640) / 1280 of gray84_pixel, as a separable sum.
// Nothing but the 7,056-byte observation is written to global memory.
constexpr uint32_t kG84Rows = 40, kG84Out = 14;
static_assert(kFrameH % kG84Rows == 0 && kG84Rows * kGray == kG84Out * kFrameH, "strip geometry");
static_assert((2 * 14 * kGray) % 16 == 0 && (kGray * kGray) % 16 == 0,
              "bulk copies move multiples of 16 bytes to 16-byte aligned rows");

constexpr uint32_t kG84PairBytes = 2 * kG84Out * kGray;  // output rows of two strips: 2,352 B

struct Gray84Smem {
    __align__(16) uint8_t obs[kG84PairBytes];  // two strips of the observation, written out by one bulk copy
    uint32_t tiles[kG84Rows * kRowTiles];
    __align__(16) uint8_t luma[kG84Rows * kFrameW];
    uint16_t h[kG84Rows + 1][kGray];  // + a zero row read with weight 0
    uint16_t list[kG84Rows * 32];
    uint32_t hx[kGray];               // first source column | 4 weights x 5 bits from bit 8
    uint32_t vy[kG84Out];             // first strip row | 4 weights x 5 bits from bit 8
    uint32_t group_luma[4];           // luma version of group_colors
    uint32_t count;
    uint8_t lut[64];                  // luma of each NES colour
};

__device__ __forceinline__ uint32_t span_weights(uint32_t first, uint32_t unit, uint32_t lo, uint32_t hi) {
    uint32_t w = first;
    for (uint32_t j = 0; j < 4; ++j) {
        const uint32_t a = (first + j) * unit, b = a + unit;
        const uint32_t x = umin(b, hi) > umax(a, lo) ? umin(b, hi) - umax(a, lo) : 0u;
        w |= x << (8 + 5 * j);
    }
    return w;
}

__global__ void __launch_bounds__(kRenderThreads, kGrayMinBlocks)
gray84_kernel(const BatchView* __restrict__ vp, uint8_t* __restrict__ out, uint32_t env0) {
    __shared__ __align__(16) SnapSmem sm;
    __shared__ Gray84Smem g;
    const BatchView& v = *vp;
    const uint32_t env = env0 + blockIdx.x, tid = threadIdx.x;
    if (tid < 64) g.lut[tid] = (uint8_t)luma_of_rgb(kPaletteRgb[tid * 3], kPaletteRgb[tid * 3 + 1], kPaletteRgb[tid * 3 + 2]);
    if (tid < kGray) {
        g.hx[tid] = span_weights(64u * tid / 21u, 21u, 64u * tid, 64u * tid + 64u);
        g.h[kG84Rows][tid] = 0;
    }
    if (tid < kG84Out) g.vy[tid] = span_weights(20u * tid / 7u, 7u, 20u * tid, 20u * tid + 20u);
    const RenderEnv e = stage_snapshot(v, env, sm);  // its barriers also cover the tables above
    if (tid < 4) {  // read after render_strip's first barrier
        const uint32_t w = group_colors(sm, tid);
        uint32_t l = 0;
        for (uint32_t b = 0; b < 4; ++b) l |= (uint32_t)g.lut[(w >> (8 * b)) & 0xFFu] << (8 * b);
        g.group_luma[tid] = l;
    }
    uint8_t* dst = out + (size_t)env * kGray * kGray;
    for (uint32_t k = 0; k < kFrameH / kG84Rows; ++k) {
        render_strip<true>(e, sm, g.tiles, k * kG84Rows, kG84Rows, g.group_luma, g.lut, g.luma, g.list, g.count);
        // Threads 0..251: output column ox = tid % 84, every third row from tid / 84,
        // so each thread decodes its column's weights once.
        if (tid < 3 * kGray) {
            const uint32_t ox = tid % kGray, first = tid / kGray, w = g.hx[ox];
            const uint32_t w0 = (w >> 8) & 31u, w1 = (w >> 13) & 31u, w2 = (w >> 18) & 31u, w3 = (w >> 23) & 31u;
            const uint8_t* l = &g.luma[w & 0xFFu];
            for (uint32_t r = first; r < kG84Rows; r += 3) {
                const uint8_t* q = l + r * kFrameW;
                g.h[r][ox] = (uint16_t)(q[0] * w0 + q[1] * w1 + q[2] * w2 + q[3] * w3);
            }
        }
        // The previous pair's bulk copy has read the buffer (issued a strip ago,
        // so this wait is normally already satisfied) before it is written again.
        if (tid == 0 && (k & 1u) == 0 && k > 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        __syncthreads();
        if (tid < 3 * kGray) {
            const uint32_t ox = tid % kGray;
            for (uint32_t oyl = tid / kGray; oyl < kG84Out; oyl += 3) {
                const uint32_t w = g.vy[oyl], r = w & 0xFFu;
                const uint32_t acc = g.h[r][ox] * ((w >> 8) & 31u) + g.h[r + 1][ox] * ((w >> 13) & 31u) +
                                     g.h[r + 2][ox] * ((w >> 18) & 31u) + g.h[r + 3][ox] * ((w >> 23) & 31u);
                g.obs[((k & 1u) * kG84Out + oyl) * kGray + ox] = (uint8_t)((acc + 640u) / 1280u);
            }
        }
        // Every second strip, the pair's 2,352 bytes leave shared memory as one
        // bulk copy (TMA engine, no multicast): each thread fences its writes for
        // the async proxy, the barrier collects them, one thread issues the copy.
        if (k & 1u) asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncthreads();
        if ((k & 1u) && tid == 0) {
            const uint32_t src = static_cast<uint32_t>(__cvta_generic_to_shared(g.obs));
            asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst + (k / 2) * kG84PairBytes),
                         "r"(src), "r"(kG84PairBytes)
                         : "memory");
            asm volatile("cp.async.bulk.commit_group;" ::: "memory");
        }
    }
    // The CTA's shared memory must outlive the last copy's read of it.
    if (tid == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// --------------------------------------------------------------------------
// Launchers.
// --------------------------------------------------------------------------
size_t step_smem_bytes() { return kPrgSmem + kDecSmem + (size_t)kStepSlots * kRamBytes; }

// In-place step placements: (zero-page slot, operand mode, interleaved copy).
struct GlobalPlacement {
    bool hybrid;
    int operand;  // 0 read at execution, 1 cp.async ahead, 2 register load ahead
    bool interleave;
};
constexpr GlobalPlacement global_placement(uint32_t variant) {
    switch (variant) {
        case kStepHybridRam: case kStepHybridStackRam: return {true, 0, false};
        case kStepGlobalAsync: return {false, 1, false};
        case kStepHybridAsync: return {true, 1, false};
        case kStepInterleaved: return {true, 0, true};
        case kStepInterleavedAsync: return {true, 1, true};
        case kStepGlobalPreload: return {false, 2, false};
        case kStepHybridPreload: return {true, 2, false};
        case kStepInterleavedPreload: return {true, 2, true};
        default: return {false, 0, false};  // kStepGlobalRam
    }
}

size_t global_step_smem(uint32_t variant, uint32_t threads) {
    const GlobalPlacement g = global_placement(variant);
    return kPrgSmem + kDecSmem + (g.hybrid ? (size_t)threads * 256 : 0) +
           (g.operand == 1 ? (size_t)threads * kAsyncSmemPerLane : 0);
}

template <uint32_t kVariant, bool kBoard = false>
cudaError_t configure_global() {
    constexpr GlobalPlacement g = global_placement(kVariant);
    return cudaFuncSetAttribute(step_kernel_global<false, g.hybrid, g.operand, g.interleave, kBoard>,
                                cudaFuncAttributeMaxDynamicSharedMemorySize,
                                (int)global_step_smem(kVariant, kGlobalMaxThreads));
}

template <uint32_t kVariant, bool kBoard = false>
void launch_global(const BatchView* dv, uint32_t num_envs, const uint8_t* act8, const long long* act64,
                   uint32_t flags, uint32_t threads, cudaStream_t s) {
    constexpr GlobalPlacement g = global_placement(kVariant);
    const uint32_t blocks = (num_envs + threads - 1) / threads;
    step_kernel_global<false, g.hybrid, g.operand, g.interleave, kBoard><<<blocks, threads,
                                                                          global_step_smem(kVariant, threads), s>>>(
        dv, act8, act64, flags, nullptr, nullptr, kVariant == kStepHybridStackRam ? 0x100u : 0u);
}

cudaError_t configure_kernels() {
    cudaError_t e = cudaFuncSetAttribute(step_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)step_smem_bytes());
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(step_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)step_smem_bytes());
    if (e == cudaSuccess) e = configure_global<kStepGlobalRam, true>();
    if (e == cudaSuccess) e = configure_global<kStepHybridRam, true>();
    if (e == cudaSuccess) e = configure_global<kStepGlobalRam>();
    if (e == cudaSuccess) e = configure_global<kStepHybridRam>();
    if (e == cudaSuccess) e = configure_global<kStepGlobalAsync>();
    if (e == cudaSuccess) e = configure_global<kStepHybridAsync>();
    if (e == cudaSuccess) e = configure_global<kStepInterleaved>();
    if (e == cudaSuccess) e = configure_global<kStepInterleavedAsync>();
    if (e == cudaSuccess) e = configure_global<kStepGlobalPreload>();
    if (e == cudaSuccess) e = configure_global<kStepHybridPreload>();
    if (e == cudaSuccess) e = configure_global<kStepInterleavedPreload>();
    // step_profile's instantiations (above the 48 KB default with the 16 KB v2 table reserved)
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(step_kernel_global<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)(kPrgSmem + kDecSmem));
    if (e == cudaSuccess)
        e = cudaFuncSetAttribute(step_kernel_global<true, false, 0, false, true>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize, (int)(kPrgSmem + kDecSmem));
    return e;
}

// Threads per in-place step CTA: one CTA per SM when the batch fits in one
// wave (65,536 envs on 148 SMs -> 448 threads x 147 CTAs), so every SM holds the
// same number of warps; larger batches use 448-thread CTAs in several waves.
uint32_t global_step_threads(uint32_t num_envs, uint32_t num_sms) {
    const uint32_t per_sm = (num_envs + num_sms - 1) / (num_sms ? num_sms : 1);
    uint32_t t = (per_sm + 31) / 32 * 32;
    if (t < 32) t = 32;
    if (t > kGlobalMaxThreads) t = kGlobalMaxThreads;
    return t;
}

cudaError_t launch_step(const BatchView* dv, uint32_t num_envs, const uint8_t* act8, const long long* act64,
                        uint32_t flags, uint32_t variant, uint32_t threads, cudaStream_t s,
                        unsigned long long* prof_op, unsigned long long* prof_pc, bool board) {
    if (prof_op || prof_pc) {  // step_profile: the in-place kernel with histograms
        if (!prof_op || !prof_pc) return cudaErrorInvalidValue;
        const uint32_t blocks = (num_envs + threads - 1) / threads;
        if (board)
            step_kernel_global<true, false, 0, false, true><<<blocks, threads, kPrgSmem + kDecSmem, s>>>(
                dv, act8, act64, flags, prof_op, prof_pc, 0);
        else
            step_kernel_global<true, false><<<blocks, threads, kPrgSmem + kDecSmem, s>>>(dv, act8, act64, flags,
                                                                                        prof_op, prof_pc, 0);
    } else if (board) {  // UxROM / CNROM: the shared, in-place and hybrid placements
        if (variant == kStepGlobalRam) {
            launch_global<kStepGlobalRam, true>(dv, num_envs, act8, act64, flags, threads, s);
        } else if (variant == kStepHybridRam) {
            launch_global<kStepHybridRam, true>(dv, num_envs, act8, act64, flags, threads, s);
        } else {
            const uint32_t blocks = (num_envs + kStepSlots - 1) / kStepSlots;
            step_kernel<true><<<blocks, kStepSlots, step_smem_bytes(), s>>>(dv, act8, act64, flags);
        }
    } else {
        switch (variant) {
            case kStepGlobalRam: launch_global<kStepGlobalRam>(dv, num_envs, act8, act64, flags, threads, s); break;
            case kStepHybridRam: launch_global<kStepHybridRam>(dv, num_envs, act8, act64, flags, threads, s); break;
            case kStepHybridStackRam:
                launch_global<kStepHybridStackRam>(dv, num_envs, act8, act64, flags, threads, s);
                break;
            case kStepGlobalAsync: launch_global<kStepGlobalAsync>(dv, num_envs, act8, act64, flags, threads, s); break;
            case kStepHybridAsync: launch_global<kStepHybridAsync>(dv, num_envs, act8, act64, flags, threads, s); break;
            case kStepInterleaved: launch_global<kStepInterleaved>(dv, num_envs, act8, act64, flags, threads, s); break;
            case kStepInterleavedAsync:
                launch_global<kStepInterleavedAsync>(dv, num_envs, act8, act64, flags, threads, s);
                break;
            case kStepGlobalPreload:
                launch_global<kStepGlobalPreload>(dv, num_envs, act8, act64, flags, threads, s);
                break;
            case kStepHybridPreload:
                launch_global<kStepHybridPreload>(dv, num_envs, act8, act64, flags, threads, s);
                break;
            case kStepInterleavedPreload:
                launch_global<kStepInterleavedPreload>(dv, num_envs, act8, act64, flags, threads, s);
                break;
            default: {
                const uint32_t blocks = (num_envs + kStepSlots - 1) / kStepSlots;
                step_kernel<false><<<blocks, kStepSlots, step_smem_bytes(), s>>>(dv, act8, act64, flags);
            }
        }
    }
    return cudaGetLastError();
}

cudaError_t launch_reset(const BatchView* dv, uint32_t num_envs, const uint8_t* mask, bool full, cudaStream_t s) {
    const uint64_t threads = (uint64_t)num_envs * 32;  // a warp per env
    reset_kernel<<<(uint32_t)((threads + 127) / 128), 128, 0, s>>>(dv, mask, full ? 1u : 0u);
    return cudaGetLastError();
}

cudaError_t launch_state(const BatchView* dv, const uint32_t* envs, uint32_t count, uint8_t* blobs, bool save,
                         cudaStream_t s) {
    if (count) state_kernel<<<count, 128, 0, s>>>(dv, envs, blobs, save ? 1u : 0u);
    return cudaGetLastError();
}

cudaError_t launch_poke(const BatchView* dv, uint32_t num_envs, uint32_t address, uint32_t value, cudaStream_t s) {
    poke_kernel<<<(num_envs + 255) / 256, 256, 0, s>>>(dv, address, value);
    return cudaGetLastError();
}

// Envs [env0, env0 + count) into their rows of `out` (row = env index).
cudaError_t launch_render(const BatchView* dv, uint32_t env0, uint32_t count, uint8_t* out, int mode, cudaStream_t s) {
    if (!count) return cudaSuccess;
    if (mode == 2) {
        gray84_kernel<<<count, kRenderThreads, 0, s>>>(dv, out, env0);
    } else {
        render_kernel<<<count, kRenderThreads, 0, s>>>(dv, out, mode == 0 ? 1u : 0u, env0);
    }
    return cudaGetLastError();
}

}  // namespace nesle
