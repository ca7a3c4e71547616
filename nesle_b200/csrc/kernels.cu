// kernels.cu -- sm_100a kernels of the batched NES core.
//
//   step_kernel_global  one env-step per thread, env RAM in place (default)
//   step_kernel     one env-step per thread, env RAM staged in shared memory
//   reset_kernel    masked or full snapshot/cold reset
//   poke_kernel     one RAM byte in every env
//   render_kernel   colour index or RGB per pixel from the presentation snapshot
//   gray84_kernel   84x84 area-resampled luma observation
#include <cuda_runtime.h>
#include <stdlib.h>

#include "kernels.h"
#include "nes_core.cuh"
#include "nes_render.cuh"

namespace nesle {

__constant__ EntryTable kEntriesConst = dt::build_entries();
__constant__ uint8_t kPaletteRgb[192] = NESLE_PALETTE_RGB;

// --------------------------------------------------------------------------
// Env step with RAM staged in shared memory.  One CTA = kStepSlots envs =
// kStepSlots threads: 32 KB PRG + 8 KB execution entries + kStepSlots x 2 KB
// interleaved RAM.  Kept as the alternative placement (NESLE_STEP_KERNEL=shared);
// the in-place kernel below is the default.
// --------------------------------------------------------------------------
constexpr uint32_t kPrgSmem = 32768 + 16;  // +16: the two-word fetch at $FFFC-$FFFD reads one word past the ROM
constexpr uint32_t kDecSmem = 256 * sizeof(Entry);

__device__ __forceinline__ uint32_t* ram_word(uint8_t* slot, uint32_t word) {
    return reinterpret_cast<uint32_t*>(slot + word * 4u * kStepSlots);
}

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
    const uint4* ent_src = reinterpret_cast<const uint4*>(&kEntriesConst);
    for (uint32_t i = tid; i < kDecSmem / 16; i += blockDim.x) reinterpret_cast<uint4*>(s_dec)[i] = ent_src[i];

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
    c.view = vp;
    c.env = env;
    c.frameskip = v.frameskip;
    c.max_instr = v.max_instructions;
    c.prg_ram = v.prg_ram + (size_t)env * kPrgRamBytes;
    c.nt = v.nt + (size_t)env * kNtBytes;
    c.pal = v.pal + (size_t)env * kPalBytes;
    c.oam = v.oam + (size_t)env * kOamBytes;

    EnvRecord rec = v.rec[env];
    const uint32_t status_before = rec.status;
    const uint8_t action = act64 ? (uint8_t)(act64[env] & 0xFF) : act8[env];
    float reward;
    uint8_t done;
    run_env_step(c, rec, action, reward, done);

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

// kHybrid: each env's zero page ($0000-$00FF) is staged into shared memory for
// the launch (interleaved 4 bytes per lane: every lane keeps to its own bank)
// and written back before the env's done/auto-reset; the rest of RAM stays in
// place.  Zero-page operands and indirect pointers then cost a shared-memory
// access instead of a global one.
template <bool kProfile, bool kHybrid>
__global__ void __launch_bounds__(kGlobalMaxThreads, 1)
step_kernel_global(const BatchView* __restrict__ vp, const uint8_t* __restrict__ act8,
                   const long long* __restrict__ act64, uint32_t flags, unsigned long long* __restrict__ prof_op,
                   unsigned long long* __restrict__ prof_pc, uint32_t slot_page) {
    extern __shared__ __align__(16) uint8_t smem[];
    __shared__ uint32_t s_op[kProfile ? 256 : 1];
    uint8_t* s_prg = smem;
    Entry* s_dec = reinterpret_cast<Entry*>(smem + kPrgSmem);
    uint32_t* s_zp = reinterpret_cast<uint32_t*>(smem + kPrgSmem + kDecSmem);  // [64 words][blockDim lanes]
    const BatchView& v = *vp;
    const uint32_t tid = threadIdx.x;
    const uint4* prg_src = reinterpret_cast<const uint4*>(v.prg);
    for (uint32_t i = tid; i < 2048; i += blockDim.x) reinterpret_cast<uint4*>(s_prg)[i] = prg_src[i];
    if (tid == 0) reinterpret_cast<uint4*>(s_prg)[2048] = make_uint4(0, 0, 0, 0);
    const uint4* ent_src = reinterpret_cast<const uint4*>(&kEntriesConst);
    for (uint32_t i = tid; i < kDecSmem / 16; i += blockDim.x) reinterpret_cast<uint4*>(s_dec)[i] = ent_src[i];
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
        c.prg = s_prg;
        c.dec = s_dec;
        c.view = vp;
        c.env = env;
        c.frameskip = v.frameskip;
        c.max_instr = v.max_instructions;
        c.prg_ram = v.prg_ram + (size_t)env * kPrgRamBytes;
        c.nt = v.nt + (size_t)env * kNtBytes;
        c.pal = v.pal + (size_t)env * kPalBytes;
        c.oam = v.oam + (size_t)env * kOamBytes;

        EnvRecord rec = v.rec[env];
        const uint32_t status_before = rec.status;
        const uint8_t action = act64 ? (uint8_t)(act64[env] & 0xFF) : act8[env];
        float reward;
        uint8_t done;
        if (kProfile) run_env_step<false>(c, rec, action, reward, done, DeviceProfile{s_op, prof_pc});
        else run_env_step<false>(c, rec, action, reward, done);
        if (kHybrid) {  // back in place before a possible auto-reset rewrites the row
            uint4* dst = reinterpret_cast<uint4*>(c.ram + slot_page);
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
        if (s) {
            f[0] = v.rewards[env];
            f[1] = v.last_rewards[env];
            u[0] = v.done[env];
            u[1] = v.last_done[env];
        } else {
            v.rewards[env] = f[0];
            v.last_rewards[env] = f[1];
            v.done[env] = u[0];
            v.last_done[env] = u[1];
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
        if (full) seed_presentation_record(rec);
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

__device__ __forceinline__ RenderEnv stage_snapshot(const BatchView& v, uint32_t env, SnapSmem& sm) {
    const uint32_t tid = threadIdx.x;
    const uint32_t chr_size = v.chr_size <= kChrMax ? v.chr_size : 0u;
    for (uint32_t i = tid; i < chr_size / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sm.chr)[i] = reinterpret_cast<const uint4*>(v.chr)[i];
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

// Per strip of 20 rows: the background tile entries of each row.
struct StripSmem {
    uint32_t tiles[kGrayStripRows][kRowTiles];
};

// One strip of 20 rows: the tile entries (built by the whole CTA), then one
// pixel per thread from its row's entries and the sprite tables.
__device__ __forceinline__ void build_strip(const RenderEnv& e, uint32_t row0, StripSmem& st) {
    for (uint32_t i = threadIdx.x; i < kGrayStripRows * kRowTiles; i += blockDim.x) {
        const uint32_t r = i / kRowTiles, j = i % kRowTiles, y = row0 + r;
        st.tiles[r][j] = slot_entry(bg_view(e, y), y, j);
    }
}
__device__ __forceinline__ uint32_t strip_pixel(const RenderEnv& e, const SnapSmem& sm, const StripSmem& st,
                                                uint32_t row0, uint32_t x, uint32_t y) {
    const RenderView& v = bg_view(e, y);
    const uint32_t bgc = bg_from_entry_tables(v, sm.res, st.tiles[y - row0][tile_slot(v, x)], x, v.sx + x);
    return compose_pixel_tables(e, sm.res, x, y, bgc, sm.rows[y] & sm.cols[x >> 3], sm.spat);
}

__global__ void __launch_bounds__(kRenderThreads)
render_kernel(const BatchView* __restrict__ vp, uint8_t* __restrict__ out, uint32_t rgb) {
    __shared__ __align__(16) SnapSmem sm;
    __shared__ StripSmem st;
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x;
    const RenderEnv e = stage_snapshot(v, env, sm);
    uint8_t* dst = out + (size_t)env * (kFrameW * kFrameH) * (rgb ? 3u : 1u);
    for (uint32_t row0 = 0; row0 < kFrameH; row0 += kGrayStripRows) {
        build_strip(e, row0, st);
        __syncthreads();
        for (uint32_t p = threadIdx.x; p < kGrayStripRows * kFrameW; p += kRenderThreads) {
            const uint32_t y = row0 + p / kFrameW, x = p % kFrameW;
            const uint32_t c = strip_pixel(e, sm, st, row0, x, y);
            const size_t q = (size_t)y * kFrameW + x;
            if (rgb) {
                dst[q * 3 + 0] = kPaletteRgb[c * 3 + 0];
                dst[q * 3 + 1] = kPaletteRgb[c * 3 + 1];
                dst[q * 3 + 2] = kPaletteRgb[c * 3 + 2];
            } else {
                dst[q] = (uint8_t)c;
            }
        }
        __syncthreads();
    }
}

// 84x84 grey observation, one CTA per env, on the same staged snapshot.  The
// frame is done in 12 strips of 20 source rows: every source pixel is rendered
// once into a shared luma strip, from which the strip's 7 x 84 outputs are
// area-summed (gray84_pixel).  Nothing but the 7,056-byte observation is written.
__global__ void __launch_bounds__(kRenderThreads)
gray84_kernel(const BatchView* __restrict__ vp, uint8_t* __restrict__ out) {
    __shared__ __align__(16) SnapSmem sm;
    __shared__ StripSmem st;
    __shared__ __align__(16) uint8_t s_luma[kGrayStripRows * kFrameW];
    __shared__ uint8_t s_lut[64];
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x, tid = threadIdx.x;
    if (tid < 64) s_lut[tid] = (uint8_t)luma_of_rgb(kPaletteRgb[tid * 3], kPaletteRgb[tid * 3 + 1], kPaletteRgb[tid * 3 + 2]);
    const RenderEnv e = stage_snapshot(v, env, sm);  // its barriers also cover s_lut

    uint8_t* dst = out + (size_t)env * kGray * kGray;
    for (uint32_t k = 0; k < kFrameH / kGrayStripRows; ++k) {
        const uint32_t row0 = k * kGrayStripRows;
        build_strip(e, row0, st);
        __syncthreads();
        for (uint32_t p = tid; p < kGrayStripRows * kFrameW; p += kRenderThreads) {
            const uint32_t y = row0 + p / kFrameW, x = p % kFrameW;
            s_luma[p] = s_lut[strip_pixel(e, sm, st, row0, x, y)];
        }
        __syncthreads();
        for (uint32_t o = tid; o < kGrayStripOut * kGray; o += kRenderThreads) {
            const uint32_t oy = k * kGrayStripOut + o / kGray, ox = o % kGray;
            dst[oy * kGray + ox] = (uint8_t)gray84_pixel(s_luma, row0, ox, oy);
        }
        __syncthreads();
    }
}

// --------------------------------------------------------------------------
// Launchers.
// --------------------------------------------------------------------------
size_t step_smem_bytes() { return kPrgSmem + kDecSmem + (size_t)kStepSlots * kRamBytes; }

constexpr size_t kHybridSmemMax = kPrgSmem + kDecSmem + (size_t)kGlobalMaxThreads * 256;

cudaError_t configure_kernels() {
    cudaError_t e = cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)step_smem_bytes());
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(step_kernel_global<false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)kHybridSmemMax);
    if (e != cudaSuccess) return e;
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
                        unsigned long long* prof_op, unsigned long long* prof_pc) {
    if (prof_op || prof_pc) {  // step_profile: the in-place kernel with histograms
        if (!prof_op || !prof_pc) return cudaErrorInvalidValue;
        const uint32_t blocks = (num_envs + threads - 1) / threads;
        step_kernel_global<true, false><<<blocks, threads, kPrgSmem + kDecSmem, s>>>(dv, act8, act64, flags, prof_op,
                                                                                    prof_pc, 0);
    } else if (variant == kStepGlobalRam) {
        const uint32_t blocks = (num_envs + threads - 1) / threads;
        step_kernel_global<false, false><<<blocks, threads, kPrgSmem + kDecSmem, s>>>(dv, act8, act64, flags, nullptr,
                                                                                      nullptr, 0);
    } else if (variant == kStepHybridRam || variant == kStepHybridStackRam) {
        const uint32_t blocks = (num_envs + threads - 1) / threads;
        step_kernel_global<false, true><<<blocks, threads, kPrgSmem + kDecSmem + (size_t)threads * 256, s>>>(
            dv, act8, act64, flags, nullptr, nullptr, variant == kStepHybridStackRam ? 0x100u : 0u);
    } else {
        const uint32_t blocks = (num_envs + kStepSlots - 1) / kStepSlots;
        step_kernel<<<blocks, kStepSlots, step_smem_bytes(), s>>>(dv, act8, act64, flags);
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

cudaError_t launch_render(const BatchView* dv, uint32_t num_envs, uint8_t* out, int mode, cudaStream_t s) {
    if (mode == 2) {
        gray84_kernel<<<num_envs, kRenderThreads, 0, s>>>(dv, out);
    } else {
        render_kernel<<<num_envs, kRenderThreads, 0, s>>>(dv, out, mode == 0 ? 1u : 0u);
    }
    return cudaGetLastError();
}

}  // namespace nesle
