// kernels.cu -- sm_100a kernels of the batched NES core.
//
//   step_kernel_global  one env-step per thread, env RAM in place (default)
//   step_kernel     one env-step per thread, env RAM staged in shared memory
//   reset_kernel    masked or full snapshot/cold reset
//   poke_kernel     one RAM byte in every env
//   render_kernel   colour index or RGB per pixel from the presentation snapshot
//   gray84_kernel   84x84 area-resampled luma observation
#include <cuda_runtime.h>

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
// Env step, RAM in place.  The env's RAM row stays in global memory (L2
// resident for moderate batches) and only PRG + decode table are staged, so a
// CTA is 256 envs and every env of a 65,536-env batch is resident at once:
// warp parallelism, not shared-memory latency, hides the memory latency.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(kGlobalMaxThreads, 1)
step_kernel_global(const BatchView* __restrict__ vp, const uint8_t* __restrict__ act8,
                   const long long* __restrict__ act64, uint32_t flags) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint8_t* s_prg = smem;
    Entry* s_dec = reinterpret_cast<Entry*>(smem + kPrgSmem);
    const BatchView& v = *vp;
    const uint32_t tid = threadIdx.x;
    const uint4* prg_src = reinterpret_cast<const uint4*>(v.prg);
    for (uint32_t i = tid; i < 2048; i += blockDim.x) reinterpret_cast<uint4*>(s_prg)[i] = prg_src[i];
    if (tid == 0) reinterpret_cast<uint4*>(s_prg)[2048] = make_uint4(0, 0, 0, 0);
    const uint4* ent_src = reinterpret_cast<const uint4*>(&kEntriesConst);
    for (uint32_t i = tid; i < kDecSmem / 16; i += blockDim.x) reinterpret_cast<uint4*>(s_dec)[i] = ent_src[i];
    __syncthreads();
    const uint32_t env = blockIdx.x * blockDim.x + tid;
    if (env >= v.num_envs) return;

    Ctx c;
    c.ram = v.ram + (size_t)env * kRamBytes;
    c.slots = 1;
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
    run_env_step<false>(c, rec, action, reward, done);
    const bool faulted = finish_env(v, env, rec, status_before, reward, done, flags & kStepDeviceApi,
                                    flags & kStepAutoReset);
    v.rec[env] = rec;
    if (faulted) atomicAdd(v.fault_count, 1u);
}

// --------------------------------------------------------------------------
// Resets.
// --------------------------------------------------------------------------
__global__ void reset_kernel(const BatchView* __restrict__ vp, const uint8_t* __restrict__ mask, uint32_t full) {
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x * blockDim.x + threadIdx.x;
    if (env >= v.num_envs) return;
    if (!full && !mask[env]) return;
    EnvRecord rec = v.rec[env];
    if (full) rec.episode = 0;
    else rec.episode++;
    reset_env(v, env, rec);
    v.rewards[env] = 0.0f;
    v.done[env] = 0;
    if (full) seed_presentation(v, env, rec);
    v.rec[env] = rec;
}

__global__ void poke_kernel(const BatchView* __restrict__ vp, uint32_t address, uint32_t value) {
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x * blockDim.x + threadIdx.x;
    if (env < v.num_envs) v.ram[(size_t)env * kRamBytes + (address & 0x7FF)] = (uint8_t)value;
}

// --------------------------------------------------------------------------
// Rendering.  grid.x = env, grid.y = band of 16 rows; 256 threads = 1 column.
// --------------------------------------------------------------------------
__global__ void __launch_bounds__(256)
render_kernel(const BatchView* __restrict__ vp, uint8_t* __restrict__ out, uint32_t rgb) {
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x;
    const RenderEnv e = render_env(v, v.rec[env], env);
    const uint32_t x = threadIdx.x;
    for (uint32_t y = blockIdx.y * 16; y < blockIdx.y * 16 + 16; ++y) {
        const uint32_t c = render_pixel(e, x, y);
        const size_t px = (size_t)env * (kFrameW * kFrameH) + y * kFrameW + x;
        if (rgb) {
            out[px * 3 + 0] = kPaletteRgb[c * 3 + 0];
            out[px * 3 + 1] = kPaletteRgb[c * 3 + 1];
            out[px * 3 + 2] = kPaletteRgb[c * 3 + 2];
        } else {
            out[px] = (uint8_t)c;
        }
    }
}

// 84x84 grey: output (ox, oy) is the integer area average of the luma of the
// source pixels it covers.  In units of 1/21 px horizontally and 1/7 px
// vertically, source column sx spans [21 sx, 21 sx + 21) and output column ox
// [64 ox, 64 ox + 64); source row sy spans [7 sy, 7 sy + 7) and output row oy
// [20 oy, 20 oy + 20).  Result = (sum(luma * wx * wy) + 640) / 1280.
__device__ __forceinline__ uint32_t luma_of(uint32_t c) {
    return (299u * kPaletteRgb[c * 3] + 587u * kPaletteRgb[c * 3 + 1] + 114u * kPaletteRgb[c * 3 + 2] + 500u) / 1000u;
}

__global__ void __launch_bounds__(128)
gray84_kernel(const BatchView* __restrict__ vp, uint8_t* __restrict__ out) {
    const BatchView& v = *vp;
    const uint32_t env = blockIdx.x;
    const RenderEnv e = render_env(v, v.rec[env], env);
    for (uint32_t o = threadIdx.x; o < kGray * kGray; o += blockDim.x) {
        const uint32_t oy = o / kGray, ox = o % kGray;
        const uint32_t y0 = (20 * oy) / 7, y1 = (20 * oy + 19) / 7;
        const uint32_t x0 = (64 * ox) / 21, x1 = (64 * ox + 63) / 21;
        uint32_t acc = 0;
        for (uint32_t sy = y0; sy <= y1; ++sy) {
            const uint32_t wy = min(7 * sy + 7, 20 * oy + 20) - max(7 * sy, 20 * oy);
            for (uint32_t sx = x0; sx <= x1; ++sx) {
                const uint32_t wx = min(21 * sx + 21, 64 * ox + 64) - max(21 * sx, 64 * ox);
                acc += luma_of(render_pixel(e, sx, sy)) * wx * wy;
            }
        }
        out[(size_t)env * kGray * kGray + o] = (uint8_t)((acc + 640) / 1280);
    }
}

// --------------------------------------------------------------------------
// Launchers.
// --------------------------------------------------------------------------
size_t step_smem_bytes() { return kPrgSmem + kDecSmem + (size_t)kStepSlots * kRamBytes; }

cudaError_t configure_kernels() {
    return cudaFuncSetAttribute(step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)step_smem_bytes());
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
                        uint32_t flags, uint32_t variant, uint32_t threads, cudaStream_t s) {
    if (variant == kStepGlobalRam) {
        const uint32_t blocks = (num_envs + threads - 1) / threads;
        step_kernel_global<<<blocks, threads, kPrgSmem + kDecSmem, s>>>(dv, act8, act64, flags);
    } else {
        const uint32_t blocks = (num_envs + kStepSlots - 1) / kStepSlots;
        step_kernel<<<blocks, kStepSlots, step_smem_bytes(), s>>>(dv, act8, act64, flags);
    }
    return cudaGetLastError();
}

cudaError_t launch_reset(const BatchView* dv, uint32_t num_envs, const uint8_t* mask, bool full, cudaStream_t s) {
    reset_kernel<<<(num_envs + 127) / 128, 128, 0, s>>>(dv, mask, full ? 1u : 0u);
    return cudaGetLastError();
}

cudaError_t launch_poke(const BatchView* dv, uint32_t num_envs, uint32_t address, uint32_t value, cudaStream_t s) {
    poke_kernel<<<(num_envs + 255) / 256, 256, 0, s>>>(dv, address, value);
    return cudaGetLastError();
}

cudaError_t launch_render(const BatchView* dv, uint32_t num_envs, uint8_t* out, int mode, cudaStream_t s) {
    if (mode == 2) {
        gray84_kernel<<<num_envs, 128, 0, s>>>(dv, out);
    } else {
        render_kernel<<<dim3(num_envs, kFrameH / 16), 256, 0, s>>>(dv, out, mode == 0 ? 1u : 0u);
    }
    return cudaGetLastError();
}

}  // namespace nesle
