/*
 * nesle_b200.h -- C ABI of the B200 batched NES env-step core.
 *
 * This is the drop-in boundary for the reference's pybind11 module
 * `nesle._cuda_core` (hbofz/NeSLE cpp/bindings/cuda_module.cu).  Every entry
 * point names the binding method it replaces.  Plain pointers and sizes only;
 * no torch or pybind types.  All functions return NESLE_OK (0) or an error
 * code, with a message retrievable through nesle_last_error() (thread-local).
 * Error classes mirror the binding's exception mapping (cuda_module.cu:185-189):
 * NESLE_ERR_INVALID <-> std::invalid_argument (Python ValueError),
 * NESLE_ERR_RUNTIME and NESLE_ERR_CUDA <-> std::runtime_error (RuntimeError).
 *
 * Streams: every call that issues device work takes a cudaStream_t as `void*`
 * (NULL = the legacy default stream, which is what the reference uses) and
 * records a completion event; nesle_stream_wait() orders another stream after
 * that work (the DLPack producer/consumer hand-off) without a host sync.
 */
#ifndef NESLE_B200_H
#define NESLE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define NESLE_OK 0
#define NESLE_ERR_INVALID 1 /* bad argument, ROM or snapshot  -> ValueError */
#define NESLE_ERR_RUNTIME 2 /* unsupported operation           -> RuntimeError */
#define NESLE_ERR_CUDA 3    /* CUDA runtime failure            -> RuntimeError */

typedef struct nesle_batch nesle_batch;

/* Done predicates.  NESLE_DONE_SMB is the reference's in-kernel predicate
 * (cpp/include/nesle/cuda/batch_step.cuh:100-103).  The other two implement the
 * benchmark configurations and have no counterpart in the reference. */
#define NESLE_DONE_SMB 0
#define NESLE_DONE_RAM_EQ 1      /* done = RAM[done_a] == done_b */
#define NESLE_DONE_FRAME_LIMIT 2 /* done = frames since reset >= U[done_a, done_b], drawn per episode */

typedef struct nesle_create_args {
    int device;                           /* CUDA device ordinal */
    uint32_t num_envs;                    /* envs on this device */
    uint32_t frameskip;                   /* frames per env-step (> 0) */
    const uint8_t* rom;                   /* iNES image: mapper 0 NROM (the reference's only board), 2 UxROM, 3 CNROM */
    size_t rom_len;
    const uint8_t* const* snapshots;      /* uncompressed FCS save states, may be NULL */
    const size_t* snapshot_lens;
    uint32_t num_snapshots;               /* 0 = cold (power-on) resets; at most 255 */
    const uint8_t* env_to_level;          /* host [num_envs], NULL = all slot 0 */
    uint32_t done_mode, done_a, done_b;   /* NESLE_DONE_* and its two parameters */
    uint64_t seed;                        /* key of the frame-limit RNG */
    uint32_t env_offset;                  /* global index of env 0 (multi-GPU sharding) */
    uint32_t max_instructions_per_frame;  /* 0 = 200000, the binding's default (cuda_module.cu:1467) */
} nesle_create_args;

/* Replaces the CudaBatch(num_envs, frameskip, rom_bytes[, snapshot_bytes |
 * snapshot_bytes_list, env_to_level]) constructors (cuda_module.cu:381-460):
 * validates, allocates every device array and performs the initial reset. */
int nesle_create(const nesle_create_args* args, nesle_batch** out);

/* Replaces ~CudaBatchBinding / release() (cuda_module.cu:465-467, 1120-1207). */
int nesle_destroy(nesle_batch* b);

/* Device part of CudaBatch.reset() / reset_device() (cuda_module.cu:469-531,
 * 1417-1463): snapshot (or cold) reset of every env, actions cleared,
 * episode counters restarted, presentation snapshot seeded from live state. */
int nesle_reset(nesle_batch* b, void* stream);

/* Replaces CudaBatch.reset_envs(mask) (cuda_module.cu:917-937).  `mask` is
 * num_envs bytes, host or device memory. */
int nesle_reset_envs(nesle_batch* b, const uint8_t* mask, int mask_on_device, void* stream);

#define NESLE_ACTIONS_U8 0  /* uint8 button masks */
#define NESLE_ACTIONS_I64 1 /* int64 values already encoded as masks (low byte used) */

/* One env-step of every env.  device_api = 1 replaces CudaBatch.step_device()
 * (cuda_module.cu:594-666): rewards/done are also copied to the last_* arrays
 * and, with auto_reset, envs whose done is set are reset in the same launch.
 * device_api = 0 replaces the kernel part of CudaBatch.step() (:533-592). */
int nesle_step(nesle_batch* b, const void* actions, int action_dtype, int actions_on_device,
               int device_api, int auto_reset, void* stream);

/* Replaces CudaBatch.step_profile(actions) (cuda_module.cu:734-818): a
 * step() (no last_* copy, no auto-reset) that also counts every executed
 * instruction by opcode and by the address it was fetched from, as
 * console_step_kernel does (kernels.cu:59-64).  The histograms are cleared
 * first, then copied to opcode_counts[256] and pc_counts[65536] (host memory;
 * either may be NULL).  Synchronous. */
int nesle_step_profile(nesle_batch* b, const void* actions, int action_dtype, int actions_on_device, void* stream,
                       uint64_t* opcode_counts, uint64_t* pc_counts);

#define NESLE_RENDER_RGB 0    /* (N,240,256,3) uint8, as launch_render_kernel (kernels.cu:160-174) */
#define NESLE_RENDER_INDEX 1  /* (N,240,256) NES colour indices; no counterpart in the reference */
#define NESLE_RENDER_GRAY84 2 /* (N,84,84) area-resampled luma; no counterpart in the reference */

/* Replaces CudaBatch.render_device() (cuda_module.cu:860-863, 1435-1438). */
int nesle_render(nesle_batch* b, int mode, void* stream);

/* No counterpart in the reference.  The 84x84 grey observation of every env
 * copied into `host_out` (num_envs * 7056 bytes), without allocating device
 * memory: for callers that cannot take a device allocation at call time, such
 * as an evaluation or visualisation loop running beside a trainer whose
 * caching allocator already holds the device's memory.  The kernel renders
 * into a static device scratch of 1,024 envs (7,225,344 bytes, a global of the
 * library's module).  The scratch is committed on a device, and its address
 * looked up, by the first nesle_create on that device, so this call itself
 * never asks the device for memory.  Batches of more than 1,024 envs are
 * rejected (NESLE_ERR_INVALID).  The call copies the result out and
 * synchronizes its stream before returning, so it must not be made while that
 * stream is capturing.  The scratch is shared by all batches of a device, so
 * calls that overlap on the GPU race; serialise them.  A device reset while
 * the library is in use is not supported (the looked-up address would be
 * stale). */
int nesle_render_gray84_noalloc(nesle_batch* b, uint8_t* host_out, uint64_t bytes, void* stream);

/* Env state save / restore; the device-side capture and restore of
 * device_reset.cuh:72-263 (capture_device_reset_snapshot /
 * restore_device_reset_snapshot) over an index list.  A state is one flat
 * blob of nesle_state_bytes() bytes: the env record (CPU and PPU registers,
 * counters, controller, reward baselines, episode), RAM, PRG-RAM, nametables,
 * palette, OAM, the presentation snapshot, and the reward/done words.
 * save copies envs[0..count) into count consecutive blobs at `dst`; load
 * writes blobs into envs (any env may receive any saved state).  Env lists
 * and blobs may be host or device memory; host indices are range-checked
 * (NESLE_ERR_INVALID); device indices past the batch are skipped without an
 * error: on save their blobs keep whatever they held, on load nothing is
 * written for them.  With host
 * blobs the call synchronises; with device blobs it is asynchronous on
 * `stream`.  The blob layout is this library's and can change with
 * nesle_abi_version().  Loaded blobs are taken as saved: a hand-edited
 * controller state outside what the bus can produce (count > 8, or shift bits
 * at or above bit 8 - count) is normalised by the next step. */
uint64_t nesle_state_bytes(void);
int nesle_save_states(nesle_batch* b, const uint32_t* envs, uint32_t count, int envs_on_device, void* dst,
                      int dst_on_device, void* stream);
int nesle_load_states(nesle_batch* b, const uint32_t* envs, uint32_t count, int envs_on_device, const void* src,
                      int src_on_device, void* stream);

/* Replaces the render + copy inside CudaBatch.step(copy_obs=True) and render()
 * (cuda_module.cu:566-588, 820-840): the frames (`mode` as nesle_render) of
 * every env rendered and copied into `host_out` (num_envs x bytes per env).
 * The work is split into 8 env ranges; each range is copied on a stream of the
 * batch's own as soon as it is rendered, so copies overlap rendering.  Returns
 * when the copies are complete.  Page-locked `host_out` (nesle_host_alloc)
 * copies at the link's full rate. */
int nesle_render_copy(nesle_batch* b, int mode, void* host_out, uint64_t bytes, void* stream);

/* No counterpart in the reference (its observation copies land in pageable
 * numpy arrays).  Page-locked host memory for the host-side copies of frames
 * and observations: cudaHostAlloc with the portable flag, so every context of
 * the process copies into it at the link's full rate.  The Python binding
 * pools these buffers and hands each out as a fresh array. */
int nesle_host_alloc(uint64_t bytes, void** out);
int nesle_host_free(void* ptr);

/* Replaces CudaBatch.poke_ram(address, value) (cuda_module.cu:939-945). */
int nesle_poke_ram(nesle_batch* b, uint16_t address, uint8_t value, void* stream);

#define NESLE_PTR_RAM 0          /* uint8 [N][2048]       ram_device()        (:854-863) */
#define NESLE_PTR_LAST_REWARDS 1 /* float [N]             rewards_device()    (:888-894) */
#define NESLE_PTR_LAST_DONE 2    /* uint8 [N]             last_done_device()  (:896-902) */
#define NESLE_PTR_FRAMES_RGB 3   /* uint8 [N][240][256][3] frames_device()    (:871-886) */
#define NESLE_PTR_FRAMES_INDEX 4 /* uint8 [N][240][256] */
#define NESLE_PTR_OBS_GRAY84 5   /* uint8 [N][84][84] */
#define NESLE_PTR_REWARDS 6      /* float [N] rewards of the last kernel (step() semantics) */
#define NESLE_PTR_DONE 7         /* uint8 [N] done of the last kernel */

/* Device pointer and size of one batch array (frame buffers are allocated
 * on first use).  Replaces the *_device() view constructors listed above. */
int nesle_device_ptr(nesle_batch* b, int which, void** ptr, uint64_t* bytes);

/* Synchronous host copy of one per-env field: "ram", "oam", "prg_ram",
 * "nametable", "palette", "pc", "a", "x", "y", "sp", "p", "cycles", "frame",
 * "status", "stat_instructions", "stat_frames", "stat_budget_hits", the output
 * arrays "rewards", "done", "last_rewards", "last_done" and the rendered
 * "frames_rgb", "frames_index", "obs_gray84" (replaces ram(), oam() and
 * render()'s copy, cuda_module.cu:820-852, 904-915, and the host copies of
 * step_stats(), :668-732).  `bytes` must match num_envs * width. */
int nesle_copy_field(nesle_batch* b, const char* name, void* host_out, uint64_t bytes);

/* Host wait for all work this batch issued (replaces blocking_stream_sync,
 * cuda_module.cu:199-210). */
int nesle_sync(nesle_batch* b);

/* Makes `consumer_stream` wait for the batch's last issued work (the
 * synchronisation CudaDeviceArrayView.__dlpack__ performs, :142-149, as a
 * device-side dependency instead of a host sync). */
int nesle_stream_wait(nesle_batch* b, void* consumer_stream);

/* Number of env faults since creation: an env faults when it meets an illegal
 * opcode, where the reference kernel executes `trap` (cpu.hpp:716-720); the
 * env then stops for the rest of the step and its status word (field
 * "status") holds the opcode and address until the env is reset.  Synchronous. */
int nesle_fault_count(nesle_batch* b, uint32_t* count);

typedef struct nesle_info {
    uint32_t num_envs, frameskip, num_levels, device;
    uint32_t envs_per_block, smem_bytes_per_block;
    uint32_t step_placement; /* where the step kernel keeps env RAM: NESLE_PLACEMENT_* */
} nesle_info;

#define NESLE_PLACEMENT_SHARED 0       /* whole RAM row staged in shared memory (small batches) */
#define NESLE_PLACEMENT_GLOBAL 1       /* RAM row in place in device memory */
#define NESLE_PLACEMENT_HYBRID 2       /* in place, zero page staged in shared memory */
#define NESLE_PLACEMENT_HYBRID_STACK 3 /* in place, stack page staged in shared memory */
#define NESLE_PLACEMENT_GLOBAL_ASYNC 4 /* in place, operands loaded ahead asynchronously */
#define NESLE_PLACEMENT_HYBRID_ASYNC 5 /* hybrid, operands outside the zero page loaded ahead asynchronously */
#define NESLE_PLACEMENT_INTERLEAVED 6  /* hybrid, the rest of RAM env-interleaved in a device working copy */
#define NESLE_PLACEMENT_INTERLEAVED_ASYNC 7 /* the same with operands loaded ahead asynchronously */
#define NESLE_PLACEMENT_GLOBAL_PRELOAD 8   /* in place, operands loaded one instruction ahead into registers */
#define NESLE_PLACEMENT_HYBRID_PRELOAD 9   /* hybrid, the same for operands outside the zero page */
#define NESLE_PLACEMENT_INTERLEAVED_PRELOAD 10 /* interleaved, the same */

/* name / has_snapshot / num_levels properties (cuda_module.cu:947-957). */
int nesle_get_info(nesle_batch* b, nesle_info* out);

typedef struct nesle_fcs_state {
    uint16_t pc;
    uint8_t a, x, y, sp, p;
    uint64_t cycles;
    uint8_t ppu_ctrl, ppu_mask, ppu_status, ppu_oam_addr, ppu_open_bus, ppu_read_buffer, ppu_x, ppu_w;
    uint16_t ppu_v, ppu_t;
    uint8_t cpu_ram[2048];
    uint8_t prg_ram[8192];
    uint8_t nametable_ram[2048];
    uint8_t palette_ram[32];
    uint8_t oam[256];
} nesle_fcs_state;

/* Replaces the module function parse_fcs_state(bytes) (cuda_module.cu:1579-1620). */
int nesle_parse_fcs(const uint8_t* data, size_t len, nesle_fcs_state* out);

/* Message of the last failed call on this thread ("" if none). */
const char* nesle_last_error(void);

/* ABI version (bumped on incompatible changes). */
int nesle_abi_version(void);

#ifdef __cplusplus
}
#endif
#endif /* NESLE_B200_H */
