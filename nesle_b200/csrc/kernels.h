// kernels.h -- host-side launchers of the batched NES kernels.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/nesle_b200.h"
#include "nesle_state.h"

namespace nesle {

constexpr uint32_t kStepSlots = 64;       // envs (threads) per shared-RAM step CTA (multiple of 32: conflict-free banks)
constexpr uint32_t kGlobalMaxThreads = 448;  // max envs (threads) per in-place step CTA

enum : uint32_t {
    kStepSharedRam = 0,       // whole RAM row staged in shared memory
    kStepGlobalRam = 1,       // RAM row in place
    kStepHybridRam = 2,       // in place, zero page staged in a shared-memory slot
    kStepHybridStackRam = 3,  // in place, stack page in the slot
    kStepGlobalAsync = 4,     // in place, operands loaded ahead asynchronously
    kStepHybridAsync = 5,     // hybrid, operands outside the slot loaded ahead asynchronously
    kStepInterleaved = 6,     // hybrid, the rest of RAM in an env-interleaved working copy in device memory
    kStepInterleavedAsync = 7,  // the same with operands loaded ahead asynchronously
    kStepGlobalPreload = 8,   // in place, operands loaded one iteration ahead into a register
    kStepHybridPreload = 9,   // hybrid, the same for operands outside the slot
    kStepInterleavedPreload = 10,  // interleaved, the same
};
inline bool step_interleaved(uint32_t variant) {
    return variant == kStepInterleaved || variant == kStepInterleavedAsync || variant == kStepInterleavedPreload;
}
static_assert(kStepSharedRam == NESLE_PLACEMENT_SHARED && kStepHybridAsync == NESLE_PLACEMENT_HYBRID_ASYNC,
              "step variants are the ABI's placement codes");
// Dynamic shared memory of one in-place step CTA of `threads` lanes.
size_t global_step_smem(uint32_t variant, uint32_t threads);

enum : uint32_t { kStepDeviceApi = 1, kStepAutoReset = 2 };

size_t step_smem_bytes();
cudaError_t configure_kernels();
uint32_t global_step_threads(uint32_t num_envs, uint32_t num_sms);
// prof_op (256) / prof_pc (65536): step_profile histograms to add to, or both null.
// board: the cartridge is UxROM or CNROM (variant must then be shared, global or hybrid).
cudaError_t launch_step(const BatchView* dv, uint32_t num_envs, const uint8_t* act8, const long long* act64,
                        uint32_t flags, uint32_t variant, uint32_t threads, cudaStream_t s,
                        unsigned long long* prof_op = nullptr, unsigned long long* prof_pc = nullptr,
                        bool board = false);
cudaError_t launch_reset(const BatchView* dv, uint32_t num_envs, const uint8_t* mask, bool full, cudaStream_t s);
// envs: device array of `count` env indices; blobs: count x kStateBytes (device).
cudaError_t launch_state(const BatchView* dv, const uint32_t* envs, uint32_t count, uint8_t* blobs, bool save,
                         cudaStream_t s);
cudaError_t launch_poke(const BatchView* dv, uint32_t num_envs, uint32_t address, uint32_t value, cudaStream_t s);
cudaError_t launch_render(const BatchView* dv, uint32_t env0, uint32_t count, uint8_t* out, int mode, cudaStream_t s);

}  // namespace nesle
