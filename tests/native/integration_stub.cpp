// integration_stub.cpp -- the minimal C++ host loop over the C ABI that a
// maintainer of a non-Python trainer would write (quoted in the integration
// guide).  tests/test_capi_exports.py type-checks it against
// include/nesle_b200.h with `g++ -fsyntax-only`; it is never linked or run.
#include <cuda_runtime.h>

#include <cstdio>
#include <vector>

#include "nesle_b200.h"

// rom: an iNES image; snaps/lens: 8 FCS snapshots; levels: host uint8[num_envs];
// d_actions: device uint8[num_envs] written on `stream` by the policy.
int run_loop(std::vector<uint8_t>& rom, const uint8_t* const* snaps, const size_t* lens, const uint8_t* levels,
             void* d_actions, void* stream, int steps) {
    nesle_create_args a = {};
    a.device = 0; a.num_envs = 65536; a.frameskip = 4;
    a.rom = rom.data(); a.rom_len = rom.size();
    a.snapshots = snaps; a.snapshot_lens = lens; a.num_snapshots = 8;
    a.env_to_level = levels;                      // host uint8[num_envs]
    a.done_mode = NESLE_DONE_SMB;
    nesle_batch* b = nullptr;
    if (nesle_create(&a, &b) != NESLE_OK) {
        fprintf(stderr, "%s\n", nesle_last_error());
        return 1;
    }

    void* ram; uint64_t ram_bytes;               // (N, 2048) uint8, stays valid for b's lifetime
    nesle_device_ptr(b, NESLE_PTR_RAM, &ram, &ram_bytes);
    void* rew; uint64_t rew_bytes;
    nesle_device_ptr(b, NESLE_PTR_LAST_REWARDS, &rew, &rew_bytes);

    for (int i = 0; i < steps; ++i) {
        // actions: device uint8[N] (or int64 with NESLE_ACTIONS_I64) produced on `stream`
        nesle_step(b, d_actions, NESLE_ACTIONS_U8, /*on_device=*/1, /*device_api=*/1, /*auto_reset=*/1, stream);
        // consume ram / rew on `stream` (or call nesle_stream_wait(b, other_stream) first)
    }
    nesle_destroy(b);
    return 0;
}
