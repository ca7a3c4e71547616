/*
 * nes_oracle.h -- CPU checker for the batched NES env-step path.
 *
 * TEST INFRASTRUCTURE ONLY.  This is a plain-C restatement of the reference
 * CUDA kernel's semantics (hbofz/NeSLE cpp/src/cuda/kernels.cu:19-104 and the
 * batch_* headers it includes), used by tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py as the parity checker.  The product path
 * (nesle_b200/, include/nesle_b200.h) never links or calls it.
 *
 * Pinning: tests/test_oracle_pin.py checks this restatement against the
 * reference sources compiled unchanged into oracle/_ref/ (oracle/Makefile) and
 * against the committed golden vectors under tests/golden/.
 */
#ifndef NES_ORACLE_H
#define NES_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct nes_oracle nes_oracle;

/* Done predicates.  ORACLE_DONE_SMB is the reference's in-kernel predicate
 * (cpp/include/nesle/cuda/batch_step.cuh:100-103); the other two are the
 * benchmark-configuration predicates, which the reference does not have. */
enum { ORACLE_DONE_SMB = 0, ORACLE_DONE_RAM_EQ = 1, ORACLE_DONE_FRAME_LIMIT = 2 };

/* Per-env status word: 0 = healthy.  Bit 31 set = illegal opcode, with the
 * opcode in bits 16-23 and its address in bits 0-15.  The env stops executing
 * for the rest of the step; the word is cleared by any reset of that env. */
#define ORACLE_STATUS_ILLEGAL 0x80000000u

nes_oracle *oracle_create(uint32_t num_envs, uint32_t frameskip, const uint8_t *rom,
                          size_t rom_len, const uint8_t *const *snapshots,
                          const size_t *snapshot_lens, uint32_t num_snapshots,
                          const uint8_t *env_to_level, uint32_t done_mode, uint32_t done_a,
                          uint32_t done_b, uint64_t seed, uint32_t env_offset);
const char *oracle_last_error(void);
void oracle_destroy(nes_oracle *o);

/* CudaBatch.reset(): snapshot or cold reset of every env, then seed the
 * presentation snapshot from live state (cuda_module.cu:469-480,1417-1463). */
void oracle_reset(nes_oracle *o);
/* CudaBatch.reset_envs(mask) (cuda_module.cu:917-937). */
void oracle_reset_envs(nes_oracle *o, const uint8_t *mask);
/* step_device semantics when device_api != 0 (cuda_module.cu:594-666):
 * run the kernel, copy rewards/done to last_*, auto-reset where last_done.
 * With device_api == 0: CudaBatch.step() semantics (cuda_module.cu:533-592):
 * run the kernel only. */
void oracle_step(nes_oracle *o, const uint8_t *actions, int device_api, int auto_reset);
void oracle_poke_ram(nes_oracle *o, uint16_t address, uint8_t value);

/* Render every env from its presentation snapshot (batch_render.cuh:333-434).
 * Any output pointer may be NULL.  index: N*240*256 NES colour indices;
 * rgb: N*240*256*3; gray84: N*84*84 (this build's area-resampled luma). */
void oracle_render(const nes_oracle *o, uint8_t *index, uint8_t *rgb, uint8_t *gray84);

/* Field export.  `field` names one per-env quantity; `out` must hold
 * num_envs * width bytes, with width given by oracle_field_width(). */
int oracle_field_width(const char *field);
int oracle_get_field(const nes_oracle *o, const char *field, void *out);
uint32_t oracle_num_envs(const nes_oracle *o);

/* Instruction trace of one env during the next oracle_step calls: after every
 * executed instruction one record {op_pc, opcode, a, x, y, p, sp, pad,
 * cycles(u64)} (16 bytes) is appended to `buf` until `cap` records.  Returns
 * the number of records written so far via oracle_trace_count(). */
void oracle_set_trace(nes_oracle *o, uint32_t env, uint8_t *buf, uint32_t cap);
uint32_t oracle_trace_count(const nes_oracle *o);

/* step_profile histograms (cuda_module.cu:734-818): while set, every executed
 * instruction adds one to opcode_counts[opcode] (256 entries) and to
 * pc_counts[address] (65536 entries).  The caller clears them.  NULL stops. */
void oracle_set_profile(nes_oracle *o, uint64_t *opcode_counts, uint64_t *pc_counts);

/* Decode-table export for pinning: per opcode {mode, base_cycles, flags}. */
void oracle_decode_table(uint8_t *mode, uint8_t *base_cycles, uint8_t *flags);

/* Counter RNG shared with the product kernel (SplitMix64 finaliser). */
uint64_t oracle_counter_rand(uint64_t seed, uint32_t stream, uint64_t a, uint64_t b);

#ifdef __cplusplus
}
#endif
#endif
