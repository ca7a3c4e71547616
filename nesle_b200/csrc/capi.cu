// capi.cu -- the C ABI (include/nesle_b200.h): validation, device memory,
// snapshot bank upload and kernel launches for one batch.
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>
#include <string>
#include <vector>

#include "../../include/nesle_b200.h"
#include "formats.h"
#include "kernels.h"
#include "nesle_state.h"

using namespace nesle;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

#define CUDA_TRY(expr, label)                                                              \
    do {                                                                                   \
        cudaError_t e_ = (expr);                                                           \
        if (e_ != cudaSuccess) return fail(NESLE_ERR_CUDA, std::string(label) + ": " + cudaGetErrorString(e_)); \
    } while (0)

// Restores the caller's current device on scope exit.
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

int bcd3(const uint8_t* ram, int a) { return (ram[a] & 0xF) * 100 + (ram[a + 1] & 0xF) * 10 + (ram[a + 2] & 0xF); }

}  // namespace

constexpr uint32_t kRenderChunks = 8;  // env ranges of nesle_render_copy

struct nesle_batch {
    int device = 0;
    uint32_t n = 0, frameskip = 0, num_levels = 0;
    BatchView hv{};
    BatchView* dv = nullptr;
    std::vector<void*> allocations;
    uint8_t* d_host_actions = nullptr;  // staging for host-memory action arrays
    uint8_t* d_mask = nullptr;          // staging for host-memory reset masks
    uint8_t* d_frames_rgb = nullptr;
    uint8_t* d_frames_index = nullptr;
    uint8_t* d_gray84 = nullptr;
    unsigned long long* d_prof = nullptr;  // step_profile histograms: 256 opcode + 65536 PC counts
    uint32_t* d_state_envs = nullptr;      // staging of host env lists / state blobs (grown on demand)
    uint8_t* d_state_blobs = nullptr;
    uint32_t state_cap = 0;
    cudaEvent_t done_event = nullptr;
    cudaStream_t copy_stream = nullptr;         // nesle_render_copy: device-to-host copies
    cudaEvent_t chunk_events[kRenderChunks] = {};  // nesle_render_copy: one per rendered range
    uint32_t step_variant = kStepGlobalRam;
    uint32_t step_threads = 0;
    bool board = false;  // UxROM / CNROM cartridge

    template <class T>
    int alloc(T** out, size_t count, const char* label) {
        void* p = nullptr;
        cudaError_t e = cudaMalloc(&p, count * sizeof(T) > 0 ? count * sizeof(T) : 16);
        if (e != cudaSuccess) return fail(NESLE_ERR_CUDA, std::string("cudaMalloc ") + label + ": " + cudaGetErrorString(e));
        allocations.push_back(p);
        *out = static_cast<T*>(p);
        return NESLE_OK;
    }
    // Frees one allocation made by alloc() (a no-op for null).
    void free_one(void* p) {
        if (!p) return;
        for (size_t i = 0; i < allocations.size(); ++i)
            if (allocations[i] == p) {
                cudaFree(p);
                allocations.erase(allocations.begin() + (long)i);
                return;
            }
    }
    void release() {
        for (void* p : allocations) cudaFree(p);
        allocations.clear();
        if (done_event) cudaEventDestroy(done_event);
        done_event = nullptr;
        for (cudaEvent_t& e : chunk_events) {
            if (e) cudaEventDestroy(e);
            e = nullptr;
        }
        if (copy_stream) cudaStreamDestroy(copy_stream);
        copy_stream = nullptr;
    }
};

#define TRY(expr)                     \
    do {                              \
        int rc_ = (expr);             \
        if (rc_ != NESLE_OK) return rc_; \
    } while (0)

// Static scratch of nesle_render_gray84_noalloc: 1,024 envs x 7,056 bytes
// (7,225,344 B), a module global rather than a cudaMalloc.  Under lazy module
// loading (the CUDA default) the module that holds it -- this file's, which has
// no kernels -- is loaded, and the scratch committed on the device, by the
// first cudaGetSymbolAddress.  nesle_create does that lookup, so the scratch
// is committed while a batch is being allocated anyway, never later inside
// the no-allocation call.  The cached address belongs to the device's current
// context: resetting the device (cudaDeviceReset) while the library is in use
// is not supported.
constexpr uint32_t kNoAllocGrayEnvs = 1024;
static __device__ __align__(256) uint8_t g_gray84_scratch[(size_t)kNoAllocGrayEnvs * kGray * kGray];
constexpr int kNoAllocMaxDevices = 64;
static std::mutex g_noalloc_mu;
static uint8_t* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Address of the scratch on `device`, which must be current (looked up once per device).
static int noalloc_scratch(int device, uint8_t** out) {
    if (device < 0 || device >= kNoAllocMaxDevices) return fail(NESLE_ERR_INVALID, "render_gray84_noalloc: device ordinal");
    std::lock_guard<std::mutex> lock(g_noalloc_mu);
    if (!g_noalloc_ptr[device]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_gray84_scratch);
        if (e != cudaSuccess)
            return fail(NESLE_ERR_CUDA, std::string("render_gray84_noalloc scratch: ") + cudaGetErrorString(e));
        g_noalloc_ptr[device] = static_cast<uint8_t*>(p);
    }
    *out = g_noalloc_ptr[device];
    return NESLE_OK;
}

extern "C" {

const char* nesle_last_error(void) { return g_err.c_str(); }

int nesle_abi_version(void) { return 2; }

int nesle_parse_fcs(const uint8_t* data, size_t len, nesle_fcs_state* out) {
    if (!data || !out) return fail(NESLE_ERR_INVALID, "parse_fcs: null argument");
    FcsState s;
    std::string err;
    if (!parse_fcs(data, len, s, err)) return fail(NESLE_ERR_INVALID, err);
    out->pc = s.pc; out->a = s.a; out->x = s.x; out->y = s.y; out->sp = s.sp; out->p = s.p;
    out->cycles = s.cycles;
    out->ppu_ctrl = s.ppu_ctrl; out->ppu_mask = s.ppu_mask; out->ppu_status = s.ppu_status;
    out->ppu_oam_addr = s.ppu_oam_addr; out->ppu_open_bus = s.ppu_open_bus;
    out->ppu_read_buffer = s.ppu_read_buffer; out->ppu_x = s.ppu_x; out->ppu_w = s.ppu_w;
    out->ppu_v = s.ppu_v; out->ppu_t = s.ppu_t;
    memcpy(out->cpu_ram, s.cpu_ram, 2048); memcpy(out->prg_ram, s.prg_ram, 8192);
    memcpy(out->nametable_ram, s.nametable_ram, 2048); memcpy(out->palette_ram, s.palette_ram, 32);
    memcpy(out->oam, s.oam, 256);
    return NESLE_OK;
}

static int create_impl(const nesle_create_args* a, nesle_batch* b) {
    b->device = a->device;
    b->n = a->num_envs;
    b->frameskip = a->frameskip;
    // ROM (cuda_module.cu:381-398) and snapshots (:403-460).
    Cartridge cart;
    std::string err;
    if (!a->rom || !parse_ines(a->rom, a->rom_len, cart, err)) return fail(NESLE_ERR_INVALID, a->rom ? err : "rom is required");
    if (a->num_snapshots > 255) return fail(NESLE_ERR_INVALID, "at most 255 snapshot levels supported per CudaBatch");
    std::vector<FcsState> snaps(a->num_snapshots);
    for (uint32_t i = 0; i < a->num_snapshots; ++i) {
        if (!parse_fcs(a->snapshots[i], a->snapshot_lens[i], snaps[i], err)) return fail(NESLE_ERR_INVALID, err);
    }
    std::vector<uint8_t> e2l(b->n, 0);
    if (a->env_to_level) {
        for (uint32_t e = 0; e < b->n; ++e) {
            const uint32_t lvl = a->env_to_level[e];
            if (a->num_snapshots && lvl >= a->num_snapshots)
                return fail(NESLE_ERR_INVALID, "env_to_level[" + std::to_string(e) + "]=" + std::to_string(lvl) +
                                                   " out of range (have " + std::to_string(a->num_snapshots) + " levels)");
            e2l[e] = static_cast<uint8_t>(lvl);
        }
    }
    if (a->done_mode > NESLE_DONE_FRAME_LIMIT) return fail(NESLE_ERR_INVALID, "unknown done_mode");
    if (a->done_mode == NESLE_DONE_FRAME_LIMIT && a->done_b < a->done_a)
        return fail(NESLE_ERR_INVALID, "frame-limit done needs done_a <= done_b");

    int ndev = 0;
    CUDA_TRY(cudaGetDeviceCount(&ndev), "cudaGetDeviceCount");
    if (a->device < 0 || a->device >= ndev) return fail(NESLE_ERR_INVALID, "device ordinal out of range");
    DeviceGuard guard(a->device);
    CUDA_TRY(configure_kernels(), "configure kernels");
    uint8_t* noalloc = nullptr;  // commits the no-allocation scratch now (see noalloc_scratch)
    TRY(noalloc_scratch(a->device, &noalloc));

    const size_t n = b->n;
    BatchView& v = b->hv;
    TRY(b->alloc(&v.rec, n, "records"));
    TRY(b->alloc(&v.ram, n * kRamBytes, "ram"));
    TRY(b->alloc(&v.prg_ram, n * kPrgRamBytes, "prg ram"));
    TRY(b->alloc(&v.nt, n * kNtBytes, "nametable"));
    TRY(b->alloc(&v.pal, n * kPalBytes, "palette"));
    TRY(b->alloc(&v.oam, n * kOamBytes, "oam"));
    TRY(b->alloc(&v.snap_nt, n * kNtBytes, "snapshot nametable"));
    TRY(b->alloc(&v.snap_pal, n * kPalBytes, "snapshot palette"));
    TRY(b->alloc(&v.snap_oam, n * kOamBytes, "snapshot oam"));
    TRY(b->alloc(&v.rewards, n, "rewards"));
    TRY(b->alloc(&v.done, n, "done"));
    TRY(b->alloc(&v.last_rewards, n, "last rewards"));
    TRY(b->alloc(&v.last_done, n, "last done"));
    TRY(b->alloc(&v.fault_count, 1, "fault count"));
    TRY(b->alloc(&b->d_host_actions, n, "action staging"));
    TRY(b->alloc(&b->d_mask, n, "mask staging"));
    CUDA_TRY(cudaMemset(v.rec, 0, n * sizeof(EnvRecord)), "clear records");
    CUDA_TRY(cudaMemset(v.last_rewards, 0, n * sizeof(float)), "clear last rewards");
    CUDA_TRY(cudaMemset(v.last_done, 0, n), "clear last done");
    CUDA_TRY(cudaMemset(v.fault_count, 0, sizeof(uint32_t)), "clear fault count");

    // Cartridge: the 32 KB window at $8000 the kernels stage.  16 KB PRG
    // images are mirrored to 32 KB so the kernel masks every PRG address with
    // $7FFF (cpp/include/nesle/cuda/batch_bus.cuh:24-33); for UxROM the window
    // is bank 0 and the fixed last bank (the kernels serve $8000-$BFFF from
    // the env's bank of the whole ROM instead).
    std::vector<uint8_t> prg32(32768);
    const size_t last = cart.prg.size() - 16384;
    for (size_t i = 0; i < 32768; ++i)
        prg32[i] = cart.mapper == kMapperUxrom ? cart.prg[i < 16384 ? i : last + i - 16384] : cart.prg[i % cart.prg.size()];
    uint8_t* d_prg = nullptr;
    TRY(b->alloc(&d_prg, 32768 + 16, "prg rom"));
    CUDA_TRY(cudaMemset(d_prg, 0, 32768 + 16), "clear prg");
    CUDA_TRY(cudaMemcpy(d_prg, prg32.data(), 32768, cudaMemcpyHostToDevice), "copy prg rom");
    v.prg = d_prg;
    v.prg_rom = d_prg;
    if (cart.mapper == kMapperUxrom) {
        uint8_t* d_rom = nullptr;
        TRY(b->alloc(&d_rom, cart.prg.size(), "prg banks"));
        CUDA_TRY(cudaMemcpy(d_rom, cart.prg.data(), cart.prg.size(), cudaMemcpyHostToDevice), "copy prg banks");
        v.prg_rom = d_rom;
    }
    v.mapper = cart.mapper;
    v.prg_banks = cart.prg_banks;
    v.chr_banks = cart.chr_banks;
    TRY(b->alloc(&v.mstate, n, "board registers"));
    CUDA_TRY(cudaMemset(v.mstate, 0, n * sizeof(MapperState)), "clear board registers");
    v.chr = nullptr;
    v.chr_size = static_cast<uint32_t>(cart.chr.size());
    if (!cart.chr.empty()) {
        uint8_t* d_chr = nullptr;
        TRY(b->alloc(&d_chr, cart.chr.size(), "chr rom"));
        CUDA_TRY(cudaMemcpy(d_chr, cart.chr.data(), cart.chr.size(), cudaMemcpyHostToDevice), "copy chr rom");
        v.chr = d_chr;
    }
    v.horizontal = cart.horizontal ? 1u : 0u;
    v.reset_vector = static_cast<uint16_t>(prg32[0x7FFC] | (prg32[0x7FFD] << 8));

    // Snapshot bank (cuda_module.cu:1291-1415).
    const size_t k = snaps.size();
    b->num_levels = static_cast<uint32_t>(k);
    v.num_levels = b->num_levels;
    {
        std::vector<BankRecord> recs(k ? k : 1);
        std::vector<uint8_t> ram(k * kRamBytes), prg_ram(k * kPrgRamBytes), nt(k * kNtBytes), pal(k * kPalBytes),
            oam(k * kOamBytes);
        for (size_t i = 0; i < k; ++i) {
            const FcsState& s = snaps[i];
            BankRecord r{};
            r.pc = s.pc; r.a = s.a; r.x = s.x; r.y = s.y; r.sp = s.sp; r.p = s.p; r.cycles = s.cycles;
            r.ctrl = s.ppu_ctrl; r.mask = s.ppu_mask; r.status = s.ppu_status; r.oam_addr = s.ppu_oam_addr;
            r.open_bus = s.ppu_open_bus; r.read_buffer = s.ppu_read_buffer; r.fine_x = s.ppu_x; r.w = s.ppu_w;
            r.v = s.ppu_v; r.t = s.ppu_t;
            // Reward baselines seeded from the slot's RAM (batch_step.cuh:232-239).
            r.prev_x = s.cpu_ram[0x6D] * 0x100 + s.cpu_ram[0x86];
            r.prev_time = bcd3(s.cpu_ram, 0x7F8);
            recs[i] = r;
            memcpy(&ram[i * kRamBytes], s.cpu_ram, kRamBytes);
            memcpy(&prg_ram[i * kPrgRamBytes], s.prg_ram, kPrgRamBytes);
            memcpy(&nt[i * kNtBytes], s.nametable_ram, kNtBytes);
            memcpy(&pal[i * kPalBytes], s.palette_ram, kPalBytes);
            memcpy(&oam[i * kOamBytes], s.oam, kOamBytes);
        }
        BankRecord* d_bank = nullptr;
        uint8_t *d_ram = nullptr, *d_prg_ram = nullptr, *d_nt = nullptr, *d_pal = nullptr, *d_oam = nullptr, *d_e2l = nullptr;
        TRY(b->alloc(&d_bank, recs.size(), "bank records"));
        TRY(b->alloc(&d_ram, ram.size(), "bank ram"));
        TRY(b->alloc(&d_prg_ram, prg_ram.size(), "bank prg ram"));
        TRY(b->alloc(&d_nt, nt.size(), "bank nametable"));
        TRY(b->alloc(&d_pal, pal.size(), "bank palette"));
        TRY(b->alloc(&d_oam, oam.size(), "bank oam"));
        TRY(b->alloc(&d_e2l, n, "env_to_level"));
        CUDA_TRY(cudaMemcpy(d_bank, recs.data(), recs.size() * sizeof(BankRecord), cudaMemcpyHostToDevice), "bank upload");
        if (k) {
            CUDA_TRY(cudaMemcpy(d_ram, ram.data(), ram.size(), cudaMemcpyHostToDevice), "bank upload");
            CUDA_TRY(cudaMemcpy(d_prg_ram, prg_ram.data(), prg_ram.size(), cudaMemcpyHostToDevice), "bank upload");
            CUDA_TRY(cudaMemcpy(d_nt, nt.data(), nt.size(), cudaMemcpyHostToDevice), "bank upload");
            CUDA_TRY(cudaMemcpy(d_pal, pal.data(), pal.size(), cudaMemcpyHostToDevice), "bank upload");
            CUDA_TRY(cudaMemcpy(d_oam, oam.data(), oam.size(), cudaMemcpyHostToDevice), "bank upload");
        }
        CUDA_TRY(cudaMemcpy(d_e2l, e2l.data(), n, cudaMemcpyHostToDevice), "env_to_level upload");
        v.bank = d_bank; v.bank_ram = d_ram; v.bank_prg_ram = d_prg_ram; v.bank_nt = d_nt;
        v.bank_pal = d_pal; v.bank_oam = d_oam; v.env_to_level = d_e2l;
    }
    v.num_envs = b->n;
    v.frameskip = b->frameskip;
    v.max_instructions = a->max_instructions_per_frame ? a->max_instructions_per_frame : 200000u;
    v.done_mode = a->done_mode;
    v.done_a = a->done_a;
    v.done_b = a->done_b;
    v.env_offset = a->env_offset;
    v.seed = a->seed;
    v.actions = nullptr;
    TRY(b->alloc(&b->dv, 1, "batch view"));
    CUDA_TRY(cudaMemcpy(b->dv, &v, sizeof(BatchView), cudaMemcpyHostToDevice), "batch view upload");
    // Step-kernel placement of env RAM.  Up to two waves of shared-memory CTAs
    // (kStepSlots envs per SM per wave) the RAM is staged in shared memory: with
    // few warps per SM the latency of each env's instruction chain decides, and
    // shared memory has the shorter one (B200, config-4 workload: 185k vs 77k
    // env-steps/s at 2,048 envs, 740k vs 592k at 16,384).  Larger batches keep
    // every env resident with the zero page in shared memory and the rest of RAM
    // in the env-interleaved working copy (B200, 65,536 envs: config 4 2.36 M
    // env-steps/s against 2.27 M in place with the zero page staged, config 2
    // 3.29 M against 3.26 M; config 3's step is 4% slower than in place).
    // NESLE_STEP_KERNEL=<placement name> overrides.
    int sms = 0;
    CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, a->device), "SM count");
    b->step_variant = b->n <= 2u * (uint32_t)sms * kStepSlots ? kStepSharedRam : kStepInterleaved;
    if (const char* sv = getenv("NESLE_STEP_KERNEL")) {
        // Names in kStep* order (the Python mirror's PLACEMENTS).
        static const char* const kNames[] = {"shared", "global", "hybrid", "hybrid-stack", "global-async",
                                             "hybrid-async", "interleaved", "interleaved-async",
                                             "global-preload", "hybrid-preload", "interleaved-preload"};
        static_assert(sizeof(kNames) / sizeof(kNames[0]) == kStepInterleavedPreload + 1, "placement names");
        int found = -1;
        for (int i = 0; i <= kStepInterleavedPreload; ++i)
            if (strcmp(sv, kNames[i]) == 0) found = i;
        if (found < 0) return fail(NESLE_ERR_INVALID, std::string("NESLE_STEP_KERNEL: unknown placement '") + sv + "'");
        b->step_variant = found;
    }
    b->board = cart.mapper != kMapperNrom;
    if (b->board && b->step_variant != kStepSharedRam && b->step_variant != kStepGlobalRam)
        b->step_variant = kStepHybridRam;  // the placements built for UxROM / CNROM
    b->step_threads = global_step_threads(b->n, static_cast<uint32_t>(sms));
    if (step_interleaved(b->step_variant)) {  // the interleaved working copy: one 2 KB word column per lane
        const size_t blocks = (b->n + b->step_threads - 1) / b->step_threads;
        TRY(b->alloc(&v.ram_work, blocks * b->step_threads * kRamBytes, "interleaved ram"));
        CUDA_TRY(cudaMemcpy(b->dv, &v, sizeof(BatchView), cudaMemcpyHostToDevice), "batch view upload");
    }
    CUDA_TRY(cudaEventCreateWithFlags(&b->done_event, cudaEventDisableTiming), "create event");
    CUDA_TRY(launch_reset(b->dv, b->n, nullptr, true, nullptr), "initial reset");
    CUDA_TRY(cudaEventRecord(b->done_event, nullptr), "record event");
    CUDA_TRY(cudaEventSynchronize(b->done_event), "initial reset synchronize");
    return NESLE_OK;
}

int nesle_create(const nesle_create_args* a, nesle_batch** out) {
    if (!a || !out) return fail(NESLE_ERR_INVALID, "create: null argument");
    *out = nullptr;
    if (a->num_envs == 0) return fail(NESLE_ERR_INVALID, "num_envs must be positive");
    if (a->frameskip == 0) return fail(NESLE_ERR_INVALID, "frameskip must be positive");
    auto* b = new nesle_batch();
    const int rc = create_impl(a, b);
    if (rc != NESLE_OK) {
        DeviceGuard guard(a->device >= 0 ? a->device : 0);
        b->release();
        delete b;
        return rc;
    }
    *out = b;
    return NESLE_OK;
}

int nesle_destroy(nesle_batch* b) {
    if (!b) return NESLE_OK;
    {
        DeviceGuard guard(b->device);
        if (b->done_event) cudaEventSynchronize(b->done_event);
        b->release();
    }
    delete b;
    return NESLE_OK;
}

static int finish(nesle_batch* b, cudaStream_t s, cudaError_t launch, const char* label) {
    if (launch != cudaSuccess) return fail(NESLE_ERR_CUDA, std::string(label) + ": " + cudaGetErrorString(launch));
    CUDA_TRY(cudaEventRecord(b->done_event, s), "record event");
    return NESLE_OK;
}

int nesle_reset(nesle_batch* b, void* stream) {
    if (!b) return fail(NESLE_ERR_INVALID, "null batch");
    DeviceGuard guard(b->device);
    auto s = static_cast<cudaStream_t>(stream);
    return finish(b, s, launch_reset(b->dv, b->n, nullptr, true, s), "reset kernel");
}

int nesle_reset_envs(nesle_batch* b, const uint8_t* mask, int mask_on_device, void* stream) {
    if (!b || !mask) return fail(NESLE_ERR_INVALID, "reset_envs: null argument");
    DeviceGuard guard(b->device);
    auto s = static_cast<cudaStream_t>(stream);
    const uint8_t* dmask = mask;
    if (!mask_on_device) {
        CUDA_TRY(cudaMemcpyAsync(b->d_mask, mask, b->n, cudaMemcpyHostToDevice, s), "copy reset mask");
        dmask = b->d_mask;
    }
    return finish(b, s, launch_reset(b->dv, b->n, dmask, false, s), "reset_envs kernel");
}

// Shared by nesle_step and nesle_step_profile: action ingest (cuda_module.cu:259-317) and the launch.
static int step_impl(nesle_batch* b, const void* actions, int dtype, int on_device, int device_api, int auto_reset,
                     cudaStream_t s, unsigned long long* prof_op, unsigned long long* prof_pc) {
    if (!b || !actions) return fail(NESLE_ERR_INVALID, "step: null argument");
    if (dtype != NESLE_ACTIONS_U8 && dtype != NESLE_ACTIONS_I64)
        return fail(NESLE_ERR_INVALID, "CUDA actions must be uint8 masks or int64 values already encoded as masks");
    const uint8_t* a8 = nullptr;
    const long long* a64 = nullptr;
    if (on_device) {
        if (dtype == NESLE_ACTIONS_U8) a8 = static_cast<const uint8_t*>(actions);
        else a64 = static_cast<const long long*>(actions);
    } else {
        if (dtype != NESLE_ACTIONS_U8) return fail(NESLE_ERR_INVALID, "host actions must be uint8 masks");
        CUDA_TRY(cudaMemcpyAsync(b->d_host_actions, actions, b->n, cudaMemcpyHostToDevice, s), "copy actions");
        a8 = b->d_host_actions;
    }
    uint32_t flags = (device_api ? kStepDeviceApi : 0u) | (auto_reset ? kStepAutoReset : 0u);
    return finish(b, s, launch_step(b->dv, b->n, a8, a64, flags, b->step_variant, b->step_threads, s, prof_op, prof_pc,
                              b->board),
                  "step kernel");
}

int nesle_step(nesle_batch* b, const void* actions, int dtype, int on_device, int device_api, int auto_reset,
               void* stream) {
    if (!b) return fail(NESLE_ERR_INVALID, "step: null argument");
    DeviceGuard guard(b->device);
    return step_impl(b, actions, dtype, on_device, device_api, auto_reset, static_cast<cudaStream_t>(stream), nullptr,
                     nullptr);
}

int nesle_step_profile(nesle_batch* b, const void* actions, int dtype, int on_device, void* stream,
                       uint64_t* opcode_counts, uint64_t* pc_counts) {
    if (!b) return fail(NESLE_ERR_INVALID, "step_profile: null argument");
    DeviceGuard guard(b->device);
    auto s = static_cast<cudaStream_t>(stream);
    if (!b->d_prof) TRY(b->alloc(&b->d_prof, 256 + 65536, "profile histograms"));
    CUDA_TRY(cudaMemsetAsync(b->d_prof, 0, (256 + 65536) * sizeof(unsigned long long), s), "clear profile");
    TRY(step_impl(b, actions, dtype, on_device, 0, 0, s, b->d_prof, b->d_prof + 256));
    if (opcode_counts)
        CUDA_TRY(cudaMemcpyAsync(opcode_counts, b->d_prof, 256 * sizeof(uint64_t), cudaMemcpyDeviceToHost, s),
                 "copy opcode profile");
    if (pc_counts)
        CUDA_TRY(cudaMemcpyAsync(pc_counts, b->d_prof + 256, 65536 * sizeof(uint64_t), cudaMemcpyDeviceToHost, s),
                 "copy pc profile");
    CUDA_TRY(cudaStreamSynchronize(s), "step profile synchronize");
    return NESLE_OK;
}

static int ensure_frames(nesle_batch* b, int which) {
    const size_t n = b->n;
    if (which == NESLE_PTR_FRAMES_RGB && !b->d_frames_rgb)
        return b->alloc(&b->d_frames_rgb, n * kFrameW * kFrameH * 3, "frames rgb");
    if (which == NESLE_PTR_FRAMES_INDEX && !b->d_frames_index)
        return b->alloc(&b->d_frames_index, n * kFrameW * kFrameH, "frames index");
    if (which == NESLE_PTR_OBS_GRAY84 && !b->d_gray84) return b->alloc(&b->d_gray84, n * kGray * kGray, "gray84");
    return NESLE_OK;
}

int nesle_render(nesle_batch* b, int mode, void* stream) {
    if (!b) return fail(NESLE_ERR_INVALID, "null batch");
    if (mode < NESLE_RENDER_RGB || mode > NESLE_RENDER_GRAY84) return fail(NESLE_ERR_INVALID, "unknown render mode");
    DeviceGuard guard(b->device);
    const int which = mode == NESLE_RENDER_RGB ? NESLE_PTR_FRAMES_RGB
                      : mode == NESLE_RENDER_INDEX ? NESLE_PTR_FRAMES_INDEX : NESLE_PTR_OBS_GRAY84;
    TRY(ensure_frames(b, which));
    uint8_t* out = mode == NESLE_RENDER_RGB ? b->d_frames_rgb : mode == NESLE_RENDER_INDEX ? b->d_frames_index : b->d_gray84;
    auto s = static_cast<cudaStream_t>(stream);
    return finish(b, s, launch_render(b->dv, 0, b->n, out, mode, s), "render kernel");
}

// Rendered in kRenderChunks env ranges on `stream`; each range's rows are
// copied to the host on the batch's copy stream as soon as they are done, so
// the copy of one range overlaps the rendering of the next.
int nesle_render_copy(nesle_batch* b, int mode, void* host_out, uint64_t bytes, void* stream) {
    if (!b || !host_out) return fail(NESLE_ERR_INVALID, "render_copy: null argument");
    if (mode < NESLE_RENDER_RGB || mode > NESLE_RENDER_GRAY84) return fail(NESLE_ERR_INVALID, "unknown render mode");
    const uint64_t per_env = mode == NESLE_RENDER_RGB ? (uint64_t)kFrameW * kFrameH * 3
                             : mode == NESLE_RENDER_INDEX ? (uint64_t)kFrameW * kFrameH : (uint64_t)kGray * kGray;
    if (bytes != (uint64_t)b->n * per_env) return fail(NESLE_ERR_INVALID, "render_copy: wrong output size");
    DeviceGuard guard(b->device);
    const int which = mode == NESLE_RENDER_RGB ? NESLE_PTR_FRAMES_RGB
                      : mode == NESLE_RENDER_INDEX ? NESLE_PTR_FRAMES_INDEX : NESLE_PTR_OBS_GRAY84;
    TRY(ensure_frames(b, which));
    uint8_t* dev = mode == NESLE_RENDER_RGB ? b->d_frames_rgb : mode == NESLE_RENDER_INDEX ? b->d_frames_index : b->d_gray84;
    if (!b->copy_stream) CUDA_TRY(cudaStreamCreateWithFlags(&b->copy_stream, cudaStreamNonBlocking), "copy stream");
    for (cudaEvent_t& e : b->chunk_events)
        if (!e) CUDA_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "chunk event");
    auto s = static_cast<cudaStream_t>(stream);
    const uint32_t per_chunk = (b->n + kRenderChunks - 1) / kRenderChunks;
    auto* host = static_cast<uint8_t*>(host_out);
    for (uint32_t k = 0; k < kRenderChunks; ++k) {
        const uint32_t env0 = k * per_chunk;
        if (env0 >= b->n) break;
        const uint32_t count = per_chunk < b->n - env0 ? per_chunk : b->n - env0;
        CUDA_TRY(launch_render(b->dv, env0, count, dev, mode, s), "render kernel");
        CUDA_TRY(cudaEventRecord(b->chunk_events[k], s), "record chunk event");
        CUDA_TRY(cudaStreamWaitEvent(b->copy_stream, b->chunk_events[k], 0), "copy stream wait");
        CUDA_TRY(cudaMemcpyAsync(host + env0 * per_env, dev + env0 * per_env, count * per_env, cudaMemcpyDeviceToHost,
                                 b->copy_stream), "copy rendered chunk");
    }
    CUDA_TRY(cudaEventRecord(b->done_event, s), "record event");
    CUDA_TRY(cudaStreamSynchronize(b->copy_stream), "synchronize copies");
    return NESLE_OK;
}

int nesle_host_alloc(uint64_t bytes, void** out) {
    if (!out || !bytes) return fail(NESLE_ERR_INVALID, "host_alloc: null output or zero size");
    *out = nullptr;
    CUDA_TRY(cudaHostAlloc(out, bytes, cudaHostAllocPortable), "host alloc");
    return NESLE_OK;
}

int nesle_host_free(void* ptr) {
    if (ptr) CUDA_TRY(cudaFreeHost(ptr), "host free");
    return NESLE_OK;
}

uint64_t nesle_state_bytes(void) { return kStateBytes; }

static int state_io(nesle_batch* b, const uint32_t* envs, uint32_t count, int envs_on_device, void* blobs,
                    int blobs_on_device, bool save, void* stream) {
    if (!b || (count && (!envs || !blobs))) return fail(NESLE_ERR_INVALID, "state: null argument");
    DeviceGuard guard(b->device);
    auto s = static_cast<cudaStream_t>(stream);
    if (!envs_on_device)
        for (uint32_t i = 0; i < count; ++i)
            if (envs[i] >= b->n)
                return fail(NESLE_ERR_INVALID, "env index " + std::to_string(envs[i]) + " out of range (batch of " +
                                                   std::to_string(b->n) + ")");
    if ((!envs_on_device || !blobs_on_device) && count > b->state_cap) {
        // staging grows to the largest request; the outgrown pair is freed
        CUDA_TRY(cudaStreamSynchronize(s), "state staging synchronize");
        b->free_one(b->d_state_envs);
        b->free_one(b->d_state_blobs);
        b->d_state_envs = nullptr;
        b->d_state_blobs = nullptr;
        b->state_cap = 0;
        TRY(b->alloc(&b->d_state_envs, count, "state env list"));
        TRY(b->alloc(&b->d_state_blobs, (size_t)count * kStateBytes, "state blobs"));
        b->state_cap = count;
    }
    const uint32_t* d_envs = static_cast<const uint32_t*>(static_cast<const void*>(envs));
    if (!envs_on_device) {
        CUDA_TRY(cudaMemcpyAsync(b->d_state_envs, envs, count * sizeof(uint32_t), cudaMemcpyHostToDevice, s),
                 "copy env list");
        d_envs = b->d_state_envs;
    }
    uint8_t* d_blobs = blobs_on_device ? static_cast<uint8_t*>(blobs) : b->d_state_blobs;
    if (!save && !blobs_on_device)
        CUDA_TRY(cudaMemcpyAsync(d_blobs, blobs, (size_t)count * kStateBytes, cudaMemcpyHostToDevice, s),
                 "copy state blobs");
    TRY(finish(b, s, launch_state(b->dv, d_envs, count, d_blobs, save, s), save ? "save states" : "load states"));
    if (save && !blobs_on_device) {
        CUDA_TRY(cudaMemcpyAsync(blobs, d_blobs, (size_t)count * kStateBytes, cudaMemcpyDeviceToHost, s),
                 "copy state blobs");
        CUDA_TRY(cudaStreamSynchronize(s), "save states synchronize");
    }
    if (!save && !blobs_on_device) CUDA_TRY(cudaStreamSynchronize(s), "load states synchronize");
    return NESLE_OK;
}

int nesle_save_states(nesle_batch* b, const uint32_t* envs, uint32_t count, int envs_on_device, void* dst,
                      int dst_on_device, void* stream) {
    return state_io(b, envs, count, envs_on_device, dst, dst_on_device, true, stream);
}

int nesle_load_states(nesle_batch* b, const uint32_t* envs, uint32_t count, int envs_on_device, const void* src,
                      int src_on_device, void* stream) {
    return state_io(b, envs, count, envs_on_device, const_cast<void*>(src), src_on_device, false, stream);
}

int nesle_poke_ram(nesle_batch* b, uint16_t address, uint8_t value, void* stream) {
    if (!b) return fail(NESLE_ERR_INVALID, "null batch");
    DeviceGuard guard(b->device);
    auto s = static_cast<cudaStream_t>(stream);
    return finish(b, s, launch_poke(b->dv, b->n, address, value, s), "poke kernel");
}

int nesle_device_ptr(nesle_batch* b, int which, void** ptr, uint64_t* bytes) {
    if (!b || !ptr || !bytes) return fail(NESLE_ERR_INVALID, "device_ptr: null argument");
    DeviceGuard guard(b->device);
    const uint64_t n = b->n;
    switch (which) {
        case NESLE_PTR_RAM: *ptr = b->hv.ram; *bytes = n * kRamBytes; return NESLE_OK;
        case NESLE_PTR_LAST_REWARDS: *ptr = b->hv.last_rewards; *bytes = n * 4; return NESLE_OK;
        case NESLE_PTR_LAST_DONE: *ptr = b->hv.last_done; *bytes = n; return NESLE_OK;
        case NESLE_PTR_REWARDS: *ptr = b->hv.rewards; *bytes = n * 4; return NESLE_OK;
        case NESLE_PTR_DONE: *ptr = b->hv.done; *bytes = n; return NESLE_OK;
        case NESLE_PTR_FRAMES_RGB:
            TRY(ensure_frames(b, which)); *ptr = b->d_frames_rgb; *bytes = n * kFrameW * kFrameH * 3; return NESLE_OK;
        case NESLE_PTR_FRAMES_INDEX:
            TRY(ensure_frames(b, which)); *ptr = b->d_frames_index; *bytes = n * kFrameW * kFrameH; return NESLE_OK;
        case NESLE_PTR_OBS_GRAY84:
            TRY(ensure_frames(b, which)); *ptr = b->d_gray84; *bytes = n * kGray * kGray; return NESLE_OK;
        default: return fail(NESLE_ERR_INVALID, "unknown device array");
    }
}

namespace {
struct FieldDesc { const char* name; size_t off, width; };
#define RF(nm, member) {nm, offsetof(EnvRecord, member), sizeof(((EnvRecord*)nullptr)->member)}
const FieldDesc kRecordFields[] = {
    RF("pc", pc), RF("a", a), RF("x", x), RF("y", y), RF("sp", sp), RF("p", p), RF("nmi_pending", nmi_pending),
    RF("cycles", cycles), RF("frame", frame), RF("frame_dot", frame_dot), RF("ppu_ctrl", ppu_ctrl),
    RF("ppu_mask", ppu_mask), RF("ppu_status", ppu_status), RF("oam_addr", oam_addr), RF("v", v), RF("t", t),
    RF("fine_x", fine_x), RF("w", w), RF("open_bus", open_bus), RF("read_buffer", read_buffer),
    RF("scroll_x", scroll_x), RF("scroll_y", scroll_y), RF("lat_sx", lat_sx), RF("lat_sy", lat_sy),
    RF("lat_ctrl", lat_ctrl), RF("snap_sx_start", snap_sx_start), RF("snap_sy_start", snap_sy_start),
    RF("snap_ctrl_start", snap_ctrl_start), RF("snap_sx_end", snap_sx_end), RF("snap_sy_end", snap_sy_end),
    RF("snap_ctrl_end", snap_ctrl_end), RF("snap_mask", snap_mask), RF("ctrl_shift", ctrl_shift),
    RF("ctrl_count", ctrl_count), RF("ctrl_strobe", ctrl_strobe), RF("prev_x", prev_x), RF("prev_time", prev_time),
    RF("pending_dma", pending_dma), RF("episode", episode), RF("status", status),
    RF("stat_instructions", stat_instructions), RF("stat_frames", stat_frames),
    RF("stat_budget_hits", stat_budget_hits),
};
#undef RF
}  // namespace

int nesle_copy_field(nesle_batch* b, const char* name, void* host_out, uint64_t bytes) {
    if (!b || !name || !host_out) return fail(NESLE_ERR_INVALID, "copy_field: null argument");
    DeviceGuard guard(b->device);
    CUDA_TRY(cudaEventSynchronize(b->done_event), "synchronize");
    const std::string f = name;
    const uint64_t n = b->n;
    struct Arr { const char* name; const void* ptr; uint64_t width; };
    const Arr arrays[] = {
        {"ram", b->hv.ram, kRamBytes}, {"prg_ram", b->hv.prg_ram, kPrgRamBytes}, {"nametable", b->hv.nt, kNtBytes},
        {"palette", b->hv.pal, kPalBytes}, {"oam", b->hv.oam, kOamBytes}, {"snap_nametable", b->hv.snap_nt, kNtBytes},
        {"snap_palette", b->hv.snap_pal, kPalBytes}, {"snap_oam", b->hv.snap_oam, kOamBytes},
        {"rewards", b->hv.rewards, 4}, {"done", b->hv.done, 1}, {"last_rewards", b->hv.last_rewards, 4},
        {"last_done", b->hv.last_done, 1}, {"frames_rgb", b->d_frames_rgb, kFrameW * kFrameH * 3},
        {"frames_index", b->d_frames_index, kFrameW * kFrameH}, {"obs_gray84", b->d_gray84, kGray * kGray},
    };
    for (const auto& a : arrays) {
        if (f == a.name) {
            if (!a.ptr) return fail(NESLE_ERR_RUNTIME, "copy_field: " + f + " has not been rendered yet");
            if (bytes != n * a.width) return fail(NESLE_ERR_INVALID, "copy_field: wrong output size for " + f);
            CUDA_TRY(cudaMemcpy(host_out, a.ptr, bytes, cudaMemcpyDeviceToHost), "copy field");
            return NESLE_OK;
        }
    }
    const char* board_fields[] = {"prg_bank", "chr_bank", "snap_chr_bank"};
    for (uint32_t k = 0; k < 3; ++k) {
        if (f == board_fields[k]) {
            if (bytes != n) return fail(NESLE_ERR_INVALID, "copy_field: wrong output size for " + f);
            std::vector<MapperState> ms(n);
            CUDA_TRY(cudaMemcpy(ms.data(), b->hv.mstate, n * sizeof(MapperState), cudaMemcpyDeviceToHost),
                     "copy board registers");
            auto* out = static_cast<uint8_t*>(host_out);
            for (uint64_t e = 0; e < n; ++e) out[e] = reinterpret_cast<const uint8_t*>(&ms[e])[k];
            return NESLE_OK;
        }
    }
    for (const auto& d : kRecordFields) {
        if (f == d.name) {
            if (bytes != n * d.width) return fail(NESLE_ERR_INVALID, "copy_field: wrong output size for " + f);
            std::vector<EnvRecord> recs(n);
            CUDA_TRY(cudaMemcpy(recs.data(), b->hv.rec, n * sizeof(EnvRecord), cudaMemcpyDeviceToHost), "copy records");
            auto* out = static_cast<uint8_t*>(host_out);
            for (uint64_t e = 0; e < n; ++e)
                memcpy(out + e * d.width, reinterpret_cast<const uint8_t*>(&recs[e]) + d.off, d.width);
            return NESLE_OK;
        }
    }
    return fail(NESLE_ERR_INVALID, "unknown field " + f);
}

int nesle_sync(nesle_batch* b) {
    if (!b) return fail(NESLE_ERR_INVALID, "null batch");
    DeviceGuard guard(b->device);
    CUDA_TRY(cudaEventSynchronize(b->done_event), "synchronize");
    return NESLE_OK;
}

int nesle_stream_wait(nesle_batch* b, void* consumer_stream) {
    if (!b) return fail(NESLE_ERR_INVALID, "null batch");
    DeviceGuard guard(b->device);
    CUDA_TRY(cudaStreamWaitEvent(static_cast<cudaStream_t>(consumer_stream), b->done_event, 0), "stream wait");
    return NESLE_OK;
}

int nesle_fault_count(nesle_batch* b, uint32_t* count) {
    if (!b || !count) return fail(NESLE_ERR_INVALID, "fault_count: null argument");
    DeviceGuard guard(b->device);
    CUDA_TRY(cudaEventSynchronize(b->done_event), "synchronize");
    CUDA_TRY(cudaMemcpy(count, b->hv.fault_count, sizeof(uint32_t), cudaMemcpyDeviceToHost), "copy fault count");
    return NESLE_OK;
}

// No-allocation 84x84 observation: the render kernel writes into a file-scope
// device scratch (module memory, set up once per device by
// cudaGetSymbolAddress at nesle_create) and the result is copied to the
// caller's host buffer.  No cudaMalloc / cudaFree.  Concurrent calls on one
// device share the scratch and race.  Every scratch byte the call reads is
// written by the kernel first, so nothing needs clearing.  The call ends with
// a synchronisation of its stream, so it cannot be made while that stream is
// capturing.
int nesle_render_gray84_noalloc(nesle_batch* b, uint8_t* host_out, uint64_t bytes, void* stream) {
    if (!b || !host_out) return fail(NESLE_ERR_INVALID, "render_gray84_noalloc: null argument");
    if (b->n > kNoAllocGrayEnvs)
        return fail(NESLE_ERR_INVALID, "render_gray84_noalloc: batch of " + std::to_string(b->n) +
                                           " envs exceeds its static scratch (at most " +
                                           std::to_string(kNoAllocGrayEnvs) + " envs)");
    if (bytes != (uint64_t)b->n * kGray * kGray)
        return fail(NESLE_ERR_INVALID, "render_gray84_noalloc: expected " + std::to_string((uint64_t)b->n * kGray * kGray) +
                                           " bytes, got " + std::to_string(bytes));
    DeviceGuard guard(b->device);
    uint8_t* scratch = nullptr;
    TRY(noalloc_scratch(b->device, &scratch));
    auto s = static_cast<cudaStream_t>(stream);
    CUDA_TRY(launch_render(b->dv, 0, b->n, scratch, NESLE_RENDER_GRAY84, s), "render_gray84_noalloc kernel");
    CUDA_TRY(cudaMemcpyAsync(host_out, scratch, bytes, cudaMemcpyDeviceToHost, s), "render_gray84_noalloc copy");
    CUDA_TRY(cudaEventRecord(b->done_event, s), "record event");
    CUDA_TRY(cudaStreamSynchronize(s), "render_gray84_noalloc synchronize");
    return NESLE_OK;
}

int nesle_get_info(nesle_batch* b, nesle_info* out) {
    if (!b || !out) return fail(NESLE_ERR_INVALID, "get_info: null argument");
    out->num_envs = b->n;
    out->frameskip = b->frameskip;
    out->num_levels = b->num_levels;
    out->device = static_cast<uint32_t>(b->device);
    out->envs_per_block = b->step_variant == kStepSharedRam ? kStepSlots : b->step_threads;
    out->step_placement = b->step_variant;  // the kStep* values equal NESLE_PLACEMENT_*
    out->smem_bytes_per_block = b->step_variant == kStepSharedRam
                                    ? static_cast<uint32_t>(step_smem_bytes())
                                    : static_cast<uint32_t>(global_step_smem(b->step_variant, b->step_threads));
    return NESLE_OK;
}

}  // extern "C"
