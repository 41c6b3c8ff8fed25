// Runtime core of libvolta_cuda_backend.so (B200 / sm_100a).
//
// One Context per (host thread, GPU): a single non-blocking stream, a
// generational device arena addressed by opaque u64 ids, a pinned host pool,
// private workspaces, and the measurement observer that backs the reference's
// RawStats ABI.  Semantics follow the reference seam
// (cuda/volta_cuda_backend.cu:182-330 context/arena, 355-403 errors,
//  1035-1240 timing, 3148-3960 ABI entry points); the implementation is this
// project's own.
#pragma once

#include <cuda_runtime.h>

#include <array>
#include <chrono>
#include <cstdint>
#include <cstring>
#include <limits>
#include <set>
#include <string>
#include <vector>

#include "../../include/volta_b200_ext.h"
#include "field.cuh"

namespace vzb {

constexpr uint32_t kAbiVersion = 37;

// Operation classes of the stats ABI (rust/volta-accel/src/lib.rs:27-59).
enum Op : int {
    kOpGemm = 0,
    kOpLogup = 1,
    kOpPcsRows = 2,
    kOpPcsNtt = 3,
    kOpPcsMerkle = 4,
    kOpAuthMasks = 5,
    kOpMailbox = 6,
    kOpCount = 7,
};

// Observation modes (cuda/volta_cuda_backend.cu:42-46).
enum TimingMode : uint32_t {
    kTimingEvents = 1,       // events + one synchronisation per primitive
    kTimingHostBarrier = 2,  // host barriers (runtimes without elapsed time)
    kTimingDeferred = 3,     // ring of events resolved at host boundaries
    kTimingCounters = 4,     // counters only, no CUDA events
};

constexpr size_t kRingSize = 512;
constexpr uint64_t kSlotMask = 0xFFFFFFFFull;
constexpr uint32_t kGenerationMax = 0xFFFFFFFFu;
constexpr uint64_t kMockReservedDomainBits = (1ull << 63) | (1ull << 62) | (1ull << 61);

// ---- C ABI structs (layouts frozen by rust/volta-accel/src/cuda.rs:21-121) ----
using RawStats = ::vz_raw_stats;
using RawPinnedMemoryStats = ::vz_raw_pinned_stats;
using RawX4cControlState = ::vz_raw_control_state;
static_assert(sizeof(RawStats) == 504, "RawStats layout is part of the C ABI");
static_assert(sizeof(RawPinnedMemoryStats) == 104, "pinned stats layout is part of the C ABI");
static_assert(sizeof(RawX4cControlState) == 104, "control-state layout is part of the C ABI");

enum class Sync { HostOutput, UploadLifetime, TimingFlush, ProfilingLegacy, AllocatorFlush };

// Device allocation owned by the arena.  Freed slots keep their storage for
// best-fit reuse; an id is (generation << 32) | (slot + 1).
struct Slot {
    void* ptr = nullptr;
    size_t capacity = 0;
    size_t logical = 0;
    uint32_t generation = 0;
    bool active = false;
};

struct PinnedSlot {
    void* ptr = nullptr;
    size_t capacity = 0;
    size_t logical = 0;
    cudaEvent_t ready = nullptr;  // recorded after the last H2D that read it
    uint32_t generation = 0;
    bool active = false;
    bool in_flight = false;
};

enum class RecordKind : uint8_t { Primitive, Coarse, Upload, Download };

struct Record {
    cudaEvent_t ev[4] = {};
    RecordKind kind = RecordKind::Primitive;
    int op = -1;
    uint8_t mask = 0;
    bool committed = false;
    uint64_t h2d = 0, d2h = 0, d2d = 0, zeroed = 0, generated = 0;
    uint64_t ns[3] = {};
};

// Grow-only private workspace (never visible through the arena).
constexpr int kTimingMarkers = 16;  // measurement marker slots (extension ABI)

struct Workspace {
    void* ptr = nullptr;
    size_t capacity = 0;
};

enum WorkspaceSlot : int {
    kWsPartials = 0,   // per-block reduction partials
    kWsMailbox = 1,    // device mailbox for host-bound round messages
    kWsCounter = 2,    // last-block-done counters (zeroed once)
    kWsTwiddles = 3,   // NTT twiddles
    kWsStageA = 4,     // staged (hybrid) inputs
    kWsStageB = 5,
    kWsStageC = 6,
    kWsStageD = 7,
    kWsStageE = 8,
    kWsStageF = 9,
    kWsStageG = 10,
    kWsStageH = 11,
    kWsScratch = 12,   // miscellaneous scratch
    kWsScratch2 = 13,
    kWsGemm = 14,      // byte planes of the GEMM operands
    kWsScratch3 = 15,  // split-k partial sums of the few-row products
    kWsCount = 16,
};

constexpr size_t kStageSlotBytes = size_t{64} << 10;
constexpr int kStageSlots = 64;

struct Context {
    int device = 0;
    int sm_count = 148;
    cudaStream_t stream = nullptr;
    cudaEvent_t sync_ev[4] = {};
    Workspace ws[kWsCount];
    // Mapped pinned mailbox: kernels write host-bound messages here directly.
    void* host_mailbox = nullptr;
    void* host_mailbox_dev = nullptr;

    std::vector<Slot> slots;
    // Free slots: with memory, ordered by (capacity, slot) for the best fit
    // in O(log n); without memory (trimmed); retired (generation exhausted)
    // but still holding memory until the next trim.
    std::set<std::pair<size_t, size_t>> free_fit;
    std::vector<size_t> free_empty, free_retired;
    std::vector<PinnedSlot> pinned;
    std::vector<size_t> free_pinned;

    RawStats stats{};
    uint32_t mode = kTimingEvents;
    std::array<Record, kRingSize> ring;
    size_t ring_head = 0, ring_pending = 0;
    size_t active_record = kRingSize;
    uint32_t inject_no_write = 0;

    bool coarse = false;        // inside a coarse scope
    bool coarse_inner = false;  // a primitive is running inside it
    bool coarse_work = false;   // the scope already accounted work
    int coarse_op = -1;
    bool counter_active = false;
    bool counter_pending = false;
    bool poisoned = false;
    uint64_t outstanding = 0;
    std::chrono::steady_clock::time_point phase_start{};
    uint64_t phase_ns[3] = {};
    size_t twiddle_n = 0;
    uint32_t mail_seq = 0;               // sequence number of host-bound messages
    uint64_t launches = 0;               // kernels launched by this context
    cudaEvent_t bench_ev[kTimingMarkers] = {};        // measurement markers (extension ABI)
    // Pinned, device-mapped staging ring for small uploads: the bytes are
    // copied into a slot at call time and a one-block kernel on the compute
    // stream copies the slot into device memory.  A pageable source could
    // make cudaMemcpyAsync synchronise with the stream, and a copy-engine
    // transfer queued behind this stream's kernels would hold up other
    // streams' copies behind it (another context's bulk uploads share the
    // engine), so small uploads do not use the copy engine at all.
    void* stage = nullptr;
    void* stage_dev = nullptr;
    cudaEvent_t stage_ev[kStageSlots] = {};
    bool stage_used[kStageSlots] = {};
    int stage_next = 0;
    // asynchronous uploads (extension): a copy stream and the event of its
    // last copy, which volta_b200_wait_uploads makes the compute stream wait on
    cudaStream_t copy_stream = nullptr;
    cudaEvent_t copy_ev = nullptr;
    // asynchronous downloads (extension): a second copy stream; dl_ev orders
    // each copy after the compute work enqueued before it, dl_done_ev orders
    // later compute work (which may reuse a freed buffer) after the copies
    cudaStream_t dl_stream = nullptr;
    cudaEvent_t dl_ev = nullptr, dl_done_ev = nullptr;
    bool dl_pending = false;
    std::string error;
};

// A context may be driven from any host thread: make its device the
// calling thread's current device (a new thread starts on device 0).
inline int bind_device(Context* c) {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur == c->device) return 0;
    return cudaSetDevice(c->device) == cudaSuccess ? 0 : -1;
}

// ---- errors -------------------------------------------------------------
int fail_message(Context* c, const char* message) noexcept;
int fail_cuda(Context* c, const char* what, cudaError_t e) noexcept;
int reject(Context* c, const char* message) noexcept;

// After every kernel launch: count it and surface launch errors.
#define VZB_LAUNCHED(c)                                                  \
    do {                                                                 \
        ++(c)->launches;                                                 \
        cudaError_t vzb_l_ = cudaGetLastError();                         \
        if (vzb_l_ != cudaSuccess) return ::vzb::fail_cuda((c), "kernel launch", vzb_l_); \
    } while (0)

#define VZB_CUDA(c, call)                                            \
    do {                                                             \
        cudaError_t vzb_e_ = (call);                                 \
        if (vzb_e_ != cudaSuccess) return ::vzb::fail_cuda((c), #call, vzb_e_); \
    } while (0)

// ---- arithmetic helpers ---------------------------------------------------
inline bool mul_ok(size_t a, size_t b, size_t* out) {
    if (a && b > std::numeric_limits<size_t>::max() / a) return false;
    *out = a * b;
    return true;
}
inline bool add_ok(size_t a, size_t b, size_t* out) {
    if (b > std::numeric_limits<size_t>::max() - a) return false;
    *out = a + b;
    return true;
}

// ---- arena ------------------------------------------------------------------
Slot* find_slot(Context* c, uint64_t id);
// Resolve [offset_bytes, offset_bytes + bytes) of buffer `id`.
int region(Context* c, uint64_t id, size_t offset_bytes, size_t bytes, void** out);
// Same with element offsets/counts (overflow-checked).
int region_elems(Context* c, uint64_t id, size_t offset, size_t count, size_t elem, void** out);
int strided_region(Context* c, uint64_t id, size_t offset, size_t stride, size_t row_bytes,
                   size_t rows, void** out, size_t* span);
int ensure_ws(Context* c, int slot, size_t bytes);
template <typename T>
T* ws(Context* c, int slot) {
    return static_cast<T*>(c->ws[slot].ptr);
}

// ---- measurement -----------------------------------------------------------
int sync_stream(Context* c, Sync reason);
int op_begin(Context* c);
int op_mark(Context* c, int which);  // 1 = inputs staged, 2 = kernels enqueued
int op_finish(Context* c, int op, uint64_t h2d, uint64_t d2h, uint64_t d2d = 0,
              uint64_t zeroed = 0, uint64_t generated = 0);
// Host-bound round messages: the reducing kernel writes the message into the
// mapped mailbox, then (after a system fence) `seq` into the flag word.
constexpr size_t kMailboxFlagOffset = 1024;
// Word of the mailbox in which a kernel whose bounded wait ran out of time
// records a nonzero code; every stream synchronisation checks and clears it.
constexpr size_t kMailboxFaultOffset = 2048;
inline unsigned* device_fault_word(Context* c) {
    return reinterpret_cast<unsigned*>(static_cast<char*>(c->host_mailbox_dev) + kMailboxFaultOffset);
}
// Finish a primitive whose output is a message in the mapped mailbox.  In the
// wall-only counter mode the host waits on the flag (no stream
// synchronisation); the other modes synchronise as op_finish does.
int op_finish_message(Context* c, int op, uint64_t d2h_bytes, uint32_t seq);
int xfer_begin(Context* c);
int xfer_finish(Context* c, size_t bytes, bool h2d);

// Launch geometry: blocks for a grid-stride kernel over `items`.
inline unsigned grid_for(Context* c, size_t items, unsigned threads, unsigned per_sm = 8) {
    size_t need = (items + threads - 1) / threads;
    size_t cap = static_cast<size_t>(c->sm_count) * per_sm;
    if (need < 1) need = 1;
    return static_cast<unsigned>(need < cap ? need : cap);
}

}  // namespace vzb
