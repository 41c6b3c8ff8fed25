// Context, arena, pinned pool, measurement observer and their C ABI.
//
// Reference semantics (okrame/volta-zk cuda/volta_cuda_backend.cu):
//   ids / arena / regions       182-330, 3733-3960
//   errors                      355-403
//   timing modes and stats      42-124, 1035-1270, 3213-3420
//   pinned pool                 194-203, 3570-3730
#include "runtime.cuh"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>

namespace vzb {

// ---------------------------------------------------------------------------
// errors
// ---------------------------------------------------------------------------

static void drop_active_record(Context* c) noexcept {
    if (!c) return;
    if (c->coarse_work) c->poisoned = true;
    if (c->active_record != kRingSize) {
        c->ring[c->active_record].mask = 0;
        c->ring[c->active_record].committed = false;
    }
    c->active_record = kRingSize;
    c->coarse = false;
    c->coarse_inner = false;
    c->counter_active = false;
    c->coarse_work = false;
    c->coarse_op = -1;
}

int fail_message(Context* c, const char* message) noexcept {
    drop_active_record(c);
    if (c) {
        try {
            c->error = message;
        } catch (...) {
        }
    }
    return -1;
}

int fail_cuda(Context* c, const char* what, cudaError_t e) noexcept {
    drop_active_record(c);
    // consume a non-sticky error so it cannot surface again at a later launch
    (void)cudaGetLastError();
    if (c) {
        try {
            c->error = std::string(what) + ": " + cudaGetErrorString(e);
        } catch (...) {
        }
    }
    return e == cudaSuccess ? -1 : static_cast<int>(e);
}

int reject(Context* c, const char* message) noexcept {
    if (c) {
        try {
            c->error = message;
        } catch (...) {
        }
    }
    return -1;
}

// ---------------------------------------------------------------------------
// arena
// ---------------------------------------------------------------------------

static uint64_t make_id(size_t slot, uint32_t gen) {
    return (static_cast<uint64_t>(gen) << 32) | static_cast<uint64_t>(slot + 1);
}

Slot* find_slot(Context* c, uint64_t id) {
    if (!c || !id) return nullptr;
    const uint64_t enc = id & kSlotMask;
    const uint32_t gen = static_cast<uint32_t>(id >> 32);
    if (!enc || !gen) return nullptr;
    const size_t slot = static_cast<size_t>(enc - 1);
    if (slot >= c->slots.size()) return nullptr;
    Slot& s = c->slots[slot];
    return (s.active && s.generation == gen) ? &s : nullptr;
}

int region(Context* c, uint64_t id, size_t offset, size_t bytes, void** out) {
    Slot* s = find_slot(c, id);
    if (!s) return fail_message(c, "unknown resident buffer id");
    if (offset > s->logical || bytes > s->logical - offset)
        return fail_message(c, "resident buffer region is out of bounds");
    *out = static_cast<unsigned char*>(s->ptr) + offset;
    return 0;
}

int region_elems(Context* c, uint64_t id, size_t offset, size_t count, size_t elem, void** out) {
    size_t ob = 0, nb = 0;
    if (!mul_ok(offset, elem, &ob) || !mul_ok(count, elem, &nb))
        return fail_message(c, "resident geometry overflows size_t");
    return region(c, id, ob, nb, out);
}

int strided_region(Context* c, uint64_t id, size_t offset, size_t stride, size_t row_bytes,
                   size_t rows, void** out, size_t* span) {
    if (!rows || !row_bytes || stride < row_bytes)
        return fail_message(c, "invalid resident strided-row geometry");
    size_t prefix = 0;
    if (!mul_ok(rows - 1, stride, &prefix) || !add_ok(prefix, row_bytes, span))
        return fail_message(c, "resident strided-row geometry overflows size_t");
    return region(c, id, offset, *span, out);
}

int sync_stream_raw(Context* c) {
    const auto t0 = std::chrono::steady_clock::now();
    const cudaError_t e = cudaStreamSynchronize(c->stream);
    const auto t1 = std::chrono::steady_clock::now();
    if (e != cudaSuccess) return fail_cuda(c, "cudaStreamSynchronize", e);
    volatile unsigned* fault =
        reinterpret_cast<volatile unsigned*>(static_cast<char*>(c->host_mailbox) + kMailboxFaultOffset);
    if (*fault) {
        *fault = 0;
        return fail_message(c, "a tensor-core pipeline wait timed out; the results of the last operation are invalid");
    }
    c->counter_pending = false;
    c->outstanding = 0;
    ++c->stats.synchronizations;
    c->stats.synchronization_ns +=
        std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
    return 0;
}

static uint64_t& sync_counter(RawStats& s, Sync r) {
    switch (r) {
        case Sync::HostOutput: return s.sync_host_output;
        case Sync::UploadLifetime: return s.sync_upload_lifetime;
        case Sync::TimingFlush: return s.sync_timing_flush;
        case Sync::AllocatorFlush: return s.sync_allocator_flush;
        case Sync::ProfilingLegacy: break;
    }
    return s.sync_profiling_legacy;
}

int sync_stream(Context* c, Sync reason) {
    if (sync_stream_raw(c)) return -1;
    ++sync_counter(c->stats, reason);
    return 0;
}

static int flush_ring(Context* c, Sync reason);

static int sync_for_reclaim(Context* c) {
    if (c->mode == kTimingDeferred && c->ring_pending) return flush_ring(c, Sync::AllocatorFlush);
    return sync_stream(c, Sync::AllocatorFlush);
}

int ensure_ws(Context* c, int slot, size_t bytes) {
    if (slot < 0 || slot >= kWsCount) return fail_message(c, "invalid workspace slot");
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    Workspace& w = c->ws[slot];
    if (w.capacity >= bytes) return 0;
    if (c->coarse) {
        const std::string m = "workspace slot " + std::to_string(slot) + " growth from " +
                              std::to_string(w.capacity) + " to " + std::to_string(bytes) +
                              " bytes is forbidden inside a coarse timing scope";
        return reject(c, m.c_str());
    }
    // grow geometrically so repeated shapes settle quickly
    size_t want = std::max(bytes, w.capacity + w.capacity / 2);
    want = (want + 255) & ~size_t{255};
    if (w.ptr) {
        if (sync_for_reclaim(c)) return -1;
        VZB_CUDA(c, cudaFree(w.ptr));
        ++c->stats.physical_free_calls;
        c->stats.live_device_bytes -= w.capacity;
        w = Workspace{};
    }
    VZB_CUDA(c, cudaMalloc(&w.ptr, want));
    w.capacity = want;
    ++c->stats.allocation_calls;
    c->stats.live_device_bytes += want;
    c->stats.peak_device_bytes = std::max(c->stats.peak_device_bytes, c->stats.live_device_bytes);
    if (slot == kWsCounter) VZB_CUDA(c, cudaMemsetAsync(w.ptr, 0, want, c->stream));
    return 0;
}

// ---------------------------------------------------------------------------
// measurement observer
// ---------------------------------------------------------------------------

static cudaError_t ev_record(Context* c, cudaEvent_t e) {
    ++c->stats.timing_event_api_calls;
    return cudaEventRecord(e, c->stream);
}

static int elapsed_once(Context* c, cudaEvent_t a, cudaEvent_t b, uint64_t* out, bool* ok) {
    ++c->stats.timing_elapsed_query_attempts;
    if (c->inject_no_write) {
        --c->inject_no_write;
        ++c->stats.timing_elapsed_no_write;
        *ok = false;
        return 0;
    }
    float ms = -1.0f;
    ++c->stats.timing_event_api_calls;
    const cudaError_t e = cudaEventElapsedTime(&ms, a, b);
    if (e != cudaSuccess) return fail_cuda(c, "cudaEventElapsedTime", e);
    if (std::isfinite(ms) && ms >= 0.0f) {
        *out = static_cast<uint64_t>(ms * 1.0e6f);
        ++c->stats.timing_event_queries;
        *ok = true;
    } else {
        ++c->stats.timing_elapsed_no_write;
        *ok = false;
    }
    return 0;
}

static int elapsed(Context* c, cudaEvent_t a, cudaEvent_t b, uint64_t* out) {
    for (int i = 0; i < 4; ++i) {
        bool ok = false;
        if (elapsed_once(c, a, b, out, &ok)) return -1;
        if (ok) return 0;
    }
    return fail_message(c, "cudaEventElapsedTime returned success without a duration after bounded retries");
}

static uint8_t full_mask(RecordKind k) { return k == RecordKind::Primitive ? 0x0f : 0x03; }

static int flush_ring(Context* c, Sync reason) {
    if (c->mode != kTimingDeferred || !c->ring_pending) return 0;
    if (sync_stream(c, reason)) return -1;
    ++c->stats.timing_flush_count;
    for (size_t k = 0; k < c->ring_pending; ++k) {
        Record& r = c->ring[(c->ring_head + k) % kRingSize];
        if (!r.committed || r.mask != full_mask(r.kind))
            return fail_message(c, "invalid deferred timing record");
        if (r.kind == RecordKind::Primitive) {
            if (r.h2d && elapsed(c, r.ev[0], r.ev[1], &r.ns[0])) return -1;
            if (elapsed(c, r.ev[1], r.ev[2], &r.ns[1])) return -1;
            if (r.d2h && elapsed(c, r.ev[2], r.ev[3], &r.ns[2])) return -1;
        } else if (r.kind == RecordKind::Coarse) {
            if (elapsed(c, r.ev[0], r.ev[1], &r.ns[1])) return -1;
        } else {
            if (elapsed(c, r.ev[0], r.ev[1], &r.ns[0])) return -1;
        }
    }
    for (size_t k = 0; k < c->ring_pending; ++k) {
        Record& r = c->ring[(c->ring_head + k) % kRingSize];
        RawStats& s = c->stats;
        if (r.kind == RecordKind::Primitive) {
            ++s.calls[r.op];
            s.h2d_bytes += r.h2d;
            s.d2h_bytes += r.d2h;
            s.d2d_bytes += r.d2d;
            s.device_zeroed_bytes += r.zeroed;
            s.device_generated_bytes += r.generated;
            if (r.h2d) s.h2d_ns += r.ns[0];
            s.kernel_ns[r.op] += r.ns[1];
            if (r.d2h) s.d2h_ns += r.ns[2];
        } else if (r.kind == RecordKind::Coarse) {
            s.kernel_ns[r.op] += r.ns[1];
            s.coarse_timing_ns += r.ns[1];
        } else if (r.kind == RecordKind::Upload) {
            s.h2d_bytes += r.h2d;
            s.h2d_ns += r.ns[0];
        } else {
            s.d2h_bytes += r.d2h;
            s.d2h_ns += r.ns[0];
        }
        r.committed = false;
        r.mask = 0;
    }
    c->ring_head = (c->ring_head + c->ring_pending) % kRingSize;
    c->ring_pending = 0;
    return 0;
}

static int discard_ring(Context* c, Sync reason) {
    if (c->mode != kTimingDeferred || !c->ring_pending) return 0;
    if (sync_stream(c, reason)) return -1;
    for (size_t k = 0; k < c->ring_pending; ++k) {
        Record& r = c->ring[(c->ring_head + k) % kRingSize];
        r.committed = false;
        r.mask = 0;
    }
    c->ring_head = (c->ring_head + c->ring_pending) % kRingSize;
    c->ring_pending = 0;
    return 0;
}

static int ring_open(Context* c, RecordKind kind, int events) {
    if (c->active_record != kRingSize) return fail_message(c, "nested deferred timing record");
    if (c->ring_pending == kRingSize && flush_ring(c, Sync::TimingFlush)) return -1;
    const size_t slot = (c->ring_head + c->ring_pending) % kRingSize;
    Record& r = c->ring[slot];
    if (r.committed) return fail_message(c, "deferred timing ring would overwrite a committed record");
    for (int i = 0; i < events; ++i) {
        if (!r.ev[i]) {
            ++c->stats.timing_event_api_calls;
            VZB_CUDA(c, cudaEventCreate(&r.ev[i]));
        }
    }
    r.kind = kind;
    r.op = -1;
    r.mask = 0;
    r.h2d = r.d2h = r.d2d = r.zeroed = r.generated = 0;
    r.ns[0] = r.ns[1] = r.ns[2] = 0;
    VZB_CUDA(c, ev_record(c, r.ev[0]));
    r.mask |= 1;
    c->active_record = slot;
    return 0;
}

static int ring_commit(Context* c) {
    if (c->active_record == kRingSize) return fail_message(c, "no active deferred timing record");
    Record& r = c->ring[c->active_record];
    if (r.committed || r.mask != full_mask(r.kind))
        return fail_message(c, "deferred timing commit has incomplete event markers");
    r.committed = true;
    c->active_record = kRingSize;
    ++c->ring_pending;
    ++c->stats.timing_records;
    c->stats.timing_pending_high_water =
        std::max<uint64_t>(c->stats.timing_pending_high_water, c->ring_pending);
    return 0;
}

int op_begin(Context* c) {
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    c->phase_ns[0] = c->phase_ns[1] = c->phase_ns[2] = 0;
    if (c->coarse) {
        if (c->coarse_inner) return reject(c, "nested primitive timing inside a coarse timing scope");
        c->coarse_inner = true;
        return 0;
    }
    switch (c->mode) {
        case kTimingCounters:
            if (c->counter_active) return reject(c, "nested counter-only timing record");
            c->counter_active = true;
            return 0;
        case kTimingDeferred:
            return ring_open(c, RecordKind::Primitive, 4);
        case kTimingEvents:
            VZB_CUDA(c, ev_record(c, c->sync_ev[0]));
            return 0;
        default:
            c->phase_start = std::chrono::steady_clock::now();
            return 0;
    }
}

static int host_phase(Context* c, int phase) {
    if (sync_stream_raw(c)) return -1;
    const auto t = std::chrono::steady_clock::now();
    c->phase_ns[phase] =
        std::chrono::duration_cast<std::chrono::nanoseconds>(t - c->phase_start).count();
    c->phase_start = t;
    return 0;
}

int op_mark(Context* c, int which) {
    if (which != 1 && which != 2) return fail_message(c, "invalid timing event");
    if (c->coarse) {
        if (!c->coarse_inner) return fail_message(c, "coarse timing marker without an active primitive");
        return 0;
    }
    switch (c->mode) {
        case kTimingCounters:
            if (!c->counter_active) return fail_message(c, "counter-only timing marker without active operation");
            return 0;
        case kTimingDeferred: {
            if (c->active_record == kRingSize) return fail_message(c, "deferred timing marker without active record");
            Record& r = c->ring[c->active_record];
            VZB_CUDA(c, ev_record(c, r.ev[which]));
            r.mask |= static_cast<uint8_t>(1u << which);
            return 0;
        }
        case kTimingEvents:
            VZB_CUDA(c, ev_record(c, c->sync_ev[which]));
            return 0;
        default:
            return host_phase(c, which - 1);
    }
}

int op_finish(Context* c, int op, uint64_t h2d, uint64_t d2h, uint64_t d2d, uint64_t zeroed,
              uint64_t generated) {
    ++c->outstanding;
    RawStats& s = c->stats;
    if (c->coarse) {
        if (!c->coarse_inner) return fail_message(c, "coarse timing finish without an active primitive");
        if (op != c->coarse_op)
            return fail_message(c, "coarse timing scope received a different operation kind");
        if (h2d || d2h) {
            if (sync_stream(c, d2h ? Sync::HostOutput : Sync::UploadLifetime)) return -1;
            return fail_message(c, "host transfer is forbidden inside a coarse timing scope");
        }
        ++s.calls[op];
        s.d2d_bytes += d2d;
        s.device_zeroed_bytes += zeroed;
        s.device_generated_bytes += generated;
        c->coarse_work = true;
        if (c->mode == kTimingCounters) c->counter_pending = true;
        c->coarse_inner = false;
        return 0;
    }
    uint64_t ns0 = 0, ns1 = 0, ns2 = 0;
    if (c->mode == kTimingCounters) {
        if (!c->counter_active) return fail_message(c, "counter-only finish without active operation");
        c->counter_active = false;
        c->counter_pending = true;
        if (d2h && sync_stream(c, Sync::HostOutput)) return -1;
        ++s.calls[op];
        s.h2d_bytes += h2d;
        s.d2h_bytes += d2h;
        s.d2d_bytes += d2d;
        s.device_zeroed_bytes += zeroed;
        s.device_generated_bytes += generated;
        return 0;
    }
    if (c->mode == kTimingDeferred) {
        if (c->active_record == kRingSize) return fail_message(c, "deferred finish without active record");
        Record& r = c->ring[c->active_record];
        VZB_CUDA(c, ev_record(c, r.ev[3]));
        r.mask |= 1u << 3;
        r.kind = RecordKind::Primitive;
        r.op = op;
        r.h2d = h2d;
        r.d2h = d2h;
        r.d2d = d2d;
        r.zeroed = zeroed;
        r.generated = generated;
        if (ring_commit(c)) return -1;
        return d2h ? flush_ring(c, Sync::HostOutput) : 0;
    }
    if (c->mode == kTimingEvents) {
        VZB_CUDA(c, ev_record(c, c->sync_ev[3]));
        const Sync why = d2h ? Sync::HostOutput : (h2d ? Sync::UploadLifetime : Sync::ProfilingLegacy);
        if (sync_stream(c, why)) return -1;
        if (elapsed(c, c->sync_ev[0], c->sync_ev[1], &ns0) ||
            elapsed(c, c->sync_ev[1], c->sync_ev[2], &ns1) ||
            elapsed(c, c->sync_ev[2], c->sync_ev[3], &ns2))
            return -1;
    } else {
        if (host_phase(c, 2)) return -1;
        if (h2d) ++s.sync_upload_lifetime;
        if (d2h) ++s.sync_host_output;
        s.sync_profiling_legacy += 3 - (h2d ? 1 : 0) - (d2h ? 1 : 0);
        ns0 = c->phase_ns[0];
        ns1 = c->phase_ns[1];
        ns2 = c->phase_ns[2];
    }
    ++s.calls[op];
    s.h2d_bytes += h2d;
    s.d2h_bytes += d2h;
    s.d2d_bytes += d2d;
    s.device_zeroed_bytes += zeroed;
    s.device_generated_bytes += generated;
    if (h2d) s.h2d_ns += ns0;
    s.kernel_ns[op] += ns1;
    if (d2h) s.d2h_ns += ns2;
    return 0;
}

int op_finish_message(Context* c, int op, uint64_t d2h, uint32_t seq) {
    if (c->coarse || c->mode != kTimingCounters) return op_finish(c, op, 0, d2h);
    if (!c->counter_active) return fail_message(c, "counter-only finish without active operation");
    c->counter_active = false;
    c->counter_pending = true;
    ++c->outstanding;
    volatile uint32_t* flag =
        reinterpret_cast<volatile uint32_t*>(static_cast<char*>(c->host_mailbox) + kMailboxFlagOffset);
    const auto t0 = std::chrono::steady_clock::now();
    uint64_t spins = 0;
    while (*flag != seq) {
        if ((++spins & 255) == 0) {
            const cudaError_t q = cudaStreamQuery(c->stream);
            if (q == cudaSuccess) {
                if (*flag == seq) break;
                return fail_message(c, "round message flag missing after the stream completed");
            }
            if (q != cudaErrorNotReady) return fail_cuda(c, "cudaStreamQuery(round message)", q);
            if (std::chrono::steady_clock::now() - t0 > std::chrono::seconds(120))
                return fail_message(c, "timed out waiting for a round message");
        }
    }
    std::atomic_thread_fence(std::memory_order_acquire);  // message words are read after the flag
    const auto t1 = std::chrono::steady_clock::now();
    RawStats& s = c->stats;
    ++s.calls[op];
    s.d2h_bytes += d2h;
    ++s.synchronizations;
    ++s.sync_host_output;
    s.synchronization_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
    return 0;
}

int xfer_begin(Context* c) {
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    if (c->coarse) return reject(c, "host transfer is forbidden inside a coarse timing scope");
    switch (c->mode) {
        case kTimingCounters:
            if (c->counter_active) return reject(c, "nested counter-only timing record");
            c->counter_active = true;
            return 0;
        case kTimingDeferred:
            return ring_open(c, RecordKind::Upload, 2);
        case kTimingEvents:
            VZB_CUDA(c, ev_record(c, c->sync_ev[0]));
            return 0;
        default:
            c->phase_start = std::chrono::steady_clock::now();
            return 0;
    }
}

int xfer_finish(Context* c, size_t bytes, bool h2d) {
    ++c->outstanding;
    uint64_t ns = 0;
    if (c->mode == kTimingCounters) {
        if (!c->counter_active) return fail_message(c, "counter-only transfer finish without active transfer");
        c->counter_active = false;
        c->counter_pending = true;
        if (!h2d && sync_stream(c, Sync::HostOutput)) return -1;
        if (h2d) c->stats.h2d_bytes += bytes;
        else c->stats.d2h_bytes += bytes;
        return 0;
    }
    if (c->mode == kTimingDeferred) {
        if (c->active_record == kRingSize) return fail_message(c, "deferred transfer finish without active record");
        Record& r = c->ring[c->active_record];
        VZB_CUDA(c, ev_record(c, r.ev[1]));
        r.mask |= 1u << 1;
        r.kind = h2d ? RecordKind::Upload : RecordKind::Download;
        r.h2d = h2d ? bytes : 0;
        r.d2h = h2d ? 0 : bytes;
        if (ring_commit(c)) return -1;
        return h2d ? 0 : flush_ring(c, Sync::HostOutput);
    }
    if (c->mode == kTimingEvents) {
        VZB_CUDA(c, ev_record(c, c->sync_ev[1]));
        if (sync_stream(c, h2d ? Sync::UploadLifetime : Sync::HostOutput)) return -1;
        if (elapsed(c, c->sync_ev[0], c->sync_ev[1], &ns)) return -1;
    } else {
        if (sync_stream(c, h2d ? Sync::UploadLifetime : Sync::HostOutput)) return -1;
        ns = std::chrono::duration_cast<std::chrono::nanoseconds>(
                 std::chrono::steady_clock::now() - c->phase_start).count();
    }
    if (h2d) {
        c->stats.h2d_bytes += bytes;
        c->stats.h2d_ns += ns;
    } else {
        c->stats.d2h_bytes += bytes;
        c->stats.d2h_ns += ns;
    }
    return 0;
}

static int probe_timing(Context* c) {
    VZB_CUDA(c, ev_record(c, c->sync_ev[0]));
    VZB_CUDA(c, ev_record(c, c->sync_ev[1]));
    VZB_CUDA(c, cudaStreamSynchronize(c->stream));
    float ms = -1.0f;
    ++c->stats.timing_event_api_calls;
    const cudaError_t e = cudaEventElapsedTime(&ms, c->sync_ev[0], c->sync_ev[1]);
    if (e == cudaSuccess && ms >= 0.0f) {
        c->mode = kTimingEvents;
    } else {
        (void)cudaGetLastError();
        c->mode = kTimingHostBarrier;
    }
    c->stats.timing_mode = c->mode;
    return 0;
}

// ---- pinned pool helpers ----------------------------------------------------

static PinnedSlot* find_pinned(Context* c, uint64_t id) {
    if (!c || !id) return nullptr;
    const uint64_t enc = id & kSlotMask;
    const uint32_t gen = static_cast<uint32_t>(id >> 32);
    if (!enc || !gen) return nullptr;
    const size_t slot = static_cast<size_t>(enc - 1);
    if (slot >= c->pinned.size()) return nullptr;
    PinnedSlot& p = c->pinned[slot];
    return (p.active && p.generation == gen) ? &p : nullptr;
}

static int pinned_ready(Context* c, PinnedSlot* p, bool* ready) {
    if (!p->in_flight) {
        *ready = true;
        return 0;
    }
    const cudaError_t st = cudaEventQuery(p->ready);
    if (st == cudaSuccess) {
        p->in_flight = false;
        *ready = true;
        return 0;
    }
    if (st == cudaErrorNotReady) {
        *ready = false;
        return 0;
    }
    return fail_cuda(c, "cudaEventQuery(pinned ready)", st);
}

static int trim_resident(Context* c) {
    if (c->free_fit.empty() && c->free_retired.empty()) return 0;
    if (sync_for_reclaim(c)) return -1;
    auto release = [&](size_t s) -> int {
        Slot& b = c->slots[s];
        VZB_CUDA(c, cudaFree(b.ptr));
        ++c->stats.physical_free_calls;
        c->stats.live_device_bytes -= b.capacity;
        b.ptr = nullptr;
        b.capacity = 0;
        b.logical = 0;
        return 0;
    };
    while (!c->free_fit.empty()) {
        const size_t s = c->free_fit.begin()->second;
        c->free_fit.erase(c->free_fit.begin());
        if (release(s)) return -1;
        c->free_empty.push_back(s);
    }
    while (!c->free_retired.empty()) {  // retired slots are never handed out again
        const size_t s = c->free_retired.back();
        c->free_retired.pop_back();
        if (release(s)) return -1;
    }
    return 0;
}

static int trim_pinned(Context* c) {
    bool any = false;
    for (size_t s : c->free_pinned)
        if (!c->pinned[s].active && c->pinned[s].ptr) any = true;
    if (!any) return 0;
    if (sync_for_reclaim(c)) return -1;
    for (size_t s : c->free_pinned) {
        PinnedSlot& b = c->pinned[s];
        if (b.active || !b.ptr) continue;
        const uint32_t gen = b.generation;
        const size_t cap = b.capacity;
        if (b.ready) VZB_CUDA(c, cudaEventDestroy(b.ready));
        VZB_CUDA(c, cudaFreeHost(b.ptr));
        ++c->stats.pinned_physical_free_calls;
        c->stats.live_pinned_bytes -= cap;
        b = PinnedSlot{};
        b.generation = gen;
    }
    return 0;
}

}  // namespace vzb

using namespace vzb;

// ===========================================================================
// C ABI: context
// ===========================================================================

extern "C" uint32_t volta_cuda_abi_version(void) { return kAbiVersion; }

extern "C" int volta_cuda_create(void** out) {
    if (!out) return -1;
    *out = nullptr;
    Context* c = new (std::nothrow) Context;
    if (!c) return -1;
    *out = c;
    try {
        int count = 0;
        cudaError_t e = cudaGetDeviceCount(&count);
        if (e != cudaSuccess) return fail_cuda(c, "cudaGetDeviceCount", e);
        if (count < 1) return fail_message(c, "no CUDA device is available");
        VZB_CUDA(c, cudaGetDevice(&c->device));
        cudaDeviceProp prop{};
        VZB_CUDA(c, cudaGetDeviceProperties(&prop, c->device));
        if (prop.major < 10)
            return fail_message(c, "libvolta_cuda_backend (B200 build) requires an sm_100 device");
        c->sm_count = prop.multiProcessorCount;
        VZB_CUDA(c, cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking));
        for (auto& ev : c->sync_ev) {
            ++c->stats.timing_event_api_calls;
            VZB_CUDA(c, cudaEventCreate(&ev));
        }
        VZB_CUDA(c, cudaHostAlloc(&c->host_mailbox, 4096, cudaHostAllocMapped));
        VZB_CUDA(c, cudaHostGetDevicePointer(&c->host_mailbox_dev, c->host_mailbox, 0));
        std::memset(c->host_mailbox, 0, 4096);  // the message flag starts below every sequence number
        VZB_CUDA(c, cudaHostAlloc(&c->stage, kStageSlotBytes * kStageSlots, cudaHostAllocMapped));
        VZB_CUDA(c, cudaHostGetDevicePointer(&c->stage_dev, c->stage, 0));
        for (auto& e : c->stage_ev) VZB_CUDA(c, cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        if (ensure_ws(c, kWsCounter, 4096)) return -1;
        // per-block partials of the single-launch reductions: at most 8 blocks
        // per SM and 9 Fp2 accumulators per block (the aux round)
        if (ensure_ws(c, kWsPartials, static_cast<size_t>(c->sm_count) * 8 * 9 * sizeof(Fp2))) return -1;
        if (probe_timing(c)) return -1;
        return 0;
    } catch (...) {
        return fail_message(c, "CUDA context construction threw a C++ exception");
    }
}

extern "C" void volta_cuda_destroy(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return;
    if (c->coarse) drop_active_record(c);
    if (c->mode == kTimingDeferred) (void)flush_ring(c, Sync::TimingFlush);
    if (c->stream) (void)cudaStreamSynchronize(c->stream);
    for (auto& w : c->ws)
        if (w.ptr) cudaFree(w.ptr);
    for (auto& s : c->slots)
        if (s.ptr) cudaFree(s.ptr);
    for (auto& p : c->pinned) {
        if (p.ready) cudaEventDestroy(p.ready);
        if (p.ptr) cudaFreeHost(p.ptr);
    }
    for (auto& r : c->ring)
        for (auto e : r.ev)
            if (e) cudaEventDestroy(e);
    for (auto e : c->sync_ev)
        if (e) cudaEventDestroy(e);
    for (auto e : c->bench_ev)
        if (e) cudaEventDestroy(e);
    if (c->host_mailbox) cudaFreeHost(c->host_mailbox);
    for (auto e : c->stage_ev)
        if (e) cudaEventDestroy(e);
    if (c->stage) cudaFreeHost(c->stage);
    if (c->copy_stream) cudaStreamSynchronize(c->copy_stream);
    if (c->copy_ev) cudaEventDestroy(c->copy_ev);
    if (c->copy_stream) cudaStreamDestroy(c->copy_stream);
    if (c->dl_stream) cudaStreamSynchronize(c->dl_stream);
    if (c->dl_ev) cudaEventDestroy(c->dl_ev);
    if (c->dl_done_ev) cudaEventDestroy(c->dl_done_ev);
    if (c->dl_stream) cudaStreamDestroy(c->dl_stream);
    if (c->stream) cudaStreamDestroy(c->stream);
    delete c;
}

extern "C" const char* volta_cuda_last_error(void* raw) {
    Context* c = static_cast<Context*>(raw);
    return c ? c->error.c_str() : "null CUDA context";
}

extern "C" int volta_cuda_set_resident_timing_policy(void* raw, int policy) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->active_record != kRingSize || c->coarse || c->counter_active || c->ring_pending ||
        c->counter_pending)
        return reject(c, "cannot change resident timing policy after work has started");
    if (policy == 0) {
        if (c->mode == kTimingEvents) c->mode = kTimingDeferred;
    } else if (policy == 1) {
        c->mode = kTimingCounters;
    } else {
        return reject(c, "unknown resident timing policy");
    }
    c->stats.timing_elapsed_query_attempts = 0;
    c->stats.timing_elapsed_no_write = 0;
    c->stats.timing_event_queries = 0;
    c->stats.timing_event_api_calls = 0;
    c->stats.timing_mode = c->mode;
    return 0;
}

extern "C" int volta_cuda_test_inject_elapsed_no_write_once(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->active_record != kRingSize)
        return reject(c, "cannot inject elapsed no-write during an active record");
    c->inject_no_write = 1;
    return 0;
}

extern "C" int volta_cuda_begin_coarse_timing(void* raw, int operation) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->mode != kTimingDeferred && c->mode != kTimingCounters)
        return reject(c, "coarse timing requires a resident observation mode");
    if (c->poisoned) return reject(c, "measurement timing is poisoned; reset stats before continuing");
    if (operation < 0 || operation >= kOpCount) return reject(c, "invalid coarse timing operation");
    if (c->coarse || c->active_record != kRingSize || c->counter_active)
        return reject(c, "nested coarse timing scope");
    if (c->mode == kTimingDeferred && ring_open(c, RecordKind::Coarse, 2)) return -1;
    c->coarse_op = operation;
    c->coarse = true;
    c->coarse_inner = false;
    c->coarse_work = false;
    if (c->mode == kTimingDeferred) c->ring[c->active_record].op = operation;
    return 0;
}

extern "C" int volta_cuda_end_coarse_timing(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->mode != kTimingDeferred && c->mode != kTimingCounters)
        return reject(c, "coarse timing requires a resident observation mode");
    if (!c->coarse || (c->mode == kTimingDeferred && c->active_record == kRingSize))
        return reject(c, "no active coarse timing scope");
    if (c->coarse_inner) return reject(c, "cannot end coarse timing during an active primitive");
    if (c->mode == kTimingDeferred) {
        Record& r = c->ring[c->active_record];
        VZB_CUDA(c, ev_record(c, r.ev[1]));
        r.mask |= 1u << 1;
        r.kind = RecordKind::Coarse;
        r.op = c->coarse_op;
    }
    c->coarse = false;
    c->coarse_op = -1;
    if (c->mode == kTimingDeferred && ring_commit(c)) return -1;
    c->coarse_work = false;
    ++c->stats.coarse_timing_scopes;
    return 0;
}

extern "C" int volta_cuda_abort_coarse_timing(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->mode != kTimingDeferred && c->mode != kTimingCounters)
        return reject(c, "coarse timing requires a resident observation mode");
    if (c->coarse) drop_active_record(c);
    return 0;
}

extern "C" int volta_cuda_ensure_timing_capacity(void* raw, size_t bound, size_t* before,
                                                 size_t* after, int* flushed) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !before || !after || !flushed) return reject(c, "invalid timing-capacity output");
    if (c->mode != kTimingDeferred && c->mode != kTimingCounters)
        return reject(c, "timing-capacity preflight requires a resident observation mode");
    if (c->active_record != kRingSize || c->counter_active)
        return reject(c, "cannot preflight timing capacity during an active record");
    if (bound > kRingSize) return reject(c, "deferred timing cohort bound exceeds ring capacity");
    *before = c->mode == kTimingDeferred ? c->ring_pending : 0;
    *flushed = 0;
    if (c->mode == kTimingCounters) {
        *after = 0;
        return 0;
    }
    if (c->ring_pending > kRingSize - bound) {
        if (flush_ring(c, Sync::TimingFlush)) return -1;
        *flushed = 1;
    }
    *after = c->ring_pending;
    return 0;
}

extern "C" int volta_cuda_flush_profiling(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->poisoned) return reject(c, "measurement timing is poisoned; reset stats before reading it");
    if (c->active_record != kRingSize || c->counter_active)
        return reject(c, "cannot flush an active timing record");
    if (c->mode == kTimingCounters && c->counter_pending) return sync_stream(c, Sync::TimingFlush);
    return flush_ring(c, Sync::TimingFlush);
}

extern "C" int volta_cuda_reset_stats(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (c->active_record != kRingSize || c->counter_active)
        return reject(c, "cannot reset stats during an active timing record");
    const bool pending = (c->mode == kTimingDeferred && c->ring_pending) ||
                         (c->mode == kTimingCounters && c->counter_pending);
    if (discard_ring(c, Sync::TimingFlush)) return -1;
    if (c->mode == kTimingCounters && c->counter_pending && sync_stream(c, Sync::TimingFlush))
        return -1;
    if (c->poisoned && !pending && sync_stream(c, Sync::TimingFlush)) return -1;
    const uint64_t live = c->stats.live_device_bytes, pinned = c->stats.live_pinned_bytes;
    c->stats = RawStats{};
    c->stats.live_device_bytes = live;
    c->stats.peak_device_bytes = live;
    c->stats.live_pinned_bytes = pinned;
    c->stats.peak_pinned_bytes = pinned;
    c->stats.timing_mode = c->mode;
    c->poisoned = false;
    c->coarse_work = false;
    c->counter_active = false;
    c->counter_pending = false;
    return 0;
}

extern "C" int volta_cuda_get_stats(void* raw, RawStats* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !out) return -1;
    if (c->poisoned) return reject(c, "measurement timing is poisoned; reset stats before reading it");
    if (c->active_record != kRingSize || c->counter_active)
        return reject(c, "cannot read stats during an active timing record");
    if (volta_cuda_flush_profiling(raw)) return -1;
    const RawStats& s = c->stats;
    if (s.sync_host_output + s.sync_upload_lifetime + s.sync_timing_flush + s.sync_profiling_legacy +
            s.sync_allocator_flush != s.synchronizations)
        return fail_message(c, "synchronization reason accounting mismatch");
    if (s.timing_elapsed_query_attempts != s.timing_event_queries + s.timing_elapsed_no_write)
        return fail_message(c, "elapsed timing query accounting mismatch");
    if (c->mode == kTimingCounters) {
        uint64_t k = 0;
        for (uint64_t v : s.kernel_ns) k += v;
        if (s.timing_records || s.timing_elapsed_query_attempts || s.timing_elapsed_no_write ||
            s.timing_event_queries || s.timing_event_api_calls || s.timing_pending_high_water ||
            s.timing_flush_count || s.h2d_ns || s.d2h_ns || s.coarse_timing_ns || k)
            return fail_message(c, "wall-only counter mode emitted CUDA-event attribution");
    }
    *out = s;
    return 0;
}

extern "C" int volta_cuda_memory_breakdown(void* raw, uint64_t* workspace, uint64_t* resident,
                                           uint64_t* cached) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !workspace || !resident || !cached) return fail_message(c, "invalid memory-breakdown output");
    uint64_t w = 0, r = 0, k = 0;
    for (const auto& x : c->ws) w += x.capacity;
    for (const auto& s : c->slots) {
        if (!s.ptr) continue;
        (s.active ? r : k) += s.capacity;
    }
    if (w + r + k != c->stats.live_device_bytes) return fail_message(c, "device-memory accounting mismatch");
    *workspace = w;
    *resident = r;
    *cached = k;
    return 0;
}

extern "C" int volta_cuda_trim_resident_cache(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return fail_message(c, "invalid resident-cache trim context");
    if (c->coarse) return reject(c, "resident-cache trim is forbidden inside a coarse timing scope");
    return trim_resident(c);
}

extern "C" int volta_cuda_pinned_memory_stats(void* raw, RawPinnedMemoryStats* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !out) return fail_message(c, "invalid pinned-memory stats output");
    RawPinnedMemoryStats r{};
    for (auto& p : c->pinned) {
        if (!p.ptr) continue;
        bool ready = false;
        if (pinned_ready(c, &p, &ready)) return -1;
        if (p.active) {
            r.active_bytes += p.capacity;
            ++r.active_allocations;
        } else {
            r.cached_bytes += p.capacity;
            ++r.cached_allocations;
        }
        if (!ready) ++r.in_flight_allocations;
    }
    if (r.active_bytes + r.cached_bytes != c->stats.live_pinned_bytes)
        return fail_message(c, "pinned-memory accounting mismatch");
    r.physical_allocation_calls = c->stats.pinned_allocation_calls;
    r.allocation_requests = c->stats.pinned_alloc_requests;
    r.reuse_hits = c->stats.pinned_reuse_hits;
    r.free_requests = c->stats.pinned_free_requests;
    r.physical_free_calls = c->stats.pinned_physical_free_calls;
    r.host_write_calls = c->stats.pinned_host_write_calls;
    r.host_write_bytes = c->stats.pinned_host_write_bytes;
    r.peak_bytes = c->stats.peak_pinned_bytes;
    *out = r;
    return 0;
}

extern "C" int volta_cuda_x4c_control_state(void* raw, RawX4cControlState* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !out) return fail_message(c, "invalid X4c control-state output");
    ++c->stats.x4c_control_peek_calls;
    const cudaError_t st = cudaStreamQuery(c->stream);
    uint32_t state = 0;
    if (st == cudaSuccess) {
        c->outstanding = 0;
        c->counter_pending = false;
        for (auto& p : c->pinned) p.in_flight = false;
    } else if (st == cudaErrorNotReady) {
        state = 1;
        ++c->stats.x4c_control_peek_pending;
    } else {
        return fail_cuda(c, "cudaStreamQuery(X4c control state)", st);
    }
    RawX4cControlState r{};
    r.stream_state = state;
    r.flags = (c->coarse ? 1u : 0u) | ((c->active_record != kRingSize || c->counter_active) ? 2u : 0u) |
              (c->poisoned ? 4u : 0u);
    r.outstanding_cuda_operations = c->outstanding;
    r.pending_timing_records = c->ring_pending;
    for (const auto& w : c->ws) r.workspace_device_bytes += w.capacity;
    for (const auto& s : c->slots) {
        if (!s.ptr) continue;
        if (s.active) {
            ++r.active_device_allocations;
            r.active_device_bytes += s.capacity;
        } else {
            ++r.cached_device_allocations;
            r.cached_device_bytes += s.capacity;
        }
    }
    for (const auto& p : c->pinned) {
        if (!p.ptr) continue;
        if (p.active) {
            ++r.active_pinned_allocations;
            r.active_pinned_bytes += p.capacity;
        } else {
            ++r.cached_pinned_allocations;
            r.cached_pinned_bytes += p.capacity;
        }
        if (p.in_flight) ++r.in_flight_pinned_allocations;
    }
    if (r.workspace_device_bytes + r.active_device_bytes + r.cached_device_bytes !=
        c->stats.live_device_bytes)
        return fail_message(c, "X4c control-state device ownership mismatch");
    if (r.active_pinned_bytes + r.cached_pinned_bytes != c->stats.live_pinned_bytes)
        return fail_message(c, "X4c control-state pinned ownership mismatch");
    *out = r;
    return 0;
}

// ===========================================================================
// C ABI: pinned pool
// ===========================================================================

extern "C" int volta_cuda_pinned_alloc(void* raw, size_t bytes, uint64_t* out_id) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !bytes || !out_id) return fail_message(c, "invalid pinned allocation");
    if (c->coarse) return reject(c, "pinned allocation is forbidden inside a coarse timing scope");
    try {
        ++c->stats.pinned_alloc_requests;
        // best fit among cached, ready allocations (ties to the lowest slot)
        size_t best_pos = SIZE_MAX, best_slot = SIZE_MAX, best_cap = SIZE_MAX;
        for (size_t pos = 0; pos < c->free_pinned.size(); ++pos) {
            const size_t s = c->free_pinned[pos];
            PinnedSlot& p = c->pinned[s];
            bool ready = false;
            if (p.ptr && pinned_ready(c, &p, &ready)) return -1;
            if (p.active || !p.ptr || !ready || p.generation == kGenerationMax || p.capacity < bytes)
                continue;
            if (p.capacity < best_cap || (p.capacity == best_cap && s < best_slot)) {
                best_pos = pos;
                best_cap = p.capacity;
                best_slot = s;
            }
        }
        if (best_pos != SIZE_MAX) {
            c->free_pinned[best_pos] = c->free_pinned.back();
            c->free_pinned.pop_back();
            PinnedSlot& p = c->pinned[best_slot];
            ++p.generation;
            p.logical = bytes;
            p.active = true;
            ++c->stats.pinned_reuse_hits;
            *out_id = make_id(best_slot, p.generation);
            return 0;
        }
        void* ptr = nullptr;
        cudaError_t st = cudaMallocHost(&ptr, bytes);
        if (st != cudaSuccess) return fail_cuda(c, "cudaMallocHost(&pinned, bytes)", st);
        cudaEvent_t ready = nullptr;
        st = cudaEventCreateWithFlags(&ready, cudaEventDisableTiming);
        if (st != cudaSuccess) {
            (void)cudaFreeHost(ptr);
            return fail_cuda(c, "cudaEventCreateWithFlags(pinned ready)", st);
        }
        ++c->stats.pinned_allocation_calls;
        c->stats.live_pinned_bytes += bytes;
        c->stats.peak_pinned_bytes = std::max(c->stats.peak_pinned_bytes, c->stats.live_pinned_bytes);
        size_t slot = SIZE_MAX;
        for (size_t pos = 0; pos < c->free_pinned.size(); ++pos) {
            const size_t s = c->free_pinned[pos];
            const PinnedSlot& p = c->pinned[s];
            if (!p.active && !p.ptr && p.generation != kGenerationMax) {
                slot = s;
                c->free_pinned[pos] = c->free_pinned.back();
                c->free_pinned.pop_back();
                break;
            }
        }
        if (slot == SIZE_MAX) {
            if (c->pinned.size() >= kSlotMask) return fail_message(c, "pinned slot id space exhausted");
            c->pinned.emplace_back();
            slot = c->pinned.size() - 1;
        }
        PinnedSlot& p = c->pinned[slot];
        ++p.generation;
        p.ptr = ptr;
        p.capacity = bytes;
        p.logical = bytes;
        p.ready = ready;
        p.active = true;
        p.in_flight = false;
        *out_id = make_id(slot, p.generation);
        return 0;
    } catch (...) {
        return fail_message(c, "pinned allocation threw a C++ exception");
    }
}

extern "C" int volta_cuda_pinned_write(void* raw, uint64_t id, size_t offset, const void* src,
                                       size_t bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !src || !bytes) return fail_message(c, "invalid pinned write");
    PinnedSlot* p = find_pinned(c, id);
    if (!p) return fail_message(c, "unknown pinned buffer id");
    if (offset > p->logical || bytes > p->logical - offset)
        return fail_message(c, "pinned buffer region is out of bounds");
    bool ready = false;
    if (pinned_ready(c, p, &ready)) return -1;
    if (!ready) return reject(c, "pinned buffer is still consumed by an outstanding H2D");
    std::memcpy(static_cast<unsigned char*>(p->ptr) + offset, src, bytes);
    ++c->stats.pinned_host_write_calls;
    c->stats.pinned_host_write_bytes += bytes;
    return 0;
}

extern "C" int volta_cuda_pinned_wait_ready(void* raw, uint64_t id) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !id) return fail_message(c, "invalid pinned wait");
    if (c->coarse || c->coarse_inner || c->counter_active || c->active_record != kRingSize)
        return reject(c, "pinned wait inside an active timing scope");
    PinnedSlot* p = find_pinned(c, id);
    if (!p) return fail_message(c, "unknown pinned buffer id");
    bool ready = false;
    if (pinned_ready(c, p, &ready)) return -1;
    if (ready) return 0;
    const auto t0 = std::chrono::steady_clock::now();
    const cudaError_t st = cudaEventSynchronize(p->ready);
    const auto t1 = std::chrono::steady_clock::now();
    if (st != cudaSuccess) return fail_cuda(c, "cudaEventSynchronize(pinned ready)", st);
    p->in_flight = false;
    ++c->stats.synchronizations;
    ++c->stats.sync_upload_lifetime;
    c->stats.synchronization_ns += std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
    return 0;
}

extern "C" int volta_cuda_pinned_free(void* raw, uint64_t id) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !id) return fail_message(c, "invalid pinned free");
    if (c->coarse) return reject(c, "pinned free is forbidden inside a coarse timing scope");
    PinnedSlot* p = find_pinned(c, id);
    if (!p) return fail_message(c, "unknown or stale pinned buffer id");
    ++c->stats.pinned_free_requests;
    c->free_pinned.push_back(static_cast<size_t>((id & kSlotMask) - 1));
    p->logical = 0;
    p->active = false;
    return 0;
}

extern "C" int volta_cuda_trim_pinned_cache(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return fail_message(c, "invalid pinned-cache trim context");
    if (c->coarse) return reject(c, "pinned-cache trim is forbidden inside a coarse timing scope");
    return trim_pinned(c);
}

// ===========================================================================
// C ABI: resident arena
// ===========================================================================

extern "C" int volta_cuda_resident_alloc(void* raw, size_t bytes, uint64_t* out_id) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !bytes || !out_id) return fail_message(c, "invalid resident allocation");
    if (c->coarse) return reject(c, "resident allocation is forbidden inside a coarse timing scope");
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    try {
        ++c->stats.resident_alloc_requests;
        // best fit: the smallest free capacity >= bytes, the lowest slot among equals
        const auto fit = c->free_fit.lower_bound({bytes, 0});
        if (fit != c->free_fit.end()) {
            const size_t best_slot = fit->second;
            c->free_fit.erase(fit);
            Slot& b = c->slots[best_slot];
            ++b.generation;
            b.logical = bytes;
            b.active = true;
            ++c->stats.resident_reuse_hits;
            *out_id = make_id(best_slot, b.generation);
            return 0;
        }
        void* ptr = nullptr;
        cudaError_t e = cudaMalloc(&ptr, bytes);
        if (e == cudaErrorMemoryAllocation) {
            (void)cudaGetLastError();
            if (trim_resident(c)) return -1;
            e = cudaMalloc(&ptr, bytes);
        }
        if (e != cudaSuccess) return fail_cuda(c, "cudaMalloc(&resident, bytes)", e);
        ++c->stats.allocation_calls;
        c->stats.live_device_bytes += bytes;
        c->stats.peak_device_bytes = std::max(c->stats.peak_device_bytes, c->stats.live_device_bytes);
        size_t slot = SIZE_MAX;
        if (!c->free_empty.empty()) {  // a trimmed slot's id
            slot = c->free_empty.back();
            c->free_empty.pop_back();
        }
        if (slot == SIZE_MAX) {
            if (c->slots.size() >= kSlotMask) {
                cudaFree(ptr);
                return fail_message(c, "resident slot id space exhausted");
            }
            c->slots.emplace_back();
            slot = c->slots.size() - 1;
        }
        Slot& b = c->slots[slot];
        ++b.generation;
        b.ptr = ptr;
        b.capacity = bytes;
        b.logical = bytes;
        b.active = true;
        *out_id = make_id(slot, b.generation);
        return 0;
    } catch (...) {
        return fail_message(c, "resident allocation threw a C++ exception");
    }
}

extern "C" int volta_cuda_resident_free(void* raw, uint64_t id) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !id) return fail_message(c, "invalid resident free");
    if (c->coarse) return reject(c, "resident free is forbidden inside a coarse timing scope");
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    ++c->stats.resident_free_requests;
    Slot* b = find_slot(c, id);
    if (!b) return fail_message(c, "unknown or stale resident buffer id");
    if (c->dl_pending) {  // a later owner of this memory writes only after the pending downloads read it
        VZB_CUDA(c, cudaEventRecord(c->dl_done_ev, c->dl_stream));
        VZB_CUDA(c, cudaStreamWaitEvent(c->stream, c->dl_done_ev, 0));
    }
    try {
        const size_t s = static_cast<size_t>((id & kSlotMask) - 1);
        if (b->generation == kGenerationMax)
            c->free_retired.push_back(s);
        else
            c->free_fit.insert({b->capacity, s});
    } catch (...) {
        return fail_message(c, "resident free threw a C++ exception");
    }
    b->logical = 0;
    b->active = false;
    return 0;
}

// Small upload from the mapped staging ring (at most 64 KiB; 4 KiB per block).
__global__ void stage_copy_kernel(unsigned char* __restrict__ dst, const unsigned char* __restrict__ src,
                                  size_t bytes) {
    const size_t lo = static_cast<size_t>(blockIdx.x) * 4096, hi = lo + 4096 < bytes ? lo + 4096 : bytes;
    if (((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src) | lo | hi) & 15) == 0) {
        for (size_t i = lo + 16 * threadIdx.x; i < hi; i += 16 * blockDim.x)
            *reinterpret_cast<uint4*>(dst + i) = *reinterpret_cast<const uint4*>(src + i);
    } else {
        for (size_t i = lo + threadIdx.x; i < hi; i += blockDim.x) dst[i] = src[i];
    }
}

extern "C" int volta_cuda_resident_upload(void* raw, uint64_t id, size_t offset, const void* src,
                                          size_t bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !src || !bytes) return fail_message(c, "invalid resident upload");
    void* dst = nullptr;
    if (region(c, id, offset, bytes, &dst)) return -1;
    if (xfer_begin(c)) return -1;
    const auto t0 = std::chrono::steady_clock::now();
    cudaError_t e;
    if (bytes <= kStageSlotBytes && c->stage) {
        // small upload through a pinned staging slot (reused once its copy is done)
        const int slot = c->stage_next;
        c->stage_next = (slot + 1) % kStageSlots;
        if (c->stage_used[slot]) VZB_CUDA(c, cudaEventSynchronize(c->stage_ev[slot]));
        const size_t at = static_cast<size_t>(slot) * kStageSlotBytes;
        std::memcpy(static_cast<char*>(c->stage) + at, src, bytes);
        stage_copy_kernel<<<static_cast<unsigned>((bytes + 4095) / 4096), 256, 0, c->stream>>>(
            static_cast<unsigned char*>(dst), static_cast<const unsigned char*>(c->stage_dev) + at, bytes);
        e = cudaGetLastError();
        ++c->launches;
        if (e == cudaSuccess) e = cudaEventRecord(c->stage_ev[slot], c->stream);
        c->stage_used[slot] = true;
    } else {
        e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->stream);
    }
    const auto t1 = std::chrono::steady_clock::now();
    if (e != cudaSuccess) return fail_cuda(c, "cudaMemcpyAsync(resident H2D)", e);
    ++c->stats.resident_h2d_host_calls;
    c->stats.resident_h2d_host_call_ns +=
        std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
    return xfer_finish(c, bytes, true);
}

// Many small uploads at once (extension): the host buffers are packed into
// staging slots (16-byte aligned pieces) and each slot's pieces are copied to
// their destinations by one launch, one CTA per piece.
struct StagePiece {
    unsigned char* dst;
    size_t src_at;  // offset in the mapped staging ring
    size_t bytes;
};
constexpr int kPiecesPerLaunch = 96;
struct StagePieces {
    StagePiece p[kPiecesPerLaunch];
};

__global__ void stage_pieces_kernel(const __grid_constant__ StagePieces pieces, const unsigned char* __restrict__ stage) {
    const StagePiece& g = pieces.p[blockIdx.x];
    const unsigned char* src = stage + g.src_at;
    if (((reinterpret_cast<uintptr_t>(g.dst) | g.bytes) & 15) == 0) {
        for (size_t i = 16 * threadIdx.x; i < g.bytes; i += 16 * blockDim.x)
            *reinterpret_cast<uint4*>(g.dst + i) = *reinterpret_cast<const uint4*>(src + i);
    } else {
        for (size_t i = threadIdx.x; i < g.bytes; i += blockDim.x) g.dst[i] = src[i];
    }
}

extern "C" int volta_b200_upload_batch(void* raw, const vzb_upload* items, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || (count && !items)) return fail_message(c, "invalid upload batch");
    if (!c->stage) return fail_message(c, "upload batch needs the staging ring");
    std::vector<void*> dsts(count);
    for (size_t i = 0; i < count; ++i) {  // every destination checked before anything is staged
        if (!items[i].src || !items[i].bytes || items[i].bytes > kStageSlotBytes)
            return fail_message(c, "invalid upload batch item (1 byte .. 64 KiB each)");
        if (region(c, items[i].dst_id, items[i].dst_offset, items[i].bytes, &dsts[i])) return -1;
    }
    if (xfer_begin(c)) return -1;
    size_t total = 0, i = 0;
    while (i < count) {  // fill one slot, launch its copies
        const int slot = c->stage_next;
        c->stage_next = (slot + 1) % kStageSlots;
        if (c->stage_used[slot]) VZB_CUDA(c, cudaEventSynchronize(c->stage_ev[slot]));
        const size_t base = static_cast<size_t>(slot) * kStageSlotBytes;
        StagePieces batch{};
        int n = 0;
        size_t used = 0;
        while (i < count && n < kPiecesPerLaunch && used + items[i].bytes <= kStageSlotBytes) {
            std::memcpy(static_cast<char*>(c->stage) + base + used, items[i].src, items[i].bytes);
            batch.p[n++] = StagePiece{static_cast<unsigned char*>(dsts[i]), base + used, items[i].bytes};
            used += (items[i].bytes + 15) & ~size_t{15};
            total += items[i].bytes;
            ++i;
        }
        stage_pieces_kernel<<<static_cast<unsigned>(n), 128, 0, c->stream>>>(
            batch, static_cast<const unsigned char*>(c->stage_dev));
        cudaError_t e = cudaGetLastError();
        ++c->launches;
        if (e == cudaSuccess) e = cudaEventRecord(c->stage_ev[slot], c->stream);
        if (e != cudaSuccess) return fail_cuda(c, "upload batch", e);
        c->stage_used[slot] = true;
    }
    ++c->stats.resident_h2d_host_calls;
    return xfer_finish(c, total, true);
}

extern "C" int volta_cuda_resident_download(void* raw, uint64_t id, size_t offset, void* dst,
                                            size_t bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !dst || !bytes) return fail_message(c, "invalid resident download");
    void* src = nullptr;
    if (region(c, id, offset, bytes, &src)) return -1;
    if (xfer_begin(c)) return -1;
    const auto t0 = std::chrono::steady_clock::now();
    const cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->stream);
    const auto t1 = std::chrono::steady_clock::now();
    if (e != cudaSuccess) return fail_cuda(c, "cudaMemcpyAsync(resident D2H)", e);
    ++c->stats.resident_d2h_host_calls;
    c->stats.resident_d2h_host_call_ns +=
        std::chrono::duration_cast<std::chrono::nanoseconds>(t1 - t0).count();
    return xfer_finish(c, bytes, false);
}

extern "C" int volta_cuda_resident_zero(void* raw, uint64_t id, size_t offset, size_t bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !bytes) return fail_message(c, "invalid resident zero");
    void* dst = nullptr;
    if (region(c, id, offset, bytes, &dst)) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    VZB_CUDA(c, cudaMemsetAsync(dst, 0, bytes, c->stream));
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0, 0, bytes, 0);
}

// Strided device-to-device rows as a kernel on the compute stream, in the
// widest unit that every address, stride and row length allows (a copy
// engine transfer queued behind this stream's kernels could hold up other
// streams' uploads on the same engine).
template <typename T>
__global__ void copy_rows_kernel(unsigned char* __restrict__ dst, size_t dst_stride,
                                 const unsigned char* __restrict__ src, size_t src_stride, size_t rows,
                                 size_t row_units) {
    const size_t total = rows * row_units, step = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += step) {
        size_t r, u;
        if (total <= 0xFFFFFFFFull) {
            r = static_cast<uint32_t>(i) / static_cast<uint32_t>(row_units);
            u = static_cast<uint32_t>(i) - static_cast<uint32_t>(r) * static_cast<uint32_t>(row_units);
        } else {
            r = i / row_units;
            u = i - r * row_units;
        }
        *reinterpret_cast<T*>(dst + r * dst_stride + u * sizeof(T)) =
            *reinterpret_cast<const T*>(src + r * src_stride + u * sizeof(T));
    }
}

static int copy_rows(Context* c, uint64_t src_id, size_t src_off, size_t src_stride,
                     uint64_t dst_id, size_t dst_off, size_t dst_stride, size_t rows,
                     size_t row_bytes, int op) {
    if (!c) return fail_message(c, "invalid resident D2D copy context");
    void *src = nullptr, *dst = nullptr;
    size_t src_span = 0, dst_span = 0;
    if (strided_region(c, src_id, src_off, src_stride, row_bytes, rows, &src, &src_span) ||
        strided_region(c, dst_id, dst_off, dst_stride, row_bytes, rows, &dst, &dst_span))
        return -1;
    if (src_id == dst_id) {
        size_t se = 0, de = 0;
        if (!add_ok(src_off, src_span, &se) || !add_ok(dst_off, dst_span, &de))
            return fail_message(c, "resident D2D copy envelope overflows size_t");
        if (src_off < de && dst_off < se)
            return fail_message(c, "resident D2D copy source and destination overlap");
    }
    size_t total = 0;
    if (!mul_ok(rows, row_bytes, &total)) return fail_message(c, "resident D2D byte count overflows size_t");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const uintptr_t align = reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst) | src_stride |
                            dst_stride | row_bytes;
    const int unit = (align & 15) == 0 ? 16 : (align & 7) == 0 ? 8 : (align & 3) == 0 ? 4 : 1;
    const size_t units = total / unit;
    const unsigned grid = static_cast<unsigned>(
        std::min<size_t>((units + 255) / 256, static_cast<size_t>(c->sm_count) * 8));
    unsigned char* d = static_cast<unsigned char*>(dst);
    const unsigned char* sp = static_cast<const unsigned char*>(src);
    switch (unit) {
        case 16: copy_rows_kernel<uint4><<<grid, 256, 0, c->stream>>>(d, dst_stride, sp, src_stride, rows, row_bytes / 16); break;
        case 8: copy_rows_kernel<uint2><<<grid, 256, 0, c->stream>>>(d, dst_stride, sp, src_stride, rows, row_bytes / 8); break;
        case 4: copy_rows_kernel<uint32_t><<<grid, 256, 0, c->stream>>>(d, dst_stride, sp, src_stride, rows, row_bytes / 4); break;
        default: copy_rows_kernel<unsigned char><<<grid, 256, 0, c->stream>>>(d, dst_stride, sp, src_stride, rows, row_bytes); break;
    }
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, op, 0, 0, total, 0, 0);
}

extern "C" int volta_cuda_resident_copy_rows(void* raw, uint64_t src_id, size_t src_off,
                                             size_t src_stride, uint64_t dst_id, size_t dst_off,
                                             size_t dst_stride, size_t rows, size_t row_bytes) {
    return copy_rows(static_cast<Context*>(raw), src_id, src_off, src_stride, dst_id, dst_off,
                     dst_stride, rows, row_bytes, kOpPcsRows);
}

extern "C" int volta_cuda_resident_mailbox_copy_rows(void* raw, uint64_t src_id, size_t src_off,
                                                     size_t src_stride, uint64_t dst_id,
                                                     size_t dst_off, size_t dst_stride,
                                                     size_t rows, size_t row_bytes) {
    return copy_rows(static_cast<Context*>(raw), src_id, src_off, src_stride, dst_id, dst_off,
                     dst_stride, rows, row_bytes, kOpMailbox);
}

// Many small device-to-device copies in one launch (extension): one CTA per
// segment, 16-byte units when both ends and the length allow it.
struct CopySeg {
    const unsigned char* src;
    unsigned char* dst;
    size_t bytes;
};
constexpr int kSegsPerLaunch = 96;
struct CopySegs {
    CopySeg s[kSegsPerLaunch];
};

__global__ void copy_segments_kernel(const __grid_constant__ CopySegs segs) {
    const CopySeg& g = segs.s[blockIdx.x];
    const bool wide = ((reinterpret_cast<uintptr_t>(g.src) | reinterpret_cast<uintptr_t>(g.dst) | g.bytes) & 15) == 0;
    if (wide) {
        for (size_t i = threadIdx.x; i < g.bytes / 16; i += blockDim.x)
            reinterpret_cast<uint4*>(g.dst)[i] = reinterpret_cast<const uint4*>(g.src)[i];
    } else {
        for (size_t i = threadIdx.x; i < g.bytes; i += blockDim.x) g.dst[i] = g.src[i];
    }
}

extern "C" int volta_b200_copy_segments_device(void* raw, const vzb_copy_seg* segs, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || (count && !segs)) return fail_message(c, "invalid copy segments");
    std::vector<CopySeg> resolved(count);  // every segment checked before anything is launched
    size_t total = 0;
    for (size_t i = 0; i < count; ++i) {
        void *src = nullptr, *dst = nullptr;
        if (region_elems(c, segs[i].src_id, segs[i].src_offset, segs[i].bytes, 1, &src) ||
            region_elems(c, segs[i].dst_id, segs[i].dst_offset, segs[i].bytes, 1, &dst))
            return -1;
        resolved[i] = CopySeg{static_cast<const unsigned char*>(src), static_cast<unsigned char*>(dst), segs[i].bytes};
        total += segs[i].bytes;
    }
    if (op_begin(c) || op_mark(c, 1)) return -1;
    for (size_t base = 0; base < count; base += kSegsPerLaunch) {
        const size_t n = std::min(count - base, static_cast<size_t>(kSegsPerLaunch));
        CopySegs batch{};
        for (size_t i = 0; i < n; ++i) batch.s[i] = resolved[base + i];
        copy_segments_kernel<<<static_cast<unsigned>(n), 256, 0, c->stream>>>(batch);
        VZB_LAUNCHED(c);
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0, total, 0, 0);
}

// ===========================================================================
// Extensions (include/volta_b200_ext.h): measurement markers, launch count
// ===========================================================================

extern "C" int volta_b200_timing_mark(void* raw, int slot) {
    Context* c = static_cast<Context*>(raw);
    if (!c || slot < 0 || slot >= kTimingMarkers) return fail_message(c, "invalid timing marker slot");
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    if (!c->bench_ev[slot]) VZB_CUDA(c, cudaEventCreate(&c->bench_ev[slot]));
    VZB_CUDA(c, cudaEventRecord(c->bench_ev[slot], c->stream));
    return 0;
}

extern "C" int volta_b200_timing_elapsed(void* raw, int start, int end, float* ms) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !ms || start < 0 || start >= kTimingMarkers || end < 0 || end >= kTimingMarkers || !c->bench_ev[start] ||
        !c->bench_ev[end])
        return fail_message(c, "invalid timing marker pair");
    VZB_CUDA(c, cudaEventSynchronize(c->bench_ev[end]));
    VZB_CUDA(c, cudaEventElapsedTime(ms, c->bench_ev[start], c->bench_ev[end]));
    return 0;
}

extern "C" int volta_b200_launch_count(void* raw, uint64_t* launches) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !launches) return fail_message(c, "invalid launch-count output");
    *launches = c->launches;
    return 0;
}

// ---------------------------------------------------------------------------
// Extensions: asynchronous uploads (include/volta_b200_ext.h)
// ---------------------------------------------------------------------------

extern "C" int volta_b200_upload_async(void* raw, uint64_t id, size_t offset, const void* src, size_t bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !src || !bytes) return fail_message(c, "invalid asynchronous upload");
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    void* dst = nullptr;
    if (region(c, id, offset, bytes, &dst)) return -1;
    if (!c->copy_stream) {
        VZB_CUDA(c, cudaStreamCreateWithFlags(&c->copy_stream, cudaStreamNonBlocking));
        VZB_CUDA(c, cudaEventCreateWithFlags(&c->copy_ev, cudaEventDisableTiming));
    }
    VZB_CUDA(c, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, c->copy_stream));
    VZB_CUDA(c, cudaEventRecord(c->copy_ev, c->copy_stream));
    return 0;
}

extern "C" int volta_b200_download_async(void* raw, uint64_t id, size_t offset, void* dst, size_t bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !dst || !bytes) return fail_message(c, "invalid asynchronous download");
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    void* src = nullptr;
    if (region(c, id, offset, bytes, &src)) return -1;
    if (!c->dl_stream) {
        VZB_CUDA(c, cudaStreamCreateWithFlags(&c->dl_stream, cudaStreamNonBlocking));
        VZB_CUDA(c, cudaEventCreateWithFlags(&c->dl_ev, cudaEventDisableTiming));
        VZB_CUDA(c, cudaEventCreateWithFlags(&c->dl_done_ev, cudaEventDisableTiming));
    }
    // the copy sees everything enqueued on the compute stream so far
    VZB_CUDA(c, cudaEventRecord(c->dl_ev, c->stream));
    VZB_CUDA(c, cudaStreamWaitEvent(c->dl_stream, c->dl_ev, 0));
    VZB_CUDA(c, cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, c->dl_stream));
    c->dl_pending = true;
    return 0;
}

extern "C" int volta_b200_wait_downloads(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    if (c->dl_stream) VZB_CUDA(c, cudaStreamSynchronize(c->dl_stream));
    c->dl_pending = false;
    return 0;
}

extern "C" int volta_b200_wait_uploads(void* raw) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    if (bind_device(c)) return fail_message(c, "cannot select the context's device");
    if (c->copy_ev) VZB_CUDA(c, cudaStreamWaitEvent(c->stream, c->copy_ev, 0));
    return 0;
}
