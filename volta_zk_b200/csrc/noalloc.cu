// Triple-product round message with a statically allocated reduction
// scratch (include/volta_b200_ext.h: volta_b200_triple_product_round_noalloc).
//
// For callers that cannot allocate device memory: a host framework whose
// caching allocator owns the GPU's memory, or a latency-critical round loop
// that must not risk the synchronisation cudaMalloc/cudaFree can cause.
// The scratch lives in this file as fixed-size __device__ arrays; nothing
// here calls cudaMalloc, cudaFree or an allocating library routine.
#include <mutex>

#include "../../include/volta_b200_ext.h"
#include "reduce.cuh"

namespace {

using vzb::Acc;
using vzb::Fp2;

constexpr unsigned kThreads = 256;
constexpr size_t kPairsPerBlock = 1024;      // 4 pairs per thread
constexpr size_t kScratchFp2 = 65536;        // 1 MiB of per-block partials
constexpr size_t kMaxBlocks = kScratchFp2 / 3;
constexpr size_t kMaxPairs = kMaxBlocks * kPairsPerBlock;
static_assert(kMaxPairs == VOLTA_B200_NOALLOC_MAX_PAIRS, "header limit");
static_assert(kScratchFp2 * sizeof(Fp2) + 256 == VOLTA_B200_NOALLOC_SCRATCH_BYTES, "header size");

// Shared by every call on a device; contents persist between calls.
static __device__ __align__(256) Fp2 g_noalloc_partials[kScratchFp2];
static __device__ __align__(256) unsigned g_noalloc_counter[64];

struct TripleTerms {
    const Fp2 *a, *b, *c;
    __device__ __forceinline__ void operator()(size_t i, Acc<3>& acc) const {
        using namespace vzb;
        const Fp2 a0 = ldcs2(a + 2 * i), a1 = ldcs2(a + 2 * i + 1);
        const Fp2 b0 = ldcs2(b + 2 * i), b1 = ldcs2(b + 2 * i + 1);
        const Fp2 c0 = ldcs2(c + 2 * i), c1 = ldcs2(c + 2 * i + 1);
        const Fp2 da = f2sub(a1, a0), db = f2sub(b1, b0), dc = f2sub(c1, c0);
        const Fp2 a2 = f2add(a1, da), b2 = f2add(b1, db), c2 = f2add(c1, dc);
        const Fp2 a3 = f2add(a2, da), b3 = f2add(b2, db), c3 = f2add(c2, dc);
        acc.v[0] = f2add(acc.v[0], f2mul(f2mul(a0, b0), c0));
        acc.v[1] = f2add(acc.v[1], f2mul(f2mul(a2, b2), c2));
        acc.v[2] = f2add(acc.v[2], f2mul(f2mul(a3, b3), c3));
    }
};

struct Store3 {
    Fp2* out;
    __device__ __forceinline__ void operator()(const Acc<3>& s) const {
        out[0] = s.v[0];
        out[1] = s.v[1];
        out[2] = s.v[2];
    }
};

__global__ void __launch_bounds__(kThreads) noalloc_triple_kernel(TripleTerms t, size_t pairs, Fp2* partials,
                                                                  unsigned* counter, Store3 epi) {
    Acc<3> acc;
    acc.zero();
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < pairs; i += stride) t(i, acc);
    vzb::grid_finish<3>(acc, partials, counter, epi);
}

struct DeviceScratch {
    unsigned long long context_id = 0;  // driver context the addresses belong to
    Fp2* partials = nullptr;
    unsigned* counter = nullptr;
};

constexpr int kMaxDevices = 64;
std::mutex g_setup_mutex;
DeviceScratch g_scratch[kMaxDevices];

// The unique id of the current driver context (cuCtxGetCurrent + cuCtxGetId,
// reached through the runtime's driver entry points so the library does not
// link libcuda).  0 when no context is current yet or the query is missing.
unsigned long long current_context_id() {
    using GetCurrent = int (*)(void**);
    using GetId = int (*)(void*, unsigned long long*);
    static GetCurrent get_current = nullptr;
    static GetId get_id = nullptr;
    static bool looked_up = false;
    if (!looked_up) {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrent>(f);
        f = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetId>(f);
        looked_up = true;
    }
    void* ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != 0 || !ctx || get_id(ctx, &id) != 0) return 0;
    return id;
}

// Resolve the scratch addresses for the current device: once per device and
// driver context, with that device current.  A context created after the
// previous one was destroyed (cudaDeviceReset) has a new id, so its
// addresses are resolved again instead of reusing stale ones.
cudaError_t scratch_for_current_device(DeviceScratch* out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
    std::lock_guard<std::mutex> lock(g_setup_mutex);
    DeviceScratch& s = g_scratch[dev];
    const unsigned long long ctx = current_context_id();
    if (!s.partials || ctx == 0 || ctx != s.context_id) {
        void* p = nullptr;
        void* q = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_partials);  // makes the device's primary context current
        if (e != cudaSuccess) return e;
        e = cudaGetSymbolAddress(&q, g_noalloc_counter);
        if (e != cudaSuccess) return e;
        s.partials = static_cast<Fp2*>(p);
        s.counter = static_cast<unsigned*>(q);
        s.context_id = current_context_id();
    }
    *out = s;
    return cudaSuccess;
}

}  // namespace

extern "C" int volta_b200_triple_product_round_noalloc(const vz_fp2* a, const vz_fp2* b, const vz_fp2* c,
                                                       size_t pairs, vz_fp2* output, void* stream) {
    if (!a || !b || !c || !output || !pairs) return -1;
    if (pairs > kMaxPairs) return VOLTA_B200_NOALLOC_TOO_LARGE;
    DeviceScratch s;
    cudaError_t e = scratch_for_current_device(&s);
    if (e != cudaSuccess) return static_cast<int>(e);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // the last-block counter must start at zero; partials are fully rewritten
    e = cudaMemsetAsync(s.counter, 0, sizeof(unsigned), st);
    if (e != cudaSuccess) return static_cast<int>(e);
    const unsigned blocks = static_cast<unsigned>((pairs + kPairsPerBlock - 1) / kPairsPerBlock);
    noalloc_triple_kernel<<<blocks, kThreads, 0, st>>>(TripleTerms{a, b, c}, pairs, s.partials, s.counter,
                                                       Store3{output});
    e = cudaGetLastError();
    return e == cudaSuccess ? 0 : static_cast<int>(e);
}
