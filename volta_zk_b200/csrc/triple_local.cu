// Triple-product sumcheck rounds that stay on chip (extension,
// include/volta_b200_ext.h: volta_b200_triple_local_device and
// volta_b200_triple_flush_device).
//
// The triple-product sumcheck (reference semantics: hadamard.rs:222-240 for
// one round, cuda/volta_cuda_backend.cu:5106-5153 for the device round) pairs
// entries (2i, 2i + 1) in every round and folds pair i into entry i of the
// next round's tables.  A run of 2^13 consecutive entries therefore folds
// into one entry after 13 rounds without ever reading an entry outside the
// run.  With the challenges drawn in advance (a seeded stream that does not
// depend on the messages), one CTA runs all 13 rounds of its tile on chip:
//   rounds 0 and 1  in registers, straight from the loaded columns (each
//                   thread takes 4 consecutive entries: two pairs of round 0,
//                   one pair of round 1, one entry of round 2);
//   rounds 2 .. 6   through shared memory (2048 entries per table down to 64);
//   rounds 7 .. 12  in a second kernel, one warp per tile, one pair per lane,
//                   partners by shuffle (a warp per CTA idled the other seven
//                   through these short dependent rounds).
// The tables are read once; what is written back is the tiles' round-7
// tables (3 KB per 8192-entry tile, read once by the second kernel) and their
// three folded values.  The layer-by-layer chain (one launch per round, each
// reading and writing half of the previous tables) moved about six times
// the bytes and paid a launch and a grid reduction per round.
//
// Each tile's share of a round message is added to a u64 accumulator with
// integer atomics, split into 32-bit halves (4 counters per Fp2 value), so
// any number of tiles (and of launches, e.g. one per uploaded chunk) sum
// exactly and in any order; the flush turns the counters into canonical
// messages and zeroes them.  Messages are therefore bit-identical to the
// round-by-round path.
#include "reduce.cuh"
#include "runtime.cuh"

namespace vzb {

constexpr int kLocLog = 13;                      // entries per tile: 8192
constexpr int kLocThreads = 256;
constexpr int kLocWarps = kLocThreads / 32;
constexpr int kLocL2 = 1 << (kLocLog - 2);       // round-2 entries per table: 2048
constexpr int kLocQuads = kLocL2 / kLocThreads;  // quads per thread: 8
constexpr int kLocPairs = kLocL2 / 2 / kLocThreads;  // round-2 pairs per thread: 4
constexpr int kLocAccWords = kLocLog * 3 * 4;    // u64 counters per pass: round, term, coefficient, half
constexpr size_t kLocSmem = 3 * kLocL2 * sizeof(Fp2);
constexpr int kLocSmemRounds = 7;                // rounds 0 .. 6 in the tile kernel

namespace {

__device__ __forceinline__ void acc_add(unsigned long long* acc, uint64_t v) {
    atomicAdd(acc, v & 0xFFFFFFFFull);
    atomicAdd(acc + 1, v >> 32);
}

// Round terms of one pair: g(0), g(2), g(3) of a * b * c on the line
// through (0, x0) and (1, x1), accumulated lazily.
__device__ __forceinline__ void pair_terms(const Fp2 (&x0)[3], const Fp2 (&x1)[3], const Fp2 (&d)[3], Fp2W (&w)[3]) {
    const Fp2 a2 = d2add_weak(x1[0], d[0]), b2 = d2add_weak(x1[1], d[1]), c2 = d2add_weak(x1[2], d[2]);
    const Fp2 a3 = d2add_weak(a2, d[0]), b3 = d2add_weak(b2, d[1]), c3 = d2add_weak(c2, d[2]);
    f2w_mac(w[0], d2mul(x0[0], x0[1]), x0[2]);
    f2w_mac(w[1], d2mul(a2, b2), c2);
    f2w_mac(w[2], d2mul(a3, b3), c3);
}

__device__ __forceinline__ Fp2 warp_sum2(Fp2 v) {
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) v = f2add(v, shfl_down2(v, s));
    return v;
}

__device__ __forceinline__ Fp2 shfl2(Fp2 v, int src) {
    return Fp2{__shfl_sync(0xFFFFFFFFu, v.c0, src), __shfl_sync(0xFFFFFFFFu, v.c1, src)};
}

// Round-0 terms of a base-field pair (products in Fp; the message's c1 is 0)
// and its fold with r0: x0 + r0 (x1 - x0).
__device__ __forceinline__ void base_pair(const uint64_t (&v0)[3], const uint64_t (&v1)[3], Fp2 r0, W5 (&w)[3],
                                          Fp2 (&out)[3]) {
    uint64_t d[3], t2[3], t3[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) {
        d[k] = dsub(v1[k], v0[k]);
        t2[k] = dadd_weak(v1[k], d[k]);
        t3[k] = dadd_weak(t2[k], d[k]);
        out[k] = Fp2{dadd(v0[k], dmul(r0.c0, d[k])), dmul(r0.c1, d[k])};
    }
    wadd(w[0], dmul_wide(dmul(v0[0], v0[1]), v0[2]));
    wadd(w[1], dmul_wide(dmul(t2[0], t2[1]), t2[2]));
    wadd(w[2], dmul_wide(dmul(t3[0], t3[1]), t3[2]));
}

// Round-0 terms of an Fp2 pair and its fold with r0.
__device__ __forceinline__ void ext_pair(const Fp2 (&v0)[3], const Fp2 (&v1)[3], Fp2 r0, Fp2W (&w)[3],
                                         Fp2 (&out)[3]) {
    Fp2 d[3];
#pragma unroll
    for (int k = 0; k < 3; ++k) d[k] = d2sub(v1[k], v0[k]);
    pair_terms(v0, v1, d, w);
#pragma unroll
    for (int k = 0; k < 3; ++k) out[k] = d2add(v0[k], d2mul(d[k], r0));
}

template <bool kBase>
__global__ void __launch_bounds__(kLocThreads, 2)
    triple_local_kernel(const void* __restrict__ ta, const void* __restrict__ tb, const void* __restrict__ tc,
                        size_t tile0, const Fp2* __restrict__ rs, unsigned long long* __restrict__ acc,
                        Fp2* __restrict__ lvl7) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    Fp2* v = reinterpret_cast<Fp2*>(smem_raw);  // [3][kLocL2]
    __shared__ Fp2 red[kLocSmemRounds][3][kLocWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t tile = tile0 + blockIdx.x;
    const size_t first = tile << kLocLog;
    const Fp2 r0 = ldg2(rs), r1 = ldg2(rs + 1);

    // ---- rounds 0 and 1 from the columns ----------------------------------
    {
        W5 w0b[3];       // round 0, base tables
        Fp2W w0[3], w1[3];
#pragma unroll
        for (int e = 0; e < 3; ++e) {
            f2w_zero(w0[e]);
            f2w_zero(w1[e]);
#pragma unroll
            for (int i = 0; i < 5; ++i) w0b[e].w[i] = 0;
        }
#pragma unroll 1
        for (int m = 0; m < kLocQuads; ++m) {
            const int q = threadIdx.x + m * kLocThreads;
            Fp2 x0[3], x1[3];
            if constexpr (kBase) {
                uint64_t v0[3], v1[3], v2[3], v3[3];
                const uint64_t* src[3] = {static_cast<const uint64_t*>(ta), static_cast<const uint64_t*>(tb),
                                          static_cast<const uint64_t*>(tc)};
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    const ulonglong2* p = reinterpret_cast<const ulonglong2*>(src[k] + first + 4 * size_t(q));
                    const ulonglong2 lo = __ldcs(p), hi = __ldcs(p + 1);
                    v0[k] = lo.x;
                    v1[k] = lo.y;
                    v2[k] = hi.x;
                    v3[k] = hi.y;
                }
                base_pair(v0, v1, r0, w0b, x0);
                base_pair(v2, v3, r0, w0b, x1);
            } else {
                const Fp2* src[3] = {static_cast<const Fp2*>(ta), static_cast<const Fp2*>(tb),
                                     static_cast<const Fp2*>(tc)};
#pragma unroll
                for (int h = 0; h < 2; ++h) {  // one round-0 pair at a time
                    Fp2 v0[3], v1[3];
#pragma unroll
                    for (int k = 0; k < 3; ++k) {
                        const Fp2* p = src[k] + first + 4 * size_t(q) + 2 * h;
                        v0[k] = ldcs2(p);
                        v1[k] = ldcs2(p + 1);
                    }
                    ext_pair(v0, v1, r0, w0, h ? x1 : x0);
                }
            }
            Fp2 d[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) d[k] = d2sub(x1[k], x0[k]);
            pair_terms(x0, x1, d, w1);
#pragma unroll
            for (int k = 0; k < 3; ++k) v[k * kLocL2 + q] = d2add(x0[k], d2mul(d[k], r1));
        }
#pragma unroll
        for (int e = 0; e < 3; ++e) {
            const Fp2 s0 = warp_sum2(kBase ? Fp2{wreduce(w0b[e]), 0} : f2w_reduce(w0[e]));
            const Fp2 s1 = warp_sum2(f2w_reduce(w1[e]));
            if (lane == 0) {
                red[0][e][warp] = s0;
                red[1][e][warp] = s1;
            }
        }
    }
    __syncthreads();

    // ---- rounds 2 .. 6 through shared memory -------------------------------
    int j = 2;
#pragma unroll 1
    for (; (kLocL2 >> (j - 2)) > 64; ++j) {
        const int pairs = kLocL2 >> (j - 1);
        const Fp2 r = ldg2(rs + j);
        Fp2W w[3];
#pragma unroll
        for (int e = 0; e < 3; ++e) f2w_zero(w[e]);
        // Pair i reads entries 2i, 2i + 1 and writes entry i, which pair i / 2
        // reads: only the lower half's writes can overtake a read, so that
        // half is held in registers across a barrier and the upper half
        // (reading [pairs, 2 pairs), writing [pairs / 2, pairs)) stores at once.
        Fp2 f[3][2];
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const int i = threadIdx.x + m * kLocThreads;
            if (i < pairs / 2) {
                Fp2 x0[3], x1[3], d[3];
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    x0[k] = v[k * kLocL2 + 2 * i];
                    x1[k] = v[k * kLocL2 + 2 * i + 1];
                    d[k] = d2sub(x1[k], x0[k]);
                }
                pair_terms(x0, x1, d, w);
#pragma unroll
                for (int k = 0; k < 3; ++k) f[k][m] = d2add(x0[k], d2mul(d[k], r));
            }
        }
        __syncthreads();  // the lower half's pairs are read before its entries land
#pragma unroll
        for (int m = 0; m < 2; ++m) {
            const int i = threadIdx.x + m * kLocThreads;
            if (i < pairs / 2)
#pragma unroll
                for (int k = 0; k < 3; ++k) v[k * kLocL2 + i] = f[k][m];
        }
        // one copy of the pair code for the upper half (instruction-cache
        // pressure: every inlined copy is about a thousand instructions)
#pragma unroll 1
        for (int m = 0; m < kLocPairs; ++m) {
            const int i = threadIdx.x + m * kLocThreads;
            if (i >= pairs / 2 && i < pairs) {
                Fp2 x0[3], x1[3], d[3];
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    x0[k] = v[k * kLocL2 + 2 * i];
                    x1[k] = v[k * kLocL2 + 2 * i + 1];
                    d[k] = d2sub(x1[k], x0[k]);
                }
                pair_terms(x0, x1, d, w);
#pragma unroll
                for (int k = 0; k < 3; ++k) v[k * kLocL2 + i] = d2add(x0[k], d2mul(d[k], r));
            }
        }
        if (warp * 32 < pairs) {
#pragma unroll
            for (int e = 0; e < 3; ++e) {
                const Fp2 s = warp_sum2(f2w_reduce(w[e]));
                if (lane == 0) red[j][e][warp] = s;
            }
        }
        __syncthreads();
    }

    // ---- round-7 tables (64 entries each) to the warp-per-tile kernel -------
    if (threadIdx.x < 3 * 64)
        st2(lvl7 + static_cast<size_t>(blockIdx.x) * 3 * 64 + threadIdx.x,
            v[(threadIdx.x / 64) * kLocL2 + threadIdx.x % 64]);

    // ---- this tile's share of the messages of rounds 0 .. 6 ---------------
    if (threadIdx.x < kLocSmemRounds * 3) {
        const int round = threadIdx.x / 3, e = threadIdx.x % 3;
        // warps that held pairs of this round (8 for rounds 0 .. 4, then 4, 2)
        const int warps = round < 2 ? kLocWarps : min(kLocWarps, (kLocL2 >> (round - 1)) / 32);
        Fp2 s = red[round][e][0];
        for (int w = 1; w < warps; ++w) s = f2add(s, red[round][e][w]);
        unsigned long long* slot = acc + 4 * threadIdx.x;
        acc_add(slot, s.c0);
        acc_add(slot + 2, s.c1);
    }
}

// Rounds 7 .. 12: one warp per tile, lane i holding the pair (2i, 2i + 1) of
// the 64-entry tables, partners of the next round by shuffle.  Thousands of
// independent warps hide the latency of these short dependent rounds, which
// one warp per CTA could not.
__global__ void __launch_bounds__(kLocThreads) triple_local_warp_kernel(const Fp2* __restrict__ lvl7, size_t tiles,
                                                                        size_t tile0, const Fp2* __restrict__ rs,
                                                                        unsigned long long* __restrict__ acc,
                                                                        Fp2* __restrict__ fa, Fp2* __restrict__ fb,
                                                                        Fp2* __restrict__ fc) {
    constexpr int kRounds = kLocLog - kLocSmemRounds;  // 6
    __shared__ Fp2 red[kRounds][3][kLocWarps];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t t = static_cast<size_t>(blockIdx.x) * kLocWarps + warp;
    if (t < tiles) {
        const Fp2* src = lvl7 + t * 3 * 64;
        Fp2 x0[3], x1[3];
#pragma unroll
        for (int k = 0; k < 3; ++k) {
            x0[k] = ldcs2(src + k * 64 + 2 * lane);
            x1[k] = ldcs2(src + k * 64 + 2 * lane + 1);
        }
#pragma unroll 1
        for (int jj = 0; jj < kRounds; ++jj) {
            const int pairs = 32 >> jj;
            const Fp2 r = ldg2(rs + kLocSmemRounds + jj);
            Fp2W w[3];
#pragma unroll
            for (int e = 0; e < 3; ++e) f2w_zero(w[e]);
            Fp2 d[3], y[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) d[k] = d2sub(x1[k], x0[k]);
            if (lane < pairs) pair_terms(x0, x1, d, w);
#pragma unroll
            for (int k = 0; k < 3; ++k) y[k] = d2add(x0[k], d2mul(d[k], r));
#pragma unroll
            for (int e = 0; e < 3; ++e) {
                const Fp2 sum = warp_sum2(f2w_reduce(w[e]));
                if (lane == 0) red[jj][e][warp] = sum;
            }
            if (jj == kRounds - 1) {
                if (lane == 0) {
                    st2(fa + tile0 + t, y[0]);
                    st2(fb + tile0 + t, y[1]);
                    st2(fc + tile0 + t, y[2]);
                }
            } else {
                // entry i of the next round sits in lane i: pair i takes lanes 2i, 2i + 1
                const int a = (2 * lane) & 31, b = (2 * lane + 1) & 31;
#pragma unroll
                for (int k = 0; k < 3; ++k) {
                    x0[k] = shfl2(y[k], a);
                    x1[k] = shfl2(y[k], b);
                }
            }
        }
    } else if (lane == 0) {
#pragma unroll
        for (int jj = 0; jj < kRounds; ++jj)
#pragma unroll
            for (int e = 0; e < 3; ++e) red[jj][e][warp] = Fp2{0, 0};
    }
    __syncthreads();
    if (threadIdx.x < kRounds * 3) {
        const int jj = threadIdx.x / 3, e = threadIdx.x % 3;
        Fp2 s = red[jj][e][0];
#pragma unroll
        for (int w = 1; w < kLocWarps; ++w) s = f2add(s, red[jj][e][w]);
        unsigned long long* slot = acc + 4 * (kLocSmemRounds * 3 + threadIdx.x);
        acc_add(slot, s.c0);
        acc_add(slot + 2, s.c1);
    }
}

// Canonical value of lo + hi 2^32 (lo, hi < 2^64).
__device__ __forceinline__ uint64_t acc_value(unsigned long long lo, unsigned long long hi) {
    const uint64_t h = dmul(hi >= kP ? hi - kP : hi, 0x100000000ull);
    return dadd(lo >= kP ? lo - kP : lo, h);
}

__global__ void triple_flush_kernel(unsigned long long* acc, int rounds, Fp2* out) {
    const int i = threadIdx.x;
    if (i >= rounds * 3) return;
    unsigned long long* slot = acc + 4 * i;
    st2(out + i, Fp2{acc_value(slot[0], slot[1]), acc_value(slot[2], slot[3])});
#pragma unroll
    for (int k = 0; k < 4; ++k) slot[k] = 0;
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_b200_triple_local_device(void* raw, int base, uint64_t a_id, uint64_t b_id, uint64_t c_id,
                                              size_t len, size_t tile0, size_t tiles, uint64_t r_id,
                                              size_t r_offset, uint64_t acc_id, uint64_t fa_id, uint64_t fb_id,
                                              uint64_t fc_id) {
    Context* c = static_cast<Context*>(raw);
    constexpr size_t kTile = size_t{1} << kLocLog;
    if (!c || len < kTile || (len & (len - 1)) || !tiles || tile0 + tiles > len / kTile || tiles > 0x7FFFFFFFu)
        return fail_message(c, "invalid on-chip triple-product geometry");
    const size_t esize = base ? sizeof(uint64_t) : sizeof(Fp2), total = len / kTile;
    void *a = nullptr, *b = nullptr, *cc = nullptr, *r = nullptr, *acc = nullptr, *fa = nullptr, *fb = nullptr,
         *fc = nullptr;
    if (region_elems(c, a_id, 0, len, esize, &a) || region_elems(c, b_id, 0, len, esize, &b) ||
        region_elems(c, c_id, 0, len, esize, &cc) || region_elems(c, r_id, r_offset, kLocLog, sizeof(Fp2), &r) ||
        region_elems(c, acc_id, 0, kLocAccWords, sizeof(uint64_t), &acc) ||
        region_elems(c, fa_id, 0, total, sizeof(Fp2), &fa) || region_elems(c, fb_id, 0, total, sizeof(Fp2), &fb) ||
        region_elems(c, fc_id, 0, total, sizeof(Fp2), &fc))
        return -1;
    // the tiles' round-7 tables (3 x 64 entries each) between the two kernels
    if (ensure_ws(c, kWsScratch, tiles * 3 * 64 * sizeof(Fp2))) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const Fp2* rs = static_cast<const Fp2*>(r);
    unsigned long long* ac = static_cast<unsigned long long*>(acc);
    Fp2* lvl7 = ws<Fp2>(c, kWsScratch);
    if (base) {
        VZB_CUDA(c, cudaFuncSetAttribute(triple_local_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kLocSmem)));
        triple_local_kernel<true><<<static_cast<unsigned>(tiles), kLocThreads, kLocSmem, c->stream>>>(
            a, b, cc, tile0, rs, ac, lvl7);
    } else {
        VZB_CUDA(c, cudaFuncSetAttribute(triple_local_kernel<false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kLocSmem)));
        triple_local_kernel<false><<<static_cast<unsigned>(tiles), kLocThreads, kLocSmem, c->stream>>>(
            a, b, cc, tile0, rs, ac, lvl7);
    }
    VZB_LAUNCHED(c);
    triple_local_warp_kernel<<<static_cast<unsigned>((tiles + kLocWarps - 1) / kLocWarps), kLocThreads, 0,
                               c->stream>>>(lvl7, tiles, tile0, rs, ac, static_cast<Fp2*>(fa),
                                            static_cast<Fp2*>(fb), static_cast<Fp2*>(fc));
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_b200_triple_flush_device(void* raw, uint64_t acc_id, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c) return -1;
    void *acc = nullptr, *out = nullptr;
    if (region_elems(c, acc_id, 0, kLocAccWords, sizeof(uint64_t), &acc) ||
        region_elems(c, out_id, out_offset, 3 * kLocLog, sizeof(Fp2), &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    triple_flush_kernel<<<1, 64, 0, c->stream>>>(static_cast<unsigned long long*>(acc), kLocLog,
                                                 static_cast<Fp2*>(out));
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}
