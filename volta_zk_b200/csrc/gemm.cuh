// Exact int16 x int16 -> int64 GEMM on the tensor cores.
//
// Each int16 operand splits into a signed high and an unsigned low byte,
// x = 256 xh + xl (xh in [-128, 127], xl in [0, 255]), so
//   a b = 65536 ah bh + 256 (ah bl + al bh) + al bl.
// The three partial sums are int8 tensor-core products with int32
// accumulation (exact while k <= 16384: |partial| <= k 2^16 < 2^31); longer
// reductions flush the int32 partials into int64 every 16384 terms.  The
// epilogue recombines them in int64, so every accumulator equals the
// reference's scalar i64 loop (cuda/volta_cuda_backend.cu:1412-1440,
// rust/volta-gpt2/src/gemm.rs:40-60) bit for bit.
//
// Layout: the operands are first split into byte planes, A with m rows and B
// with n rows, each row holding its k bytes zero-padded to Kp (a multiple of
// 64) and the row count padded to a multiple of 128.  A plane is stored as
// Kp / 64 k-slices; inside a slice, rows come in groups of 8 and each group
// holds four 8 x 16-byte core matrices (see plane_off).  A 128-row slab of one
// k-slice is therefore one contiguous 8 KiB block that a single bulk copy
// moves into shared memory already in the tensor core's canonical K-major
// layout.
//
// gemm_tc_kernel (K <= 16384) is a persistent kernel on the 5th generation
// tensor cores, one CTA per SM walking 128 x 128 output tiles: one lane
// streams the slabs with cp.async.bulk into a 5-stage mbarrier ring, one lane
// issues tcgen05.mma kind::i8 into three int32 accumulators in tensor memory,
// and eight epilogue warps empty tensor memory into registers right after
// each tile so that the next tile's MMAs overlap the stores.  gemm_planes_kernel (longer K) is the mma.sync form
// with 64 x 64 tiles, which flushes int32 partials into int64 registers.
#pragma once

#include "runtime.cuh"

namespace vzb {

constexpr int kGemmBM = 64, kGemmBN = 64, kGemmBK = 64;
constexpr int kGemmRow = kGemmBK + 16;  // shared-memory row pitch in bytes
constexpr int kGemmThreads = 128;
constexpr size_t kGemmChunkK = 16384;   // int32 partials stay exact below this
constexpr size_t kPlaneRowAlign = 128;  // plane row counts are padded to this

// Byte offset of element (r, k) in a plane of `rpad` rows.
__host__ __device__ __forceinline__ size_t plane_off(size_t r, size_t k, size_t rpad) {
    return (k >> 6) * (rpad << 6) + ((r >> 3) << 9) + (((k & 63) >> 4) << 7) + ((r & 7) << 4) + (k & 15);
}
inline size_t plane_rows(size_t rows) { return (rows + kPlaneRowAlign - 1) / kPlaneRowAlign * kPlaneRowAlign; }

// Byte planes of `batches` independent products (batch z at z * a_batch /
// z * b_batch bytes into each plane; a_batch = mpad * kp, b_batch = npad * kp).
struct GemmPlanes {
    const int8_t* a_hi;
    const uint8_t* a_lo;
    const int8_t* b_hi;
    const uint8_t* b_lo;
    size_t m, n, kp;
    size_t mpad = 0, npad = 0;  // plane row counts (multiples of kPlaneRowAlign)
    size_t a_batch = 0, b_batch = 0;
    unsigned batches = 1;
};

#ifdef __CUDACC__

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool valid) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    const int bytes = valid ? 16 : 0;  // zero-fill rows beyond m / n
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(s), "l"(gmem), "r"(bytes));
}

__device__ __forceinline__ void ldsm_x4(const void* smem, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    const unsigned s = static_cast<unsigned>(__cvta_generic_to_shared(smem));
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(s));
}

#define VZB_MMA_I8(TA, TB, d, a, b)                                                                   \
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32." TA "." TB ".s32 {%0,%1,%2,%3}, "          \
                 "{%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};\n"                                          \
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])                                    \
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]))

// epi(z, i, j, acc) is called once per output element of batch z inside
// [0,m) x [0,n); tiles for which epi.active(z, m0, n0, tile_rows) is false
// are skipped.
template <class Epi, bool kLongK>
__global__ void __launch_bounds__(kGemmThreads) gemm_planes_kernel(GemmPlanes g, Epi epi) {
    __shared__ __align__(16) unsigned char sm[2][4][kGemmBM][kGemmRow];  // stage, plane, row, k bytes
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 1, wn = warp & 1;
    const size_t m0 = static_cast<size_t>(blockIdx.y) * kGemmBM, n0 = static_cast<size_t>(blockIdx.x) * kGemmBN;
    const size_t bz = blockIdx.z;
    if (!epi.active(bz, m0, n0, kGemmBM)) return;
    g.a_hi += bz * g.a_batch;
    g.a_lo += bz * g.a_batch;
    g.b_hi += bz * g.b_batch;
    g.b_lo += bz * g.b_batch;
    const size_t ktiles = g.kp / kGemmBK;

    auto load = [&](int stage, size_t kt) {
        const size_t k0 = kt * kGemmBK;
#pragma unroll
        for (int it = 0; it < 8; ++it) {
            const int chunk = tid + it * kGemmThreads;  // 0..1023
            const int plane = chunk >> 8, r = (chunk >> 2) & 63, c = chunk & 3;
            const bool is_a = plane < 2;
            const size_t row = (is_a ? m0 : n0) + r;
            const bool valid = row < (is_a ? g.m : g.n);
            const size_t rr = valid ? row : 0;
            const void* base = plane == 0 ? static_cast<const void*>(g.a_hi)
                               : plane == 1 ? static_cast<const void*>(g.a_lo)
                               : plane == 2 ? static_cast<const void*>(g.b_hi)
                                            : static_cast<const void*>(g.b_lo);
            const unsigned char* src =
                static_cast<const unsigned char*>(base) + plane_off(rr, k0 + c * 16, is_a ? g.mpad : g.npad);
            cp_async16(&sm[stage][plane][r][c * 16], src, valid);
        }
        asm volatile("cp.async.commit_group;\n" ::);
    };

    int32_t acc[3][2][4][4];  // [hh, mid, ll][mt][nt][frag]
    int64_t wide[kLongK ? 2 : 1][kLongK ? 4 : 1][kLongK ? 4 : 1];
#pragma unroll
    for (int s = 0; s < 3; ++s)
#pragma unroll
        for (int a = 0; a < 2; ++a)
#pragma unroll
            for (int b = 0; b < 4; ++b)
#pragma unroll
                for (int e = 0; e < 4; ++e) acc[s][a][b][e] = 0;
    if (kLongK) {
#pragma unroll
        for (int a = 0; a < (kLongK ? 2 : 1); ++a)
#pragma unroll
            for (int b = 0; b < (kLongK ? 4 : 1); ++b)
#pragma unroll
                for (int e = 0; e < (kLongK ? 4 : 1); ++e) wide[a][b][e] = 0;
    }
    auto flush = [&]() {
        if constexpr (kLongK) {
#pragma unroll
        for (int mt = 0; mt < 2; ++mt)
#pragma unroll
            for (int nt = 0; nt < 4; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    wide[kLongK ? mt : 0][kLongK ? nt : 0][kLongK ? e : 0] +=
                        65536 * static_cast<int64_t>(acc[0][mt][nt][e]) +
                        256 * static_cast<int64_t>(acc[1][mt][nt][e]) + static_cast<int64_t>(acc[2][mt][nt][e]);
                    acc[0][mt][nt][e] = acc[1][mt][nt][e] = acc[2][mt][nt][e] = 0;
                }
        }
    };

    if (ktiles) load(0, 0);
    for (size_t kt = 0; kt < ktiles; ++kt) {
        if (kt + 1 < ktiles) {
            load(static_cast<int>((kt + 1) & 1), kt + 1);
            asm volatile("cp.async.wait_group 1;\n" ::);
        } else {
            asm volatile("cp.async.wait_group 0;\n" ::);
        }
        __syncthreads();
        const int st = static_cast<int>(kt & 1);
#pragma unroll
        for (int kk = 0; kk < 2; ++kk) {
            uint32_t a[2][2][4];  // [hi, lo][mt][reg]
            uint32_t b[2][4][2];  // [hi, lo][nt][reg]
#pragma unroll
            for (int pl = 0; pl < 2; ++pl)
#pragma unroll
                for (int mt = 0; mt < 2; ++mt)
                    ldsm_x4(&sm[st][pl][wm * 32 + mt * 16 + (lane & 15)][kk * 32 + (lane >> 4) * 16], a[pl][mt][0],
                            a[pl][mt][1], a[pl][mt][2], a[pl][mt][3]);
#pragma unroll
            for (int pl = 0; pl < 2; ++pl)
#pragma unroll
                for (int p = 0; p < 2; ++p) {
                    const int q = lane >> 3;
                    ldsm_x4(&sm[st][2 + pl][wn * 32 + p * 16 + (q >> 1) * 8 + (lane & 7)][kk * 32 + (q & 1) * 16],
                            b[pl][2 * p][0], b[pl][2 * p][1], b[pl][2 * p + 1][0], b[pl][2 * p + 1][1]);
                }
#pragma unroll
            for (int mt = 0; mt < 2; ++mt)
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    VZB_MMA_I8("s8", "s8", acc[0][mt][nt], a[0][mt], b[0][nt]);
                    VZB_MMA_I8("s8", "u8", acc[1][mt][nt], a[0][mt], b[1][nt]);
                    VZB_MMA_I8("u8", "s8", acc[1][mt][nt], a[1][mt], b[0][nt]);
                    VZB_MMA_I8("u8", "u8", acc[2][mt][nt], a[1][mt], b[1][nt]);
                }
        }
        __syncthreads();
        if (kLongK && ((kt + 1) % (kGemmChunkK / kGemmBK)) == 0) flush();
    }
    if (kLongK) flush();
    // epilogue: fragment element e -> row g (+8 for e >= 2), column 2 tig + (e & 1)
    const int grp = lane >> 2, tig = lane & 3;
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
        for (int nt = 0; nt < 4; ++nt)
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const size_t i = m0 + wm * 32 + mt * 16 + grp + (e >> 1) * 8;
                const size_t j = n0 + wn * 32 + nt * 8 + tig * 2 + (e & 1);
                if (i < g.m && j < g.n) {
                    const int64_t v = kLongK ? wide[kLongK ? mt : 0][kLongK ? nt : 0][kLongK ? e : 0]
                                             : 65536 * static_cast<int64_t>(acc[0][mt][nt][e]) +
                                                   256 * static_cast<int64_t>(acc[1][mt][nt][e]) +
                                                   static_cast<int64_t>(acc[2][mt][nt][e]);
                    epi(bz, i, j, v);
                }
            }
}
#undef VZB_MMA_I8

// ---- tcgen05 form -----------------------------------------------------------

constexpr int kTcBM = 128, kTcBN = 128, kTcStages = 5;
constexpr int kTcEpiWarps = 8, kTcThreads = 64 + 32 * kTcEpiWarps;  // producer, MMA, epilogue warps
constexpr int kTcEpiCols = kTcBN / (kTcEpiWarps / 4);             // columns per epilogue warp
constexpr uint32_t kTcTileA = kTcBM * kGemmBK;                    // one A plane tile (8 KiB)
constexpr uint32_t kTcTileB = kTcBN * kGemmBK;                    // one B plane tile (8 KiB)
constexpr uint32_t kTcStageBytes = 2 * kTcTileA + 2 * kTcTileB;   // hi + lo of A and B
constexpr int kTcPitch = 17;                                      // epilogue transpose row pitch (int64)
constexpr size_t kTcTransBytes = static_cast<size_t>(kTcEpiWarps) * 32 * kTcPitch * 8;
constexpr size_t kTcSmem = static_cast<size_t>(kTcStages) * kTcStageBytes + kTcTransBytes;
constexpr uint32_t kTcTmemCols = 512;                             // hh, mid, ll: 3 x kTcBN columns
constexpr unsigned long long kTcWaitNs = 2000000000ull;           // bound of every pipeline wait
static_assert(kTcSmem <= 227 * 1024, "stage ring + transpose buffer fit one CTA");

__device__ __forceinline__ uint32_t tc_smem(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long tc_clock() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Bounded wait for the completion of phase `parity` of an mbarrier; gives up
// at once when another role of the CTA has already failed (unless `failed`
// is null).
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, const volatile int* failed) {
    const unsigned long long t0 = tc_clock();
    for (;;) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}\n"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
        if ((failed && *failed) || tc_clock() - t0 > kTcWaitNs) return false;
    }
}

__device__ __forceinline__ void tc_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(bar) : "memory");
}

// Shared-memory matrix descriptor, no swizzle (version 1 = tcgen05): start,
// leading-dimension (K direction) and stride-dimension (M/N direction) byte
// offsets between 8 x 16-byte core matrices.
__device__ __forceinline__ uint64_t tc_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFF) | (static_cast<uint64_t>((lbo >> 4) & 0x3FFF) << 16) |
           (static_cast<uint64_t>((sbo >> 4) & 0x3FFF) << 32) | (uint64_t{1} << 46);
}

// Instruction descriptor of kind::i8 with s32 accumulation, both operands
// K-major, M = kTcBM, N = kTcBN; the flags select signed (1) or unsigned (0)
// bytes.
__host__ __device__ constexpr uint32_t tc_idesc(uint32_t a_signed, uint32_t b_signed) {
    return (2u << 4) | (a_signed << 7) | (b_signed << 10) | (static_cast<uint32_t>(kTcBN >> 3) << 17) |
           (static_cast<uint32_t>(kTcBM >> 4) << 24);
}

__device__ __forceinline__ void tc_mma(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d),
        "l"(a), "l"(b), "r"(idesc), "r"(accumulate));
}

__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(bar)
                 : "memory");
}

__device__ __forceinline__ void tc_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}

// Tile t of the product, batches slowest.  Inside a batch the tiles of the
// smaller operand vary fastest, so that consecutive tiles (running on
// neighbouring SMs at the same time) share a slab of the larger operand.
struct TcTile {
    size_t m0, n0, bz;
};
__device__ __forceinline__ TcTile tc_tile(size_t t, size_t tiles_n, size_t tiles_m, bool m_fast) {
    const size_t per = tiles_n * tiles_m, bz = t / per, r = t - bz * per;
    if (m_fast) {
        const size_t tx = r / tiles_m;
        return TcTile{(r - tx * tiles_m) * kTcBM, tx * kTcBN, bz};
    }
    const size_t ty = r / tiles_n;
    return TcTile{ty * kTcBM, (r - ty * tiles_n) * kTcBN, bz};
}

// Persistent GEMM: CTA b handles tiles b, b + gridDim.x, ... (those with
// epi.active).  Warp 0 streams the 128-row slabs of each k-slice with
// cp.async.bulk into a kTcStages ring; warp 1 issues the tcgen05.mma of each
// tile into the three accumulators in tensor memory; warps 2..9 move each
// finished tile into registers, release tensor memory for the next tile and
// run the epilogue while it accumulates.  Only k-slices below
// epi.k_end(z, m0, tile_rows, kp) are read (all-zero slices of causal
// operands are skipped).  Requires g.kp <= kGemmChunkK (int32 accumulators
// stay exact).  A wait that runs out of time records 1 in *fault; the CTA
// then stops issuing work, waits (bounded) for its MMAs and releases tensor
// memory.
template <class Epi>
__global__ void __launch_bounds__(kTcThreads, 1) gemm_tc_kernel(GemmPlanes g, Epi epi, unsigned* fault) {
    extern __shared__ __align__(128) unsigned char tc_ring[];
    __shared__ __align__(8) uint64_t full_bar[kTcStages], empty_bar[kTcStages];
    __shared__ __align__(8) uint64_t acc_full, acc_empty, drain_bar;
    __shared__ uint32_t tmem_base;
    __shared__ volatile int failed;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const size_t tiles_n = (g.n + kTcBN - 1) / kTcBN, tiles_m = (g.m + kTcBM - 1) / kTcBM;
    const size_t tiles = tiles_n * tiles_m * g.batches;
    const bool m_fast = g.n > g.m;

    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(tc_smem(&tmem_base)),
                     "r"(kTcTmemCols));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::);
    }
    if (tid == 0) {
        for (int s = 0; s < kTcStages; ++s) {
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_smem(&full_bar[s])));
            asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_smem(&empty_bar[s])));
        }
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_smem(&acc_full)));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(tc_smem(&acc_empty)), "r"(kTcEpiWarps));
        asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;\n" ::"r"(tc_smem(&drain_bar)));
        asm volatile("fence.mbarrier_init.release.cluster;\n" ::);
        failed = 0;
    }
    __syncthreads();
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::);
    const uint32_t tmem = tmem_base;
    const uint32_t ring = tc_smem(tc_ring);

    if (warp == 0) {
        if (lane == 0) {
            // producer: the slab of each plane for k-slice kt is one
            // contiguous block at kt * rpad * 64 + row0 * 64
            const size_t step_a = g.mpad * kGemmBK, step_b = g.npad * kGemmBK;
            size_t slice = 0;  // k-slices streamed so far (all tiles)
            for (size_t t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
                const TcTile tl = tc_tile(t, tiles_n, tiles_m, m_fast);
                if (!epi.active(tl.bz, tl.m0, tl.n0, kTcBM)) continue;
                const size_t kts = epi.k_end(tl.bz, tl.m0, kTcBM, g.kp) / kGemmBK;
                const unsigned char* src[4] = {
                    reinterpret_cast<const unsigned char*>(g.a_hi) + tl.bz * g.a_batch + tl.m0 * kGemmBK,
                    g.a_lo + tl.bz * g.a_batch + tl.m0 * kGemmBK,
                    reinterpret_cast<const unsigned char*>(g.b_hi) + tl.bz * g.b_batch + tl.n0 * kGemmBK,
                    g.b_lo + tl.bz * g.b_batch + tl.n0 * kGemmBK};
                for (size_t kt = 0; kt < kts; ++kt, ++slice) {
                    const int s = static_cast<int>(slice % kTcStages);
                    if (slice >= static_cast<size_t>(kTcStages) &&
                        !tc_wait(tc_smem(&empty_bar[s]), static_cast<uint32_t>((slice / kTcStages - 1) & 1),
                                 &failed)) {
                        failed = 1;
                        break;
                    }
                    const uint32_t bar = tc_smem(&full_bar[s]);
                    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(bar),
                                 "r"(kTcStageBytes)
                                 : "memory");
                    const uint32_t dst = ring + s * kTcStageBytes;
                    const uint32_t off[4] = {0, kTcTileA, 2 * kTcTileA, 2 * kTcTileA + kTcTileB};
                    const uint32_t bytes[4] = {kTcTileA, kTcTileA, kTcTileB, kTcTileB};
#pragma unroll
                    for (int p = 0; p < 4; ++p) {
                        const unsigned char* from = src[p] + kt * (p < 2 ? step_a : step_b);
                        asm volatile(
                            "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];\n" ::
                                "r"(dst + off[p]),
                            "l"(from), "r"(bytes[p]), "r"(bar)
                            : "memory");
                    }
                }
            }
            if (failed) {
                // copies still in flight land before the CTA can exit
                for (size_t q = slice > static_cast<size_t>(kTcStages) ? slice - kTcStages : 0; q < slice; ++q)
                    tc_wait(tc_smem(&full_bar[q % kTcStages]), static_cast<uint32_t>((q / kTcStages) & 1), nullptr);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            // MMA issuer: per 64-byte k-slice, two K = 32 steps of the three
            // partial products (hh, hl + lh, ll); tile j starts once the
            // epilogue has taken tile j - 1 out of tensor memory
            constexpr uint32_t lbo = 128;             // next 16-byte k chunk
            constexpr uint32_t sbo = 8 * kGemmBK;     // next group of 8 rows
            size_t slice = 0, j = 0;
            for (size_t t = blockIdx.x; t < tiles && !failed; t += gridDim.x) {
                const TcTile tl = tc_tile(t, tiles_n, tiles_m, m_fast);
                if (!epi.active(tl.bz, tl.m0, tl.n0, kTcBM)) continue;
                const size_t kts = epi.k_end(tl.bz, tl.m0, kTcBM, g.kp) / kGemmBK;
                if (j >= 1 && !tc_wait(tc_smem(&acc_empty), static_cast<uint32_t>((j - 1) & 1), &failed)) {
                    failed = 1;
                    break;
                }
                asm volatile("tcgen05.fence::after_thread_sync;\n" ::);
                const uint32_t d = tmem;
                bool ok = true;
                for (size_t kt = 0; kt < kts; ++kt, ++slice) {
                    const int s = static_cast<int>(slice % kTcStages);
                    if (!tc_wait(tc_smem(&full_bar[s]), static_cast<uint32_t>((slice / kTcStages) & 1), &failed)) {
                        ok = false;
                        break;
                    }
                    asm volatile("tcgen05.fence::after_thread_sync;\n" ::);
                    const uint32_t a_hi = ring + s * kTcStageBytes, a_lo = a_hi + kTcTileA;
                    const uint32_t b_hi = a_hi + 2 * kTcTileA, b_lo = b_hi + kTcTileB;
#pragma unroll
                    for (int ks = 0; ks < kGemmBK / 32; ++ks) {
                        const uint32_t ko = ks * 2 * lbo;
                        const uint32_t acc = (kt > 0 || ks > 0) ? 1u : 0u;
                        const uint64_t dah = tc_desc(a_hi + ko, lbo, sbo), dal = tc_desc(a_lo + ko, lbo, sbo);
                        const uint64_t dbh = tc_desc(b_hi + ko, lbo, sbo), dbl = tc_desc(b_lo + ko, lbo, sbo);
                        tc_mma(d, dah, dbh, tc_idesc(1, 1), acc);
                        tc_mma(d + kTcBN, dah, dbl, tc_idesc(1, 0), acc);
                        tc_mma(d + kTcBN, dal, dbh, tc_idesc(0, 1), 1u);
                        tc_mma(d + 2 * kTcBN, dal, dbl, tc_idesc(0, 0), acc);
                    }
                    tc_commit(tc_smem(&empty_bar[s]));
                }
                if (!ok) {
                    failed = 1;
                    break;
                }
                tc_commit(tc_smem(&acc_full));
                ++j;
            }
            // completes once every MMA issued above has finished
            tc_commit(tc_smem(&drain_bar));
        }
    } else {
        // epilogue warps: warp w owns accumulator rows 32 (w % 4) .. + 31
        // (its tensor-memory lane quarter) and half of the columns.  It
        // pulls its 32 x 64 block into registers (combined into int64),
        // hands tensor memory back to the MMA warp, then stores the block 16
        // columns at a time through a private transpose buffer so that each
        // store covers 16 consecutive columns of two rows.
        const int quarter = warp & 3, col0 = ((warp - 2) >> 2) * kTcEpiCols;
        int64_t* tr = reinterpret_cast<int64_t*>(tc_ring + static_cast<size_t>(kTcStages) * kTcStageBytes) +
                      (warp - 2) * 32 * kTcPitch;
        const uint32_t lane_base = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + col0;
        size_t j = 0;
        for (size_t t = blockIdx.x; t < tiles; t += gridDim.x) {
            const TcTile tl = tc_tile(t, tiles_n, tiles_m, m_fast);
            if (!epi.active(tl.bz, tl.m0, tl.n0, kTcBM)) continue;
            if (!tc_wait(tc_smem(&acc_full), static_cast<uint32_t>(j & 1), &failed)) {
                failed = 1;
                break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;\n" ::);
            int64_t v[kTcEpiCols];
#pragma unroll
            for (int cc = 0; cc < kTcEpiCols; cc += 16) {
                uint32_t hh[16], mid[16], ll[16];
                tc_ld16(lane_base + cc, hh);
                tc_ld16(lane_base + kTcBN + cc, mid);
                tc_ld16(lane_base + 2 * kTcBN + cc, ll);
                asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::);
#pragma unroll
                for (int q = 0; q < 16; ++q)
                    v[cc + q] = 65536 * static_cast<int64_t>(static_cast<int32_t>(hh[q])) +
                                256 * static_cast<int64_t>(static_cast<int32_t>(mid[q])) +
                                static_cast<int64_t>(static_cast<int32_t>(ll[q]));
            }
            asm volatile("tcgen05.fence::before_thread_sync;\n" ::);
            __syncwarp();
            if (lane == 0) tc_arrive(tc_smem(&acc_empty));
#pragma unroll
            for (int cc = 0; cc < kTcEpiCols; cc += 16) {
#pragma unroll
                for (int q = 0; q < 16; ++q) tr[lane * kTcPitch + q] = v[cc + q];
                __syncwarp();
#pragma unroll 4
                for (int r2 = 0; r2 < 16; ++r2) {
                    const int row = 2 * r2 + (lane >> 4), col = lane & 15;
                    const size_t i = tl.m0 + quarter * 32 + row, jj = tl.n0 + col0 + cc + col;
                    if (i < g.m && jj < g.n) epi(tl.bz, i, jj, tr[row * kTcPitch + col]);
                }
                __syncwarp();
            }
            ++j;
        }
    }
    __syncwarp();
    // every MMA this CTA issued has finished before tensor memory is released
    if (!tc_wait(tc_smem(&drain_bar), 0, nullptr)) failed = 1;
    __syncthreads();
    if (failed && tid == 0) {
        *reinterpret_cast<volatile unsigned*>(fault) = 1u;
        __threadfence_system();
    }
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::);
    __syncthreads();
    if (warp == 1)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(tmem), "r"(kTcTmemCols));
}

// Byte planes of `batches` row-major matrices [rows][k] (row stride ld,
// batch b starting at x + b * boff) into planes of rpad rows, zero beyond k
// and beyond `rows`.
__global__ void split_planes_kernel(const int16_t* x, size_t rows, size_t k, size_t ld, int8_t* hi, uint8_t* lo,
                                    size_t kp, size_t rpad, unsigned batches, size_t boff);
// Byte planes of the transposes: batch b of x is [k][n] row-major (stride ld,
// starting at x + b * boff); planes have npad rows (one per column of x).
__global__ void split_planes_t_kernel(const int16_t* x, size_t k, size_t n, size_t ld, int8_t* hi, uint8_t* lo,
                                      size_t kp, size_t npad, unsigned batches, size_t boff);

#endif  // __CUDACC__

// Split A (m x k, row-major) and B (k x n row-major, or n x k when b_nk) into
// byte planes in the context's GEMM workspace; `batches` products whose
// operands start a_boff / b_boff elements apart.
int gemm_prepare(Context* c, const int16_t* a, size_t m, size_t k, size_t lda, const int16_t* b, size_t n,
                 size_t ldb, bool b_nk, GemmPlanes* out, unsigned batches = 1, size_t a_boff = 0,
                 size_t b_boff = 0);
// Planes for A supplied by the caller's own split (fills b only).
int gemm_prepare_b(Context* c, const int16_t* b, size_t k, size_t n, size_t ldb, bool b_nk, size_t kp,
                   unsigned batches, size_t b_boff, size_t a_bytes, GemmPlanes* out);

#ifdef __CUDACC__
template <class Epi>
int gemm_launch(Context* c, const GemmPlanes& g, const Epi& epi) {
    if (g.kp <= kGemmChunkK) {
        const size_t tiles = (g.n + kTcBN - 1) / kTcBN * ((g.m + kTcBM - 1) / kTcBM) * g.batches;
        const unsigned ctas = static_cast<unsigned>(tiles < static_cast<size_t>(c->sm_count) ? tiles : c->sm_count);
        VZB_CUDA(c, cudaFuncSetAttribute(gemm_tc_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(kTcSmem)));
        gemm_tc_kernel<Epi><<<ctas, kTcThreads, kTcSmem, c->stream>>>(g, epi, device_fault_word(c));
    } else {
        const dim3 grid(static_cast<unsigned>((g.n + kGemmBN - 1) / kGemmBN),
                        static_cast<unsigned>((g.m + kGemmBM - 1) / kGemmBM), g.batches);
        if (grid.y > 65535 || grid.z > 65535) return fail_message(c, "GEMM shape exceeds the launch grid");
        gemm_planes_kernel<Epi, true><<<grid, kGemmThreads, 0, c->stream>>>(g, epi);
    }
    VZB_LAUNCHED(c);
    return 0;
}
#endif

}  // namespace vzb
