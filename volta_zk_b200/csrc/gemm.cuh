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
// Layout: the operands are first split into byte planes, A as [m][Kp] and B
// as [n][Kp] (k contiguous, zero-padded to Kp = 64-multiple), then a CTA
// computes a 64 x 64 tile with 4 warps (32 x 32 each) from a 2-stage cp.async
// pipeline of 64-byte k slices (rows padded to 80 B: conflict-free ldmatrix).
#pragma once

#include "runtime.cuh"

namespace vzb {

constexpr int kGemmBM = 64, kGemmBN = 64, kGemmBK = 64;
constexpr int kGemmRow = kGemmBK + 16;  // shared-memory row pitch in bytes
constexpr int kGemmThreads = 128;
constexpr size_t kGemmChunkK = 16384;   // int32 partials stay exact below this

// Byte planes of `batches` independent products (batch z at z * a_batch /
// z * b_batch bytes into each plane).
struct GemmPlanes {
    const int8_t* a_hi;
    const uint8_t* a_lo;
    const int8_t* b_hi;
    const uint8_t* b_lo;
    size_t m, n, kp;
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
// [0,m) x [0,n); tiles for which epi.active(z, m0, n0) is false are skipped.
template <class Epi, bool kLongK>
__global__ void __launch_bounds__(kGemmThreads) gemm_planes_kernel(GemmPlanes g, Epi epi) {
    __shared__ __align__(16) unsigned char sm[2][4][kGemmBM][kGemmRow];  // stage, plane, row, k bytes
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int wm = warp >> 1, wn = warp & 1;
    const size_t m0 = static_cast<size_t>(blockIdx.y) * kGemmBM, n0 = static_cast<size_t>(blockIdx.x) * kGemmBN;
    const size_t bz = blockIdx.z;
    if (!epi.active(bz, m0, n0)) return;
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
            const unsigned char* src = static_cast<const unsigned char*>(base) + rr * g.kp + k0 + c * 16;
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

// Byte planes of `batches` row-major matrices [rows][k] (row stride ld,
// batch b starting at x + b * boff) into hi/lo [batches][rows][kp], zero
// beyond k.
__global__ void split_planes_kernel(const int16_t* x, size_t rows, size_t k, size_t ld, int8_t* hi, uint8_t* lo,
                                    size_t kp, unsigned batches, size_t boff);
// Byte planes of the transposes: batch b of x is [k][n] row-major (stride ld,
// starting at x + b * boff); planes are [batches][n][kp].
__global__ void split_planes_t_kernel(const int16_t* x, size_t k, size_t n, size_t ld, int8_t* hi, uint8_t* lo,
                                      size_t kp, size_t boff);

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
    const dim3 grid(static_cast<unsigned>((g.n + kGemmBN - 1) / kGemmBN),
                    static_cast<unsigned>((g.m + kGemmBM - 1) / kGemmBM), g.batches);
    if (grid.y > 65535 || grid.z > 65535) return fail_message(c, "GEMM shape exceeds the launch grid");
    if (g.kp > kGemmChunkK)
        gemm_planes_kernel<Epi, true><<<grid, kGemmThreads, 0, c->stream>>>(g, epi);
    else
        gemm_planes_kernel<Epi, false><<<grid, kGemmThreads, 0, c->stream>>>(g, epi);
    VZB_LAUNCHED(c);
    return 0;
}
#endif

}  // namespace vzb
