// Reed-Solomon row encoding: forward DFT over Goldilocks, natural order in
// and out, a_j = sum_i a_i w^(ij) with w = 7^((p-1) >> log2 n)
// (rust/volta-pcs/src/ntt.rs:9-70; seam entry points
// cuda/volta_cuda_backend.cu:5534-5576, 6545-6579).  Fp2 rows transform
// each coordinate with the same base-field twiddles (the reference's
// fp2_mul_base butterflies, backend.cu:2600-2619).
//
// B200 design.  The reference runs a bit-reversal pass and one global
// kernel per stage (log2 n + 1 full HBM round trips per row).  Here:
//   * n <= 2^11: one CTA holds whole rows in shared memory (the bit
//     reversal happens on the load), runs every stage there and writes the
//     rows back: one read and one write of the data.
//   * 2^12 <= n <= 2^16 (the Ligero code lengths): the six-step split
//     n = n1 * n2 (n1, n2 in 64..256).  Pass 1 runs the n2 column DFTs of
//     length n1, applies w^(j2 k1) and stores the result transposed; pass 2
//     runs the n1 row DFTs of length n2 and stores X[k1 + n1 k2].  Each
//     length-m DFT is m = RA x RB in registers (radix-8/16 sub-DFTs whose
//     twiddles are powers of two, i.e. shifts) with a single shared-memory
//     exchange; every global access covers 16 adjacent elements (128 B for
//     Fp).  Rows go through in chunks whose transposed intermediate stays in
//     L2, so HBM sees one read of the input and one write of the output.
//   * 2^17 <= n <= 2^22: the same split with shared-memory radix-2 sub-DFTs.
//   * larger n: the per-stage global algorithm (correct, not tuned).
#include "runtime.cuh"

namespace vzb {
namespace {

constexpr int kNttThreads = 256;
constexpr int kSmallMaxBits = 11;
constexpr size_t kNttChunkBytes = size_t{48} << 20;  // transposed intermediate kept in L2

// x * 2^s mod p for 0 <= s < 192 (2 has order 192: 2^96 = -1).  With s a
// compile-time constant after unrolling this is a few funnel shifts and one
// reduction of the 160-bit shifted value.
__device__ __forceinline__ uint64_t mul_pow2(uint64_t x, int s) {
    const bool neg = s >= 96;
    s = neg ? s - 96 : s;
    if (s == 0) return neg ? dsub(0, x) : x;
    const int q = s >> 5, r = s & 31;
    const uint32_t x0 = lo32(x), x1 = hi32(x);
    const uint32_t l0 = r ? x0 << r : x0;
    const uint32_t l1 = r ? __funnelshift_l(x0, x1, r) : x1;
    const uint32_t l2 = r ? x1 >> (32 - r) : 0;
    W5 w;
    w.w[0] = q == 0 ? l0 : 0;
    w.w[1] = q == 0 ? l1 : (q == 1 ? l0 : 0);
    w.w[2] = q == 0 ? l2 : (q == 1 ? l1 : l0);
    w.w[3] = q == 1 ? l2 : (q == 2 ? l1 : 0);
    w.w[4] = q == 2 ? l2 : 0;
    const uint64_t y = wreduce(w);
    return neg ? dsub(0, y) : y;
}

// Butterfly arithmetic on the carry-chain forms (canonical in, canonical out).
struct FpOps {
    using T = uint64_t;
    static __device__ __forceinline__ T add(T a, T b) { return dadd(a, b); }
    static __device__ __forceinline__ T sub(T a, T b) { return dsub(a, b); }
    static __device__ __forceinline__ T mulb(T a, uint64_t w) { return dmul(a, w); }
    static __device__ __forceinline__ T mulp2(T a, int s) { return mul_pow2(a, s); }
};
struct Fp2Ops {
    using T = Fp2;
    static __device__ __forceinline__ T add(T a, T b) { return d2add(a, b); }
    static __device__ __forceinline__ T sub(T a, T b) { return d2sub(a, b); }
    static __device__ __forceinline__ T mulb(T a, uint64_t w) { return Fp2{dmul(a.c0, w), dmul(a.c1, w)}; }
    static __device__ __forceinline__ T mulp2(T a, int s) { return Fp2{mul_pow2(a.c0, s), mul_pow2(a.c1, s)}; }
};

// Register DFT of R <= 16 values, natural order in and out (radix-2 DIT on
// the bit-reversed registers).  The R-th roots of unity of the reference's
// generator are powers of two: w_2 = 2^96, w_4 = 2^48, w_8 = 2^120,
// w_16 = 2^156 (w_R = 7^((p-1)/R)), so every twiddle is a shift.
constexpr int ilog2c(int r) { return r <= 1 ? 0 : 1 + ilog2c(r >> 1); }
constexpr int root_exp(int r) { return r == 2 ? 96 : r == 4 ? 48 : r == 8 ? 120 : 156; }

template <class Ops, int R>
__device__ __forceinline__ void reg_dft(typename Ops::T (&v)[R]) {
    using T = typename Ops::T;
    constexpr int kLog = ilog2c(R);
    constexpr int kE = root_exp(R);
    T a[R];
    // (flat loops with intrinsic index arithmetic unroll completely, so the
    // arrays stay in registers)
#pragma unroll
    for (int i = 0; i < R; ++i) a[__brev(i) >> (32 - kLog)] = v[i];
#pragma unroll
    for (int lg = 0; lg < kLog; ++lg) {
#pragma unroll
        for (int b = 0; b < R / 2; ++b) {
            const int k = b & ((1 << lg) - 1);
            const int i0 = ((b >> lg) << (lg + 1)) + k, i1 = i0 + (1 << lg);
            const T u = a[i0];
            const T w = k == 0 ? a[i1] : Ops::mulp2(a[i1], (kE * k * (R >> (lg + 1))) % 192);
            a[i0] = Ops::add(u, w);
            a[i1] = Ops::sub(u, w);
        }
    }
#pragma unroll
    for (int i = 0; i < R; ++i) v[i] = a[i];
}

// One six-step pass over 16 sequences of length m = RA * RB per CTA, all
// arithmetic in registers with one shared-memory exchange:
//   step A (16 RB threads): DFT_RA over x[t + RB u] (u < RA), times w_m^(t k)
//   step B (16 RA threads): DFT_RB over t, giving X[k + RA k'].
// kCols: the sequences are 16 adjacent columns j2 of the n1 x n2 view (pass
// 1: length n1, output times w_n^(j2 k1), stored transposed as
// Y[k1][j2]); otherwise 16 adjacent rows k1 of Y (pass 2: length n2, output
// X[k1 + n1 k2]).  Every global access covers 16 adjacent elements.
template <class Ops, int RA, int RB, bool kCols>
__global__ void __launch_bounds__(16 * (RA > RB ? RA : RB)) ntt_pass_kernel(const typename Ops::T* in,
                                                                           typename Ops::T* out, int bits1,
                                                                           int bits2, const uint64_t* tw) {
    using T = typename Ops::T;
    constexpr int M = RA * RB;
    constexpr int kPitchT = RA + 1;              // odd: conflict-free 8-byte accesses
    constexpr int kPitchSeq = RB * kPitchT + 1;  // odd
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* S = reinterpret_cast<T*>(smem_raw);
    uint64_t* twm = reinterpret_cast<uint64_t*>(S + 16 * kPitchSeq);  // w_m^i, i < m
    const int n1 = 1 << bits1, n2 = 1 << bits2;
    const int bits = bits1 + bits2;
    const size_t n = size_t{1} << bits;
    const int seq_len_bits = kCols ? bits1 : bits2;  // = log2 M
    const int tiles = (kCols ? n2 : n1) / 16;
    const size_t row = blockIdx.x / tiles;
    const int base = (blockIdx.x - static_cast<int>(row * tiles)) * 16;
    const T* src = in + row * n;
    T* dst = out + row * n;
    for (int i = threadIdx.x; i < M; i += blockDim.x) {
        const size_t e = static_cast<size_t>(i) << (bits - seq_len_bits);
        twm[i] = e < n / 2 ? __ldg(tw + e) : dsub(0, __ldg(tw + (e - n / 2)));
    }
    __syncthreads();
    // ---- step A
    if (threadIdx.x < 16 * RB) {
        int seq, t;
        if (kCols) {
            seq = threadIdx.x & 15;
            t = threadIdx.x >> 4;
        } else {
            t = threadIdx.x % RB;
            seq = threadIdx.x / RB;
        }
        T v[RA];
#pragma unroll
        for (int u = 0; u < RA; ++u) {
            const int j = t + RB * u;
            v[u] = kCols ? src[static_cast<size_t>(j) * n2 + base + seq] : src[static_cast<size_t>(base + seq) * n2 + j];
        }
        reg_dft<Ops, RA>(v);
        T* srow = S + seq * kPitchSeq + t * kPitchT;
        srow[0] = v[0];
#pragma unroll
        for (int k = 1; k < RA; ++k) srow[k] = Ops::mulb(v[k], twm[t * k]);
    }
    __syncthreads();
    // ---- step B
    if (threadIdx.x < 16 * RA) {
        const int seq = threadIdx.x & 15, k = threadIdx.x >> 4;
        T v[RB];
#pragma unroll
        for (int t = 0; t < RB; ++t) v[t] = S[seq * kPitchSeq + t * kPitchT + k];
        reg_dft<Ops, RB>(v);
#pragma unroll
        for (int kp = 0; kp < RB; ++kp) {
            const int kk = k + RA * kp;  // output index within the sequence
            if (kCols) {
                const size_t j2 = base + seq;
                const size_t e = j2 * static_cast<size_t>(kk);  // < n
                const uint64_t w = e < n / 2 ? __ldg(tw + e) : dsub(0, __ldg(tw + (e - n / 2)));
                dst[static_cast<size_t>(kk) * n2 + j2] = e ? Ops::mulb(v[kp], w) : v[kp];
            } else {
                dst[base + seq + static_cast<size_t>(n1) * kk] = v[kp];
            }
        }
    }
}

__device__ __forceinline__ unsigned brev_bits(unsigned i, int bits) { return bits ? __brev(i) >> (32 - bits) : 0; }

// w^e for 0 <= e < n from the half table tw[i] = w^i (i < n/2): w^(n/2) = -1.
__device__ __forceinline__ uint64_t tw_at(const uint64_t* tw, size_t e, size_t n) {
    const size_t h = n / 2;
    return e < h ? __ldg(tw + e) : fsub(0, __ldg(tw + (e - h)));
}

// In-place DIT DFT of `count` bit-reversed sequences of length m = 2^bits
// held in shared memory at s[r * pitch + i].  Twiddles of stage `len` are
// w_n^(k n / len).
template <class Ops>
__device__ __forceinline__ void smem_dft(typename Ops::T* s, int count, int pitch, int bits, const uint64_t* tw,
                                         size_t n) {
    const int m = 1 << bits, half_m = m >> 1;
    for (int sb = 1; sb <= bits; ++sb) {
        const int half = 1 << (sb - 1);
        const size_t step = n >> sb;
        for (int b = threadIdx.x; b < count * half_m; b += blockDim.x) {
            const int r = b / half_m, i = b - r * half_m;
            const int k = i & (half - 1), group = i >> (sb - 1);
            const int i0 = r * pitch + (group << sb) + k, i1 = i0 + half;
            const typename Ops::T u = s[i0];
            const typename Ops::T v = Ops::mulb(s[i1], __ldg(tw + k * step));
            s[i0] = Ops::add(u, v);
            s[i1] = Ops::sub(u, v);
        }
        __syncthreads();
    }
}

// Whole rows in shared memory: `rpc` rows of n = 2^bits per CTA.
template <class Ops>
__global__ void __launch_bounds__(kNttThreads) ntt_small_kernel(const typename Ops::T* in, typename Ops::T* out,
                                                                 size_t rows, int bits, int rpc,
                                                                 const uint64_t* tw) {
    using T = typename Ops::T;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* s = reinterpret_cast<T*>(smem_raw);
    const int n = 1 << bits;
    const size_t row0 = static_cast<size_t>(blockIdx.x) * rpc;
    const int nrows = static_cast<int>(rows - row0 < static_cast<size_t>(rpc) ? rows - row0 : rpc);
    const int pitch = n;
    for (int idx = threadIdx.x; idx < nrows * n; idx += blockDim.x) {
        const int r = idx >> bits, i = idx & (n - 1);
        s[r * pitch + brev_bits(i, bits)] = in[(row0 + r) * n + i];
    }
    __syncthreads();
    smem_dft<Ops>(s, nrows, pitch, bits, tw, n);
    for (int idx = threadIdx.x; idx < nrows * n; idx += blockDim.x) out[row0 * n + idx] = s[idx];
}

// Six-step pass 1: column DFTs of length n1 (stride n2) for T adjacent
// columns, times w^(j2 k1), stored transposed as Y[row][k1][j2].
template <class Ops>
__global__ void __launch_bounds__(kNttThreads) ntt_cols_kernel(const typename Ops::T* in, typename Ops::T* y,
                                                                int bits1, int bits2, int tcols,
                                                                const uint64_t* tw) {
    using T = typename Ops::T;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* s = reinterpret_cast<T*>(smem_raw);
    const int n1 = 1 << bits1, n2 = 1 << bits2;
    const size_t n = size_t{1} << (bits1 + bits2);
    const int tiles = n2 / tcols;
    const size_t row = blockIdx.x / tiles;
    const int j20 = (blockIdx.x - row * tiles) * tcols;
    const int pitch = n1 + 1;
    const T* src = in + row * n;
    for (int idx = threadIdx.x; idx < n1 * tcols; idx += blockDim.x) {
        const int j1 = idx / tcols, t = idx - j1 * tcols;
        s[t * pitch + brev_bits(j1, bits1)] = src[static_cast<size_t>(j1) * n2 + j20 + t];
    }
    __syncthreads();
    smem_dft<Ops>(s, tcols, pitch, bits1, tw, n);
    T* dst = y + row * n;
    for (int idx = threadIdx.x; idx < n1 * tcols; idx += blockDim.x) {
        const int k1 = idx / tcols, t = idx - k1 * tcols;
        const size_t e = (static_cast<size_t>(j20 + t) * k1) & (n - 1);
        dst[static_cast<size_t>(k1) * n2 + j20 + t] = Ops::mulb(s[t * pitch + k1], tw_at(tw, e, n));
    }
}

// Six-step pass 2: row DFTs of length n2 over Y[row][k1][*] for T adjacent
// k1, stored as X[row][k1 + n1 k2].
template <class Ops>
__global__ void __launch_bounds__(kNttThreads) ntt_rows_kernel(const typename Ops::T* y, typename Ops::T* out,
                                                                int bits1, int bits2, int trows,
                                                                const uint64_t* tw) {
    using T = typename Ops::T;
    extern __shared__ __align__(16) unsigned char smem_raw[];
    T* s = reinterpret_cast<T*>(smem_raw);
    const int n1 = 1 << bits1, n2 = 1 << bits2;
    const size_t n = size_t{1} << (bits1 + bits2);
    const int tiles = n1 / trows;
    const size_t row = blockIdx.x / tiles;
    const int k10 = (blockIdx.x - row * tiles) * trows;
    const int pitch = n2 + 1;
    const T* src = y + row * n + static_cast<size_t>(k10) * n2;
    for (int idx = threadIdx.x; idx < n2 * trows; idx += blockDim.x) {
        const int t = idx >> bits2, j2 = idx & (n2 - 1);
        s[t * pitch + brev_bits(j2, bits2)] = src[idx];
    }
    __syncthreads();
    smem_dft<Ops>(s, trows, pitch, bits2, tw, n);
    T* dst = out + row * n;
    for (int idx = threadIdx.x; idx < n2 * trows; idx += blockDim.x) {
        const int k2 = idx / trows, t = idx - k2 * trows;
        dst[k10 + t + static_cast<size_t>(n1) * k2] = s[t * pitch + k2];
    }
}

// Fallback for n > 2^22: bit reversal, then one launch per stage.
template <class T>
__global__ void bitrev_kernel(const T* in, T* out, size_t rows, int bits) {
    const size_t n = size_t{1} << bits, total = rows * n;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = z >> bits, i = z & (n - 1);
        out[(r << bits) + (__brevll(i) >> (64 - bits))] = in[z];
    }
}

template <class Ops>
__global__ void stage_kernel(typename Ops::T* v, size_t rows, int bits, int sb, const uint64_t* tw) {
    const size_t n = size_t{1} << bits, per_row = n / 2, total = rows * per_row;
    const size_t half = size_t{1} << (sb - 1), step = n >> sb;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = z / per_row, i = z - r * per_row;
        const size_t k = i & (half - 1), group = i >> (sb - 1);
        const size_t i0 = r * n + (group << sb) + k, i1 = i0 + half;
        const typename Ops::T u = v[i0];
        const typename Ops::T w = Ops::mulb(v[i1], __ldg(tw + k * step));
        v[i0] = Ops::add(u, w);
        v[i1] = Ops::sub(u, w);
    }
}

__global__ void twiddle_kernel(uint64_t* tw, size_t count, uint64_t w) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        tw[i] = fpow(w, i);
}

int ensure_twiddles(Context* c, size_t n) {
    if (ensure_ws(c, kWsTwiddles, (n / 2) * sizeof(uint64_t))) return -1;
    if (c->twiddle_n == n) return 0;
    int bits = 0;
    while ((size_t{1} << bits) < n) ++bits;
    const uint64_t w = fpow(7, (kP - 1) >> bits);
    twiddle_kernel<<<grid_for(c, n / 2, 256), 256, 0, c->stream>>>(ws<uint64_t>(c, kWsTwiddles), n / 2, w);
    VZB_LAUNCHED(c);
    c->twiddle_n = n;
    return 0;
}

template <class Ops, int RA, int RB, bool kCols>
int launch_pass_rr(Context* c, const typename Ops::T* in, typename Ops::T* out, int bits1, int bits2, size_t rows,
                   const uint64_t* tw) {
    using T = typename Ops::T;
    constexpr int kPitchSeq = RB * (RA + 1) + 1;
    const size_t smem = 16 * kPitchSeq * sizeof(T) + RA * RB * sizeof(uint64_t);
    auto k = ntt_pass_kernel<Ops, RA, RB, kCols>;
    VZB_CUDA(c, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    const size_t tiles = (size_t{1} << (kCols ? bits2 : bits1)) / 16;
    k<<<static_cast<unsigned>(rows * tiles), 16 * (RA > RB ? RA : RB), smem, c->stream>>>(in, out, bits1, bits2, tw);
    VZB_LAUNCHED(c);
    return 0;
}

// Sequence length 2^len_bits (6..8) split into register radices RA x RB.
template <class Ops, bool kCols>
int launch_pass(Context* c, const typename Ops::T* in, typename Ops::T* out, int bits1, int bits2, size_t rows,
                int len_bits, const uint64_t* tw) {
    switch (len_bits) {
        case 6: return launch_pass_rr<Ops, 8, 8, kCols>(c, in, out, bits1, bits2, rows, tw);
        case 7: return launch_pass_rr<Ops, 16, 8, kCols>(c, in, out, bits1, bits2, rows, tw);
        case 8: return launch_pass_rr<Ops, 16, 16, kCols>(c, in, out, bits1, bits2, rows, tw);
        default: return fail_message(c, "internal: unsupported NTT pass length");
    }
}

template <class Ops>
int launch_ntt(Context* c, const typename Ops::T* in, typename Ops::T* out, size_t rows, size_t n) {
    using T = typename Ops::T;
    int bits = 0;
    while ((size_t{1} << bits) < n) ++bits;
    if (ensure_twiddles(c, n)) return -1;
    const uint64_t* tw = ws<uint64_t>(c, kWsTwiddles);
    if (bits <= kSmallMaxBits) {
        const int rpc = n >= 1024 ? 1 : static_cast<int>(1024 / n);
        const size_t smem = static_cast<size_t>(rpc) * n * sizeof(T);
        const size_t blocks = (rows + rpc - 1) / rpc;
        auto k = ntt_small_kernel<Ops>;
        VZB_CUDA(c, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
        for (size_t b0 = 0; b0 < blocks; b0 += 0x7fffffff) {
            const size_t nb = blocks - b0 < 0x7fffffff ? blocks - b0 : 0x7fffffff;
            const size_t r0 = b0 * rpc;
            k<<<static_cast<unsigned>(nb), kNttThreads, smem, c->stream>>>(in + r0 * n, out + r0 * n, rows - r0,
                                                                           bits, rpc, tw);
            VZB_LAUNCHED(c);
        }
        return 0;
    }
    if (bits >= 12 && bits <= 16) {
        // register six-step: n1 = 2^ceil(bits/2), n2 = 2^floor(bits/2), each 64..256
        const int bits2 = bits / 2, bits1 = bits - bits2;
        size_t chunk = kNttChunkBytes / (n * sizeof(T));
        if (chunk < 1) chunk = 1;
        if (chunk > rows) chunk = rows;
        if (ensure_ws(c, kWsScratch2, chunk * n * sizeof(T))) return -1;
        T* y = ws<T>(c, kWsScratch2);
        for (size_t r0 = 0; r0 < rows; r0 += chunk) {
            const size_t nr = rows - r0 < chunk ? rows - r0 : chunk;
            if (launch_pass<Ops, true>(c, in + r0 * n, y, bits1, bits2, nr, bits1, tw)) return -1;
            if (launch_pass<Ops, false>(c, y, out + r0 * n, bits1, bits2, nr, bits2, tw)) return -1;
        }
        return 0;
    }
    if (bits <= 2 * kSmallMaxBits) {
        const int bits2 = bits / 2, bits1 = bits - bits2;  // n1 >= n2
        const int n1 = 1 << bits1, n2 = 1 << bits2;
        auto tile = [](int len) {  // adjacent sequences per CTA: <= 64 KB of shared memory
            int t = 16;
            while (t > 1 && static_cast<size_t>(t) * (len + 1) * sizeof(T) > (size_t{64} << 10)) t >>= 1;
            return t;
        };
        const int tc = tile(n1) < n2 ? tile(n1) : n2, tr = tile(n2) < n1 ? tile(n2) : n1;
        const size_t smem1 = static_cast<size_t>(tc) * (n1 + 1) * sizeof(T);
        const size_t smem2 = static_cast<size_t>(tr) * (n2 + 1) * sizeof(T);
        auto k1 = ntt_cols_kernel<Ops>;
        auto k2 = ntt_rows_kernel<Ops>;
        VZB_CUDA(c, cudaFuncSetAttribute(k1, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem1)));
        VZB_CUDA(c, cudaFuncSetAttribute(k2, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem2)));
        size_t chunk = kNttChunkBytes / (n * sizeof(T));
        if (chunk < 1) chunk = 1;
        if (chunk > rows) chunk = rows;
        if (ensure_ws(c, kWsScratch2, chunk * n * sizeof(T))) return -1;
        T* y = ws<T>(c, kWsScratch2);
        for (size_t r0 = 0; r0 < rows; r0 += chunk) {
            const size_t nr = rows - r0 < chunk ? rows - r0 : chunk;
            k1<<<static_cast<unsigned>(nr * (n2 / tc)), kNttThreads, smem1, c->stream>>>(in + r0 * n, y, bits1,
                                                                                        bits2, tc, tw);
            VZB_LAUNCHED(c);
            k2<<<static_cast<unsigned>(nr * (n1 / tr)), kNttThreads, smem2, c->stream>>>(y, out + r0 * n, bits1,
                                                                                        bits2, tr, tw);
            VZB_LAUNCHED(c);
        }
        return 0;
    }
    // very long rows: out-of-place bit reversal (through scratch when in place)
    T* dst = out;
    if (in == out) {
        if (ensure_ws(c, kWsScratch2, rows * n * sizeof(T))) return -1;
        VZB_CUDA(c, cudaMemcpyAsync(ws<T>(c, kWsScratch2), in, rows * n * sizeof(T), cudaMemcpyDeviceToDevice,
                                    c->stream));
        in = ws<T>(c, kWsScratch2);
    }
    bitrev_kernel<T><<<grid_for(c, rows * n, 256), 256, 0, c->stream>>>(in, dst, rows, bits);
    VZB_LAUNCHED(c);
    for (int sb = 1; sb <= bits; ++sb) {
        stage_kernel<Ops><<<grid_for(c, rows * n / 2, 256), 256, 0, c->stream>>>(dst, rows, bits, sb, tw);
        VZB_LAUNCHED(c);
    }
    return 0;
}

bool pow2(size_t n) { return n && !(n & (n - 1)); }

// Hybrid rows: upload `rows` messages of msg_len into zero-padded rows of n.
template <class T>
int stage_padded(Context* c, int slot, const T* host, size_t rows, size_t msg_len, size_t n, uint64_t* h2d) {
    if (ensure_ws(c, slot, rows * n * sizeof(T))) return -1;
    T* d = ws<T>(c, slot);
    if (msg_len < n) VZB_CUDA(c, cudaMemsetAsync(d, 0, rows * n * sizeof(T), c->stream));
    if (msg_len)
        VZB_CUDA(c, cudaMemcpy2DAsync(d, n * sizeof(T), host, msg_len * sizeof(T), msg_len * sizeof(T), rows,
                                      cudaMemcpyHostToDevice, c->stream));
    *h2d += rows * msg_len * sizeof(T);
    return 0;
}

template <class Ops>
int ntt_hybrid(Context* c, const typename Ops::T* msg, size_t rows, size_t msg_len, size_t n,
               typename Ops::T* out) {
    using T = typename Ops::T;
    uint64_t h2d = 0;
    if (ensure_ws(c, kWsStageB, rows * n * sizeof(T))) return -1;
    if (op_begin(c)) return -1;
    if (stage_padded<T>(c, kWsStageA, msg, rows, msg_len, n, &h2d)) return -1;
    if (op_mark(c, 1)) return -1;
    if (launch_ntt<Ops>(c, ws<T>(c, kWsStageA), ws<T>(c, kWsStageB), rows, n)) return -1;
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(out, ws<T>(c, kWsStageB), rows * n * sizeof(T), cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpPcsNtt, h2d, rows * n * sizeof(T));
}

template <class Ops>
int ntt_device(Context* c, uint64_t in_id, size_t in_off, size_t rows, size_t n, uint64_t out_id, size_t out_off,
               const char* what) {
    using T = typename Ops::T;
    if (!c || !rows || n < 2 || !pow2(n)) return fail_message(c, what);
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, rows * n, sizeof(T), &in) ||
        region_elems(c, out_id, out_off, rows * n, sizeof(T), &out))
        return -1;
    const char* a = static_cast<const char*>(in);
    const char* b = static_cast<const char*>(out);
    const size_t bytes = rows * n * sizeof(T);
    if (a != b && a < b + bytes && b < a + bytes) return fail_message(c, "NTT input and output overlap partially");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (launch_ntt<Ops>(c, static_cast<const T*>(in), static_cast<T*>(out), rows, n)) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsNtt, 0, 0);
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_ntt_fp(void* raw, const uint64_t* msg, size_t msg_len, size_t n, uint64_t* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || (!msg && msg_len) || !out || n < 2 || !pow2(n) || msg_len > n) return -1;
    return ntt_hybrid<FpOps>(c, msg, 1, msg_len, n, out);
}

extern "C" int volta_cuda_ntt_fp_batch(void* raw, const uint64_t* messages, size_t rows, size_t msg_len, size_t n,
                                       uint64_t* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || (!messages && msg_len) || !out || !rows || n < 2 || !pow2(n) || msg_len > n) return -1;
    return ntt_hybrid<FpOps>(c, messages, rows, msg_len, n, out);
}

extern "C" int volta_cuda_ntt_fp2(void* raw, const Fp2* msg, size_t msg_len, size_t n, Fp2* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || (!msg && msg_len) || !out || n < 2 || !pow2(n) || msg_len > n) return -1;
    return ntt_hybrid<Fp2Ops>(c, msg, 1, msg_len, n, out);
}

extern "C" int volta_cuda_ntt_fp_batch_device(void* raw, uint64_t input_id, size_t input_offset, size_t rows,
                                              size_t n, uint64_t output_id, size_t output_offset) {
    return ntt_device<FpOps>(static_cast<Context*>(raw), input_id, input_offset, rows, n, output_id, output_offset,
                             "invalid resident Fp NTT geometry");
}

extern "C" int volta_cuda_ntt_fp2_batch_device(void* raw, uint64_t input_id, size_t input_offset, size_t rows,
                                               size_t n, uint64_t output_id, size_t output_offset) {
    return ntt_device<Fp2Ops>(static_cast<Context*>(raw), input_id, input_offset, rows, n, output_id,
                              output_offset, "invalid resident Fp2 NTT geometry");
}
