// ChaCha8 FpStream expansion (prover-secret PCS pads, mock-PCG sub masks,
// zero-knowledge Fp2 mask rows).
//
// Semantics: rust/volta-field/src/lib.rs:222-268 -- row r is
// FpStream::domain_separated(seed, base + r), i.e. rand_chacha 0.3.1's
// ChaCha8Rng with stream id base + r, read as little-endian u64 words with
// values >= p rejected.  Reference entry points:
// cuda/volta_cuda_backend.cu:3955-4047 (one thread per row, serial).
//
// B200 design: one thread per 64-byte ChaCha block, so a row of 16384
// values is spread over 2048 threads.  Rejection (probability ~2^-32 per
// draw) shifts every later value of its row, so the block-parallel pass
// writes values assuming no rejection and flags any row where a draw was
// >= p; a second pass recomputes only flagged rows serially.  The fast pass
// is exact for every row it does not flag.
#include "runtime.cuh"

namespace vzb {

struct ChachaKey {
    uint32_t w[8];
};

__device__ __forceinline__ uint32_t rotl32(uint32_t x, int n) { return __funnelshift_l(x, x, n); }

#define VZB_QR(a, b, c, d)              \
    a += b; d = rotl32(d ^ a, 16);      \
    c += d; b = rotl32(b ^ c, 12);      \
    a += b; d = rotl32(d ^ a, 8);       \
    c += d; b = rotl32(b ^ c, 7);

// ChaCha8 block: constants | key | counter (64-bit) | stream (64-bit).
__device__ __forceinline__ void chacha8_block(const ChachaKey& k, uint64_t stream, uint64_t counter,
                                              uint32_t out[16]) {
    uint32_t x[16] = {0x61707865u, 0x3320646eu, 0x79622d32u, 0x6b206574u,
                      k.w[0], k.w[1], k.w[2], k.w[3], k.w[4], k.w[5], k.w[6], k.w[7],
                      static_cast<uint32_t>(counter), static_cast<uint32_t>(counter >> 32),
                      static_cast<uint32_t>(stream), static_cast<uint32_t>(stream >> 32)};
    uint32_t s[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) s[i] = x[i];
#pragma unroll
    for (int r = 0; r < 4; ++r) {
        VZB_QR(s[0], s[4], s[8], s[12]);
        VZB_QR(s[1], s[5], s[9], s[13]);
        VZB_QR(s[2], s[6], s[10], s[14]);
        VZB_QR(s[3], s[7], s[11], s[15]);
        VZB_QR(s[0], s[5], s[10], s[15]);
        VZB_QR(s[1], s[6], s[11], s[12]);
        VZB_QR(s[2], s[7], s[8], s[13]);
        VZB_QR(s[3], s[4], s[9], s[14]);
    }
#pragma unroll
    for (int i = 0; i < 16; ++i) out[i] = s[i] + x[i];
}

// Sequential reference path for one row (used only for flagged rows).
struct SerialStream {
    ChachaKey key;
    uint64_t stream, counter;
    uint32_t words[16];
    int idx;
    __device__ SerialStream(const ChachaKey& k, uint64_t s) : key(k), stream(s), counter(0), idx(8) {}
    __device__ uint64_t next_u64() {
        if (idx == 8) {
            chacha8_block(key, stream, counter++, words);
            idx = 0;
        }
        const uint64_t v = static_cast<uint64_t>(words[2 * idx]) | (static_cast<uint64_t>(words[2 * idx + 1]) << 32);
        ++idx;
        return v;
    }
    __device__ uint64_t next_fp() {
        for (;;) {
            const uint64_t v = next_u64();
            if (v < kP) return v;
        }
    }
};

// Row layout: `draws` accepted values per row written as u64 words at
// out[row * row_words + j] for j < draws (Fp2 rows are the same words: c0, c1
// interleaved), padding words [draws, row_words) are zeroed.
__global__ void __launch_bounds__(256) chacha_rows_fast_kernel(ChachaKey key, uint64_t base,
                                                               size_t rows, size_t draws,
                                                               size_t row_words, uint64_t* out,
                                                               uint8_t* flags) {
    const size_t blocks_per_row = (draws + 7) / 8;
    const size_t pad_words = row_words - draws;
    const size_t pad_blocks = (pad_words + 7) / 8;
    const size_t per_row = blocks_per_row + pad_blocks;
    const size_t total = rows * per_row;
    const size_t gs = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t t = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < total; t += gs) {
        const size_t row = t / per_row, b = t - row * per_row;
        uint64_t* dst = out + row * row_words;
        if (b >= blocks_per_row) {  // zero padding
            const size_t j0 = draws + (b - blocks_per_row) * 8;
            for (size_t j = j0; j < j0 + 8 && j < row_words; ++j) dst[j] = 0;
            continue;
        }
        uint32_t w[16];
        chacha8_block(key, base + row, b, w);
        bool reject = false;
        const size_t j0 = b * 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint64_t v = static_cast<uint64_t>(w[2 * i]) | (static_cast<uint64_t>(w[2 * i + 1]) << 32);
            const size_t j = j0 + i;
            if (j < draws) {
                reject |= v >= kP;
                dst[j] = v;
            }
        }
        if (reject) flags[row] = 1;
    }
}

__global__ void chacha_rows_fixup_kernel(ChachaKey key, uint64_t base, size_t rows, size_t draws,
                                         size_t row_words, uint64_t* out, const uint8_t* flags) {
    const size_t gs = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t row = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; row < rows; row += gs) {
        if (!flags[row]) continue;
        SerialStream s(key, base + row);
        uint64_t* dst = out + row * row_words;
        for (size_t j = 0; j < draws; ++j) dst[j] = s.next_fp();
    }
}

static ChachaKey key_from(const uint8_t* seed) {
    ChachaKey k{};
    for (int i = 0; i < 8; ++i)
        k.w[i] = static_cast<uint32_t>(seed[4 * i]) | (static_cast<uint32_t>(seed[4 * i + 1]) << 8) |
                 (static_cast<uint32_t>(seed[4 * i + 2]) << 16) | (static_cast<uint32_t>(seed[4 * i + 3]) << 24);
    return k;
}

int chacha_rows(Context* c, const uint8_t* seed, uint64_t base, size_t rows, size_t draws,
                size_t row_words, uint64_t* out) {
    if (ensure_ws(c, kWsScratch2, rows)) return -1;
    uint8_t* flags = ws<uint8_t>(c, kWsScratch2);
    VZB_CUDA(c, cudaMemsetAsync(flags, 0, rows, c->stream));
    const ChachaKey key = key_from(seed);
    const size_t per_row = (draws + 7) / 8 + (row_words - draws + 7) / 8;
    chacha_rows_fast_kernel<<<grid_for(c, rows * per_row, 256), 256, 0, c->stream>>>(
        key, base, rows, draws, row_words, out, flags);
    VZB_LAUNCHED(c);
    chacha_rows_fixup_kernel<<<grid_for(c, rows, 128, 2), 128, 0, c->stream>>>(key, base, rows, draws,
                                                                             row_words, out, flags);
    VZB_LAUNCHED(c);
    return 0;
}

static int fp_rows_impl(Context* c, uint64_t out_id, size_t out_off_bytes, const uint8_t* seed,
                        uint64_t base, size_t rows, size_t count, int op) {
    if (!c || !seed || !rows || !count) return fail_message(c, "invalid ChaCha8 Fp row generation");
    if (rows - 1 > UINT64_MAX - base) return fail_message(c, "ChaCha8 Fp row domain overflows u64");
    const uint64_t last = base + static_cast<uint64_t>(rows - 1);
    if (op == kOpAuthMasks && ((base | last) & kMockReservedDomainBits))
        return fail_message(c, "mock correlation mask domain sets reserved correlation bits");
    size_t elems = 0, bytes = 0;
    if (!mul_ok(rows, count, &elems) || !mul_ok(elems, sizeof(uint64_t), &bytes))
        return fail_message(c, "ChaCha8 Fp row geometry overflows size_t");
    void* out = nullptr;
    if (region(c, out_id, out_off_bytes, bytes, &out)) return -1;
    if ((reinterpret_cast<uintptr_t>(out) & 7) != 0)
        return fail_message(c, "ChaCha8 Fp rows must be 8-byte aligned");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (chacha_rows(c, seed, base, rows, count, count, static_cast<uint64_t*>(out))) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, op, 0, 0, 0, 0, bytes);
}

}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_chacha8_prover_secret_fp_rows_device(void* raw, uint64_t out_id,
                                                               size_t out_off_bytes,
                                                               const uint8_t* seed, uint64_t base,
                                                               size_t rows, size_t count) {
    return fp_rows_impl(static_cast<Context*>(raw), out_id, out_off_bytes, seed, base, rows, count,
                        kOpPcsRows);
}

extern "C" int volta_cuda_mock_correlation_sub_masks_device(void* raw, uint64_t out_id,
                                                            size_t out_off_bytes,
                                                            const uint8_t* seed, uint64_t base,
                                                            size_t rows, size_t cols) {
    return fp_rows_impl(static_cast<Context*>(raw), out_id, out_off_bytes, seed, base, rows, cols,
                        kOpAuthMasks);
}

extern "C" int volta_cuda_chacha8_prover_secret_fp2_rows_padded_device(
    void* raw, uint64_t out_id, size_t out_off_bytes, const uint8_t* seed, uint64_t base,
    size_t rows, size_t count, size_t padded) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !seed || !rows || !count || padded < count)
        return fail_message(c, "invalid ChaCha8 Fp2 row generation");
    if (rows - 1 > UINT64_MAX - base) return fail_message(c, "ChaCha8 Fp2 row domain overflows u64");
    size_t elems = 0, bytes = 0, generated = 0;
    if (!mul_ok(rows, padded, &elems) || !mul_ok(elems, sizeof(Fp2), &bytes) ||
        !mul_ok(rows, count * sizeof(Fp2), &generated))
        return fail_message(c, "ChaCha8 Fp2 row geometry overflows size_t");
    void* out = nullptr;
    if (region(c, out_id, out_off_bytes, bytes, &out)) return -1;
    if ((reinterpret_cast<uintptr_t>(out) & 7) != 0)
        return fail_message(c, "ChaCha8 Fp2 rows must be 8-byte aligned");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (chacha_rows(c, seed, base, rows, 2 * count, 2 * padded, static_cast<uint64_t*>(out))) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0, 0, bytes - generated, generated);
}
