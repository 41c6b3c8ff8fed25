// Lookup-column preparation, subfield corrections, padding, broadcasts and
// matrix folds (MLE evaluation of GEMM operand tables along one axis).
//
// Reference entry points (okrame/volta-zk cuda/volta_cuda_backend.cu):
//   subfield_corrections / pad_base_vector / matrix_fold     4612-4713
//   ln_hadamard_factors / base_broadcast / repeat / compact  5155-5253
//   attention_above_mask                                     5254-5276
//   requant_columns / pair_columns / histograms / u32 add /
//   pack_lookup_leaf / deinterleave_base_columns             5378-5532
// Kernels 1924-2039, 2174-2215, 2455-2580.  Scalar kinds: 0 i16, 1 i64,
// 2 canonical Fp, 3 Fp2, 4 u32.
#include <algorithm>

#include "reduce.cuh"
#include "runtime.cuh"

namespace vzb {

enum Kind : int { kI16 = 0, kI64 = 1, kFp = 2, kFp2 = 3, kU32 = 4 };

inline size_t kind_size(int kind) {
    switch (kind) {
        case kI16: return 2;
        case kU32: return 4;
        case kI64:
        case kFp: return 8;
        case kFp2: return 16;
        default: return 0;
    }
}

__device__ __forceinline__ uint64_t load_base(const void* in, size_t i, int kind) {
    switch (kind) {
        case kI16: return ffrom_i64(static_cast<const int16_t*>(in)[i]);
        case kI64: return ffrom_i64(static_cast<const int64_t*>(in)[i]);
        case kU32: return static_cast<const uint32_t*>(in)[i];
        default: return static_cast<const uint64_t*>(in)[i];
    }
}

#define VZB_GRID_LOOP(i, n)                                                                  \
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < (n);     \
         i += static_cast<size_t>(gridDim.x) * blockDim.x)

__global__ void subfield_corr_kernel(const void* in, const uint64_t* masks, uint64_t* out, size_t n,
                                     int kind) {
    VZB_GRID_LOOP(i, n) out[i] = fsub(load_base(in, i, kind), masks[i]);
}

__global__ void pad_base_kernel(const void* in, uint64_t* out, size_t real, size_t padded, uint64_t pad,
                                int kind) {
    VZB_GRID_LOOP(i, padded) out[i] = i < real ? load_base(in, i, kind) : pad;
}

__global__ void broadcast_kernel(const void* in, Fp2* out, size_t repeat, size_t out_len, int kind) {
    VZB_GRID_LOOP(i, out_len) st2(out + i, Fp2{load_base(in, i / repeat, kind), 0});
}

__global__ void ln_factors_kernel(const int16_t* in, const uint64_t* means, const uint64_t* rsqrt,
                                  const int16_t* gain, Fp2* centered, Fp2* scaled, size_t rows,
                                  size_t cols, size_t row_pad, size_t col_pad) {
    VZB_GRID_LOOP(z, row_pad * col_pad) {
        const size_t row = z / col_pad, col = z - row * col_pad;
        Fp2 cv{0, 0};
        if (row < rows) cv = Fp2{fsub(col < cols ? ffrom_i64(in[row * cols + col]) : 0, means[row]), 0};
        st2(centered + z, cv);
        st2(scaled + z, col < cols ? Fp2{fmul(rsqrt[row], ffrom_i64(gain[col])), 0} : Fp2{0, 0});
    }
}

__global__ void above_mask_kernel(Fp2* eq, size_t entries, size_t rows, size_t seq, size_t pos0,
                                  size_t heads, size_t query_pad, size_t seq_pad) {
    const size_t sp2 = query_pad * seq_pad;
    VZB_GRID_LOOP(z, entries) {
        const size_t head = z / sp2, rem = z - head * sp2;
        const size_t row = rem / seq_pad, col = rem - row * seq_pad;
        if (head >= heads || row >= rows || col >= seq || col < pos0 + row + 1) st2(eq + z, Fp2{0, 0});
    }
}

__device__ __forceinline__ int64_t round_stage(int64_t v, uint32_t shift) {
    return (v + (int64_t{1} << (shift - 1))) >> shift;
}

// Requant witness columns (layer.rs:103-115): rem = acc + 2^(s-1) - y 2^s in
// [0, 2^s); shifts above 16 are chained through an intermediate y1.
__global__ void requant_columns_kernel(const void* acc_in, const int16_t* outs, uint64_t* cols_out,
                                       uint32_t* error, size_t rows, size_t cols, size_t row_pad,
                                       size_t col_pad, int acc_kind, uint32_t shift) {
    const size_t padded = row_pad * col_pad;
    VZB_GRID_LOOP(z, padded) {
        const size_t row = z / col_pad, col = z - row * col_pad;
        const bool real = row < rows && col < cols;
        int64_t acc = 0, out = 0;
        if (real) {
            acc = acc_kind == kI16 ? static_cast<const int16_t*>(acc_in)[row * cols + col]
                                   : static_cast<const int64_t*>(acc_in)[row * cols + col];
            out = outs[row * cols + col];
        }
        if (shift <= 16) {
            const int64_t rem = acc + (int64_t{1} << (shift - 1)) - out * (int64_t{1} << shift);
            if (real && (rem < 0 || rem >= (int64_t{1} << shift) || round_stage(acc, shift) != out))
                atomicExch(error, 1u);
            cols_out[z] = static_cast<uint64_t>(rem);
            cols_out[padded + z] = ffrom_i64(out);
        } else {
            const uint32_t first = shift - 16;
            const int64_t y1 = round_stage(acc, first);
            const int64_t rem1 = acc + (int64_t{1} << (first - 1)) - y1 * (int64_t{1} << first);
            const int64_t rem2 = y1 + (int64_t{1} << 15) - out * (int64_t{1} << 16);
            if (real && (rem1 < 0 || rem1 >= (int64_t{1} << first) || rem2 < 0 ||
                         rem2 >= (int64_t{1} << 16) || round_stage(y1, 16) != out))
                atomicExch(error, 1u);
            cols_out[z] = static_cast<uint64_t>(rem1);
            cols_out[padded + z] = ffrom_i64(y1);
            cols_out[2 * padded + z] = static_cast<uint64_t>(rem2);
            cols_out[3 * padded + z] = ffrom_i64(out);
        }
    }
}

__global__ void pair_columns_kernel(const void* in, const void* outs, uint64_t* cols_out, size_t rows,
                                    size_t cols, size_t row_pad, size_t col_pad, uint64_t pad_in,
                                    uint64_t pad_out, int in_kind, int out_kind) {
    const size_t padded = row_pad * col_pad;
    VZB_GRID_LOOP(z, padded) {
        const size_t row = z / col_pad, col = z - row * col_pad;
        const bool real = row < rows && col < cols;
        cols_out[z] = real ? load_base(in, row * cols + col, in_kind) : pad_in;
        cols_out[padded + z] = real ? load_base(outs, row * cols + col, out_kind) : pad_out;
    }
}

// Multiplicity histograms.  Lookup columns are dominated by a few values
// (every pad entry holds the same value, and remainders and table indices
// cluster), so one global atomic per element serialises on the hot bins.
// A warp whose 32 elements share one bin (a run of pads) adds them with one
// atomic; in other warps the lanes holding the same bin (softmax remainders
// of rows where most exp values underflow to 0, small table indices) add
// once with their count.  Tables of at most kSmemBins bins are
// counted in a per-block shared-memory copy that is added to the global
// table once per block (blocks are sized so that this flush stays small
// against the column).  Each warp walks 32 consecutive elements per step.
constexpr size_t kSmemBins = 16384;  // 64 KB of u32 counters

__device__ __forceinline__ uint32_t lut_bin(uint64_t v, int signed_input, bool& ok) {
    ok = true;
    if (!signed_input) {
        ok = v < (uint64_t{1} << 16);
        return static_cast<uint32_t>(v);
    }
    if (v <= 32767) return static_cast<uint32_t>(v);
    ok = v >= kP - (uint64_t{1} << 15);
    return static_cast<uint32_t>((uint64_t{1} << 16) - (kP - v));
}

// mode 0: bins = values below `bins`; mode 1: u16 table index (signed_input)
template <bool kShared>
__global__ void histogram_kernel(const uint64_t* in, uint32_t* out, size_t n, size_t bins, int mode,
                                 int signed_input) {
    extern __shared__ uint32_t sm_hist[];
    if (kShared) {
        for (size_t b = threadIdx.x; b < bins; b += blockDim.x) sm_hist[b] = 0;
        __syncthreads();
    }
    uint32_t* target = kShared ? sm_hist : out;
    const unsigned lane = threadIdx.x & 31;
    const size_t warp = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const size_t warps = (static_cast<size_t>(gridDim.x) * blockDim.x) >> 5;
    for (size_t base = warp * 32; base < n; base += warps * 32) {
        const size_t i = base + lane;
        bool ok = i < n;
        uint32_t bin = 0;
        if (ok) {
            const uint64_t v = __ldcs(in + i);
            if (mode == 0) {
                ok = v < bins;
                bin = static_cast<uint32_t>(v);
            } else {
                bin = lut_bin(v, signed_input, ok);
            }
        }
        const uint32_t first = __shfl_sync(0xffffffffu, bin, 0);
        const unsigned ok_mask = __ballot_sync(0xffffffffu, ok);
        if (__all_sync(0xffffffffu, ok && bin == first)) {
            if (lane == 0) atomicAdd(target + first, 32u);
        } else if (ok) {
            // lanes holding the same bin add once, with their count
            const unsigned peers = __match_any_sync(ok_mask, bin);
            if (lane == static_cast<unsigned>(__ffs(peers) - 1)) atomicAdd(target + bin, __popc(peers));
        }
    }
    if (kShared) {
        __syncthreads();
        for (size_t b = threadIdx.x; b < bins; b += blockDim.x)
            if (sm_hist[b]) atomicAdd(out + b, sm_hist[b]);
    }
}

// Tables of up to 2^16 bins (the u16 lookup tables and 16-bit ranges): two
// 16-bit counters per shared-memory word, 128 KB for 2^16 bins.  A CTA
// counts a contiguous slice of the column in chunks of kPackedChunk
// elements and adds its nonzero counters to the global table after each
// chunk, so no counter can pass 65535 and wrap.
constexpr size_t kPackedBins = size_t{1} << 16;
constexpr unsigned kPackedThreads = 1024;
constexpr size_t kPackedChunk = 63 * kPackedThreads;  // <= 65535 elements per flush

__global__ void __launch_bounds__(kPackedThreads) histogram_packed_kernel(const uint64_t* in, uint32_t* out, size_t n,
                                                                         size_t bins, int mode, int signed_input) {
    extern __shared__ uint32_t sm_pair[];
    const size_t words = (bins + 1) / 2;
    for (size_t w = threadIdx.x; w < words; w += blockDim.x) sm_pair[w] = 0;
    const size_t per = (n + gridDim.x - 1) / gridDim.x;
    const size_t begin = min(n, per * blockIdx.x), end = min(n, begin + per);
    const unsigned lane = threadIdx.x & 31;
    for (size_t chunk = begin; chunk < end; chunk += kPackedChunk) {
        __syncthreads();  // counters zeroed (first chunk) or flushed
        const size_t stop = min(end, chunk + kPackedChunk);
        for (size_t base = chunk + (threadIdx.x & ~31u); base < stop; base += blockDim.x) {
            const size_t i = base + lane;
            bool ok = i < stop;
            uint32_t bin = 0;
            if (ok) {
                const uint64_t v = __ldcs(in + i);
                if (mode == 0) {
                    ok = v < bins;
                    bin = static_cast<uint32_t>(v);
                } else {
                    bin = lut_bin(v, signed_input, ok);
                }
            }
            const uint32_t first = __shfl_sync(0xffffffffu, bin, 0);
            const unsigned ok_mask = __ballot_sync(0xffffffffu, ok);
            if (__all_sync(0xffffffffu, ok && bin == first)) {
                if (lane == 0) atomicAdd(sm_pair + (first >> 1), 32u << (16 * (first & 1)));
            } else if (ok) {
                const unsigned peers = __match_any_sync(ok_mask, bin);
                if (lane == static_cast<unsigned>(__ffs(peers) - 1))
                    atomicAdd(sm_pair + (bin >> 1), static_cast<uint32_t>(__popc(peers)) << (16 * (bin & 1)));
            }
        }
        __syncthreads();
        for (size_t w = threadIdx.x; w < words; w += blockDim.x) {
            const uint32_t v = sm_pair[w];
            if (!v) continue;
            sm_pair[w] = 0;
            if (v & 0xFFFFu) atomicAdd(out + 2 * w, v & 0xFFFFu);
            if (v >> 16) atomicAdd(out + 2 * w + 1, v >> 16);
        }
    }
}

int launch_histogram(Context* c, const uint64_t* in, uint32_t* out, size_t n, size_t bins, int mode,
                     int signed_input) {
    if (bins > kSmemBins && bins <= kPackedBins && n >= 4 * kPackedChunk) {
        // one CTA per SM (128 KB of counters), each a contiguous slice
        const size_t smem = (bins + 1) / 2 * sizeof(uint32_t);
        VZB_CUDA(c, cudaFuncSetAttribute(histogram_packed_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
        const unsigned blocks = static_cast<unsigned>(
            std::max<size_t>(1, std::min<size_t>(static_cast<size_t>(c->sm_count), n / kPackedChunk)));
        histogram_packed_kernel<<<blocks, kPackedThreads, smem, c->stream>>>(in, out, n, bins, mode, signed_input);
        VZB_LAUNCHED(c);
        return 0;
    }
    if (bins <= kSmemBins) {
        // one flush of `bins` atomics per block: at most one block per 8 x
        // bins elements, up to two 1024-thread blocks per SM
        const size_t want = n / (8 * bins);
        const unsigned blocks = static_cast<unsigned>(
            std::max<size_t>(1, std::min<size_t>(want, static_cast<size_t>(c->sm_count) * 2)));
        const size_t smem = bins * sizeof(uint32_t);
        if (smem > 48 * 1024)
            VZB_CUDA(c, cudaFuncSetAttribute(histogram_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem)));
        histogram_kernel<true><<<blocks, 1024, smem, c->stream>>>(in, out, n, bins, mode, signed_input);
    } else {
        histogram_kernel<false><<<grid_for(c, n, 256), 256, 0, c->stream>>>(in, out, n, bins, mode, signed_input);
    }
    VZB_LAUNCHED(c);
    return 0;
}

// out[i] = in[i % len] for elements of 2, 4, 8 or 16 bytes
template <typename T>
__global__ void repeat_kernel(const T* in, T* out, size_t len, size_t total) {
    VZB_GRID_LOOP(i, total) out[i] = in[i % len];
}

__global__ void u32_add_kernel(uint32_t* t, const uint32_t* a, size_t n) {
    VZB_GRID_LOOP(i, n) t[i] += a[i];
}

// leaf = alpha0 - sum_c col_c * 2^shift_c (shift == u32::MAX skips a column)
__global__ void pack_leaf_kernel(const uint64_t* cols, const uint32_t* shifts, uint64_t* leaf,
                                 size_t column_count, size_t n, uint64_t alpha0) {
    VZB_GRID_LOOP(i, n) {
        uint64_t packed = 0;
        for (size_t c = 0; c < column_count; ++c) {
            const uint32_t s = shifts[c];
            if (s != 0xFFFFFFFFu) packed = dadd(packed, dmul(cols[c * n + i], s < 64 ? (uint64_t{1} << s) : fpow(2, s)));
        }
        leaf[i] = dsub(alpha0, packed);
    }
}

// per column: evens then odds, lifted to Fp2
__global__ void deinterleave_base_kernel(const uint64_t* cols, Fp2* out, size_t column_count, size_t n) {
    const size_t half = n / 2;
    VZB_GRID_LOOP(z, column_count * n) {
        const size_t c = z / n, local = z - c * n;
        const size_t src = local < half ? 2 * local : 2 * (local - half) + 1;
        st2(out + z, Fp2{cols[c * n + src], 0});
    }
}

// ---- matrix folds -----------------------------------------------------------
// axis 0: out[j] = sum_t w[t] M[t*stride + off + j]   (columns, coalesced in j)
// axis 1: out[i] = sum_t w[t] M[i*stride + off + t]   (rows, coalesced in t)

__device__ __forceinline__ Fp2 fold_term(const void* in, size_t idx, int kind, Fp2 w) {
    if (kind == kFp2) return f2mul(w, ldg2(static_cast<const Fp2*>(in) + idx));
    const uint64_t v = load_base(in, idx, kind);
    return v ? f2mul_base(w, v) : Fp2{0, 0};
}

// block (32, 8): lanes own 32 consecutive outputs, warps split the terms of
// this block's term chunk; partial sums go to part[chunk * cols + j].
__global__ void __launch_bounds__(256) fold_axis0_kernel(const void* in, const Fp2* w, Fp2* part,
                                                         size_t rows, size_t stride, size_t off,
                                                         size_t cols, size_t chunk_terms, int kind) {
    __shared__ Fp2 sm[8][32];
    const size_t j = static_cast<size_t>(blockIdx.x) * 32 + threadIdx.x;
    const size_t t0 = static_cast<size_t>(blockIdx.y) * chunk_terms;
    const size_t t1 = min(rows, t0 + chunk_terms);
    Fp2 acc{0, 0};
    if (j < cols)
        for (size_t t = t0 + threadIdx.y; t < t1; t += 8)
            acc = f2add(acc, fold_term(in, t * stride + off + j, kind, ldg2(w + t)));
    sm[threadIdx.y][threadIdx.x] = acc;
    __syncthreads();
    if (threadIdx.y == 0 && j < cols) {
        Fp2 sum = sm[0][threadIdx.x];
        for (int k = 1; k < 8; ++k) sum = f2add(sum, sm[k][threadIdx.x]);
        part[static_cast<size_t>(blockIdx.y) * cols + j] = sum;
    }
}

// out[j] = sum over chunks of part[chunk * cols + j]; zero for j >= cols
__global__ void fold_finish_kernel(const Fp2* part, Fp2* out, size_t chunks, size_t cols, size_t out_pad) {
    VZB_GRID_LOOP(j, out_pad) {
        Fp2 s{0, 0};
        if (j < cols)
            for (size_t c = 0; c < chunks; ++c) s = f2add(s, ldg2(part + c * cols + j));
        st2(out + j, s);
    }
}

// one block per output row (grid-stride over rows), threads over terms
__global__ void __launch_bounds__(256) fold_axis1_kernel(const void* in, const Fp2* w, Fp2* out,
                                                         size_t rows, size_t stride, size_t off,
                                                         size_t cols, size_t out_pad, int kind) {
    for (size_t i = blockIdx.x; i < out_pad; i += gridDim.x) {
        Acc<1> acc;
        acc.zero();
        if (i < rows)
            for (size_t t = threadIdx.x; t < cols; t += blockDim.x)
                acc.v[0] = f2add(acc.v[0], fold_term(in, i * stride + off + t, kind, ldg2(w + t)));
        acc = block_sum<1>(acc);
        if (threadIdx.x == 0) out[i] = acc.v[0];
    }
}

}  // namespace vzb

using namespace vzb;

#define VZB_OP_BEGIN(c) \
    if (op_begin(c) || op_mark(c, 1)) return -1
#define VZB_OP_END(c, op) \
    VZB_LAUNCHED(c); \
    if (op_mark(c, 2)) return -1; \
    return op_finish(c, op, 0, 0)
// for primitives that enqueue a copy instead of a kernel
#define VZB_OP_END_COPY(c, op) \
    if (op_mark(c, 2)) return -1; \
    return op_finish(c, op, 0, 0)

extern "C" int volta_cuda_subfield_corrections_device(void* raw, uint64_t in_id, size_t in_off,
                                                      uint64_t m_id, size_t m_off, uint64_t out_id,
                                                      size_t out_off, size_t n, int kind) {
    Context* c = static_cast<Context*>(raw);
    const size_t e = kind_size(kind);
    if (!c || !n || !e || kind == kFp2) return fail_message(c, "invalid resident subfield-correction geometry");
    void *in = nullptr, *m = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, n, e, &in) || region_elems(c, m_id, m_off, n, 8, &m) ||
        region_elems(c, out_id, out_off, n, 8, &out))
        return -1;
    VZB_OP_BEGIN(c);
    subfield_corr_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(in, static_cast<const uint64_t*>(m),
                                                                     static_cast<uint64_t*>(out), n, kind);
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_pad_base_vector_device(void* raw, uint64_t in_id, size_t in_off, uint64_t out_id,
                                                 size_t out_off, size_t real, size_t padded, uint64_t pad,
                                                 int kind) {
    Context* c = static_cast<Context*>(raw);
    const size_t e = kind_size(kind);
    if (!c || !real || padded < real || (padded & (padded - 1)) || !e || kind == kFp2 || pad >= kP)
        return fail_message(c, "invalid resident base-vector padding geometry");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, real, e, &in) || region_elems(c, out_id, out_off, padded, 8, &out))
        return -1;
    VZB_OP_BEGIN(c);
    pad_base_kernel<<<grid_for(c, padded, 256), 256, 0, c->stream>>>(in, static_cast<uint64_t*>(out), real,
                                                                     padded, pad, kind);
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_matrix_fold_device(void* raw, uint64_t in_id, size_t in_off, uint64_t w_id,
                                             size_t w_off, uint64_t out_id, size_t out_off, size_t rows,
                                             size_t stride, size_t column_offset, size_t cols,
                                             size_t out_pad, int kind, int axis) {
    Context* c = static_cast<Context*>(raw);
    const size_t e = kind_size(kind);
    const size_t terms = axis == 0 ? rows : cols;
    const size_t real = axis == 0 ? cols : rows;
    if (!c || !rows || !stride || !cols || column_offset > stride || cols > stride - column_offset || !e ||
        (axis != 0 && axis != 1) || out_pad < real || (out_pad & (out_pad - 1)))
        return fail_message(c, "invalid resident matrix-window fold geometry");
    size_t n_in = 0;
    if (!mul_ok(rows, stride, &n_in)) return fail_message(c, "matrix fold geometry overflows size_t");
    void *in = nullptr, *w = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, n_in, e, &in) || region_elems(c, w_id, w_off, terms, sizeof(Fp2), &w) ||
        region_elems(c, out_id, out_off, out_pad, sizeof(Fp2), &out))
        return -1;
    size_t chunks = 1, chunk_terms = rows;
    if (axis == 0) {
        // enough blocks to cover every SM several times
        const size_t col_blocks = (cols + 31) / 32;
        const size_t want = static_cast<size_t>(c->sm_count) * 8;
        if (col_blocks < want) chunks = std::min<size_t>((want + col_blocks - 1) / col_blocks, (rows + 63) / 64);
        if (chunks < 1) chunks = 1;
        if (chunks > 65535) chunks = 65535;
        chunk_terms = (rows + chunks - 1) / chunks;
        chunks = (rows + chunk_terms - 1) / chunk_terms;
        if (ensure_ws(c, kWsScratch, chunks * cols * sizeof(Fp2))) return -1;
    }
    VZB_OP_BEGIN(c);
    if (axis == 0) {
        dim3 grid(static_cast<unsigned>((cols + 31) / 32), static_cast<unsigned>(chunks));
        fold_axis0_kernel<<<grid, dim3(32, 8), 0, c->stream>>>(in, static_cast<const Fp2*>(w),
                                                               ws<Fp2>(c, kWsScratch), rows, stride,
                                                               column_offset, cols, chunk_terms, kind);
        VZB_LAUNCHED(c);
        fold_finish_kernel<<<grid_for(c, out_pad, 256), 256, 0, c->stream>>>(ws<Fp2>(c, kWsScratch),
                                                                            static_cast<Fp2*>(out), chunks,
                                                                            cols, out_pad);
    } else {
        const unsigned blocks = static_cast<unsigned>(std::min<size_t>(out_pad, 65535));
        fold_axis1_kernel<<<blocks, 256, 0, c->stream>>>(in, static_cast<const Fp2*>(w), static_cast<Fp2*>(out),
                                                         rows, stride, column_offset, cols, out_pad, kind);
    }
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_ln_hadamard_factors_device(void* raw, uint64_t in_id, size_t in_off,
                                                     uint64_t mean_id, size_t mean_off, uint64_t rs_id,
                                                     size_t rs_off, uint64_t gain_id, size_t gain_off,
                                                     uint64_t cen_id, size_t cen_off, uint64_t sc_id,
                                                     size_t sc_off, size_t rows, size_t cols,
                                                     size_t row_pad, size_t col_pad) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !cols || row_pad < rows || col_pad < cols || (row_pad & (row_pad - 1)) ||
        (col_pad & (col_pad - 1)))
        return fail_message(c, "invalid resident LN Hadamard factor geometry");
    const size_t total = row_pad * col_pad;
    void *in = nullptr, *mean = nullptr, *rs = nullptr, *gain = nullptr, *cen = nullptr, *sc = nullptr;
    if (region_elems(c, in_id, in_off, rows * cols, 2, &in) || region_elems(c, mean_id, mean_off, row_pad, 8, &mean) ||
        region_elems(c, rs_id, rs_off, row_pad, 8, &rs) || region_elems(c, gain_id, gain_off, cols, 2, &gain) ||
        region_elems(c, cen_id, cen_off, total, sizeof(Fp2), &cen) ||
        region_elems(c, sc_id, sc_off, total, sizeof(Fp2), &sc))
        return -1;
    VZB_OP_BEGIN(c);
    ln_factors_kernel<<<grid_for(c, total, 256), 256, 0, c->stream>>>(
        static_cast<const int16_t*>(in), static_cast<const uint64_t*>(mean), static_cast<const uint64_t*>(rs),
        static_cast<const int16_t*>(gain), static_cast<Fp2*>(cen), static_cast<Fp2*>(sc), rows, cols, row_pad,
        col_pad);
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_base_broadcast_fp2_device(void* raw, uint64_t in_id, size_t in_off, uint64_t out_id,
                                                    size_t out_off, size_t input_len, size_t repeat, int kind) {
    Context* c = static_cast<Context*>(raw);
    const size_t e = kind_size(kind);
    if (!c || !input_len || !repeat || !e || kind == kFp2)
        return fail_message(c, "invalid resident base broadcast geometry");
    const size_t out_len = input_len * repeat;
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, input_len, e, &in) ||
        region_elems(c, out_id, out_off, out_len, sizeof(Fp2), &out))
        return -1;
    VZB_OP_BEGIN(c);
    broadcast_kernel<<<grid_for(c, out_len, 256), 256, 0, c->stream>>>(in, static_cast<Fp2*>(out), repeat,
                                                                      out_len, kind);
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_repeat_vector_device(void* raw, uint64_t in_id, size_t in_off, uint64_t out_id,
                                               size_t out_off, size_t input_len, size_t repeat, int kind) {
    Context* c = static_cast<Context*>(raw);
    const size_t e = kind_size(kind);
    if (!c || !input_len || !repeat || !e) return fail_message(c, "invalid resident vector repeat geometry");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, input_len, e, &in) ||
        region_elems(c, out_id, out_off, input_len * repeat, e, &out))
        return -1;
    const size_t total = input_len * repeat;
    VZB_OP_BEGIN(c);
    const unsigned grid = grid_for(c, total, 256);
    switch (e) {
        case 2: repeat_kernel<<<grid, 256, 0, c->stream>>>(static_cast<const uint16_t*>(in), static_cast<uint16_t*>(out), input_len, total); break;
        case 4: repeat_kernel<<<grid, 256, 0, c->stream>>>(static_cast<const uint32_t*>(in), static_cast<uint32_t*>(out), input_len, total); break;
        case 8: repeat_kernel<<<grid, 256, 0, c->stream>>>(static_cast<const uint64_t*>(in), static_cast<uint64_t*>(out), input_len, total); break;
        default: repeat_kernel<<<grid, 256, 0, c->stream>>>(static_cast<const ulonglong2*>(in), static_cast<ulonglong2*>(out), input_len, total); break;
    }
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_compact_strided_rows_device(void* raw, uint64_t in_id, size_t in_off,
                                                      uint64_t out_id, size_t out_off, size_t rows,
                                                      size_t source_stride, size_t width, int kind) {
    Context* c = static_cast<Context*>(raw);
    const size_t e = kind_size(kind);
    if (!c || !rows || !width || source_stride < width || !e)
        return fail_message(c, "invalid resident strided-copy geometry");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, (rows - 1) * source_stride + width, e, &in) ||
        region_elems(c, out_id, out_off, rows * width, e, &out))
        return -1;
    VZB_OP_BEGIN(c);
    VZB_CUDA(c, cudaMemcpy2DAsync(out, width * e, in, source_stride * e, width * e, rows,
                                  cudaMemcpyDeviceToDevice, c->stream));
    VZB_OP_END_COPY(c, kOpGemm);
}

extern "C" int volta_cuda_attention_above_mask_device(void* raw, uint64_t eq_id, size_t eq_off, size_t entries,
                                                      size_t rows, size_t seq, size_t pos0, size_t heads,
                                                      size_t head_pad, size_t query_pad, size_t seq_pad) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !entries || !rows || !seq || !heads || head_pad < heads || (head_pad & (head_pad - 1)) ||
        query_pad < rows || (query_pad & (query_pad - 1)) || seq_pad < seq || (seq_pad & (seq_pad - 1)) ||
        pos0 + rows != seq || entries != head_pad * query_pad * seq_pad)
        return fail_message(c, "invalid resident above-causal mask geometry");
    void* eq = nullptr;
    if (region_elems(c, eq_id, eq_off, entries, sizeof(Fp2), &eq)) return -1;
    VZB_OP_BEGIN(c);
    above_mask_kernel<<<grid_for(c, entries, 256), 256, 0, c->stream>>>(static_cast<Fp2*>(eq), entries, rows, seq,
                                                                       pos0, heads, query_pad, seq_pad);
    VZB_OP_END(c, kOpGemm);
}

extern "C" int volta_cuda_requant_columns_device(void* raw, uint64_t acc_id, size_t acc_off, uint64_t out_id,
                                                 size_t out_off, uint64_t col_id, size_t col_off,
                                                 uint64_t err_id, size_t err_off, size_t rows, size_t cols,
                                                 size_t row_pad, size_t col_pad, int acc_kind, uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    const size_t ae = kind_size(acc_kind);
    if (!c || !rows || !cols || row_pad < rows || col_pad < cols || (row_pad & (row_pad - 1)) ||
        (col_pad & (col_pad - 1)) || (acc_kind != kI16 && acc_kind != kI64) || !ae || !shift || shift >= 63)
        return fail_message(c, "invalid resident requant-column geometry");
    const size_t real = rows * cols, padded = row_pad * col_pad, count = shift > 16 ? 4 : 2;
    void *acc = nullptr, *out = nullptr, *col = nullptr, *err = nullptr;
    if (region_elems(c, acc_id, acc_off, real, ae, &acc) || region_elems(c, out_id, out_off, real, 2, &out) ||
        region_elems(c, col_id, col_off, count * padded, 8, &col) || region_elems(c, err_id, err_off, 1, 4, &err))
        return -1;
    VZB_OP_BEGIN(c);
    requant_columns_kernel<<<grid_for(c, padded, 256), 256, 0, c->stream>>>(
        acc, static_cast<const int16_t*>(out), static_cast<uint64_t*>(col), static_cast<uint32_t*>(err), rows,
        cols, row_pad, col_pad, acc_kind, shift);
    VZB_OP_END(c, kOpLogup);
}

extern "C" int volta_cuda_pair_columns_device(void* raw, uint64_t in_id, size_t in_off, uint64_t out_id,
                                              size_t out_off, uint64_t col_id, size_t col_off, size_t rows,
                                              size_t cols, size_t row_pad, size_t col_pad, uint64_t pad_in,
                                              uint64_t pad_out, int in_kind, int out_kind) {
    Context* c = static_cast<Context*>(raw);
    const size_t ie = kind_size(in_kind), oe = kind_size(out_kind);
    if (!c || !rows || !cols || row_pad < rows || col_pad < cols || (row_pad & (row_pad - 1)) ||
        (col_pad & (col_pad - 1)) || !ie || !oe || in_kind == kFp2 || out_kind == kFp2 || pad_in >= kP ||
        pad_out >= kP)
        return fail_message(c, "invalid resident pair-column geometry");
    const size_t real = rows * cols, padded = row_pad * col_pad;
    void *in = nullptr, *out = nullptr, *col = nullptr;
    if (region_elems(c, in_id, in_off, real, ie, &in) || region_elems(c, out_id, out_off, real, oe, &out) ||
        region_elems(c, col_id, col_off, 2 * padded, 8, &col))
        return -1;
    VZB_OP_BEGIN(c);
    pair_columns_kernel<<<grid_for(c, padded, 256), 256, 0, c->stream>>>(
        in, out, static_cast<uint64_t*>(col), rows, cols, row_pad, col_pad, pad_in, pad_out, in_kind, out_kind);
    VZB_OP_END(c, kOpLogup);
}

extern "C" int volta_cuda_histogram_lut_device(void* raw, uint64_t in_id, size_t in_off, uint64_t out_id,
                                               size_t out_off, size_t n, int signed_input) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || (signed_input != 0 && signed_input != 1))
        return fail_message(c, "invalid resident LUT histogram geometry");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, n, 8, &in) || region_elems(c, out_id, out_off, size_t{1} << 16, 4, &out))
        return -1;
    VZB_OP_BEGIN(c);
    VZB_CUDA(c, cudaMemsetAsync(out, 0, (size_t{1} << 16) * 4, c->stream));
    if (launch_histogram(c, static_cast<const uint64_t*>(in), static_cast<uint32_t*>(out), n, size_t{1} << 16, 1,
                         signed_input))
        return -1;
    VZB_OP_END_COPY(c, kOpLogup);  // launch_histogram counted the launch
}

extern "C" int volta_cuda_histogram_fp_device(void* raw, uint64_t in_id, size_t in_off, uint64_t out_id,
                                              size_t out_off, size_t n, size_t bins) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || !bins) return fail_message(c, "invalid resident histogram geometry");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_off, n, 8, &in) || region_elems(c, out_id, out_off, bins, 4, &out)) return -1;
    VZB_OP_BEGIN(c);
    VZB_CUDA(c, cudaMemsetAsync(out, 0, bins * 4, c->stream));
    if (launch_histogram(c, static_cast<const uint64_t*>(in), static_cast<uint32_t*>(out), n, bins, 0, 0)) return -1;
    VZB_OP_END_COPY(c, kOpLogup);  // launch_histogram counted the launch
}

extern "C" int volta_cuda_u32_add_inplace_device(void* raw, uint64_t t_id, size_t t_off, uint64_t a_id,
                                                 size_t a_off, size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n) return fail_message(c, "invalid resident u32-add geometry");
    void *t = nullptr, *a = nullptr;
    if (region_elems(c, t_id, t_off, n, 4, &t) || region_elems(c, a_id, a_off, n, 4, &a)) return -1;
    VZB_OP_BEGIN(c);
    u32_add_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<uint32_t*>(t),
                                                               static_cast<const uint32_t*>(a), n);
    VZB_OP_END(c, kOpLogup);
}

extern "C" int volta_cuda_pack_lookup_leaf_device(void* raw, uint64_t col_id, size_t col_off, uint64_t sh_id,
                                                  size_t sh_off, uint64_t leaf_id, size_t leaf_off,
                                                  size_t column_count, size_t n, uint64_t alpha0) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !column_count || n < 2 || (n & (n - 1))) return fail_message(c, "invalid resident lookup-leaf geometry");
    void *col = nullptr, *sh = nullptr, *leaf = nullptr;
    if (region_elems(c, col_id, col_off, column_count * n, 8, &col) ||
        region_elems(c, sh_id, sh_off, column_count, 4, &sh) || region_elems(c, leaf_id, leaf_off, n, 8, &leaf))
        return -1;
    VZB_OP_BEGIN(c);
    pack_leaf_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<const uint64_t*>(col),
                                                                 static_cast<const uint32_t*>(sh),
                                                                 static_cast<uint64_t*>(leaf), column_count, n,
                                                                 alpha0);
    VZB_OP_END(c, kOpLogup);
}

extern "C" int volta_cuda_deinterleave_base_columns_device(void* raw, uint64_t col_id, size_t col_off,
                                                           uint64_t out_id, size_t out_off, size_t column_count,
                                                           size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !column_count || n < 2 || n % 2)
        return fail_message(c, "invalid resident base-column deinterleave geometry");
    void *col = nullptr, *out = nullptr;
    if (region_elems(c, col_id, col_off, column_count * n, 8, &col) ||
        region_elems(c, out_id, out_off, column_count * n, sizeof(Fp2), &out))
        return -1;
    VZB_OP_BEGIN(c);
    deinterleave_base_kernel<<<grid_for(c, column_count * n, 256), 256, 0, c->stream>>>(
        static_cast<const uint64_t*>(col), static_cast<Fp2*>(out), column_count, n);
    VZB_OP_END(c, kOpLogup);
}

// ---------------------------------------------------------------------------
// Extension: int16 column to canonical Fp (negative v -> p + v), the
// embedding of rust/volta-gpt2 witness values, on the device
// ---------------------------------------------------------------------------

namespace vzb {
namespace {
__global__ void embed_i16_kernel(const int16_t* in, uint64_t* out, size_t n) {
    VZB_GRID_LOOP(i, n) {
        const int64_t v = in[i];
        out[i] = v < 0 ? kP - static_cast<uint64_t>(-v) : static_cast<uint64_t>(v);
    }
}
}  // namespace
}  // namespace vzb

extern "C" int volta_b200_embed_i16_device(void* raw, uint64_t in_id, size_t in_offset, uint64_t out_id,
                                           size_t out_offset, size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n) return fail_message(c, "invalid int16 embedding geometry");
    void *in = nullptr, *out = nullptr;
    if (region_elems(c, in_id, in_offset, n, sizeof(int16_t), &in) ||
        region_elems(c, out_id, out_offset, n, sizeof(uint64_t), &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    embed_i16_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(static_cast<const int16_t*>(in),
                                                               static_cast<uint64_t*>(out), n);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}
