// Ligero row preparation and opening gathers (seam entry points
// cuda/volta_cuda_backend.cu:7064-7100, 7206-7254; kernels 2946-3028):
//   messages   row r = (embed(w[r, 0..cols)) || pads[r, 0..pad) || 0...) to
//              code_len (ligero.rs:553-561)
//   combine    out[c, j] = sum_r coeffs[c, r] * row_r[j] over the message
//              rows (pcs_combine_rows; ligero.rs:1187-1555 opening)
//   gather     out[q, i] = matrix[i, idx[q]] (opened columns, ligero.rs:1444)
#include "runtime.cuh"

#include <algorithm>

namespace vzb {
namespace {

__device__ __forceinline__ uint64_t from_i16(int16_t x) {
    return x >= 0 ? static_cast<uint64_t>(x) : kP - static_cast<uint64_t>(-static_cast<int32_t>(x));
}

// One thread per output word, row-major: consecutive threads write (and
// read) consecutive words of a row.
__global__ void messages_kernel(const int16_t* w, const uint64_t* pads, uint64_t* out, size_t rows, size_t cols,
                                size_t pad, size_t code_len) {
    const size_t total = rows * code_len;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t r = z / code_len, j = z - r * code_len;
        uint64_t v = 0;
        if (j < cols)
            v = from_i16(w[r * cols + j]);
        else if (j < cols + pad)
            v = pads[r * pad + (j - cols)];
        __stcs(out + z, v);
    }
}

// out[c, j] = sum_r coeffs[c, r] x[r, j]: each thread owns one column j of
// the message rows and up to kCombos combinations, so every message word is
// read once per kCombos combinations; products accumulate unreduced.
constexpr int kCombos = 4;

__global__ void combine_kernel(const int16_t* w, const uint64_t* pads, const Fp2* coeffs, Fp2* out, size_t rows,
                               size_t cols, size_t pad, size_t combinations) {
    const size_t msg_len = cols + pad;
    const size_t groups = (combinations + kCombos - 1) / kCombos;
    const size_t total = groups * msg_len;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t g = z / msg_len, j = z - g * msg_len;
        const size_t c0 = g * kCombos;
        const int nc = static_cast<int>(combinations - c0 < kCombos ? combinations - c0 : kCombos);
        Fp2W acc[kCombos];
#pragma unroll
        for (int k = 0; k < kCombos; ++k) f2w_zero(acc[k]);
        for (size_t r = 0; r < rows; ++r) {
            const uint64_t x = j < cols ? from_i16(w[r * cols + j]) : pads[r * pad + (j - cols)];
#pragma unroll
            for (int k = 0; k < kCombos; ++k) {
                if (k < nc) {
                    const Fp2 cf = ldg2(coeffs + (c0 + k) * rows + r);
                    wadd(acc[k].c0, dmul_wide(cf.c0, x));
                    wadd(acc[k].c1, dmul_wide(cf.c1, x));
                }
            }
        }
#pragma unroll
        for (int k = 0; k < kCombos; ++k)
            if (k < nc) out[(c0 + k) * msg_len + j] = f2w_reduce(acc[k]);
    }
}

template <class T>
__global__ void gather_kernel(const T* m, const uint32_t* idx, T* out, size_t rows, size_t cols, size_t queries) {
    const size_t total = rows * queries;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t q = z / rows, i = z - q * rows;
        const size_t col = idx[q];
        // an out-of-range column index yields zeros instead of a stray read
        out[z] = col < cols ? m[i * cols + col] : T{};
    }
}

// The same sums over a band of rows per grid row (blockIdx.y): partial
// out[band][combination][j] into `part`, summed by combine_finish_kernel.
// With few combinations there are only cols + pad columns of work, so one
// thread per column walking every row waits out a dependent HBM load per row
// (8192 rows: milliseconds); bands give every SM independent rows to stream.
__global__ void combine_band_kernel(const int16_t* w, const uint64_t* pads, const Fp2* coeffs, Fp2* part,
                                    size_t rows, size_t cols, size_t pad, size_t combinations, size_t band_rows) {
    const size_t msg_len = cols + pad;
    const size_t groups = (combinations + kCombos - 1) / kCombos;
    const size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (z >= groups * msg_len) return;
    const size_t g = z / msg_len, j = z - g * msg_len;
    const size_t c0 = g * kCombos, band = blockIdx.y;
    const size_t r0 = band * band_rows, r1 = min(rows, r0 + band_rows);
    const int nc = static_cast<int>(combinations - c0 < kCombos ? combinations - c0 : kCombos);
    Fp2W acc[kCombos];
#pragma unroll
    for (int k = 0; k < kCombos; ++k) f2w_zero(acc[k]);
#pragma unroll 4
    for (size_t r = r0; r < r1; ++r) {
        const uint64_t x = j < cols ? from_i16(w[r * cols + j]) : pads[r * pad + (j - cols)];
#pragma unroll
        for (int k = 0; k < kCombos; ++k) {
            if (k < nc) {
                const Fp2 cf = ldg2(coeffs + (c0 + k) * rows + r);
                wadd(acc[k].c0, dmul_wide(cf.c0, x));
                wadd(acc[k].c1, dmul_wide(cf.c1, x));
            }
        }
    }
#pragma unroll
    for (int k = 0; k < kCombos; ++k)
        if (k < nc) part[(band * combinations + c0 + k) * msg_len + j] = f2w_reduce(acc[k]);
}

__global__ void combine_finish_kernel(const Fp2* part, Fp2* out, size_t bands, size_t entries) {
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < entries; z += stride) {
        Fp2 s{0, 0};
        for (size_t b = 0; b < bands; ++b) s = f2add(s, ldg2(part + b * entries + z));
        st2(out + z, s);
    }
}

int combine(Context* c, const int16_t* w, const uint64_t* pads, const Fp2* coeffs, Fp2* out, size_t rows,
            size_t cols, size_t pad, size_t combinations) {
    const size_t msg_len = cols + pad;
    const size_t items = ((combinations + kCombos - 1) / kCombos) * msg_len;
    // aim for about 2 x 1024 threads per SM, with bands of at least 32 rows
    const size_t want = static_cast<size_t>(c->sm_count) * 2048;
    size_t bands = items >= want ? 1 : (want + items - 1) / items;
    bands = std::min<size_t>(std::min(bands, (rows + 31) / 32), 65535);
    if (bands <= 1) {
        combine_kernel<<<grid_for(c, items, 256), 256, 0, c->stream>>>(w, pads, coeffs, out, rows, cols, pad,
                                                                       combinations);
        VZB_LAUNCHED(c);
        return 0;
    }
    const size_t band_rows = (rows + bands - 1) / bands;
    bands = (rows + band_rows - 1) / band_rows;
    const size_t entries = combinations * msg_len;
    if (ensure_ws(c, kWsScratch, bands * entries * sizeof(Fp2))) return -1;
    Fp2* part = ws<Fp2>(c, kWsScratch);
    const dim3 grid(static_cast<unsigned>((items + 255) / 256), static_cast<unsigned>(bands));
    combine_band_kernel<<<grid, 256, 0, c->stream>>>(w, pads, coeffs, part, rows, cols, pad, combinations,
                                                     band_rows);
    VZB_LAUNCHED(c);
    combine_finish_kernel<<<grid_for(c, entries, 256), 256, 0, c->stream>>>(part, out, bands, entries);
    VZB_LAUNCHED(c);
    return 0;
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_pcs_messages_device(void* raw, uint64_t weights_id, size_t weights_offset,
                                              uint64_t pads_id, size_t pads_offset, size_t rows, size_t cols,
                                              size_t pad, size_t code_len, uint64_t output_id,
                                              size_t output_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !cols || !code_len || cols + pad > code_len)
        return fail_message(c, "invalid resident PCS message geometry");
    void *w = nullptr, *pads = nullptr, *out = nullptr;
    if (region_elems(c, weights_id, weights_offset, rows * cols, sizeof(int16_t), &w) ||
        (pad && region_elems(c, pads_id, pads_offset, rows * pad, sizeof(uint64_t), &pads)) ||
        region_elems(c, output_id, output_offset, rows * code_len, sizeof(uint64_t), &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    messages_kernel<<<grid_for(c, rows * code_len, 256), 256, 0, c->stream>>>(
        static_cast<const int16_t*>(w), static_cast<const uint64_t*>(pads), static_cast<uint64_t*>(out), rows, cols,
        pad, code_len);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_pcs_combine_rows_device(void* raw, uint64_t weights_id, size_t weights_offset,
                                                  uint64_t pads_id, size_t pads_offset, uint64_t coeffs_id,
                                                  size_t coeffs_offset, size_t rows, size_t cols, size_t pad,
                                                  size_t combinations, uint64_t output_id, size_t output_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !cols || !combinations) return fail_message(c, "invalid resident PCS combination geometry");
    const size_t msg_len = cols + pad;
    void *w = nullptr, *pads = nullptr, *coeffs = nullptr, *out = nullptr;
    if (region_elems(c, weights_id, weights_offset, rows * cols, sizeof(int16_t), &w) ||
        (pad && region_elems(c, pads_id, pads_offset, rows * pad, sizeof(uint64_t), &pads)) ||
        region_elems(c, coeffs_id, coeffs_offset, combinations * rows, sizeof(Fp2), &coeffs) ||
        region_elems(c, output_id, output_offset, combinations * msg_len, sizeof(Fp2), &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (combine(c, static_cast<const int16_t*>(w), static_cast<const uint64_t*>(pads),
                static_cast<const Fp2*>(coeffs), static_cast<Fp2*>(out), rows, cols, pad, combinations))
        return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_pcs_combine_rows(void* raw, const int16_t* weights, const uint64_t* pads,
                                           const Fp2* coeffs, size_t rows, size_t cols, size_t pad,
                                           size_t combinations, Fp2* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !weights || !coeffs || !out || !rows || !cols || !combinations || (pad && !pads)) return -1;
    const size_t wb = rows * cols * sizeof(int16_t), pb = rows * pad * sizeof(uint64_t),
                 cb = combinations * rows * sizeof(Fp2), ob = combinations * (cols + pad) * sizeof(Fp2);
    if (ensure_ws(c, kWsStageA, wb) || ensure_ws(c, kWsStageB, pb ? pb : 8) || ensure_ws(c, kWsStageC, cb) ||
        ensure_ws(c, kWsStageD, ob))
        return -1;
    if (op_begin(c)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(ws<int16_t>(c, kWsStageA), weights, wb, cudaMemcpyHostToDevice, c->stream));
    if (pb) VZB_CUDA(c, cudaMemcpyAsync(ws<uint64_t>(c, kWsStageB), pads, pb, cudaMemcpyHostToDevice, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(ws<Fp2>(c, kWsStageC), coeffs, cb, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    if (combine(c, ws<int16_t>(c, kWsStageA), ws<uint64_t>(c, kWsStageB), ws<Fp2>(c, kWsStageC),
                ws<Fp2>(c, kWsStageD), rows, cols, pad, combinations))
        return -1;
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(out, ws<Fp2>(c, kWsStageD), ob, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpPcsRows, wb + pb + cb, ob);
}

extern "C" int volta_cuda_pcs_gather_columns_device(void* raw, uint64_t matrix_id, size_t matrix_offset,
                                                    size_t rows, size_t cols, uint64_t indices_id,
                                                    size_t indices_offset, size_t queries, uint64_t output_id,
                                                    size_t output_offset, int fp2) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !cols || !queries) return fail_message(c, "invalid resident PCS gather geometry");
    const size_t elem = fp2 ? sizeof(Fp2) : sizeof(uint64_t);
    void *m = nullptr, *idx = nullptr, *out = nullptr;
    if (region_elems(c, matrix_id, matrix_offset, rows * cols, elem, &m) ||
        region_elems(c, indices_id, indices_offset, queries, sizeof(uint32_t), &idx) ||
        region_elems(c, output_id, output_offset, rows * queries, elem, &out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const unsigned grid = grid_for(c, rows * queries, 256);
    if (fp2)
        gather_kernel<Fp2><<<grid, 256, 0, c->stream>>>(static_cast<const Fp2*>(m), static_cast<const uint32_t*>(idx),
                                                        static_cast<Fp2*>(out), rows, cols, queries);
    else
        gather_kernel<uint64_t><<<grid, 256, 0, c->stream>>>(static_cast<const uint64_t*>(m),
                                                             static_cast<const uint32_t*>(idx),
                                                             static_cast<uint64_t*>(out), rows, cols, queries);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsRows, 0, 0);
}

extern "C" int volta_cuda_pcs_gather_columns(void* raw, const uint64_t* matrix, size_t rows, size_t cols,
                                             const uint32_t* indices, size_t queries, uint64_t* out) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !matrix || !indices || !out || !rows || !cols || !queries) return -1;
    const size_t mb = rows * cols * sizeof(uint64_t), ib = queries * sizeof(uint32_t),
                 ob = rows * queries * sizeof(uint64_t);
    if (ensure_ws(c, kWsStageA, mb) || ensure_ws(c, kWsStageB, ib) || ensure_ws(c, kWsStageC, ob)) return -1;
    if (op_begin(c)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(ws<uint64_t>(c, kWsStageA), matrix, mb, cudaMemcpyHostToDevice, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(ws<uint32_t>(c, kWsStageB), indices, ib, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    gather_kernel<uint64_t><<<grid_for(c, rows * queries, 256), 256, 0, c->stream>>>(
        ws<uint64_t>(c, kWsStageA), ws<uint32_t>(c, kWsStageB), ws<uint64_t>(c, kWsStageC), rows, cols, queries);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(out, ws<uint64_t>(c, kWsStageC), ob, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpPcsRows, mb + ib, ob);
}
