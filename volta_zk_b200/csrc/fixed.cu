// int16 fixed-point GPT-2 forward primitives at the seam (entry points
// cuda/volta_cuda_backend.cu:4208-4500, kernels 1442-1740; the arithmetic
// they freeze is rust/volta-gpt2/src/layer.rs / scripts/gpt2_fixed.py).
//
// B200 design: the GEMM-shaped primitives (projections, attention scores,
// attention-weighted values, logits) run on the tensor cores through the
// exact int8-limb GEMM (gemm.cuh) with their epilogues fused: bias fold,
// requant (chained above 2^16), residual add, causal packing and the sticky
// error word.  Row reductions (layer norm, softmax) use one warp per row with
// shuffle reductions; the integer sums are exact, so the order is free.
#include "gemm.cuh"

namespace vzb {
namespace {

__device__ __forceinline__ void flag(uint32_t* error) { atomicExch(error, 1u); }

// backend.cu:1442-1446
__device__ __forceinline__ int64_t floor_div(int64_t a, int64_t b) {
    const int64_t q = a / b, r = a % b;
    return r < 0 ? q - 1 : q;
}

// backend.cu:1448-1457: round half up, chained through 2^16 above 16 bits
__device__ __forceinline__ int64_t requant_rounded(int64_t acc, uint32_t shift) {
    int64_t stage = acc;
    uint32_t fin = shift;
    if (shift > 16) {
        const uint32_t first = shift - 16;
        stage = (stage + (int64_t{1} << (first - 1))) >> first;
        fin = 16;
    }
    return (stage + (int64_t{1} << (fin - 1))) >> fin;
}

__device__ __forceinline__ int16_t requant_no_clamp(int64_t acc, uint32_t shift, bool& bad) {
    const int64_t r = requant_rounded(acc, shift);
    bad |= r < INT16_MIN || r > INT16_MAX;
    return static_cast<int16_t>(r);
}

__device__ __forceinline__ size_t packed_prefix(size_t row, size_t pos0) { return row * pos0 + row * (row + 1) / 2; }

__device__ __forceinline__ int64_t warp_sum(int64_t v) {
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) v += __shfl_xor_sync(0xffffffffu, v, d);
    return v;
}

// ---------------------------------------------------------------------------
// element-wise primitives
// ---------------------------------------------------------------------------

__global__ void embed_kernel(const uint32_t* tokens, const int16_t* wte, const int16_t* wpe, int64_t* acc_out,
                             int16_t* out, uint32_t* error, size_t rows, size_t d, size_t vocab, size_t positions,
                             size_t pos0, int32_t shift) {
    const size_t total = rows * d;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = z / d, col = z - row * d;
        const uint32_t tok = tokens[row];
        bool bad = false;
        if (tok >= vocab || pos0 + row >= positions) {
            acc_out[z] = 0;
            out[z] = 0;
            flag(error);
            continue;
        }
        const int64_t acc = static_cast<int64_t>(wte[static_cast<size_t>(tok) * d + col]) +
                            static_cast<int64_t>(wpe[(pos0 + row) * d + col]);
        acc_out[z] = acc;
        if (shift > 0) {
            out[z] = requant_no_clamp(acc, static_cast<uint32_t>(shift), bad);
        } else {
            const int64_t v = acc << static_cast<uint32_t>(-shift);
            bad = v < INT16_MIN || v > INT16_MAX;
            out[z] = static_cast<int16_t>(v);
        }
        if (bad) flag(error);
    }
}

__global__ void qkv_split_kernel(const int16_t* qkv, int16_t* q, int16_t* k, int16_t* v, size_t rows, size_t d) {
    const size_t total = rows * d;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t row = z / d, col = z - row * d;
        const int16_t* src = qkv + row * 3 * d;
        q[z] = src[col];
        k[z] = src[d + col];
        v[z] = src[2 * d + col];
    }
}

__global__ void lookup_kernel(const int16_t* in, const int16_t* lut, int16_t* out, size_t n) {
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < n;
         z += static_cast<size_t>(gridDim.x) * blockDim.x)
        out[z] = __ldg(lut + static_cast<uint16_t>(in[z]));
}

__global__ void requant_i16_kernel(const int16_t* in, int16_t* out, uint32_t* error, size_t n, uint32_t shift) {
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < n;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        bool bad = false;
        out[z] = shift == 0 ? in[z] : requant_no_clamp(in[z], shift, bad);
        if (bad) flag(error);
    }
}

// ---------------------------------------------------------------------------
// layer norm (backend.cu:1510-1549): one warp per row
// ---------------------------------------------------------------------------

__global__ void layer_norm_kernel(const int16_t* input, const int16_t* gain, const int16_t* bias, const int16_t* lut,
                                  int64_t* means, int64_t* vars, int64_t* rin, int16_t* rout, int64_t* accs,
                                  int16_t* outs, uint32_t* error, size_t rows, size_t d, uint32_t var_shift,
                                  uint32_t norm_shift) {
    const size_t row_index = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (row_index >= rows) return;
    const int16_t* row = input + row_index * d;
    int64_t sum = 0;
    for (size_t j = lane; j < d; j += 32) sum += row[j];
    sum = warp_sum(sum);
    const int64_t di = static_cast<int64_t>(d);
    const int64_t mean = floor_div(sum + di / 2, di);
    int64_t vs = 0;
    for (size_t j = lane; j < d; j += 32) {
        const int64_t dl = static_cast<int64_t>(row[j]) - mean;
        vs += dl * dl;
    }
    vs = warp_sum(vs);
    const int64_t var = floor_div(vs + di / 2, di);
    int64_t ri = var >> var_shift;
    bool bad = false;
    if (ri < 0 || ri >= (int64_t{1} << 16)) {
        bad = true;
        ri = 0;
    }
    const int16_t ro = __ldg(lut + ri);
    if (lane == 0) {
        means[row_index] = mean;
        vars[row_index] = var;
        rin[row_index] = ri;
        rout[row_index] = ro;
    }
    for (size_t j = lane; j < d; j += 32) {
        const int64_t dl = static_cast<int64_t>(row[j]) - mean;
        const int64_t acc = dl * static_cast<int64_t>(ro) * static_cast<int64_t>(gain[j]) +
                            (static_cast<int64_t>(bias[j]) << norm_shift);
        accs[row_index * d + j] = acc;
        outs[row_index * d + j] = requant_no_clamp(acc, norm_shift, bad);
    }
    if (__any_sync(0xffffffffu, bad) && lane == 0) flag(error);
}

// ---------------------------------------------------------------------------
// softmax over causal packed rows (backend.cu:1619-1687): one warp per row
// ---------------------------------------------------------------------------

__device__ __forceinline__ int16_t recip_value(int64_t input, const int16_t* lut, uint32_t den_shift,
                                               uint32_t recip_log2, int use_row_shift, bool& bad) {
    const int64_t limit = use_row_shift ? (int64_t{1} << 18) : (int64_t{1} << 16);
    if (input < 0 || input >= limit) {
        bad = true;
        return lut[0];
    }
    if (input < (int64_t{1} << 16)) return lut[static_cast<size_t>(input)];
    const uint64_t den_back = (static_cast<uint64_t>(input) << den_shift) + (uint64_t{1} << (den_shift - 1));
    uint64_t v = ((uint64_t{1} << recip_log2) + den_back / 2) / den_back;
    if (v > static_cast<uint64_t>(INT16_MAX)) v = INT16_MAX;
    return static_cast<int16_t>(v);
}

__global__ void softmax_kernel(const int16_t* scores, const int16_t* exp_lut, const int16_t* recip_lut,
                               int16_t* row_shifts, int16_t* exp_out, int64_t* denoms, int16_t* recips,
                               int16_t* weights, uint32_t* error, size_t rows, size_t pos0, size_t heads,
                               uint32_t recip_den_shift, uint32_t recip_log2, uint32_t norm_shift, int use_row_shift) {
    const size_t z = (static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (z >= heads * rows) return;
    const size_t row = z % rows, head = z / rows;
    const size_t width = pos0 + row + 1;
    const size_t per_head = rows * pos0 + rows * (rows + 1) / 2;
    const size_t start = head * per_head + packed_prefix(row, pos0);
    bool bad = false;
    int32_t sv = 0;
    if (use_row_shift) {
        int32_t mx = INT32_MIN;
        for (size_t j = lane; j < width; j += 32) mx = max(mx, static_cast<int32_t>(scores[start + j]));
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) mx = max(mx, __shfl_xor_sync(0xffffffffu, mx, d));
        sv = mx;
    }
    if (lane == 0) row_shifts[head * rows + row] = static_cast<int16_t>(sv);
    int64_t denom = 0;
    for (size_t j = lane; j < width; j += 32) {
        const int32_t s = scores[start + j];
        int16_t v = 0;
        if (use_row_shift) {
            const int32_t gap = sv - s;
            if (gap < 0 || gap > UINT16_MAX) {
                bad = true;
            } else if (gap <= 32768) {
                v = __ldg(exp_lut + static_cast<uint16_t>(static_cast<int16_t>(-gap)));
            } else if (__ldg(exp_lut + static_cast<uint16_t>(INT16_MIN)) != 0) {
                bad = true;
            }
        } else {
            v = __ldg(exp_lut + static_cast<uint16_t>(s));
        }
        exp_out[start + j] = v;
        denom += v;
    }
    denom = warp_sum(denom);
    const int16_t rc = recip_value(denom >> recip_den_shift, recip_lut, recip_den_shift, recip_log2, use_row_shift,
                                   bad);
    if (lane == 0) {
        denoms[head * rows + row] = denom;
        recips[head * rows + row] = rc;
    }
    for (size_t j = lane; j < width; j += 32)
        weights[start + j] = requant_no_clamp(static_cast<int64_t>(exp_out[start + j]) * rc, norm_shift, bad);
    if (__any_sync(0xffffffffu, bad) && lane == 0) flag(error);
}

// ---------------------------------------------------------------------------
// GEMM epilogues
// ---------------------------------------------------------------------------

// backend.cu:1551-1574
struct FixedGemmEpi {
    const int16_t* bias;
    const int16_t* residual;
    int64_t* accs;
    int16_t* req;
    int16_t* res_out;
    uint32_t* error;
    size_t n;
    uint32_t shift;
    __device__ __forceinline__ bool active(size_t, size_t, size_t, size_t) const { return true; }
    __device__ __forceinline__ size_t k_end(size_t, size_t, size_t, size_t kp) const { return kp; }
    __device__ __forceinline__ void operator()(size_t, size_t i, size_t j, int64_t acc) const {
        if (bias) acc += static_cast<int64_t>(bias[j]) << shift;
        const size_t z = i * n + j;
        accs[z] = acc;
        bool bad = false;
        const int16_t q = requant_no_clamp(acc, shift, bad);
        req[z] = q;
        if (res_out) {
            const int32_t v = static_cast<int32_t>(q) + residual[z];
            bad |= v < INT16_MIN || v > INT16_MAX;
            res_out[z] = static_cast<int16_t>(v);
        }
        if (bad) flag(error);
    }
};

// causal packed scores, batch = head (backend.cu:1593-1617)
struct ScoresEpi {
    int64_t* accs;
    int16_t* outs;
    uint32_t* error;
    size_t rows, pos0, per_head;
    uint32_t shift;
    // tiles entirely above the causal diagonal produce nothing
    __device__ __forceinline__ bool active(size_t, size_t m0, size_t n0, size_t tile_rows) const {
        return n0 <= pos0 + m0 + tile_rows - 1;
    }
    __device__ __forceinline__ size_t k_end(size_t, size_t, size_t, size_t kp) const { return kp; }
    __device__ __forceinline__ void operator()(size_t h, size_t i, size_t j, int64_t acc) const {
        if (j > pos0 + i) return;
        const size_t p = h * per_head + packed_prefix(i, pos0) + j;
        accs[p] = acc;
        const int64_t r = requant_rounded(acc, shift);
        if (r < -(int64_t{1} << 16) || r >= (int64_t{1} << 16)) flag(error);
        outs[p] = static_cast<int16_t>(r < INT16_MIN ? INT16_MIN : (r > INT16_MAX ? INT16_MAX : r));
    }
};

// attention-weighted values, batch = head (backend.cu:1689-1709)
struct AvEpi {
    int64_t* accs;
    int16_t* outs;
    uint32_t* error;
    size_t d, head_dim, pos0;
    uint32_t shift;
    __device__ __forceinline__ bool active(size_t, size_t, size_t, size_t) const { return true; }
    // weight rows m0 .. m0 + tile_rows - 1 are zero from key pos0 + m0 + tile_rows on
    __device__ __forceinline__ size_t k_end(size_t, size_t m0, size_t tile_rows, size_t kp) const {
        const size_t w = (pos0 + m0 + tile_rows + kGemmBK - 1) / kGemmBK * kGemmBK;
        return w < kp ? w : kp;
    }
    __device__ __forceinline__ void operator()(size_t h, size_t i, size_t j, int64_t acc) const {
        const size_t z = i * d + h * head_dim + j;
        accs[z] = acc;
        bool bad = false;
        outs[z] = requant_no_clamp(acc, shift, bad);
        if (bad) flag(error);
    }
};

struct LogitsEpi {
    int64_t* out;
    size_t vocab;
    __device__ __forceinline__ bool active(size_t, size_t, size_t, size_t) const { return true; }
    __device__ __forceinline__ size_t k_end(size_t, size_t, size_t, size_t kp) const { return kp; }
    __device__ __forceinline__ void operator()(size_t, size_t i, size_t j, int64_t v) const { out[i * vocab + j] = v; }
};

// Few-row products (KV-cached decoding: one row per step).  The tensor-core
// path splits the whole weight matrix into byte planes per call, which for a
// single row costs more than the product; here the weights are read once,
// straight from HBM, and the sums are exact in int64 (|x w| < 2^30, k <=
// 2^16).  The epilogues are the tensor-core path's.
constexpr size_t kSmallRows = 4;

// out[i][j] = sum_t x[i][t] w[t][j] for w row-major (k x n), split over k so
// that enough bytes are in flight to stream the weights at HBM speed: CTA
// (cx, s) covers columns [256 cx, 256 cx + 256) (8 per thread, one 16-byte
// load per row) over rows [16 s, 16 s + 16) (2 per warp); the 8 warps' sums
// meet in shared memory and the CTA writes its slice's partial sums; a
// second kernel adds the slices and applies the epilogue.  Needs n % 8 == 0
// and 16-byte aligned rows.
constexpr size_t kSliceRows = 16;

__global__ void __launch_bounds__(256) small_rows_kn_kernel(const int16_t* __restrict__ x, size_t m, size_t k,
                                                            const int16_t* __restrict__ w, size_t n,
                                                            int64_t* __restrict__ part) {
    extern __shared__ int64_t red[];  // [warp][row < m][column in the CTA], 16 KB per row
    const unsigned lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t c0 = static_cast<size_t>(blockIdx.x) * 256 + lane * 8, slice = blockIdx.y;
    int64_t acc[kSmallRows][8];
#pragma unroll
    for (size_t i = 0; i < kSmallRows; ++i)
#pragma unroll
        for (int c = 0; c < 8; ++c) acc[i][c] = 0;
    if (c0 < n) {
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
            const size_t r = slice * kSliceRows + warp * 2 + rr;
            if (r < k) {
                const uint4 v = __ldcs(reinterpret_cast<const uint4*>(w + r * n + c0));
                const uint32_t words[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (size_t i = 0; i < kSmallRows; ++i) {
                    if (i >= m) break;
                    const int32_t xv = x[i * k + r];
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const int32_t wv = static_cast<int16_t>(words[c >> 1] >> (16 * (c & 1)));
                        acc[i][c] += static_cast<int64_t>(xv * wv);
                    }
                }
            }
        }
    }
#pragma unroll
    for (size_t i = 0; i < kSmallRows; ++i) {
        if (i >= m) break;
#pragma unroll
        for (int c = 0; c < 8; ++c) red[(warp * m + i) * 256 + lane * 8 + c] = acc[i][c];
    }
    __syncthreads();
    // thread t sums column t of the CTA over the warps, row by row
    const size_t col = static_cast<size_t>(blockIdx.x) * 256 + threadIdx.x;
    if (col < n)
        for (size_t i = 0; i < m; ++i) {
            int64_t a = 0;
#pragma unroll
            for (int q = 0; q < 8; ++q) a += red[(q * m + i) * 256 + threadIdx.x];
            part[(slice * m + i) * n + col] = a;
        }
}

template <class Epi>
__global__ void small_rows_finish_kernel(const int64_t* __restrict__ part, size_t slices, size_t m, size_t n, Epi epi) {
    const size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    if (z >= m * n) return;
    int64_t a = 0;
    for (size_t s = 0; s < slices; ++s) a += part[s * m * n + z];
    epi(0, z / n, z % n, a);
}

// out[i][v] = sum_t x[i][t] w[v][t] for w stored n x k (the tied wte of the
// logits): one warp per output column v, lanes along t, a shuffle sum.
template <class Epi>
__global__ void __launch_bounds__(256) small_rows_nk_kernel(const int16_t* __restrict__ x, size_t m, size_t k,
                                                            const int16_t* __restrict__ w, size_t n, Epi epi) {
    extern __shared__ int16_t xs[];
    for (size_t t = threadIdx.x; t < m * k; t += blockDim.x) xs[t] = x[t];
    __syncthreads();
    const size_t v = static_cast<size_t>(blockIdx.x) * (blockDim.x / 32) + (threadIdx.x >> 5);
    const unsigned lane = threadIdx.x & 31;
    if (v >= n) return;
    int64_t acc[kSmallRows] = {0, 0, 0, 0};
    for (size_t t = lane; t < k; t += 32) {
        const int32_t wv = __ldcs(w + v * k + t);
#pragma unroll
        for (size_t i = 0; i < kSmallRows; ++i)
            if (i < m) acc[i] += static_cast<int64_t>(static_cast<int32_t>(xs[i * k + t]) * wv);
    }
#pragma unroll
    for (size_t i = 0; i < kSmallRows; ++i) {
        int64_t a = acc[i];
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) a += __shfl_down_sync(0xffffffffu, a, d);
        if (i < m && lane == 0) epi(0, i, v, a);
    }
}

// Whether the few-row path applies: the row-major form wants 16-byte rows.
bool small_rows_ok(size_t m, size_t k, const int16_t* w, size_t n, bool w_nk) {
    if (m > kSmallRows || k > 16384) return false;
    return w_nk || ((n % 8) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0);
}

template <class Epi>
int launch_small_rows(Context* c, const int16_t* x, size_t m, size_t k, const int16_t* w, size_t n, bool w_nk,
                      const Epi& epi) {
    if (w_nk) {
        const size_t smem = m * k * sizeof(int16_t);
        if (smem > 48 * 1024)
            VZB_CUDA(c, cudaFuncSetAttribute(small_rows_nk_kernel<Epi>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             static_cast<int>(smem)));
        small_rows_nk_kernel<Epi><<<static_cast<unsigned>((n + 7) / 8), 256, smem, c->stream>>>(x, m, k, w, n, epi);
        VZB_LAUNCHED(c);
        return 0;
    }
    const size_t slices = (k + kSliceRows - 1) / kSliceRows;
    if (ensure_ws(c, kWsScratch3, slices * m * n * sizeof(int64_t))) return -1;
    int64_t* part = ws<int64_t>(c, kWsScratch3);
    const dim3 grid(static_cast<unsigned>((n + 255) / 256), static_cast<unsigned>(slices));
    const size_t smem = 8 * m * 256 * sizeof(int64_t);
    if (smem > 48 * 1024)
        VZB_CUDA(c, cudaFuncSetAttribute(small_rows_kn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
    small_rows_kn_kernel<<<grid, 256, smem, c->stream>>>(x, m, k, w, n, part);
    VZB_LAUNCHED(c);
    small_rows_finish_kernel<Epi><<<static_cast<unsigned>((m * n + 255) / 256), 256, 0, c->stream>>>(part, slices, m,
                                                                                                     n, epi);
    VZB_LAUNCHED(c);
    return 0;
}

// Byte planes of the packed causal attention weights as dense rows (rpad per
// head, zero beyond each row's width pos0 + row + 1 and beyond `rows`); one
// thread per 16-byte chunk of the planes.
__global__ void causal_planes_kernel(const int16_t* w, size_t rows, size_t pos0, size_t heads, size_t kp,
                                     size_t rpad, int8_t* hi, uint8_t* lo) {
    const size_t per_head = rows * pos0 + rows * (rows + 1) / 2;
    const size_t per = rpad * kp / 16, total = heads * per;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t h = z / per, q = z - h * per;
        const size_t slice = q / (rpad * 4), rem = q - slice * rpad * 4;
        const size_t i = (rem >> 5) * 8 + (rem & 7), j0 = slice * 64 + ((rem >> 3) & 3) * 16;
        uint32_t hv[4] = {0, 0, 0, 0}, lv[4] = {0, 0, 0, 0};
        if (i < rows) {
            const int16_t* src = w + h * per_head + packed_prefix(i, pos0);
            const size_t width = pos0 + i + 1;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const size_t j = j0 + t;
                const uint32_t v = j < width ? static_cast<uint16_t>(src[j]) : 0u;
                hv[t >> 2] |= (v >> 8) << (8 * (t & 3));
                lv[t >> 2] |= (v & 0xFFu) << (8 * (t & 3));
            }
        }
        const size_t off = h * rpad * kp + q * 16;
        *reinterpret_cast<uint4*>(hi + off) = make_uint4(hv[0], hv[1], hv[2], hv[3]);
        *reinterpret_cast<uint4*>(lo + off) = make_uint4(lv[0], lv[1], lv[2], lv[3]);
    }
}

}  // namespace
}  // namespace vzb

using namespace vzb;

namespace {
// Typed region lookup (element offsets and counts).
template <class P>
int typed_region(Context* c, uint64_t id, size_t off, size_t count, P*& out) {
    void* p = nullptr;
    if (region_elems(c, id, off, count, sizeof(P), &p)) return -1;
    out = static_cast<P*>(p);
    return 0;
}
}  // namespace

#define VZB_REGION(id, off, count, T, ptr) typed_region(c, id, off, count, ptr)

extern "C" int volta_cuda_fixed_embed_device(void* raw, uint64_t tokens_id, size_t tokens_off, uint64_t wte_id,
                                             size_t wte_off, uint64_t wpe_id, size_t wpe_off, uint64_t acc_id,
                                             size_t acc_off, uint64_t out_id, size_t out_off, uint64_t error_id,
                                             size_t error_off, size_t rows, size_t d, size_t vocab, size_t positions,
                                             size_t pos0, int32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !d || !vocab || pos0 + rows > positions || shift >= 63 || shift <= -63)
        return fail_message(c, "invalid resident embedding geometry");
    const uint32_t* tokens = nullptr;
    const int16_t *wte = nullptr, *wpe = nullptr;
    int64_t* acc = nullptr;
    int16_t* out = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(tokens_id, tokens_off, rows, uint32_t, tokens) || VZB_REGION(wte_id, wte_off, vocab * d, int16_t, wte) ||
        VZB_REGION(wpe_id, wpe_off, positions * d, int16_t, wpe) || VZB_REGION(acc_id, acc_off, rows * d, int64_t, acc) ||
        VZB_REGION(out_id, out_off, rows * d, int16_t, out) || VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    embed_kernel<<<grid_for(c, rows * d, 256), 256, 0, c->stream>>>(tokens, wte, wpe, acc, out, err, rows, d, vocab,
                                                                    positions, pos0, shift);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_layer_norm_device(void* raw, uint64_t input_id, size_t input_off, uint64_t gain_id,
                                                  size_t gain_off, uint64_t bias_id, size_t bias_off, uint64_t lut_id,
                                                  size_t lut_off, uint64_t mean_id, size_t mean_off, uint64_t var_id,
                                                  size_t var_off, uint64_t rin_id, size_t rin_off, uint64_t rout_id,
                                                  size_t rout_off, uint64_t acc_id, size_t acc_off, uint64_t out_id,
                                                  size_t out_off, uint64_t error_id, size_t error_off, size_t rows,
                                                  size_t d, uint32_t var_shift, uint32_t norm_shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !d || !norm_shift || norm_shift >= 63 || var_shift >= 63)
        return fail_message(c, "invalid resident layer-norm geometry");
    const int16_t *in = nullptr, *gain = nullptr, *bias = nullptr, *lut = nullptr;
    int64_t *mean = nullptr, *var = nullptr, *rin = nullptr, *acc = nullptr;
    int16_t *rout = nullptr, *out = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(input_id, input_off, rows * d, int16_t, in) || VZB_REGION(gain_id, gain_off, d, int16_t, gain) ||
        VZB_REGION(bias_id, bias_off, d, int16_t, bias) || VZB_REGION(lut_id, lut_off, size_t{1} << 16, int16_t, lut) ||
        VZB_REGION(mean_id, mean_off, rows, int64_t, mean) || VZB_REGION(var_id, var_off, rows, int64_t, var) ||
        VZB_REGION(rin_id, rin_off, rows, int64_t, rin) || VZB_REGION(rout_id, rout_off, rows, int16_t, rout) ||
        VZB_REGION(out_id, out_off, rows * d, int16_t, out) || VZB_REGION(acc_id, acc_off, rows * d, int64_t, acc) ||
        VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const size_t threads = rows * 32;
    layer_norm_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, c->stream>>>(
        in, gain, bias, lut, mean, var, rin, rout, acc, out, err, rows, d, var_shift, norm_shift);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_gemm_device(void* raw, uint64_t input_id, size_t input_off, uint64_t weights_id,
                                            size_t weights_off, uint64_t bias_id, size_t bias_off,
                                            uint64_t residual_id, size_t residual_off, uint64_t acc_id,
                                            size_t acc_off, uint64_t requant_id, size_t requant_off,
                                            uint64_t residual_out_id, size_t residual_out_off, uint64_t error_id,
                                            size_t error_off, size_t m, size_t k, size_t n, uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !m || !k || !n || !shift || shift >= 63 || ((residual_id == 0) != (residual_out_id == 0)))
        return fail_message(c, "invalid resident fixed GEMM geometry");
    const int16_t *in = nullptr, *w = nullptr, *bias = nullptr, *res = nullptr;
    int64_t* acc = nullptr;
    int16_t *req = nullptr, *res_out = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(input_id, input_off, m * k, int16_t, in) || VZB_REGION(weights_id, weights_off, k * n, int16_t, w) ||
        (bias_id && VZB_REGION(bias_id, bias_off, n, int16_t, bias)) ||
        (residual_id && VZB_REGION(residual_id, residual_off, m * n, int16_t, res)) ||
        VZB_REGION(acc_id, acc_off, m * n, int64_t, acc) || VZB_REGION(requant_id, requant_off, m * n, int16_t, req) ||
        (residual_out_id && VZB_REGION(residual_out_id, residual_out_off, m * n, int16_t, res_out)) ||
        VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const FixedGemmEpi epi{bias, res, acc, req, res_out, err, n, shift};
    if (small_rows_ok(m, k, w, n, false)) {
        if (launch_small_rows(c, in, m, k, w, n, false, epi)) return -1;
    } else {
        GemmPlanes g;
        if (gemm_prepare(c, in, m, k, k, w, n, n, false, &g)) return -1;
        if (gemm_launch(c, g, epi)) return -1;
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_qkv_split_device(void* raw, uint64_t input_id, size_t input_off, uint64_t q_id,
                                                 size_t q_off, uint64_t k_id, size_t k_off, uint64_t v_id,
                                                 size_t v_off, size_t rows, size_t d) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !d) return fail_message(c, "invalid resident QKV split geometry");
    const int16_t* in = nullptr;
    int16_t *q = nullptr, *k = nullptr, *v = nullptr;
    if (VZB_REGION(input_id, input_off, rows * 3 * d, int16_t, in) || VZB_REGION(q_id, q_off, rows * d, int16_t, q) ||
        VZB_REGION(k_id, k_off, rows * d, int16_t, k) || VZB_REGION(v_id, v_off, rows * d, int16_t, v))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    qkv_split_kernel<<<grid_for(c, rows * d, 256), 256, 0, c->stream>>>(in, q, k, v, rows, d);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_attention_scores_device(void* raw, uint64_t q_id, size_t q_off, uint64_t k_id,
                                                        size_t k_off, uint64_t acc_id, size_t acc_off,
                                                        uint64_t out_id, size_t out_off, uint64_t error_id,
                                                        size_t error_off, size_t rows, size_t seq, size_t pos0,
                                                        size_t heads, size_t head_dim, uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !seq || !heads || !head_dim || pos0 + rows > seq || !shift || shift >= 63)
        return fail_message(c, "invalid resident attention-score geometry");
    const size_t d = heads * head_dim;
    const size_t per_head = rows * pos0 + rows * (rows + 1) / 2;
    const int16_t *q = nullptr, *k = nullptr;
    int64_t* acc = nullptr;
    int16_t* out = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(q_id, q_off, rows * d, int16_t, q) || VZB_REGION(k_id, k_off, seq * d, int16_t, k) ||
        VZB_REGION(acc_id, acc_off, heads * per_head, int64_t, acc) ||
        VZB_REGION(out_id, out_off, heads * per_head, int16_t, out) || VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    // per head: Q_h (rows x head_dim, stride d) times K_h^T (K_h is seq x head_dim: the n x k layout)
    GemmPlanes g;
    if (gemm_prepare(c, q, rows, head_dim, d, k, pos0 + rows, d, true, &g, static_cast<unsigned>(heads), head_dim,
                     head_dim))
        return -1;
    if (gemm_launch(c, g, ScoresEpi{acc, out, err, rows, pos0, per_head, shift})) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_softmax_device(void* raw, uint64_t scores_id, size_t scores_off, uint64_t exp_lut_id,
                                               size_t exp_lut_off, uint64_t recip_lut_id, size_t recip_lut_off,
                                               uint64_t row_shift_id, size_t row_shift_off, uint64_t exp_id,
                                               size_t exp_off, uint64_t denoms_id, size_t denoms_off,
                                               uint64_t recips_id, size_t recips_off, uint64_t weights_id,
                                               size_t weights_off, uint64_t error_id, size_t error_off, size_t rows,
                                               size_t seq, size_t pos0, size_t heads, uint32_t recip_den_shift,
                                               uint32_t recip_log2, uint32_t norm_shift, int use_row_shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !seq || !heads || pos0 + rows > seq || !norm_shift || norm_shift >= 63 || !recip_den_shift ||
        recip_den_shift >= 63 || recip_log2 >= 63)
        return fail_message(c, "invalid resident softmax geometry");
    const size_t packed = heads * (rows * pos0 + rows * (rows + 1) / 2), row_count = heads * rows;
    const int16_t *scores = nullptr, *exp_lut = nullptr, *recip_lut = nullptr;
    int16_t *row_shift = nullptr, *exp = nullptr, *recips = nullptr, *weights = nullptr;
    int64_t* denoms = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(scores_id, scores_off, packed, int16_t, scores) ||
        VZB_REGION(exp_lut_id, exp_lut_off, size_t{1} << 16, int16_t, exp_lut) ||
        VZB_REGION(recip_lut_id, recip_lut_off, size_t{1} << 16, int16_t, recip_lut) ||
        VZB_REGION(row_shift_id, row_shift_off, row_count, int16_t, row_shift) ||
        VZB_REGION(exp_id, exp_off, packed, int16_t, exp) || VZB_REGION(denoms_id, denoms_off, row_count, int64_t, denoms) ||
        VZB_REGION(recips_id, recips_off, row_count, int16_t, recips) ||
        VZB_REGION(weights_id, weights_off, packed, int16_t, weights) || VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    const size_t threads = row_count * 32;
    softmax_kernel<<<static_cast<unsigned>((threads + 255) / 256), 256, 0, c->stream>>>(
        scores, exp_lut, recip_lut, row_shift, exp, denoms, recips, weights, err, rows, pos0, heads, recip_den_shift,
        recip_log2, norm_shift, use_row_shift);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_av_device(void* raw, uint64_t weights_id, size_t weights_off, uint64_t values_id,
                                          size_t values_off, uint64_t acc_id, size_t acc_off, uint64_t out_id,
                                          size_t out_off, uint64_t error_id, size_t error_off, size_t rows,
                                          size_t seq, size_t pos0, size_t d, size_t heads, uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !seq || !d || !heads || d % heads || pos0 + rows > seq || !shift || shift >= 63)
        return fail_message(c, "invalid resident AV geometry");
    const size_t packed = heads * (rows * pos0 + rows * (rows + 1) / 2), head_dim = d / heads;
    const int16_t *w = nullptr, *values = nullptr;
    int64_t* acc = nullptr;
    int16_t* out = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(weights_id, weights_off, packed, int16_t, w) || VZB_REGION(values_id, values_off, seq * d, int16_t, values) ||
        VZB_REGION(acc_id, acc_off, rows * d, int64_t, acc) || VZB_REGION(out_id, out_off, rows * d, int16_t, out) ||
        VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    // per head: dense causal weights (rows x width) times V_h (width x head_dim, stride d)
    const size_t width = pos0 + rows;
    const size_t kp = (width + kGemmBK - 1) / kGemmBK * kGemmBK;
    const size_t mpad = plane_rows(rows);
    GemmPlanes g;
    if (gemm_prepare_b(c, values, width, head_dim, d, false, kp, static_cast<unsigned>(heads), head_dim,
                       heads * mpad * kp, &g))
        return -1;
    g.m = rows;
    g.mpad = mpad;
    g.a_batch = mpad * kp;
    causal_planes_kernel<<<grid_for(c, heads * mpad * kp / 16, 256), 256, 0, c->stream>>>(
        w, rows, pos0, heads, kp, mpad, const_cast<int8_t*>(g.a_hi), const_cast<uint8_t*>(g.a_lo));
    VZB_LAUNCHED(c);
    if (gemm_launch(c, g, AvEpi{acc, out, err, d, head_dim, pos0, shift})) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_lookup_device(void* raw, uint64_t input_id, size_t input_off, uint64_t lut_id,
                                              size_t lut_off, uint64_t out_id, size_t out_off, size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n) return fail_message(c, "invalid resident lookup geometry");
    const int16_t *in = nullptr, *lut = nullptr;
    int16_t* out = nullptr;
    if (VZB_REGION(input_id, input_off, n, int16_t, in) || VZB_REGION(lut_id, lut_off, size_t{1} << 16, int16_t, lut) ||
        VZB_REGION(out_id, out_off, n, int16_t, out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    lookup_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(in, lut, out, n);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_requant_i16_device(void* raw, uint64_t input_id, size_t input_off, uint64_t out_id,
                                                   size_t out_off, uint64_t error_id, size_t error_off, size_t n,
                                                   uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || shift >= 63) return fail_message(c, "invalid resident i16 requant geometry");
    const int16_t* in = nullptr;
    int16_t* out = nullptr;
    uint32_t* err = nullptr;
    if (VZB_REGION(input_id, input_off, n, int16_t, in) || VZB_REGION(out_id, out_off, n, int16_t, out) ||
        VZB_REGION(error_id, error_off, 1, uint32_t, err))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    requant_i16_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(in, out, err, n, shift);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_fixed_logits_device(void* raw, uint64_t input_id, size_t input_off, uint64_t weights_id,
                                              size_t weights_off, uint64_t out_id, size_t out_off, size_t rows,
                                              size_t d, size_t vocab) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !rows || !d || !vocab) return fail_message(c, "invalid resident logits geometry");
    const int16_t *in = nullptr, *w = nullptr;
    int64_t* out = nullptr;
    if (VZB_REGION(input_id, input_off, rows * d, int16_t, in) || VZB_REGION(weights_id, weights_off, vocab * d, int16_t, w) ||
        VZB_REGION(out_id, out_off, rows * vocab, int64_t, out))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    // x (rows x d) times wte^T: wte (vocab x d) is already the n x k layout
    if (small_rows_ok(rows, d, w, vocab, true)) {
        if (launch_small_rows(c, in, rows, d, w, vocab, true, LogitsEpi{out, vocab})) return -1;
    } else {
        GemmPlanes g;
        if (gemm_prepare(c, in, rows, d, d, w, vocab, d, true, &g)) return -1;
        if (gemm_launch(c, g, LogitsEpi{out, vocab})) return -1;
    }
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

// ---------------------------------------------------------------------------
// Extension: greedy token selection (rust/volta-gpt2/src/decode.rs:270-272,
// argmax by Iterator::max_by_key, which returns the LAST of equal maxima)
// ---------------------------------------------------------------------------

namespace vzb {
namespace {

// One CTA: (value, index) pairs reduced with "greater value, or equal value
// and larger index" wins.
__global__ void __launch_bounds__(1024) argmax_last_kernel(const int64_t* __restrict__ x, size_t n,
                                                           uint32_t* __restrict__ out) {
    __shared__ int64_t sv[32];
    __shared__ uint32_t si[32];
    int64_t bv = INT64_MIN;
    uint32_t bi = 0;
    for (size_t i = threadIdx.x; i < n; i += blockDim.x) {
        const int64_t v = x[i];
        if (v >= bv) {  // indices grow along a thread's walk: >= keeps the last
            bv = v;
            bi = static_cast<uint32_t>(i);
        }
    }
    auto better = [](int64_t va, uint32_t ia, int64_t vb, uint32_t ib) { return vb > va || (vb == va && ib > ia); };
#pragma unroll
    for (int d = 16; d > 0; d >>= 1) {
        const int64_t ov = __shfl_down_sync(0xffffffffu, bv, d);
        const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, d);
        if (better(bv, bi, ov, oi)) {
            bv = ov;
            bi = oi;
        }
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) {
        sv[warp] = bv;
        si[warp] = bi;
    }
    __syncthreads();
    if (warp == 0) {
        const int warps = (blockDim.x + 31) >> 5;
        bv = lane < warps ? sv[lane] : INT64_MIN;
        bi = lane < warps ? si[lane] : 0;
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) {
            const int64_t ov = __shfl_down_sync(0xffffffffu, bv, d);
            const uint32_t oi = __shfl_down_sync(0xffffffffu, bi, d);
            if (better(bv, bi, ov, oi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) *out = bi;
    }
}

}  // namespace
}  // namespace vzb

extern "C" int volta_b200_argmax_i64_device(void* raw, uint64_t in_id, size_t in_off, size_t n, uint64_t out_id,
                                            size_t out_off) {
    using namespace vzb;
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || n > 0xFFFFFFFFull) return fail_message(c, "invalid argmax geometry");
    const int64_t* x = nullptr;
    uint32_t* out = nullptr;
    if (VZB_REGION(in_id, in_off, n, int64_t, x) || VZB_REGION(out_id, out_off, 1, uint32_t, out)) return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    argmax_last_kernel<<<1, 1024, 0, c->stream>>>(x, n, out);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}
