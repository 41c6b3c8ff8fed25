// Witness GEMMs on the tensor cores (seam entry points
// cuda/volta_cuda_backend.cu:4128-4200; semantics rust/volta-gpt2/src/gemm.rs):
//   gemm_i64            acc = a b exactly (i64)
//   gemm_requant_auth   y = clamp(round_half_up(acc / 2^s)) as i16 and the MAC
//                       correction corr = embed(y) - mask (gemm.rs:19-22, 120-154)
#include "gemm.cuh"

namespace vzb {

// Packs 16 int16 values into the 16 high bytes and 16 low bytes of one
// core-matrix row of each plane.
__device__ __forceinline__ void pack16(const uint32_t (&v)[16], int8_t* hi, uint8_t* lo) {
    uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
#pragma unroll
    for (int t = 0; t < 16; ++t) {
        h[t >> 2] |= (v[t] >> 8) << (8 * (t & 3));
        l[t >> 2] |= (v[t] & 0xFFu) << (8 * (t & 3));
    }
    *reinterpret_cast<uint4*>(hi) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4*>(lo) = make_uint4(l[0], l[1], l[2], l[3]);
}

// One thread per 16-byte core-matrix row of the output planes (consecutive
// threads write consecutive 16-byte chunks); a row's 16 values are read as
// two 16-byte vectors when the source allows it.
__global__ void split_planes_kernel(const int16_t* x, size_t rows, size_t k, size_t ld, int8_t* hi, uint8_t* lo,
                                    size_t kp, size_t rpad, unsigned batches, size_t boff) {
    const size_t per = rpad * kp / 16, total = per * batches;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t b = z / per, q = z - b * per;
        // q -> (k-slice, row group, 16-byte chunk, row in group), the order of plane_off
        const size_t slice = q / (rpad * 4), rem = q - slice * rpad * 4;
        const size_t r = (rem >> 5) * 8 + (rem & 7), k0 = slice * 64 + ((rem >> 3) & 3) * 16;
        uint32_t v[16];
        const int16_t* src = x + b * boff + r * ld + k0;
        if (r < rows && k0 + 16 <= k && (reinterpret_cast<uintptr_t>(src) & 15) == 0) {
            const uint4 w0 = __ldg(reinterpret_cast<const uint4*>(src)), w1 = __ldg(reinterpret_cast<const uint4*>(src) + 1);
            const uint32_t w[8] = {w0.x, w0.y, w0.z, w0.w, w1.x, w1.y, w1.z, w1.w};
#pragma unroll
            for (int t = 0; t < 8; ++t) {
                v[2 * t] = w[t] & 0xFFFFu;
                v[2 * t + 1] = w[t] >> 16;
            }
        } else {
#pragma unroll
            for (int t = 0; t < 16; ++t) v[t] = (r < rows && k0 + t < k) ? static_cast<uint16_t>(src[t]) : 0u;
        }
        const size_t off = b * rpad * kp + q * 16;
        pack16(v, hi + off, lo + off);
    }
}

// Transposing split: plane row nn holds column nn of x ([k][n] row-major,
// stride ld, batch b at x + b * boff).  One thread per 16-byte core-matrix
// row (16 consecutive k of one column); the 32 threads of a warp take 32
// consecutive columns, so each of the 16 reads is one coalesced 64-byte
// access and each plane store covers four 128-byte row groups.  Rows n..npad
// are written as zeros.
__global__ void split_planes_t_kernel(const int16_t* x, size_t k, size_t n, size_t ld, int8_t* hi, uint8_t* lo,
                                      size_t kp, size_t npad, unsigned batches, size_t boff) {
    const size_t chunks = kp / 16, per = npad * chunks, total = per * batches;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t b = z / per, q = z - b * per;
        const size_t nb = q / (32 * chunks), rem = q - nb * 32 * chunks;
        const size_t kc = rem >> 5, nn = nb * 32 + (rem & 31), k0 = kc * 16;
        const int16_t* src = x + b * boff + nn;
        uint32_t v[16];
#pragma unroll
        for (int t = 0; t < 16; ++t) v[t] = (nn < n && k0 + t < k) ? static_cast<uint16_t>(src[(k0 + t) * ld]) : 0u;
        const size_t off = b * npad * kp + plane_off(nn, k0, npad);
        pack16(v, hi + off, lo + off);
    }
}

int gemm_prepare_b(Context* c, const int16_t* b, size_t k, size_t n, size_t ldb, bool b_nk, size_t kp,
                   unsigned batches, size_t b_boff, size_t a_bytes, GemmPlanes* out) {
    const size_t npad = plane_rows(n);
    const size_t bbytes = npad * kp * batches;
    if (ensure_ws(c, kWsGemm, 2 * a_bytes + 2 * bbytes + 64)) return -1;
    unsigned char* w = ws<unsigned char>(c, kWsGemm);
    out->a_hi = reinterpret_cast<int8_t*>(w);
    out->a_lo = w + a_bytes;
    out->b_hi = reinterpret_cast<int8_t*>(w + 2 * a_bytes);
    out->b_lo = w + 2 * a_bytes + bbytes;
    out->n = n;
    out->npad = npad;
    out->kp = kp;
    out->batches = batches;
    out->b_batch = npad * kp;
    if (b_nk) {
        split_planes_kernel<<<grid_for(c, bbytes / 16, 256), 256, 0, c->stream>>>(
            b, n, k, ldb, const_cast<int8_t*>(out->b_hi), const_cast<uint8_t*>(out->b_lo), kp, npad, batches, b_boff);
    } else {
        split_planes_t_kernel<<<grid_for(c, bbytes / 16, 256), 256, 0, c->stream>>>(
            b, k, n, ldb, const_cast<int8_t*>(out->b_hi), const_cast<uint8_t*>(out->b_lo), kp, npad, batches, b_boff);
    }
    VZB_LAUNCHED(c);
    return 0;
}

int gemm_prepare(Context* c, const int16_t* a, size_t m, size_t k, size_t lda, const int16_t* b, size_t n,
                 size_t ldb, bool b_nk, GemmPlanes* out, unsigned batches, size_t a_boff, size_t b_boff) {
    const size_t kp = (k + kGemmBK - 1) / kGemmBK * kGemmBK;
    const size_t mpad = plane_rows(m);
    const size_t abytes = mpad * kp * batches;
    if (gemm_prepare_b(c, b, k, n, ldb, b_nk, kp, batches, b_boff, abytes, out)) return -1;
    out->m = m;
    out->mpad = mpad;
    out->a_batch = mpad * kp;
    split_planes_kernel<<<grid_for(c, abytes / 16, 256), 256, 0, c->stream>>>(
        a, m, k, lda, const_cast<int8_t*>(out->a_hi), const_cast<uint8_t*>(out->a_lo), kp, mpad, batches, a_boff);
    VZB_LAUNCHED(c);
    return 0;
}

namespace {

struct I64Epi {
    int64_t* out;
    size_t ldo;
    __device__ __forceinline__ bool active(size_t, size_t, size_t, size_t) const { return true; }
    __device__ __forceinline__ size_t k_end(size_t, size_t, size_t, size_t kp) const { return kp; }
    __device__ __forceinline__ void operator()(size_t, size_t i, size_t j, int64_t v) const { out[i * ldo + j] = v; }
};

__device__ __forceinline__ int16_t requant_clamped(int64_t acc, uint32_t shift) {
    const int64_t r = (acc + (int64_t{1} << (shift - 1))) >> shift;
    return static_cast<int16_t>(r < -32768 ? -32768 : (r > 32767 ? 32767 : r));
}

struct RequantAuthEpi {
    const uint64_t* masks;
    int16_t* out;
    uint64_t* corr;
    size_t n;
    uint32_t shift;
    __device__ __forceinline__ bool active(size_t, size_t, size_t, size_t) const { return true; }
    __device__ __forceinline__ size_t k_end(size_t, size_t, size_t, size_t kp) const { return kp; }
    __device__ __forceinline__ void operator()(size_t, size_t i, size_t j, int64_t v) const {
        const size_t z = i * n + j;
        const int16_t y = requant_clamped(v, shift);
        out[z] = y;
        corr[z] = fsub(ffrom_i64(y), __ldg(masks + z));
    }
};

int gemm_i64_run(Context* c, const int16_t* a, const int16_t* b, int64_t* out, size_t m, size_t k, size_t n) {
    GemmPlanes g;
    if (gemm_prepare(c, a, m, k, k, b, n, n, false, &g)) return -1;
    return gemm_launch(c, g, I64Epi{out, n});
}

int gemm_auth_run(Context* c, const int16_t* a, const int16_t* b, const uint64_t* masks, int16_t* out,
                  uint64_t* corr, size_t m, size_t k, size_t n, uint32_t shift) {
    GemmPlanes g;
    if (gemm_prepare(c, a, m, k, k, b, n, n, false, &g)) return -1;
    return gemm_launch(c, g, RequantAuthEpi{masks, out, corr, n, shift});
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_gemm_i64(void* raw, const int16_t* a, const int16_t* b, int64_t* out, size_t m, size_t k,
                                   size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !a || !b || !out || !m || !k || !n) return -1;
    const size_t ab = m * k * 2, bb = k * n * 2, ob = m * n * 8;
    if (ensure_ws(c, kWsStageA, ab) || ensure_ws(c, kWsStageB, bb) || ensure_ws(c, kWsStageC, ob)) return -1;
    if (op_begin(c)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(ws<int16_t>(c, kWsStageA), a, ab, cudaMemcpyHostToDevice, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(ws<int16_t>(c, kWsStageB), b, bb, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    if (gemm_i64_run(c, ws<int16_t>(c, kWsStageA), ws<int16_t>(c, kWsStageB), ws<int64_t>(c, kWsStageC), m, k, n))
        return -1;
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(out, ws<int64_t>(c, kWsStageC), ob, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpGemm, ab + bb, ob);
}

extern "C" int volta_cuda_gemm_i64_device(void* raw, uint64_t a_id, size_t a_off, uint64_t b_id, size_t b_off,
                                          uint64_t out_id, size_t out_off, size_t m, size_t k, size_t n) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !m || !k || !n) return fail_message(c, "invalid resident GEMM geometry");
    void *a = nullptr, *b = nullptr, *o = nullptr;
    if (region_elems(c, a_id, a_off, m * k, sizeof(int16_t), &a) ||
        region_elems(c, b_id, b_off, k * n, sizeof(int16_t), &b) ||
        region_elems(c, out_id, out_off, m * n, sizeof(int64_t), &o))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (gemm_i64_run(c, static_cast<const int16_t*>(a), static_cast<const int16_t*>(b), static_cast<int64_t*>(o), m, k,
                     n))
        return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_cuda_gemm_requant_auth(void* raw, const int16_t* a, const int16_t* b, const uint64_t* masks,
                                            int16_t* out, uint64_t* corr, size_t m, size_t k, size_t n,
                                            uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !a || !b || !masks || !out || !corr || !shift || shift >= 63) return -1;
    if (!m || !k || !n) return fail_message(c, "invalid fused GEMM geometry");
    const size_t ab = m * k * 2, bb = k * n * 2, mb = m * n * 8, ob = m * n * 2, cb = m * n * 8;
    if (ensure_ws(c, kWsStageA, ab) || ensure_ws(c, kWsStageB, bb) || ensure_ws(c, kWsStageC, mb) ||
        ensure_ws(c, kWsStageD, ob) || ensure_ws(c, kWsStageE, cb))
        return -1;
    if (op_begin(c)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(ws<int16_t>(c, kWsStageA), a, ab, cudaMemcpyHostToDevice, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(ws<int16_t>(c, kWsStageB), b, bb, cudaMemcpyHostToDevice, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(ws<uint64_t>(c, kWsStageC), masks, mb, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    if (gemm_auth_run(c, ws<int16_t>(c, kWsStageA), ws<int16_t>(c, kWsStageB), ws<uint64_t>(c, kWsStageC),
                      ws<int16_t>(c, kWsStageD), ws<uint64_t>(c, kWsStageE), m, k, n, shift))
        return -1;
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(out, ws<int16_t>(c, kWsStageD), ob, cudaMemcpyDeviceToHost, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(corr, ws<uint64_t>(c, kWsStageE), cb, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpGemm, ab + bb + mb, ob + cb);
}

extern "C" int volta_cuda_gemm_requant_auth_device(void* raw, uint64_t a_id, size_t a_off, uint64_t b_id,
                                                   size_t b_off, uint64_t masks_id, size_t masks_off,
                                                   uint64_t out_id, size_t out_off, uint64_t corr_id,
                                                   size_t corr_off, size_t m, size_t k, size_t n, uint32_t shift) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !m || !k || !n || !shift || shift >= 63) return fail_message(c, "invalid resident fused GEMM geometry");
    void *a = nullptr, *b = nullptr, *mk = nullptr, *o = nullptr, *cr = nullptr;
    if (region_elems(c, a_id, a_off, m * k, sizeof(int16_t), &a) ||
        region_elems(c, b_id, b_off, k * n, sizeof(int16_t), &b) ||
        region_elems(c, masks_id, masks_off, m * n, sizeof(uint64_t), &mk) ||
        region_elems(c, out_id, out_off, m * n, sizeof(int16_t), &o) ||
        region_elems(c, corr_id, corr_off, m * n, sizeof(uint64_t), &cr))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (gemm_auth_run(c, static_cast<const int16_t*>(a), static_cast<const int16_t*>(b),
                      static_cast<const uint64_t*>(mk), static_cast<int16_t*>(o), static_cast<uint64_t*>(cr), m, k, n,
                      shift))
        return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}
