// Witness GEMMs on the tensor cores (seam entry points
// cuda/volta_cuda_backend.cu:4128-4200; semantics rust/volta-gpt2/src/gemm.rs):
//   gemm_i64            acc = a b exactly (i64)
//   gemm_requant_auth   y = clamp(round_half_up(acc / 2^s)) as i16 and the MAC
//                       correction corr = embed(y) - mask (gemm.rs:19-22, 120-154)
#include "gemm.cuh"

namespace vzb {

// One thread per 16-byte core-matrix row of the output planes (consecutive
// threads write consecutive 16-byte chunks).
__global__ void split_planes_kernel(const int16_t* x, size_t rows, size_t k, size_t ld, int8_t* hi, uint8_t* lo,
                                    size_t kp, size_t rpad, unsigned batches, size_t boff) {
    const size_t per = rpad * kp / 16, total = per * batches;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t b = z / per, q = z - b * per;
        // q -> (k-slice, row group, 16-byte chunk, row in group), the order of plane_off
        const size_t slice = q / (rpad * 4), rem = q - slice * rpad * 4;
        const size_t r = (rem >> 5) * 8 + (rem & 7), k0 = slice * 64 + ((rem >> 3) & 3) * 16;
        uint32_t h[4] = {0, 0, 0, 0}, l[4] = {0, 0, 0, 0};
        if (r < rows) {
            const int16_t* src = x + b * boff + r * ld;
#pragma unroll
            for (int t = 0; t < 16; ++t) {
                const size_t kk = k0 + t;
                const uint32_t v = kk < k ? static_cast<uint16_t>(src[kk]) : 0u;
                h[t >> 2] |= (v >> 8) << (8 * (t & 3));
                l[t >> 2] |= (v & 0xFFu) << (8 * (t & 3));
            }
        }
        const size_t off = b * rpad * kp + q * 16;
        *reinterpret_cast<uint4*>(hi + off) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(lo + off) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}

// 32 x 32 tiles through shared memory: coalesced reads of x rows; blockIdx.z
// is the batch; rows n..npad of the planes are written as zeros.
__global__ void split_planes_t_kernel(const int16_t* x, size_t k, size_t n, size_t ld, int8_t* hi, uint8_t* lo,
                                      size_t kp, size_t npad, size_t boff) {
    __shared__ int16_t t[32][33];
    const size_t k0 = static_cast<size_t>(blockIdx.x) * 32, n0 = static_cast<size_t>(blockIdx.y) * 32;
    const size_t b = blockIdx.z;
    x += b * boff;
    hi += b * npad * kp;
    lo += b * npad * kp;
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const size_t kk = k0 + r, nn = n0 + threadIdx.x;
        t[r][threadIdx.x] = (kk < k && nn < n) ? x[kk * ld + nn] : 0;
    }
    __syncthreads();
    for (int r = threadIdx.y; r < 32; r += blockDim.y) {
        const size_t nn = n0 + r, kk = k0 + threadIdx.x;
        if (nn < npad && kk < kp) {
            const int v = t[threadIdx.x][r];
            const size_t o = plane_off(nn, kk, npad);
            hi[o] = static_cast<int8_t>(v >> 8);
            lo[o] = static_cast<uint8_t>(v & 0xFF);
        }
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
        const dim3 grid(static_cast<unsigned>(kp / 32), static_cast<unsigned>(npad / 32), batches);
        if (grid.y > 65535 || grid.z > 65535) return fail_message(c, "GEMM column count exceeds the launch grid");
        split_planes_t_kernel<<<grid, dim3(32, 8), 0, c->stream>>>(b, k, n, ldb, const_cast<int8_t*>(out->b_hi),
                                                                   const_cast<uint8_t*>(out->b_lo), kp, npad, b_boff);
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
