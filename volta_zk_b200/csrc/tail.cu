// Small sumchecks in one CTA (extensions, include/volta_b200_ext.h).
//
// Once the vectors of a sumcheck have at most 2^11 entries, each further
// round is a few microseconds of launch and grid-reduction latency around a
// few hundred field operations.  With the challenges known in advance (the
// clear sink / private transcript draws them from a seeded stream), one CTA
// can run every remaining round back to back in shared memory: evaluate the
// round (exactly the terms of logup_general_round / triple_product_round),
// fold with that round's challenge, reduce the block, write the message,
// repeat.  A LogUp layer job starts either from four vectors or from the
// interleaved children of a fraction-tree level (the deinterleave is the
// load), builds its suffix-eq tables in shared memory from its claim point,
// and ends with the four split values.  Independent jobs run as separate
// CTAs of one launch.
#include "reduce.cuh"
#include "runtime.cuh"

namespace vzb {
namespace {

constexpr int kTailMaxLog = 11;
constexpr int kTailThreads = 512;
constexpr int kMaxJobs = 64;
constexpr int kTailPer = (1 << kTailMaxLog) / 2 / kTailThreads;  // pairs per thread, at most

struct LayerJob {
    const Fp2* v[4];   // separate vectors (when il_p is null)
    const Fp2* il_p;   // interleaved children: p[2i], p[2i+1], q[2i], q[2i+1]
    const Fp2* il_q;
    const Fp2* point;  // `rounds` claim-point coordinates
    const Fp2* r;      // `rounds` round challenges
    Fp2* out;          // 4 per round, then the 4 final values
    int rounds;
};

struct LayerJobs {
    LayerJob j[kMaxJobs];
};

// Suffix table k (size 2^k) lives at offset 2^k - 1 of `tab`; table k is
// table k-1 expanded by coordinate point[L - k] as its low bit
// (logup.rs:284-305).
__device__ void build_suffix_tables(Fp2* tab, const Fp2* point, int L) {
    if (threadIdx.x == 0) tab[0] = Fp2{1, 0};
    __syncthreads();
    for (int k = 1; k < L; ++k) {
        const Fp2 p = point[L - k];
        const Fp2* in = tab + (1 << (k - 1)) - 1;
        Fp2* o = tab + (1 << k) - 1;
        for (int i = threadIdx.x; i < (1 << (k - 1)); i += blockDim.x) {
            const Fp2 v1 = d2mul(in[i], p);
            o[2 * i] = d2sub(in[i], v1);
            o[2 * i + 1] = v1;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(kTailThreads) logup_layers_kernel(LayerJobs jobs) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const LayerJob& job = jobs.j[blockIdx.x];
    const int L = job.rounds;
    const int n = 1 << L;
    Fp2* v[4];
    Fp2* base = reinterpret_cast<Fp2*>(smem_raw);
    for (int k = 0; k < 4; ++k) v[k] = base + k * n;
    Fp2* tab = base + 4 * n;  // 2^L - 1 entries
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        if (job.il_p) {
            v[0][i] = ldg2(job.il_p + 2 * i);
            v[1][i] = ldg2(job.il_p + 2 * i + 1);
            v[2][i] = ldg2(job.il_q + 2 * i);
            v[3][i] = ldg2(job.il_q + 2 * i + 1);
        } else {
            for (int k = 0; k < 4; ++k) v[k][i] = ldg2(job.v[k] + i);
        }
    }
    build_suffix_tables(tab, job.point, L);  // syncs, also after the loads
    __syncthreads();
    int len = n;
    for (int j = 0; j < L; ++j) {
        const int half = len >> 1;
        const Fp2* S = tab + (1 << (L - 1 - j)) - 1;
        const Fp2 r = ldg2(job.r + j);
        Fp2W w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) f2w_zero(w[e]);
        Fp2 folded[4][kTailPer];
#pragma unroll
        for (int m = 0; m < kTailPer; ++m) {
            const int i = threadIdx.x + m * kTailThreads;
            if (i >= half) break;
            const Fp2 a0 = v[0][2 * i], a1 = v[0][2 * i + 1], b0 = v[1][2 * i], b1 = v[1][2 * i + 1];
            const Fp2 c0 = v[2][2 * i], c1 = v[2][2 * i + 1], d0 = v[3][2 * i], d1 = v[3][2 * i + 1];
            const Fp2 si = S[i];
            const Fp2 a2 = d2add_weak(a1, d2sub(a1, a0)), b2 = d2add_weak(b1, d2sub(b1, b0));
            const Fp2 c2 = d2add_weak(c1, d2sub(c1, c0)), d2 = d2add_weak(d1, d2sub(d1, d0));
            Fp2W t;
            f2w_zero(t);
            f2w_mac(t, a0, d0);
            f2w_mac(t, b0, c0);
            f2w_mac(w[0], si, f2w_reduce(t));
            f2w_zero(t);
            f2w_mac(t, a2, d2);
            f2w_mac(t, b2, c2);
            f2w_mac(w[1], si, f2w_reduce(t));
            f2w_mac(w[2], si, d2mul(c0, d0));
            f2w_mac(w[3], si, d2mul(c2, d2));
            folded[0][m] = d2fold(a0, a1, r);
            folded[1][m] = d2fold(b0, b1, r);
            folded[2][m] = d2fold(c0, c1, r);
            folded[3][m] = d2fold(d0, d1, r);
        }
        __syncthreads();  // every pair is read before any folded value lands
#pragma unroll
        for (int m = 0; m < kTailPer; ++m) {
            const int i = threadIdx.x + m * kTailThreads;
            if (i >= half) break;
#pragma unroll
            for (int k = 0; k < 4; ++k) v[k][i] = folded[k][m];
        }
        Acc<4> acc;
#pragma unroll
        for (int e = 0; e < 4; ++e) acc.v[e] = f2w_reduce(w[e]);
        acc = block_sum<4>(acc);  // its barriers also publish the folded values
        if (threadIdx.x == 0)
            for (int e = 0; e < 4; ++e) st2(job.out + 4 * j + e, acc.v[e]);
        len = half;
    }
    if (threadIdx.x < 4) st2(job.out + 4 * L + threadIdx.x, v[threadIdx.x][0]);
}

__global__ void __launch_bounds__(kTailThreads) triple_tail_kernel(const Fp2* a, const Fp2* b, const Fp2* c, int L,
                                                                   const Fp2* rs, Fp2* out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int n = 1 << L;
    Fp2* v[3];
    Fp2* base = reinterpret_cast<Fp2*>(smem_raw);
    for (int k = 0; k < 3; ++k) v[k] = base + k * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        v[0][i] = ldg2(a + i);
        v[1][i] = ldg2(b + i);
        v[2][i] = ldg2(c + i);
    }
    __syncthreads();
    int len = n;
    for (int j = 0; j < L; ++j) {
        const int half = len >> 1;
        const Fp2 r = ldg2(rs + j);
        Fp2W w[3];
#pragma unroll
        for (int e = 0; e < 3; ++e) f2w_zero(w[e]);
        Fp2 folded[3][kTailPer];
#pragma unroll
        for (int m = 0; m < kTailPer; ++m) {
            const int i = threadIdx.x + m * kTailThreads;
            if (i >= half) break;
            Fp2 x0[3], x1[3];
#pragma unroll
            for (int k = 0; k < 3; ++k) {
                x0[k] = v[k][2 * i];
                x1[k] = v[k][2 * i + 1];
            }
            const Fp2 da = d2sub(x1[0], x0[0]), db = d2sub(x1[1], x0[1]), dc = d2sub(x1[2], x0[2]);
            const Fp2 a2 = d2add_weak(x1[0], da), b2 = d2add_weak(x1[1], db), c2 = d2add_weak(x1[2], dc);
            const Fp2 a3 = d2add_weak(a2, da), b3 = d2add_weak(b2, db), c3 = d2add_weak(c2, dc);
            f2w_mac(w[0], d2mul(x0[0], x0[1]), x0[2]);
            f2w_mac(w[1], d2mul(a2, b2), c2);
            f2w_mac(w[2], d2mul(a3, b3), c3);
#pragma unroll
            for (int k = 0; k < 3; ++k) folded[k][m] = d2fold(x0[k], x1[k], r);
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < kTailPer; ++m) {
            const int i = threadIdx.x + m * kTailThreads;
            if (i >= half) break;
#pragma unroll
            for (int k = 0; k < 3; ++k) v[k][i] = folded[k][m];
        }
        Acc<3> acc;
#pragma unroll
        for (int e = 0; e < 3; ++e) acc.v[e] = f2w_reduce(w[e]);
        acc = block_sum<3>(acc);
        if (threadIdx.x == 0)
            for (int e = 0; e < 3; ++e) st2(out + 3 * j + e, acc.v[e]);
        len = half;
    }
    if (threadIdx.x < 3) st2(out + 3 * L + threadIdx.x, v[threadIdx.x][0]);
}

template <class P>
int typed_region(Context* c, uint64_t id, size_t off, size_t count, P*& out) {
    void* p = nullptr;
    if (region_elems(c, id, off, count, sizeof(P), &p)) return -1;
    out = static_cast<P*>(p);
    return 0;
}

// All rounds of a product sumcheck on two vectors of 2^L <= 2^11 entries:
// per round [g(0), g(2)] of a*b (as fp2_product_round) then the fold with
// that round's challenge; out: 2 per round, then the two final values.
__global__ void __launch_bounds__(kTailThreads) product_tail_kernel(const Fp2* a, const Fp2* b, int L, const Fp2* rs,
                                                                    Fp2* out) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    const int n = 1 << L;
    Fp2* v[2];
    Fp2* base = reinterpret_cast<Fp2*>(smem_raw);
    for (int k = 0; k < 2; ++k) v[k] = base + k * n;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        v[0][i] = ldg2(a + i);
        v[1][i] = ldg2(b + i);
    }
    __syncthreads();
    int len = n;
    for (int j = 0; j < L; ++j) {
        const int half = len >> 1;
        const Fp2 r = ldg2(rs + j);
        Fp2W w[2];
        f2w_zero(w[0]);
        f2w_zero(w[1]);
        Fp2 folded[2][kTailPer];
#pragma unroll
        for (int m = 0; m < kTailPer; ++m) {
            const int i = threadIdx.x + m * kTailThreads;
            if (i >= half) break;
            const Fp2 a0 = v[0][2 * i], a1 = v[0][2 * i + 1], b0 = v[1][2 * i], b1 = v[1][2 * i + 1];
            f2w_mac(w[0], a0, b0);
            f2w_mac(w[1], d2add_weak(a1, d2sub(a1, a0)), d2add_weak(b1, d2sub(b1, b0)));
            folded[0][m] = d2fold(a0, a1, r);
            folded[1][m] = d2fold(b0, b1, r);
        }
        __syncthreads();
#pragma unroll
        for (int m = 0; m < kTailPer; ++m) {
            const int i = threadIdx.x + m * kTailThreads;
            if (i >= half) break;
            v[0][i] = folded[0][m];
            v[1][i] = folded[1][m];
        }
        Acc<2> acc;
        acc.v[0] = f2w_reduce(w[0]);
        acc.v[1] = f2w_reduce(w[1]);
        acc = block_sum<2>(acc);
        if (threadIdx.x == 0) {
            st2(out + 2 * j, acc.v[0]);
            st2(out + 2 * j + 1, acc.v[1]);
        }
        len = half;
    }
    if (threadIdx.x < 2) st2(out + 2 * L + threadIdx.x, v[threadIdx.x][0]);
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_b200_logup_layers_device(void* raw, const vzb_layer_job* jobs, size_t count) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !jobs || !count) return fail_message(c, "invalid LogUp layer jobs");
    for (size_t first = 0; first < count; first += kMaxJobs) {
        const size_t batch = count - first < kMaxJobs ? count - first : kMaxJobs;
        LayerJobs lj{};
        int max_log = 0;
        for (size_t i = 0; i < batch; ++i) {
            const vzb_layer_job& in = jobs[first + i];
            LayerJob& j = lj.j[i];
            if (in.rounds > static_cast<size_t>(kTailMaxLog))
                return fail_message(c, "LogUp layer job beyond 2^11 entries");
            const size_t L = in.rounds, n = size_t{1} << L;
            j.rounds = static_cast<int>(L);
            max_log = j.rounds > max_log ? j.rounds : max_log;
            if (in.il_p_id) {
                if (typed_region(c, in.il_p_id, in.il_offset, 2 * n, j.il_p) ||
                    typed_region(c, in.il_q_id, in.il_offset, 2 * n, j.il_q))
                    return -1;
            } else {
                for (int k = 0; k < 4; ++k)
                    if (typed_region(c, in.v_id[k], in.v_offset[k], n, j.v[k])) return -1;
            }
            if (L && (typed_region(c, in.point_id, in.point_offset, L, j.point) ||
                      typed_region(c, in.r_id, in.r_offset, L, j.r)))
                return -1;
            if (typed_region(c, in.out_id, in.out_offset, 4 * L + 4, j.out)) return -1;
        }
        const size_t smem = (4 * (size_t{1} << max_log) + (size_t{1} << max_log)) * sizeof(Fp2);
        VZB_CUDA(c, cudaFuncSetAttribute(logup_layers_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
        if (op_begin(c) || op_mark(c, 1)) return -1;
        logup_layers_kernel<<<static_cast<unsigned>(batch), kTailThreads, smem, c->stream>>>(lj);
        VZB_LAUNCHED(c);
        if (op_mark(c, 2) || op_finish(c, kOpLogup, 0, 0)) return -1;
    }
    return 0;
}

extern "C" int volta_b200_triple_tail_device(void* raw, uint64_t a_id, uint64_t b_id, uint64_t c_id, size_t len,
                                             uint64_t r_id, size_t r_offset, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !len || (len & (len - 1)) || len > (size_t{1} << kTailMaxLog))
        return fail_message(c, "invalid triple-product tail geometry");
    int L = 0;
    while ((size_t{1} << L) < len) ++L;
    const Fp2 *a = nullptr, *b = nullptr, *cc = nullptr, *r = nullptr;
    Fp2* out = nullptr;
    if (typed_region(c, a_id, 0, len, a) || typed_region(c, b_id, 0, len, b) || typed_region(c, c_id, 0, len, cc) ||
        (L && typed_region(c, r_id, r_offset, L, r)) || typed_region(c, out_id, out_offset, 3 * L + 3, out))
        return -1;
    const size_t smem = 3 * len * sizeof(Fp2);
    VZB_CUDA(c, cudaFuncSetAttribute(triple_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    if (op_begin(c) || op_mark(c, 1)) return -1;
    triple_tail_kernel<<<1, kTailThreads, smem, c->stream>>>(a, b, cc, L, r, out);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}

extern "C" int volta_b200_product_tail_device(void* raw, uint64_t a_id, uint64_t b_id, size_t len, uint64_t r_id,
                                              size_t r_offset, uint64_t out_id, size_t out_offset) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !len || (len & (len - 1)) || len > (size_t{1} << kTailMaxLog))
        return fail_message(c, "invalid product tail geometry");
    int L = 0;
    while ((size_t{1} << L) < len) ++L;
    const Fp2 *a = nullptr, *b = nullptr, *r = nullptr;
    Fp2* out = nullptr;
    if (typed_region(c, a_id, 0, len, a) || typed_region(c, b_id, 0, len, b) ||
        (L && typed_region(c, r_id, r_offset, L, r)) || typed_region(c, out_id, out_offset, 2 * L + 2, out))
        return -1;
    const size_t smem = 2 * len * sizeof(Fp2);
    if (smem > 48 * 1024)
        VZB_CUDA(c, cudaFuncSetAttribute(product_tail_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(smem)));
    if (op_begin(c) || op_mark(c, 1)) return -1;
    product_tail_kernel<<<1, kTailThreads, smem, c->stream>>>(a, b, L, r, out);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpGemm, 0, 0);
}
