// LogUp fraction tree (Papini-Haboeck GKR) and leaf materialisation.
//
// Semantics: rust/volta-proto/src/logup.rs:136-240 (build_tree_cpu) with the
// flattened root-to-leaf layout of rust/volta-accel/src/lib.rs:5511-5513
// (level k, 2^k nodes, at offset 2^k - 1).  Reference entry points:
// cuda/volta_cuda_backend.cu:6581-6653.
//
// B200 design: the reference launches one kernel per level (24 launches for
// 2^24 leaves, each a full HBM pass over its level).  Here one block owns a
// 2^11-leaf tile, performs the structured first combine and the next ten
// general combines in shared memory and writes every level it produced;
// a 2^24-leaf tree takes three launches and reads the leaves once.
#include "runtime.cuh"

namespace vzb {

constexpr int kTreeTileBits = 11;
constexpr int kTreeTile = 1 << kTreeTileBits;  // children per block

__device__ __forceinline__ Fp2 shfl_idx2(Fp2 v, int src) {
    return Fp2{__shfl_sync(0xffffffffu, v.c0, src), __shfl_sync(0xffffffffu, v.c1, src)};
}

// Parent of two fractions: p = pa qb + pb qa (one lazy sum, one reduction),
// q = qa qb, on the carry-chain arithmetic.
__device__ __forceinline__ void combine(Fp2 pa, Fp2 pb, Fp2 qa, Fp2 qb, Fp2& p, Fp2& q) {
    Fp2W t;
    f2w_zero(t);
    f2w_mac(t, pa, qb);
    f2w_mac(t, pb, qa);
    p = f2w_reduce(t);
    q = d2mul(qa, qb);
}

// Combine `levels` times starting from a child level of 2^child_bits entries.
// first == true: children are leaves (a_i, alpha1) with numerators 1 or -mult.
// kColumn: the leaves are alpha0 - leaf[i] (`leaf` is a query column).
template <bool kFirst, bool kColumn = false>
__global__ void __launch_bounds__(256, 4) tree_tile_kernel(
    const uint64_t* __restrict__ leaf, const uint32_t* __restrict__ mult, const Fp2* __restrict__ cp,
    const Fp2* __restrict__ cq, Fp2* __restrict__ p, Fp2* __restrict__ q, int child_bits, int levels,
    uint64_t alpha1, uint64_t w7a1sq, int neg_mult, uint64_t alpha0 = 0) {
    // Two shared buffers in turn (level k in A, k + 1 in B, ...): a level
    // reads one and writes the other, so one barrier per level suffices.
    __shared__ Fp2 ap[kTreeTile / 2], aq[kTreeTile / 2], bp[kTreeTile / 4], bq[kTreeTile / 4];
    const size_t tile = size_t{1} << levels;  // children handled by this block
    const size_t child0 = static_cast<size_t>(blockIdx.x) * tile;
    // first combine into shared memory, level child_bits - 1; the loop is
    // unrolled over its at most 4 parents per thread so that all of a thread's
    // loads can be in flight before the first combine (the outputs are
    // __restrict__, so no store orders them)
    int half = static_cast<int>(tile / 2);
    {
        const int lvl = child_bits - 1;
        Fp2* po = p + ((size_t{1} << lvl) - 1) + child0 / 2;
        Fp2* qo = q + ((size_t{1} << lvl) - 1) + child0 / 2;
        constexpr int kPer = kTreeTile / 2 / 256;
#pragma unroll
        for (int m = 0; m < kPer; ++m) {
            const int i = threadIdx.x + m * 256;
            if (i >= half) break;
            Fp2 pv, qv;
            if (kFirst) {
                uint64_t a = __ldcs(leaf + child0 + 2 * i), b = __ldcs(leaf + child0 + 2 * i + 1);
                if (kColumn) {
                    a = dsub(alpha0, a);
                    b = dsub(alpha0, b);
                }
                const uint64_t sum = dadd(a, b);
                if (neg_mult) {
                    const uint64_t ma = __ldcs(mult + child0 + 2 * i), mb = __ldcs(mult + child0 + 2 * i + 1);
                    pv = Fp2{dsub(0, dadd(dmul(ma, b), dmul(mb, a))), dsub(0, dmul(dadd(ma, mb), alpha1))};
                } else {
                    pv = Fp2{sum, dadd(alpha1, alpha1)};
                }
                qv = Fp2{dadd(dmul(a, b), w7a1sq), dmul(sum, alpha1)};
            } else {
                const Fp2 pa = ldcs2(cp + child0 + 2 * i), pb = ldcs2(cp + child0 + 2 * i + 1);
                const Fp2 qa = ldcs2(cq + child0 + 2 * i), qb = ldcs2(cq + child0 + 2 * i + 1);
                combine(pa, pb, qa, qb, pv, qv);
            }
            ap[i] = pv;
            aq[i] = qv;
            st2(po + i, pv);
            st2(qo + i, qv);
        }
    }
    __syncthreads();
    // remaining combines inside the tile through shared memory while a level
    // has more than 32 nodes ...
    int step = 1;
    bool in_a = true;
    for (; step < levels && half > 32; ++step) {
        const int parents = half / 2;
        const int lvl = child_bits - 1 - step;
        const size_t base = child0 >> (step + 1);
        Fp2* po = p + ((size_t{1} << lvl) - 1) + base;
        Fp2* qo = q + ((size_t{1} << lvl) - 1) + base;
        const Fp2 *sp = in_a ? ap : bp, *sq = in_a ? aq : bq;
        Fp2 *dp = in_a ? bp : ap, *dq = in_a ? bq : aq;
        for (int i = threadIdx.x; i < parents; i += 256) {
            Fp2 np, nq;
            combine(sp[2 * i], sp[2 * i + 1], sq[2 * i], sq[2 * i + 1], np, nq);
            dp[i] = np;
            dq[i] = nq;
            st2(po + i, np);
            st2(qo + i, nq);
        }
        __syncthreads();
        half = parents;
        in_a = !in_a;
    }
    // ... then warp 0 alone, node j of a level in lane j, with shuffles
    if (step < levels && threadIdx.x < 32) {
        const int lane = threadIdx.x;
        const Fp2 *sp = in_a ? ap : bp, *sq = in_a ? aq : bq;
        Fp2 pv = lane < half ? sp[lane] : Fp2{0, 0};
        Fp2 qv = lane < half ? sq[lane] : Fp2{0, 0};
        for (; step < levels; ++step) {
            const int parents = half / 2;
            const int lvl = child_bits - 1 - step;
            const size_t base = child0 >> (step + 1);
            const int a = (2 * lane) & 31, b = (2 * lane + 1) & 31;
            const Fp2 pa = shfl_idx2(pv, a), pb = shfl_idx2(pv, b), qa = shfl_idx2(qv, a), qb = shfl_idx2(qv, b);
            if (lane < parents) {
                combine(pa, pb, qa, qb, pv, qv);
                st2(p + ((size_t{1} << lvl) - 1) + base + lane, pv);
                st2(q + ((size_t{1} << lvl) - 1) + base + lane, qv);
            }
            half = parents;
        }
    }
}

__global__ void materialize_leaves_kernel(const uint64_t* leaf, const uint32_t* mult, Fp2* p, Fp2* q,
                                          size_t n, uint64_t alpha1, int neg_mult) {
    const size_t gs = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += gs) {
        st2(p + i, neg_mult ? Fp2{fneg(static_cast<uint64_t>(mult[i])), 0} : Fp2{1, 0});
        st2(q + i, Fp2{leaf[i], alpha1});
    }
}

int build_tree(Context* c, const uint64_t* leaf, const uint32_t* mult, size_t n, uint64_t alpha1,
               int neg_mult, Fp2* p, Fp2* q, bool column = false, uint64_t alpha0 = 0) {
    int depth = 0;
    while ((size_t{1} << depth) < n) ++depth;
    const uint64_t w7a1sq = fmul7(fmul(alpha1, alpha1));
    int child_bits = depth;
    bool first = true;
    while (child_bits > 0) {
        const int levels = child_bits < kTreeTileBits ? child_bits : kTreeTileBits;
        const unsigned blocks = static_cast<unsigned>((size_t{1} << child_bits) >> levels);
        if (first && column) {
            tree_tile_kernel<true, true><<<blocks, 256, 0, c->stream>>>(leaf, nullptr, nullptr, nullptr, p, q,
                                                                        child_bits, levels, alpha1, w7a1sq, 0,
                                                                        alpha0);
        } else if (first) {
            tree_tile_kernel<true><<<blocks, 256, 0, c->stream>>>(leaf, mult, nullptr, nullptr, p, q,
                                                                  child_bits, levels, alpha1, w7a1sq,
                                                                  neg_mult);
        } else {
            const size_t off = (size_t{1} << child_bits) - 1;
            tree_tile_kernel<false><<<blocks, 256, 0, c->stream>>>(nullptr, nullptr, p + off, q + off,
                                                                   p, q, child_bits, levels, alpha1,
                                                                   w7a1sq, neg_mult);
        }
        VZB_LAUNCHED(c);
        child_bits -= levels;
        first = false;
    }
    return 0;
}

}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_logup_tree(void* raw, const uint64_t* leaf, const uint32_t* mult, size_t n,
                                     uint64_t alpha1, int neg_mult, Fp2* hp, Fp2* hq) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !leaf || !hp || !hq || n < 2 || (n & (n - 1)) || (neg_mult && !mult)) return -1;
    const size_t lb = n * 8, mb = neg_mult ? n * 4 : 0, tb = (n - 1) * sizeof(Fp2);
    if (ensure_ws(c, kWsStageA, lb) || ensure_ws(c, kWsStageB, mb ? mb : 16) ||
        ensure_ws(c, kWsStageC, tb) || ensure_ws(c, kWsStageD, tb))
        return -1;
    if (op_begin(c)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(c->ws[kWsStageA].ptr, leaf, lb, cudaMemcpyHostToDevice, c->stream));
    if (neg_mult)
        VZB_CUDA(c, cudaMemcpyAsync(c->ws[kWsStageB].ptr, mult, mb, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    if (build_tree(c, ws<uint64_t>(c, kWsStageA), ws<uint32_t>(c, kWsStageB), n, alpha1, neg_mult,
                   ws<Fp2>(c, kWsStageC), ws<Fp2>(c, kWsStageD)))
        return -1;
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(hp, c->ws[kWsStageC].ptr, tb, cudaMemcpyDeviceToHost, c->stream));
    VZB_CUDA(c, cudaMemcpyAsync(hq, c->ws[kWsStageD].ptr, tb, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpLogup, lb + mb, 2 * tb);
}

extern "C" int volta_cuda_logup_tree_device(void* raw, uint64_t leaf_id, size_t leaf_off,
                                            uint64_t mult_id, size_t mult_off, size_t n,
                                            uint64_t alpha1, int neg_mult, uint64_t p_id,
                                            size_t p_off, uint64_t q_id, size_t q_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || n < 2 || (n & (n - 1)) || (neg_mult && !mult_id))
        return fail_message(c, "invalid resident LogUp tree geometry");
    void *leaf = nullptr, *mult = nullptr, *p = nullptr, *q = nullptr;
    if (region_elems(c, leaf_id, leaf_off, n, sizeof(uint64_t), &leaf) ||
        (neg_mult && region_elems(c, mult_id, mult_off, n, sizeof(uint32_t), &mult)) ||
        region_elems(c, p_id, p_off, n - 1, sizeof(Fp2), &p) ||
        region_elems(c, q_id, q_off, n - 1, sizeof(Fp2), &q))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (build_tree(c, static_cast<const uint64_t*>(leaf), static_cast<const uint32_t*>(mult), n, alpha1,
                   neg_mult, static_cast<Fp2*>(p), static_cast<Fp2*>(q)))
        return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_cuda_logup_materialize_leaves_device(void* raw, uint64_t leaf_id,
                                                          size_t leaf_off, uint64_t mult_id,
                                                          size_t mult_off, size_t n,
                                                          uint64_t alpha1, int neg_mult,
                                                          uint64_t p_id, size_t p_off,
                                                          uint64_t q_id, size_t q_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !n || (neg_mult && !mult_id)) return fail_message(c, "invalid resident LogUp leaf geometry");
    void *leaf = nullptr, *mult = nullptr, *p = nullptr, *q = nullptr;
    if (region_elems(c, leaf_id, leaf_off, n, sizeof(uint64_t), &leaf) ||
        (neg_mult && region_elems(c, mult_id, mult_off, n, sizeof(uint32_t), &mult)) ||
        region_elems(c, p_id, p_off, n, sizeof(Fp2), &p) || region_elems(c, q_id, q_off, n, sizeof(Fp2), &q))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    materialize_leaves_kernel<<<grid_for(c, n, 256), 256, 0, c->stream>>>(
        static_cast<const uint64_t*>(leaf), static_cast<const uint32_t*>(mult), static_cast<Fp2*>(p),
        static_cast<Fp2*>(q), n, alpha1, neg_mult);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}

extern "C" int volta_b200_logup_tree_column_device(void* raw, uint64_t col_id, size_t col_off, uint64_t alpha0,
                                                   size_t n, uint64_t alpha1, uint64_t p_id, size_t p_off,
                                                   uint64_t q_id, size_t q_off) {
    Context* c = static_cast<Context*>(raw);
    if (!c || n < 2 || (n & (n - 1)) || alpha0 >= kP || alpha1 >= kP)
        return fail_message(c, "invalid resident LogUp column-tree geometry");
    void *col = nullptr, *p = nullptr, *q = nullptr;
    if (region_elems(c, col_id, col_off, n, sizeof(uint64_t), &col) ||
        region_elems(c, p_id, p_off, n - 1, sizeof(Fp2), &p) || region_elems(c, q_id, q_off, n - 1, sizeof(Fp2), &q))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (build_tree(c, static_cast<const uint64_t*>(col), nullptr, n, alpha1, 0, static_cast<Fp2*>(p),
                   static_cast<Fp2*>(q), true, alpha0))
        return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpLogup, 0, 0);
}
