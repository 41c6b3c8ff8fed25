// Single-launch reductions of K Fp2 accumulators.
//
// Every sumcheck round message in the reference is a sum over pairs followed
// by a log-depth chain of relaunched pairwise reduce kernels
// (cuda/volta_cuda_backend.cu:2091, 2161, 2798).  Here a grid-stride
// evaluation accumulates in registers, warps reduce with shuffles, blocks
// publish one partial each and the last block to finish folds the partials
// and runs the epilogue, all in one launch.  Field addition is exact, so the
// result equals the reference's bit for bit regardless of order.
#pragma once

#include "field.cuh"

namespace vzb {

constexpr int kReduceThreads = 256;

template <int K>
struct Acc {
    Fp2 v[K];
    __device__ __forceinline__ void zero() {
#pragma unroll
        for (int k = 0; k < K; ++k) v[k] = Fp2{0, 0};
    }
    __device__ __forceinline__ void add(const Acc& o) {
#pragma unroll
        for (int k = 0; k < K; ++k) v[k] = f2add(v[k], o.v[k]);
    }
};

// Sum of `a` over the block (up to 1024 threads); valid in thread 0.
template <int K>
__device__ __forceinline__ Acc<K> block_sum(Acc<K> a) {
    __shared__ Fp2 sm[K][32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int d = 16; d > 0; d >>= 1)
#pragma unroll
        for (int k = 0; k < K; ++k) a.v[k] = f2add(a.v[k], shfl_down2(a.v[k], d));
    if (lane == 0)
#pragma unroll
        for (int k = 0; k < K; ++k) sm[k][warp] = a.v[k];
    __syncthreads();
    const int warps = (blockDim.x + 31) >> 5;
    if (warp == 0) {
#pragma unroll
        for (int k = 0; k < K; ++k) a.v[k] = lane < warps ? sm[k][lane] : Fp2{0, 0};
#pragma unroll
        for (int d = 16; d > 0; d >>= 1)
#pragma unroll
            for (int k = 0; k < K; ++k) a.v[k] = f2add(a.v[k], shfl_down2(a.v[k], d));
    }
    __syncthreads();
    return a;
}

// Reduce the per-thread accumulators of the whole grid; the last block hands
// the total to `epi(total)` in thread 0.  `partials` holds gridDim.x * K Fp2
// and `counter` is a zeroed u32 that the last block resets.
template <int K, class Epi>
__device__ __forceinline__ void grid_finish(Acc<K> a, Fp2* partials, unsigned* counter,
                                            const Epi& epi) {
    a = block_sum<K>(a);
    if (gridDim.x == 1) {
        if (threadIdx.x == 0) epi(a);
        return;
    }
    __shared__ bool last;
    if (threadIdx.x == 0) {
#pragma unroll
        for (int k = 0; k < K; ++k) st2(partials + static_cast<size_t>(blockIdx.x) * K + k, a.v[k]);
        __threadfence();
        last = atomicAdd(counter, 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last) return;
    __threadfence();
    Acc<K> t;
    t.zero();
    for (unsigned b = threadIdx.x; b < gridDim.x; b += blockDim.x) {
#pragma unroll
        for (int k = 0; k < K; ++k) {
            const ulonglong2 v = __ldcg(reinterpret_cast<const ulonglong2*>(partials + static_cast<size_t>(b) * K + k));
            t.v[k] = f2add(t.v[k], Fp2{v.x, v.y});
        }
    }
    t = block_sum<K>(t);
    if (threadIdx.x == 0) {
        epi(t);
        *counter = 0;
    }
}

#ifdef __CUDACC__
// Grid-stride evaluation into lazily reduced accumulators (sums of 128-bit
// products, one canonical reduction per accumulator per thread), then the
// single-launch grid reduction.  `eval(i, w)` adds item i's terms into w[K].
template <int K, class Eval, class Epi>
__global__ void __launch_bounds__(kReduceThreads) reduce_wide_kernel(Eval eval, size_t items, Fp2* partials,
                                                                     unsigned* counter, Epi epi) {
    Fp2W w[K];
#pragma unroll
    for (int k = 0; k < K; ++k) f2w_zero(w[k]);
    const size_t stride = static_cast<size_t>(gridDim.x) * blockDim.x;
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < items; i += stride)
        eval(i, w);
    Acc<K> acc;
#pragma unroll
    for (int k = 0; k < K; ++k) acc.v[k] = f2w_reduce(w[k]);
    grid_finish<K>(acc, partials, counter, epi);
}
#endif

// Epilogue that stores the K sums, optionally multiplied by a scale.
// When `flag` is set (host-bound message in the mapped mailbox) the message
// is published by a system-scope fence followed by the sequence number.
template <int K>
struct StoreEpi {
    Fp2* out;
    Fp2 scale;
    bool scaled;
    unsigned* flag;
    unsigned seq;
    __device__ __forceinline__ void operator()(const Acc<K>& a) const {
#pragma unroll
        for (int k = 0; k < K; ++k) out[k] = scaled ? f2mul(a.v[k], scale) : a.v[k];
        if (flag) {
            __threadfence_system();
            *reinterpret_cast<volatile unsigned*>(flag) = seq;
        }
    }
};

}  // namespace vzb
