// Ligero column commitment: BLAKE3 column leaves and the binary Merkle tree
// over them (rust/volta-pcs/src/ligero.rs:351-359, 595-616 and
// merkle.rs:9-79; seam entry points cuda/volta_cuda_backend.cu:7151-7264).
//
//   leaf(col)      = BLAKE3(LE bytes of column col: rows x u64, or rows x
//                    (c0, c1) for Fp2), the standard unkeyed hash (1 KiB
//                    chunks, binary chunk tree, ROOT flag on the last
//                    compression).  BLAKE3 is the third-party crate blake3
//                    1.8.5; the compression function below is written from
//                    the published BLAKE3 specification.
//   parent(l, r)   = BLAKE3(l || r) (a single 64-byte block).
//   tree storage   = levels leaf -> root, (2 cols - 1) x 32 B, root last.
//
// B200 design.  The reference hashes one column per thread (65,536 threads,
// 64 chunks each in series, then one launch per tree level).  Here a CTA
// owns 32 adjacent columns: its 8 warps hash the chunks of those columns in
// parallel (each warp reads 32 adjacent columns of one row = 256 contiguous
// bytes per load), the chunk chaining values meet in shared memory where the
// chunk tree is merged level by level, and the same CTA then builds the 5
// Merkle levels above its 32 leaves.  One more launch finishes the tree from
// the cols/32 subtree roots.  Compression count equals the reference's.
#include "runtime.cuh"

namespace vzb {
namespace {

constexpr uint32_t kChunkStart = 1, kChunkEnd = 2, kParent = 4, kRoot = 8;
constexpr int kColsPerCta = 32;
constexpr int kHashWarps = 8;
constexpr int kMaxSmemChunks = 64;  // chunk CVs of 32 columns kept in shared memory (64 KiB)

struct H32 {
    uint32_t w[8];
};

__device__ __constant__ uint32_t kIv[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                                           0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};

__device__ __forceinline__ uint32_t rotr32(uint32_t x, int n) { return __funnelshift_r(x, x, n); }

#define VZB_G(a, b, c, d, x, y)           \
    do {                                  \
        s[a] = s[a] + s[b] + (x);         \
        s[d] = rotr32(s[d] ^ s[a], 16);   \
        s[c] = s[c] + s[d];               \
        s[b] = rotr32(s[b] ^ s[c], 12);   \
        s[a] = s[a] + s[b] + (y);         \
        s[d] = rotr32(s[d] ^ s[a], 8);    \
        s[c] = s[c] + s[d];               \
        s[b] = rotr32(s[b] ^ s[c], 7);    \
    } while (0)

// BLAKE3 compression (specification section 2.2): 7 rounds of the
// column/diagonal G steps with the fixed message permutation between rounds.
// Returns the first 8 output words (the chaining value / hash).
__device__ __forceinline__ H32 compress(const uint32_t cv[8], const uint32_t m_in[16], uint64_t counter,
                                        uint32_t block_len, uint32_t flags) {
    uint32_t s[16], m[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) s[i] = cv[i];
#pragma unroll
    for (int i = 0; i < 4; ++i) s[8 + i] = kIv[i];
    s[12] = static_cast<uint32_t>(counter);
    s[13] = static_cast<uint32_t>(counter >> 32);
    s[14] = block_len;
    s[15] = flags;
#pragma unroll
    for (int i = 0; i < 16; ++i) m[i] = m_in[i];
#pragma unroll
    for (int r = 0; r < 7; ++r) {
        VZB_G(0, 4, 8, 12, m[0], m[1]);
        VZB_G(1, 5, 9, 13, m[2], m[3]);
        VZB_G(2, 6, 10, 14, m[4], m[5]);
        VZB_G(3, 7, 11, 15, m[6], m[7]);
        VZB_G(0, 5, 10, 15, m[8], m[9]);
        VZB_G(1, 6, 11, 12, m[10], m[11]);
        VZB_G(2, 7, 8, 13, m[12], m[13]);
        VZB_G(3, 4, 9, 14, m[14], m[15]);
        if (r < 6) {  // message permutation 2,6,3,10,7,0,4,13,1,11,12,5,9,14,15,8
            const uint32_t t[16] = {m[2], m[6], m[3], m[10], m[7], m[0], m[4], m[13],
                                    m[1], m[11], m[12], m[5], m[9], m[14], m[15], m[8]};
#pragma unroll
            for (int i = 0; i < 16; ++i) m[i] = t[i];
        }
    }
    H32 h;
#pragma unroll
    for (int i = 0; i < 8; ++i) h.w[i] = s[i] ^ s[i + 8];
    return h;
}
#undef VZB_G

__device__ __forceinline__ H32 parent_cv(const H32& l, const H32& r, uint32_t extra) {
    uint32_t m[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m[i] = l.w[i];
        m[8 + i] = r.w[i];
    }
    return compress(kIv, m, 0, 64, kParent | extra);
}

// Merkle node = BLAKE3 of the 64-byte concatenation: one chunk of one block.
__device__ __forceinline__ H32 merkle_pair(const H32& l, const H32& r) {
    uint32_t m[16];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        m[i] = l.w[i];
        m[8 + i] = r.w[i];
    }
    return compress(kIv, m, 0, 64, kChunkStart | kChunkEnd | kRoot);
}

// Word w (u64) of the column's byte stream.
template <int WPV>
__device__ __forceinline__ uint64_t column_word(const uint64_t* m, size_t cols, size_t col, size_t w) {
    if (WPV == 1) return __ldcs(m + w * cols + col);
    const size_t row = w >> 1;
    return __ldcs(m + 2 * (row * cols + col) + (w & 1));
}

// Chaining value of chunk `chunk` of a column of `words` u64 words, compressed
// with chunk counter `counter`; with `root` set (single-chunk column) the last
// block carries the ROOT flag (and counter 0).
template <int WPV>
__device__ __forceinline__ H32 chunk_cv(const uint64_t* m, size_t cols, size_t col, size_t words, size_t chunk,
                                        uint64_t counter, bool root) {
    const size_t w0 = chunk * 128;
    const size_t take = words - w0 < 128 ? words - w0 : 128;
    const int blocks = static_cast<int>((take + 7) / 8);
    uint32_t cv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) cv[i] = kIv[i];
    H32 h{};
    for (int b = 0; b < blocks; ++b) {
        const size_t bw = take - static_cast<size_t>(b) * 8 < 8 ? take - static_cast<size_t>(b) * 8 : 8;
        uint32_t blk[16];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint64_t x = i < static_cast<int>(bw) ? column_word<WPV>(m, cols, col, w0 + b * 8 + i) : 0;
            blk[2 * i] = static_cast<uint32_t>(x);
            blk[2 * i + 1] = static_cast<uint32_t>(x >> 32);
        }
        const bool last = b + 1 == blocks;
        const uint32_t flags = (b == 0 ? kChunkStart : 0) | (last ? kChunkEnd : 0) | (last && root ? kRoot : 0);
        h = compress(cv, blk, root ? 0 : counter, static_cast<uint32_t>(bw * 8), flags);
#pragma unroll
        for (int i = 0; i < 8; ++i) cv[i] = h.w[i];
    }
    return h;
}

// Offset (in nodes) of Merkle level `l` for `leaves` leaves.
__device__ __host__ __forceinline__ size_t level_offset(size_t leaves, int l) {
    size_t off = 0, len = leaves;
    for (int i = 0; i < l; ++i) {
        off += len;
        len >>= 1;
    }
    return off;
}

// One CTA: 32 adjacent columns.  Leaves (and, when `build` is set, the Merkle
// levels above them up to the CTA's subtree root) go to `tree`.  With `root`
// clear the result per column is the non-root chaining value of the chunk
// subtree whose first chunk has global index chunk_base (a row slab of a
// taller column).
template <int WPV>
__global__ void __launch_bounds__(kColsPerCta * kHashWarps) column_leaves_kernel(const uint64_t* m, size_t rows,
                                                                                  size_t cols, H32* tree,
                                                                                  H32* scratch, int build,
                                                                                  uint64_t chunk_base, int root) {
    extern __shared__ H32 cvs_flat[];  // [min(chunks, 64) or 1][32] chunk CVs, then the subtree nodes
    auto cvs = [&](size_t ch, int ln) -> H32& { return cvs_flat[ch * kColsPerCta + ln]; };
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t col0 = static_cast<size_t>(blockIdx.x) * kColsPerCta;
    const int ncols = static_cast<int>(cols - col0 < kColsPerCta ? cols - col0 : kColsPerCta);
    const size_t col = col0 + lane;
    const size_t words = rows * WPV;
    const size_t chunks = (words + 127) / 128;
    const bool in_smem = chunks <= kMaxSmemChunks;
    // chunk chaining values, warps striding over the chunks
    if (lane < ncols) {
        for (size_t ch = warp; ch < chunks; ch += kHashWarps) {
            const H32 h = chunk_cv<WPV>(m, cols, col, words, ch, chunk_base + ch, chunks == 1 && root);
            if (in_smem)
                cvs(ch, lane) = h;
            else
                scratch[ch * cols + col] = h;
        }
    }
    __syncthreads();
    H32 leaf{};
    if (chunks == 1) {
        leaf = cvs(0, lane);
    } else if (in_smem) {
        // left-balanced chunk tree, merged level by level; ROOT on the last merge
        size_t count = chunks;
        while (count > 1) {
            const size_t pairs = count / 2;
            H32 mine[kMaxSmemChunks / 2 / kHashWarps];
            int nm = 0;
            for (size_t p = warp; p < pairs; p += kHashWarps)
                mine[nm++] = parent_cv(cvs(2 * p, lane), cvs(2 * p + 1, lane), count == 2 && root ? kRoot : 0);
            H32 carry{};
            const bool odd = count & 1;
            if (odd && warp == 0) carry = cvs(count - 1, lane);
            __syncthreads();
            nm = 0;
            for (size_t p = warp; p < pairs; p += kHashWarps) cvs(p, lane) = mine[nm++];
            if (odd && warp == 0) cvs(pairs, lane) = carry;
            __syncthreads();
            count = pairs + (odd ? 1 : 0);
        }
        leaf = cvs(0, lane);
    } else if (warp == 0 && lane < ncols) {
        // long columns: eager stack merge over the chunk CVs in global scratch
        // (complete subtrees merge as soon as they close), the last chunk is
        // pushed unmerged and the right spine folds with ROOT on the final merge
        H32 stack[48];
        int depth = 0;
        for (size_t ch = 0; ch + 1 < chunks; ++ch) {
            H32 cv = scratch[ch * cols + col];
            size_t total = ch;
            while (total & 1) {
                cv = parent_cv(stack[--depth], cv, 0);
                total >>= 1;
            }
            stack[depth++] = cv;
        }
        H32 cv = scratch[(chunks - 1) * cols + col];
        while (depth) {
            --depth;
            cv = parent_cv(stack[depth], cv, depth == 0 && root ? kRoot : 0);
        }
        leaf = cv;
    }
    __syncthreads();
    // leaves and the CTA's Merkle subtree (levels 1..5)
    H32* level_nodes = cvs_flat;
    if (warp == 0) {
        if (lane < ncols) {
            tree[col] = leaf;
            level_nodes[lane] = leaf;
        }
    }
    __syncthreads();
    if (!build) return;
    int len = ncols;  // a power of two (cols is)
    for (int l = 1; len > 1; ++l) {
        const int half = len / 2;
        H32 p{};
        if (threadIdx.x < half) p = merkle_pair(level_nodes[2 * threadIdx.x], level_nodes[2 * threadIdx.x + 1]);
        __syncthreads();
        if (threadIdx.x < half) {
            level_nodes[threadIdx.x] = p;
            tree[level_offset(cols, l) + (col0 >> l) + threadIdx.x] = p;
        }
        __syncthreads();
        len = half;
    }
}

// Merkle levels from `start_level` (len nodes at offset off) upward, one CTA
// with all nodes of the starting level in shared memory.
__global__ void __launch_bounds__(1024) merkle_top_kernel(H32* tree, size_t leaves, int start_level) {
    extern __shared__ H32 nodes[];
    size_t off = level_offset(leaves, start_level);
    size_t len = leaves >> start_level;
    for (size_t i = threadIdx.x; i < len; i += blockDim.x) nodes[i] = tree[off + i];
    __syncthreads();
    int l = start_level;
    while (len > 1) {
        const size_t half = len / 2;
        const size_t next = off + len;
        for (size_t base = 0; base < half; base += blockDim.x) {
            const size_t i = base + threadIdx.x;
            H32 p{};
            if (i < half) p = merkle_pair(nodes[2 * i], nodes[2 * i + 1]);
            __syncthreads();
            if (i < half) {
                nodes[i] = p;
                tree[next + i] = p;
            }
            __syncthreads();
        }
        off = next;
        len = half;
        ++l;
    }
}

// One Merkle level across many CTAs (trees too wide for one CTA's memory).
__global__ void merkle_level_kernel(const H32* children, H32* parents, size_t count) {
    for (size_t i = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < count;
         i += static_cast<size_t>(gridDim.x) * blockDim.x)
        parents[i] = merkle_pair(children[2 * i], children[2 * i + 1]);
}

__global__ void merkle_paths_kernel(const H32* tree, const uint32_t* idx, H32* paths, size_t leaves, size_t queries,
                                    int bits) {
    const size_t total = queries * bits;
    for (size_t z = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; z < total;
         z += static_cast<size_t>(gridDim.x) * blockDim.x) {
        const size_t q = z / bits;
        const int level = static_cast<int>(z - q * bits);
        const size_t leaf = idx[q];
        if (leaf >= leaves) {  // out-of-range opening: an all-zero sibling instead of a stray read
            paths[z] = H32{};
            continue;
        }
        paths[z] = tree[level_offset(leaves, level) + ((leaf >> level) ^ 1)];
    }
}

int column_leaves(Context* c, const void* matrix, size_t rows, size_t cols, bool fp2, H32* tree, bool build,
                  uint64_t chunk_base = 0, bool root = true) {
    const size_t words = rows * (fp2 ? 2 : 1);
    const size_t chunks = (words + 127) / 128;
    H32* scratch = nullptr;
    if (chunks > kMaxSmemChunks) {
        if (ensure_ws(c, kWsScratch, chunks * cols * sizeof(H32))) return -1;
        scratch = ws<H32>(c, kWsScratch);
    }
    const unsigned blocks = static_cast<unsigned>((cols + kColsPerCta - 1) / kColsPerCta);
    const auto* m = static_cast<const uint64_t*>(matrix);
    const size_t smem_chunks = chunks > kMaxSmemChunks ? 1 : chunks;
    const size_t smem = smem_chunks * kColsPerCta * sizeof(H32);
    auto k = fp2 ? column_leaves_kernel<2> : column_leaves_kernel<1>;
    VZB_CUDA(c, cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem)));
    k<<<blocks, kColsPerCta * kHashWarps, smem, c->stream>>>(m, rows, cols, tree, scratch, build ? 1 : 0,
                                                             chunk_base, root ? 1 : 0);
    VZB_LAUNCHED(c);
    return 0;
}

// Merkle levels above `level` (whose nodes are already in `tree`).
int merkle_up(Context* c, H32* tree, size_t leaves, int level) {
    size_t len = leaves >> level;
    if (len <= 1) return 0;
    constexpr size_t kTopNodes = 2048;  // 64 KiB of shared memory
    while (len > kTopNodes) {
        const size_t off = level_offset(leaves, level);
        merkle_level_kernel<<<grid_for(c, len / 2, 256), 256, 0, c->stream>>>(tree + off, tree + off + len, len / 2);
        VZB_LAUNCHED(c);
        len /= 2;
        ++level;
    }
    const size_t smem = len * sizeof(H32);
    VZB_CUDA(c, cudaFuncSetAttribute(merkle_top_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                     static_cast<int>(smem)));
    merkle_top_kernel<<<1, 1024, smem, c->stream>>>(tree, leaves, level);
    VZB_LAUNCHED(c);
    return 0;
}

int hash_tree(Context* c, const void* matrix, size_t rows, size_t cols, bool fp2, H32* tree) {
    if (column_leaves(c, matrix, rows, cols, fp2, tree, true)) return -1;
    if (cols <= kColsPerCta) return 0;
    // subtree roots of the column CTAs sit at level log2(32) = 5
    return merkle_up(c, tree, cols, 5);
}

// Column leaves from `shards` subtree chaining values per column
// (in[g * cols + col]), merged pairwise left to right with ROOT on the final
// merge: the BLAKE3 tree of a column whose chunk tree splits into `shards`
// aligned complete subtrees.
constexpr int kMaxCvShards = 64;

__global__ void cvs_merge_kernel(const H32* in, int shards, size_t cols, H32* leaves) {
    for (size_t col = static_cast<size_t>(blockIdx.x) * blockDim.x + threadIdx.x; col < cols;
         col += static_cast<size_t>(gridDim.x) * blockDim.x) {
        H32 cv[kMaxCvShards];
        for (int g = 0; g < shards; ++g) cv[g] = in[static_cast<size_t>(g) * cols + col];
        for (int n = shards; n > 1; n >>= 1)
            for (int i = 0; i < n / 2; ++i) cv[i] = parent_cv(cv[2 * i], cv[2 * i + 1], n == 2 ? kRoot : 0);
        leaves[col] = cv[0];
    }
}

bool pow2(size_t n) { return n && !(n & (n - 1)); }

int tree_device(Context* c, uint64_t matrix_id, size_t matrix_offset, size_t rows, size_t cols, uint64_t tree_id,
                size_t tree_offset_bytes, bool fp2) {
    if (!c || !rows || !pow2(cols))
        return fail_message(c, fp2 ? "invalid resident Fp2 Merkle geometry" : "invalid resident Fp Merkle geometry");
    const size_t elem = fp2 ? sizeof(Fp2) : sizeof(uint64_t);
    void *matrix = nullptr, *tree = nullptr;
    if (region_elems(c, matrix_id, matrix_offset, rows * cols, elem, &matrix) ||
        region(c, tree_id, tree_offset_bytes, (2 * cols - 1) * sizeof(H32), &tree))
        return -1;
    if (reinterpret_cast<uintptr_t>(tree) % alignof(H32)) return fail_message(c, "Merkle tree offset is not 4-byte aligned");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (hash_tree(c, matrix, rows, cols, fp2, static_cast<H32*>(tree))) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsMerkle, 0, 0);
}

}  // namespace
}  // namespace vzb

using namespace vzb;

extern "C" int volta_cuda_hash_fp_tree_device(void* raw, uint64_t matrix_id, size_t matrix_offset, size_t rows,
                                              size_t cols, uint64_t tree_id, size_t tree_offset_bytes) {
    return tree_device(static_cast<Context*>(raw), matrix_id, matrix_offset, rows, cols, tree_id, tree_offset_bytes,
                       false);
}

extern "C" int volta_cuda_hash_fp2_tree_device(void* raw, uint64_t matrix_id, size_t matrix_offset, size_t rows,
                                               size_t cols, uint64_t tree_id, size_t tree_offset_bytes) {
    return tree_device(static_cast<Context*>(raw), matrix_id, matrix_offset, rows, cols, tree_id, tree_offset_bytes,
                       true);
}

// Hybrid leaves only (backend.cu:7256): rows a positive multiple of 8.
extern "C" int volta_cuda_hash_fp_columns(void* raw, const uint64_t* matrix, size_t rows, size_t cols,
                                          uint8_t* leaves) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !matrix || !leaves || rows < 8 || rows % 8 || !pow2(cols)) return -1;
    const size_t mb = rows * cols * sizeof(uint64_t), hb = cols * sizeof(H32);
    if (ensure_ws(c, kWsStageA, mb) || ensure_ws(c, kWsStageB, hb)) return -1;
    if (op_begin(c)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(ws<uint64_t>(c, kWsStageA), matrix, mb, cudaMemcpyHostToDevice, c->stream));
    if (op_mark(c, 1)) return -1;
    if (column_leaves(c, ws<uint64_t>(c, kWsStageA), rows, cols, false, ws<H32>(c, kWsStageB), false)) return -1;
    if (op_mark(c, 2)) return -1;
    VZB_CUDA(c, cudaMemcpyAsync(leaves, ws<H32>(c, kWsStageB), hb, cudaMemcpyDeviceToHost, c->stream));
    return op_finish(c, kOpPcsMerkle, mb, hb);
}

extern "C" int volta_cuda_merkle_paths_device(void* raw, uint64_t tree_id, size_t tree_offset_bytes, size_t leaves,
                                              uint64_t indices_id, size_t indices_offset, size_t queries,
                                              uint64_t paths_id, size_t paths_offset_bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || leaves < 2 || !pow2(leaves) || !queries) return fail_message(c, "invalid resident Merkle path geometry");
    const int bits = __builtin_ctzll(leaves);
    void *tree = nullptr, *idx = nullptr, *paths = nullptr;
    if (region(c, tree_id, tree_offset_bytes, (2 * leaves - 1) * sizeof(H32), &tree) ||
        region_elems(c, indices_id, indices_offset, queries, sizeof(uint32_t), &idx) ||
        region(c, paths_id, paths_offset_bytes, queries * bits * sizeof(H32), &paths))
        return -1;
    if (op_begin(c) || op_mark(c, 1)) return -1;
    merkle_paths_kernel<<<grid_for(c, queries * bits, 256), 256, 0, c->stream>>>(
        static_cast<const H32*>(tree), static_cast<const uint32_t*>(idx), static_cast<H32*>(paths), leaves, queries,
        bits);
    VZB_LAUNCHED(c);
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsMerkle, 0, 0);
}

// ===========================================================================
// Extensions: column trees of row-sharded matrices
// ===========================================================================

extern "C" int volta_b200_hash_fp_column_cvs_device(void* raw, uint64_t matrix_id, size_t matrix_offset, size_t rows,
                                                    size_t cols, uint64_t chunk_base, uint64_t out_id,
                                                    size_t out_offset_bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !cols || !rows || rows % 128 || !pow2(rows / 128))
        return fail_message(c, "column chaining values need rows = 128 * 2^k");
    void *matrix = nullptr, *out = nullptr;
    if (region_elems(c, matrix_id, matrix_offset, rows * cols, sizeof(uint64_t), &matrix) ||
        region(c, out_id, out_offset_bytes, cols * sizeof(H32), &out))
        return -1;
    if (reinterpret_cast<uintptr_t>(out) % alignof(H32)) return fail_message(c, "chaining-value output is not 4-byte aligned");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (column_leaves(c, matrix, rows, cols, false, static_cast<H32*>(out), false, chunk_base, false)) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsMerkle, 0, 0);
}

extern "C" int volta_b200_merkle_from_cvs_device(void* raw, uint64_t cvs_id, size_t cvs_offset_bytes, size_t shards,
                                                 size_t cols, uint64_t tree_id, size_t tree_offset_bytes) {
    Context* c = static_cast<Context*>(raw);
    if (!c || shards < 2 || shards > static_cast<size_t>(kMaxCvShards) || !pow2(shards) || !pow2(cols))
        return fail_message(c, "invalid sharded column-tree geometry");
    void *in = nullptr, *tree = nullptr;
    if (region(c, cvs_id, cvs_offset_bytes, shards * cols * sizeof(H32), &in) ||
        region(c, tree_id, tree_offset_bytes, (2 * cols - 1) * sizeof(H32), &tree))
        return -1;
    if ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(tree)) % alignof(H32))
        return fail_message(c, "Merkle buffers are not 4-byte aligned");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    cvs_merge_kernel<<<grid_for(c, cols, 128), 128, 0, c->stream>>>(static_cast<const H32*>(in),
                                                                    static_cast<int>(shards), cols,
                                                                    static_cast<H32*>(tree));
    VZB_LAUNCHED(c);
    if (merkle_up(c, static_cast<H32*>(tree), cols, 0)) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsMerkle, 0, 0);
}

extern "C" int volta_b200_merkle_levels_device(void* raw, uint64_t tree_id, size_t tree_offset_bytes, size_t leaves) {
    Context* c = static_cast<Context*>(raw);
    if (!c || !pow2(leaves)) return fail_message(c, "invalid Merkle level geometry");
    void* tree = nullptr;
    if (region(c, tree_id, tree_offset_bytes, (2 * leaves - 1) * sizeof(H32), &tree)) return -1;
    if (reinterpret_cast<uintptr_t>(tree) % alignof(H32)) return fail_message(c, "Merkle tree is not 4-byte aligned");
    if (op_begin(c) || op_mark(c, 1)) return -1;
    if (merkle_up(c, static_cast<H32*>(tree), leaves, 0)) return -1;
    if (op_mark(c, 2)) return -1;
    return op_finish(c, kOpPcsMerkle, 0, 0);
}
