// Resident Ligero commitment and column openings over the seam, restating
// the reference's resident callers call for call:
//   commit   rust/volta-pcs/src/ligero.rs:465-505 (finish_resident_commit:
//            ChaCha8 rows -> PCS messages -> batched NTT -> BLAKE3 column tree
//            -> root download)
//   open     ligero.rs:1440-1480 (query indices challenge_fp2().c0 mod
//            code_len, column gather, Merkle paths, downloads)
// The messages here are seeded Fp rows (msg_len words per row) zero-padded to
// code_len, the shape of the weight-matrix commitment benchmark.
#include <cstring>

#include "protocol.hpp"

namespace vzh {

LigeroOpening ligero_commit_open_resident(Backend& b, const uint8_t row_seed[32], size_t rows, size_t msg_len,
                                          size_t code_len, size_t queries, FpStream& tx) {
    const Api& A = b.api();
    void* ctx = b.ctx();
    if (!rows || !msg_len || msg_len > code_len || !code_len || (code_len & (code_len - 1)) || !queries)
        throw AccelError("invalid Ligero geometry");
    Owned own(b);
    LigeroOpening out;
    // rows of the message matrix, then zero-padded codeword rows
    const uint64_t msgs = own.add(b.alloc(rows * msg_len * sizeof(uint64_t)));
    b.check(A.volta_cuda_chacha8_prover_secret_fp_rows_device(ctx, msgs, 0, row_seed, 0, rows, msg_len),
            "chacha8_prover_secret_fp_rows_device");
    const size_t code_bytes = rows * code_len * sizeof(uint64_t);
    const uint64_t code = own.add(b.alloc(code_bytes));
    if (msg_len < code_len) b.check(A.volta_cuda_resident_zero(ctx, code, 0, code_bytes), "resident_zero");
    b.check(A.volta_cuda_resident_copy_rows(ctx, msgs, 0, msg_len * sizeof(uint64_t), code, 0,
                                            code_len * sizeof(uint64_t), rows, msg_len * sizeof(uint64_t)),
            "resident_copy_rows");
    own.release(msgs);
    // Reed-Solomon encoding in place, then the column tree
    b.check(A.volta_cuda_ntt_fp_batch_device(ctx, code, 0, rows, code_len, code, 0), "ntt_fp_batch_device");
    const uint64_t tree = own.add(b.alloc((2 * code_len - 1) * 32));
    b.check(A.volta_cuda_hash_fp_tree_device(ctx, code, 0, rows, code_len, tree, 0), "hash_fp_tree_device");
    b.download(tree, (2 * code_len - 2) * 32, out.root, 32);
    // openings
    out.indices.resize(queries);
    for (auto& j : out.indices) j = static_cast<uint32_t>(tx.next_fp2().c0 % code_len);
    const uint64_t idx = own.add(b.alloc(queries * sizeof(uint32_t)));
    b.upload(idx, 0, out.indices.data(), queries * sizeof(uint32_t));
    const uint64_t cols = own.add(b.alloc(queries * rows * sizeof(uint64_t)));
    b.check(A.volta_cuda_pcs_gather_columns_device(ctx, code, 0, rows, code_len, idx, 0, queries, cols, 0, 0),
            "pcs_gather_columns_device");
    size_t bits = 0;
    while ((size_t{1} << bits) < code_len) ++bits;
    out.columns.resize(queries * rows);
    out.paths.resize(queries * bits * 32);
    if (bits) {
        const uint64_t paths = own.add(b.alloc(out.paths.size()));
        b.check(A.volta_cuda_merkle_paths_device(ctx, tree, 0, code_len, idx, 0, queries, paths, 0),
                "merkle_paths_device");
        b.download(paths, 0, out.paths.data(), out.paths.size());
    }
    b.download(cols, 0, out.columns.data(), out.columns.size() * sizeof(uint64_t));
    return out;
}

}  // namespace vzh
