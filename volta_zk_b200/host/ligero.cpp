// Resident Ligero commitment and column openings over the seam, restating
// the reference's resident callers call for call:
//   commit   rust/volta-pcs/src/ligero.rs:465-505 (finish_resident_commit:
//            ChaCha8 rows -> PCS messages -> batched NTT -> BLAKE3 column tree
//            -> root download)
//   open     ligero.rs:1440-1480 (query indices challenge_fp2().c0 mod
//            code_len, column gather, Merkle paths, downloads)
// The messages here are seeded Fp rows (msg_len words per row) zero-padded to
// code_len, the shape of the weight-matrix commitment benchmark.
#include <algorithm>
#include <chrono>
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

static size_t claim_row0(const LigeroShape& sh, const ZkClaim& cl) {
    // ligero.rs:953-972 (resident_claim_row0)
    if (cl.point.size() < sh.col_bits) throw AccelError("PCS claim block is smaller than a matrix row");
    if (cl.point.size() >= 8 * sizeof(size_t)) throw AccelError("PCS claim geometry overflow");
    const size_t block = size_t{1} << cl.point.size();
    if (cl.offset % block) throw AccelError("PCS claim block offset is not aligned");
    const size_t row_count = size_t{1} << (cl.point.size() - sh.col_bits), row0 = cl.offset >> sh.col_bits;
    if (row0 + row_count > sh.rows || row0 + row_count < row0) throw AccelError("PCS claim rows exceed matrix");
    return row0;
}

LigeroZkOpening ligero_commit_open_zk(Backend& b, const int16_t* weights, const LigeroShape& sh,
                                      const uint8_t pad_seed[32], const std::vector<ZkClaim>& claims,
                                      const uint8_t mask_seed[32], Fp2 c, const std::vector<uint32_t>& indices,
                                      double phase_ms[2]) {
    const Api& A = b.api();
    void* ctx = b.ctx();
    const size_t rows = sh.rows, cols = sh.cols(), pad = sh.pad, msg_len = sh.msg_len(), code_len = sh.code_len();
    if (!rows || sh.col_bits >= 31 || sh.code_bits >= 31 || msg_len > code_len || !weights)
        throw AccelError("invalid Ligero geometry");
    if (claims.empty()) throw AccelError("PCS opening needs a claim");
    if (indices.empty()) throw AccelError("PCS opening needs a query");
    for (uint32_t j : indices)
        if (j >= code_len) throw AccelError("PCS query index beyond the code length");
    std::vector<size_t> row0(claims.size());
    for (size_t g = 0; g < claims.size(); ++g) row0[g] = claim_row0(sh, claims[g]);
    const size_t n = claims.size(), mrows = n + 1, q = indices.size(), bits = sh.code_bits;
    Owned own(b);
    LigeroZkOpening out;
    const auto t0 = std::chrono::steady_clock::now();

    // ---- commit (ligero.rs:465-505) -----------------------------------------
    const uint64_t w = own.add(b.alloc(rows * cols * sizeof(int16_t)));
    b.upload(w, 0, weights, rows * cols * sizeof(int16_t));
    const uint64_t pads = own.add(b.alloc(std::max<size_t>(rows * pad, 1) * sizeof(uint64_t)));
    if (pad)
        b.check(A.volta_cuda_chacha8_prover_secret_fp_rows_device(ctx, pads, 0, pad_seed, 0, rows, pad),
                "chacha8_prover_secret_fp_rows_device");
    const uint64_t code = own.add(b.alloc(rows * code_len * sizeof(uint64_t)));
    b.check(A.volta_cuda_pcs_messages_device(ctx, w, 0, pads, 0, rows, cols, pad, code_len, code, 0),
            "pcs_messages_device");
    b.check(A.volta_cuda_ntt_fp_batch_device(ctx, code, 0, rows, code_len, code, 0), "ntt_fp_batch_device");
    const uint64_t tree = own.add(b.alloc((2 * code_len - 1) * 32));
    b.check(A.volta_cuda_hash_fp_tree_device(ctx, code, 0, rows, code_len, tree, 0), "hash_fp_tree_device");
    b.download(tree, (2 * code_len - 2) * 32, out.root, 32);
    const auto t1 = std::chrono::steady_clock::now();

    // ---- 1. mask rows: generated padded, compact copy, encoded, committed ----
    const uint64_t mask_msgs = own.add(b.alloc(mrows * code_len * sizeof(Fp2)));
    b.check(A.volta_cuda_chacha8_prover_secret_fp2_rows_padded_device(ctx, mask_msgs, 0, mask_seed, 0, mrows,
                                                                      msg_len, code_len),
            "chacha8_prover_secret_fp2_rows_padded_device");
    const uint64_t mask_compact = own.add(b.alloc(mrows * msg_len * sizeof(Fp2)));
    b.check(A.volta_cuda_resident_copy_rows(ctx, mask_msgs, 0, code_len * sizeof(Fp2), mask_compact, 0,
                                            msg_len * sizeof(Fp2), mrows, msg_len * sizeof(Fp2)),
            "resident_copy_rows");
    const uint64_t mask_code = own.add(b.alloc(mrows * code_len * sizeof(Fp2)));
    b.check(A.volta_cuda_ntt_fp2_batch_device(ctx, mask_msgs, 0, mrows, code_len, mask_code, 0),
            "ntt_fp2_batch_device");
    own.release(mask_msgs);
    const uint64_t mask_tree = own.add(b.alloc((2 * code_len - 1) * 32));
    b.check(A.volta_cuda_hash_fp2_tree_device(ctx, mask_code, 0, mrows, code_len, mask_tree, 0),
            "hash_fp2_tree_device");

    // ---- 2. proximity row: u_c = sum_r c^r row_r + mask_0 -------------------
    const uint64_t cpow = own.add(b.alloc(rows * sizeof(Fp2)));
    b.check(A.volta_cuda_fp2_powers_device(ctx, c.c0, c.c1, cpow, 0, rows), "fp2_powers_device");
    const uint64_t u_c = own.add(b.alloc(msg_len * sizeof(Fp2)));
    b.check(A.volta_cuda_pcs_combine_rows_device(ctx, w, 0, pads, 0, cpow, 0, rows, cols, pad, 1, u_c, 0),
            "pcs_combine_rows_device");
    b.check(A.volta_cuda_fp2_add_inplace_device(ctx, u_c, 0, mask_compact, 0, msg_len), "fp2_add_inplace_device");

    // ---- 3. claim rows: u_g = sum_r eq_g(r) row_r + mask_{g+1} ---------------
    // A claim's coefficients vanish outside its own 2^k rows, so each claim
    // combines just those rows (the same sums as one pass over every row with
    // the zero coefficients, ligero.rs:1296-1345, at a fraction of the reads).
    const uint64_t u_g = own.add(b.alloc(n * msg_len * sizeof(Fp2)));
    for (size_t g = 0; g < n; ++g) {
        const size_t k = claims[g].point.size() - sh.col_bits, len = size_t{1} << k;
        uint64_t pts = 0;
        if (k) {
            pts = own.add(b.alloc(k * sizeof(Fp2)));
            b.upload(pts, 0, claims[g].point.data() + sh.col_bits, k * sizeof(Fp2));
        }
        const uint64_t eq = own.add(b.alloc(len * sizeof(Fp2)));
        b.check(A.volta_cuda_logup_eq_rows_device(ctx, pts, 0, 1, k, eq, 0), "logup_eq_rows_device");
        b.check(A.volta_cuda_pcs_combine_rows_device(ctx, w, row0[g] * cols, pads, pad ? row0[g] * pad : 0, eq, 0, len,
                                                     cols, pad, 1, u_g, g * msg_len),
                "pcs_combine_rows_device");
        own.release(eq);
        if (pts) own.release(pts);
    }
    b.check(A.volta_cuda_fp2_add_inplace_device(ctx, u_g, 0, mask_compact, msg_len, n * msg_len),
            "fp2_add_inplace_device");

    // ---- 4. s_g = <mask_{g+1}[0 .. cols), eq(point_g[.. col_bits])> --------
    std::vector<Fp2> mpts(n * sh.col_bits);
    for (size_t g = 0; g < n; ++g)
        std::copy(claims[g].point.begin(), claims[g].point.begin() + sh.col_bits, mpts.begin() + g * sh.col_bits);
    uint64_t mp = 0;
    if (!mpts.empty()) {
        mp = own.add(b.alloc(mpts.size() * sizeof(Fp2)));
        b.upload(mp, 0, mpts.data(), mpts.size() * sizeof(Fp2));
    }
    const uint64_t meq = own.add(b.alloc(n * cols * sizeof(Fp2)));
    b.check(A.volta_cuda_logup_eq_rows_device(ctx, mp, 0, n, sh.col_bits, meq, 0), "logup_eq_rows_device");
    const uint64_t dots = own.add(b.alloc(n * sizeof(Fp2)));
    b.check(A.volta_cuda_fp2_row_dots_device(ctx, mask_compact, msg_len, msg_len, meq, 0, cols, dots, 0, n, cols),
            "fp2_row_dots_device");

    // ---- 5. query columns and Merkle paths ---------------------------------
    const uint64_t idx = own.add(b.alloc(q * sizeof(uint32_t)));
    b.upload(idx, 0, indices.data(), q * sizeof(uint32_t));
    const uint64_t dcols = own.add(b.alloc(q * rows * sizeof(uint64_t)));
    b.check(A.volta_cuda_pcs_gather_columns_device(ctx, code, 0, rows, code_len, idx, 0, q, dcols, 0, 0),
            "pcs_gather_columns_device");
    const uint64_t mcols = own.add(b.alloc(q * mrows * sizeof(Fp2)));
    b.check(A.volta_cuda_pcs_gather_columns_device(ctx, mask_code, 0, mrows, code_len, idx, 0, q, mcols, 0, 1),
            "pcs_gather_columns_device");
    out.paths.resize(q * bits * 32);
    out.mask_paths.resize(q * bits * 32);
    uint64_t dpaths = 0, mpaths = 0;
    if (bits) {
        dpaths = own.add(b.alloc(out.paths.size()));
        mpaths = own.add(b.alloc(out.mask_paths.size()));
        b.check(A.volta_cuda_merkle_paths_device(ctx, tree, 0, code_len, idx, 0, q, dpaths, 0), "merkle_paths_device");
        b.check(A.volta_cuda_merkle_paths_device(ctx, mask_tree, 0, code_len, idx, 0, q, mpaths, 0),
                "merkle_paths_device");
    }
    // downloads (the first one waits for everything above)
    b.download(mask_tree, (2 * code_len - 2) * 32, out.mask_root, 32);
    out.u_c.resize(msg_len);
    b.download(u_c, 0, out.u_c.data(), msg_len * sizeof(Fp2));
    out.u_g.resize(n * msg_len);
    b.download(u_g, 0, out.u_g.data(), n * msg_len * sizeof(Fp2));
    out.s.resize(n);
    b.download(dots, 0, out.s.data(), n * sizeof(Fp2));
    out.columns.resize(q * rows);
    b.download(dcols, 0, out.columns.data(), q * rows * sizeof(uint64_t));
    out.mask_columns.resize(q * mrows);
    b.download(mcols, 0, out.mask_columns.data(), q * mrows * sizeof(Fp2));
    if (bits) {
        b.download(dpaths, 0, out.paths.data(), out.paths.size());
        b.download(mpaths, 0, out.mask_paths.data(), out.mask_paths.size());
    }
    const auto t2 = std::chrono::steady_clock::now();
    if (phase_ms) {
        phase_ms[0] = std::chrono::duration<double, std::milli>(t1 - t0).count();
        phase_ms[1] = std::chrono::duration<double, std::milli>(t2 - t1).count();
    }
    return out;
}

}  // namespace vzh
