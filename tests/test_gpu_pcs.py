"""Ligero PCS kernels against the oracle: NTT (every size regime: whole rows
in shared memory, the six-step split, the per-stage path beyond 2^22),
BLAKE3 column leaves and Merkle trees (single-chunk, shared-memory chunk
trees and the long-column path), Merkle paths, PCS messages, row
combinations and column gathers.  Plus the reference's own golden vectors
(batched NTT checksum, column-Merkle roots) at their full sizes."""

import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=0)
    yield b
    b.close()


def rand_fp(rng, n):
    return rng.integers(0, P, size=n, dtype=np.uint64)


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def mod_affine(i, mul, add):
    x = i.astype(np.uint64) * np.uint64(mul) + np.uint64(add)
    return np.where(x >= np.uint64(P), x - np.uint64(P), x).astype(np.uint64)


# ---- NTT ----------------------------------------------------------------------

@pytest.mark.parametrize("rows,bits", [(1, 1), (3, 2), (5, 6), (2, 10), (3, 11), (2, 12), (3, 13), (4, 16),
                                       (2, 17), (1, 20), (1, 23)])
def test_ntt_fp_batch_device(be, oracle, rows, bits):
    n = 1 << bits
    rng = np.random.default_rng(bits * 10 + rows)
    x = rand_fp(rng, rows * n)
    src = be.upload_new(x)
    dst = be.alloc(8 * rows * n)
    be.call("ntt_fp_batch_device", src, 0, rows, n, dst, 0)
    exp = oracle.ntt_batch(x, rows, n, n)
    assert np.array_equal(be.download(dst, 8 * rows * n), exp)
    # in place (same buffer) gives the same result
    be.call("ntt_fp_batch_device", src, 0, rows, n, src, 0)
    assert np.array_equal(be.download(src, 8 * rows * n), exp)
    be.free(src)
    be.free(dst)


@pytest.mark.parametrize("rows,bits", [(1, 1), (3, 5), (2, 11), (2, 12), (3, 15), (1, 23)])
def test_ntt_fp2_batch_device(be, oracle, rows, bits):
    n = 1 << bits
    rng = np.random.default_rng(bits + 100 * rows)
    x = rng.integers(0, P, size=(rows * n, 2), dtype=np.uint64)
    src = be.upload_new(x)
    dst = be.alloc(16 * rows * n)
    be.call("ntt_fp2_batch_device", src, 0, rows, n, dst, 0)
    exp = oracle.ntt_fp2_batch(x, rows, n, n)
    assert np.array_equal(be.download_fp2(dst, rows * n), exp)
    be.free(src)
    be.free(dst)


@pytest.mark.parametrize("rows,msg_len,bits", [(1, 0, 1), (1, 5, 4), (3, 100, 8), (7, 2304, 12), (2, 16384, 16)])
def test_ntt_hybrid(be, oracle, rows, msg_len, bits):
    n = 1 << bits
    rng = np.random.default_rng(msg_len + bits)
    msgs = rand_fp(rng, max(rows * msg_len, 1))
    exp = oracle.ntt_batch(msgs, rows, msg_len, n)
    out = np.zeros(rows * n, dtype=np.uint64)
    assert be.lib.volta_cuda_ntt_fp_batch(be.ctx, ptr(msgs), rows, msg_len, n, ptr(out)) == 0, be.last_error()
    assert np.array_equal(out, exp)
    one = np.zeros(n, dtype=np.uint64)
    assert be.lib.volta_cuda_ntt_fp(be.ctx, ptr(msgs), msg_len, n, ptr(one)) == 0, be.last_error()
    assert np.array_equal(one, exp[:n])
    m2 = rng.integers(0, P, size=(max(msg_len, 1), 2), dtype=np.uint64)
    out2 = np.zeros((n, 2), dtype=np.uint64)
    assert be.lib.volta_cuda_ntt_fp2(be.ctx, ptr(m2), msg_len, n, ptr(out2)) == 0, be.last_error()
    assert np.array_equal(out2, oracle.ntt_fp2_batch(m2, 1, msg_len, n))


def test_ntt_rejects_bad_geometry(be):
    buf = be.alloc(8 * 64)
    assert be.lib.volta_cuda_ntt_fp_batch_device(be.ctx, buf, 0, 1, 48, buf, 0) != 0
    assert be.lib.volta_cuda_ntt_fp_batch_device(be.ctx, buf, 0, 2, 64, buf, 0) != 0  # beyond the buffer
    assert be.lib.volta_cuda_ntt_fp_batch_device(be.ctx, buf, 0, 1, 1, buf, 0) != 0
    one = np.zeros(64, dtype=np.uint64)
    assert be.lib.volta_cuda_ntt_fp(be.ctx, ptr(one), 65, 64, ptr(one)) != 0
    be.free(buf)


@pytest.mark.parametrize("rows,bits,msg_len,checksum", [
    (32, 12, 2304, 0xa87a560725f2d016),
    (1024, 15, 16896, 0xbe7b90425a4c7229),
])
def test_ntt_golden(be, oracle, rows, bits, msg_len, checksum):
    """cuda/p7_pcs_arithmetic.cu:204-262 batched NTT checksums (published run)."""
    n = 1 << bits
    idx = np.arange(rows * n, dtype=np.uint64).reshape(rows, n)
    full = mod_affine(idx, 0x9E3779B9, 17)
    full[:, msg_len:] = 0
    src = be.upload_new(full)
    be.call("ntt_fp_batch_device", src, 0, rows, n, src, 0)
    assert oracle.fnv_u64(be.download(src, 8 * rows * n)) == checksum
    be.free(src)


# ---- BLAKE3 columns and Merkle trees -----------------------------------------

def device_tree(be, m, rows, cols, fp2=False, tree_offset=0):
    src = be.upload_new(m)
    tree = be.alloc(tree_offset + 32 * (2 * cols - 1))
    be.call("hash_fp2_tree_device" if fp2 else "hash_fp_tree_device", src, 0, rows, cols, tree, tree_offset)
    out = be.download(tree, 32 * (2 * cols - 1), dtype=np.uint8, offset_bytes=tree_offset).reshape(-1, 32)
    be.free(src)
    be.free(tree)
    return out


@pytest.mark.parametrize("rows,cols", [(1, 1), (1, 2), (8, 4), (100, 32), (128, 64), (129, 64), (1000, 256),
                                       (8192, 64), (8200, 32), (16, 4096), (3, 1 << 16)])
def test_hash_fp_tree(be, oracle, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols)
    m = rand_fp(rng, rows * cols)
    got = device_tree(be, m, rows, cols, tree_offset=64)
    exp = oracle.merkle_tree(oracle.hash_fp_columns(m, rows, cols))
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("rows,cols", [(1, 1), (7, 8), (64, 32), (65, 64), (4096, 32), (4100, 64)])
def test_hash_fp2_tree(be, oracle, rows, cols):
    rng = np.random.default_rng(rows + cols)
    m = rng.integers(0, P, size=(rows * cols, 2), dtype=np.uint64)
    got = device_tree(be, m, rows, cols, fp2=True)
    exp = oracle.merkle_tree(oracle.hash_fp2_columns(m, rows, cols))
    assert np.array_equal(got, exp)


@pytest.mark.parametrize("rows,cols,root", [
    (32, 1024, "f427c1a8e4024b372e694b20215a860cfbf94c2463e2a5f76021243f1f8722e1"),
    (1024, 32768, "c90027afa35e9f24dd436d51d734b63e52c9788f50a1658c7a6a2a2685ca4d5f"),
])
def test_column_merkle_golden(be, rows, cols, root):
    """cuda/p7_blake3_merkle.cu:231-243 roots (published run)."""
    m = mod_affine(np.arange(rows * cols, dtype=np.uint64), 0x9E3779B9, 17)
    tree = device_tree(be, m, rows, cols)
    assert tree[-1].tobytes().hex() == root


def test_hash_fp_columns_hybrid(be, oracle):
    rows, cols = 256, 512
    m = rand_fp(np.random.default_rng(9), rows * cols)
    out = np.zeros((cols, 32), dtype=np.uint8)
    assert be.lib.volta_cuda_hash_fp_columns(be.ctx, ptr(m), rows, cols, ptr(out)) == 0, be.last_error()
    assert np.array_equal(out, oracle.hash_fp_columns(m, rows, cols))
    assert be.lib.volta_cuda_hash_fp_columns(be.ctx, ptr(m), 12, cols, ptr(out)) != 0  # rows % 8


@pytest.mark.parametrize("leaves,queries", [(2, 1), (16, 16), (1024, 37), (1 << 16, 128)])
def test_merkle_paths(be, oracle, leaves, queries):
    rng = np.random.default_rng(leaves + queries)
    leaf_hashes = rng.integers(0, 256, size=(leaves, 32), dtype=np.uint8)
    tree = oracle.merkle_tree(leaf_hashes)
    idx = rng.integers(0, leaves, size=queries, dtype=np.uint32)
    tid, iid = be.upload_new(tree), be.upload_new(idx)
    bits = leaves.bit_length() - 1
    pid = be.alloc(32 * queries * bits)
    be.call("merkle_paths_device", tid, 0, leaves, iid, 0, queries, pid, 0)
    got = be.download(pid, 32 * queries * bits, dtype=np.uint8).reshape(-1, 32)
    assert np.array_equal(got, oracle.merkle_paths(tree, leaves, idx))
    for i in (tid, iid, pid):
        be.free(i)


# ---- messages, combinations, gathers --------------------------------------------

@pytest.mark.parametrize("rows,cols,pad,code_len", [(1, 1, 0, 1), (3, 5, 2, 16), (4, 700, 37, 2048), (64, 1000, 24, 4096)])
def test_pcs_messages(be, oracle, rows, cols, pad, code_len):
    rng = np.random.default_rng(cols + pad)
    w = rng.integers(-32768, 32768, size=rows * cols, dtype=np.int64).astype(np.int16)
    pads = rand_fp(rng, max(rows * pad, 1))
    wid, pid = be.upload_new(w), be.upload_new(pads)
    out = be.alloc(8 * rows * code_len)
    be.call("pcs_messages_device", wid, 0, pid, 0, rows, cols, pad, code_len, out, 0)
    exp = oracle.pcs_messages(w, pads, rows, cols, pad, code_len)
    assert np.array_equal(be.download(out, 8 * rows * code_len), exp)
    for i in (wid, pid, out):
        be.free(i)


@pytest.mark.parametrize("rows,cols,pad,combos", [(1, 1, 0, 1), (3, 17, 4, 2), (16, 300, 8, 5), (128, 2048, 64, 9),
                                                   (1000, 64, 3, 1), (4096, 512, 0, 2)])  # row bands, ragged last
def test_pcs_combine_rows(be, oracle, rows, cols, pad, combos):
    rng = np.random.default_rng(rows * cols + combos)
    w = rng.integers(-32768, 32768, size=rows * cols, dtype=np.int64).astype(np.int16)
    pads = rand_fp(rng, max(rows * pad, 1))
    coeffs = rng.integers(0, P, size=(combos * rows, 2), dtype=np.uint64)
    exp = oracle.pcs_combine_rows(w, pads, coeffs, rows, cols, pad, combos)
    ids = [be.upload_new(x) for x in (w, pads, coeffs)]
    out = be.alloc(16 * combos * (cols + pad))
    be.call("pcs_combine_rows_device", ids[0], 0, ids[1], 0, ids[2], 0, rows, cols, pad, combos, out, 0)
    assert np.array_equal(be.download_fp2(out, combos * (cols + pad)), exp)
    host = np.zeros((combos * (cols + pad), 2), dtype=np.uint64)
    rc = be.lib.volta_cuda_pcs_combine_rows(be.ctx, ptr(w), ptr(pads) if pad else None, ptr(coeffs), rows, cols,
                                            pad, combos, ptr(host))
    assert rc == 0, be.last_error()
    assert np.array_equal(host, exp)
    for i in ids + [out]:
        be.free(i)


@pytest.mark.parametrize("rows,cols,queries", [(1, 1, 1), (5, 64, 3), (8192, 1 << 10, 128)])
def test_pcs_gather_columns(be, rows, cols, queries):
    rng = np.random.default_rng(rows + cols)
    m = rand_fp(rng, rows * cols)
    idx = rng.integers(0, cols, size=queries, dtype=np.uint32)
    exp = m.reshape(rows, cols)[:, idx].T.reshape(-1)
    mid, iid = be.upload_new(m), be.upload_new(idx)
    out = be.alloc(8 * rows * queries)
    be.call("pcs_gather_columns_device", mid, 0, rows, cols, iid, 0, queries, out, 0, 0)
    assert np.array_equal(be.download(out, 8 * rows * queries), exp)
    host = np.zeros(rows * queries, dtype=np.uint64)
    assert be.lib.volta_cuda_pcs_gather_columns(be.ctx, ptr(m), rows, cols, ptr(idx), queries, ptr(host)) == 0
    assert np.array_equal(host, exp)
    # Fp2 matrix
    m2 = rng.integers(0, P, size=(rows * cols, 2), dtype=np.uint64)
    m2id = be.upload_new(m2)
    out2 = be.alloc(16 * rows * queries)
    be.call("pcs_gather_columns_device", m2id, 0, rows, cols, iid, 0, queries, out2, 0, 1)
    exp2 = m2.reshape(rows, cols, 2)[:, idx, :].transpose(1, 0, 2).reshape(-1, 2)
    assert np.array_equal(be.download_fp2(out2, rows * queries), exp2)
    for i in (mid, iid, out, m2id, out2):
        be.free(i)
