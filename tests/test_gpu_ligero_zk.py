"""Weight-matrix Ligero commitment and the device part of its
zero-knowledge multi-claim opening (vzh_ligero_commit_open_zk) against the
oracle's functions composed in the order of rust/volta-pcs/src/ligero.rs
(finish_resident_commit 465-505, open_multi_zk_resident 1187-1480): root,
mask root, proximity row u_c, claim rows u_g, masked row dots s_g, queried
data and mask columns, both Merkle paths."""

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


def fp2_mul(a, b):
    a0, a1, b0, b1 = (int(x) for x in (a[0], a[1], b[0], b[1]))
    return ((a0 * b0 + 7 * a1 * b1) % P, (a0 * b1 + a1 * b0) % P)


def fp2_add_rows(x, y):
    """Entry-wise Fp2 sum of two (n, 2) u64 arrays."""
    s = (x.astype(object) + y.astype(object)) % P
    return s.astype(np.uint64)


def expected(oracle, w, rows, col_bits, pad, code_bits, pad_seed, claims, mask_seed, c, idx):
    cols, code_len = 1 << col_bits, 1 << code_bits
    msg_len, n, mrows = cols + pad, len(claims), len(claims) + 1
    pads = oracle.chacha_fp_rows(pad_seed, 0, rows, pad) if pad else np.zeros((rows, 0), np.uint64)
    msgs = oracle.pcs_messages(np.ascontiguousarray(w), np.ascontiguousarray(pads), rows, cols, pad, code_len)
    code = oracle.ntt_batch(msgs.reshape(rows, code_len)[:, :msg_len].copy(), rows, msg_len, code_len)
    tree = oracle.merkle_tree(oracle.hash_fp_columns(code, rows, code_len))
    masks = oracle.chacha_fp2_rows_padded(mask_seed, 0, mrows, msg_len, code_len).reshape(mrows, code_len, 2)
    compact = np.ascontiguousarray(masks[:, :msg_len])
    mcode = oracle.ntt_fp2_batch(compact.reshape(-1, 2), mrows, msg_len, code_len)
    mtree = oracle.merkle_tree(oracle.hash_fp2_columns(mcode, mrows, code_len))
    powers, x = [], (1, 0)
    for _ in range(rows):  # c^1 .. c^rows (ligero.rs:1630-1635)
        x = fp2_mul(x, c)
        powers.append(x)
    cpow = np.array(powers, dtype=np.uint64)
    u_c = fp2_add_rows(oracle.pcs_combine_rows(w, pads, cpow, rows, cols, pad, 1), compact[0])
    coeff = np.zeros((n * rows, 2), dtype=np.uint64)
    for g, (offset, point) in enumerate(claims):
        k = len(point) - col_bits
        eq = oracle.eq_rows(np.ascontiguousarray(point[col_bits:]), 1, k) if k else np.array([[1, 0]], np.uint64)
        row0 = offset >> col_bits
        coeff[g * rows + row0: g * rows + row0 + (1 << k)] = eq
    u_g = oracle.pcs_combine_rows(w, pads, coeff, rows, cols, pad, n).reshape(n, msg_len, 2)
    u_g = np.stack([fp2_add_rows(u_g[g], compact[g + 1]) for g in range(n)])
    s = []
    for g, (_, point) in enumerate(claims):
        eq = oracle.eq_rows(np.ascontiguousarray(point[:col_bits]), 1, col_bits)
        acc = (0, 0)
        for j in range(cols):
            t = fp2_mul(compact[g + 1, j], eq[j])
            acc = ((acc[0] + t[0]) % P, (acc[1] + t[1]) % P)
        s.append(acc)
    code2 = code.reshape(rows, code_len)
    mcode2 = mcode.reshape(mrows, code_len, 2)
    return {
        "root": tree[-1], "mask_root": mtree[-1], "u_c": u_c, "u_g": u_g.reshape(-1, 2),
        "s": np.array(s, dtype=np.uint64),
        "columns": np.concatenate([code2[:, j] for j in idx]),
        "mask_columns": np.concatenate([mcode2[:, j] for j in idx]),
        "paths": oracle.merkle_paths(tree, code_len, idx).reshape(-1),
        "mask_paths": oracle.merkle_paths(mtree, code_len, idx).reshape(-1),
    }


@pytest.mark.parametrize("rows,col_bits,pad,code_bits,blocks", [
    (40, 6, 8, 8, [(4, 2), (7, 0), (0, 3)]),     # non-power-of-two rows; one-row, 4-row and 8-row claims
    (64, 7, 0, 8, [(32, 5)]),                    # no pads; one claim over half the matrix
    (128, 5, 31, 7, [(r, 0) for r in range(0, 128, 37)] + [(64, 6)]),
])
def test_commit_open_zk_matches_oracle(prover, oracle, rows, col_bits, pad, code_bits, blocks):
    rng = np.random.default_rng(rows + col_bits + pad)
    cols = 1 << col_bits
    w = rng.integers(-32768, 32768, size=(rows, cols), dtype=np.int64).astype(np.int16)
    claims = []
    for row0, k in blocks:
        point = rng.integers(0, P, size=(col_bits + k, 2), dtype=np.uint64)
        claims.append((row0 << col_bits, point))
    c = tuple(int(x) for x in rng.integers(0, P, size=2, dtype=np.uint64))
    idx = rng.integers(0, 1 << code_bits, size=17).astype(np.uint32)
    pad_seed, mask_seed = bytes(range(32)), bytes([0xA5] * 32)
    got = prover.ligero_commit_open_zk(w, rows, col_bits, pad, code_bits, pad_seed, claims, mask_seed, c, idx)
    exp = expected(oracle, w, rows, col_bits, pad, code_bits, pad_seed, claims, mask_seed, c, idx)
    for key in ("root", "mask_root", "u_c", "u_g", "s", "columns", "mask_columns", "paths", "mask_paths"):
        assert np.array_equal(np.asarray(got[key]).reshape(np.asarray(exp[key]).shape), exp[key]), key


def test_commit_open_zk_rejects_bad_claims(prover):
    from volta_zk_b200.accel import AccelError

    rows, col_bits, pad, code_bits = 16, 4, 4, 6
    w = np.zeros((rows, 1 << col_bits), dtype=np.int16)
    pt = lambda n: np.zeros((n, 2), dtype=np.uint64)  # noqa: E731
    for claims in ([(0, pt(col_bits - 1))],             # smaller than a row
                   [(16, pt(col_bits + 1))],            # offset not aligned to the 2-row block
                   [(15 << col_bits, pt(col_bits + 1))],  # rows past the matrix
                   []):
        with pytest.raises(AccelError):
            prover.ligero_commit_open_zk(w, rows, col_bits, pad, code_bits, bytes(32), claims, bytes(32), (1, 0),
                                         [0])
    with pytest.raises(AccelError):  # query index past the code
        prover.ligero_commit_open_zk(w, rows, col_bits, pad, code_bits, bytes(32), [(0, pt(col_bits))], bytes(32),
                                     (1, 0), [1 << code_bits])
