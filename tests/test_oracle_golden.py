"""Pin the CPU oracle against the reference's own golden vectors.

Every expected value below is published by the reference (okrame/volta-zk)
in benchmarks/results/*.json or asserted in its Rust unit tests; the input
recipes are the closed forms in the cited cuda/p7_*.cu drivers.
"""

import hashlib

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
FNV0 = 0xCBF29CE484222325
FNV_PRIME = 0x00000100000001B3
M64 = (1 << 64) - 1


def fnv(h, x):
    return ((h ^ x) * FNV_PRIME) & M64


def fnv_fp2_pairs(o, h, arr):
    return o.fnv_u64(np.ascontiguousarray(arr).reshape(-1), h)


# --------------------------------------------------------------------------
# Field (rust/volta-field/src/lib.rs:297-365)
# --------------------------------------------------------------------------

def test_field_edge_cases(oracle):
    o = oracle
    assert o.fp_mul(P - 1, P - 1) == 1
    assert o.lib().or_fp_add(P - 1, 1) == 0
    assert o.lib().or_fp_sub(0, 1) == P - 1
    assert o.lib().or_fp_pow(2, 64) == 0xFFFFFFFF
    assert o.lib().or_fp_pow(2, 96) == P - 1
    # 7 is a quadratic non-residue (lib.rs:337-341)
    assert o.lib().or_fp_pow(7, (P - 1) // 2) == P - 1


def test_field_differential_u128(oracle):
    rng = np.random.default_rng(0xB0)
    a = rng.integers(0, P, size=20000, dtype=np.uint64)
    b = rng.integers(0, P, size=20000, dtype=np.uint64)
    got = oracle.fp_mul_batch(a, b)
    for i in range(0, 20000, 97):
        assert int(got[i]) == (int(a[i]) * int(b[i])) % P


def test_fp2_inverse(oracle):
    rng = np.random.default_rng(2)
    for _ in range(50):
        x = (int(rng.integers(0, P, dtype=np.uint64)), int(rng.integers(0, P, dtype=np.uint64)))
        inv = oracle.fp2_inv(x)
        assert oracle.fp2_mul(x, inv) == (1, 0)


# --------------------------------------------------------------------------
# ChaCha8 FpStream byte identity
# (benchmarks/results/p7b-chacha8-fp-diff-2026-07-13-32653fd7e076.json; output
# format of rust/volta-bench/src/bin/p7b_chacha8_fp_vectors.rs:130-160)
# --------------------------------------------------------------------------

def chacha_vectors_text(o, mode, seed_hex, base, rows, count):
    seed = bytes.fromhex(seed_hex)
    lines = ["{", '  "schema":"p7b-chacha8-fp-diff-v1",', f'  "mode":"{mode}",',
             f'  "seed_hex":"{seed_hex}",', f'  "base_domain":"0x{base:016x}",',
             f'  "rows":{rows},', f'  "count":{count},', '  "values":[']
    for row in range(rows):
        s = o.FpStream(seed, base + row)
        items = []
        for _ in range(count):
            if mode == "fp":
                items.append(f'"0x{s.next_fp():016x}"')
            else:
                c0, c1 = s.next_fp2()
                items.append(f'["0x{c0:016x}","0x{c1:016x}"]')
        lines.append("    [" + ",".join(items) + "]" + ("" if row + 1 == rows else ","))
    lines += ["  ]", "}"]
    return ("\n".join(lines) + "\n").encode()


@pytest.mark.parametrize("mode,seed_hex,base,rows,count,nbytes,sha", [
    ("fp", "000102030405060708090a0b0c0d0e0f101112131415161718191a1b1c1d1e1f",
     0x0123456789ABCDEF, 3, 10, 868,
     "1570f825215b0e38da4857fc32b40a97b8bf0efed7f90f6c44431e801b7c2634"),
    ("fp2", "fffefdfcfbfaf9f8f7f6f5f4f3f2f1f0efeeedecebeae9e8e7e6e5e4e3e2e1e0",
     0xFEDCBA9876543210, 4, 17, 3238,
     "90abbd2a0773f9c455313a3eab8172a1647a2c7cea152fa71324ef996c220051"),
])
def test_chacha8_fpstream_golden(oracle, mode, seed_hex, base, rows, count, nbytes, sha):
    text = chacha_vectors_text(oracle, mode, seed_hex, base, rows, count)
    assert len(text) == nbytes
    assert hashlib.sha256(text).hexdigest() == sha


def test_chacha_rows_match_stream(oracle):
    seed = bytes(range(32))
    rows = oracle.chacha_fp_rows(seed, 5, 3, 11)
    for r in range(3):
        s = oracle.FpStream(seed, 5 + r)
        assert [s.next_fp() for _ in range(11)] == [int(x) for x in rows[r]]


# --------------------------------------------------------------------------
# BLAKE3 / Merkle
# --------------------------------------------------------------------------

def test_blake3_matches_pinned_crate(oracle):
    blake3 = pytest.importorskip("blake3")
    rng = np.random.default_rng(7)
    for n in [0, 1, 63, 64, 65, 1023, 1024, 1025, 2048, 3000, 4096, 8192, 65536 + 17]:
        data = rng.integers(0, 256, size=n, dtype=np.uint8).tobytes()
        assert oracle.blake3(data) == blake3.blake3(data).digest(), n


def test_merkle_known_answer_root(oracle):
    # rust/volta-pcs/src/merkle.rs:85-96
    leaves = np.array([np.frombuffer(oracle.blake3(bytes([i])), np.uint8) for i in range(16)])
    tree = oracle.merkle_tree(leaves)
    assert tree[-1].tobytes().hex() == (
        "4514d7cbd7a1955608774ff4ce369840a4e40e722caa2a8ccee2f6d0539d9f17")
    paths = oracle.merkle_paths(tree, 16, np.arange(16, dtype=np.uint32))
    assert paths.shape == (64, 32)


@pytest.mark.parametrize("rows,cols,root", [
    (32, 1024, "f427c1a8e4024b372e694b20215a860cfbf94c2463e2a5f76021243f1f8722e1"),
    (1024, 32768, "c90027afa35e9f24dd436d51d734b63e52c9788f50a1658c7a6a2a2685ca4d5f"),
])
def test_column_merkle_golden(oracle, rows, cols, root):
    # cuda/p7_blake3_merkle.cu:231-243; p7-gpu-blake3-merkle(-quick)-2026-07-11-3b0a916.json
    i = np.arange(rows * cols, dtype=np.uint64)
    m = oracle_mod_affine(i, 0x9E3779B9, 17)
    leaves = oracle.hash_fp_columns(m, rows, cols)
    tree = oracle.merkle_tree(leaves)
    assert tree[-1].tobytes().hex() == root


def oracle_mod_affine(i, mul, add):
    """(i*mul + add) mod p for i < 2^32 (exact in uint64 for these recipes)."""
    x = i.astype(np.uint64) * np.uint64(mul) + np.uint64(add)
    return np.where(x >= np.uint64(P), x - np.uint64(P), x).astype(np.uint64)


# --------------------------------------------------------------------------
# LogUp fraction tree (cuda/p7_logup_tree.cu:218-300)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("log2n,root_p,root_q,checksum", [
    (18, (10980606684603994831, 1600439578519942692),
     (14103360986930473702, 7831365882393612510), 0xac5455f699d2b292),
    (24, (10777469287391840112, 8202572568769278114),
     (17742598280587501369, 7640914676155300303), 0x0350749ee82bd237),
])
def test_logup_tree_golden(oracle, log2n, root_p, root_q, checksum):
    n = 1 << log2n
    alpha0 = 0x123456789ABCDEF0
    alpha1 = 0x0FEDCBA987654321
    i = np.arange(n, dtype=np.uint64)
    vals = ((i * np.uint64(37) + np.uint64(11)) & np.uint64(0xFFFF)).astype(np.uint16).view(np.int16)
    v64 = vals.astype(np.int64)
    x = np.where(v64 >= 0, v64.astype(np.uint64),
                 np.uint64(P) - (-v64).astype(np.uint64)).astype(np.uint64)
    a0 = np.uint64(alpha0)
    leaf = np.where(a0 >= x, a0 - x, a0 + (np.uint64(P) - x)).astype(np.uint64)
    p, q = oracle.logup_tree(leaf, None, n, alpha1, False)
    assert tuple(int(v) for v in p[0]) == root_p
    assert tuple(int(v) for v in q[0]) == root_q
    # checksum: per level from the leaves' parents up, interleaving (p_i, q_i)
    h = FNV0
    level = log2n - 1
    while level >= 0:
        off = (1 << level) - 1
        cnt = 1 << level
        inter = np.stack([p[off:off + cnt], q[off:off + cnt]], axis=1)
        h = oracle.fnv_u64(inter.reshape(-1), h)
        level -= 1
    assert h == checksum


# --------------------------------------------------------------------------
# LogUp general rounds + folds (cuda/p7_logup_rounds.cu:250-400)
# --------------------------------------------------------------------------

def rounds_inputs(log2n):
    n = 1 << log2n
    i = np.arange(n, dtype=np.uint64)
    cols = []
    for col in range(4):
        c0 = oracle_mod_affine(i, 0x9E3779B9 + 2 * col, 17 + col)
        c1 = oracle_mod_affine(i, 0x85EBCA6B + 4 * col, 29 + col)
        cols.append(np.ascontiguousarray(np.stack([c0, c1], axis=1)))
    j = np.arange(n // 2, dtype=np.uint64)
    s = np.ascontiguousarray(np.stack([oracle_mod_affine(j, 0xC2B2AE35, 31),
                                       oracle_mod_affine(j, 0x27D4EB2F, 43)], axis=1))
    chals = [(101 + 2 * k, 211 + 3 * k) for k in range(log2n)]
    return cols, s, chals


@pytest.mark.parametrize("log2n,checksum,blind_checksum", [
    (16, 0x7eaefbd02661f35b, 0xa0cd787a9d565b4d),
    (22, 0x26139daf10dc7707, 0x232b3848930c2f15),
])
def test_logup_rounds_golden(oracle, log2n, checksum, blind_checksum):
    """The clear rounds checksum (p7-gpu-logup-rounds*.json) and, over the
    same rounds, the blind one (cuda/p7_logup_blind_rounds.cu:505-551,
    p7-gpu-logup-blind-rounds*.json): the blind sink's root / round / split /
    product corrections hashed after the round messages and folds."""
    from oracle import blind
    cols, s, chals = rounds_inputs(log2n)
    h = FNV0
    length = 1 << log2n
    accs = []
    for rnd in range(log2n):
        pairs = length // 2
        acc = oracle.logup_general_round(*cols, s, pairs)
        accs.append([tuple(int(v) for v in a) for a in acc.reshape(4, 2)])
        h = oracle.fnv_u64(acc.reshape(-1), h)
        nxt = []
        for col in range(4):
            f = oracle.fold_rows(cols[col], 1, length, chals[rnd])
            h = oracle.fnv_u64(f.reshape(-1), h)
            nxt.append(f)
        cols = nxt
        length = pairs
    assert h == checksum
    splits = [tuple(int(v) for v in cols[col][0]) for col in range(4)]
    art = blind.blind_artifacts(accs, splits, blind.golden_inputs(log2n))
    assert blind.hash_artifacts(h, art) == blind_checksum


# --------------------------------------------------------------------------
# Batched NTT (cuda/p7_pcs_arithmetic.cu:204-262) and combine rows (263-318)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("rows,bits,msg_len,checksum", [
    (32, 12, 2304, 0xa87a560725f2d016),
    (1024, 15, 16896, 0xbe7b90425a4c7229),
])
def test_ntt_golden(oracle, rows, bits, msg_len, checksum):
    n = 1 << bits
    idx = np.arange(rows * n, dtype=np.uint64).reshape(rows, n)
    full = oracle_mod_affine(idx, 0x9E3779B9, 17)
    msgs = np.ascontiguousarray(full[:, :msg_len])
    out = oracle.ntt_batch(msgs, rows, msg_len, n)
    assert oracle.fnv_u64(out) == checksum


def test_ntt_matches_naive_dft(oracle):
    # rust/volta-pcs/src/ntt.rs:89-104: forward NTT equals the naive DFT
    n = 16
    rng = np.random.default_rng(3)
    a = rng.integers(0, P, size=n, dtype=np.uint64)
    out = oracle.ntt_batch(a, 1, n, n)
    w = pow(7, (P - 1) >> 4, P)
    for j in range(n):
        acc = 0
        for i in range(n):
            acc = (acc + int(a[i]) * pow(w, i * j, P)) % P
        assert acc == int(out[j])


# --------------------------------------------------------------------------
# Fused GEMM + requant + MAC correction (cuda/p7_fused_epilogue.cu:172-263)
# --------------------------------------------------------------------------

@pytest.mark.parametrize("m,k,n,out_ck,corr_ck", [
    (16, 128, 768, 0xd627d7c8948ce1e4, 0xdd63d6266710a934),
    (16, 128, 2304, 0xcdf862e2f38c3d44, 0x61b14ea07fa256bf),
    (16, 128, 3072, 0xed00f0c37fa1b89a, 0xc0fe66101c12085d),
    (100, 768, 768, 0x7fac93d5b09e3279, 0x6602b2041ac9cfc4),
    (100, 768, 2304, 0x98d0ad1723fb5ba4, 0x657f2372e3e080c3),
    (100, 768, 3072, 0x622a3f3b6103a2a0, 0x0a16ee945a99dea3),
])
def test_fused_epilogue_golden(oracle, m, k, n, out_ck, corr_ck):
    a = (((np.arange(m * k, dtype=np.int64) * 37 + 11) % 4001) - 2000).astype(np.int16)
    b = (((np.arange(k * n, dtype=np.int64) * 53 + 5) % 4001) - 2000).astype(np.int16)
    masks = oracle_mod_affine(np.arange(m * n, dtype=np.uint64), 0x9E3779B9, 17)
    out, corr = oracle.gemm_requant_auth(a, b, masks, m, k, n, 8)
    assert oracle.fnv_u64(out.view(np.uint16).astype(np.uint64)) == out_ck
    assert oracle.fnv_u64(corr) == corr_ck


def test_oracle_matches_reference_chacha_header(oracle):
    """Diff the oracle's FpStream against the reference's own host-compilable
    header cuda/volta_chacha8_fp.cuh (built into oracle/_ref by oracle/Makefile
    when the reference tree is present)."""
    import ctypes as C
    import os

    path = os.path.join(os.path.dirname(oracle.LIB_PATH), "..", "_ref", "libref_chacha.so")
    if not os.path.exists(path):
        pytest.skip("reference cross-check library not built (reference tree absent)")
    ref = C.CDLL(path)
    ref.ref_chacha_fp_rows.argtypes = [C.c_char_p, C.c_uint64, C.c_size_t, C.c_size_t, C.c_void_p]
    for seed, base, rows, count in [(bytes(range(32)), 0x0123456789ABCDEF, 3, 10),
                                    (bytes([0xA5] * 32), 2**64 - 5, 4, 1000)]:
        out = np.zeros(rows * count, dtype=np.uint64)
        ref.ref_chacha_fp_rows(seed, base, rows, count, out.ctypes.data_as(C.c_void_p))
        assert np.array_equal(out.reshape(rows, count), oracle.chacha_fp_rows(seed, base, rows, count))


# --------------------------------------------------------------------------
# int16 fixed-point layer (scripts/gpt2_fixed.py forward_layer fixture)
# --------------------------------------------------------------------------

def test_fixed_layer_oracle_matches_reference_mirror(oracle):
    """The oracle's forward primitives, composed as forward_layer, reproduce
    every intermediate of the reference's NumPy mirror (digests in
    tests/golden/fixed_layer_t8.npz, made by tests/golden/make_fixed_golden.py)."""
    import fixed_layer as fl

    g = np.load(fl.GOLDEN)
    seed, t = (int(v) for v in g["seed_t"])
    w, x = fl.synthetic_layer(seed, t)
    assert fl.weights_digest(w) == str(g["weights_digest"])
    assert fl.digest(x) == str(g["input_digest"])
    luts = {k: g[k] for k in ("exp", "gelu", "ln_rsqrt", "softmax_recip")}
    res = fl.forward_layer(fl.OracleOps(oracle), x, w, luts, t)
    assert res["errors"] == [0] * len(res["errors"])
    assert fl.check_against_golden(res) == []


def test_oracle_stream_skips_rejected_draw(oracle):
    """FpStream rejection sampling (lib.rs:255-262): the raw draw >= p at index
    45451 of FpStream([0x11;32], 2215) is skipped."""
    seed = bytes([0x11] * 32)
    raw = oracle.stream_u64(seed, 2215, 45460)
    assert raw[45451] >= np.uint64(P)
    rows = oracle.chacha_fp_rows(seed, 2215, 1, 45455)[0]
    assert np.array_equal(rows[:45451], raw[:45451])
    assert np.array_equal(rows[45451:], raw[45452:45456])
