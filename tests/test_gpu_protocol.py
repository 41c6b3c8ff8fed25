"""End-to-end protocol parity: the resident callers of libvolta_accel.so
(restating rust/volta-proto hadamard.rs and logup.rs) against the oracle's
clear provers, message for message."""

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


# (timing policy, fused fold + round extensions, scheduled drivers, cross-layer
# batches): the reference's round-by-round call sequence under deferred
# events, the fused round-by-round drivers under both policies, and the
# scheduled drivers (challenges first, one message download) without fusion,
# with fusion layer after layer, and with the cross-layer round batches.
@pytest.fixture(scope="module",
                params=[(0, False, False, False), (0, True, False, False), (1, True, False, False),
                        (1, False, True, False), (1, True, True, False), (1, True, True, True)],
                ids=["events-unfused", "events-fused", "counters-fused", "scheduled-unfused", "scheduled-fused",
                     "scheduled-batched"])
def prover(request):
    from volta_zk_b200 import accel

    policy, fused, scheduled, batched = request.param
    p = accel.Prover(policy=policy, fused=fused, scheduled=scheduled, batched=batched)
    yield p
    p.close()


def embed_i16(v):
    v64 = v.astype(np.int64)
    return np.where(v64 >= 0, v64.astype(np.uint64), np.uint64(P) - (-v64).astype(np.uint64)).astype(np.uint64)


@pytest.mark.parametrize("log2n", [1, 2, 10, 13, 16])
def test_triple_sumcheck_matches_oracle(prover, oracle, log2n):
    n = 1 << log2n
    seed = bytes([0x51] * 32)
    # config-1 style tables: FpStream rows lifted to Fp2 (c1 = 0), plus one Fp2 table
    a = np.zeros((n, 2), dtype=np.uint64)
    a[:, 0] = oracle.chacha_fp_rows(seed, 0, 1, n)[0]
    b = np.zeros((n, 2), dtype=np.uint64)
    b[:, 0] = oracle.chacha_fp_rows(seed, 1, 1, n)[0]
    c = oracle.chacha_fp2_rows_padded(seed, 2, 1, n, n)
    be = prover.backend
    ids = [be.upload_new(x) for x in (a, b, c)]
    chal = bytes([0x5A] * 32)
    msgs, finals = prover.triple_sumcheck(ids[0], ids[1], ids[2], n, chal)
    emsgs, efinals = oracle.triple_sumcheck(a, b, c, chal)
    assert np.array_equal(msgs, emsgs)
    assert np.array_equal(finals, efinals)
    # inputs are left untouched (resident callers fold into fresh buffers)
    assert np.array_equal(be.download_fp2(ids[0], n), a)
    for i in ids:
        be.free(i)


@pytest.mark.parametrize("log2n", [1, 2, 3, 10, 12, 13, 14, 16, 17])
def test_triple_sumcheck_fp_columns_match_oracle(prover, oracle, log2n):
    """Fp columns (tables with c1 = 0) give the proof of the lifted tables."""
    n = 1 << log2n
    seed = bytes([0x51] * 32)
    cols = [oracle.chacha_fp_rows(seed, t, 1, n)[0] for t in range(3)]
    lifted = []
    for col in cols:
        x = np.zeros((n, 2), dtype=np.uint64)
        x[:, 0] = col
        lifted.append(x)
    be = prover.backend
    ids = [be.upload_new(np.ascontiguousarray(col)) for col in cols]
    chal = bytes([0x5A] * 32)
    msgs, finals = prover.triple_sumcheck_fp(ids[0], ids[1], ids[2], n, chal)
    emsgs, efinals = oracle.triple_sumcheck(*lifted, chal)
    assert np.array_equal(msgs, emsgs)
    assert np.array_equal(finals, efinals)
    assert np.array_equal(be.download(ids[0], 8 * n), cols[0])  # the columns are left untouched
    for i in ids:
        be.free(i)


@pytest.mark.parametrize("log2f,log2t", [(1, 1), (4, 3), (10, 8), (14, 10), (16, 13)])
def test_logup_prove_matches_oracle(prover, oracle, log2f, log2t):
    nf, nt = 1 << log2f, 1 << log2t
    rng = np.random.default_rng(log2f * 100 + log2t)
    table = rng.integers(-32768, 32768, size=nt, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    f = table[idx]
    mult = np.bincount(idx, minlength=nt).astype(np.uint32)
    be = prover.backend
    f_col, t_col, m_col = be.upload_new(embed_i16(f)), be.upload_new(embed_i16(table)), be.upload_new(mult)
    seed, domain = bytes([0x4C] * 32), 0x1004
    cap = oracle.logup_prove_words(nf, nt)
    got = prover.logup_prove(f_col, nf, t_col, nt, m_col, seed, domain, cap)
    exp = oracle.logup_prove(f, table, mult, seed, domain)
    assert got.shape == exp.shape
    assert np.array_equal(got, exp)
    for i in (f_col, t_col, m_col):
        be.free(i)


def test_logup_roots_cross_check(prover, oracle):
    """LogUp soundness identity on the device proof: p_f q_t + p_t q_f = 0
    (logup.rs:1779-1784)."""
    nf, nt = 1 << 12, 1 << 9
    rng = np.random.default_rng(5)
    table = rng.integers(-32768, 32768, size=nt, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    mult = np.bincount(idx, minlength=nt).astype(np.uint32)
    be = prover.backend
    ids = [be.upload_new(embed_i16(table[idx])), be.upload_new(embed_i16(table)), be.upload_new(mult)]
    proof = prover.logup_prove(ids[0], nf, ids[1], nt, ids[2], bytes(32), 7, oracle.logup_prove_words(nf, nt))
    side_f = 2 + sum(2 * l + 4 for l in range(12))
    pf, qf = tuple(map(int, proof[1])), tuple(map(int, proof[2]))
    pt, qt = tuple(map(int, proof[1 + side_f])), tuple(map(int, proof[2 + side_f]))
    x = oracle.fp2_mul(pf, qt)
    y = oracle.fp2_mul(pt, qf)
    assert ((x[0] + y[0]) % P, (x[1] + y[1]) % P) == (0, 0)
    for i in ids:
        be.free(i)


@pytest.mark.parametrize("rows,msg_len,code_len,queries", [(1, 1, 2, 1), (8, 16, 64, 5), (64, 256, 1024, 32),
                                                           (256, 4096, 16384, 128)])
def test_ligero_commit_open_matches_oracle(prover, oracle, rows, msg_len, code_len, queries):
    row_seed, chal_seed = bytes([0x11] * 32), bytes([0x5A] * 32)
    got = prover.ligero_commit_open(row_seed, rows, msg_len, code_len, queries, chal_seed)
    exp = oracle.ligero_commit_open(row_seed, rows, msg_len, code_len, queries, chal_seed)
    assert got[0] == exp[0]
    for g, e in zip(got[1:], exp[1:]):
        assert np.array_equal(g, e)
