"""Sharded single proofs with the device engine: each shard's local work
runs through libvolta_accel on its slice (here G shards take turns on one
GPU), the product's host logic combines them, and the result must equal the
oracle's one-process proof word for word."""

import numpy as np
import pytest

import sharded_emulation as em
from volta_zk_b200 import sharded as sh

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


@pytest.mark.parametrize("base", [False, True], ids=["fp2-tables", "fp-columns"])
@pytest.mark.parametrize("log2n,G", [(1, 2), (6, 2), (12, 4), (16, 8)])
def test_sharded_triple(prover, oracle, log2n, G, base):
    n = 1 << log2n
    seed = bytes([0x5A] * 32)
    rng = np.random.default_rng(log2n)
    a, b, c = (rng.integers(0, 2**64 - 2**32 + 1, size=(n, 2), dtype=np.uint64) for _ in range(3))
    if base:  # Fp columns: tables with c1 = 0
        for x in (a, b, c):
            x[:, 1] = 0
    be = prover.backend
    parts = []
    for g in range(G):
        sl = slice(g * n // G, (g + 1) * n // G)
        if base:
            ids = [be.upload_new(np.ascontiguousarray(x[sl, 0])) for x in (a, b, c)]
            m, f = prover.triple_sumcheck_fp(*ids, n // G, seed)
        else:
            ids = [be.upload_new(np.ascontiguousarray(x[sl])) for x in (a, b, c)]
            m, f = prover.triple_sumcheck(*ids, n // G, seed)
        parts.append(np.concatenate([m, f]))
        for i in ids:
            be.free(i)
    msgs, finals = sh.triple_finish(parts, n, seed)
    em_msgs, em_finals = oracle.triple_sumcheck(a, b, c, seed)
    assert np.array_equal(msgs, em_msgs)
    assert np.array_equal(finals, em_finals)


@pytest.mark.parametrize("log2f,log2t,G", [(2, 2, 2), (10, 6, 2), (14, 10, 4), (16, 8, 8)])
def test_sharded_logup(prover, oracle, log2f, log2t, G):
    rng = np.random.default_rng(log2f + G)
    table = rng.integers(-32768, 32768, size=1 << log2t, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, 1 << log2t, size=1 << log2f)
    f = table[idx]
    mult = np.bincount(idx, minlength=1 << log2t).astype(np.uint32)
    nf, nt = 1 << log2f, 1 << log2t
    fe, te = em.embed_i16(f), em.embed_i16(table)
    seed, domain = bytes([0x4C] * 32), 0x1004
    be = prover.backend
    parts = []
    for g in range(G):
        ids = [be.upload_new(np.ascontiguousarray(x[g * len(x) // G:(g + 1) * len(x) // G])) for x in (fe, te, mult)]
        parts.append(prover.logup_local(ids[0], nf // G, ids[1], nt // G, ids[2], G.bit_length() - 1, seed, domain))
        for i in ids:
            be.free(i)
    got = sh.logup_finish(parts, nf, nt, seed, domain)
    exp = oracle.logup_prove(f, table, mult, seed, domain)
    assert np.array_equal(got, exp)


def test_local_engine_matches_cpu_emulation(prover, oracle):
    """The device shard engine's raw words equal the CPU emulation's."""
    rng = np.random.default_rng(5)
    table = rng.integers(-32768, 32768, size=64, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, 64, size=512)
    f, mult = table[idx], np.bincount(idx, minlength=64).astype(np.uint32)
    fe, te = em.embed_i16(f), em.embed_i16(table)
    seed, domain = bytes([0x4C] * 32), 7
    be = prover.backend
    ids = [be.upload_new(np.ascontiguousarray(x[: len(x) // 4])) for x in (fe, te, mult)]
    got = prover.logup_local(ids[0], 128, ids[1], 16, ids[2], 2, seed, domain)
    exp, _ = em.logup_local(oracle, fe[:128], te[:16], mult[:16], 2, seed, domain)
    assert np.array_equal(got, exp)
    for i in ids:
        be.free(i)


@pytest.mark.parametrize("rows,msg_len,code_len,queries,G", [(256, 64, 256, 8, 2), (1024, 256, 1024, 16, 4),
                                                              (2048, 1024, 4096, 32, 8)])
def test_sharded_ligero_matches_single_gpu(prover, rows, msg_len, code_len, queries, G):
    """The row-sharded commitment (G shards taking turns on one GPU, exchanges
    done in-process) equals the one-GPU commitment and openings."""
    be = prover.backend
    seed, chal = bytes([0x11] * 32), bytes([0x5A] * 32)
    rl, slab = rows // G, code_len // G
    enc = [sh.ligero_shard_encode(be, seed, g * rl, rl, msg_len, code_len) for g in range(G)]
    trees, roots = [], []
    for s in range(G):
        recv = np.stack([enc[g][1].reshape(G, slab, 32)[s] for g in range(G)])
        t, r = sh.ligero_shard_tree(be, recv, G, slab)
        trees.append(t)
        roots.append(r)
    top = sh.ligero_top_tree(be, np.stack(roots))
    idx = sh.ligero_query_indices(chal, queries, code_len)
    opened = [sh.ligero_shard_open(be, enc[g][0], rl, code_len, trees[g], slab, g, idx) for g in range(G)]
    cols, paths = sh.ligero_assemble([o[0] for o in opened], [o[1] for o in opened], top, idx, slab)
    root, eidx, ecols, epaths = prover.ligero_commit_open(seed, rows, msg_len, code_len, queries, chal)
    assert top[-1].tobytes() == root
    assert np.array_equal(idx, eidx)
    assert np.array_equal(cols, ecols)
    assert np.array_equal(paths, epaths)
    for g in range(G):
        be.free(enc[g][0])
        be.free(trees[g])


@pytest.mark.parametrize("log2n,log2f,log2t,G", [(6, 6, 4, 2), (14, 14, 10, 4), (16, 16, 12, 8)])
def test_sharded_proof_local_matches_oracle(prover, oracle, log2n, log2f, log2t, G):
    """vzh_proof_local (triple on Fp columns + both LogUp sides, one
    download) per shard, then the two finishes, equal the one-process
    proofs; this is ShardedProver.prove's flow with the shards taking turns."""
    n, nf, nt = 1 << log2n, 1 << log2f, 1 << log2t
    rng = np.random.default_rng(log2n * 7 + G)
    cols = [rng.integers(0, 2**64 - 2**32 + 1, size=n, dtype=np.uint64) for _ in range(3)]
    lifted = [np.stack([x, np.zeros_like(x)], axis=1) for x in cols]
    table = rng.integers(-32768, 32768, size=nt, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    f = table[idx]
    mult = np.bincount(idx, minlength=nt).astype(np.uint32)
    fe, te = em.embed_i16(f), em.embed_i16(table)
    tseed, lseed, domain = bytes([0x5A] * 32), bytes([0x4C] * 32), 0x1004
    be = prover.backend
    parts = []
    for g in range(G):
        def part(x):
            return np.ascontiguousarray(x[g * len(x) // G:(g + 1) * len(x) // G])
        ids = [be.upload_new(part(x)) for x in cols + [fe, te, mult]]
        parts.append(prover.proof_local(ids[0], ids[1], ids[2], n // G, True, tseed, ids[3], nf // G, ids[4],
                                        nt // G, ids[5], G.bit_length() - 1, lseed, domain))
        for i in ids:
            be.free(i)
    kt = 3 * ((n // G).bit_length() - 1) + 3
    msgs, finals = sh.triple_finish([p[:kt] for p in parts], n, tseed)
    em_msgs, em_finals = oracle.triple_sumcheck(*lifted, tseed)
    assert np.array_equal(msgs, em_msgs)
    assert np.array_equal(finals, em_finals)
    got = sh.logup_finish([p[kt:] for p in parts], nf, nt, lseed, domain)
    assert np.array_equal(got, oracle.logup_prove(f, table, mult, lseed, domain))


@pytest.mark.parametrize("m,k,n,G", [(1024, 768, 768, 4), (100, 768, 2304, 3), (5, 3072, 768, 8)])
def test_auth_rows_shards_match_single_gpu_and_oracle(prover, oracle, m, k, n, G):
    """The VOLE-MAC epilogue split by row blocks (G shards taking turns on
    one GPU): each block's device masks and fused GEMM epilogue equal the
    single-call output and corrections rows, and the oracle's."""
    be = prover.backend
    rng = np.random.default_rng(m + n + G)
    a = rng.integers(-900, 900, size=m * k).astype(np.int16)
    b = rng.integers(-900, 900, size=k * n).astype(np.int16)
    seed, tag, shift = bytes([0x4D] * 32), 0x0A0B0C, 10
    ai, bi = be.upload_new(a), be.upload_new(b)
    _, _, wy, wc = sh.auth_gemm_rows_shard(be, 0, 1, ai, bi, m, k, n, shift, seed, tag)
    whole_y = be.download(wy, 2 * m * n, dtype=np.int16)
    whole_c = be.download(wc, 8 * m * n)
    ey, ec = oracle.gemm_requant_auth(a, b, oracle.chacha_fp_rows(seed, tag << 32, m, n).reshape(-1), m, k, n, shift)
    assert np.array_equal(whole_y, ey) and np.array_equal(whole_c, ec)
    for g in range(G):
        row0, rows, out, corr = sh.auth_gemm_rows_shard(be, g, G, ai, bi, m, k, n, shift, seed, tag)
        if not rows:
            continue
        assert np.array_equal(be.download(out, 2 * rows * n, dtype=np.int16), whole_y[row0 * n:(row0 + rows) * n])
        assert np.array_equal(be.download(corr, 8 * rows * n), whole_c[row0 * n:(row0 + rows) * n])
        be.free(out)
        be.free(corr)
    for i in (ai, bi, wy, wc):
        be.free(i)
