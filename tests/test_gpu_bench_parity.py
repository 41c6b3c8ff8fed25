"""Parity at the sizes the benchmark measures.

* the whole config-1 proof with bench.py's exact seeds and sizes (triple
  sumcheck over three 2^24 FpStream tables, LogUp of 2^24 GELU-table queries
  against the 2^16 table) against the oracle's clear provers;
* the reference's published 2^22 LogUp rounds+folds checksum
  (cuda/p7_logup_rounds.cu:250-400, p7-gpu-logup-rounds-2026-07-11-f7f54a2.json)
  and the 2^24 fraction-tree roots + all-layer checksum
  (cuda/p7_logup_tree.cu:218-315, p7-gpu-logup-tree-2026-07-11-5f7b443.json),
  both computed on the device;
* the config-2 commitment (8192 x 2^14 -> 2^16, 128 openings) against the
  oracle's composed commit + openings;
* the GPT2_FULL zero-knowledge commitment of bench.py's ligero_zk leg
  against the oracle's functions composed in the order of ligero.rs.
"""

import numpy as np
import pytest

import bench

P = 0xFFFFFFFF00000001
FNV0 = 0xCBF29CE484222325
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


def test_config1_proof_at_bench_size(prover, oracle):
    from volta_zk_b200 import accel

    log2n, log2q, log2t = 24, 24, 16
    n, n_f, n_t = 1 << log2n, 1 << log2q, 1 << log2t
    be = prover.backend
    cols = []
    for t in range(3):  # the bench's resident tables: FpStream rows generated on the device
        col = be.alloc(8 * n)
        be.call("chacha8_prover_secret_fp_rows_device", col, 0, bench.SUMCHECK_SEED, t, 1, n)
        cols.append(col)
    f, table, mult = bench.logup_inputs(log2q, log2t, accel.fpstream_u64)
    ids = [be.upload_new(bench.embed_i16(f)), be.upload_new(bench.embed_i16(table)), be.upload_new(mult)]
    msgs, finals = prover.triple_sumcheck_fp(*cols, n, bench.TRANSCRIPT_SEED)
    proof = prover.logup_prove(ids[0], n_f, ids[1], n_t, ids[2], bench.LOGUP_SEED, bench.LOGUP_DOMAIN,
                               bench.proof_words(n_f, n_t))
    tabs = []
    for col in cols:
        x = np.zeros((n, 2), dtype=np.uint64)
        x[:, 0] = be.download(col, 8 * n)
        tabs.append(x)
        be.free(col)
    for i in ids:
        be.free(i)
    # the device tables are the host stream's values
    assert np.array_equal(tabs[2][:4096, 0], accel.fpstream_fp_rows(bench.SUMCHECK_SEED, 2, 4096))
    emsgs, efinals = oracle.triple_sumcheck(*tabs, bench.TRANSCRIPT_SEED)
    assert np.array_equal(msgs, emsgs) and np.array_equal(finals, efinals)
    del tabs
    eproof = oracle.logup_prove(f, table, mult, bench.LOGUP_SEED, bench.LOGUP_DOMAIN)
    assert np.array_equal(proof, eproof)


def _fp2c(v):
    from volta_zk_b200 import accel

    return accel.fp2(v)


def test_logup_rounds_golden_2_22_on_device(prover, oracle):
    """22 rounds of logup_general_round_device + logup_fold4_device over the
    closed-form 2^22 inputs; FNV checksum of every message and fold."""
    import ctypes as C

    from tests.test_oracle_golden import rounds_inputs

    be = prover.backend
    log2n = 22
    cols, s, chals = rounds_inputs(log2n)
    ids = [be.upload_new(c) for c in cols]
    sid = be.upload_new(s)
    del cols
    h = FNV0
    length = 1 << log2n
    for rnd in range(log2n):
        pairs = length // 2
        acc = np.zeros((4, 2), dtype=np.uint64)
        be.call("logup_general_round_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, sid, 0, pairs,
                acc.ctypes.data_as(C.c_void_p))
        h = oracle.fnv_u64(acc.reshape(-1), h)
        outs = [be.alloc(16 * pairs) for _ in range(4)]
        be.call("logup_fold4_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, pairs, _fp2c(chals[rnd]),
                outs[0], 0, outs[1], 0, outs[2], 0, outs[3], 0)
        for k in range(4):
            h = oracle.fnv_u64(be.download_fp2(outs[k], pairs).reshape(-1), h)
            be.free(ids[k])
        ids = outs
        length = pairs
    for i in ids + [sid]:
        be.free(i)
    assert h == 0x26139daf10dc7707


def test_logup_tree_golden_2_24_on_device(prover, oracle):
    be = prover.backend
    n = 1 << 24
    a0, a1 = 0x123456789ABCDEF0, 0x0FEDCBA987654321
    i = np.arange(n, dtype=np.uint64)
    vals = ((i * np.uint64(37) + np.uint64(11)) & np.uint64(0xFFFF)).astype(np.uint16).view(np.int16)
    x = bench.embed_i16(vals)
    leaf = np.where(np.uint64(a0) >= x, np.uint64(a0) - x, np.uint64(a0) + (np.uint64(P) - x)).astype(np.uint64)
    il = be.upload_new(leaf)
    ip, iq = be.alloc(16 * (n - 1)), be.alloc(16 * (n - 1))
    be.call("logup_tree_device", il, 0, 0, 0, n, a1, 0, ip, 0, iq, 0)
    p, q = be.download_fp2(ip, n - 1), be.download_fp2(iq, n - 1)
    for b in (il, ip, iq):
        be.free(b)
    assert tuple(int(v) for v in p[0]) == (10777469287391840112, 8202572568769278114)
    assert tuple(int(v) for v in q[0]) == (17742598280587501369, 7640914676155300303)
    h = FNV0
    for level in range(23, -1, -1):
        off, cnt = (1 << level) - 1, 1 << level
        h = oracle.fnv_u64(np.ascontiguousarray(np.stack([p[off:off + cnt], q[off:off + cnt]], axis=1)).reshape(-1),
                           h)
    assert h == 0x0350749ee82bd237


def test_config2_commitment_at_bench_size(prover, oracle):
    rows, msg_len, code_len, queries = 8192, 1 << 14, 1 << 16, 128
    got = prover.ligero_commit_open(bench.LIGERO_ROW_SEED, rows, msg_len, code_len, queries, bench.TRANSCRIPT_SEED)
    exp = oracle.ligero_commit_open(bench.LIGERO_ROW_SEED, rows, msg_len, code_len, queries, bench.TRANSCRIPT_SEED)
    assert got[0] == exp[0]
    for g, e in zip(got[1:], exp[1:]):
        assert np.array_equal(g, e)


def test_gpt2_full_zk_commitment_at_bench_size(prover, oracle):
    from tests.test_gpu_ligero_zk import expected

    z = bench.ligero_zk_inputs()
    args = (z["w"], z["rows"], z["col_bits"], z["pad"], z["code_bits"], bench.LIGERO_ROW_SEED, z["claims"],
            bench.LIGERO_MASK_SEED, z["c"], z["idx"])
    got = prover.ligero_commit_open_zk(*args)
    exp = expected(oracle, *args)
    for key in ("root", "mask_root", "u_c", "u_g", "s", "columns", "mask_columns", "paths", "mask_paths"):
        assert np.array_equal(np.asarray(got[key]).reshape(np.asarray(exp[key]).shape), exp[key]), key
