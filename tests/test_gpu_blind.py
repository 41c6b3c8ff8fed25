"""Blind LogUp on the device: the all-rounds driver and the blind corrections.

The reference's blind-rounds benchmark (cuda/p7_logup_blind_rounds.cu,
published all_rounds_checksum in benchmarks/results/p7-gpu-logup-blind-
rounds*.json) runs the general LogUp rounds and folds over four closed-form
vectors and turns every message into a correction against a mask
(blind_begin / blind_round / blind_finish, the arithmetic of BlindSink in
rust/volta-proto/src/logup.rs:1903-2000).  Here the rounds run through
volta_b200_logup_rounds_device and the corrections through
volta_b200_logup_blind_corrections_device; the checksum is FNV over each
round's accumulators and folded vectors, then the corrections, exactly as
the benchmark hashes them.  Random cases compare with the oracle.
"""

import ctypes as C

import numpy as np
import pytest

from tests.test_oracle_golden import rounds_inputs

P = 0xFFFFFFFF00000001
FNV0 = 0xCBF29CE484222325
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=0)
    yield b
    b.close()


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def run_rounds(be, cols, s, chals):
    """Upload, run every round, return (ids to free, ladder ids, msgs (L+1)x4x2)."""
    n = cols[0].shape[0]
    L = n.bit_length() - 1
    ids = [be.upload_new(c) for c in cols]
    sid = be.upload_new(s)
    lad = [be.alloc(16 * max(n - 2, 1)) for _ in range(4)]
    out = be.alloc(16 * (4 * L + 4))
    r = np.ascontiguousarray(np.array(chals, dtype=np.uint64).reshape(L, 2))
    be.check(be.lib.volta_b200_logup_rounds_device(be.ctx, *ids, n, sid, 0, ptr(r), *lad, out, 0), "logup_rounds")
    msgs = be.download_fp2(out, 4 * L + 4).reshape(L + 1, 4, 2)
    return ids + [sid], lad, out, msgs


def blind_call(be, jobs):
    from volta_zk_b200 import accel

    arr = (accel.BlindJob * len(jobs))(*jobs)
    be.check(be.lib.volta_b200_logup_blind_corrections_device(be.ctx, arr, len(jobs)), "blind_corrections")


def job(raw, raw_off, root, sched, sched_off, mask, mask_off, out, out_off, lam, rounds):
    from volta_zk_b200 import accel

    return accel.BlindJob(raw, raw_off, root, 0, sched, sched_off, mask, mask_off, out, out_off,
                          accel.fp2(lam), rounds, 0)


def mask_vector(inp):
    flat = list(inp["root_masks"]) + [m for pair in inp["round_masks"] for m in pair] \
        + list(inp["split_masks"]) + list(inp["prod_masks"])
    return np.array(flat, dtype=np.uint64).reshape(-1, 2)


def artifacts_flat(art):
    flat = art["root"] + [x for row in art["rounds"] for x in row] + art["split"] + art["prod"]
    return np.array(flat, dtype=np.uint64).reshape(-1, 2)


@pytest.mark.parametrize("log2n,clear,blind", [
    (16, 0x7eaefbd02661f35b, 0xa0cd787a9d565b4d),
    (22, 0x26139daf10dc7707, 0x232b3848930c2f15),
])
def test_blind_rounds_golden(be, oracle, log2n, clear, blind):
    from oracle import blind as ob

    cols, s, chals = rounds_inputs(log2n)
    n = 1 << log2n
    inp = ob.golden_inputs(log2n)
    free, lad, out, msgs = run_rounds(be, cols, s, chals)
    levels = [be.download_fp2(lad[k], n - 2) for k in range(4)]
    h = FNV0
    for j in range(log2n):
        h = oracle.fnv_u64(msgs[j].reshape(-1), h)
        for k in range(4):
            if j + 1 < log2n:
                at, cnt = n - 2 * (n >> (j + 1)), n >> (j + 1)
                h = oracle.fnv_u64(levels[k][at:at + cnt].reshape(-1), h)
            else:
                h = oracle.fnv_u64(msgs[log2n][k].reshape(-1), h)
    assert h == clear
    # blind corrections on the device from the resident messages
    sched = np.array(inp["points"] + inp["challenges"], dtype=np.uint64).reshape(-1, 2)
    sid, mid = be.upload_new(sched), be.upload_new(mask_vector(inp))
    rid = be.upload_new(np.array(inp["roots"], dtype=np.uint64))
    nout = 2 + 2 * log2n + 7
    cid = be.alloc(16 * nout)
    blind_call(be, [job(out, 0, rid, sid, 0, mid, 0, cid, 0, inp["lambda"], log2n)])
    corr = be.download_fp2(cid, nout)
    h2 = h
    for x in corr:
        h2 = ob.fnv_fp2(h2, x)
    assert h2 == blind
    # and the same artifacts from the oracle's blind sink on the device messages
    accs = [[tuple(int(v) for v in a) for a in msgs[j]] for j in range(log2n)]
    splits = [tuple(int(v) for v in msgs[log2n][k]) for k in range(4)]
    assert np.array_equal(corr, artifacts_flat(ob.blind_artifacts(accs, splits, inp)))
    for i in free + lad + [out, sid, mid, rid, cid]:
        be.free(i)


@pytest.mark.parametrize("log2n", [1, 2, 3, 7, 12, 15])
def test_rounds_driver_matches_oracle(be, oracle, log2n):
    n = 1 << log2n
    rng = np.random.default_rng(log2n)
    cols = [rng.integers(0, P, size=(n, 2), dtype=np.uint64) for _ in range(4)]
    s = rng.integers(0, P, size=(max(n // 2, 1), 2), dtype=np.uint64)
    chals = [tuple(int(v) for v in rng.integers(0, P, size=2, dtype=np.uint64)) for _ in range(log2n)]
    free, lad, out, msgs = run_rounds(be, cols, s, chals)
    cur, length = cols, n
    for j in range(log2n):
        exp = oracle.logup_general_round(*cur, s, length // 2)
        assert np.array_equal(msgs[j], exp.reshape(4, 2)), j
        cur = [oracle.fold_rows(cur[k], 1, length, chals[j]) for k in range(4)]
        length //= 2
    assert np.array_equal(msgs[log2n], np.stack([cur[k][0] for k in range(4)]))
    for i in free + lad + [out]:
        be.free(i)


def test_blind_corrections_many_jobs(be, oracle):
    """130 layer jobs in one call (three launches of 64), mixed rounds, with
    and without a root, at offsets inside shared buffers; each against the
    oracle's blind sink."""
    from oracle import blind as ob

    rng = np.random.default_rng(11)
    rounds = [int(x) for x in rng.integers(0, 24, size=130)]
    rounds[0], rounds[1] = 0, 64
    raw_off, sched_off, mask_off, out_off = [], [], [], []
    a = b = m = o = 0
    roots = []
    for i, rd in enumerate(rounds):
        root = i % 3 == 0
        roots.append(root)
        raw_off.append(a)
        sched_off.append(b)
        mask_off.append(m)
        out_off.append(o)
        a += 4 * rd + 4 + 1
        b += 2 * rd + 3
        m += 2 * rd + 7 + (2 if root else 0)
        o += 2 * rd + 7 + (2 if root else 0) + 1
    raw = rng.integers(0, P, size=(a, 2), dtype=np.uint64)
    sched = rng.integers(0, P, size=(max(b, 1), 2), dtype=np.uint64)
    masks = rng.integers(0, P, size=(m, 2), dtype=np.uint64)
    rootv = rng.integers(0, P, size=(2 * len(rounds), 2), dtype=np.uint64)
    lams = rng.integers(0, P, size=(len(rounds), 2), dtype=np.uint64)
    ids = [be.upload_new(x) for x in (raw, sched, masks, rootv)]
    cid = be.alloc(16 * o)
    jobs = []
    for i, rd in enumerate(rounds):
        jb = job(ids[0], raw_off[i], ids[3] if roots[i] else 0, ids[1], sched_off[i], ids[2], mask_off[i],
                 cid, out_off[i], lams[i], rd)
        jb.root_offset = 2 * i
        jobs.append(jb)
    blind_call(be, jobs)
    got = be.download_fp2(cid, o)
    for i, rd in enumerate(rounds):
        acc = raw[raw_off[i]:raw_off[i] + 4 * rd].reshape(rd, 4, 2)
        splits = raw[raw_off[i] + 4 * rd:raw_off[i] + 4 * rd + 4]
        mk = masks[mask_off[i]:]
        lead = 2 if roots[i] else 0
        inp = {
            "roots": rootv[2 * i:2 * i + 2] if roots[i] else [(0, 0), (0, 0)],
            "root_masks": mk[:2] if roots[i] else [(0, 0), (0, 0)],
            "lambda": lams[i],
            "points": sched[sched_off[i]:sched_off[i] + rd],
            "challenges": sched[sched_off[i] + rd:sched_off[i] + 2 * rd],
            "round_masks": mk[lead:lead + 2 * rd].reshape(rd, 2, 2),
            "split_masks": mk[lead + 2 * rd:lead + 2 * rd + 4],
            "prod_masks": mk[lead + 2 * rd + 4:lead + 2 * rd + 7],
        }
        art = ob.blind_artifacts(acc, splits, inp)
        exp = artifacts_flat(art)
        if not roots[i]:
            exp = exp[2:]
        assert np.array_equal(got[out_off[i]:out_off[i] + len(exp)], exp), i
    for i in ids + [cid]:
        be.free(i)


def test_blind_entry_points_reject_bad_geometry(be):
    from volta_zk_b200 import accel

    ids = [be.alloc(16 * 8) for _ in range(4)]
    sid, out = be.alloc(16 * 8), be.alloc(16 * 64)
    r = np.zeros((4, 2), dtype=np.uint64)
    # not a power of two
    assert be.lib.volta_b200_logup_rounds_device(be.ctx, *ids, 6, sid, 0, ptr(r), *ids, out, 0) != 0
    # non-canonical challenge
    r[1, 0] = P
    assert be.lib.volta_b200_logup_rounds_device(be.ctx, *ids, 8, sid, 0, ptr(r), *ids, out, 0) != 0
    # more than 64 rounds in one blind job, and a region past a buffer's end
    too_many = job(out, 0, 0, sid, 0, out, 0, out, 0, (1, 2), 65)
    arr = (accel.BlindJob * 1)(too_many)
    assert be.lib.volta_b200_logup_blind_corrections_device(be.ctx, arr, 1) != 0
    past_end = job(out, 60, 0, sid, 0, out, 0, out, 0, (1, 2), 3)
    arr = (accel.BlindJob * 1)(past_end)
    assert be.lib.volta_b200_logup_blind_corrections_device(be.ctx, arr, 1) != 0
    for i in ids + [sid, out]:
        be.free(i)


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


def embed_i16(x):
    v = np.asarray(x, dtype=np.int64)
    out = v.astype(np.uint64)
    out[v < 0] -= np.uint64(0xFFFFFFFF)  # 2^64 + v - (2^32 - 1) = p + v
    return out


@pytest.mark.parametrize("log2f,log2t", [(1, 1), (4, 3), (10, 8), (14, 10), (16, 13)])
def test_blind_logup_prove_matches_oracle(prover, oracle, log2f, log2t):
    """The whole blind LogUp proof (logup.rs:3184-3225) on the device's
    scheduled rounds: the BlindLogupProof wire bytes, the transcript's
    canonical binding digest, its charged bytes and the correlation-domain
    cursor equal the oracle's blind prover."""
    from oracle import blind as ob

    rng = np.random.default_rng(log2f * 100 + log2t)
    nf, nt = 1 << log2f, 1 << log2t
    table = rng.integers(-32768, 32768, size=nt).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    f = table[idx]
    mult = np.bincount(idx, minlength=nt).astype(np.uint32)
    be = prover.backend
    ids = [be.upload_new(x) for x in (embed_i16(f), embed_i16(table), mult)]
    tx_seed, corr_seed, base = bytes([0x5A] * 32), bytes([0x4D] * 32), 0x3_0000
    got = prover.blind_logup_prove(ids[0], nf, ids[1], nt, ids[2], tx_seed, corr_seed, base)
    exp = ob.blind_logup_prove(oracle, f, table, mult, tx_seed, corr_seed, base)
    assert got[0] == exp[0]
    assert got[1:] == exp[1:]
    for i in ids:
        be.free(i)
