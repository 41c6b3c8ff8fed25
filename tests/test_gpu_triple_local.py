"""On-chip triple-product rounds (volta_b200_triple_local_device and
volta_b200_triple_flush_device) against the oracle's round-by-round
functions: 13 rounds of triple_product_round + fold_rows, tile launches in
any order and any split, Fp columns and Fp2 tables."""

import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
TILE = 8192
ROUNDS = 13
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=1)
    yield b
    b.close()


def expected(oracle, tables, rs):
    """Messages of rounds 0 .. 12 and the round-13 tables, round by round."""
    cur = [t.copy() for t in tables]
    msgs = []
    for r in rs:
        n = cur[0].shape[0]
        msgs.append(oracle.triple_product_round(cur[0], cur[1], cur[2], n // 2))
        cur = [oracle.fold_rows(x, 1, n, tuple(int(v) for v in r)) for x in cur]
    return np.concatenate(msgs), cur


def run_local(be, base, ids, n, rs, splits):
    lib = be.lib
    tiles = n // TILE
    r_id = be.upload_new(np.ascontiguousarray(rs))
    acc = be.alloc(ROUNDS * 3 * 4 * 8)
    assert lib.volta_cuda_resident_zero(be.ctx, acc, 0, ROUNDS * 3 * 4 * 8) == 0
    folds = [be.alloc(16 * tiles) for _ in range(3)]
    out = be.alloc(16 * 3 * ROUNDS)
    for tile0, count in splits:
        rc = lib.volta_b200_triple_local_device(be.ctx, int(base), ids[0], ids[1], ids[2], n, tile0, count, r_id, 0,
                                                acc, folds[0], folds[1], folds[2])
        assert rc == 0, be.last_error()
    assert lib.volta_b200_triple_flush_device(be.ctx, acc, out, 0) == 0, be.last_error()
    msgs = be.download_fp2(out, 3 * ROUNDS)
    fold = [be.download_fp2(f, tiles) for f in folds]
    zero = be.download(acc, ROUNDS * 3 * 4 * 8)
    for x in [r_id, acc, out] + folds:
        be.free(x)
    return msgs, fold, zero


@pytest.mark.parametrize("base", [True, False], ids=["fp-columns", "fp2-tables"])
@pytest.mark.parametrize("log2n,splits", [
    (13, [(0, 1)]),
    (15, [(2, 2), (0, 2)]),          # chunks in reverse order
    (16, [(7, 1), (0, 3), (3, 4)]),  # uneven chunks, out of order
    (18, [(0, 32)]),
])
def test_local_rounds_match_round_by_round(be, oracle, base, log2n, splits):
    n = 1 << log2n
    rng = np.random.default_rng(log2n * 7 + base)
    if base:
        cols = [rng.integers(0, P, size=n, dtype=np.uint64) for _ in range(3)]
        tables = []
        for col in cols:
            x = np.zeros((n, 2), dtype=np.uint64)
            x[:, 0] = col
            tables.append(x)
        ids = [be.upload_new(col) for col in cols]
    else:
        tables = [rng.integers(0, P, size=(n, 2), dtype=np.uint64) for _ in range(3)]
        ids = [be.upload_new(t) for t in tables]
    rs = rng.integers(0, P, size=(ROUNDS, 2), dtype=np.uint64)
    msgs, fold, acc_after = run_local(be, base, ids, n, rs, splits)
    emsgs, efold = expected(oracle, tables, rs)
    assert np.array_equal(msgs, emsgs)
    for got, want in zip(fold, efold):
        assert np.array_equal(got, want)
    assert not acc_after.any()  # the flush leaves the counters zeroed
    for i in ids:
        be.free(i)


def test_local_rounds_extreme_values(be, oracle):
    """Entries at p - 1 and 0 (largest differences, every carry path)."""
    n = 1 << 14
    rng = np.random.default_rng(5)
    pick = rng.integers(0, 2, size=(n, 2)).astype(bool)
    tables = [np.where(pick, np.uint64(P - 1), np.uint64(0)).astype(np.uint64) for _ in range(3)]
    tables[1] = np.where(~pick, np.uint64(P - 1), np.uint64(0)).astype(np.uint64)
    ids = [be.upload_new(t) for t in tables]
    rs = np.full((ROUNDS, 2), P - 1, dtype=np.uint64)
    msgs, fold, _ = run_local(be, False, ids, n, rs, [(0, 2)])
    emsgs, efold = expected(oracle, tables, rs)
    assert np.array_equal(msgs, emsgs)
    for got, want in zip(fold, efold):
        assert np.array_equal(got, want)
    for i in ids:
        be.free(i)


def test_local_rejects_bad_geometry(be):
    lib = be.lib
    a = be.alloc(8 * 4 * TILE)
    acc = be.alloc(ROUNDS * 3 * 4 * 8)
    r = be.alloc(16 * ROUNDS)
    f = be.alloc(16 * 4)
    # shorter than one tile; not a power of two; tiles past the end; no tiles
    for n, tile0, tiles in [(4096, 0, 1), (3 * TILE, 0, 1), (TILE, 1, 1), (TILE, 0, 0)]:
        rc = lib.volta_b200_triple_local_device(be.ctx, 1, a, a, a, n, tile0, tiles, r, 0, acc, f, f, f)
        assert rc != 0
    # a fold output shorter than the tiles
    g = be.alloc(16)
    assert lib.volta_b200_triple_local_device(be.ctx, 1, a, a, a, 4 * TILE, 0, 4, r, 0, acc, g, f, f) != 0
    for x in (a, acc, r, f, g):
        be.free(x)
