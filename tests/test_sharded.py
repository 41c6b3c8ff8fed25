"""Sharded single proof (volta_zk_b200/sharded.py) on the CPU: shard work
emulated with the oracle, combined by the product's host logic, compared
with the oracle's one-process proof; and the same across two gloo ranks
through torch.distributed (the multi-GPU path's host side)."""

import os
import socket

import numpy as np
import pytest

import sharded_emulation as em
from volta_zk_b200 import sharded as sh

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.usefixtures("package_built")


def tables(oracle, n):
    seed = bytes([0x51] * 32)
    out = []
    for t in range(3):
        x = np.zeros((n, 2), dtype=np.uint64)
        x[:, 0] = oracle.chacha_fp_rows(seed, t, 1, n)[0]
        out.append(x)
    out[2][:, 1] = oracle.chacha_fp_rows(seed, 7, 1, n)[0]
    return out


@pytest.mark.parametrize("log2n,G", [(1, 2), (5, 2), (8, 4), (10, 8)])
def test_triple_finish(oracle, log2n, G):
    n = 1 << log2n
    a, b, c = tables(oracle, n)
    seed = bytes([0x5A] * 32)
    parts = []
    for g in range(G):
        sl = slice(g * n // G, (g + 1) * n // G)
        parts.append(em.triple_local(oracle, a[sl], b[sl], c[sl], seed))
    msgs, finals = sh.triple_finish([np.concatenate(p) for p in parts], n, seed)
    em_msgs, em_finals = oracle.triple_sumcheck(a, b, c, seed)
    assert np.array_equal(msgs, em_msgs)
    assert np.array_equal(finals, em_finals)


def lookup_case(log2f, log2t, seed):
    rng = np.random.default_rng(seed)
    table = rng.integers(-32768, 32768, size=1 << log2t, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, 1 << log2t, size=1 << log2f)
    return table[idx], table, np.bincount(idx, minlength=1 << log2t).astype(np.uint32)


@pytest.mark.parametrize("log2f,log2t,G", [(2, 2, 2), (6, 4, 2), (9, 5, 4), (10, 4, 8)])
def test_logup_finish(oracle, log2f, log2t, G):
    f, table, mult = lookup_case(log2f, log2t, log2f * 10 + G)
    seed, domain = bytes([0x4C] * 32), 0x1004
    nf, nt = 1 << log2f, 1 << log2t
    fe, te = em.embed_i16(f), em.embed_i16(table)
    s = G.bit_length() - 1
    parts = []
    for g in range(G):
        w, _ = em.logup_local(oracle, fe[g * nf // G:(g + 1) * nf // G], te[g * nt // G:(g + 1) * nt // G],
                              mult[g * nt // G:(g + 1) * nt // G], s, seed, domain)
        parts.append(w)
    got = sh.logup_finish(parts, nf, nt, seed, domain)
    exp = oracle.logup_prove(f, table, mult, seed, domain)
    assert got.shape == exp.shape
    assert np.array_equal(got, exp)


def _rank(rank, world, port, q):
    import torch.distributed as dist

    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        gather = sh.torch_all_gather()
        f, table, mult = lookup_case(8, 4, 3)
        nf, nt = f.size, table.size
        fe, te = em.embed_i16(f), em.embed_i16(table)
        seed, domain = bytes([0x4C] * 32), 0x1004
        w, _ = em.logup_local(oracle, fe[rank * nf // world:(rank + 1) * nf // world],
                              te[rank * nt // world:(rank + 1) * nt // world],
                              mult[rank * nt // world:(rank + 1) * nt // world], world.bit_length() - 1, seed,
                              domain)
        proof = sh.logup_finish(gather(w), nf, nt, seed, domain)
        ok = np.array_equal(proof, oracle.logup_prove(f, table, mult, seed, domain))
        a, b, c = tables(oracle, 64)
        sl = slice(rank * 64 // world, (rank + 1) * 64 // world)
        m, fin = em.triple_local(oracle, a[sl], b[sl], c[sl], bytes([0x5A] * 32))
        parts = gather(np.concatenate([m, fin]))
        msgs, _ = sh.triple_finish(parts, 64, bytes([0x5A] * 32))
        em_msgs, _ = oracle.triple_sumcheck(a, b, c, bytes([0x5A] * 32))
        ok = ok and np.array_equal(msgs, em_msgs)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


class _EmuProver:
    """Stand-in for accel.Prover inside ShardedProver: each shard's local work
    by the oracle emulation, on arrays registered under integer ids."""

    def __init__(self, oracle, store):
        import types

        self.o, self.store = oracle, store
        self.backend = types.SimpleNamespace(wait_uploads=lambda: None)

    def triple_sumcheck(self, a, b, c, n, seed):
        return em.triple_local(self.o, self.store[a], self.store[b], self.store[c], seed)

    def logup_local(self, f, nf, t, nt, mult, s, seed, domain):
        w, _ = em.logup_local(self.o, self.store[f], self.store[t], self.store[mult], s, seed, domain)
        return w


def _rank_split(rank, world, port, q):
    """ShardedProver.prove with two lanes and the LogUp gather on a second
    communicator: the LogUp lane gathers and finishes while the triple lane
    still works, over gloo, twice in a row."""
    import torch.distributed as dist

    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        second = dist.new_group(backend="gloo")
        f, table, mult = lookup_case(8, 4, 5)
        nf, nt, n = f.size, table.size, 64
        fe, te = em.embed_i16(f), em.embed_i16(table)
        a, b, c = tables(oracle, n)
        sl = lambda x, m: x[rank * m // world:(rank + 1) * m // world]  # noqa: E731
        store = {1: sl(a, n), 2: sl(b, n), 3: sl(c, n), 4: sl(fe, nf), 5: sl(te, nt), 6: sl(mult, nt)}
        sp = sh.ShardedProver(_EmuProver(oracle, store), rank, world, sh.torch_all_gather(),
                              logup_prover=_EmuProver(oracle, store),
                              logup_gather=sh.torch_all_gather(group=second))
        tseed, lseed, domain = bytes([0x5A] * 32), bytes([0x4C] * 32), 0x1004
        em_msgs, em_finals = oracle.triple_sumcheck(a, b, c, tseed)
        em_proof = oracle.logup_prove(f, table, mult, lseed, domain)
        ok = True
        for _ in range(2):
            msgs, finals, proof = sp.prove(1, 2, 3, n, tseed, 4, nf, 5, nt, 6, lseed, domain)
            ok = ok and np.array_equal(msgs, em_msgs) and np.array_equal(finals, em_finals)
            ok = ok and np.array_equal(proof, em_proof)
        q.put((rank, ok))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_split_gathers():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_split, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)


def test_concurrently_lane_semantics():
    """sh.concurrently: both results in order, the second function on one
    persistent lane thread, its error re-raised, and the lane finishes its
    work even when the first function raises."""
    import threading
    import time

    main = threading.get_ident()
    a, b = sh.concurrently(lambda: 1, lambda: threading.get_ident())
    assert a == 1 and b != main
    _, b2 = sh.concurrently(lambda: 2, lambda: threading.get_ident())
    assert b2 == b  # the same lane thread serves every call

    with pytest.raises(ValueError, match="lane"):
        sh.concurrently(lambda: 3, lambda: (_ for _ in ()).throw(ValueError("lane")))

    done = []

    def slow():
        time.sleep(0.05)
        done.append(True)
        return 4

    with pytest.raises(KeyError):
        sh.concurrently(lambda: {}["missing"], slow)
    assert done == [True]  # the lane's work completed before the error surfaced
    assert sh.concurrently(lambda: 5, lambda: 6) == (5, 6)


# ---- VOLE-MAC epilogue rows split over shards ----------------------------------

class _EmuBackend:
    """The two device calls of sh.auth_gemm_rows_shard, by the oracle, on
    byte buffers registered under integer ids (element offsets as the C ABI)."""

    def __init__(self, oracle):
        self.o, self.store, self.next = oracle, {}, 1

    def alloc(self, nbytes):
        self.store[self.next] = np.zeros(nbytes, dtype=np.uint8)
        self.next += 1
        return self.next - 1

    def free(self, buf):
        del self.store[buf]

    def upload_new(self, a):
        buf = self.alloc(a.nbytes)
        self.store[buf][:] = np.ascontiguousarray(a).view(np.uint8).reshape(-1)
        return buf

    def view(self, buf, dtype):
        return self.store[buf].view(dtype)

    def call(self, name, *args):
        if name == "mock_correlation_sub_masks_device":
            out, off_bytes, seed, base, rows, cols = args
            rows_ = self.o.chacha_fp_rows(seed, base, rows, cols).reshape(-1)
            self.view(out, np.uint64)[off_bytes // 8:off_bytes // 8 + rows * cols] = rows_
        elif name == "gemm_requant_auth_device":
            a, ao, b, bo, mk, mo, out, oo, corr, co, m, k, n, shift = args
            av = self.view(a, np.int16)[ao:ao + m * k]
            bv = self.view(b, np.int16)[bo:bo + k * n]
            y, c = self.o.gemm_requant_auth(av, bv, self.view(mk, np.uint64)[mo:mo + m * n], m, k, n, shift)
            self.view(out, np.int16)[oo:oo + m * n] = y
            self.view(corr, np.uint64)[co:co + m * n] = c
        else:
            raise AssertionError(name)


@pytest.mark.parametrize("m,world", [(1, 1), (7, 2), (12, 4), (5, 8), (1024, 3)])
def test_row_blocks_partition_the_rows(m, world):
    blocks = [sh.row_block(m, g, world) for g in range(world)]
    assert blocks[0][0] == 0 and sum(r for _, r in blocks) == m
    assert all(blocks[g][0] + blocks[g][1] == blocks[g + 1][0] for g in range(world - 1))
    assert max(r for _, r in blocks) - min(r for _, r in blocks) <= 1
    with pytest.raises(Exception):
        sh.row_block(m, world, world)


def _auth_case(rng, m, k, n):
    a = rng.integers(-600, 600, size=m * k).astype(np.int16)
    b = rng.integers(-600, 600, size=k * n).astype(np.int16)
    return a, b


@pytest.mark.parametrize("m,world", [(9, 2), (10, 3), (3, 4)])
def test_auth_rows_shards_concatenate_to_the_whole(oracle, m, world):
    k, n, shift, tag, seed = 40, 24, 6, 0x33, bytes([0x4D] * 32)
    a, b = _auth_case(np.random.default_rng(m), m, k, n)
    whole_y, whole_c = oracle.gemm_requant_auth(a, b, oracle.chacha_fp_rows(seed, tag << 32, m, n).reshape(-1),
                                                m, k, n, shift)
    be = _EmuBackend(oracle)
    ai, bi = be.upload_new(a), be.upload_new(b)
    ys, cs = [], []
    for g in range(world):
        row0, rows, out, corr = sh.auth_gemm_rows_shard(be, g, world, ai, bi, m, k, n, shift, seed, tag)
        if rows:
            ys.append(be.view(out, np.int16)[:rows * n].copy())
            cs.append(be.view(corr, np.uint64)[:rows * n].copy())
            be.free(out)
            be.free(corr)
    assert np.array_equal(np.concatenate(ys), whole_y) and np.array_equal(np.concatenate(cs), whole_c)
    assert set(be.store) == {ai, bi}  # the shard freed its masks


def _rank_auth(rank, world, port, q):
    """Each gloo rank authenticates its row block; one all-gather of the
    (padded) blocks rebuilds the single-process output and corrections."""
    import torch.distributed as dist

    from oracle import oracle

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=60))
    try:
        m, k, n, shift, tag, seed = 11, 32, 16, 5, 0x21, bytes([0x4D] * 32)
        a, b = _auth_case(np.random.default_rng(4), m, k, n)
        be = _EmuBackend(oracle)
        ai, bi = be.upload_new(a), be.upload_new(b)
        row0, rows, out, corr = sh.auth_gemm_rows_shard(be, rank, world, ai, bi, m, k, n, shift, seed, tag)
        cap = -(-m // world)
        mine = np.zeros((cap, n, 2), dtype=np.uint64)
        mine[:rows, :, 0] = be.view(out, np.int16)[:rows * n].astype(np.int64).view(np.uint64).reshape(rows, n)
        mine[:rows, :, 1] = be.view(corr, np.uint64)[:rows * n].reshape(rows, n)
        parts = sh.torch_all_gather()(mine)
        got = np.concatenate([parts[g][:sh.row_block(m, g, world)[1]] for g in range(world)])
        y, c = oracle.gemm_requant_auth(a, b, oracle.chacha_fp_rows(seed, tag << 32, m, n).reshape(-1), m, k, n,
                                        shift)
        ok = np.array_equal(got[:, :, 0].view(np.int64).reshape(-1), y.astype(np.int64))
        q.put((rank, bool(ok and np.array_equal(got[:, :, 1].reshape(-1), c))))
    finally:
        dist.destroy_process_group()


def test_two_gloo_ranks_auth_rows():
    import torch.multiprocessing as mp

    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_auth, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    results = dict(q.get(timeout=5) for _ in range(2))
    assert results == {0: True, 1: True}
    assert all(p.exitcode == 0 for p in procs)
