"""Asynchronous uploads and the int16 embedding (include/volta_b200_ext.h):
data uploaded on the copy stream is what later kernels and downloads see
once wait_uploads has been called, and a local proof whose tables arrive
that way equals the oracle's."""

import numpy as np
import pytest

import sharded_emulation as em
from volta_zk_b200 import sharded as sh

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def prover():
    from volta_zk_b200 import accel

    p = accel.Prover(policy=1)
    yield p
    p.close()


def test_embed_i16_matches_definition(prover):
    be = prover.backend
    rng = np.random.default_rng(3)
    x = np.concatenate([np.array([-32768, -1, 0, 1, 32767], dtype=np.int16),
                        rng.integers(-32768, 32768, size=100_003, dtype=np.int64).astype(np.int16)])
    src = be.upload_new(x)
    dst = be.alloc(8 * x.size)
    be.embed_i16(src, dst, x.size)
    got = be.download(dst, 8 * x.size)
    v = x.astype(np.int64)
    exp = np.where(v >= 0, v.astype(np.uint64), np.uint64(P) - (-v).astype(np.uint64))
    assert np.array_equal(got, exp)
    # beyond the buffers: rejected, and the context stays usable
    assert be.lib.volta_b200_embed_i16_device(be.ctx, src, 0, dst, 0, x.size + 1) == -1
    be.embed_i16(src, dst, 5)
    be.free(src)
    be.free(dst)


def test_upload_async_then_wait(prover):
    import torch

    be = prover.backend
    rng = np.random.default_rng(4)
    data = rng.integers(0, 2**63, size=(1 << 22), dtype=np.int64)
    host = torch.from_numpy(data).pin_memory()
    buf = be.alloc(8 * data.size + 64)
    be.upload_async(buf, host.data_ptr(), 8 * data.size, 64)
    be.wait_uploads()
    got = be.download(buf, 8 * data.size, offset_bytes=64)
    assert np.array_equal(got.view(np.int64), data)
    assert be.lib.volta_b200_upload_async(be.ctx, buf, 65, host.data_ptr(), 8 * data.size) == -1  # beyond
    be.wait_uploads()
    be.free(buf)


def test_proof_local_waits_for_async_tables(prover, oracle):
    """The triple columns are still in flight on the copy stream when the
    local call starts; its triple part waits for them."""
    import torch

    n, nf, nt = 1 << 16, 1 << 14, 1 << 10
    rng = np.random.default_rng(9)
    cols = [rng.integers(0, P, size=n, dtype=np.uint64) for _ in range(3)]
    lifted = [np.stack([x, np.zeros_like(x)], axis=1) for x in cols]
    table = rng.integers(-32768, 32768, size=nt, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    f = table[idx]
    mult = np.bincount(idx, minlength=nt).astype(np.uint32)
    be = prover.backend
    f16, t16 = be.upload_new(f), be.upload_new(table)
    fe, te = be.alloc(8 * nf), be.alloc(8 * nt)
    be.embed_i16(f16, fe, nf)
    be.embed_i16(t16, te, nt)
    m = be.upload_new(mult)
    pinned = [torch.from_numpy(x.view(np.int64)).pin_memory() for x in cols]
    ids = [be.alloc(8 * n) for _ in range(3)]
    for buf, t in zip(ids, pinned):
        be.upload_async(buf, t.data_ptr(), 8 * n)
    tseed, lseed, domain = bytes([0x5A] * 32), bytes([0x4C] * 32), 0x1004
    words = prover.proof_local(*ids, n, True, tseed, fe, nf, te, nt, m, 0, lseed, domain)
    k = 3 * 16 + 3
    em_msgs, em_finals = oracle.triple_sumcheck(*lifted, tseed)
    assert np.array_equal(words[: 3 * 16], em_msgs)
    assert np.array_equal(words[3 * 16:k], em_finals)
    got = sh.logup_finish([words[k:]], nf, nt, lseed, domain)
    assert np.array_equal(got, oracle.logup_prove(f, table, mult, lseed, domain))
    for x in ids + [f16, t16, fe, te, m]:
        be.free(x)


@pytest.mark.parametrize("log2n,chunk", [(10, 0), (13, 0), (16, 8192), (16, 3 * 8192), (17, 0), (18, 5000)])
def test_triple_sumcheck_from_host_columns(prover, oracle, log2n, chunk):
    """vzh_triple_sumcheck_fp_host: the columns stream in from pinned host
    memory (by chunks, each proved on chip once landed, from 8192 entries on;
    all at once below) and the proof is the oracle's; the device columns end
    up holding the host columns."""
    import torch

    n = 1 << log2n
    rng = np.random.default_rng(log2n + chunk)
    cols = [rng.integers(0, P, size=n, dtype=np.uint64) for _ in range(3)]
    lifted = [np.stack([x, np.zeros_like(x)], axis=1) for x in cols]
    pinned = [torch.from_numpy(x.view(np.int64)).pin_memory() for x in cols]
    be = prover.backend
    ids = [be.alloc(8 * n) for _ in range(3)]
    tseed = bytes([0x5A] * 32)
    msgs, finals = prover.triple_sumcheck_fp_host(*ids, [t.data_ptr() for t in pinned], n, tseed, chunk)
    emsgs, efinals = oracle.triple_sumcheck(*lifted, tseed)
    assert np.array_equal(msgs, emsgs)
    assert np.array_equal(finals, efinals)
    for buf, col in zip(ids, cols):
        assert np.array_equal(be.download(buf, 8 * n), col)
    for x in ids:
        be.free(x)


def test_proof_local_from_host_columns(prover, oracle):
    """vzh_proof_local_host: the LogUp part computes while the triple columns
    stream in by chunks; the words equal the oracle's proofs."""
    import torch

    n, nf, nt = 1 << 16, 1 << 14, 1 << 10
    rng = np.random.default_rng(19)
    cols = [rng.integers(0, P, size=n, dtype=np.uint64) for _ in range(3)]
    lifted = [np.stack([x, np.zeros_like(x)], axis=1) for x in cols]
    table = rng.integers(-32768, 32768, size=nt, dtype=np.int64).astype(np.int16)
    idx = rng.integers(0, nt, size=nf)
    f = table[idx]
    mult = np.bincount(idx, minlength=nt).astype(np.uint32)
    be = prover.backend
    f16, t16 = be.upload_new(f), be.upload_new(table)
    fe, te = be.alloc(8 * nf), be.alloc(8 * nt)
    be.embed_i16(f16, fe, nf)
    be.embed_i16(t16, te, nt)
    m = be.upload_new(mult)
    pinned = [torch.from_numpy(x.view(np.int64)).pin_memory() for x in cols]
    ids = [be.alloc(8 * n) for _ in range(3)]
    tseed, lseed, domain = bytes([0x5A] * 32), bytes([0x4C] * 32), 0x1004
    words = prover.proof_local(*ids, n, True, tseed, fe, nf, te, nt, m, 0, lseed, domain,
                               host=[t.data_ptr() for t in pinned], chunk=2 * 8192)
    k = 3 * 16 + 3
    em_msgs, em_finals = oracle.triple_sumcheck(*lifted, tseed)
    assert np.array_equal(words[: 3 * 16], em_msgs)
    assert np.array_equal(words[3 * 16:k], em_finals)
    got = sh.logup_finish([words[k:]], nf, nt, lseed, domain)
    assert np.array_equal(got, oracle.logup_prove(f, table, mult, lseed, domain))
    for x in ids + [f16, t16, fe, te, m]:
        be.free(x)


def test_two_contexts_concurrently(prover, oracle):
    """The triple sumcheck on one context and the LogUp proof on another,
    driven from two host threads at once (bench.py's two lanes), give the
    oracle's proofs; repeated to let the launches interleave."""
    from volta_zk_b200 import accel

    other = accel.Prover(policy=1)
    try:
        n, nf, nt = 1 << 16, 1 << 15, 1 << 10
        rng = np.random.default_rng(21)
        cols = [rng.integers(0, P, size=n, dtype=np.uint64) for _ in range(3)]
        lifted = [np.stack([x, np.zeros_like(x)], axis=1) for x in cols]
        table = rng.integers(-32768, 32768, size=nt, dtype=np.int64).astype(np.int16)
        idx = rng.integers(0, nt, size=nf)
        f = table[idx]
        mult = np.bincount(idx, minlength=nt).astype(np.uint32)
        tseed, lseed, domain = bytes([0x5A] * 32), bytes([0x4C] * 32), 0x1004
        ids = [prover.backend.upload_new(x) for x in cols]
        be_b = other.backend
        lids = [be_b.upload_new(em.embed_i16(f)), be_b.upload_new(em.embed_i16(table)), be_b.upload_new(mult)]
        em_msgs, em_finals = oracle.triple_sumcheck(*lifted, tseed)
        em_proof = oracle.logup_prove(f, table, mult, lseed, domain)
        cap = oracle.logup_prove_words(nf, nt)
        for _ in range(3):
            (msgs, finals), proof = sh.concurrently(
                lambda: prover.triple_sumcheck_fp(*ids, n, tseed),
                lambda: other.logup_prove(lids[0], nf, lids[1], nt, lids[2], lseed, domain, cap))
            assert np.array_equal(msgs, em_msgs) and np.array_equal(finals, em_finals)
            assert np.array_equal(proof, em_proof)
        for i in ids:
            prover.backend.free(i)
        for i in lids:
            be_b.free(i)
    finally:
        other.close()


def test_resident_arena_best_fit_reuse_and_trim():
    """The arena's free list: a request reuses the smallest free buffer that
    fits (the lowest slot among equal capacities), a stale id is rejected,
    and a trim releases every free buffer (later requests allocate anew)."""
    from volta_zk_b200 import accel

    be = accel.CudaBackend(policy=0)
    try:
        s0 = be.stats()
        sizes = [4096, 1 << 20, 65536, 65536, 1 << 16 | 16]
        ids = [be.alloc(n) for n in sizes]
        slot = lambda i: i & 0xFFFFFFFF
        for i in ids:
            be.free(i)
        s1 = be.stats()
        assert s1.allocation_calls - s0.allocation_calls == len(sizes)
        a = be.alloc(60000)  # best fit: a 65536 buffer, the lower slot of the two
        assert slot(a) == min(slot(ids[2]), slot(ids[3]))
        b = be.alloc(65536)  # the other 65536 buffer
        assert slot(b) == max(slot(ids[2]), slot(ids[3]))
        c = be.alloc(65540)  # 65552 fits before 1 MiB
        assert slot(c) == slot(ids[4])
        d = be.alloc(100)  # the 4 KiB buffer
        assert slot(d) == slot(ids[0])
        s2 = be.stats()
        assert s2.resident_reuse_hits - s1.resident_reuse_hits == 4
        assert s2.allocation_calls == s1.allocation_calls
        with pytest.raises(accel.AccelError):
            be.free(ids[0])  # stale generation
        x = be.upload_new(np.arange(8192, dtype=np.uint64))  # the 1 MiB buffer (64 KiB requested)
        assert np.array_equal(be.download(x, 8 * 8192), np.arange(8192, dtype=np.uint64))
        for i in (a, b, c, d, x):
            be.free(i)
        be.call("trim_resident_cache")
        s3 = be.stats()
        assert s3.physical_free_calls - s2.physical_free_calls == len(sizes)
        y = be.alloc(4096)  # nothing free with memory: a fresh allocation in a trimmed slot
        assert be.stats().allocation_calls == s3.allocation_calls + 1
        assert slot(y) in {slot(i) for i in ids}
        be.free(y)
    finally:
        be.close()
