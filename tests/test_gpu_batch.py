"""Cross-layer LogUp round batches (volta_b200_logup_round_batch_device)
against the oracle's fold and round functions: every job of a batch must
equal its single-layer call (round on interleaved children, fold + round on
interleaved children, fold + round, fold only), whatever else shares the
launch."""

import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


class RoundJob(C.Structure):
    """include/volta_b200_ext.h: vzb_round_job."""

    _fields_ = [("kind", C.c_uint32), ("flags", C.c_uint32), ("in_id", C.c_uint64 * 4),
                ("in_offset", C.c_size_t * 4), ("len", C.c_size_t), ("r", C.c_uint64 * 2),
                ("out_id", C.c_uint64 * 4), ("out_offset", C.c_size_t * 4), ("s_id", C.c_uint64),
                ("s_offset", C.c_size_t), ("msg_id", C.c_uint64), ("msg_offset", C.c_size_t),
                ("q_alpha", C.c_uint64 * 2)]


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=1)
    yield b
    b.close()


def rand_fp2(rng, n):
    return rng.integers(0, P, size=(n, 2), dtype=np.uint64)


def run_batch(be, jobs):
    arr = (RoundJob * len(jobs))(*jobs)
    return be.lib.volta_b200_logup_round_batch_device(be.ctx, C.cast(arr, C.c_void_p), len(jobs))


class Case:
    """One job with its inputs, outputs and the oracle's expectation."""

    def __init__(self, be, oracle, rng, kind, length, msg_id, msg_slot, p_one=False):
        self.kind, self.length, self.p_one = kind, length, p_one
        il = kind <= 1
        fold = kind != 0
        self.r = tuple(int(x) for x in rand_fp2(rng, 1)[0])
        pairs = length // 4 if fold else length // 2
        s_off = int(rng.integers(0, 5))
        self.suffix = rand_fp2(rng, s_off + pairs)
        self.ids = []
        job = RoundJob()
        job.kind, job.len = kind, length
        job.flags = 1 if p_one else 0
        job.r[0], job.r[1] = self.r
        ones = lambda n: np.tile(np.array([[1, 0]], dtype=np.uint64), (n, 1))  # noqa: E731
        if il:
            child_off = int(rng.integers(0, 3))
            self.P = ones(child_off + 2 * length) if p_one else rand_fp2(rng, child_off + 2 * length)
            self.Q = rand_fp2(rng, child_off + 2 * length)
            # with all-one numerators P is not read: no buffer is passed
            job.in_id[0] = 0 if p_one else be.upload_new(self.P)
            job.in_id[1] = be.upload_new(self.Q)
            job.in_offset[0] = child_off
            self.ids += [x for x in (job.in_id[0], job.in_id[1]) if x]
            ch_p, ch_q = self.P[child_off:], self.Q[child_off:]
            # deinterleaved p0, p1, q0, q1
            v = [np.ascontiguousarray(x) for x in (ch_p[0::2], ch_p[1::2], ch_q[0::2], ch_q[1::2])]
        else:
            v = [ones(length) if (p_one and k < 2) else rand_fp2(rng, length) for k in range(4)]
            for k in range(4):
                if p_one and k < 2:
                    continue
                off = int(rng.integers(0, 3))
                job.in_id[k] = be.upload_new(np.concatenate([rand_fp2(rng, off), v[k]]))
                job.in_offset[k] = off
                self.ids.append(job.in_id[k])
        if fold:
            self.folded = [oracle.fold_rows(x, 1, length, self.r) for x in v]
            self.out_off = []
            for k in range(4):
                off = int(rng.integers(0, 3))
                self.out_off.append(off)
                if p_one and k < 2 and kind != 3:  # numerator outputs are not written
                    continue
                job.out_id[k] = be.alloc(16 * (off + length // 2))
                job.out_offset[k] = off
                self.ids.append(job.out_id[k])
            after = self.folded
        else:
            after = v
        self.expect_msg = None
        if kind != 3:
            job.s_id = be.upload_new(self.suffix)
            job.s_offset = s_off
            self.ids.append(job.s_id)
            job.msg_id, job.msg_offset = msg_id, 4 * msg_slot
            self.expect_msg = oracle.logup_general_round(*after, self.suffix[s_off:], pairs)
        self.job, self.msg_slot = job, msg_slot

    def check(self, be, msgs):
        if self.kind != 0:
            for k in range(4):
                if self.p_one and k < 2 and self.kind != 3:
                    continue
                got = be.download_fp2(self.job.out_id[k], self.length // 2, offset=self.out_off[k])
                assert np.array_equal(got, self.folded[k]), (self.kind, self.length, k)
        if self.expect_msg is not None:
            assert np.array_equal(msgs[4 * self.msg_slot: 4 * self.msg_slot + 4], self.expect_msg), \
                (self.kind, self.length)

    def free(self, be):
        for i in self.ids:
            be.free(i)


@pytest.mark.parametrize("spec", [
    [(0, 2)], [(1, 4)], [(2, 4)], [(3, 4)],
    [(0, 1 << 12), (1, 1 << 14), (2, 1 << 13), (3, 1 << 12), (2, 1 << 16), (0, 8)],
    [(2, 1 << 20), (2, 4096), (1, 1 << 18), (0, 1 << 17), (3, 1 << 15)] + [(2, 64)] * 10,
], ids=["round-il", "fold-round-il", "fold-round", "fold", "mixed-6", "mixed-15"])
def test_round_batch_matches_single_layer_calls(be, oracle, spec):
    rng = np.random.default_rng(len(spec) * 1000 + spec[0][1])
    msg_id = be.alloc(16 * 4 * len(spec))
    cases = [Case(be, oracle, rng, kind, length, msg_id, j) for j, (kind, length) in enumerate(spec)]
    assert run_batch(be, [c.job for c in cases]) == 0, be.last_error()
    msgs = be.download_fp2(msg_id, 4 * len(spec))
    for c in cases:
        c.check(be, msgs)
    # repeated launches reuse the per-job counters
    assert run_batch(be, [c.job for c in cases]) == 0, be.last_error()
    assert np.array_equal(be.download_fp2(msg_id, 4 * len(spec)), msgs)
    for c in cases:
        c.free(be)
    be.free(msg_id)


@pytest.mark.parametrize("spec", [
    [(0, 2)], [(1, 4)], [(2, 4)], [(3, 4)],
    [(0, 1 << 16), (1, 1 << 15), (2, 1 << 14), (3, 1 << 12), (2, 1 << 18)],
], ids=["round-il", "fold-round-il", "fold-round", "fold", "mixed-5"])
def test_round_batch_all_one_numerators(be, oracle, spec):
    """flags = VZB_ROUND_P_ONE: the same results as on all-one numerators,
    without reading them (kind 3 writes the folded ones)."""
    rng = np.random.default_rng(len(spec) * 77 + spec[0][1])
    msg_id = be.alloc(16 * 4 * (len(spec) + 1))
    cases = [Case(be, oracle, rng, kind, length, msg_id, j, p_one=True) for j, (kind, length) in enumerate(spec)]
    # an ordinary job shares the launch
    cases.append(Case(be, oracle, rng, 2, 4096, msg_id, len(spec)))
    assert run_batch(be, [c.job for c in cases]) == 0, be.last_error()
    msgs = be.download_fp2(msg_id, 4 * (len(spec) + 1))
    for c in cases:
        c.check(be, msgs)
    for c in cases:
        c.free(be)
    be.free(msg_id)


def test_round_batch_rejects_bad_jobs(be):
    ids = [be.alloc(16 * 64) for _ in range(10)]
    job = RoundJob()
    job.kind, job.len = 2, 16
    for k in range(4):
        job.in_id[k], job.out_id[k] = ids[k], ids[4 + k]
    job.s_id, job.msg_id = ids[8], ids[9]
    assert run_batch(be, [job]) == 0, be.last_error()
    bad = RoundJob.from_buffer_copy(job)
    bad.kind = 4
    assert run_batch(be, [bad]) == -1 and "kind" in be.last_error()
    bad = RoundJob.from_buffer_copy(job)
    bad.flags = 8  # no such flag
    assert run_batch(be, [bad]) == -1 and "flags" in be.last_error()
    bad = RoundJob.from_buffer_copy(job)
    bad.len = 6
    assert run_batch(be, [bad]) == -1 and "length" in be.last_error()
    bad = RoundJob.from_buffer_copy(job)
    bad.len = 256  # beyond the buffers
    assert run_batch(be, [bad]) == -1
    bad = RoundJob.from_buffer_copy(job)
    bad.r[0] = P
    assert run_batch(be, [bad]) == -1 and "canonical" in be.last_error()
    assert run_batch(be, [job] * 25) == -1 and "24" in be.last_error()
    assert run_batch(be, []) == -1
    # the context stays usable
    assert run_batch(be, [job]) == 0, be.last_error()
    for i in ids:
        be.free(i)


class SuffixJob(C.Structure):
    """include/volta_b200_ext.h: vzb_suffix_job."""

    _fields_ = [("points_id", C.c_uint64), ("points_offset", C.c_size_t), ("point_len", C.c_size_t),
                ("out_id", C.c_uint64), ("out_offset", C.c_size_t)]


def test_suffix_eq_batch_matches_single_layer_calls(be):
    """Every job of one batch equals volta_cuda_logup_suffix_eq_device on the
    same point (tables of 1 to 2^23 entries, two outer-product bands)."""
    lens = [1, 5, 11, 12, 13, 16, 23, 24]
    rng = np.random.default_rng(11)
    pts = rand_fp2(rng, 3 + sum(lens))
    pid = be.upload_new(pts)
    jobs, singles, off = [], [], 3
    for L in lens:
        total = (1 << L) - 1
        out_off = int(rng.integers(0, 4))
        batch_out, single_out = be.alloc(16 * (out_off + total)), be.alloc(16 * total)
        jobs.append(SuffixJob(pid, off, L, batch_out, out_off))
        be.call("logup_suffix_eq_device", pid, off, L, single_out, 0)
        singles.append((batch_out, out_off, single_out, total))
        off += L
    arr = (SuffixJob * len(jobs))(*jobs)
    assert be.lib.volta_b200_logup_suffix_eq_batch_device(be.ctx, C.cast(arr, C.c_void_p), len(jobs)) == 0, \
        be.last_error()
    for batch_out, out_off, single_out, total in singles:
        assert np.array_equal(be.download_fp2(batch_out, total, offset=out_off), be.download_fp2(single_out, total))
        be.free(batch_out)
        be.free(single_out)
    # a job beyond its output buffer is rejected and the context stays usable
    small = be.alloc(16 * 7)
    bad = (SuffixJob * 1)(SuffixJob(pid, 3, 4, small, 0))
    assert be.lib.volta_b200_logup_suffix_eq_batch_device(be.ctx, C.cast(bad, C.c_void_p), 1) == -1
    ok = (SuffixJob * 1)(SuffixJob(pid, 3, 3, small, 0))
    assert be.lib.volta_b200_logup_suffix_eq_batch_device(be.ctx, C.cast(ok, C.c_void_p), 1) == 0, be.last_error()
    be.free(small)
    be.free(pid)


@pytest.mark.parametrize("kind,length", [(0, 2), (1, 4), (0, 1 << 16), (1, 1 << 15), (1, 1 << 18)])
def test_round_batch_leaf_children_from_column(be, oracle, kind, length):
    """VZB_ROUND_Q_COLUMN: children j = (p = 1, q = (a0 - f_j, a1)) read from a
    query column equal the same job on materialised leaves."""
    rng = np.random.default_rng(kind * 100 + length)
    a0, a1 = (int(x) for x in rng.integers(0, P, size=2, dtype=np.uint64))
    off = 3
    f = rng.integers(0, P, size=off + 2 * length, dtype=np.uint64)
    # leaves on the host: q_j = (a0 - f_j mod p, a1)
    qc0 = np.array([(a0 - int(v)) % P for v in f[off:]], dtype=np.uint64)
    Q = np.stack([qc0, np.full_like(qc0, a1)], axis=1)
    v = [np.tile(np.array([[1, 0]], dtype=np.uint64), (length, 1)) for _ in range(2)]
    v += [np.ascontiguousarray(Q[0::2]), np.ascontiguousarray(Q[1::2])]
    r = tuple(int(t) for t in rand_fp2(rng, 1)[0])
    pairs = length // 4 if kind == 1 else length // 2
    suffix = rand_fp2(rng, pairs)
    fid, sid, msg = be.upload_new(f), be.upload_new(suffix), be.alloc(64)
    job = RoundJob()
    job.kind, job.len, job.flags = kind, length, 3
    job.r[0], job.r[1] = r
    job.q_alpha[0], job.q_alpha[1] = a0, a1
    job.in_id[1], job.in_offset[0] = fid, off
    job.s_id, job.msg_id = sid, msg
    outs = []
    if kind == 1:
        for k in (2, 3):
            job.out_id[k] = be.alloc(16 * (length // 2))
            outs.append(job.out_id[k])
    assert run_batch(be, [job]) == 0, be.last_error()
    after = [oracle.fold_rows(t, 1, length, r) for t in v] if kind == 1 else v
    assert np.array_equal(be.download_fp2(msg, 4), oracle.logup_general_round(*after, suffix, pairs))
    if kind == 1:
        for k, o in zip((2, 3), outs):
            assert np.array_equal(be.download_fp2(o, length // 2), after[k])
    # the flag needs all-one numerators and kind 0 or 1
    bad = RoundJob.from_buffer_copy(job)
    bad.flags = 2
    assert run_batch(be, [bad]) == -1 and "numerators" in be.last_error()
    for t in [fid, sid, msg] + outs:
        be.free(t)


def _fp2_mul(x, y):
    return ((x[0] * y[0] + 7 * x[1] * y[1]) % P, (x[0] * y[1] + x[1] * y[0]) % P)


@pytest.mark.parametrize("length", [2, 64, 1 << 12])
def test_round_batch_parents_shortcut(be, oracle, length):
    """VZB_ROUND_PARENTS: round 0 with the parent level given equals round 0
    computed from the children alone."""
    rng = np.random.default_rng(length + 5)
    P_ = rand_fp2(rng, 2 * length)
    Q_ = rand_fp2(rng, 2 * length)
    par_p, par_q = np.zeros((length, 2), dtype=np.uint64), np.zeros((length, 2), dtype=np.uint64)
    for j in range(length):  # parent j of children (2j, 2j + 1): p = pa qb + pb qa, q = qa qb
        pa, pb = tuple(int(t) for t in P_[2 * j]), tuple(int(t) for t in P_[2 * j + 1])
        qa, qb = tuple(int(t) for t in Q_[2 * j]), tuple(int(t) for t in Q_[2 * j + 1])
        x, y = _fp2_mul(pa, qb), _fp2_mul(pb, qa)
        par_p[j] = ((x[0] + y[0]) % P, (x[1] + y[1]) % P)
        par_q[j] = _fp2_mul(qa, qb)
    off = 2
    suffix = rand_fp2(rng, length // 2)
    ids = [be.upload_new(P_), be.upload_new(Q_), be.upload_new(np.concatenate([rand_fp2(rng, off), par_p])),
           be.upload_new(np.concatenate([rand_fp2(rng, off), par_q])), be.upload_new(suffix), be.alloc(16 * 8)]
    plain = RoundJob()
    plain.kind, plain.len = 0, length
    plain.in_id[0], plain.in_id[1] = ids[0], ids[1]
    plain.s_id, plain.msg_id = ids[4], ids[5]
    par = RoundJob.from_buffer_copy(plain)
    par.flags = 4
    par.out_id[0], par.out_id[1], par.out_offset[0] = ids[2], ids[3], off
    par.msg_offset = 4
    assert run_batch(be, [plain, par]) == 0, be.last_error()
    msgs = be.download_fp2(ids[5], 8)
    assert np.array_equal(msgs[:4], msgs[4:])
    v = [np.ascontiguousarray(x) for x in (P_[0::2], P_[1::2], Q_[0::2], Q_[1::2])]
    assert np.array_equal(msgs[:4], oracle.logup_general_round(*v, suffix, length // 2))
    bad = RoundJob.from_buffer_copy(par)
    bad.flags = 5  # with all-one numerators: rejected
    assert run_batch(be, [bad]) == -1 and "parents" in be.last_error()
    for t in ids:
        be.free(t)
