"""Parity of the sumcheck engine entry points with the CPU oracle.

Every test calls the C ABI of libvolta_cuda_backend.so (the drop-in for the
reference seam) and compares bit for bit with oracle/ (the restatement of
the reference's Rust CPU path).  Sizes cover single pairs, odd pair counts,
block-boundary and multi-block grids.
"""

import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=0)
    yield b
    b.close()


def rand_fp2(rng, n):
    return rng.integers(0, P, size=(n, 2), dtype=np.uint64)


def rand_fp(rng, n):
    return rng.integers(0, P, size=n, dtype=np.uint64)


def fp2c(v):
    from volta_zk_b200 import accel

    return accel.fp2(v)


def host_out(n):
    return np.zeros((n, 2), dtype=np.uint64)


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


PAIRS = [1, 2, 3, 255, 256, 257, 1000, (1 << 16) + 7, 1 << 18]


@pytest.mark.parametrize("pairs", PAIRS)
def test_triple_product_round(be, oracle, pairs):
    rng = np.random.default_rng(pairs)
    a, b, c = (rand_fp2(rng, 2 * pairs) for _ in range(3))
    ids = [be.upload_new(x) for x in (a, b, c)]
    out = host_out(3)
    be.call("fp2_triple_product_round_device", ids[0], 0, ids[1], 0, ids[2], 0, pairs, ptr(out))
    exp = oracle.triple_product_round(a, b, c, pairs)
    assert np.array_equal(out, exp)
    mbox = be.alloc(3 * 16)
    be.call("fp2_triple_product_round_into_device", ids[0], 0, ids[1], 0, ids[2], 0, pairs, mbox, 0)
    assert np.array_equal(be.download_fp2(mbox, 3), exp)
    for i in ids + [mbox]:
        be.free(i)


@pytest.mark.parametrize("pairs", [1, 3, 256, 4097, 1 << 17])
def test_product_round_and_scaled(be, oracle, pairs):
    rng = np.random.default_rng(7 + pairs)
    a, b = rand_fp2(rng, 2 * pairs), rand_fp2(rng, 2 * pairs)
    ia, ib = be.upload_new(a), be.upload_new(b)
    exp = oracle.product_round(a, b, pairs)
    out = host_out(2)
    be.call("fp2_product_round_device", ia, 0, ib, 0, pairs, ptr(out))
    assert np.array_equal(out, exp)
    mbox = be.alloc(32)
    be.call("fp2_product_round_into_device", ia, 0, ib, 0, pairs, mbox, 0)
    assert np.array_equal(be.download_fp2(mbox, 2), exp)
    scale = tuple(int(x) for x in rand_fp2(rng, 1)[0])
    be.call("fp2_product_round_scaled_into_device", ia, 0, ib, 0, pairs, fp2c(scale), mbox, 0)
    got = be.download_fp2(mbox, 2)
    for k in range(2):
        assert tuple(int(x) for x in got[k]) == oracle.fp2_mul(tuple(int(x) for x in exp[k]), scale)
    for i in (ia, ib, mbox):
        be.free(i)


@pytest.mark.parametrize("pairs", [1, 2, 255, 1000, (1 << 15) + 1, 1 << 19])
def test_logup_general_round(be, oracle, pairs):
    rng = np.random.default_rng(100 + pairs)
    v = [rand_fp2(rng, 2 * pairs) for _ in range(4)]
    s = rand_fp2(rng, pairs)
    ids = [be.upload_new(x) for x in v]
    sid = be.upload_new(s)
    exp = oracle.logup_general_round(*v, s, pairs)
    out = host_out(4)
    be.call("logup_general_round_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, sid, 0, pairs, ptr(out))
    assert np.array_equal(out, exp)
    mbox = be.alloc(64)
    be.call("logup_general_round_into_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, sid, 0, pairs,
            mbox, 0)
    assert np.array_equal(be.download_fp2(mbox, 4), exp)
    if pairs <= 4096:  # staged (hybrid) variant: host buffers in, message out
        out2 = host_out(4)
        rc = be.lib.volta_cuda_logup_general_round(be.ctx, ptr(v[0]), ptr(v[1]), ptr(v[2]), ptr(v[3]), ptr(s),
                                                   pairs, ptr(out2))
        assert rc == 0, be.last_error()
        assert np.array_equal(out2, exp)
    for i in ids + [sid, mbox]:
        be.free(i)


@pytest.mark.parametrize("rows,length", [(1, 2), (1, 4096), (3, 10), (5, 1 << 14), (1, 1 << 21)])
def test_fold_rows(be, oracle, rows, length):
    rng = np.random.default_rng(rows * length)
    x = rand_fp2(rng, rows * length)
    r = tuple(int(v) for v in rand_fp2(rng, 1)[0])
    ix = be.upload_new(x)
    out = be.alloc(rows * (length // 2) * 16)
    be.call("fp2_fold_rows_device", ix, 0, rows, length, fp2c(r), out, 0)
    assert np.array_equal(be.download_fp2(out, rows * (length // 2)), oracle.fold_rows(x, rows, length, r))
    be.free(ix)
    be.free(out)


@pytest.mark.parametrize("pairs", [1, 7, 4096, 100003])
def test_logup_fold4_and_deinterleave(be, oracle, pairs):
    rng = np.random.default_rng(pairs + 5)
    v = [rand_fp2(rng, 2 * pairs) for _ in range(4)]
    r = tuple(int(x) for x in rand_fp2(rng, 1)[0])
    ids = [be.upload_new(x) for x in v]
    outs = [be.alloc(16 * pairs) for _ in range(4)]
    be.call("logup_fold4_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, pairs, fp2c(r),
            outs[0], 0, outs[1], 0, outs[2], 0, outs[3], 0)
    for k in range(4):
        assert np.array_equal(be.download_fp2(outs[k], pairs), oracle.fold_rows(v[k], 1, 2 * pairs, r))
    if pairs <= 4096:
        host = [host_out(pairs) for _ in range(4)]
        rc = be.lib.volta_cuda_logup_fold4(be.ctx, ptr(v[0]), ptr(v[1]), ptr(v[2]), ptr(v[3]), pairs, fp2c(r),
                                           *[ptr(h) for h in host])
        assert rc == 0, be.last_error()
        for k in range(4):
            assert np.array_equal(host[k], oracle.fold_rows(v[k], 1, 2 * pairs, r))
    be.call("fp2_deinterleave_device", ids[0], 0, pairs, outs[0], 0, outs[1], 0)
    assert np.array_equal(be.download_fp2(outs[0], pairs), v[0][0::2])
    assert np.array_equal(be.download_fp2(outs[1], pairs), v[0][1::2])
    for i in ids + outs:
        be.free(i)


@pytest.mark.parametrize("L", [1, 2, 5, 11, 12, 13, 14, 20, 23, 24])
def test_suffix_eq(be, oracle, L):
    rng = np.random.default_rng(L)
    pts = rand_fp2(rng, L)
    ip = be.upload_new(pts)
    total = (1 << L) - 1
    out = be.alloc(16 * total)
    be.call("logup_suffix_eq_device", ip, 0, L, out, 0)
    got = be.download_fp2(out, total)
    assert np.array_equal(got, oracle.suffix_eq(pts))
    be.free(ip)
    be.free(out)


@pytest.mark.parametrize("rows,dims", [(1, 0), (3, 1), (4, 7), (2, 11), (3, 12), (2, 13), (1, 23)])
def test_eq_rows(be, oracle, rows, dims):
    rng = np.random.default_rng(rows * 31 + dims)
    pts = rand_fp2(rng, max(rows * dims, 1))
    ip = be.upload_new(pts) if dims else 0
    out = be.alloc(16 * (rows << dims))
    be.call("logup_eq_rows_device", ip, 0, rows, dims, out, 0)
    got = be.download_fp2(out, rows << dims)
    exp = oracle.eq_rows(np.ascontiguousarray(pts[: rows * dims]) if dims else pts, rows, dims)
    assert np.array_equal(got, exp)
    if ip:
        be.free(ip)
    be.free(out)


def lifted_leaves(rng, n):
    return rand_fp(rng, n)


@pytest.mark.parametrize("log2n", [1, 2, 5, 11, 12, 13, 16, 22])
@pytest.mark.parametrize("neg", [False, True])
def test_logup_tree(be, oracle, log2n, neg):
    n = 1 << log2n
    rng = np.random.default_rng(log2n * 2 + neg)
    leaf = lifted_leaves(rng, n)
    alpha1 = int(rand_fp(rng, 1)[0])
    mult = rng.integers(0, 1 << 20, size=n, dtype=np.uint32) if neg else None
    il = be.upload_new(leaf)
    im = be.upload_new(mult) if neg else 0
    ip, iq = be.alloc(16 * (n - 1)), be.alloc(16 * (n - 1))
    be.call("logup_tree_device", il, 0, im, 0, n, alpha1, int(neg), ip, 0, iq, 0)
    ep, eq = oracle.logup_tree(leaf, mult, n, alpha1, neg)
    assert np.array_equal(be.download_fp2(ip, n - 1), ep)
    assert np.array_equal(be.download_fp2(iq, n - 1), eq)
    if log2n <= 13:
        hp, hq = host_out(n - 1), host_out(n - 1)
        rc = be.lib.volta_cuda_logup_tree(be.ctx, ptr(leaf), ptr(mult) if neg else None, n, alpha1, int(neg),
                                          ptr(hp), ptr(hq))
        assert rc == 0, be.last_error()
        assert np.array_equal(hp, ep) and np.array_equal(hq, eq)
    lp, lq = be.alloc(16 * n), be.alloc(16 * n)
    be.call("logup_materialize_leaves_device", il, 0, im, 0, n, alpha1, int(neg), lp, 0, lq, 0)
    mp, mq = oracle.materialize_leaves(leaf, mult, n, alpha1, neg)
    assert np.array_equal(be.download_fp2(lp, n), mp) and np.array_equal(be.download_fp2(lq, n), mq)
    for i in (il, ip, iq, lp, lq) + ((im,) if neg else ()):
        be.free(i)


def test_logup_tree_golden_2_18(be, oracle):
    """cuda/p7_logup_tree.cu recipe on the device; published roots for 2^18."""
    n = 1 << 18
    a0, a1 = 0x123456789ABCDEF0, 0x0FEDCBA987654321
    i = np.arange(n, dtype=np.uint64)
    vals = ((i * np.uint64(37) + np.uint64(11)) & np.uint64(0xFFFF)).astype(np.uint16).view(np.int16)
    v64 = vals.astype(np.int64)
    x = np.where(v64 >= 0, v64.astype(np.uint64), np.uint64(P) - (-v64).astype(np.uint64)).astype(np.uint64)
    leaf = np.where(np.uint64(a0) >= x, np.uint64(a0) - x, np.uint64(a0) + (np.uint64(P) - x)).astype(np.uint64)
    il = be.upload_new(leaf)
    ip, iq = be.alloc(16 * (n - 1)), be.alloc(16 * (n - 1))
    be.call("logup_tree_device", il, 0, 0, 0, n, a1, 0, ip, 0, iq, 0)
    p, q = be.download_fp2(ip, n - 1), be.download_fp2(iq, n - 1)
    assert tuple(int(v) for v in p[0]) == (10980606684603994831, 1600439578519942692)
    assert tuple(int(v) for v in q[0]) == (14103360986930473702, 7831365882393612510)
    h = 0xCBF29CE484222325
    for level in range(17, -1, -1):
        off, cnt = (1 << level) - 1, 1 << level
        h = oracle.fnv_u64(np.stack([p[off:off + cnt], q[off:off + cnt]], axis=1).reshape(-1), h)
    assert h == 0xac5455f699d2b292
    for b in (il, ip, iq):
        be.free(b)


def test_logup_rounds_golden_2_16(be, oracle):
    """cuda/p7_logup_rounds.cu recipe through the resident round/fold ABI;
    published all_rounds_checksum for 2^16 (p7-gpu-logup-rounds-quick)."""
    from tests.test_oracle_golden import rounds_inputs

    log2n = 16
    cols, s, chals = rounds_inputs(log2n)
    ids = [be.upload_new(c) for c in cols]
    sid = be.upload_new(s)
    h = 0xCBF29CE484222325
    length = 1 << log2n
    for rnd in range(log2n):
        pairs = length // 2
        acc = host_out(4)
        be.call("logup_general_round_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, sid, 0, pairs, ptr(acc))
        h = oracle.fnv_u64(acc.reshape(-1), h)
        outs = [be.alloc(16 * pairs) for _ in range(4)]
        be.call("logup_fold4_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, pairs, fp2c(chals[rnd]),
                outs[0], 0, outs[1], 0, outs[2], 0, outs[3], 0)
        for k in range(4):
            h = oracle.fnv_u64(be.download_fp2(outs[k], pairs).reshape(-1), h)
            be.free(ids[k])
        ids = outs
        length = pairs
    assert h == 0x7eaefbd02661f35b
    for i in ids + [sid]:
        be.free(i)


@pytest.mark.parametrize("claims", [0, 1, 3])
@pytest.mark.parametrize("vector_len", [2, 64, 4096])
def test_aux_round(be, oracle, claims, vector_len):
    rng = np.random.default_rng(claims * 1000 + vector_len)
    column_count = 3
    q0, q1 = rand_fp2(rng, vector_len), rand_fp2(rng, vector_len)
    s = rand_fp2(rng, vector_len // 2)
    cols = rand_fp2(rng, 2 * column_count * vector_len)
    eq = rand_fp2(rng, max(claims, 1) * vector_len)
    cc = np.array([2, 0, 7][:claims] or [0], dtype=np.uint32)  # column 7 is out of range: skipped
    w = rand_fp2(rng, 2 * max(claims, 1))
    lam, cpref, point = (tuple(int(x) for x in v) for v in rand_fp2(rng, 3))
    ids = [be.upload_new(x) for x in (q0, q1, s, cols, eq, cc, w)]
    out = host_out(3)
    be.call("logup_aux_round_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, ids[4], 0, ids[5], 0,
            ids[6], 0, column_count, claims, vector_len, fp2c(lam), fp2c(cpref), fp2c(point), ptr(out))
    exp = oracle.aux_round(q0, q1, s, cols, eq, cc, w, column_count, claims, vector_len, lam, cpref, point)
    assert np.array_equal(out, exp)
    mbox = be.alloc(48)
    be.call("logup_aux_round_into_device", ids[0], 0, ids[1], 0, ids[2], 0, ids[3], 0, ids[4], 0, ids[5], 0,
            ids[6], 0, column_count, claims, vector_len, fp2c(lam), fp2c(cpref), fp2c(point), mbox, 0)
    assert np.array_equal(be.download_fp2(mbox, 3), exp)
    for i in ids + [mbox]:
        be.free(i)


@pytest.mark.parametrize("n", [1, 5, 1000, 1 << 18])
def test_dot_pair_sum_scaled(be, oracle, n):
    rng = np.random.default_rng(n + 77)
    a, b = rand_fp2(rng, n), rand_fp2(rng, n)
    ia, ib = be.upload_new(a), be.upload_new(b)
    out = host_out(1)
    be.call("fp2_dot_device", ia, 0, ib, 0, n, ptr(out))
    # dot = sum a_i b_i: the product-round g(0) of a and b interleaved with zeros
    ones = np.zeros((2 * n, 2), dtype=np.uint64)
    ones[0::2] = a
    zb = np.zeros((2 * n, 2), dtype=np.uint64)
    zb[0::2] = b
    exp = oracle.product_round(ones, zb, n)[0]
    assert np.array_equal(out[0], exp)
    scale = tuple(int(x) for x in rand_fp2(rng, 1)[0])
    mbox = be.alloc(32)
    be.call("fp2_dot_scaled_pair_into_device", ia, 0, ib, 0, n, fp2c(scale), mbox, 0)
    got = be.download_fp2(mbox, 2)
    v = oracle.fp2_mul(tuple(int(x) for x in exp), scale)
    assert tuple(int(x) for x in got[0]) == v
    assert tuple(int(x) for x in got[1]) == ((P - v[0]) % P, (P - v[1]) % P)
    pairs_in = rand_fp2(rng, 2 * n)
    ipairs = be.upload_new(pairs_in)
    out2 = host_out(2)
    be.call("fp2_pair_sum_device", ipairs, 0, n, ptr(out2))
    for k in range(2):
        part = pairs_in[k::2].astype(object)
        assert tuple(int(x) for x in out2[k]) == (int(part[:, 0].sum()) % P, int(part[:, 1].sum()) % P)
    for i in (ia, ib, mbox, ipairs):
        be.free(i)


@pytest.mark.parametrize("n_vars", [1, 4, 11, 12, 14])
def test_claim_reduce_and_link(be, oracle, n_vars):
    rng = np.random.default_rng(n_vars)
    pts = rand_fp2(rng, 2 * n_vars + 2)
    ip = be.upload_new(pts)
    length = 1 << n_vars
    out, s1, s2, s3 = (be.alloc(16 * length) for _ in range(4))
    be.call("claim_reduce_f_two_into_device", ip, 0, n_vars, out, 0, s1, 0, s2, 0, s3, 0)
    e1 = oracle.eq_rows(np.ascontiguousarray(pts[:n_vars]), 1, n_vars)
    e2 = oracle.eq_rows(np.ascontiguousarray(pts[n_vars:2 * n_vars]), 1, n_vars)
    sc1 = tuple(int(x) for x in pts[2 * n_vars])
    sc2 = tuple(int(x) for x in pts[2 * n_vars + 1])
    got = be.download_fp2(out, length)
    for i in list(range(min(length, 64))) + [length - 1]:
        t1 = oracle.fp2_mul(tuple(int(x) for x in e1[i]), sc1)
        t2 = oracle.fp2_mul(tuple(int(x) for x in e2[i]), sc2)
        assert tuple(int(x) for x in got[i]) == ((t1[0] + t2[0]) % P, (t1[1] + t2[1]) % P)
    # link accumulate: target = s * eq(point) (initialize) then += again
    lp = rand_fp2(rng, n_vars + 1)
    il = be.upload_new(lp)
    tgt = be.alloc(16 * length)
    be.call("x4d_link_eq_accumulate_device", il, 0, n_vars, tgt, 0, s1, 0, s2, 0, 1)
    be.call("x4d_link_eq_accumulate_device", il, 0, n_vars, tgt, 0, s1, 0, s2, 0, 0)
    el = oracle.eq_rows(np.ascontiguousarray(lp[:n_vars]), 1, n_vars)
    sc = tuple(int(x) for x in lp[n_vars])
    got = be.download_fp2(tgt, length)
    for i in list(range(min(length, 32))) + [length - 1]:
        t = oracle.fp2_mul(tuple(int(x) for x in el[i]), sc)
        assert tuple(int(x) for x in got[i]) == ((2 * t[0]) % P, (2 * t[1]) % P)
    for b in (ip, out, s1, s2, s3, il, tgt):
        be.free(b)


@pytest.mark.parametrize("n", [1, 2, 8, 4096, 1 << 14])
def test_mobius_and_affine_eq(be, oracle, n):
    rng = np.random.default_rng(n + 3)
    v = rand_fp2(rng, n)
    iv = be.upload_new(v)
    be.call("fp2_mobius_inverse_inplace_device", iv, 0, n)
    got = be.download_fp2(iv, n)
    # subset sums over index bits
    exp = v.astype(object)
    stride = 1
    while stride < n:
        for i in range(n):
            if i & stride:
                exp[i] = [(exp[i][0] + exp[i ^ stride][0]) % P, (exp[i][1] + exp[i ^ stride][1]) % P]
        stride <<= 1
    assert np.array_equal(got.astype(object), np.array(exp.tolist(), dtype=object))
    be.free(iv)
    if n >= 2:
        L = n.bit_length() - 1
        pts = rand_fp2(rng, L)
        vals = rand_fp2(rng, n)
        src = max(1, n // 3)
        iv = be.upload_new(vals)
        ip = be.upload_new(pts)
        rho, gamma = (tuple(int(x) for x in y) for y in rand_fp2(rng, 2))
        be.call("fp2_affine_eq_weights_inplace_device", iv, n, src, ip, 0, L, rho[0], rho[1], gamma[0], gamma[1])
        got = be.download_fp2(iv, n)
        eqv = oracle.eq_rows(pts, 1, L)
        for i in list(range(min(n, 40))) + [n - 1]:
            t = oracle.fp2_mul(rho, tuple(int(x) for x in eqv[i]))
            u = oracle.fp2_mul(gamma, tuple(int(x) for x in vals[i])) if i < src else (0, 0)
            assert tuple(int(x) for x in got[i]) == ((t[0] + u[0]) % P, (t[1] + u[1]) % P)
        be.free(iv)
        be.free(ip)


def test_powers_and_row_dots(be, oracle):
    rng = np.random.default_rng(11)
    base = tuple(int(x) for x in rand_fp2(rng, 1)[0])
    out = be.alloc(16 * 300)
    be.call("fp2_powers_device", base[0], base[1], out, 0, 300)
    got = be.download_fp2(out, 300)
    cur = base
    for i in range(300):
        assert tuple(int(x) for x in got[i]) == cur
        cur = oracle.fp2_mul(cur, base)
    be.free(out)
    rows, length, stride = 5, 700, 712
    a, b = rand_fp2(rng, rows * stride), rand_fp2(rng, rows * stride)
    ia, ib, io = be.upload_new(a), be.upload_new(b), be.alloc(16 * rows)
    be.call("fp2_row_dots_device", ia, 0, stride, ib, 0, stride, io, 0, rows, length)
    got = be.download_fp2(io, rows)
    for r in range(rows):
        x = np.zeros((2 * length, 2), dtype=np.uint64)
        y = np.zeros((2 * length, 2), dtype=np.uint64)
        x[0::2] = a[r * stride:r * stride + length]
        y[0::2] = b[r * stride:r * stride + length]
        assert np.array_equal(got[r], oracle.product_round(x, y, length)[0])
    for i in (ia, ib, io):
        be.free(i)


def test_errors_are_reported_not_faulted(be):
    """Geometry and id validation happen on the host (lib.rs:6829-6958)."""
    from volta_zk_b200 import accel

    with pytest.raises(accel.AccelError, match="unknown resident buffer id"):
        be.call("fp2_fold_rows_device", 12345, 0, 1, 4, accel.fp2((1, 0)), 999, 0)
    buf = be.alloc(64)
    with pytest.raises(accel.AccelError, match="out of bounds"):
        be.call("fp2_fold_rows_device", buf, 0, 1, 8, accel.fp2((1, 0)), buf, 0)
    with pytest.raises(accel.AccelError, match="invalid resident row-fold geometry"):
        be.call("fp2_fold_rows_device", buf, 0, 1, 3, accel.fp2((1, 0)), buf, 0)
    be.free(buf)
    with pytest.raises(accel.AccelError, match="stale"):
        be.free(buf)
    with pytest.raises(accel.AccelError, match="unsupported in the B200 build"):
        be.call("x4c_session_reusable_boundary")
