"""Fixed-point GPT-2 forward primitives on the device against the oracle
(which tests/test_oracle_golden.py pins to the reference's NumPy mirror):
the whole layer composition against the golden digests, then each primitive
on ragged shapes, decode offsets (pos0 > 0), the row-shifted softmax, the
chained requant above 2^16 and the sticky error word."""

import numpy as np
import pytest

import fixed_layer as fl

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=0)
    yield b
    b.close()


@pytest.fixture(scope="module")
def dev(be):
    return fl.DeviceOps(be)


def i16(rng, n, lo=-32768, hi=32768):
    return rng.integers(lo, hi, size=n, dtype=np.int64).astype(np.int16)


def test_layer_matches_reference_mirror(dev, oracle):
    g = np.load(fl.GOLDEN)
    seed, t = (int(v) for v in g["seed_t"])
    w, x = fl.synthetic_layer(seed, t)
    luts = {k: g[k] for k in ("exp", "gelu", "ln_rsqrt", "softmax_recip")}
    res = fl.forward_layer(dev, x, w, luts, t)
    assert res["errors"] == [0] * len(res["errors"])
    assert fl.check_against_golden(res) == []


@pytest.mark.parametrize("m,k,n,shift,with_bias,with_res", [(1, 1, 1, 1, False, False), (5, 70, 9, 10, True, True),
                                                            (64, 768, 128, 10, True, False),
                                                            (33, 3072, 65, 20, False, True),
                                                            (7, 100, 300, 3, True, True),
                                                            # decode rows (the few-row path)
                                                            (1, 768, 2304, 10, False, False),
                                                            (2, 3072, 768, 10, True, True),
                                                            (4, 768, 3072, 17, True, False),
                                                            (3, 100, 1000, 5, False, True)])
def test_fixed_gemm(dev, oracle, m, k, n, shift, with_bias, with_res):
    rng = np.random.default_rng(m + k + n)
    x, w = i16(rng, m * k, -600, 600), i16(rng, k * n, -600, 600)
    bias = i16(rng, n, -2000, 2000) if with_bias else None
    res = i16(rng, m * n) if with_res else None
    got = dev.gemm(x, w, bias, res, m, k, n, shift)
    exp = oracle.fixed_gemm(x, w, bias, res, m, k, n, shift)
    for g_, e_ in zip(got, exp):
        if e_ is None:
            assert g_ is None
        elif isinstance(e_, int):
            assert g_ == e_
        else:
            assert np.array_equal(g_, e_)


def test_fixed_gemm_few_rows_extremes(dev, oracle):
    """The few-row path at the int16 extremes over k = 3072 (exact int64 sums)
    and for a width that is not a multiple of its 32-column blocks."""
    for m, k, n in ((1, 3072, 777), (4, 3072, 33)):
        x = np.where(np.arange(m * k) % 3 == 0, -32768, 32767).astype(np.int16)
        w = np.where(np.arange(k * n) % 5 == 0, -32768, 32767).astype(np.int16)
        got = dev.gemm(x, w, None, None, m, k, n, 30)
        exp = oracle.fixed_gemm(x, w, None, None, m, k, n, 30)
        assert np.array_equal(got[0], exp[0]) and np.array_equal(got[1], exp[1]) and got[3] == exp[3]


def test_logits_one_row_full_vocabulary(be, oracle):
    rng = np.random.default_rng(5)
    rows, d, vocab = 1, 768, 50257
    xin, w = i16(rng, rows * d, -3000, 3000), i16(rng, vocab * d, -3000, 3000)
    a, b, o = be.upload_new(xin), be.upload_new(w), be.alloc(8 * rows * vocab)
    be.call("fixed_logits_device", a, 0, b, 0, o, 0, rows, d, vocab)
    assert np.array_equal(be.download(o, 8 * rows * vocab, dtype=np.int64), oracle.fixed_logits(xin, w, rows, d, vocab))
    for i in (a, b, o):
        be.free(i)


def test_fixed_gemm_error_word(dev, oracle):
    """Saturating requant and residual overflow set the sticky error word."""
    m, k, n = 4, 16, 8
    x = np.full(m * k, 30000, np.int16)
    w = np.full(k * n, 30000, np.int16)
    got = dev.gemm(x, w, None, None, m, k, n, 2)
    exp = oracle.fixed_gemm(x, w, None, None, m, k, n, 2)
    assert got[3] == exp[3] == 1
    assert np.array_equal(got[1], exp[1])


@pytest.mark.parametrize("rows,pos0,heads,head_dim", [(1, 0, 1, 64), (8, 0, 12, 64), (70, 0, 2, 64), (5, 100, 3, 32),
                                                      (130, 3, 1, 16)])
def test_scores_softmax_av(dev, oracle, rows, pos0, heads, head_dim):
    rng = np.random.default_rng(rows * 7 + pos0 + heads)
    seq, d = pos0 + rows, heads * head_dim
    q, k, v = i16(rng, rows * d, -400, 400), i16(rng, seq * d, -400, 400), i16(rng, seq * d, -2000, 2000)
    got = dev.scores(q, k, rows, seq, pos0, heads, head_dim, 10)
    exp = oracle.fixed_attention_scores(q, k, rows, seq, pos0, heads, head_dim, 10)
    assert all(np.array_equal(a, b) for a, b in zip(got[:2], exp[:2])) and got[2] == exp[2]
    g = np.load(fl.GOLDEN)
    for row_shift in (0, 1):
        gs = dev.softmax(exp[1], g["exp"], g["softmax_recip"], rows, pos0, heads, 6, 26, 14, row_shift)
        es = oracle.fixed_softmax(exp[1], g["exp"], g["softmax_recip"], rows, pos0, heads, 6, 26, 14, row_shift)
        for a, b in zip(gs, es):
            assert (a == b) if isinstance(b, int) else np.array_equal(a, b)
    wts = es[4]
    ga = dev.av(wts, v, rows, seq, pos0, d, heads, 12)
    ea = oracle.fixed_av(wts, v, rows, seq, pos0, d, heads, 12)
    assert np.array_equal(ga[0], ea[0]) and np.array_equal(ga[1], ea[1]) and ga[2] == ea[2]


def test_scores_clamp17_error(dev, oracle):
    rows, heads, hd = 3, 1, 64
    q = np.full(rows * hd, 32767, np.int16)
    k = np.full(rows * hd, 32767, np.int16)
    got = dev.scores(q, k, rows, rows, 0, heads, hd, 10)
    exp = oracle.fixed_attention_scores(q, k, rows, rows, 0, heads, hd, 10)
    assert got[2] == exp[2] == 1
    assert np.array_equal(got[1], exp[1])


@pytest.mark.parametrize("rows,d", [(1, 1), (3, 768), (65, 100), (17, 3072)])
def test_layer_norm(dev, oracle, rows, d):
    rng = np.random.default_rng(rows + d)
    x = i16(rng, rows * d, -3000, 3000)
    gain, bias = i16(rng, d, 40, 90), i16(rng, d, -128, 128)
    lut = fl.np.load(fl.GOLDEN)["ln_rsqrt"]
    got = dev.layer_norm(x, gain, bias, lut, rows, d, 7, 16)
    exp = oracle.fixed_layer_norm(x, gain, bias, lut, rows, d, 7, 16)
    for a, b in zip(got, exp):
        assert (a == b) if isinstance(b, int) else np.array_equal(a, b)


def test_embed_lookup_requant_logits(be, oracle):
    rng = np.random.default_rng(11)
    vocab, positions, d, rows, pos0 = 300, 40, 96, 9, 5
    wte, wpe = i16(rng, vocab * d, -3000, 3000), i16(rng, positions * d, -3000, 3000)
    tokens = rng.integers(0, vocab, size=rows, dtype=np.uint32)
    tokens[3] = vocab + 7  # out of range: zero row and the error word
    ids = [be.upload_new(a) for a in (tokens, wte, wpe)]
    for shift in (3, 0, -2):
        acc, out, err = be.alloc(8 * rows * d), be.alloc(2 * rows * d), be.upload_new(np.zeros(1, np.uint32))
        be.call("fixed_embed_device", ids[0], 0, ids[1], 0, ids[2], 0, acc, 0, out, 0, err, 0, rows, d, vocab,
                positions, pos0, shift)
        ea, eo, ee = oracle.fixed_embed(tokens, wte, wpe, rows, d, vocab, positions, pos0, shift)
        assert np.array_equal(be.download(acc, 8 * rows * d, dtype=np.int64), ea)
        assert np.array_equal(be.download(out, 2 * rows * d, dtype=np.int16), eo)
        assert int(be.download(err, 4, dtype=np.uint32)[0]) == ee == 1
        for i in (acc, out, err):
            be.free(i)
    # lookup and requant_i16
    x = i16(rng, 5000)
    lut = i16(rng, 1 << 16)
    xi, li, oi = be.upload_new(x), be.upload_new(lut), be.alloc(2 * x.size)
    be.call("fixed_lookup_device", xi, 0, li, 0, oi, 0, x.size)
    assert np.array_equal(be.download(oi, 2 * x.size, dtype=np.int16), oracle.fixed_lookup(x, lut))
    for shift in (0, 1, 5, 17):
        err = be.upload_new(np.zeros(1, np.uint32))
        be.call("fixed_requant_i16_device", xi, 0, oi, 0, err, 0, x.size, shift)
        eo, ee = oracle.fixed_requant_i16(x, shift)
        assert np.array_equal(be.download(oi, 2 * x.size, dtype=np.int16), eo)
        assert int(be.download(err, 4, dtype=np.uint32)[0]) == ee
        be.free(err)
    # logits: x wte^T over a ragged vocabulary
    rows, d, vocab = 3, 768, 1000
    xin, w = i16(rng, rows * d, -3000, 3000), i16(rng, vocab * d, -3000, 3000)
    a, b, o = be.upload_new(xin), be.upload_new(w), be.alloc(8 * rows * vocab)
    be.call("fixed_logits_device", a, 0, b, 0, o, 0, rows, d, vocab)
    assert np.array_equal(be.download(o, 8 * rows * vocab, dtype=np.int64), oracle.fixed_logits(xin, w, rows, d, vocab))
    for i in ids + [xi, li, oi, a, b, o]:
        be.free(i)
