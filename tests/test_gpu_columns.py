"""Parity of ChaCha8 expansion, lookup-column preparation and matrix folds."""

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def be():
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=1)
    yield b
    b.close()


def embed(v):
    v64 = np.asarray(v).astype(np.int64)
    return np.where(v64 >= 0, v64.astype(np.uint64), np.uint64(P) - (-v64).astype(np.uint64)).astype(np.uint64)


@pytest.mark.parametrize("rows,count", [(1, 1), (3, 10), (7, 17), (64, 1000), (512, 16384)])
def test_chacha_fp_rows(be, oracle, rows, count):
    seed = bytes(range(32))
    base = 0x0123456789ABCDEF
    out = be.alloc(8 * rows * count + 8)
    be.call("chacha8_prover_secret_fp_rows_device", out, 8, seed, base, rows, count)
    got = be.download(out, 8 * rows * count, offset_bytes=8).reshape(rows, count)
    assert np.array_equal(got, oracle.chacha_fp_rows(seed, base, rows, count))
    be.free(out)


@pytest.mark.parametrize("rows,count,padded", [(1, 1, 1), (4, 17, 17), (3, 5, 8), (33, 100, 128)])
def test_chacha_fp2_rows_padded(be, oracle, rows, count, padded):
    seed = bytes(range(255, 223, -1))
    base = 0xFEDCBA9876543210
    out = be.alloc(16 * rows * padded)
    be.call("chacha8_prover_secret_fp2_rows_padded_device", out, 0, seed, base, rows, count, padded)
    got = be.download_fp2(out, rows * padded)
    assert np.array_equal(got, oracle.chacha_fp2_rows_padded(seed, base, rows, count, padded))
    be.free(out)


def test_mock_masks_reserved_domains_rejected(be, oracle):
    from volta_zk_b200 import accel

    seed = bytes([3] * 32)
    out = be.alloc(8 * 4 * 8)
    be.call("mock_correlation_sub_masks_device", out, 0, seed, (5 << 32) | 7, 4, 8)
    assert np.array_equal(be.download(out, 8 * 32).reshape(4, 8), oracle.chacha_fp_rows(seed, (5 << 32) | 7, 4, 8))
    with pytest.raises(accel.AccelError, match="reserved correlation bits"):
        be.call("mock_correlation_sub_masks_device", out, 0, seed, 1 << 62, 1, 8)
    be.free(out)


def test_pack_leaf_histograms_and_u32_add(be, oracle):
    rng = np.random.default_rng(1)
    n = 1 << 12
    f = rng.integers(-32768, 32768, size=n)
    col = embed(f)
    cols = np.concatenate([col, embed(rng.integers(0, 1 << 10, size=n))])
    shifts = np.array([0, 16], dtype=np.uint32)
    icol, ish = be.upload_new(cols), be.upload_new(shifts)
    leaf = be.alloc(8 * n)
    alpha0 = int(rng.integers(0, P, dtype=np.uint64))
    be.call("pack_lookup_leaf_device", icol, 0, ish, 0, leaf, 0, 2, n, alpha0)
    got = be.download(leaf, 8 * n)
    second = cols[n:].astype(object)
    exp = [(alpha0 - (int(col[i]) + (int(second[i]) << 16))) % P for i in range(n)]
    assert [int(x) for x in got] == exp
    hist = be.alloc(4 << 16)
    be.call("histogram_lut_device", icol, 0, hist, 0, n, 1)
    h = be.download(hist, 4 << 16, dtype=np.uint32)
    assert np.array_equal(h, np.bincount(f.astype(np.int64) & 0xFFFF, minlength=1 << 16).astype(np.uint32))
    ih = be.upload_new(np.arange(n, dtype=np.uint64) % 37)
    bins = be.alloc(4 * 40)
    be.call("histogram_fp_device", ih, 0, bins, 0, n, 40)
    assert np.array_equal(be.download(bins, 160, dtype=np.uint32),
                          np.bincount(np.arange(n) % 37, minlength=40).astype(np.uint32))
    be.call("u32_add_inplace_device", bins, 0, bins, 0, 40)
    assert np.array_equal(be.download(bins, 160, dtype=np.uint32),
                          2 * np.bincount(np.arange(n) % 37, minlength=40).astype(np.uint32))
    for b in (icol, ish, leaf, hist, ih, bins):
        be.free(b)


@pytest.mark.parametrize("shift", [8, 12, 20])
def test_requant_and_pair_columns(be, oracle, shift):
    rng = np.random.default_rng(shift)
    rows, cols, row_pad, col_pad = 5, 6, 8, 8
    acc = rng.integers(-(1 << 30), 1 << 30, size=rows * cols, dtype=np.int64)
    out = np.clip((acc + (1 << (shift - 1))) >> shift, -32768, 32767).astype(np.int16)
    out[3] = np.int16((int(out[3]) + 1 + 32768) % 65536 - 32768)  # inconsistent entry: error flag must be set
    ia, io = be.upload_new(acc), be.upload_new(out)
    count = 4 if shift > 16 else 2
    ic = be.alloc(8 * count * row_pad * col_pad)
    err = be.upload_new(np.zeros(1, dtype=np.uint32))
    be.call("requant_columns_device", ia, 0, io, 0, ic, 0, err, 0, rows, cols, row_pad, col_pad, 1, shift)
    got = be.download(ic, 8 * count * row_pad * col_pad).reshape(count, row_pad, col_pad)
    assert be.download(err, 4, dtype=np.uint32)[0] == 1
    for r in range(rows):
        for c in range(cols):
            a, y = int(acc[r * cols + c]), int(out[r * cols + c])
            if shift <= 16:
                assert int(got[0, r, c]) == (a + (1 << (shift - 1)) - (y << shift)) % (1 << 64)
                assert int(got[1, r, c]) == y % P
            else:
                first = shift - 16
                y1 = (a + (1 << (first - 1))) >> first
                assert int(got[0, r, c]) == (a + (1 << (first - 1)) - (y1 << first)) % (1 << 64)
                assert int(got[1, r, c]) == y1 % P
                assert int(got[2, r, c]) == (y1 + (1 << 15) - (y << 16)) % (1 << 64)
                assert int(got[3, r, c]) == y % P
    # padded entries carry acc = out = 0: rem = 2^(s-1) (chained: 2^(s-17), 0, 2^15, 0)
    if shift <= 16:
        assert int(got[0, 7, 7]) == 1 << (shift - 1) and int(got[1, 7, 7]) == 0
    else:
        assert [int(got[k, 7, 7]) for k in range(4)] == [1 << (shift - 17), 0, 1 << 15, 0]
    ip = be.alloc(8 * 2 * row_pad * col_pad)
    be.call("pair_columns_device", ia, 0, io, 0, ip, 0, rows, cols, row_pad, col_pad, 5, 9, 1, 0)
    pc = be.download(ip, 16 * row_pad * col_pad).reshape(2, row_pad, col_pad)
    assert int(pc[0, 0, 0]) == int(acc[0]) % P and int(pc[1, 1, 2]) == int(out[cols + 2]) % P
    assert int(pc[0, 6, 0]) == 5 and int(pc[1, 0, 7]) == 9
    for b in (ia, io, ic, err, ip):
        be.free(b)


@pytest.mark.parametrize("kind", [0, 1, 2, 3, 4])
@pytest.mark.parametrize("axis", [0, 1])
@pytest.mark.parametrize("rows,cols", [(3, 5), (768, 96), (64, 3072), (4096, 4)])
def test_matrix_fold(be, oracle, kind, axis, rows, cols):
    rng = np.random.default_rng(kind * 10 + axis + rows)
    stride, off = cols + 3, 2
    n = rows * stride
    if kind == 0:
        m = rng.integers(-32768, 32768, size=n).astype(np.int16)
    elif kind == 1:
        m = rng.integers(-(1 << 62), 1 << 62, size=n, dtype=np.int64)
    elif kind == 2:
        m = rng.integers(0, P, size=n, dtype=np.uint64)
    elif kind == 3:
        m = rng.integers(0, P, size=(n, 2), dtype=np.uint64)
    else:
        m = rng.integers(0, 1 << 32, size=n, dtype=np.uint64).astype(np.uint32)
    cols_used = cols - off if cols > off else cols
    terms = rows if axis == 0 else cols_used
    real = cols_used if axis == 0 else rows
    out_pad = 1 << max(0, (real - 1).bit_length())
    w = rng.integers(0, P, size=(terms, 2), dtype=np.uint64)
    im, iw = be.upload_new(m), be.upload_new(w)
    io = be.alloc(16 * out_pad)
    be.call("matrix_fold_device", im, 0, iw, 0, io, 0, rows, stride, off, cols_used, out_pad, kind, axis)
    got = be.download_fp2(io, out_pad)
    exp = oracle.matrix_fold(m, w, rows, stride, off, cols_used, out_pad, kind, axis)
    assert np.array_equal(got, exp)
    for b in (im, iw, io):
        be.free(b)


def test_small_vector_ops(be, oracle):
    rng = np.random.default_rng(9)
    n = 1000
    x = rng.integers(-32768, 32768, size=n).astype(np.int16)
    masks = rng.integers(0, P, size=n, dtype=np.uint64)
    ix, im = be.upload_new(x), be.upload_new(masks)
    out = be.alloc(8 * 1024)
    be.call("subfield_corrections_device", ix, 0, im, 0, out, 0, n, 0)
    got = be.download(out, 8 * n)
    exp = [(int(embed(x)[i]) - int(masks[i])) % P for i in range(n)]
    assert [int(v) for v in got] == exp
    be.call("pad_base_vector_device", ix, 0, out, 0, n, 1024, 77, 0)
    got = be.download(out, 8 * 1024)
    assert np.array_equal(got[:n], embed(x)) and np.all(got[n:] == 77)
    bc = be.alloc(16 * n * 3)
    be.call("base_broadcast_fp2_device", ix, 0, bc, 0, n, 3, 0)
    g = be.download_fp2(bc, 3 * n)
    assert np.array_equal(g[:, 0], np.repeat(embed(x), 3)) and np.all(g[:, 1] == 0)
    rep = be.alloc(2 * n * 4)
    be.call("repeat_vector_device", ix, 0, rep, 0, n, 4, 0)
    assert np.array_equal(be.download(rep, 2 * n * 4, dtype=np.int16), np.tile(x, 4))
    cp = be.alloc(2 * 10 * 7)
    be.call("compact_strided_rows_device", ix, 0, cp, 0, 10, 90, 7, 0)
    assert np.array_equal(be.download(cp, 140, dtype=np.int16).reshape(10, 7),
                          np.stack([x[r * 90:r * 90 + 7] for r in range(10)]))
    cols = rng.integers(0, P, size=2 * 16, dtype=np.uint64)
    ic = be.upload_new(cols)
    dout = be.alloc(16 * 32)
    be.call("deinterleave_base_columns_device", ic, 0, dout, 0, 2, 16)
    d = be.download_fp2(dout, 32)
    for c in range(2):
        col = cols[c * 16:(c + 1) * 16]
        assert np.array_equal(d[c * 16:(c + 1) * 16, 0], np.concatenate([col[0::2], col[1::2]]))
    for b in (ix, im, out, bc, rep, cp, ic, dout):
        be.free(b)


def test_chacha_rows_with_rejected_draw(be, oracle):
    """FpStream([0x11;32], 2215) draws a raw value >= p at index 45451 (found by a
    CPU scan of the oracle stream); the fast row kernel flags that row and the
    fix-up regenerates it with the rejection applied."""
    seed = bytes([0x11] * 32)
    raw = oracle.stream_u64(seed, 2215, 45460)
    assert raw[45451] >= np.uint64(0xFFFFFFFF00000001)
    rows, count, base = 16, 65536, 2208
    out = be.alloc(8 * rows * count)
    be.call("chacha8_prover_secret_fp_rows_device", out, 0, seed, base, rows, count)
    got = be.download(out, 8 * rows * count).reshape(rows, count)
    exp = oracle.chacha_fp_rows(seed, base, rows, count)
    assert np.array_equal(got, exp)
    assert got[2215 - base, 45451] == raw[45452]
    be.free(out)


@pytest.mark.parametrize("n,bins,dist", [
    (1 << 22, 1 << 16, "skewed"), (1 << 22, 40000, "uniform"), ((1 << 20) + 12345, 1 << 16, "one-bin"),
    (300000, 20000, "uniform"), (1 << 24, 1 << 16, "skewed")])
def test_histogram_fp_large_tables(be, n, bins, dist):
    """Tables of 16385 .. 2^16 bins over long columns (the packed 16-bit
    shared-memory counters, flushed every 64512 elements of a CTA's slice):
    exact counts, values at or above `bins` ignored, a single hot bin past
    65535 per CTA."""
    rng = np.random.default_rng(n + bins)
    if dist == "uniform":
        v = rng.integers(0, bins + 500, size=n, dtype=np.uint64)
    elif dist == "one-bin":
        v = np.full(n, bins - 1, dtype=np.uint64)
    else:
        v = np.minimum(rng.geometric(0.01, size=n), bins + 10).astype(np.uint64)
    iv, hist = be.upload_new(v), be.alloc(4 * bins)
    be.call("resident_zero", hist, 0, 4 * bins)
    be.call("histogram_fp_device", iv, 0, hist, 0, n, bins)
    exp = np.bincount(v[v < bins].astype(np.int64), minlength=bins).astype(np.uint32)
    assert np.array_equal(be.download(hist, 4 * bins, dtype=np.uint32), exp)
    be.free(iv)
    be.free(hist)


def test_histogram_lut_large_signed_column(be):
    """u16 lookup indices of a signed column through the packed path: values
    in [-32768, 32767] embedded in Fp, out-of-domain values ignored."""
    rng = np.random.default_rng(77)
    n = (1 << 21) + 3
    f = np.clip(np.round(rng.normal(0, 300, size=n)), -32768, 32767).astype(np.int64)
    col = f.astype(np.uint64)
    col[f < 0] -= np.uint64(0xFFFFFFFF)  # 2^64 + f - (2^32 - 1) = p + f
    col[::1000] = np.uint64(1 << 20)  # outside the i16 domain: not counted
    ic, hist = be.upload_new(col), be.alloc(4 << 16)
    be.call("resident_zero", hist, 0, 4 << 16)
    be.call("histogram_lut_device", ic, 0, hist, 0, n, 1)
    keep = np.ones(n, dtype=bool)
    keep[::1000] = False
    exp = np.bincount(f[keep] & 0xFFFF, minlength=1 << 16).astype(np.uint32)
    assert np.array_equal(be.download(hist, 4 << 16, dtype=np.uint32), exp)
    be.free(ic)
    be.free(hist)
