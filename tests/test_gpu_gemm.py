"""Tensor-core witness GEMMs against the oracle's exact i64 loop
(gemm.rs:40-60, 120-154): full-range int16 operands, ragged shapes, the
long-k path (int32 partials flushed to int64), the reference's fused
epilogue golden checksums, hybrid and resident entry points."""

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


def ptr(a):
    return a.ctypes.data_as(C.c_void_p)


def rand_i16(rng, n):
    return rng.integers(-32768, 32768, size=n, dtype=np.int64).astype(np.int16)


SHAPES = [(1, 1, 1), (3, 5, 7), (64, 64, 64), (65, 130, 67), (17, 768, 2304), (128, 3072, 96), (2, 20000, 33)]


@pytest.mark.parametrize("m,k,n", SHAPES)
def test_gemm_i64(be, oracle, m, k, n):
    rng = np.random.default_rng(m * 1000 + k + n)
    a, b = rand_i16(rng, m * k), rand_i16(rng, k * n)
    exp = oracle.gemm_i64(a, b, m, k, n)
    aid, bid = be.upload_new(a), be.upload_new(b)
    oid = be.alloc(8 * m * n)
    be.call("gemm_i64_device", aid, 0, bid, 0, oid, 0, m, k, n)
    assert np.array_equal(be.download(oid, 8 * m * n, dtype=np.int64), exp)
    out = np.zeros(m * n, dtype=np.int64)
    assert be.lib.volta_cuda_gemm_i64(be.ctx, ptr(a), ptr(b), ptr(out), m, k, n) == 0, be.last_error()
    assert np.array_equal(out, exp)
    for i in (aid, bid, oid):
        be.free(i)


def test_gemm_extreme_values_long_k(be, oracle):
    """All operands -32768 (largest |a b|), k beyond the int32-exact chunk."""
    m, k, n = 3, 40000, 9
    a = np.full(m * k, -32768, dtype=np.int16)
    b = np.full(k * n, -32768, dtype=np.int16)
    b[::7] = 32767
    exp = oracle.gemm_i64(a, b, m, k, n)
    out = np.zeros(m * n, dtype=np.int64)
    assert be.lib.volta_cuda_gemm_i64(be.ctx, ptr(a), ptr(b), ptr(out), m, k, n) == 0, be.last_error()
    assert np.array_equal(out, exp)


@pytest.mark.parametrize("m,k,n,shift", [(1, 1, 1, 1), (5, 9, 13, 3), (33, 768, 100, 8), (64, 3072, 64, 17),
                                         (7, 16, 5, 62)])
def test_gemm_requant_auth(be, oracle, m, k, n, shift):
    rng = np.random.default_rng(m + k + n + shift)
    a, b = rand_i16(rng, m * k), rand_i16(rng, k * n)
    masks = rng.integers(0, P, size=m * n, dtype=np.uint64)
    eo, ec = oracle.gemm_requant_auth(a, b, masks, m, k, n, shift)
    ids = [be.upload_new(x) for x in (a, b, masks)]
    oid, cid = be.alloc(2 * m * n), be.alloc(8 * m * n)
    be.call("gemm_requant_auth_device", ids[0], 0, ids[1], 0, ids[2], 0, oid, 0, cid, 0, m, k, n, shift)
    assert np.array_equal(be.download(oid, 2 * m * n, dtype=np.int16), eo)
    assert np.array_equal(be.download(cid, 8 * m * n), ec)
    out, corr = np.zeros(m * n, dtype=np.int16), np.zeros(m * n, dtype=np.uint64)
    rc = be.lib.volta_cuda_gemm_requant_auth(be.ctx, ptr(a), ptr(b), ptr(masks), ptr(out), ptr(corr), m, k, n, shift)
    assert rc == 0, be.last_error()
    assert np.array_equal(out, eo) and np.array_equal(corr, ec)
    for i in ids + [oid, cid]:
        be.free(i)


@pytest.mark.parametrize("m,k,n,out_ck,corr_ck", [
    (16, 128, 768, 0xd627d7c8948ce1e4, 0xdd63d6266710a934),
    (100, 768, 2304, 0x98d0ad1723fb5ba4, 0x657f2372e3e080c3),
    (100, 768, 3072, 0x622a3f3b6103a2a0, 0x0a16ee945a99dea3),
])
def test_fused_epilogue_golden(be, oracle, m, k, n, out_ck, corr_ck):
    """cuda/p7_fused_epilogue.cu:172-263 output / correction checksums (published run)."""
    a = (((np.arange(m * k, dtype=np.int64) * 37 + 11) % 4001) - 2000).astype(np.int16)
    b = (((np.arange(k * n, dtype=np.int64) * 53 + 5) % 4001) - 2000).astype(np.int16)
    x = np.arange(m * n, dtype=np.uint64) * np.uint64(0x9E3779B9) + np.uint64(17)
    masks = np.where(x >= np.uint64(P), x - np.uint64(P), x).astype(np.uint64)
    out, corr = np.zeros(m * n, dtype=np.int16), np.zeros(m * n, dtype=np.uint64)
    rc = be.lib.volta_cuda_gemm_requant_auth(be.ctx, ptr(a), ptr(b), ptr(masks), ptr(out), ptr(corr), m, k, n, 8)
    assert rc == 0, be.last_error()
    assert oracle.fnv_u64(out.view(np.uint16).astype(np.uint64)) == out_ck
    assert oracle.fnv_u64(corr) == corr_ck


def test_gemm_rejects_bad_geometry(be):
    buf = be.alloc(64)
    assert be.lib.volta_cuda_gemm_i64_device(be.ctx, buf, 0, buf, 0, buf, 0, 0, 4, 4) != 0
    assert be.lib.volta_cuda_gemm_i64_device(be.ctx, buf, 0, buf, 0, buf, 0, 4, 4, 4) != 0  # beyond the buffers
    assert be.lib.volta_cuda_gemm_requant_auth_device(be.ctx, buf, 0, buf, 0, buf, 0, buf, 0, buf, 0, 1, 1, 1, 0) != 0
    be.free(buf)


def test_epilogue_output_is_mac_authenticated(be, oracle):
    """End to end through the VOLE-MAC: the device expands the mock sub masks
    of a tensor (domain (tag << 32) | row, corr.rs:1896-1915), the fused GEMM
    epilogue publishes corrections out - mask, and the verifier half
    (auth_verifier_from_epilogue, auth.rs:56-69) with the prover's lazily
    expanded tags (prover_tags_from_epilogue, auth.rs:71-95) accepts every
    output: k = m + delta out."""
    from oracle import blind as ob

    m, k, n, shift, tag = 6, 768, 96, 10, 0x0102_0304
    seed = bytes([0x4D] * 32)
    delta = (0x0DDC_0FFE_E123_4567, 0x0BAD_CAFE_7654_3210)
    rng = np.random.default_rng(21)
    a, b = rand_i16(rng, m * k), rand_i16(rng, k * n)
    ids = [be.upload_new(x) for x in (a, b)]
    mid, oid, cid = be.alloc(8 * m * n), be.alloc(2 * m * n), be.alloc(8 * m * n)
    be.call("mock_correlation_sub_masks_device", mid, 0, seed, tag << 32, m, n)
    be.call("gemm_requant_auth_device", ids[0], 0, ids[1], 0, mid, 0, oid, 0, cid, 0, m, k, n, shift)
    out = be.download(oid, 2 * m * n, dtype=np.int16).reshape(m, n)
    corr = be.download(cid, 8 * m * n).reshape(m, n)
    exp_out, _ = oracle.gemm_requant_auth(a, b, np.zeros(m * n, dtype=np.uint64), m, k, n, shift)
    assert np.array_equal(out.reshape(-1), exp_out)
    for row in range(m):
        dom = (tag << 32) | row
        tags = ob.sub_tags(oracle, seed, dom, n)
        keys = ob.auth_verifier(oracle, seed, dom, [int(c) for c in corr[row]], delta)
        assert ob.mac_holds(tags, keys, [int(v) for v in out[row]], delta), row
    # a corrupted correction is rejected
    keys = ob.auth_verifier(oracle, seed, tag << 32, [int(c) + 1 for c in corr[0]], delta)
    assert not ob.mac_holds(ob.sub_tags(oracle, seed, tag << 32, n), keys, [int(v) for v in out[0]], delta)
    for i in ids + [mid, oid, cid]:
        be.free(i)
