"""The fused fold + next-round extensions (include/volta_b200_ext.h) against
the oracle's separate fold and round functions, under both timing policies
(the wall-only policy publishes host-bound messages through the mapped
mailbox flag instead of a stream synchronisation)."""

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", params=[0, 1], ids=["events", "counters"])
def be(request):
    from volta_zk_b200 import accel

    b = accel.CudaBackend(policy=request.param)
    yield b
    b.close()


def rand_fp2(rng, n):
    return rng.integers(0, P, size=(n, 2), dtype=np.uint64)


def ext(be, name):
    return getattr(be.lib, "volta_b200_" + name)


@pytest.mark.parametrize("length", [4, 8, 12, 1024, 4100, 1 << 18])
def test_triple_fold_round_matches_fold_then_round(be, oracle, length):
    from volta_zk_b200 import accel

    rng = np.random.default_rng(length)
    v = [rand_fp2(rng, length) for _ in range(3)]
    r = tuple(int(x) for x in rand_fp2(rng, 1)[0])
    ids = [be.upload_new(x) for x in v]
    outs = [be.alloc(16 * (length // 2)) for _ in range(3)]
    msg = np.zeros((3, 2), dtype=np.uint64)
    rc = ext(be, "triple_fold_round_device")(be.ctx, *ids, length, accel.fp2(r), *outs,
                                             msg.ctypes.data_as(np.ctypeslib.ctypes.c_void_p))
    assert rc == 0, be.last_error()
    folded = [oracle.fold_rows(x, 1, length, r) for x in v]
    for k in range(3):
        assert np.array_equal(be.download_fp2(outs[k], length // 2), folded[k])
    assert np.array_equal(msg, oracle.triple_product_round(*folded, length // 4))
    for i in ids + outs:
        be.free(i)


@pytest.mark.parametrize("length", [4, 8, 64, 4096, 1 << 17])
def test_logup_fold_round_matches_fold_then_round(be, oracle, length):
    from volta_zk_b200 import accel

    rng = np.random.default_rng(length + 1)
    v = [rand_fp2(rng, length) for _ in range(4)]
    r = tuple(int(x) for x in rand_fp2(rng, 1)[0])
    s_off = 3
    suffix = rand_fp2(rng, s_off + length // 4)
    ids = [be.upload_new(x) for x in v]
    sid = be.upload_new(suffix)
    outs = [be.alloc(16 * (length // 2)) for _ in range(4)]
    msg = np.zeros((4, 2), dtype=np.uint64)
    rc = ext(be, "logup_fold_round_device")(be.ctx, *ids, length, accel.fp2(r), *outs, sid, s_off,
                                            msg.ctypes.data_as(np.ctypeslib.ctypes.c_void_p))
    assert rc == 0, be.last_error()
    folded = [oracle.fold_rows(x, 1, length, r) for x in v]
    for k in range(4):
        assert np.array_equal(be.download_fp2(outs[k], length // 2), folded[k])
    exp = oracle.logup_general_round(*folded, suffix[s_off:], length // 4)
    assert np.array_equal(msg, exp)
    for i in ids + outs + [sid]:
        be.free(i)


def test_fused_entry_points_reject_bad_geometry(be):
    from volta_zk_b200 import accel

    ids = [be.alloc(16 * 16) for _ in range(9)]
    msg = np.zeros((4, 2), dtype=np.uint64)
    p = msg.ctypes.data_as(np.ctypeslib.ctypes.c_void_p)
    f3 = ext(be, "triple_fold_round_device")
    f4 = ext(be, "logup_fold_round_device")
    zero = accel.fp2((0, 0))
    assert f3(be.ctx, ids[0], ids[1], ids[2], 6, zero, ids[3], ids[4], ids[5], p) == -1
    assert "geometry" in be.last_error()
    assert f3(be.ctx, ids[0], ids[1], ids[2], 2, zero, ids[3], ids[4], ids[5], p) == -1
    assert f3(be.ctx, ids[0], ids[1], ids[2], 64, zero, ids[3], ids[4], ids[5], p) == -1  # beyond the buffers
    assert be.last_error()
    assert f4(be.ctx, *ids[:4], 10, zero, *ids[4:8], ids[8], 0, p) == -1
    # the context stays usable
    assert f3(be.ctx, ids[0], ids[1], ids[2], 16, zero, ids[3], ids[4], ids[5], p) == 0
    for i in ids:
        be.free(i)
