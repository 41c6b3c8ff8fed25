"""The allocation-free triple-product round (volta_b200_triple_product_round_noalloc).

It exists for callers that cannot allocate device memory themselves: hosts
whose caching allocator owns the GPU's memory, and round loops that cannot
afford the synchronisation cudaMalloc/cudaFree may cause.  Its reduction
scratch is a fixed array inside the library.  This file is collected last
so that a failure here leaves every other test already run; it also passes
alone in a fresh process (the first call performs the per-device set-up).

Every result is checked against the CPU oracle's round
(oracle.triple_product_round, restating hadamard.rs:222-240) on the same
inputs, bit for bit.
"""

import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
MAX_PAIRS = 22369280  # VOLTA_B200_NOALLOC_MAX_PAIRS (include/volta_b200_ext.h)
pytestmark = pytest.mark.gpu


def _noalloc_fn(lib):
    fn = lib.volta_b200_triple_product_round_noalloc
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
    fn.restype = C.c_int
    return fn


def _tables(rng, pairs):
    return [rng.integers(0, P, size=(2 * pairs, 2), dtype=np.uint64) for _ in range(3)]


def test_noalloc_round_matches_oracle_on_two_calls(oracle):
    import torch

    from volta_zk_b200 import accel

    fn = _noalloc_fn(accel.load_cuda_library())
    rng = np.random.default_rng(2024)
    for call, pairs in enumerate((3001, (1 << 20) + 5)):
        a, b, c = _tables(rng, pairs)
        expected = oracle.triple_product_round(a, b, c, pairs)
        # the caller owns every buffer of the allocation-free call
        dev = [torch.from_numpy(x.view(np.int64)).cuda() for x in (a, b, c)]
        out = torch.full((6,), -1, dtype=torch.int64, device="cuda")
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = fn(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), pairs, out.data_ptr(), None)
        torch.cuda.synchronize()
        assert rc == 0
        got = out.cpu().numpy().view(np.uint64).reshape(3, 2)
        assert np.array_equal(got, expected), f"call {call}: {got} != {expected}"
        if call == 1:  # set-up happened on the first call; later calls allocate nothing
            assert torch.cuda.mem_get_info()[0] == free_before


def test_noalloc_round_at_its_size_limit_on_a_caller_stream(oracle):
    """pairs == VOLTA_B200_NOALLOC_MAX_PAIRS fills every per-block partial of
    the scratch; the calls go to a non-default stream, twice in a row (the
    second reuses the scratch the first left behind)."""
    import torch

    from volta_zk_b200 import accel

    fn = _noalloc_fn(accel.load_cuda_library())
    rng = np.random.default_rng(77)
    a, b, c = _tables(rng, MAX_PAIRS)
    expected = oracle.triple_product_round(a, b, c, MAX_PAIRS)
    pairs = 4097
    host = [np.ascontiguousarray(x[: 2 * pairs]) for x in (a, b, c)]
    dev = [torch.from_numpy(x.view(np.int64)).cuda() for x in (a, b, c)]
    del a, b, c
    stream = torch.cuda.Stream()
    outs = [torch.full((6,), -1, dtype=torch.int64, device="cuda") for _ in range(2)]
    torch.cuda.synchronize()
    for out in outs:
        rc = fn(dev[0].data_ptr(), dev[1].data_ptr(), dev[2].data_ptr(), MAX_PAIRS, out.data_ptr(),
                stream.cuda_stream)
        assert rc == 0
    stream.synchronize()
    for out in outs:
        assert np.array_equal(out.cpu().numpy().view(np.uint64).reshape(3, 2), expected)
    # a smaller call after the full one: partials beyond its blocks are stale
    # and must not be read
    small = [x[: 2 * pairs] for x in dev]
    out = torch.full((6,), -1, dtype=torch.int64, device="cuda")
    torch.cuda.synchronize()
    assert fn(small[0].data_ptr(), small[1].data_ptr(), small[2].data_ptr(), pairs, out.data_ptr(),
              stream.cuda_stream) == 0
    stream.synchronize()
    assert np.array_equal(out.cpu().numpy().view(np.uint64).reshape(3, 2),
                          oracle.triple_product_round(*host, pairs))


def test_noalloc_round_rejects_sizes_beyond_its_scratch():
    import torch

    from volta_zk_b200 import accel

    fn = _noalloc_fn(accel.load_cuda_library())
    buf = torch.zeros(16, dtype=torch.int64, device="cuda")
    ptr = buf.data_ptr()
    assert fn(ptr, ptr, ptr, MAX_PAIRS + 1, ptr, None) == -2  # VOLTA_B200_NOALLOC_TOO_LARGE
    assert fn(ptr, ptr, ptr, 0, ptr, None) == -1
    assert fn(None, ptr, ptr, 4, ptr, None) == -1
