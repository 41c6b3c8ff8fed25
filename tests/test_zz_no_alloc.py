"""The allocation-free triple-product round (volta_b200_triple_product_round_noalloc).

It exists for callers that cannot allocate device memory themselves: hosts
whose caching allocator owns the GPU's memory, and round loops that cannot
afford the synchronisation cudaMalloc/cudaFree may cause.  Its reduction
scratch is a fixed array inside the library.  This file is collected last
so that a failure here leaves every other test already run; it also passes
alone in a fresh process (the first call performs the per-device set-up).
"""

import ctypes as C

import numpy as np
import pytest

P = 0xFFFFFFFF00000001
pytestmark = pytest.mark.gpu


def _noalloc_fn(lib):
    fn = lib.volta_b200_triple_product_round_noalloc
    fn.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p, C.c_void_p]
    fn.restype = C.c_int
    return fn


def test_noalloc_round_matches_context_entry_point_on_two_calls():
    import torch

    from volta_zk_b200 import accel

    lib = accel.load_cuda_library()
    fn = _noalloc_fn(lib)
    be = accel.CudaBackend(policy=0)
    rng = np.random.default_rng(2024)
    try:
        for call, pairs in enumerate((3001, (1 << 20) + 5)):
            a, b, c = (rng.integers(0, P, size=(2 * pairs, 2), dtype=np.uint64) for _ in range(3))
            # reference result through the existing context-based entry point
            ids = [be.upload_new(x) for x in (a, b, c)]
            expected = np.zeros((3, 2), dtype=np.uint64)
            be.call("fp2_triple_product_round_device", ids[0], 0, ids[1], 0, ids[2], 0, pairs,
                    expected.ctypes.data_as(C.c_void_p))
            for i in ids:
                be.free(i)
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
    finally:
        be.close()


def test_noalloc_round_rejects_sizes_beyond_its_scratch():
    import torch

    from volta_zk_b200 import accel

    fn = _noalloc_fn(accel.load_cuda_library())
    buf = torch.zeros(16, dtype=torch.int64, device="cuda")
    ptr = buf.data_ptr()
    assert fn(ptr, ptr, ptr, 22369280 + 1, ptr, None) == -2  # VOLTA_B200_NOALLOC_TOO_LARGE
    assert fn(ptr, ptr, ptr, 0, ptr, None) == -1
    assert fn(None, ptr, ptr, 4, ptr, None) == -1
