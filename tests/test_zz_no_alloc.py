"""The allocation-free encoder entry point, exl3b_tailbite_noalloc.

It exists for callers that must not allocate device memory while they run
(for example code inside a process whose GPU memory is reserved by another
allocator, which treats later cudaMalloc calls as failures).  Its scratch is a
fixed array inside the library, so these tests check, through the C ABI:
  * two calls in a row give exactly the states of the regular entry point
    exl3b_tailbite (the encoder is bit-exact, so the tolerance is zero), and
    of the CPU oracle;
  * every K = 2..7 with every code (mul1, 3inst, MCG: the kernel computes the
    decode values from the code formulas), and a batch at each K's limit;
  * after one warm-up call per K, further calls leave the device's free
    memory unchanged;
  * a request larger than the fixed scratch is refused with a clear error.

Kept in its own file, named to be collected last.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

# sequences one call takes at most, per K (64 MiB / (256 steps x row bytes))
LIMIT = {2: 64, 3: 64, 4: 128, 5: 128, 6: 256, 7: 512}


def _states(L, fn, X, K, code, pivot, margin):
    n = X.shape[0]
    out = torch.full((n, 256), -1, dtype=torch.int32, device=X.device)
    if fn == "noalloc":
        rc = L.exl3b_tailbite_noalloc(X.data_ptr(), n, K, code, pivot, margin,
                                      out.data_ptr(), None)
    else:
        rc = L.exl3b_tailbite(X.data_ptr(), n, K, code, pivot, margin, out.data_ptr(),
                              None, 0, None)
    torch.cuda.synchronize()
    from exl3b import native
    assert rc == 0, native.last_error()
    return out.cpu().numpy()


def test_no_alloc_entry_point_matches_regular_one(oracle):
    from exl3b import native
    L = native.lib()
    gen = torch.Generator().manual_seed(77)
    # two calls in a row (different K, sizes, pivot/margin and code), then a
    # repeat of the first shape: the shared scratch keeps the previous call's
    # contents and must not leak into the next result
    calls = [(4, 100, 128, 0, 0), (2, 64, 0, 16, 0), (4, 128, 31, 16, 1)]
    for K, n, pivot, margin, code in calls:
        X = (torch.randn(n, 256, generator=gen) * 0.9).cuda()
        a = _states(L, "noalloc", X, K, code, pivot, margin)
        b = _states(L, "regular", X, K, code, pivot, margin)
        assert np.array_equal(a, b), (K, n, pivot, margin, code)
        assert np.all((a[:, 0] >> K) == (a[:, -1] & ((1 << (16 - K)) - 1)))
    # and the first call's shape against the CPU oracle directly
    X = (torch.randn(16, 256, generator=gen) * 0.9)
    a = _states(L, "noalloc", X.cuda(), 4, 0, 128, 0)
    ref = oracle.tailbite(X.numpy(), oracle.code_lut("exl3_mul1"), 4, pivot=128, margin=0,
                          nthreads=8)
    assert np.array_equal(a, ref)


@pytest.mark.parametrize("K", range(2, 8))
def test_no_alloc_every_width_and_code(K):
    """Every code (the in-kernel decode formulas, including MCG) at every K,
    on a small batch, and a batch at the K's sequence limit."""
    from exl3b import native
    L = native.lib()
    gen = torch.Generator().manual_seed(100 + K)
    for code in (0, 1, 2):
        X = (torch.randn(9, 256, generator=gen) * 1.1).cuda()
        a = _states(L, "noalloc", X, K, code, 77, 16)
        b = _states(L, "regular", X, K, code, 77, 16)
        assert np.array_equal(a, b), (K, code)
    X = torch.randn(LIMIT[K], 256, generator=gen).cuda()
    a = _states(L, "noalloc", X, K, 0, 128, 0)
    b = _states(L, "regular", X, K, 0, 128, 0)
    assert np.array_equal(a, b), (K, "limit batch")


def test_no_alloc_allocates_nothing_after_warm_up():
    """After one warm-up call per K (which sets the device up), calls of every
    K leave the device's free memory where it was."""
    from exl3b import native
    L = native.lib()
    X = torch.randn(64, 256, generator=torch.Generator().manual_seed(5)).cuda()
    outs = {K: torch.empty(64, 256, dtype=torch.int32, device="cuda") for K in range(2, 8)}
    for K in range(2, 8):
        assert L.exl3b_tailbite_noalloc(X.data_ptr(), 64, K, 0, 128, 0,
                                        outs[K].data_ptr(), None) == 0, native.last_error()
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for rep in range(3):
        for K in range(2, 8):
            assert L.exl3b_tailbite_noalloc(X.data_ptr(), 64, K, rep % 3, 7 * rep, 16 * rep,
                                            outs[K].data_ptr(), None) == 0, native.last_error()
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0, (free0, free1)


def test_no_alloc_rejects_oversized_request():
    from exl3b import native
    L = native.lib()
    X = torch.zeros(129, 256, device="cuda")
    out = torch.zeros(129, 256, dtype=torch.int32, device="cuda")
    rc = L.exl3b_tailbite_noalloc(X.data_ptr(), 129, 4, 0, 0, 0, out.data_ptr(), None)
    assert rc == 6
    msg = native.last_error()
    assert "at most 128 sequences" in msg and "K=4" in msg
