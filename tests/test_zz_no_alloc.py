"""The allocation-free encoder entry point, exl3b_tailbite_noalloc.

It exists for callers that must not allocate device memory while they run
(for example code inside a process whose GPU memory is reserved by another
allocator, which treats later cudaMalloc calls as failures).  Its scratch is a
fixed array inside the library, so this test checks that two calls in a row,
through the C ABI, give exactly the states of the regular entry point
exl3b_tailbite (the encoder is bit-exact, so the tolerance is zero), and that
a request larger than the fixed scratch is refused with a clear error.

Kept in its own file, named to be collected last.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


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


def test_no_alloc_entry_point_matches_regular_one():
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


def test_no_alloc_rejects_oversized_request():
    from exl3b import native
    L = native.lib()
    X = torch.zeros(129, 256, device="cuda")
    out = torch.zeros(129, 256, dtype=torch.int32, device="cuda")
    rc = L.exl3b_tailbite_noalloc(X.data_ptr(), 129, 4, 0, 0, 0, out.data_ptr(), None)
    assert rc == 6
    msg = native.last_error()
    assert "at most 128 sequences" in msg and "K=4" in msg
