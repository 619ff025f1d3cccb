"""Every device-side wait of the LDLQ sweep is bounded and reports a status
instead of hanging.

A sweep asked to encode k-blocks [0, tk - 1) on a fresh workspace waits for
block tk - 1, which nothing ever writes back (a dependency that never
arrives).  With the wait bound shortened to 50 ms through
exl3b_set_wait_limit_ms, the call must return EXL3B_DEVICE_ERROR (4) within a
fraction of a second, name the cause and the waiting tile, and leave the
device usable: the next normal sweep on it succeeds.  Both tile kernels are
covered: the one-CTA-per-tile kernel (few tiles per launch) and the
persistent lazy-argmin kernel (at least two tiles per SM).  Nothing here
faults or traps the GPU: the kernels end on their own when the bound runs
out.
"""
import ctypes
import re
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def _problem(k, n, seed):
    gen = torch.Generator().manual_seed(seed)
    A = torch.randn(k, k, generator=gen)
    H = A.t() @ A / k + 0.1 * torch.eye(k)
    Wq = torch.randn(k, n, generator=gen)
    return Wq, H


def _raw_sweep(L, Wq, Lfac, K, block_lo, block_hi, ws):
    k, n = Wq.shape
    tr = torch.empty(k // 16, n // 16, 16 * K, dtype=torch.int16, device=Wq.device)
    hatW = torch.empty(k, n, dtype=torch.float32, device=Wq.device)
    seg_c0 = (ctypes.c_int * 2)(0, n // 16)
    seg_K = (ctypes.c_int * 1)(K)
    seg_tr = (ctypes.c_void_p * 1)(tr.data_ptr())
    return L.exl3b_ldlq_sweep(Wq.data_ptr(), Lfac.data_ptr(), k, n, 1, seg_c0, seg_K, seg_tr,
                              0, 128, 0, 128, hatW.data_ptr(), None, None, block_lo, block_hi,
                              ws.data_ptr(), ws.numel(),
                              torch.cuda.current_stream().cuda_stream)


@pytest.mark.parametrize("n,kernel", [(64, "one CTA per tile"), (2560, "persistent lazy")])
def test_dependency_wait_times_out_and_device_stays_usable(n, kernel):
    from exl3b import api, native
    L = native.lib()
    dev = torch.device("cuda", 0)
    k, K = 256, 4
    Wq, H = _problem(k, n, 90 + n)
    Wq = Wq.to(dev)
    Lfac = api._damped_lfac(H, api.sign_vec(k, 3).half(), 0.01, dev)
    wsb = L.exl3b_ldlq_workspace_bytes(k, n, K, 1)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=dev)     # no block written back yet
    torch.cuda.synchronize()
    assert L.exl3b_set_wait_limit_ms(50.0) == 0
    try:
        t0 = time.perf_counter()
        rc = _raw_sweep(L, Wq, Lfac, K, 0, k // 16 - 1, ws)
        dt = time.perf_counter() - t0
        msg = native.last_error()
    finally:
        assert L.exl3b_set_wait_limit_ms(0.0) == 0          # back to the default bound
    assert rc == 4, (rc, msg)
    assert "dependency wait timed out" in msg, msg
    m = re.search(r"k-block (\d+), column (\d+)", msg)
    assert m and int(m.group(1)) <= k // 16 - 2 and int(m.group(2)) < n // 16, msg
    assert dt < 3.0, f"{kernel}: returned after {dt:.2f} s with a 50 ms bound"
    # the context is intact: a normal sweep on the same device succeeds
    hatW, trl, st, _ = api._sweep(Wq, Lfac, [K], [n], "exl3_mul1", 128, 0, 128,
                                  want_states=True)
    api.verify_trellis(trl[0], hatW, K, states=st)
    torch.cuda.synchronize()


def test_wait_limit_argument_checked():
    from exl3b import native
    L = native.lib()
    assert L.exl3b_set_wait_limit_ms(-1.0) == 7
    assert L.exl3b_set_wait_limit_ms(float("nan")) == 7
    assert L.exl3b_set_wait_limit_ms(0.0) == 0
