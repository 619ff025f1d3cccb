"""GPU parity of the CUDA tail-biting encoder against the reference's golden
states and the CPU oracle.  The bar is bit-exact states: the kernel keeps the
reference's fp32 operation order (fl(fl(f - x)^2) + best, first index on
ties), so any difference is a bug."""
import ctypes
import os

import numpy as np
import pytest
import torch

from conftest import golden

pytestmark = pytest.mark.gpu

NTHREADS = max(1, min(32, os.cpu_count() or 1))


@pytest.fixture(scope="module")
def ops():
    from exl3b import ops as _ops
    return _ops


def _run(ops, X, K, pivot, margin):
    st = ops.tailbite(torch.from_numpy(X).cuda(), K, pivot=pivot, margin=margin)
    torch.cuda.synchronize()
    return st.cpu().numpy()


@pytest.mark.parametrize("K", range(2, 8))
def test_golden_states(ops, K):
    """Every reference-generated case (Gaussian, tie-heavy, wide targets;
    six pivot/margin combinations)."""
    g = golden("viterbi")
    n = 0
    for key in g.files:
        if not key.startswith("st_") or f"_K{K}_" not in key:
            continue
        _, tag, _, p, m = key.split("_")
        st = _run(ops, g[f"X_{tag}"], K, int(p[1:]), int(m[1:]))
        assert np.array_equal(st.astype(np.uint16), g[key]), key
        n += 1
    assert n >= 8


@pytest.mark.parametrize("K,nseq,pivot,margin", [
    (4, 300, 128, 0),      # >= 2 per SM: the lazy-argmin pipeline, odd tails
    (4, 160, 0, 16),       # quantize() defaults at seed 0 (traced encoder)
    (2, 48, 77, 16), (3, 48, 255, 0), (5, 48, 3, 40),
    (6, 48, 128, 0), (7, 48, 200, 100),
    # lazy pipeline at every K with short / full / pivot-0 first passes
    (4, 444, 0, 16), (5, 301, 3, 40), (6, 297, 255, 0), (7, 445, 200, 100),
    (5, 296, 128, 0), (7, 310, 0, 0),
    (2, 300, 77, 16), (2, 297, 0, 0), (3, 298, 255, 0), (3, 333, 128, 0),
])
def test_random_vs_oracle(ops, oracle, mul1_lut, K, nseq, pivot, margin):
    rng = np.random.default_rng(1000 + K * 7 + pivot)
    X = rng.standard_normal((nseq, 256)).astype(np.float32)
    X[: nseq // 4] *= 0.05                       # small-magnitude tiles
    X[nseq // 4: nseq // 2] = np.round(X[nseq // 4: nseq // 2] * 4) / 4  # coarse grid: ties
    st = _run(ops, X, K, pivot, margin)
    ref = oracle.tailbite(X, mul1_lut, K, pivot=pivot, margin=margin, nthreads=NTHREADS)
    bad = np.nonzero((st != ref).any(1))[0]
    assert bad.size == 0, f"{bad.size} sequences differ, first {bad[:5]}"
    # tail-biting consistency (test_quantize.py:141-152)
    assert np.all((st[:, 0] >> K) == (st[:, -1] & ((1 << (16 - K)) - 1)))


def test_other_codes(ops, oracle):
    """3INST / MCG tables go through the same encoder."""
    rng = np.random.default_rng(7)
    X = rng.standard_normal((12, 256)).astype(np.float32)
    for code in ("exl3_3inst", "exl3_mcg"):
        st = ops.tailbite(torch.from_numpy(X).cuda(), 4, pivot=10, margin=0, code=code)
        ref = oracle.tailbite(X, oracle.code_lut(code), 4, pivot=10, margin=0,
                              nthreads=NTHREADS)
        assert np.array_equal(st.cpu().numpy(), ref), code


def test_xtq_vit_run_dropin(oracle, mul1_lut):
    """The reference's ctypes entry points (viterbi_esimd.cpp:935-1005):
    same signature, host buffers, mul1 at K=4, same return codes."""
    from exl3b import native
    L = native.lib()
    assert L.xtq_vit_init() == 0
    rng = np.random.default_rng(5)
    X = np.ascontiguousarray(rng.standard_normal((20, 256)).astype(np.float32))
    out = np.zeros((20, 256), dtype=np.int32)
    P = ctypes.c_void_p
    rc = L.xtq_vit_run(X.ctypes.data_as(P), 20, b"mul1p", 16, 40, out.ctypes.data_as(P))
    assert rc == 0, native.last_error()
    ref = oracle.tailbite(X, mul1_lut, 4, pivot=40, margin=16, nthreads=NTHREADS)
    assert np.array_equal(out, ref)
    assert L.xtq_vit_run(X.ctypes.data_as(P), 0, b"mul1p", 0, 0, out.ctypes.data_as(P)) == 6
    assert L.xtq_vit_run(X.ctypes.data_as(P), 20, b"ih2x2", 0, 0, out.ctypes.data_as(P)) == 7
    assert L.xtq_vit_run(X.ctypes.data_as(P), 5000, b"mul1p", 0, 0, out.ctypes.data_as(P)) == 6


def test_workspace_validation(ops):
    from exl3b import native
    L = native.lib()
    X = torch.zeros(4, 256, device="cuda")
    S = torch.zeros(4, 256, dtype=torch.int32, device="cuda")
    need = L.exl3b_tailbite_workspace_bytes(4, 4)
    ws = torch.empty(need, dtype=torch.uint8, device="cuda")
    rc = L.exl3b_tailbite(X.data_ptr(), 4, 4, 0, 0, 0, S.data_ptr(), ws.data_ptr(),
                          need - 1, None)
    assert rc == 11
    rc = L.exl3b_tailbite(X.data_ptr(), 4, 4, 0, 0, 0, S.data_ptr(), None, 0, None)
    assert rc == 0, native.last_error()
    torch.cuda.synchronize()


def test_serve_worker_matches_oracle(oracle, mul1_lut):
    """The exl3b_vit worker over the framed protocol (the reference's "proc"
    transport) returns the oracle's states, chunked across frames."""
    import torch
    from exl3b import transport as tp
    rng = np.random.default_rng(77)
    X = rng.standard_normal((37, 256)).astype(np.float32)
    ref = oracle.tailbite(X, mul1_lut, 4, pivot=128, margin=0, nthreads=NTHREADS)
    w = tp.ServeWorker(devidx=0)
    try:
        assert np.array_equal(w.run(X, "mul1p", 0, 128), ref)
        ref2 = oracle.tailbite(X, mul1_lut, 4, pivot=0, margin=16, nthreads=NTHREADS)
        assert np.array_equal(w.run(X, "mul1", 16, 0), ref2)
        # rc passthrough: bad pivot is xtq_vit_run's rc 7, worker keeps serving
        rc, _ = w.request(1, 0, 300, 2, 2048, "mul1p", X[:2])
        assert rc == 7
        assert np.array_equal(w.run(X[:5], "mul1p", 0, 128), ref[:5])
    finally:
        assert w.close() == 0
    os.environ["XTQ_VIT_MAXSEQ"] = "16"
    try:
        st = tp.tailbite_proc(torch.from_numpy(X).t(), pivot=128, margin=0)
    finally:
        del os.environ["XTQ_VIT_MAXSEQ"]
    assert np.array_equal(st.t().numpy(), ref.astype(np.int64))


def test_xtq_vit_run_lazy_batch(oracle, mul1_lut):
    """xtq_vit_run with >= 2 sequences per SM runs the lazy-argmin pipeline
    behind the reference's ctypes signature: same states as the oracle."""
    from exl3b import native
    L = native.lib()
    rng = np.random.default_rng(303)
    X = rng.standard_normal((300, 256)).astype(np.float32)
    X[:50] = np.round(X[:50] * 4) / 4                  # tie-heavy
    out = np.zeros((300, 256), np.int32)
    P = ctypes.c_void_p
    rc = L.xtq_vit_run(X.ctypes.data_as(P), 300, b"mul1p", 0, 128, out.ctypes.data_as(P))
    assert rc == 0, native.last_error()
    ref = oracle.tailbite(X, mul1_lut, 4, pivot=128, margin=0, nthreads=NTHREADS)
    assert np.array_equal(out, ref)


@pytest.fixture(scope="module")
def xq():
    import quantize as _xq     # the drop-in module (exl3xpu-mixedk_b200/quantize.py)
    return _xq


@pytest.mark.parametrize("K", (2, 4, 7))
def test_single_pass_viterbi_vs_reference(xq, K):
    """viterbi() (quantize.py:218-320) through the drop-in module against the
    reference's own outputs: free boundary, a per-sequence overlap pin, and
    back_from=40 on a 60-step sequence (the shortened first pass)."""
    g = golden("viterbi")
    X = torch.from_numpy(g["X_gauss"][:4].T.copy())          # [T=256, B=4]
    lut = xq.get_lut("exl3_mul1")
    st = xq.viterbi(X, lut, K, 16)
    assert st.shape == (256, 4) and st.dtype == torch.int64
    assert np.array_equal(st.t().numpy().astype(np.uint16), g[f"plain_K{K}"])
    ov = torch.from_numpy(g[f"overlap_in_K{K}"])
    st = xq.viterbi(X, lut, K, 16, overlap=ov)
    assert np.array_equal(st.t().numpy().astype(np.uint16), g[f"overlap_K{K}"])
    bf = xq.viterbi(X[:60], lut, K, 16, back_from=40)
    assert bf.shape == (4,)
    assert np.array_equal(bf.numpy().astype(np.uint16), g[f"backfrom40_K{K}"])


@pytest.mark.parametrize("K", range(2, 8))
def test_single_pass_viterbi_vs_oracle(xq, oracle, mul1_lut, K):
    """Every K, sequence lengths 1..256, more sequences than SMs (several
    waves), overlap pins, and back_from before, at and past the last step."""
    rng = np.random.default_rng(500 + K)
    lut = xq.get_lut("exl3_mul1")
    for T, nseq in ((256, 170), (61, 7), (1, 3), (17, 5)):
        X = rng.standard_normal((nseq, T)).astype(np.float32)
        Xt = torch.from_numpy(X.T.copy())
        st = xq.viterbi(Xt, lut, K).t().numpy()
        assert np.array_equal(st, oracle.viterbi(X, mul1_lut, K)), (T, "plain")
        ov = rng.integers(0, 1 << (16 - K), nseq)
        st = xq.viterbi(Xt, lut, K, overlap=torch.from_numpy(ov)).t().numpy()
        assert np.array_equal(st, oracle.viterbi(X, mul1_lut, K, overlap=ov)), (T, "overlap")
        for bf in sorted({0, T // 2, T - 1, T + 5}):
            got = xq.viterbi(Xt, lut, K, back_from=bf).numpy()
            ref = oracle.viterbi_back_from(X, mul1_lut, K, 16, bf)
            assert np.array_equal(got, ref), (T, "back_from", bf)


def test_viterbi_rejects_what_it_cannot_encode(xq):
    X = torch.zeros(257, 2)
    lut = xq.get_lut("exl3_mul1")
    with pytest.raises(ValueError):
        xq.viterbi(X, lut, 4)                      # longer than one 256-step pass
    with pytest.raises(ValueError):
        xq.viterbi(X[:8], lut, 4, overlap=torch.tensor([0, 1 << 12]))
    with pytest.raises(ValueError):
        xq.viterbi(X[:8], lut, 4, emit_mode="gemm")
    with pytest.raises(ValueError):
        xq.viterbi(X[:8], torch.randn(65536), 4)   # not an EXL3 table


def test_had_left_right_vs_reference_formula(xq):
    """had_left / had_right (quantize.py:135-146) against the explicit
    block-diagonal product in fp64, with the other axis not a multiple of 128."""
    gen = torch.Generator().manual_seed(12)
    h = xq.hadamard128()
    for k, n in ((256, 40), (128, 300), (384, 128)):
        w = torch.randn(k, n, generator=gen)
        ref = (h.double() @ w.double().view(k // 128, 128, n)).view(k, n)
        got = xq.had_left(w, h)
        assert got.shape == (k, n) and got.device == w.device
        assert ((got.double() - ref).abs().max() / ref.abs().max()) < 2e-6
    for k, n in ((40, 256), (300, 128), (128, 384)):
        w = torch.randn(k, n, generator=gen)
        ref = (w.double().view(k, n // 128, 128) @ h.double()).view(k, n)
        got = xq.had_right(w)
        assert ((got.double() - ref).abs().max() / ref.abs().max()) < 2e-6
    with pytest.raises(ValueError):
        xq.had_left(torch.zeros(100, 128))
    with pytest.raises(ValueError):
        xq.had_right(torch.zeros(128, 128), torch.eye(128))


def test_codes_registry(xq):
    """CODES (quantize.py:44-49): name -> (decode_fn, metadata) for the codes
    this package encodes; decode_fn reproduces get_lut."""
    for name in ("exl3_mul1", "exl3_3inst", "exl3_mcg"):
        fn, meta = xq.CODES[name]
        assert meta["V"] == 1
        s = torch.arange(0, 65536, 97)
        assert torch.equal(fn(s), xq.get_lut(name)[s])
