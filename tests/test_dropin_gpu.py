"""The reference's own in-scope checks (quantize/test_quantize.py), restated
against the drop-in module: ``import quantize as xq`` with
exl3xpu-mixedk_b200/ on sys.path, CPU tensors in and out as the reference's
tests pass them, the CUDA kernels underneath.  Same seeds, shapes and pass
criteria as the reference's functions:

  t_pack_roundtrip       test_quantize.py:73-108   (exl3xpu's ref.py is not
                                                   available: the unpack side
                                                   is checked, as the reference
                                                   does without it)
  t_tailbite_consistent  test_quantize.py:141-152
  t_gauss_mse            test_quantize.py:181-201  (the three V=1 EXL3 codes;
                                                   the QTIP 1MAD table is not a
                                                   code this encoder takes)
  t_ldlq_helps           test_quantize.py:204-219
  t_quantize_api         test_quantize.py:278-301

The reference's tiny-L brute-force case (test_quantize.py:111-138, L = 4) is
outside the L = 16 encoder; the oracle is pinned to it in
test_oracle_golden.py.
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def xq():
    import quantize
    return quantize


@pytest.mark.parametrize("K", (3, 4, 5))
def test_pack_roundtrip(xq, K):
    torch.manual_seed(0)
    L, T = 16, 256
    s = torch.randint(0, 1 << K, (7, T), dtype=torch.int64)
    for b in range(s.shape[0]):
        # a tail-bite consistent sequence: s_0's high L-K bits are s_last's
        # low bits (the reference's construction)
        cur = int(s[b, 0])
        seq = [cur]
        for t in range(1, T):
            cur = ((cur << K) | int(s[b, t] & ((1 << K) - 1))) & 0xFFFF
            seq.append(cur)
        s0 = ((seq[-1] & ((1 << (L - K)) - 1)) << K) | (seq[0] & ((1 << K) - 1))
        cur = s0
        seq = [s0]
        for t in range(1, T):
            cur = ((cur << K) | int(s[b, t] & ((1 << K) - 1))) & 0xFFFF
            seq.append(cur)
        s[b] = torch.tensor(seq, dtype=torch.int64)
    packed = xq.pack_states(s, K)
    assert packed.shape == (7, 16 * K) and packed.dtype == torch.int16
    assert torch.equal(xq.unpack_states(packed, K), s)


def test_tailbite_consistent(xq):
    torch.manual_seed(2)
    L, K, T = 16, 4, 256
    lut = xq.get_lut("exl3_mul1", L)
    X = torch.randn(T, 4)
    st = xq.quantize_seq_tailbite(X, lut, K, L)
    assert bool(((st[0] >> K) == (st[-1] & ((1 << (L - K)) - 1))).all())
    packed = xq.pack_states(st.t().contiguous(), K)
    assert torch.equal(xq.unpack_states(packed, K), st.t().contiguous())


@pytest.mark.parametrize("code", ("exl3_mul1", "exl3_3inst", "exl3_mcg"))
def test_gauss_mse(xq, code):
    torch.manual_seed(3)
    lut = xq.get_lut(code, 16)
    lut_rms = lut.double().square().mean().sqrt().float()
    for K in (2, 4):
        X = torch.randn(256, 2048)
        X = X / X.square().mean().sqrt() * lut_rms
        st = xq.quantize_seq_tailbite(X, lut, K, 16)
        dec = lut[st].t().contiguous().flatten()
        mse = (dec - X.t().reshape(-1)).square().mean() / X.square().mean()
        bound = 2.0 ** (-2 * K)
        assert float(mse) < 3.0 * bound, (code, K, float(mse), bound)


def test_ldlq_helps(xq):
    torch.manual_seed(4)
    k, n = 256, 256
    A = torch.randn(k, k)
    H = A.t() @ A / k + 0.1 * torch.eye(k)
    W = (torch.randn(n, k) @ torch.linalg.cholesky(torch.linalg.inv(H)).t()).t()
    res_l = xq.quantize_linear(W.t(), H, code="exl3_mul1", K=4, use_ldlq=True)
    res_p = xq.quantize_linear(W.t(), H, code="exl3_mul1", K=4, use_ldlq=False)
    e_l = xq.hessian_weighted_err(W.t(), res_l["W_hat"], H)
    e_p = xq.hessian_weighted_err(W.t(), res_p["W_hat"], H)
    assert e_l <= e_p * 1.001, (e_l, e_p)


@pytest.mark.parametrize("K", (2, 4))
def test_quantize_api(xq, K):
    torch.manual_seed(5)
    W = torch.randn(64, 128) * 0.03
    W_hat, packed, scale = xq.quantize(W, None, "exl3_mul1", K, seed=7)
    assert packed.shape == (128 // 16, 64 // 16, 16 * K)
    assert packed.dtype == torch.int16 and W_hat.shape == W.shape
    lut = xq.get_lut("exl3_mul1", 16)
    dec = xq.decode_trellis(packed, lut, K, 128, 64).t().contiguous() * scale
    assert torch.equal(dec, W_hat)
    _w2, p2, s2 = xq.quantize(W, None, "exl3_mul1", K, seed=7)
    assert torch.equal(p2, packed) and s2 == scale
    assert xq.rel_mse(W, W_hat) < 3.0 * 2.0 ** (-2 * K)
