"""Pin the CPU oracle against fixtures produced by the reference itself
(tests/golden/make_golden.py).  Integer/index outputs are compared bit for bit;
float linear algebra within fp32 tolerance."""
import hashlib
import itertools

import numpy as np
import pytest
import torch

from conftest import golden


def _sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def test_codebooks_and_perm(oracle):
    g = golden("codes")
    assert np.array_equal(oracle.code_lut("exl3_mul1"), g["mul1"])
    assert _sha(oracle.code_lut("exl3_3inst")) == str(g["sha_3inst"])
    assert _sha(oracle.code_lut("exl3_mcg")) == str(g["sha_mcg"])
    assert _sha(oracle.code_lut("qtip_1mad")) == str(g["sha_1mad"])
    assert np.array_equal(oracle.tensor_core_perm(), g["perm"])
    assert oracle.lut_rms(g["mul1"]) == g["lut_rms"]
    assert np.array_equal(oracle.sign_vec(1024, 20261011), g["sign_1024_20261011"])
    assert np.array_equal(oracle.sign_vec(256, 7), g["sign_256_7"])


def test_mul1_lut_depends_on_bytesum_only(oracle):
    # the mul1 value is a function of bytesum(s * 0x83DCD12D) alone
    lut = oracle.code_lut("exl3_mul1")
    s = np.arange(1 << 16, dtype=np.uint64)
    x = (s * np.uint64(0x83DCD12D)) & np.uint64(0xFFFFFFFF)
    bs = sum(((x >> np.uint64(8 * b)) & np.uint64(0xFF)) for b in range(4)).astype(np.int64)
    tab = np.full(1024, np.nan, np.float32)
    tab[bs] = lut
    assert np.array_equal(tab[bs], lut)


@pytest.mark.parametrize("K", range(2, 8))
def test_tailbite_matches_reference(oracle, mul1_lut, K):
    g = golden("viterbi")
    n_cases = 0
    for key in g.files:
        if not key.startswith("st_") or f"_K{K}_" not in key:
            continue
        _, tag, _, p, m = key.split("_")
        pv, mg = int(p[1:]), int(m[1:])
        X = g[f"X_{tag}"]
        st = oracle.tailbite(X, mul1_lut, K, pivot=pv, margin=mg, nthreads=4)
        assert np.array_equal(st.astype(np.uint16), g[key]), key
        n_cases += 1
    assert n_cases >= 8


@pytest.mark.parametrize("K", (2, 4, 7))
def test_plain_viterbi_overlap_backfrom(oracle, mul1_lut, K):
    g = golden("viterbi")
    X = g["X_gauss"][:4]
    assert np.array_equal(oracle.viterbi(X, mul1_lut, K).astype(np.uint16),
                          g[f"plain_K{K}"])
    st = oracle.viterbi(X, mul1_lut, K, overlap=g[f"overlap_in_K{K}"])
    assert np.array_equal(st.astype(np.uint16), g[f"overlap_K{K}"])
    bf = oracle.viterbi_back_from(X[:, :60], mul1_lut, K, 16, 40)
    assert np.array_equal(bf.astype(np.uint16), g[f"backfrom40_K{K}"])


def test_viterbi_bruteforce_known_answer(oracle):
    """test_quantize.py:111-138: tiny L=4 trellis against the reference's
    Viterbi output and against exhaustive search."""
    g = golden("bruteforce")
    lut, X = g["lut"], g["X"]               # X [T=6, B=3]
    L, K, T = 4, 2, 6
    st = oracle.viterbi(X.T.copy(), lut, K, L)        # [B, T]
    assert np.array_equal(st.T.astype(np.int64), g["states"])
    S = 1 << L
    best = np.full(3, np.inf)
    for s0 in range(S):
        for vs in itertools.product(range(1 << K), repeat=T - 1):
            seq = [s0]
            for v in vs:
                seq.append(((seq[-1] << K) | v) & (S - 1))
            c = ((lut[seq][:, None] - X) ** 2).sum(0)
            best = np.minimum(best, c)
    cv = ((lut[st.T] - X) ** 2).sum(0)
    assert np.abs(cv - best).max() < 1e-5


@pytest.mark.parametrize("K", range(2, 8))
def test_pack_unpack_decode(oracle, mul1_lut, K):
    g = golden("pack")
    st = g[f"states_K{K}"].astype(np.int64)
    packed = oracle.pack_states(st, K)
    assert np.array_equal(packed, g[f"packed_K{K}"])
    assert np.array_equal(oracle.unpack_states(packed, K), st)
    assert np.array_equal(oracle.unpack_states(g[f"rnd_trellis_K{K}"], K),
                          g[f"rnd_unpacked_K{K}"].astype(np.int64))
    w = oracle.decode_trellis(g[f"dec_trellis_K{K}"], mul1_lut, K, 32, 48)
    assert np.array_equal(w, g[f"dec_w_K{K}"])


def test_float_transforms(oracle):
    g = golden("transforms")
    h = oracle.hadamard128()
    W32 = np.ascontiguousarray(g["W"].T)
    Wi = oracle.to_inner(W32, g["suh"], g["svh"], h)
    np.testing.assert_allclose(Wi, g["W_inner"], rtol=0, atol=2e-7)
    np.testing.assert_allclose(oracle.from_inner(g["W_inner"], g["suh"], g["svh"], h),
                               g["W_back"], rtol=0, atol=2e-7)
    G = oracle.rotate_hessian(g["H"], g["suh"], h)
    scale = np.abs(g["G"]).max()
    np.testing.assert_allclose(G, g["G"], rtol=0, atol=2e-6 * scale)
    Gd = g["G"].copy()
    Gd[np.diag_indices_from(Gd)] += np.float32(0.01) * np.float32(np.mean(np.diagonal(Gd)))
    Lm, D = oracle.block_LDL(Gd, 16)
    np.testing.assert_allclose(Lm, g["Lfac"], rtol=0, atol=5e-5)
    np.testing.assert_allclose(D, g["D"], rtol=1e-4, atol=1e-4 * np.abs(g["D"]).max())


def test_prepare_incoherence(oracle):
    g = golden("transforms")
    pi = oracle.prepare_incoherence(g["W"], g["H"], channel_scales=True)
    np.testing.assert_allclose(pi["Wt"], g["pi_Wt"], rtol=1e-5, atol=1e-5)
    for kk in ("suh", "svh", "su_mag", "sv_mag"):
        np.testing.assert_allclose(pi[kk], g[f"pi_{kk}"], rtol=1e-5, atol=1e-7)
    assert np.array_equal(pi["zero_out"], g["pi_zero_out"])
    pi0 = oracle.prepare_incoherence(g["W"], None, channel_scales=False)
    np.testing.assert_allclose(pi0["Wt"], g["pi0_Wt"], rtol=0, atol=2e-7)


def test_quantize_linear_c1(oracle):
    """Config 1 (256x256 N(0,1) seed 0, H = I, K=4): the sweep with an
    identity Hessian carries no feedback, so the trellis is reproduced bit for
    bit whenever the fp32 rotation lands on the same W_inner bits."""
    g = golden("e2e")
    W1 = torch.randn(256, 256, generator=torch.Generator().manual_seed(0)).numpy()
    r = oracle.quantize_linear(W1, None, K=4, nthreads=8)
    assert np.array_equal(r["suh"], g["c1_suh"]) and np.array_equal(r["svh"], g["c1_svh"])
    assert abs(r["Wscale"] - float(g["c1_Wscale"])) <= 1e-6 * float(g["c1_Wscale"])
    same = (r["trellis"] == g["c1_trellis"]).all(-1)
    assert same.mean() >= 0.99, same.mean()
    mse = oracle.rel_mse(W1, r["W_hat"])
    assert abs(mse - float(g["c1_rel_mse"])) <= 1e-5 * float(g["c1_rel_mse"])


def test_quantize_api_c1(oracle, mul1_lut):
    g = golden("e2e")
    W1 = torch.randn(256, 256, generator=torch.Generator().manual_seed(0)).numpy()
    W_hat, packed, scale = oracle.quantize(W1, None, "exl3_mul1", 4, seed=0, nthreads=8)
    assert np.float32(scale) == g["q_scale"]
    assert np.array_equal(packed, g["q_packed"])
    assert hashlib.sha256(W_hat.tobytes()).hexdigest() == str(g["q_W_hat_sha"])


@pytest.mark.parametrize("K", (2, 4))
def test_quantize_linear_ldlq(oracle, K):
    """LDLQ path: float feedback differs from the reference's BLAS only in
    summation order, so the trellis agrees on (nearly) every tile and the
    Hessian-weighted error within 1e-4 relative."""
    g = golden("e2e")
    W, H = g["ldlq_W"], g["ldlq_H"]
    r = oracle.quantize_linear(W, H, K=K, nthreads=8)
    assert abs(r["Wscale"] - float(g[f"ldlq_K{K}_Wscale"])) <= 1e-5 * float(g[f"ldlq_K{K}_Wscale"])
    herr = oracle.hessian_weighted_err(W, r["W_hat"], H)
    ref = float(g[f"ldlq_K{K}_herr"])
    assert abs(herr - ref) <= 1e-4 * ref, (herr, ref)
    same = (r["trellis"] == g[f"ldlq_K{K}_trellis"]).all(-1).mean()
    assert same >= 0.95, same


def test_ldlq_block_targets_match_the_sweep(oracle, mul1_lut):
    """The fp64 LDLQ targets (quantize.py:676-686, used to check the GPU
    sweep's feedback) agree with the oracle sweep's own fp32 targets, given
    the same finished rows, to fp32 rounding of the sum of |terms|."""
    rng = np.random.default_rng(0)
    k, n = 192, 64
    A = rng.standard_normal((k, k))
    G = (A.T @ A / k + 0.1 * np.eye(k)).astype(np.float32)
    G[np.diag_indices_from(G)] += np.float32(0.01) * np.mean(np.diag(G))
    L, _ = oracle.block_LDL(G, 16)
    L = L.astype(np.float32)
    Wq = rng.standard_normal((k, n)).astype(np.float32)
    seen = {}
    hat, _ = oracle.ldlq_viterbi(Wq, L, mul1_lut, 3, nthreads=8,
                                 on_launch=lambda i, X, s: seen.__setitem__(i, X))
    for i in range(k // 16):
        Xr, Ab = oracle.ldlq_block_targets(Wq, L, hat, i)
        assert (np.abs(seen[i] - Xr) / Ab).max() <= 1e-5, i
