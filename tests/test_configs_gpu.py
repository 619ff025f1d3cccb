"""Parity on the benchmark configurations themselves,
at full size, with the reference's own method: the per-launch dual check of
quantize.py:687-717 (every tile of a sampled k-block, re-encoded by the CPU
oracle from the GPU's encoder targets, must give the GPU's states bit for
bit) plus a check of those targets -- the LDLQ feedback -- against the fp64
sum of the same terms (quantize.py:676-686), and the per-tensor transform and
scale against the oracle's transform of the same weight.

Sampled k-blocks: one per 512-row launch buffer of the sweep for config 2
(the first, middle or last block of the buffer in turn), a spread of blocks
for configs 3 and 4.  Tolerances: states bit-exact; targets within 1e-5 of
the sum of the terms' absolute values (fp32 summation-order rounding is
~1e-7 of it); W_inner within 2e-6 of its maximum; Wscale within 1e-6
relative; sign vectors exact.
"""
import os

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
NTH = max(1, min(64, os.cpu_count() or 1))
LAUNCH_BLOCKS = 32          # 512-row launch buffers of the sweep


def _prepare(Ws, H, Ks, dev):
    """The device pipeline of quantize_linear_fused up to the sweep (the
    library's kernels), returning what the sweep consumes."""
    from exl3b import api
    k = Ws[0].shape[1]
    suh = api.sign_vec(k, 20261011).half()
    Wq_parts, meta = [], []
    for W in Ws:
        svh = api.sign_vec(W.shape[0], 20261012).half()
        Wi, parts = api._encode_inner(W.to(dev).contiguous(), suh, svh, dev)
        lut_rms = api._lut_rms(api.get_lut("exl3_mul1"))
        sc = api._rms_scale(parts, Wi.numel(), float(lut_rms), dev)
        Wq_parts.append(api._div(Wi, sc))
        meta.append({"Wi": Wi, "scale": float(sc.item()), "svh": svh})
    Lfac = api._damped_lfac(H, suh, 0.01, dev)
    Wq = Wq_parts[0] if len(Ws) == 1 else torch.cat(Wq_parts, dim=1)
    widths = [W.shape[0] for W in Ws]
    hatW, trl, st, X = api._sweep(Wq, Lfac, list(Ks), widths, "exl3_mul1", 128, 0, 128,
                                  want_states=True, want_x=True)
    return suh, meta, Wq, Lfac, hatW, trl, st, X, widths


def _check_transform(oracle, W, suh, m):
    """W_inner and Wscale of one member against the oracle's transform."""
    W32 = W.float().cpu().numpy().T.copy()             # [k, n]
    svh = m["svh"].numpy()
    assert np.array_equal(svh, oracle.sign_vec(W.shape[0], 20261012).astype(np.float16))
    Wi_o = oracle.to_inner(W32, suh.numpy(), svh, oracle.hadamard128())
    Wi = m["Wi"].cpu().numpy()
    assert np.abs(Wi - Wi_o).max() <= 2e-6 * np.abs(Wi_o).max()
    lut = oracle.code_lut("exl3_mul1")
    sc_o = np.float32(np.sqrt(np.float32(np.mean(Wi_o.astype(np.float64) ** 2)))) \
        / oracle.lut_rms(lut)
    assert abs(m["scale"] - float(sc_o)) <= 1e-6 * float(sc_o), (m["scale"], sc_o)


def _check_blocks(oracle, blocks, segs, Wq, Lfac, hatW, st, X):
    """Per-launch dual check and feedback-target check of k-blocks `blocks`;
    segs: (first column tile, tiles, K) per column segment."""
    lut = oracle.code_lut("exl3_mul1")
    Wq_h, L_h, hat_h = Wq.cpu().numpy(), Lfac.cpu().numpy(), hatW.cpu().numpy()
    E = Wq_h - hat_h
    Xh, sth = X.cpu().numpy(), st.cpu().numpy()
    for i in blocks:
        Xr, A = oracle.ldlq_block_targets(Wq_h, L_h, hat_h, int(i), E)
        ratio = (np.abs(Xh[i].astype(np.float64) - Xr) / np.maximum(A, 1e-30)).max()
        assert ratio <= 1e-5, f"k-block {i}: targets off by {ratio:.3g} of |terms|"
        for c0, nt, K in segs:
            ref = oracle.tailbite(Xh[i, c0:c0 + nt], lut, K, pivot=128, margin=0,
                                  nthreads=NTH)
            bad = np.nonzero((ref != sth[i, c0:c0 + nt]).any(1))[0]
            assert bad.size == 0, f"k-block {i}, K={K}: {bad.size} tiles differ, first {bad[:5]}"


def _sampled(tk, per_buffer=True, extra=()):
    """One block per launch buffer (anchored at tk: first, middle, last in
    turn), or just the spread `extra`."""
    out = set(extra)
    if per_buffer:
        for b, cur in enumerate(range(tk, 0, -LAUNCH_BLOCKS)):
            lo = max(0, cur - LAUNCH_BLOCKS)
            out.add((cur - 1, (cur + lo) // 2, lo)[b % 3])
    return sorted(out)


def test_config2_parity():
    """Config 2: 5120 x 5120, K = 4, full LDLQ."""
    from exl3b import api, synth
    from oracle import exl3_oracle as oracle
    dev = torch.device("cuda", 0)
    W, H = synth.config2(device=dev)
    suh, meta, Wq, Lfac, hatW, trl, st, X, widths = _prepare([W], H, [4], dev)
    assert np.array_equal(suh.numpy(), oracle.sign_vec(5120, 20261011).astype(np.float16))
    _check_transform(oracle, W, suh, meta[0])
    tk = 5120 // 16
    _check_blocks(oracle, _sampled(tk), [(0, 320, 4)], Wq, Lfac, hatW, st, X)
    api.verify_trellis(trl[0], hatW, 4, states=st)
    # the public entry point composes the same kernels: identical trellis
    r = api.quantize_linear(W, H, K=4, out_device="cuda")
    assert torch.equal(r["trellis"], trl[0])
    assert r["Wscale"] == meta[0]["scale"]


def test_config3_parity():
    """Config 3: fused q/k/v (6144 | 1024 | 1024 outputs, K = 5, 7, 7), one
    shared Hessian: every segment of the sampled blocks at its own K."""
    from exl3b import api, synth
    from oracle import exl3_oracle as oracle
    dev = torch.device("cuda", 0)
    Ws, H, Ks = synth.config3(device=dev)
    suh, meta, Wq, Lfac, hatW, trl, st, X, widths = _prepare(Ws, H, Ks, dev)
    for W, m in zip(Ws, meta):
        _check_transform(oracle, W, suh, m)
    segs, c0 = [], 0
    for w, K in zip(widths, Ks):
        segs.append((c0, w // 16, K))
        c0 += w // 16
    _check_blocks(oracle, _sampled(320, per_buffer=False, extra=(319, 250, 161, 0)), segs,
                  Wq, Lfac, hatW, st, X)
    fused = api.quantize_linear_fused(Ws, H, Ks=Ks, out_device="cuda")
    for r, t in zip(fused, trl):
        assert torch.equal(r["trellis"], t)


@pytest.mark.parametrize("K", (2, 7))
def test_config4_parity(K):
    """Config 4: 17408 -> 5120 down projection at the K sweep's ends."""
    from exl3b import api, synth
    from oracle import exl3_oracle as oracle
    dev = torch.device("cuda", 0)
    W, H = synth.config4(device=dev)
    suh, meta, Wq, Lfac, hatW, trl, st, X, widths = _prepare([W], H, [K], dev)
    _check_transform(oracle, W, suh, meta[0])
    tk = 17408 // 16
    _check_blocks(oracle, _sampled(tk, per_buffer=False, extra=(tk - 1, tk - 17, 600, 545, 31, 0)),
                  [(0, 320, K)], Wq, Lfac, hatW, st, X)
    api.verify_trellis(trl[0], hatW, K, states=st)


def _check_sampled(oracle, blocks, segs, Wq, Lfac, hatW, st, X, per_seg=96):
    """_check_blocks on a spread of at most `per_seg` column tiles of every
    segment (wide fused modules: the oracle re-encodes a sample of each
    sampled k-block instead of all of its tiles; columns never interact, so
    the sampled columns' targets need only their own columns of Wq and W_hat)."""
    lut = oracle.code_lut("exl3_mul1")
    picks = [np.unique(np.linspace(c0, c0 + nt - 1, min(nt, per_seg)).astype(int))
             for c0, nt, _K in segs]
    tiles = np.concatenate(picks)
    cols = torch.from_numpy((tiles[:, None] * 16 + np.arange(16)[None, :]).reshape(-1))
    Wq_h = Wq[:, cols.to(Wq.device)].cpu().numpy()
    hat_h = hatW[:, cols.to(Wq.device)].cpu().numpy()
    L_h = Lfac.cpu().numpy()
    E = Wq_h - hat_h
    for i in blocks:
        Xr, A = oracle.ldlq_block_targets(Wq_h, L_h, hat_h, int(i), E)
        Xi = X[i][torch.from_numpy(tiles).to(X.device)].cpu().numpy()
        sti = st[i][torch.from_numpy(tiles).to(st.device)].cpu().numpy()
        ratio = (np.abs(Xi.astype(np.float64) - Xr) / np.maximum(A, 1e-30)).max()
        assert ratio <= 1e-5, f"k-block {i}: targets off by {ratio:.3g} of |terms|"
        o = 0
        for (c0, nt, K), pk in zip(segs, picks):
            sl = slice(o, o + pk.size)
            ref = oracle.tailbite(np.ascontiguousarray(Xi[sl]), lut, K, pivot=128, margin=0,
                                  nthreads=NTH)
            bad = np.nonzero((ref != sti[sl]).any(1))[0]
            assert bad.size == 0, f"k-block {i}, K={K}: {bad.size} tiles differ, first {pk[bad[:5]]}"
            o += pk.size


def test_config5_layer_parity(tmp_path):
    """Config 5, the 27B-shape mixed-K stack: layer 0 through the product
    driver (exl3b.stack: q/k/v at K = 5, 7, 7 on one Hessian, o at 6,
    gate/up at 5, 5, down at 4), written as EXL3 files.  Every group's
    sweep is rerun here with its encoder targets exposed: the stored
    trellises equal it bit for bit, and sampled k-blocks of every group
    (first, middle and last) re-encoded by the CPU oracle from those targets
    give the same states, at every member's K."""
    from exl3b import export, stack, synth
    from oracle import exl3_oracle as oracle
    dev = torch.device("cuda", 0)
    layer = 0
    stack.quantize_layer(layer, dev, out_root=tmp_path)
    for group, dim, members in synth.STACK_GROUPS:
        H = synth.hessian(dim, synth.stack_hessian_seed(layer, group), dev)
        Ws = [synth.stack_weight(layer, m, dev) for m in members]
        Ks = [synth.SC5_K[m] for m in members]
        suh, meta, Wq, Lfac, hatW, trl, st, X, widths = _prepare(Ws, H, Ks, dev)
        for m, W, mt, t in zip(members, Ws, meta, trl):
            f = export.load_quantized(tmp_path / "L00" /
                                      f"{stack.MODULE_NAMES[m]}.safetensors")
            assert torch.equal(f["trellis"], t.cpu()), (group, m)
        _check_transform(oracle, Ws[0], suh, meta[0])
        segs, c0 = [], 0
        for w, K in zip(widths, Ks):
            segs.append((c0, w // 16, K))
            c0 += w // 16
        tk = dim // 16
        _check_sampled(oracle, [tk - 1, tk // 2, 0], segs, Wq, Lfac, hatW, st, X)
        del H, Ws, Wq, Lfac, hatW, trl, st, X
        torch.cuda.empty_cache()
