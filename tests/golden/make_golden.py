#!/usr/bin/env python3
"""Generate the golden fixtures in this directory by running the REFERENCE
quantizer (SergiioB/exl3xpu-mixedk, quantize/quantize.py) on seeded inputs.

This script is the only file in the repository that imports the reference,
and it only runs in a checkout where the reference tree is present
(``--ref`` points at its ``quantize/`` directory).  The fixtures it writes are
small ``.npz`` files that the CPU and GPU tests read; nothing at test time
needs the reference itself.

Usage:
    PYTHONDONTWRITEBYTECODE=1 python tests/golden/make_golden.py --ref <ref>/quantize

Every fixture records which reference function produced it
(quantize.py line numbers in the docstrings of the helpers below).
"""
from __future__ import annotations

import argparse
import hashlib
import os
import sys
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True,
                    help="path of the reference's quantize/ directory")
    ap.add_argument("--out", default=HERE)
    args = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, args.ref)
    import quantize as xq  # the reference module (read-only import)

    torch.set_num_threads(max(1, os.cpu_count() or 1))
    out = args.out
    t_all = time.time()

    # ---------------------------------------------------------------- codes
    # quantize.py:56-97 _local_code_lut / get_lut; :101-118 tensor_core_perm
    luts = {}
    for code in ("exl3_mul1", "exl3_3inst", "exl3_mcg", "qtip_1mad"):
        luts[code] = xq.get_lut(code, 16).numpy().astype(np.float32)
    np.savez_compressed(
        os.path.join(out, "codes.npz"),
        mul1=luts["exl3_mul1"],
        sha_3inst=np.array(_sha(luts["exl3_3inst"])),
        sha_mcg=np.array(_sha(luts["exl3_mcg"])),
        sha_1mad=np.array(_sha(luts["qtip_1mad"])),
        perm=xq.tensor_core_perm().numpy().astype(np.int64),
        lut_rms=np.float32(float(
            torch.from_numpy(luts["exl3_mul1"]).double().square().mean()
            .sqrt().float())),
        sign_1024_20261011=xq.sign_vec(1024, 20261011).numpy(),
        sign_256_7=xq.sign_vec(256, 7).numpy(),
    )
    print("codes.npz", flush=True)

    # --------------------------------------------------------------- viterbi
    # quantize.py:218-320 viterbi, :323-354 quantize_seq_tailbite (emit "sq")
    lut = torch.from_numpy(luts["exl3_mul1"])
    nseq = 6
    combos = [(128, 0), (0, 16), (77, 16), (250, 16), (5, 0), (200, 40)]
    vit = {}
    rng = np.random.default_rng(12345)
    Xg = rng.standard_normal((nseq, 256), dtype=np.float32)   # verify_viterbi style
    # tie-heavy targets: exact LUT values, so many edges cost exactly 0
    Xt = luts["exl3_mul1"][rng.integers(0, 65536, size=(nseq, 256))]
    Xt[:, ::3] = Xt[:, 0:1]
    # wide targets: large costs
    Xw = (rng.standard_normal((nseq, 256)) * 7.0).astype(np.float32)
    vit["X_gauss"], vit["X_ties"], vit["X_wide"] = Xg, Xt, Xw
    for K in range(2, 8):
        for (pv, mg) in combos:
            for tag, X in (("gauss", Xg), ("ties", Xt), ("wide", Xw)):
                if tag != "gauss" and (pv, mg) not in ((128, 0), (0, 16)):
                    continue
                t0 = time.time()
                st = xq.quantize_seq_tailbite(
                    torch.from_numpy(X.T.copy()), lut, K, 16, pivot=pv,
                    margin=mg, emit_mode="sq")
                vit[f"st_{tag}_K{K}_p{pv}_m{mg}"] = \
                    st.t().contiguous().numpy().astype(np.uint16)
                print(f"  viterbi K={K} pivot={pv} margin={mg} {tag} "
                      f"{time.time() - t0:.1f}s", flush=True)
    # single-pass Viterbi (no tail-biting) with and without overlap/back_from
    for K in (2, 4, 7):
        Xs = torch.from_numpy(Xg[:4].T.copy())
        vit[f"plain_K{K}"] = xq.viterbi(Xs, lut, K, 16).t().numpy() \
            .astype(np.uint16)
        ov = torch.tensor([3, 100, 2000 % (1 << (16 - K)), 0])
        vit[f"overlap_K{K}"] = xq.viterbi(Xs, lut, K, 16, overlap=ov) \
            .t().numpy().astype(np.uint16)
        vit[f"overlap_in_K{K}"] = ov.numpy()
        vit[f"backfrom40_K{K}"] = xq.viterbi(Xs[:60], lut, K, 16,
                                             back_from=40).numpy() \
            .astype(np.uint16)
    np.savez_compressed(os.path.join(out, "viterbi.npz"), **vit)
    print("viterbi.npz", flush=True)

    # ------------------------------------------------- brute force (tiny L)
    # test_quantize.py:111-138 (L=4, K=2, T=6, torch.manual_seed(1))
    torch.manual_seed(1)
    L, K, T = 4, 2, 6
    blut = torch.randn(1 << L)
    bX = torch.randn(T, 3)
    bst = xq.viterbi(bX, blut, K, L, overlap=None)
    np.savez_compressed(os.path.join(out, "bruteforce.npz"),
                        lut=blut.numpy(), X=bX.numpy(), states=bst.numpy())
    print("bruteforce.npz", flush=True)

    # ----------------------------------------------------- pack / unpack
    # quantize.py:360-415 pack_states / unpack_states / decode_trellis
    pk = {}
    g = torch.Generator().manual_seed(3)
    for K in range(2, 8):
        # circularly consistent sequences, built like test_quantize.py:73-98
        s = torch.randint(0, 1 << K, (5, 256), dtype=torch.int64, generator=g)
        seqs = []
        for b in range(s.shape[0]):
            s_last = 0
            cur = int(s[b, 0])
            for t in range(1, 256):
                cur = ((cur << K) | int(s[b, t])) & 0xFFFF
            s_last = cur
            s0 = ((s_last & ((1 << (16 - K)) - 1)) << K) | int(s[b, 0])
            cur = s0
            seq = [s0]
            for t in range(1, 256):
                cur = ((cur << K) | int(s[b, t])) & 0xFFFF
                seq.append(cur)
            seqs.append(seq)
        st = torch.tensor(seqs, dtype=torch.int64)
        packed = xq.pack_states(st, K)
        pk[f"states_K{K}"] = st.numpy().astype(np.uint16)
        pk[f"packed_K{K}"] = packed.numpy()
        rnd = torch.randint(-32768, 32768, (3, 16 * K), dtype=torch.int64,
                            generator=g).to(torch.int16)
        pk[f"rnd_trellis_K{K}"] = rnd.numpy()
        pk[f"rnd_unpacked_K{K}"] = xq.unpack_states(rnd, K).numpy() \
            .astype(np.uint16)
        tr = torch.randint(-32768, 32768, (2, 3, 16 * K), dtype=torch.int64,
                           generator=g).to(torch.int16)
        pk[f"dec_trellis_K{K}"] = tr.numpy()
        pk[f"dec_w_K{K}"] = xq.decode_trellis(tr, lut, K, 32, 48).numpy()
    np.savez_compressed(os.path.join(out, "pack.npz"), **pk)
    print("pack.npz", flush=True)

    # ------------------------------------------------ float transforms
    # quantize.py:125-176 hadamard/to_inner/from_inner/rotate_hessian,
    # :419-437 block_LDL, :969-1058 prepare_incoherence
    tf = {}
    g = torch.Generator().manual_seed(11)
    W = torch.randn(128, 256, generator=g) * 0.02        # [out, in]
    W[5, :] = 0.0                                        # one dead out channel
    A = torch.randn(512, 256, generator=g)
    A = A * torch.exp(torch.randn(256, generator=g)).unsqueeze(0)
    H = (A.t() @ A) / 512
    suh = xq.sign_vec(256, 20261011).half()
    svh = xq.sign_vec(128, 20261012).half()
    h = xq.hadamard128()
    W32 = W.t().contiguous()
    Wi = xq.to_inner(W32, suh, svh, h)
    tf.update(W=W.numpy(), H=H.numpy(), suh=suh.numpy(), svh=svh.numpy(),
              W_inner=Wi.numpy(),
              W_back=xq.from_inner(Wi, suh, svh, h).numpy(),
              G=xq.rotate_hessian(H, suh, h).numpy())
    Gd = xq.rotate_hessian(H, suh, h)
    Gd.diagonal().add_(0.01 * Gd.diagonal().mean())
    Lm, D = xq.block_LDL(Gd.clone(), 16)
    tf.update(Lfac=Lm.numpy(), D=D.numpy())
    pi = xq.prepare_incoherence(W, H, channel_scales=True)
    for kk in ("Wt", "suh", "svh", "su_mag", "sv_mag", "zero_out"):
        tf[f"pi_{kk}"] = pi[kk].numpy()
    pi0 = xq.prepare_incoherence(W, H, channel_scales=False)
    tf["pi0_Wt"] = pi0["Wt"].numpy()
    np.savez_compressed(os.path.join(out, "transforms.npz"), **tf)
    print("transforms.npz", flush=True)

    # ------------------------------------------------ end-to-end APIs
    # quantize.py:750-875 quantize_linear, :894-966 quantize
    e2e = {}
    W1 = torch.randn(256, 256, generator=torch.Generator().manual_seed(0))
    t0 = time.time()
    r = xq.quantize_linear(W1, torch.eye(256), code="exl3_mul1", K=4)
    print(f"  C1 quantize_linear {time.time() - t0:.1f}s", flush=True)
    e2e.update(c1_trellis=r["trellis"].numpy(),
               c1_W_hat_sha=np.array(_sha(r["W_hat"].numpy())),
               c1_suh=r["suh"].numpy(),
               c1_svh=r["svh"].numpy(), c1_Wscale=np.float32(r["Wscale"]),
               c1_rel_mse=np.float64(xq.rel_mse(W1, r["W_hat"])))
    t0 = time.time()
    Wh, packed, scale = xq.quantize(W1, None, "exl3_mul1", 4, seed=0)
    print(f"  C1 quantize() {time.time() - t0:.1f}s", flush=True)
    e2e.update(q_packed=packed.numpy(),
               q_W_hat_sha=np.array(_sha(Wh.numpy())),
               q_scale=np.float32(scale),
               q_rel_mse=np.float64(xq.rel_mse(W1, Wh)))
    # LDLQ on a Hessian-correlated problem (test_quantize.py:205-219 recipe)
    torch.manual_seed(4)
    k, n = 256, 128
    A = torch.randn(k, k)
    H4 = A.t() @ A / k + 0.1 * torch.eye(k)
    W4 = (torch.randn(n, k) @ torch.linalg.cholesky(torch.linalg.inv(H4)).t()).t()
    for K in (2, 4):
        t0 = time.time()
        rl = xq.quantize_linear(W4.t(), H4, code="exl3_mul1", K=K,
                                use_ldlq=True)
        print(f"  ldlq K={K} {time.time() - t0:.1f}s", flush=True)
        e2e[f"ldlq_K{K}_trellis"] = rl["trellis"].numpy()
        e2e[f"ldlq_K{K}_Wscale"] = np.float32(rl["Wscale"])
        e2e[f"ldlq_K{K}_herr"] = np.float64(
            xq.hessian_weighted_err(W4.t(), rl["W_hat"], H4))
        e2e[f"ldlq_K{K}_rel_mse"] = np.float64(xq.rel_mse(W4.t(), rl["W_hat"]))
    e2e.update(ldlq_W=W4.t().contiguous().numpy(), ldlq_H=H4.numpy())
    # quantize() with a U factor (harness convention U^T U = G^-1)
    G4 = H4.double()
    U4 = torch.linalg.cholesky(torch.cholesky_inverse(
        torch.linalg.cholesky(G4)), upper=True).float()
    Wt4 = W4.t().contiguous() * 0.05          # [out=128, in=256]
    t0 = time.time()
    WhU, pU, sU = xq.quantize(Wt4, U4, "exl3_mul1", 5, seed=3, margin=16)
    print(f"  quantize(U) {time.time() - t0:.1f}s", flush=True)
    e2e.update(qu_U=U4.numpy(), qu_packed=pU.numpy(),
               qu_scale=np.float32(sU),
               qu_rel_mse=np.float64(xq.rel_mse(Wt4, WhU)))
    np.savez_compressed(os.path.join(out, "e2e.npz"), **e2e)
    print(f"e2e.npz  (total {time.time() - t_all:.0f}s)", flush=True)


if __name__ == "__main__":
    main()
