"""exl3_oracle -- CPU restatement of the reference EXL3 trellis quantizer.

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and the
``cpu_baseline`` / ``--impl reference`` legs of ``bench.py`` may import this
module, and only as the checker or the timed CPU baseline; the product path
(``exl3xpu-mixedk_b200``) never imports it and fails loudly when its CUDA
library is missing.

It restates, function by function, SergiioB/exl3xpu-mixedk
``quantize/quantize.py`` (line numbers cited per function) in numpy for the
integer/byte work and float linear algebra, and in plain C
(``viterbi_oracle.c``, built into ``_build/libexl3oracle.so``) for the Viterbi
dynamic program.  Its outputs are pinned against the fixtures in
``tests/golden/``, which were produced by running the reference itself
(``tests/golden/make_golden.py``).

Float linear algebra (Hadamard products, Cholesky, GEMMs) runs through numpy's
BLAS/LAPACK, whose summation order differs from the reference's torch CPU
kernels: those results match within float tolerance, not bit for bit.  The
Viterbi, codebooks, permutation and bit packing are bit-exact.
"""
from __future__ import annotations

import ctypes
import math
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

MUL1_MULT = 0x83DCD12D


# ------------------------------------------------------------------ codebooks
def _f16_from_bits(u):
    return np.asarray(u, dtype=np.uint64).astype(np.uint16).view(np.float16)


def code_lut(name: str, L: int = 16) -> np.ndarray:
    """fp32 [2^L] decode table (quantize.py:56-97 _local_code_lut/get_lut)."""
    s = np.arange(1 << L, dtype=np.uint64)
    if name in ("exl3_3inst", "exl3_mcg"):
        if name == "exl3_3inst":
            x = (s * np.uint64(89226354) + np.uint64(64248484)) & np.uint64(0xFFFFFFFF)
        else:
            x = (s * np.uint64(0xCBAC1FED)) & np.uint64(0xFFFFFFFF)
        x = (x & np.uint64(0x8FFF8FFF)) ^ np.uint64(0x3B603B60)
        lo = _f16_from_bits(x & np.uint64(0xFFFF)).astype(np.float64)
        hi = _f16_from_bits(x >> np.uint64(16)).astype(np.float64)
        return (lo + hi).astype(np.float16).astype(np.float32)
    if name == "exl3_mul1":
        x = (s * np.uint64(MUL1_MULT)) & np.uint64(0xFFFFFFFF)
        m = np.uint64(0xFF)
        bsum = ((x & m) + ((x >> np.uint64(8)) & m) + ((x >> np.uint64(16)) & m)
                + ((x >> np.uint64(24)) & m))
        h = (1024 + bsum).astype(np.float64)
        inv = float(_f16_from_bits(np.array([0x1EEE]))[0])
        bias = float(_f16_from_bits(np.array([0xC931]))[0])
        return (h * inv + bias).astype(np.float16).astype(np.float32)
    if name == "qtip_1mad":
        x = (s * np.uint64(34038481) + np.uint64(76625530)) & np.uint64(0xFFFFFFFF)
        m = np.uint64(255)
        y = ((x & m) + ((x >> np.uint64(8)) & m) + ((x >> np.uint64(16)) & m)
             + ((x >> np.uint64(24)) & m)).astype(np.float64)
        return ((y - 510.0) / 147.800537109375).astype(np.float32)
    raise KeyError(f"unknown code {name!r}")


def lut_rms(lut: np.ndarray) -> np.float32:
    """quantize.py:778: lut.double().square().mean().sqrt().float()."""
    return np.float32(math.sqrt(float(np.mean(lut.astype(np.float64) ** 2))))


def tensor_core_perm() -> np.ndarray:
    """quantize.py:101-118: sequence step t -> row-major 16x16 tile position."""
    perm = np.zeros(256, dtype=np.int64)
    for t in range(32):
        r0 = (t % 4) * 2
        c0 = t // 4
        rows = (r0, r0 + 1, r0 + 8, r0 + 9)
        for q in range(8):
            r = rows[q % 4]
            c = c0 if q < 4 else c0 + 8
            perm[t * 8 + q] = r * 16 + c
    return perm


def sign_vec(n: int, seed: int) -> np.ndarray:
    """quantize.py:179-182.  Rademacher signs from torch's CPU generator: the
    reference's sign vectors ARE torch.rand draws, so the oracle uses the same
    generator to reproduce them."""
    import torch
    g = torch.Generator().manual_seed(seed)
    return np.where(torch.rand(n, generator=g).numpy() < 0.5, -1.0, 1.0) \
        .astype(np.float32)


# ------------------------------------------------------------------ Hadamard
def hadamard128() -> np.ndarray:
    """quantize.py:125-132: normalised Sylvester H_128 built in fp64 -> fp32."""
    h = np.ones((1, 1), dtype=np.float64)
    while h.shape[0] < 128:
        h = np.block([[h, h], [h, -h]])
    return (h / math.sqrt(128)).astype(np.float32)


def had_left(w: np.ndarray, h: np.ndarray) -> np.ndarray:
    """quantize.py:135-139: H_blk @ w on the first (k) dim of [k, n]."""
    k, n = w.shape
    return np.matmul(h, w.reshape(k // 128, 128, n)).reshape(k, n)


def had_right(w: np.ndarray, h: np.ndarray) -> np.ndarray:
    """quantize.py:142-146: w @ H_blk on the last (n) dim of [k, n]."""
    k, n = w.shape
    return np.matmul(w.reshape(k, n // 128, 128), h).reshape(k, n)


def to_inner(w_orig, suh, svh, h):
    """quantize.py:149-155."""
    w = w_orig / suh.astype(np.float32)[:, None]
    w = w / svh.astype(np.float32)[None, :]
    return had_right(had_left(w, h), h)


def from_inner(w_inner, suh, svh, h):
    """quantize.py:158-164."""
    w = had_left(w_inner, h)
    w = w * suh.astype(np.float32)[:, None]
    w = had_right(w, h)
    return w * svh.astype(np.float32)[None, :]


def rotate_hessian(H_x, suh, h):
    """quantize.py:167-176: G = B diag(suh) H diag(suh) B."""
    k = H_x.shape[0]
    s = suh.astype(np.float32)
    a = H_x.astype(np.float32) * s[None, :] * s[:, None]
    return had_right(np.ascontiguousarray(had_right(a.reshape(k, k), h).T), h)


# ------------------------------------------------------------------ block LDL
def block_LDL(H: np.ndarray, b: int = 16):
    """quantize.py:419-437 (QTIP block LDL): L with identity bxb diagonal
    blocks, D block-diagonal.  Raises np.linalg.LinAlgError if not SPD."""
    n = H.shape[0]
    m = n // b
    Lm = np.linalg.cholesky(H)
    DL = np.stack([Lm[i * b:(i + 1) * b, i * b:(i + 1) * b] for i in range(m)])
    D = DL @ np.transpose(DL, (0, 2, 1))
    DLi = np.linalg.inv(DL)
    Lm = Lm.reshape(n, m, b).copy()
    for i in range(m):
        Lm[:, i, :] = Lm[:, i, :] @ DLi[i]
    Lm = Lm.reshape(n, n)
    for i in range(m):
        Lm[i * b:(i + 1) * b, i * b:(i + 1) * b] = np.eye(b, dtype=Lm.dtype)
    return Lm, D


# ------------------------------------------------------------------ Viterbi (C)
def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "_build", "libexl3oracle.so")
        if not os.path.exists(path):
            import subprocess
            subprocess.run(["make", "-s", "-C", _HERE], check=True)
        lib = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I = ctypes.c_int
        lib.oracle_tailbite.argtypes = [P, I, I, P, I, I, I, I, I, P]
        lib.oracle_tailbite.restype = I
        lib.oracle_viterbi.argtypes = [P, I, I, P, I, I, P, P]
        lib.oracle_viterbi.restype = I
        lib.oracle_viterbi_back_from.argtypes = [P, I, I, P, I, I, I, P]
        lib.oracle_viterbi_back_from.restype = I
        _LIB = lib
    return _LIB


def _ptr(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def tailbite(X: np.ndarray, lut: np.ndarray, K: int, L: int = 16,
             pivot: int | None = None, margin: int = 0,
             nthreads: int = 1) -> np.ndarray:
    """quantize_seq_tailbite (quantize.py:323-354), V=1.
    X [nseq, T] fp32 (one sequence per row) -> states [nseq, T] int32."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    nseq, T = X.shape
    if pivot is None:
        pivot = T // 2
    lut = np.ascontiguousarray(lut, dtype=np.float32)
    assert lut.shape == (1 << L,)
    out = np.empty((nseq, T), dtype=np.int32)
    rc = _lib().oracle_tailbite(_ptr(X), nseq, T, _ptr(lut), K, L, int(pivot),
                                int(margin), int(nthreads), _ptr(out))
    if rc:
        raise RuntimeError(f"oracle_tailbite rc={rc}")
    return out


def viterbi(X: np.ndarray, lut: np.ndarray, K: int, L: int = 16,
            overlap: np.ndarray | None = None) -> np.ndarray:
    """viterbi (quantize.py:218-320), V=1, full traceback.
    X [nseq, T] -> states [nseq, T] int32."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    nseq, T = X.shape
    lut = np.ascontiguousarray(lut, dtype=np.float32)
    ov = None
    if overlap is not None:
        ov = np.ascontiguousarray(overlap, dtype=np.int64)
    out = np.empty((nseq, T), dtype=np.int32)
    rc = _lib().oracle_viterbi(_ptr(X), nseq, T, _ptr(lut), K, L,
                               _ptr(ov) if ov is not None else None, _ptr(out))
    if rc:
        raise RuntimeError(f"oracle_viterbi rc={rc}")
    return out


def viterbi_back_from(X, lut, K, L, back_from):
    """viterbi(..., back_from=bf) (quantize.py:305-312) -> state at step bf."""
    X = np.ascontiguousarray(X, dtype=np.float32)
    nseq, T = X.shape
    lut = np.ascontiguousarray(lut, dtype=np.float32)
    out = np.empty(nseq, dtype=np.int64)
    rc = _lib().oracle_viterbi_back_from(_ptr(X), nseq, T, _ptr(lut), K, L,
                                         int(back_from), _ptr(out))
    if rc:
        raise RuntimeError(f"oracle_viterbi_back_from rc={rc}")
    return out


# ------------------------------------------------------------------ bitstream
def pack_states(states: np.ndarray, K: int) -> np.ndarray:
    """quantize.py:360-378: low K bits of state_t at stream bits [tK, tK+K),
    MSB first; u32 words MSB first, stored as int16 pairs low half first.
    states [nt, 256] -> int16 [nt, 16K]."""
    st = np.asarray(states, dtype=np.int64)
    nt, T = st.shape
    v = (st & ((1 << K) - 1))[..., None] >> np.arange(K - 1, -1, -1)
    stream = (v & 1).reshape(nt, T * K).astype(np.uint64)
    w32 = (stream.reshape(nt, -1, 32)
           << np.arange(31, -1, -1, dtype=np.uint64)).sum(-1).astype(np.uint64)
    lo = (w32 & np.uint64(0xFFFF)).astype(np.uint16).view(np.int16)
    hi = (w32 >> np.uint64(16)).astype(np.uint16).view(np.int16)
    return np.stack([lo, hi], axis=-1).reshape(nt, 16 * K)


def unpack_states(trellis: np.ndarray, K: int) -> np.ndarray:
    """quantize.py:381-402: state t = 16-bit circular window ending at bit
    (t+1)K.  int16 [..., 16K] -> int64 [..., 256]."""
    tr = np.asarray(trellis)
    nbits = 256 * K
    t = np.arange(256)
    b0 = (t * K + K - 16 + nbits) % nbits
    pos = (b0[:, None] + np.arange(16)[None, :]) % nbits
    flat = tr.reshape(-1, 16 * K).astype(np.int64) & 0xFFFF
    words = flat[:, 0::2] | (flat[:, 1::2] << 16)
    bits = ((words[..., None] >> np.arange(31, -1, -1)) & 1).reshape(flat.shape[0], -1)
    wts = 1 << np.arange(15, -1, -1)
    out = (bits[:, pos] * wts).sum(-1)
    return out.reshape(*tr.shape[:-1], 256)


def decode_trellis(trellis: np.ndarray, lut: np.ndarray, K: int, k: int,
                   n: int) -> np.ndarray:
    """quantize.py:405-415: int16 [k/16, n/16, 16K] -> W_inner fp32 [k, n]."""
    tk, tn, _ = trellis.shape
    perm = tensor_core_perm()
    st = unpack_states(trellis.reshape(tk * tn, 16 * K), K)
    vals = lut.astype(np.float32)[st].reshape(st.shape[0], -1)
    tiles = np.empty_like(vals)
    tiles[:, perm] = vals
    return tiles.reshape(tk, tn, 16, 16).transpose(0, 2, 1, 3).reshape(k, n)


# ------------------------------------------------------------------ LDLQ sweep
def ldlq_viterbi_steps(Wq: np.ndarray, Lfac: np.ndarray | None, lut: np.ndarray,
                       K: int, L: int = 16, buf_cols: int = 128,
                       pivot: int | None = None, margin: int = 0,
                       nthreads: int = 1, on_launch=None):
    """Generator form of quantize.py:631-746: yields the k-block index after
    each block (right to left), finally returns (hatW [k, n] fp32,
    states int64 [k/16, n/16, 256]) as the StopIteration value.  Each block
    is one launch of the reference's sweep (tn tiles)."""
    k, n = Wq.shape
    perm = tensor_core_perm()
    kp, np_ = perm // 16, perm % 16
    no_ldlq = Lfac is None or not np.any(Lfac)
    tk, tn = k // 16, n // 16
    W_t = np.ascontiguousarray(Wq.T)
    hatW_t = np.zeros_like(W_t)
    prod = np.zeros((k, n), dtype=np.float32)
    states = np.empty((tn, tk, 256), dtype=np.int64)
    buf_tiles = max(1, buf_cols // 16)
    for cur in range(tk, 0, -buf_tiles):
        lo = max(0, cur - buf_tiles)
        for i in range(cur - 1, lo - 1, -1):
            c0, c1 = 16 * i, 16 * (i + 1)
            WXWX = np.ascontiguousarray(W_t[:, c0:c1].T)
            if not no_ldlq:
                later0 = 16 * (i + 1)
                if later0 < 16 * cur:
                    WXWX = WXWX + Lfac[later0:16 * cur, c0:c1].T @ \
                        (W_t[:, later0:16 * cur] - hatW_t[:, later0:16 * cur]).T
                WXWX = WXWX + prod[c0:c1, :]
            X = WXWX[kp].reshape(256, tn, 16)[np.arange(256), :, np_]  # [256, tn]
            Xs = np.ascontiguousarray(X.T.astype(np.float32))          # [tn, 256]
            st = tailbite(Xs, lut, K, L, pivot=pivot, margin=margin,
                          nthreads=nthreads).astype(np.int64)
            if on_launch is not None:
                on_launch(i, Xs, st)
            states[:, i] = st
            vals = lut.astype(np.float32)[st]                         # [tn, 256]
            tiles = np.empty_like(vals)
            tiles[:, perm] = vals
            hatW_t[:, c0:c1] = tiles.reshape(tn, 16, 16).transpose(1, 0, 2) \
                .reshape(16, n).T
            yield i
        if not no_ldlq and lo > 0:
            prod += Lfac[16 * lo:16 * cur, :].T @ \
                (W_t[:, 16 * lo:16 * cur] - hatW_t[:, 16 * lo:16 * cur]).T
    return np.ascontiguousarray(hatW_t.T), np.ascontiguousarray(
        states.transpose(1, 0, 2))


def ldlq_block_targets(Wq: np.ndarray, Lfac: np.ndarray, hatW: np.ndarray, i: int,
                       E: np.ndarray | None = None):
    """The encoder targets of k-block i of an LDLQ sweep, in fp64, given the
    sweep's finished rows below it (quantize.py:676-686): every buffering of
    the reference (intra-buffer term plus the cached `prod` of earlier
    buffers, :680-682 and :742-744) sums the same terms,
        WXWX_i = Wq[16i:16i+16] + Lfac[16(i+1):, 16i:16i+16]^T (Wq - hatW)[16(i+1):],
    only in another fp32 order.  Returns (X [tn, 256] fp64 in sequence order
    x[t] = WXWX[perm[t]], A [tn, 256] fp64: the same sum over absolute
    values, which bounds the fp32 rounding of any summation order).  E, if
    given, is the fp32 Wq - hatW (the reference's error term, :681), computed
    once by a caller that checks several blocks."""
    k, n = Wq.shape
    perm = tensor_core_perm()
    kp, np_ = perm // 16, perm % 16
    tn = n // 16
    r0, r1 = 16 * i, 16 * (i + 1)
    Lb = Lfac[r1:, r0:r1].astype(np.float64)                 # [later, 16]
    if E is None:
        E = Wq - hatW
    E = E[r1:].astype(np.float64)
    W = Wq[r0:r1].astype(np.float64)
    WX = W + Lb.T @ E
    A = np.abs(W) + np.abs(Lb).T @ np.abs(E)

    def gather(M):
        return np.ascontiguousarray(M[kp].reshape(256, tn, 16)[np.arange(256), :, np_].T)
    return gather(WX), gather(A)


def ldlq_viterbi(Wq: np.ndarray, Lfac: np.ndarray | None, lut: np.ndarray,
                 K: int, L: int = 16, buf_cols: int = 128,
                 pivot: int | None = None, margin: int = 0,
                 nthreads: int = 1, on_launch=None):
    """quantize.py:631-746 BlockLDLQ sweep (right to left over 16-row k-blocks,
    128-row buffers).  Wq [k, n] fp32 -> (hatW [k, n] fp32,
    states int64 [k/16, n/16, 256]).  on_launch(i, X[tn, 256], states) is
    called per k-block (the per-launch hook of quantize.py:687-717)."""
    gen = ldlq_viterbi_steps(Wq, Lfac, lut, K, L, buf_cols, pivot, margin,
                             nthreads, on_launch)
    while True:
        try:
            next(gen)
        except StopIteration as e:
            return e.value


# ------------------------------------------------------------------ top level
def quantize_linear(W, H_x, code="exl3_mul1", K=4, percdamp=0.01,
                    su_seed=20261011, buf_cols=128, use_ldlq=True, margin=0,
                    nthreads=1):
    """quantize.py:750-875 (channel_scales=False).  W [out, in] -> dict."""
    W = np.asarray(W, dtype=np.float32)
    m_out, k_in = W.shape
    lut = code_lut(code)
    lrms = lut_rms(lut)
    suh = sign_vec(k_in, su_seed).astype(np.float16)
    svh = sign_vec(m_out, su_seed + 1).astype(np.float16)
    h = hadamard128()
    W32 = np.ascontiguousarray(W.T)
    W_i = to_inner(W32, suh, svh, h)
    Wscale = np.float32(np.sqrt(np.float32(np.mean(W_i.astype(np.float64) ** 2)))) / lrms
    Wscale = np.float32(Wscale)
    Wq = (W_i / Wscale).astype(np.float32)
    Lfac = None
    if use_ldlq and H_x is not None:
        G = rotate_hessian(np.asarray(H_x, np.float32), suh, h)
        dead = np.diagonal(G) == 0
        if dead.any():
            idx = np.nonzero(dead)[0]
            G[idx, idx] = 1.0
        damp = np.float32(percdamp) * np.float32(np.mean(np.diagonal(G)))
        G[np.diag_indices_from(G)] += damp
        Lfac, _ = block_LDL(G.astype(np.float32), 16)
        Lfac = Lfac.astype(np.float32)
    hatWq, states = ldlq_viterbi(Wq, Lfac, lut, K, buf_cols=buf_cols,
                                 margin=margin, nthreads=nthreads)
    trellis = pack_states(states.reshape(-1, 256), K).reshape(
        k_in // 16, m_out // 16, 16 * K)
    W_hat = np.ascontiguousarray(from_inner(hatWq * Wscale, suh, svh, h).T)
    return {"W_hat": W_hat, "trellis": trellis, "suh": suh, "svh": svh,
            "Wscale": float(Wscale), "lut_rms": float(lrms), "K": K,
            "states": states, "hatWq": hatWq}


def quantize(W_transformed, U_upper, code, K, seed, margin=16, nthreads=1):
    """quantize.py:894-966 (no su_mag/sv_mag).  -> (W_hat, packed, scale)."""
    Wt = np.asarray(W_transformed, dtype=np.float32)
    m_out, k_in = Wt.shape
    lut = code_lut(code)
    lrms = lut_rms(lut)
    Wq = np.ascontiguousarray(Wt.T)
    scale = np.float32(np.float32(np.sqrt(np.mean(Wq.astype(np.float64) ** 2))) / lrms)
    Wq = (Wq / scale).astype(np.float32)
    Lfac = None
    if U_upper is not None:
        Uu = np.asarray(U_upper, dtype=np.float64)
        Ui = np.linalg.inv(Uu)            # solve_triangular(U, I) = U^-1
        Lfac, _ = block_LDL(Ui @ Ui.T, 16)
        Lfac = Lfac.astype(np.float32)
    pivot = int(seed) % 256
    hatWq, states = ldlq_viterbi(Wq, Lfac, lut, K, pivot=pivot, margin=margin,
                                 nthreads=nthreads)
    packed = pack_states(states.reshape(-1, 256), K).reshape(
        k_in // 16, m_out // 16, 16 * K)
    W_hat = np.ascontiguousarray((hatWq * scale).T)
    return W_hat, packed, float(scale)


def prepare_incoherence(W, H_x=None, su_seed=20261011, channel_scales=True):
    """quantize.py:969-1058 (signs from sign_vec)."""
    W = np.asarray(W, dtype=np.float32)
    m_out, k_in = W.shape
    h = hadamard128()
    su_s = sign_vec(k_in, su_seed).astype(np.float16)
    sv_s = sign_vec(m_out, su_seed + 1).astype(np.float16)
    W32 = np.ascontiguousarray(W.T)
    if channel_scales:
        su, sv = su_s.astype(np.float32), sv_s.astype(np.float32)
        sv_mag = np.sqrt(np.mean(W32.astype(np.float32) ** 2, axis=0)).astype(np.float32)
        rm = np.float32(sv_mag.mean())
        if rm > 1e-30:
            sv_mag = sv_mag / rm
        zero_out = np.abs(sv_mag) < 1e-30
        sv_mag = np.where(zero_out, np.float32(0.1), sv_mag).astype(np.float32)
        w = W32 / (sv * sv_mag)[None, :]
        w = had_right(w, h)
        su_mag = np.sqrt(np.mean(w ** 2, axis=1)).astype(np.float32)
        su_mag = np.where(np.abs(su_mag) < 1e-30, np.float32(0.1), su_mag)
        w = w / (su * su_mag)[:, None]
        W_i = had_left(w, h)
        suh = su * su_mag
        svh = sv * np.where(zero_out, np.float32(0.0), sv_mag)
    else:
        W_i = to_inner(W32, su_s, sv_s, h)
        suh, svh = su_s.astype(np.float32), sv_s.astype(np.float32)
        su_mag = np.ones(k_in, np.float32)
        sv_mag = np.ones(m_out, np.float32)
        zero_out = np.zeros(m_out, bool)
    G = None
    if H_x is not None:
        G = rotate_hessian(np.asarray(H_x, np.float32), su_s, h)
    return {"Wt": np.ascontiguousarray(W_i.T), "G": G, "suh": suh, "svh": svh,
            "su_mag": su_mag, "sv_mag": sv_mag, "zero_out": zero_out}


def rel_mse(W, W_hat) -> float:
    """quantize.py:888-890."""
    d = np.asarray(W_hat, np.float64) - np.asarray(W, np.float64)
    return float((d ** 2).sum() / (np.asarray(W, np.float64) ** 2).sum())


def hessian_weighted_err(W, W_hat, H_x) -> float:
    """quantize.py:878-885: tr(dW H dW^T) / tr(W H W^T)."""
    dW = np.asarray(W_hat, np.float64) - np.asarray(W, np.float64)
    H = np.asarray(H_x, np.float64)
    Wd = np.asarray(W, np.float64)
    return float(np.einsum("ij,jk,ik->", dW, H, dW)
                 / np.einsum("ij,jk,ik->", Wd, H, Wd))
