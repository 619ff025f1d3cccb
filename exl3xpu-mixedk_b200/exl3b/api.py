"""Reference-compatible quantizer API on the B200 CUDA path.

Mirrors SergiioB/exl3xpu-mixedk ``quantize/quantize.py`` (names, argument
meaning, return structures, error behaviour) so that a caller of the
reference's quantize step can switch to this module:

    quantize_linear    quantize.py:750-875
    quantize           quantize.py:894-966
    prepare_incoherence quantize.py:969-1058
    ldlq_viterbi       quantize.py:631-746
    quantize_seq_tailbite / viterbi / pack_states / unpack_states /
    decode_trellis / block_LDL / to_inner / from_inner / rotate_hessian /
    had_left / had_right / get_lut / CODES / tensor_core_perm / sign_vec /
    hadamard128 / rel_mse / hessian_weighted_err

Like the reference, quantize_linear and quantize check every tensor they
encode before returning it (quantize.py:849-853, :958-963): the packed
trellis, decoded on device, must reproduce the encoder's output, or
RuntimeError is raised.

Every numerical step runs in hand-written CUDA kernels behind the C ABI of
``libexl3b200.so``; torch provides device memory, streams and host<->device
copies only.  There is no CPU fallback: the backends "cuda" (default) and
"esimd" (the reference's name for its native encoder, mapped to the same
CUDA path) are accepted; "torch" and "dual" -- the reference's CPU path and
its cross-check -- are not part of this package.

Outputs are returned on the caller's device choice: like the reference,
``quantize_linear`` returns CPU tensors; ``out_device="cuda"`` keeps them on
the GPU.  Codes: the V=1 EXL3 tables "exl3_mul1" (default), "exl3_3inst",
"exl3_mcg" (decode values exact in fp16), K = 2..7, L = 16.
"""
from __future__ import annotations

import math
import time

import torch

from . import native, ops
from .native import Exl3bError, call, lib

STEPS = 256
L_BITS = 16
DTYPE_IDS = {torch.float32: 0, torch.bfloat16: 1, torch.float16: 2}
_LUT_CACHE: dict = {}
_H128: dict = {}


# ------------------------------------------------------------------ helpers
def _check_backend(backend: str):
    if backend not in ("cuda", "esimd"):
        raise ValueError(
            f"backend={backend!r}: this package runs the CUDA encoder "
            "(backend='cuda'; 'esimd' is accepted as an alias)")


def _check_code(code: str, L: int = 16, V: int = 1):
    if L != L_BITS:
        raise ValueError(f"L={L}: the CUDA encoder implements the 16-bit trellis")
    if V not in (0, 1):
        raise ValueError(f"V={V}: only V=1 codes have a CUDA encoder")
    ops.code_id(code)


def _check_K(K: int):
    if not 2 <= int(K) <= 7:
        raise ValueError(f"K={K} outside 2..7")


def _cuda_device(device) -> torch.device:
    """The reference defaults to device='cpu'; the computation here always
    runs on a CUDA device: 'cpu' / None select the current one."""
    if device is None:
        return torch.device("cuda", torch.cuda.current_device())
    d = torch.device(device)
    if d.type != "cuda":
        return torch.device("cuda", torch.cuda.current_device())
    return d if d.index is not None else torch.device("cuda", torch.cuda.current_device())


def _ptr(t):
    return 0 if t is None else t.data_ptr()


def _stream(dev: torch.device) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def _out(t: torch.Tensor, od: torch.device) -> torch.Tensor:
    """Result tensor on the output device.  Device -> host copies go into pinned
    memory asynchronously on the current stream; the caller synchronises once
    (_out_done) before handing the results out."""
    if od.type == "cpu" and t.is_cuda:
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t, non_blocking=True)
        return h
    return t.to(od)


def _out_done(dev: torch.device, od: torch.device):
    if od.type == "cpu":
        torch.cuda.current_stream(dev).synchronize()


def _select(dev: torch.device):
    call("exl3b_device_init", dev.index)


# ------------------------------------------------------------------ codes
def get_lut(code: str, L: int = 16, device=None) -> torch.Tensor:
    """fp32 [2^L] decode table (quantize.py:90-97), built by the library's
    host code (no GPU needed)."""
    _check_code(code, L)
    if code not in _LUT_CACHE:
        out = torch.empty(1 << L, dtype=torch.float32)
        call("exl3b_code_lut", ops.code_id(code), out.data_ptr())
        _LUT_CACHE[code] = out
    lut = _LUT_CACHE[code].clone()
    return lut.to(device) if device is not None else lut


def _code_decoder(code: str):
    def decode(states: torch.Tensor) -> torch.Tensor:
        lut = get_lut(code)
        return lut.to(states.device)[states.long() & 0xFFFF]
    return decode


# The reference's optional code registry (quantize.py:44-49: name ->
# (decode_fn, metadata)), filled here with the V=1 codes this package encodes:
# decode_fn maps int states to their fp32 decode values.
CODES = {name: (_code_decoder(name), {"V": 1, "L": 16, "code_id": cid})
         for name, cid in native.CODE_IDS.items()}


def _lut_rms(lut: torch.Tensor) -> torch.Tensor:
    return lut.double().square().mean().sqrt().float()      # quantize.py:778


def _code_of_lut(lut: torch.Tensor) -> str:
    l = lut.detach().float().cpu().reshape(-1)
    for c in native.CODE_IDS:
        if l.numel() == 65536 and torch.equal(l, get_lut(c)):
            return c
    raise ValueError("lut is not one of the EXL3 V=1 tables with a CUDA encoder "
                     f"({sorted(native.CODE_IDS)})")


def tensor_core_perm() -> torch.Tensor:
    """quantize.py:101-118: sequence step t -> row-major 16x16 tile position."""
    perm = [0] * 256
    for t in range(32):
        r0, c0 = (t % 4) * 2, t // 4
        rows = (r0, r0 + 1, r0 + 8, r0 + 9)
        for q in range(8):
            perm[t * 8 + q] = rows[q % 4] * 16 + (c0 if q < 4 else c0 + 8)
    return torch.tensor(perm, dtype=torch.long)


def sign_vec(n: int, seed: int, device=None) -> torch.Tensor:
    """quantize.py:179-182: Rademacher signs from torch's CPU generator (the
    reference's bits are torch.rand draws, so the same generator is used)."""
    g = torch.Generator().manual_seed(seed)
    return torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0).to(device)


def hadamard128(device=None, dtype=torch.float32) -> torch.Tensor:
    """quantize.py:125-132 (the explicit matrix, for callers that want it;
    the kernels use butterflies)."""
    key = (str(device), dtype)
    if key not in _H128:
        h = torch.ones((1, 1), dtype=torch.float64)
        while h.shape[0] < 128:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        _H128[key] = (h / math.sqrt(128)).to(dtype=dtype, device=device)
    return _H128[key]


# ------------------------------------------------------------------ incoherence
def _check_h(h):
    """The reference passes the normalised block-128 Hadamard matrix around;
    the kernels use butterflies, so any other matrix is refused."""
    if h is None:
        return
    hc = h.detach().float().cpu()
    if hc.shape != (128, 128) or not torch.equal(hc, hadamard128()):
        raise ValueError("h must be hadamard128(): the CUDA transforms implement the "
                         "normalised block-128 Sylvester Hadamard")


def _had_axis(w: torch.Tensor, h, axis: int) -> torch.Tensor:
    _check_h(h)
    dev = _cuda_device(w.device)
    _select(dev)
    X = w.detach().to(dev, torch.float32).contiguous()
    Y = torch.empty_like(X)
    call("exl3b_hadamard_axis", X.data_ptr(), X.shape[0], X.shape[1], axis, Y.data_ptr(),
         _stream(dev))
    return Y.to(w.device)


def had_left(w: torch.Tensor, h=None) -> torch.Tensor:
    """quantize.py:135-139: block-128 Hadamard on the first (k) dim of
    w [k, n] (k % 128 == 0), fp32, on the CUDA device; result on w's device."""
    if w.dim() != 2 or w.shape[0] % 128:
        raise ValueError(f"had_left: w {tuple(w.shape)} needs k % 128 == 0")
    return _had_axis(w, h, 0)


def had_right(w: torch.Tensor, h=None) -> torch.Tensor:
    """quantize.py:142-146: block-128 Hadamard on the last (n) dim of
    w [k, n] (n % 128 == 0)."""
    if w.dim() != 2 or w.shape[1] % 128:
        raise ValueError(f"had_right: w {tuple(w.shape)} needs n % 128 == 0")
    return _had_axis(w, h, 1)


def to_inner(w_orig: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
             h=None, device=None) -> torch.Tensor:
    """quantize.py:149-155: W_orig [k,n] -> B diag(1/suh) W diag(1/svh) B.
    Returns fp32 on the CUDA device."""
    dev = _cuda_device(device if device is not None else w_orig.device)
    k, n = w_orig.shape
    _select(dev)
    Wt = w_orig.t().contiguous().to(dev)           # [n][k] == W [out, in]
    if Wt.dtype not in DTYPE_IDS:
        Wt = Wt.float()
    ri = (1.0 / suh.float()).to(dev).contiguous()
    ci = (1.0 / svh.float()).to(dev).contiguous()
    Wi = torch.empty(k, n, dtype=torch.float32, device=dev)
    call("exl3b_incoherence_fwd", Wt.data_ptr(), DTYPE_IDS[Wt.dtype], n, k,
         ri.data_ptr(), ci.data_ptr(), Wi.data_ptr(), None, _stream(dev))
    return Wi


def from_inner(w_inner: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor,
               h=None, device=None) -> torch.Tensor:
    """quantize.py:158-164: W_inner [k,n] -> diag(suh) B W_i B diag(svh)
    (returned [k, n] like the reference)."""
    dev = _cuda_device(device if device is not None else w_inner.device)
    k, n = w_inner.shape
    _select(dev)
    Wi = w_inner.float().contiguous().to(dev)
    su = suh.float().to(dev).contiguous()
    sv = svh.float().to(dev).contiguous()
    out = torch.empty(n, k, dtype=torch.float32, device=dev)
    call("exl3b_incoherence_inv", Wi.data_ptr(), k, n, None, su.data_ptr(),
         sv.data_ptr(), out.data_ptr(), _stream(dev))
    return out.t()


def rotate_hessian(H_x: torch.Tensor, suh: torch.Tensor, h=None, device=None) -> torch.Tensor:
    """quantize.py:167-176: G = B diag(suh) H diag(suh) B (fp32, CUDA)."""
    dev = _cuda_device(device if device is not None else H_x.device)
    k = H_x.shape[0]
    _select(dev)
    Hd = H_x.float().contiguous().to(dev, non_blocking=True)
    su = suh.float().to(dev).contiguous()
    G = torch.empty(k, k, dtype=torch.float32, device=dev)
    call("exl3b_rotate_hessian", Hd.data_ptr(), k, su.data_ptr(), G.data_ptr(), _stream(dev))
    return G


# ------------------------------------------------------------------ block LDL
def _block_ldl_dev(A: torch.Tensor, want_D: bool = False):
    """Factor A (fp32 or fp64 CUDA, destroyed) -> (Lfac fp32, D or None).
    Raises Exl3bError with rc NOT_SPD (9) if A is not positive definite."""
    dev = A.device
    k = A.shape[0]
    f64 = 1 if A.dtype == torch.float64 else 0
    Lfac = torch.empty(k, k, dtype=torch.float32, device=dev)
    D = torch.empty(k // 16, 16, 16, dtype=A.dtype, device=dev) if want_D else None
    wsb = lib().exl3b_block_ldl_workspace_bytes(k, f64)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    call("exl3b_block_ldl", A.data_ptr(), k, f64, Lfac.data_ptr(), _ptr(D),
         ws.data_ptr(), wsb, _stream(dev))
    return Lfac, D


def block_LDL(H: torch.Tensor, b: int = 16):
    """quantize.py:419-437.  H -> (L, D); L has identity 16x16 diagonal
    blocks.  H's precision (fp32 / fp64) is the factorisation precision; L is
    returned in H's dtype and device.  Raises RuntimeError if H is not SPD
    (like torch.linalg.cholesky)."""
    if b != 16:
        raise ValueError("block_LDL: the CUDA factorisation uses b = 16")
    dev = _cuda_device(H.device)
    _select(dev)
    A = H.detach().to(dev).contiguous().clone()
    if A.dtype not in (torch.float32, torch.float64):
        A = A.float()
    try:
        Lf, D = _block_ldl_dev(A, want_D=True)
    except Exl3bError as e:
        if e.rc == 9:
            raise RuntimeError(str(e)) from None
        raise
    return Lf.to(device=H.device, dtype=H.dtype if H.dtype.is_floating_point else torch.float32), \
        D.to(H.device)


def _damped_lfac(H_x: torch.Tensor, suh: torch.Tensor, percdamp: float,
                 dev: torch.device) -> torch.Tensor:
    """quantize.py:809-837: rotate, fix dead diagonal, damp, block-LDL in
    fp32; on failure escalate damping in fp64 (+0, +0.1, +1.0 x mean diag),
    raising if G is not finite."""
    k = H_x.shape[0]
    G = rotate_hessian(H_x, suh, device=dev)
    nonfinite = torch.zeros(1, dtype=torch.int32, device=dev)
    call("exl3b_damp_hessian", G.data_ptr(), k, float(percdamp), nonfinite.data_ptr(),
         _stream(dev))
    try:
        Lfac, _ = _block_ldl_dev(G.clone())
        return Lfac
    except Exl3bError as e:
        if e.rc != 9:
            raise
    if int(nonfinite.item()):
        raise RuntimeError("block_LDL: rotated Hessian is not finite")
    Gd = _f64(G)
    for extra in (0.0, 0.1, 1.0):
        if extra:
            _damp_f64(Gd, extra)
        try:
            Lfac, _ = _block_ldl_dev(Gd.clone())
            print(f"xtq_quant: block_LDL fallback used extra damping {extra} "
                  f"x mean diag", flush=True)
            return Lfac
        except Exl3bError as e:
            if e.rc != 9 or extra == 1.0:
                raise RuntimeError(str(e)) from None
    raise RuntimeError("unreachable")


def _f64(G: torch.Tensor) -> torch.Tensor:
    out = torch.empty(G.shape, dtype=torch.float64, device=G.device)
    call("exl3b_convert_f32_f64", G.data_ptr(), out.data_ptr(), G.numel(), _stream(G.device))
    return out


def _damp_f64(Gd: torch.Tensor, extra: float):
    call("exl3b_damp_hessian_f64", Gd.data_ptr(), Gd.shape[0], float(extra),
         _stream(Gd.device))


# ------------------------------------------------------------------ Viterbi
def _check_emit(dtype, emit_mode):
    if emit_mode != "sq":
        raise ValueError(f"emit_mode={emit_mode!r}: the CUDA encoder implements the "
                         "reference's fp32 'sq' emit (quantize.py:255-260)")
    if dtype not in (None, torch.float32):
        raise ValueError(f"dtype={dtype}: the CUDA encoder accumulates path costs in fp32")


def viterbi(X: torch.Tensor, lut: torch.Tensor, K: int, L: int = 16, V: int = 1,
            overlap: torch.Tensor | None = None, dtype: torch.dtype = torch.float32,
            back_from: int | None = None, compiled: bool = False,
            emit_mode: str = "sq"):
    """quantize.py:218-320: one trellis Viterbi pass on the CUDA encoder,
    bit-exact with the reference's fp32 "sq" emit.  X [T, B] (T <= 256) ->
    states int64 [T, B]; with `overlap` [B], s_0 >> K and s_{T-1} mod
    2^(16-K) are pinned to it; with `back_from`, returns only the state at
    step back_from ([B]).  Results on X's device."""
    _check_K(K)
    _check_emit(dtype, emit_mode)
    if V != 1 or L != L_BITS:
        raise ValueError("the CUDA encoder takes V=1, L=16 trellises")
    T, B = X.shape
    if not 1 <= T <= STEPS:
        raise ValueError(f"T={T}: one pass covers 1..{STEPS} steps")
    if back_from is not None and int(back_from) < 0:
        raise ValueError(f"back_from={back_from} must be >= 0")
    code = _code_of_lut(lut)
    dev = _cuda_device(X.device)
    _select(dev)
    Xs = X.detach().to(dev, torch.float32).t().contiguous()        # [B][T]
    ov = None
    if overlap is not None:
        ov_h = overlap.detach().reshape(-1).to("cpu", torch.int64)
        if ov_h.numel() != B:
            raise ValueError(f"overlap has {ov_h.numel()} entries for {B} sequences")
        if B and (int(ov_h.min()) < 0 or int(ov_h.max()) >= (1 << (16 - K))):
            raise ValueError(f"overlap values must lie in [0, 2^{16 - K})")
        ov = ov_h.to(torch.int32).to(dev)
    bf = -1 if back_from is None else int(back_from)
    out = torch.empty((B, T) if bf < 0 else (B,), dtype=torch.int32, device=dev)
    if B:
        wsb = lib().exl3b_viterbi_workspace_bytes(B, int(K))
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        call("exl3b_viterbi", Xs.data_ptr(), B, T, int(K), ops.code_id(code), _ptr(ov), bf,
             out.data_ptr(), ws.data_ptr(), wsb, _stream(dev))
    res = out.t() if bf < 0 else out
    return res.long().to(X.device)


def quantize_seq_tailbite(X: torch.Tensor, lut: torch.Tensor, K: int, L: int = 16,
                          V: int = 1, dtype: torch.dtype = torch.float32,
                          pivot: int | None = None, margin: int = 0,
                          compiled: bool = False, emit_mode: str = "sq"):
    """quantize.py:323-354 on the CUDA encoder.  X [T=256, B] -> states
    int64 [256, B] (on X's device), bit-exact with the reference's "sq" emit."""
    _check_K(K)
    _check_emit(dtype, emit_mode)
    T, B = X.shape
    if T != STEPS or V != 1 or L != L_BITS:
        raise ValueError("the CUDA encoder takes 256-step V=1 L=16 sequences")
    code = _code_of_lut(lut)
    pv = T // 2 if pivot is None else int(pivot)
    if not 0 <= pv < T:
        raise ValueError(f"pivot {pv} outside [0, {T})")
    dev = _cuda_device(X.device)
    Xs = X.detach().to(dev, torch.float32).t().contiguous()
    st = ops.tailbite(Xs, K, pivot=pv, margin=margin, code=code)
    return st.t().long().to(X.device)


# ------------------------------------------------------------------ bitstream
def pack_states(states: torch.Tensor, K: int, V: int = 1) -> torch.Tensor:
    """quantize.py:360-378: int [ntiles, 256] -> int16 [ntiles, 16K]."""
    if V != 1:
        raise ValueError("V=1 only")
    dev = _cuda_device(states.device)
    _select(dev)
    st = states.to(dev, torch.int32).contiguous()
    nt = st.shape[0]
    out = torch.empty(nt, 16 * K, dtype=torch.int16, device=dev)
    call("exl3b_pack_states", st.data_ptr(), nt, int(K), out.data_ptr(), _stream(dev))
    return out.to(states.device)


def unpack_states(trellis: torch.Tensor, K: int, V: int = 1) -> torch.Tensor:
    """quantize.py:381-402: int16 [..., 16K] -> int64 [..., 256]."""
    if V != 1:
        raise ValueError("V=1 only")
    dev = _cuda_device(trellis.device)
    _select(dev)
    tr = trellis.to(dev, torch.int16).reshape(-1, 16 * K).contiguous()
    nt = tr.shape[0]
    out = torch.empty(nt, 256, dtype=torch.int32, device=dev)
    call("exl3b_unpack_states", tr.data_ptr(), nt, int(K), out.data_ptr(), _stream(dev))
    return out.long().reshape(*trellis.shape[:-1], 256).to(trellis.device)


def decode_trellis(trellis: torch.Tensor, lut: torch.Tensor, K: int, k: int, n: int,
                   V: int = 1) -> torch.Tensor:
    """quantize.py:405-415: int16 [k/16, n/16, 16K] -> W_inner fp32 [k, n]."""
    code = _code_of_lut(lut)
    dev = _cuda_device(trellis.device)
    _select(dev)
    tk, tn, _ = trellis.shape
    tr = trellis.to(dev).contiguous()
    out = torch.empty(k, n, dtype=torch.float32, device=dev)
    call("exl3b_decode_trellis", tr.data_ptr(), tk, tn, int(K), ops.code_id(code),
         out.data_ptr(), _stream(dev))
    return out.to(trellis.device)


def _verify_async(trellis: torch.Tensor, hatW: torch.Tensor, K: int, code: str,
                  bad: torch.Tensor, states: torch.Tensor | None = None):
    """Queue the self-check of one encoded column segment (quantize.py:849-853,
    :958-963) on the current stream: every weight decoded from `trellis`
    [tk, tn, 16K] must equal `hatW` (a [k, 16 tn] view, row pitch
    hatW.stride(0)) and, with `states` ([tk, tn, 256] view), every unpacked
    state the encoder's.  Mismatches are added to the device int `bad`."""
    tk, tn, _ = trellis.shape
    dev = trellis.device
    st_ptr, ld_st = 0, 0
    if states is not None:
        st_ptr, ld_st = states.data_ptr(), states.stride(0) // 256
    call("exl3b_verify_trellis", trellis.data_ptr(), tk, tn, int(K), ops.code_id(code),
         hatW.data_ptr(), hatW.stride(0), st_ptr, ld_st, bad.data_ptr(), _stream(dev))


def _verify_raise(bad: torch.Tensor, what: str):
    n = int(bad.item())
    if n:
        raise RuntimeError(f"{what}: decode != encoder output ({n} weights or states "
                           "differ between the packed trellis and the encoder)")


def verify_trellis(trellis: torch.Tensor, hatW: torch.Tensor, K: int,
                   code: str = "exl3_mul1", states: torch.Tensor | None = None):
    """The reference's per-tensor self-check (quantize.py:849-853): the packed
    trellis [k/16, n/16, 16K] decodes to hatW [k, n] (inner domain, unit
    scale) bit for bit and, when given, unpacks to `states` [k/16, n/16, 256];
    raises RuntimeError otherwise.  Runs on the CUDA device."""
    dev = _cuda_device(trellis.device)
    _select(dev)
    tr = trellis.detach().to(dev, torch.int16).contiguous()
    hw = hatW.detach().to(dev, torch.float32).contiguous()
    tk, tn, w = tr.shape
    if w != 16 * K or hw.shape != (16 * tk, 16 * tn):
        raise ValueError(f"trellis {tuple(tr.shape)} / hatW {tuple(hw.shape)} / K={K}")
    st = None
    if states is not None:
        st = states.detach().to(dev, torch.int32).reshape(tk, tn, 256).contiguous()
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _verify_async(tr, hw, K, code, bad, st)
    _verify_raise(bad, "verify_trellis")


# ------------------------------------------------------------------ LDLQ
def _sweep(Wq: torch.Tensor, Lfac, Ks: list, widths: list, code: str, pivot: int,
           margin: int, buf_cols: int, progress=None, want_states=False, want_x=False):
    """Run the fused LDLQ sweep on device over column segments of Wq [k][n]
    (segment s: `widths[s]` columns at K = Ks[s]).  Returns (hatW, trellis
    list, states or None, X or None)."""
    import ctypes
    dev = Wq.device
    k, n = Wq.shape
    tk, tn = k // 16, n // 16
    c0 = [0]
    for w in widths:
        c0.append(c0[-1] + w // 16)
    assert c0[-1] == tn
    trellis = [torch.empty(tk, w // 16, 16 * K, dtype=torch.int16, device=dev)
               for w, K in zip(widths, Ks)]
    hatW = torch.empty(k, n, dtype=torch.float32, device=dev)
    states = torch.empty(tk, tn, 256, dtype=torch.int32, device=dev) if want_states else None
    X = torch.empty(tk, tn, 256, dtype=torch.float32, device=dev) if want_x else None
    wsb = lib().exl3b_ldlq_workspace_bytes(k, n, min(Ks), 1 if Lfac is not None else 0)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    nseg = len(Ks)
    seg_c0 = (ctypes.c_int * (nseg + 1))(*c0)
    seg_K = (ctypes.c_int * nseg)(*Ks)
    seg_tr = (ctypes.c_void_p * nseg)(*[t.data_ptr() for t in trellis])
    args = [Wq.data_ptr(), _ptr(Lfac), k, n, nseg, seg_c0, seg_K, seg_tr,
            ops.code_id(code), int(pivot), int(margin), int(buf_cols),
            hatW.data_ptr(), _ptr(states), _ptr(X)]
    s = _stream(dev)
    if progress is None:
        call("exl3b_ldlq_sweep", *args, 0, tk, ws.data_ptr(), wsb, s)
    else:
        step_i = 0
        for i in range(tk - 1, -1, -1):
            call("exl3b_ldlq_sweep", *args, i, i + 1, ws.data_ptr(), wsb, s)
            torch.cuda.current_stream(dev).synchronize()
            step_i += 2 * STEPS
            progress(i, step_i)
    return hatW, trellis, states, X


def ldlq_viterbi(Wq: torch.Tensor, Lfac: torch.Tensor | None, lut: torch.Tensor,
                 K: int, L: int = 16, buf_cols: int = 128, V: int = 1,
                 batch: int = 0, dtype: torch.dtype = torch.float32,
                 pivot: int | None = None, margin: int = 0,
                 compiled: bool = False, progress=None,
                 code: str | None = None, backend: str = "cuda"):
    """quantize.py:631-746.  Wq [k, n] -> (hatW [k, n] fp32,
    states int64 [k/16, n/16, 256]) on Wq's device."""
    _check_backend(backend)
    _check_K(K)
    if V != 1 or L != L_BITS:
        raise ValueError("V=1, L=16 only")
    code = code or _code_of_lut(lut)
    k, n = Wq.shape
    if k % 16 or n % 16:
        raise ValueError("k and n must be multiples of 16")
    dev = _cuda_device(Wq.device)
    _select(dev)
    Wd = Wq.detach().to(dev, torch.float32).contiguous()
    Ld = None
    if Lfac is not None and bool(Lfac.any()):
        Ld = Lfac.detach().to(dev, torch.float32).contiguous()
    pv = STEPS // 2 if pivot is None else int(pivot)
    hatW, _tr, st, _x = _sweep(Wd, Ld, [K], [n], code, pv, margin, buf_cols,
                               progress=progress, want_states=True)
    return hatW.to(Wq.device), st.long().to(Wq.device)


# ------------------------------------------------------------------ top level
def _rms_scale(parts: torch.Tensor, count: int, lut_rms: float, dev) -> torch.Tensor:
    tmp = torch.empty(1, dtype=torch.float64, device=dev)
    scale = torch.empty(1, dtype=torch.float32, device=dev)
    call("exl3b_rms_scale", parts.data_ptr(), parts.numel(), float(count), float(lut_rms),
         tmp.data_ptr(), scale.data_ptr(), _stream(dev))
    return scale


def _div(x: torch.Tensor, s: torch.Tensor) -> torch.Tensor:
    y = torch.empty_like(x)
    call("exl3b_div_scalar", x.data_ptr(), s.data_ptr(), y.data_ptr(), x.numel(),
         _stream(x.device))
    return y


def _encode_inner(W_dev: torch.Tensor, suh, svh, dev):
    """W [out, in] (CUDA, fp32/bf16/fp16) -> (W_i [k][n] fp32, per-block
    sums of squares)."""
    m_out, k_in = W_dev.shape
    ri = (1.0 / suh.float()).to(dev).contiguous()
    ci = (1.0 / svh.float()).to(dev).contiguous()
    Wi = torch.empty(k_in, m_out, dtype=torch.float32, device=dev)
    parts = torch.empty((k_in // 128) * (m_out // 128), dtype=torch.float64, device=dev)
    call("exl3b_incoherence_fwd", W_dev.data_ptr(), DTYPE_IDS[W_dev.dtype], m_out, k_in,
         ri.data_ptr(), ci.data_ptr(), Wi.data_ptr(), parts.data_ptr(), _stream(dev))
    return Wi, parts


def quantize_linear(W: torch.Tensor, H_x: torch.Tensor | None, code: str = "exl3_mul1",
                    K: int = 4, L: int = 16, V: int = 0, percdamp: float = 0.01,
                    su_seed: int = 20261011, buf_cols: int = 128,
                    use_ldlq: bool = True, device: str = "cpu",
                    batch: int = 0, dtype: torch.dtype = torch.float32,
                    margin: int = 0, compiled: bool = False, progress=None,
                    backend: str = "cuda", channel_scales: bool = False,
                    *, pivot: int | None = None, out_device="cpu",
                    keep_states: bool = False):
    """quantize.py:750-875: quantize one nn.Linear weight W [out, in] with
    input Gram H_x [in, in] (None -> plain trellis encode of the incoherent
    weight).  Returns the reference's dict; tensors on `out_device`
    (CPU by default, like the reference)."""
    return quantize_linear_fused(
        [W], H_x, code=code, Ks=[K], L=L, V=V, percdamp=percdamp, su_seed=su_seed,
        buf_cols=buf_cols, use_ldlq=use_ldlq, device=device, batch=batch, dtype=dtype,
        margin=margin, compiled=compiled, progress=progress, backend=backend,
        channel_scales=channel_scales, pivot=pivot, out_device=out_device,
        keep_states=keep_states)[0]


def quantize_linear_fused(Ws: list, H_x: torch.Tensor | None, code: str = "exl3_mul1",
                          Ks: list | None = None, L: int = 16, V: int = 0,
                          percdamp: float = 0.01, su_seed: int = 20261011,
                          buf_cols: int = 128, use_ldlq: bool = True, device: str = "cpu",
                          batch: int = 0, dtype: torch.dtype = torch.float32,
                          margin: int = 0, compiled: bool = False, progress=None,
                          backend: str = "cuda", channel_scales: bool = False,
                          *, pivot: int | None = None, out_device="cpu",
                          keep_states: bool = False) -> list:
    """Members of one fused module (e.g. q/k/v: W_j [out_j, in], one shared
    input Gram H_x) at per-member bit widths Ks[j] -- the mixed-K fused
    module of serve/patches/0002-vllm-plugin-mixed-k.patch.  Returns one
    quantize_linear dict per member, identical to quantize_linear(W_j, H_x,
    K=Ks[j], ...) called member by member: the members share su (same seed
    and k), hence the rotated Hessian and its block-LDL factor, which are
    computed once; the LDLQ feedback couples rows only (quantize.py:680-682,
    743-744), so one sweep over the members' columns side by side, each
    column segment at its own K, gives each member's own result."""
    _check_backend(backend)
    _check_code(code, L, V)
    if Ks is None:
        Ks = [4] * len(Ws)
    if len(Ks) != len(Ws) or not Ws:
        raise ValueError("need one K per member")
    for K in Ks:
        _check_K(K)
    k_in = Ws[0].shape[1]
    for W in Ws:
        assert W.shape[1] == k_in, "fused members share the input dimension"
        assert k_in % 128 == 0 and W.shape[0] % 128 == 0, (W.shape, "need k%128, n%128")
    dev = _cuda_device(device)
    _select(dev)
    lut = get_lut(code)
    lut_rms = _lut_rms(lut)
    suh = sign_vec(k_in, su_seed).half()

    members = []
    for W in Ws:
        m_out = W.shape[0]
        svh = sign_vec(m_out, su_seed + 1).half()
        W_dev = W.detach().to(dev, non_blocking=True)
        if W_dev.dtype not in DTYPE_IDS:
            W_dev = W_dev.float()
        W_dev = W_dev.contiguous()
        mem = {"m_out": m_out, "svh": svh}
        if channel_scales:
            from .incoherence import channel_scale_inner
            Wi, parts, mem["su_mag"], _sv_mag, mem["sv_store"] = channel_scale_inner(
                W_dev, suh, svh, dev)
        else:
            Wi, parts = _encode_inner(W_dev, suh, svh, dev)
        del W_dev
        mem["Wscale_d"] = _rms_scale(parts, Wi.numel(), float(lut_rms), dev)
        mem["Wq"] = _div(Wi, mem["Wscale_d"])
        del Wi
        members.append(mem)

    Lfac = None
    if use_ldlq and H_x is not None:
        t0 = time.time()
        Lfac = _damped_lfac(H_x, suh, percdamp, dev)
        if progress is not None:
            progress("hinv", time.time() - t0)

    widths = [m["m_out"] for m in members]
    if len(members) == 1:
        Wq = members[0].pop("Wq")
    else:
        Wq = torch.cat([m.pop("Wq") for m in members], dim=1)
    pv = STEPS // 2 if pivot is None else int(pivot)
    hatW, trl, st, _ = _sweep(Wq, Lfac, list(Ks), widths, code, pv, margin, buf_cols,
                              progress=progress, want_states=keep_states)
    del Wq, Lfac
    # self-check of every member (quantize.py:849-853), read at the sync below
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    c0 = 0
    for j, m in enumerate(members):
        w = m["m_out"]
        _verify_async(trl[j], hatW[:, c0:c0 + w], Ks[j], code, bad,
                      None if st is None else st[:, c0 // 16:(c0 + w) // 16])
        c0 += w

    od = torch.device(out_device) if out_device is not None else dev
    wscales = torch.cat([m["Wscale_d"] for m in members]).tolist()   # one host sync
    _verify_raise(bad, "quantize_linear")
    outs = []
    c0 = 0
    for j, mem in enumerate(members):
        m_out = mem["m_out"]
        hw = hatW if len(members) == 1 else hatW[:, c0:c0 + m_out].contiguous()
        su32 = suh.float().to(dev)
        sv32 = mem["svh"].float().to(dev)
        suh_j, svh_j = suh, mem["svh"]
        if channel_scales:
            from .incoherence import channel_scale_outer
            W_hat, suh_j, svh_j = channel_scale_outer(hw, suh, mem["svh"], mem["su_mag"],
                                                      mem["sv_store"], mem["Wscale_d"], dev)
        else:
            W_hat = torch.empty(m_out, k_in, dtype=torch.float32, device=dev)
            call("exl3b_incoherence_inv", hw.data_ptr(), k_in, m_out,
                 mem["Wscale_d"].data_ptr(), su32.data_ptr(), sv32.data_ptr(),
                 W_hat.data_ptr(), _stream(dev))
        out = {
            "W_hat": _out(W_hat, od),
            "trellis": _out(trl[j], od),
            "suh": _out(suh_j, od), "svh": _out(svh_j, od),
            "Wscale": float(wscales[j]), "lut_rms": float(lut_rms),
            "code": code, "K": int(Ks[j]), "L": L, "V": 1, "use_ldlq": use_ldlq,
            "channel_scales": channel_scales,
        }
        if keep_states:
            out["states"] = _out(st if len(members) == 1 else
                             st[:, c0 // 16:(c0 + m_out) // 16].contiguous(), od)
            out["hatWq"] = _out(hw, od)
        outs.append(out)
        c0 += m_out
    _out_done(dev, od)
    return outs


def hessian_weighted_err(W: torch.Tensor, W_hat: torch.Tensor, H_x: torch.Tensor) -> float:
    """quantize.py:878-885: tr(dW H dW^T) / tr(W H W^T) (diagnostic)."""
    dW = (W_hat - W).float()
    H = H_x.float().to(dW.device)
    num = torch.einsum("ij,jk,ik->", dW, H, dW)
    den = torch.einsum("ij,jk,ik->", W.float(), H, W.float())
    return float(num / den)


def rel_mse(W: torch.Tensor, W_hat: torch.Tensor) -> float:
    """quantize.py:888-890 (diagnostic)."""
    d = (W_hat.float() - W.float().to(W_hat.device))
    return float(d.square().sum() / W.float().to(W_hat.device).square().sum())


def quantize(W_transformed: torch.Tensor, U_upper: torch.Tensor | None,
             code: str, K: int, seed: int, L: int = 16,
             dtype: torch.dtype = torch.float32,
             backend: str = "cuda", margin: int = 16, batch: int = 0,
             su_mag: torch.Tensor | None = None,
             sv_mag: torch.Tensor | None = None, *, device=None):
    """quantize.py:894-966 harness entry point.  W_transformed [out, in] fp32
    (inner domain), U_upper [in, in] (U^T U = G^-1) or None ->
    (W_hat fp32 [out, in], packed int16 [in/16, out/16, 16K], scale float);
    tensors on W_transformed's device."""
    _check_backend(backend)
    _check_code(code, L)
    _check_K(K)
    m_out, k_in = W_transformed.shape
    assert k_in % 16 == 0 and m_out % 16 == 0, W_transformed.shape
    dev = _cuda_device(device if device is not None else W_transformed.device)
    _select(dev)
    s = _stream(dev)
    lut_rms = _lut_rms(get_lut(code))
    Wt = W_transformed.detach().to(dev, torch.float32).contiguous()
    su_m = sv_m = None
    if su_mag is not None or sv_mag is not None:
        su_m = (torch.ones(k_in) if su_mag is None else su_mag.float()).to(dev).contiguous()
        sv_m = (torch.ones(m_out) if sv_mag is None else sv_mag.float()).to(dev).contiguous()
    Wq0 = torch.empty(k_in, m_out, dtype=torch.float32, device=dev)
    parts = torch.empty(((m_out + 31) // 32) * ((k_in + 31) // 32), dtype=torch.float64,
                        device=dev)
    call("exl3b_transpose_scale", 0, Wt.data_ptr(), m_out, k_in, _ptr(sv_m), _ptr(su_m),
         None, Wq0.data_ptr(), parts.data_ptr(), s)
    scale = _rms_scale(parts, Wq0.numel(), float(lut_rms), dev)
    Wq = _div(Wq0, scale)
    del Wq0
    Lfac = None
    if U_upper is not None:
        Ud = U_upper.detach().to(dev, torch.float32).contiguous()
        G = torch.empty(k_in, k_in, dtype=torch.float64, device=dev)
        wsb = lib().exl3b_u_to_gram_workspace_bytes(k_in)
        ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
        call("exl3b_u_to_gram", Ud.data_ptr(), k_in, G.data_ptr(), ws.data_ptr(), wsb, s)
        del ws
        try:
            Lfac, _ = _block_ldl_dev(G)
        except Exl3bError as e:
            if e.rc == 9:
                raise RuntimeError(str(e)) from None
            raise
    pivot = int(seed) % STEPS
    hatW, trl, _st, _ = _sweep(Wq, Lfac, [K], [m_out], code, pivot, margin, 128)
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    _verify_async(trl[0], hatW, K, code, bad)          # quantize.py:958-963
    W_hat = torch.empty(m_out, k_in, dtype=torch.float32, device=dev)
    call("exl3b_transpose_scale", 1, hatW.data_ptr(), k_in, m_out, _ptr(sv_m), _ptr(su_m),
         scale.data_ptr(), W_hat.data_ptr(), None, s)
    od = W_transformed.device
    sc = float(scale.item())
    _verify_raise(bad, "quantize")
    W_hat, tr = _out(W_hat, od), _out(trl[0], od)
    _out_done(dev, od)
    return W_hat, tr, sc


def prepare_incoherence(W, H_x=None, su_seed=20261011, sv_seed=None, su_sign=None,
                        sv_sign=None, channel_scales=True, device="cpu"):
    """quantize.py:969-1058 (see exl3b.incoherence.prepare_incoherence)."""
    from .incoherence import prepare_incoherence as _pi
    return _pi(W, H_x, su_seed=su_seed, sv_seed=sv_seed, su_sign=su_sign,
               sv_sign=sv_sign, channel_scales=channel_scales, device=device)
