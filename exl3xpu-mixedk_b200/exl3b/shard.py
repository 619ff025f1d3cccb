"""Output-column sharding of one projection across the ranks of a process
group (the "row-tile" unit of the multi-GPU plan: a range of output-column
tiles of one layer's inner weight).

Why columns split without any exchange during the sweep: the LDLQ feedback
couples rows of the inner weight only (quantize.py:680-682 and :742-744 index
rows of Lfac), and the block-128 Hadamard along the output axis is block
diagonal, so a 128-aligned output-channel range [n0, n1) depends only on
W[n0:n1, :], on the Hessian, and on the per-tensor scale.  Each rank

  1. transforms the whole W (a fraction of a millisecond) so that Wscale is
     the unsplit tensor's scale, computed in the same order;
  2. factors the Hessian itself (the same rotation, damping and block LDL on
     every rank: no broadcast, and the factorisation is on each rank's
     critical path either way);
  3. sweeps its own column range and checks it (decode == encoder output);
  4. reconstructs its W_hat rows.

The result of a rank is bit-identical to the same slice of the unsplit
quantize_linear (columns never interact; tested).  Finished tensors are then
all-gathered (NCCL for CUDA tensors) when the caller wants the whole layer:
the only collective, after the quantization.

What limits the split: a column's k-blocks are sequential (each needs the
finished blocks below it), so once a rank holds fewer column tiles than the
tile kernel keeps in flight (two per SM), the per-layer time approaches the
length of one column's chain of k-blocks instead of shrinking further.
"""
from __future__ import annotations

import torch

from . import api
from .native import call

ALIGN = 128


def column_ranges(n: int, world: int, align: int = ALIGN) -> list:
    """Contiguous [n0, n1) output-channel ranges, one per rank, aligned to
    `align` and as equal as the alignment allows (earlier ranks take the
    extra blocks)."""
    if world < 1 or n < 0 or n % align:
        raise ValueError(f"n={n} must be a multiple of {align}; world={world} >= 1")
    nb = n // align
    base, extra = divmod(nb, world)
    out, c = [], 0
    for r in range(world):
        w = (base + (1 if r < extra else 0)) * align
        out.append((c, c + w))
        c += w
    return out


def quantize_linear_columns(W: torch.Tensor, H_x: torch.Tensor | None, cols: tuple,
                            code: str = "exl3_mul1", K: int = 4, percdamp: float = 0.01,
                            su_seed: int = 20261011, buf_cols: int = 128,
                            use_ldlq: bool = True, device=None, margin: int = 0,
                            pivot: int | None = None, out_device=None,
                            Lfac: torch.Tensor | None = None) -> dict:
    """Output channels [n0, n1) of quantize_linear(W [out, in], H_x, ...):
    the same dict with W_hat [n1 - n0, in], trellis [in/16, (n1 - n0)/16, 16K]
    and svh [n1 - n0] restricted to the range (suh and Wscale are the whole
    tensor's), plus "cols": (n0, n1).  Bit-identical to that slice of the
    unsplit result.  Lfac: the damped block-LDL factor of H_x already
    computed by lfac() (members of one fused module share it); H_x is then
    not used."""
    api._check_code(code)
    api._check_K(K)
    m_out, k_in = W.shape
    n0, n1 = int(cols[0]), int(cols[1])
    if not (0 <= n0 < n1 <= m_out) or n0 % ALIGN or n1 % ALIGN or k_in % ALIGN:
        raise ValueError(f"columns [{n0}, {n1}) of W {tuple(W.shape)}: need 128-aligned "
                         "ranges inside the output dim and in % 128 == 0")
    dev = api._cuda_device(device if device is not None else W.device)
    api._select(dev)
    s = api._stream(dev)
    lut_rms = api._lut_rms(api.get_lut(code))
    suh = api.sign_vec(k_in, su_seed).half()
    svh = api.sign_vec(m_out, su_seed + 1).half()
    W_dev = W.detach().to(dev, non_blocking=True)
    if W_dev.dtype not in api.DTYPE_IDS:
        W_dev = W_dev.float()
    Wi, parts = api._encode_inner(W_dev.contiguous(), suh, svh, dev)
    del W_dev
    Wscale_d = api._rms_scale(parts, Wi.numel(), float(lut_rms), dev)
    Wq = api._div(Wi[:, n0:n1].contiguous(), Wscale_d)
    del Wi
    if not use_ldlq:
        Lfac = None
    elif Lfac is None and H_x is not None:
        Lfac = lfac(H_x, k_in, percdamp, su_seed, dev)
    pv = api.STEPS // 2 if pivot is None else int(pivot)
    w = n1 - n0
    hatW, trl, _st, _ = api._sweep(Wq, Lfac, [K], [w], code, pv, margin, buf_cols)
    del Wq, Lfac
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    api._verify_async(trl[0], hatW, K, code, bad)
    su32 = suh.float().to(dev)
    sv32 = svh[n0:n1].float().to(dev).contiguous()
    W_hat = torch.empty(w, k_in, dtype=torch.float32, device=dev)
    call("exl3b_incoherence_inv", hatW.data_ptr(), k_in, w, Wscale_d.data_ptr(),
         su32.data_ptr(), sv32.data_ptr(), W_hat.data_ptr(), s)
    od = torch.device(out_device) if out_device is not None else dev
    wscale = float(Wscale_d.item())
    api._verify_raise(bad, "quantize_linear_columns")
    out = {"W_hat": api._out(W_hat, od), "trellis": api._out(trl[0], od),
           "suh": api._out(suh, od), "svh": api._out(svh[n0:n1].contiguous(), od),
           "Wscale": wscale, "lut_rms": float(lut_rms), "code": code, "K": int(K),
           "L": 16, "V": 1, "use_ldlq": use_ldlq, "channel_scales": False,
           "cols": (n0, n1)}
    api._out_done(dev, od)
    return out


def quantize_columns_fused(pieces: list, Lfac: torch.Tensor | None, code: str = "exl3_mul1",
                           su_seed: int = 20261011, buf_cols: int = 128, device=None,
                           margin: int = 0, pivot: int | None = None, out_device=None) -> list:
    """Output-channel ranges of the members of one fused module (one shared
    input Gram, so one Lfac), quantized in ONE sweep with a column segment per
    piece at its own K: pieces = [(W_j [out_j, in], (n0, n1), K_j), ...].
    Returns one quantize_linear_columns dict per piece, bit-identical to it
    (columns never interact); a single sweep keeps narrow pieces (k / v, the
    ends of a rank's range) on a full-width launch."""
    if not pieces:
        return []
    code = code or "exl3_mul1"
    api._check_code(code)
    k_in = pieces[0][0].shape[1]
    dev = api._cuda_device(device if device is not None else pieces[0][0].device)
    api._select(dev)
    s = api._stream(dev)
    lut_rms = api._lut_rms(api.get_lut(code))
    suh = api.sign_vec(k_in, su_seed).half()
    prep = []
    for W, cols, K in pieces:
        api._check_K(K)
        m_out = W.shape[0]
        n0, n1 = int(cols[0]), int(cols[1])
        if W.shape[1] != k_in or not (0 <= n0 < n1 <= m_out) or n0 % ALIGN or n1 % ALIGN:
            raise ValueError(f"piece [{n0}, {n1}) of W {tuple(W.shape)} (in = {k_in}): need "
                             "128-aligned ranges of members with one input dim")
        svh = api.sign_vec(m_out, su_seed + 1).half()
        W_dev = W.detach().to(dev, non_blocking=True)
        if W_dev.dtype not in api.DTYPE_IDS:
            W_dev = W_dev.float()
        Wi, parts = api._encode_inner(W_dev.contiguous(), suh, svh, dev)
        del W_dev
        Wscale_d = api._rms_scale(parts, Wi.numel(), float(lut_rms), dev)
        prep.append((api._div(Wi[:, n0:n1].contiguous(), Wscale_d), Wscale_d, svh, n0, n1, K))
        del Wi
    Wq = prep[0][0] if len(prep) == 1 else torch.cat([p[0] for p in prep], dim=1)
    widths = [p[4] - p[3] for p in prep]
    pv = api.STEPS // 2 if pivot is None else int(pivot)
    hatW, trl, _st, _ = api._sweep(Wq, Lfac, [p[5] for p in prep], widths, code, pv, margin,
                                   buf_cols)
    del Wq
    bad = torch.zeros(1, dtype=torch.int32, device=dev)
    su32 = suh.float().to(dev)
    outs_dev, c0 = [], 0
    for (_wq, Wscale_d, svh, n0, n1, K), t, w in zip(prep, trl, widths):
        hw = hatW[:, c0:c0 + w]
        api._verify_async(t, hw, K, code, bad)
        sv32 = svh[n0:n1].float().to(dev).contiguous()
        W_hat = torch.empty(w, k_in, dtype=torch.float32, device=dev)
        call("exl3b_incoherence_inv", hw.contiguous().data_ptr(), k_in, w,
             Wscale_d.data_ptr(), su32.data_ptr(), sv32.data_ptr(), W_hat.data_ptr(), s)
        outs_dev.append((W_hat, t))
        c0 += w
    od = torch.device(out_device) if out_device is not None else dev
    wscales = torch.cat([p[1] for p in prep]).tolist()
    api._verify_raise(bad, "quantize_columns_fused")
    outs = []
    for (_wq, _sc, svh, n0, n1, K), (W_hat, t), wscale in zip(prep, outs_dev, wscales):
        outs.append({"W_hat": api._out(W_hat, od), "trellis": api._out(t, od),
                     "suh": api._out(suh, od), "svh": api._out(svh[n0:n1].contiguous(), od),
                     "Wscale": float(wscale), "lut_rms": float(lut_rms), "code": code,
                     "K": int(K), "L": 16, "V": 1, "use_ldlq": Lfac is not None,
                     "channel_scales": False, "cols": (n0, n1)})
    api._out_done(dev, od)
    return outs


def lfac(H_x: torch.Tensor, k_in: int, percdamp: float = 0.01, su_seed: int = 20261011,
         device=None) -> torch.Tensor:
    """The damped block-LDL factor quantize_linear computes from H_x (the
    same rotation by the su sign vector of `su_seed`, damping and fallback)."""
    dev = api._cuda_device(device if device is not None else H_x.device)
    api._select(dev)
    suh = api.sign_vec(k_in, su_seed).half()
    return api._damped_lfac(H_x, suh, percdamp, dev)


def gather_columns(part: dict, n: int, group=None) -> dict:
    """All-gather the ranks' column ranges of one projection into the whole
    quantize_linear dict on every rank (torch.distributed; NCCL for CUDA
    tensors, gloo for CPU ones).  Ranges are padded to the widest one for
    the collective and cut back after it."""
    import torch.distributed as dist
    world = dist.get_world_size(group)
    ranges = column_ranges(n, world)
    wmax = max(b - a for a, b in ranges)
    tr, Wh = part["trellis"], part["W_hat"]
    tk, _, words = tr.shape
    k_in = Wh.shape[1]
    tr_pad = tr.new_zeros(tk, wmax // 16, words)
    tr_pad[:, :tr.shape[1]] = tr
    wh_pad = Wh.new_zeros(wmax, k_in)
    wh_pad[:Wh.shape[0]] = Wh
    # collectives have no int16 type: the trellis travels as its bytes
    tr_bytes = tr_pad.view(torch.uint8)
    tr_all = [torch.empty_like(tr_bytes) for _ in range(world)]
    wh_all = [torch.empty_like(wh_pad) for _ in range(world)]
    dist.all_gather(tr_all, tr_bytes, group=group)
    dist.all_gather(wh_all, wh_pad, group=group)
    trellis = torch.cat([t.view(torch.int16)[:, :(b - a) // 16]
                         for t, (a, b) in zip(tr_all, ranges)], dim=1)
    W_hat = torch.cat([h[:b - a] for h, (a, b) in zip(wh_all, ranges)], dim=0)
    svh = api.sign_vec(n, 20261012 if "su_seed" not in part else part["su_seed"] + 1).half()
    out = dict(part)
    out.update(W_hat=W_hat, trellis=trellis, svh=svh.to(part["svh"].device), cols=(0, n))
    return out


def quantize_linear_split(W: torch.Tensor, H_x: torch.Tensor | None, K: int = 4, group=None,
                          gather: bool = True, **kw) -> dict:
    """quantize_linear of one projection with its output columns spread over
    the ranks of `group` (every rank passes the same W and H_x).  Returns the
    whole layer's dict on every rank when `gather`, else this rank's range."""
    import torch.distributed as dist
    rank, world = dist.get_rank(group), dist.get_world_size(group)
    su_seed = kw.get("su_seed", 20261011)
    cols = column_ranges(W.shape[0], world)[rank]
    part = quantize_linear_columns(W, H_x, cols, K=K, **kw)
    part["su_seed"] = su_seed
    if not gather:
        return part
    out = gather_columns(part, W.shape[0], group)
    out.pop("su_seed", None)
    return out
