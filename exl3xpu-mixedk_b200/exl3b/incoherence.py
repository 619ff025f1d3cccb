"""EXL3 per-channel magnitude folds (channel_scales=True) and
prepare_incoherence, on the CUDA path.

Reference: quantize/quantize.py:785-800 and :854-862 (quantize_linear
channel_scales branch), :969-1058 (prepare_incoherence).
"""
from __future__ import annotations

import torch

from .native import call, lib


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def channel_scale_inner(W_dev: torch.Tensor, suh: torch.Tensor, svh: torch.Tensor, dev):
    """W [out, in] (CUDA) -> (W_i [k][n] fp32, su_mag [k], sv_store [n],
    sv_mag [n]) with sign vectors suh/svh (+-1)."""
    from .api import DTYPE_IDS
    m_out, k_in = W_dev.shape
    su = suh.float().to(dev).contiguous()
    sv = svh.float().to(dev).contiguous()
    Wi = torch.empty(k_in, m_out, dtype=torch.float32, device=dev)
    su_mag = torch.empty(k_in, dtype=torch.float32, device=dev)
    sv_mag = torch.empty(m_out, dtype=torch.float32, device=dev)
    sv_store = torch.empty(m_out, dtype=torch.float32, device=dev)
    parts = torch.empty((k_in // 128) * (m_out // 128), dtype=torch.float64, device=dev)
    wsb = lib().exl3b_channel_scale_workspace_bytes(m_out, k_in)
    ws = torch.empty(wsb, dtype=torch.uint8, device=dev)
    call("exl3b_channel_scale_fwd", W_dev.data_ptr(), DTYPE_IDS[W_dev.dtype], m_out, k_in,
         su.data_ptr(), sv.data_ptr(), Wi.data_ptr(), su_mag.data_ptr(), sv_mag.data_ptr(),
         sv_store.data_ptr(), parts.data_ptr(), ws.data_ptr(), wsb, _stream(dev))
    return Wi, parts, su_mag, sv_mag, sv_store


def channel_scale_outer(hatW: torch.Tensor, suh, svh, su_mag, sv_store, Wscale_d, dev):
    """Stored fields and reconstruction (quantize.py:854-862):
    suh = half(su * su_mag * Wscale), svh = half(sv * sv_store),
    W_hat = from_inner(hatW, suh, svh)^T."""
    k, n = hatW.shape
    su = suh.float().to(dev).contiguous()
    sv = svh.float().to(dev).contiguous()
    suh_s = torch.empty(k, dtype=torch.float16, device=dev)
    svh_s = torch.empty(n, dtype=torch.float16, device=dev)
    call("exl3b_channel_scale_store", su.data_ptr(), su_mag.data_ptr(), Wscale_d.data_ptr(),
         sv.data_ptr(), sv_store.data_ptr(), k, n, suh_s.data_ptr(), svh_s.data_ptr(),
         _stream(dev))
    W_hat = torch.empty(n, k, dtype=torch.float32, device=dev)
    su_f = suh_s.float()
    sv_f = svh_s.float()
    call("exl3b_incoherence_inv", hatW.data_ptr(), k, n, None, su_f.data_ptr(),
         sv_f.data_ptr(), W_hat.data_ptr(), _stream(dev))
    return W_hat, suh_s, svh_s


def prepare_incoherence(W: torch.Tensor, H_x: torch.Tensor | None = None,
                        su_seed: int = 20261011, sv_seed: int | None = None,
                        su_sign: torch.Tensor | None = None,
                        sv_sign: torch.Tensor | None = None,
                        channel_scales: bool = True, device: str = "cpu") -> dict:
    """quantize.py:969-1058.  Returns (on CPU, like the reference):
    Wt [out, in] fp32 trellis-domain weight (magnitudes folded, per-tensor
    scale not folded), G [in, in] sign-only rotated undamped Gram (or None),
    suh/svh fp32 signed magnitudes, su_mag, sv_mag, zero_out, channel_scales."""
    from .api import (DTYPE_IDS, _cuda_device, _encode_inner, _select, rotate_hessian,
                      sign_vec)
    m_out, k_in = W.shape
    assert k_in % 128 == 0 and m_out % 128 == 0, (W.shape, "need %128 dims")
    dev = _cuda_device(device)
    _select(dev)
    suh_sign = (sign_vec(k_in, su_seed).half() if su_sign is None else su_sign.half().cpu())
    svh_sign = (sign_vec(m_out, (su_seed + 1) if sv_seed is None else sv_seed).half()
                if sv_sign is None else sv_sign.half().cpu())
    W_dev = W.detach().to(dev)
    if W_dev.dtype not in DTYPE_IDS:
        W_dev = W_dev.float()
    W_dev = W_dev.contiguous()
    if channel_scales:
        Wi, _parts, su_mag, sv_mag, sv_store = channel_scale_inner(W_dev, suh_sign, svh_sign, dev)
        su = suh_sign.float().to(dev)
        sv = svh_sign.float().to(dev)
        suh = su * su_mag
        svh = sv * sv_store
        zero_out = sv_store == 0
    else:
        Wi, _parts = _encode_inner(W_dev, suh_sign, svh_sign, dev)
        suh, svh = suh_sign.float(), svh_sign.float()
        su_mag = torch.ones(k_in)
        sv_mag = torch.ones(m_out)
        zero_out = torch.zeros(m_out, dtype=torch.bool)
    G = None
    if H_x is not None:
        G = rotate_hessian(H_x, suh_sign, device=dev).cpu()
    return {"Wt": Wi.t().contiguous().cpu(), "G": G,
            "suh": suh.cpu(), "svh": svh.cpu(),
            "su_mag": su_mag.cpu(), "sv_mag": sv_mag.cpu(),
            "zero_out": zero_out.cpu(), "channel_scales": channel_scales}
