"""torch-tensor wrappers over the C ABI.

Each wrapper takes CUDA tensors, selects their device in the library, passes
raw device pointers and torch's current stream, and allocates workspaces and
outputs through torch's caching allocator (stream-ordered, so a workspace may
be released as soon as the launch is queued).
"""
from __future__ import annotations

import torch

from . import native
from .native import call, lib

STEPS = 256


def _dev_index(t: torch.Tensor) -> int:
    if not t.is_cuda:
        raise ValueError("expected a CUDA tensor")
    return t.device.index if t.device.index is not None else torch.cuda.current_device()


def select_device(t: torch.Tensor) -> int:
    """Make the tensor's device current in the library (it links its own CUDA
    runtime, whose current device is separate from torch's)."""
    dev = _dev_index(t)
    call("exl3b_device_init", dev)
    return dev


def stream_handle(dev: int) -> int:
    return torch.cuda.current_stream(dev).cuda_stream


def code_id(code: str) -> int:
    try:
        return native.CODE_IDS[code]
    except KeyError:
        raise ValueError(f"code {code!r} has no CUDA encoder; supported: "
                         f"{sorted(native.CODE_IDS)}") from None


def tailbite(X: torch.Tensor, K: int, pivot: int = 128, margin: int = 0,
             code: str = "exl3_mul1") -> torch.Tensor:
    """Tail-biting Viterbi encode (quantize_seq_tailbite, quantize.py:323-354).

    X: [nseq, 256] fp32 CUDA tensor, one 16x16 tile per row in sequence order.
    Returns int32 [nseq, 256] full 16-bit states (bit-exact with the
    reference's fp32 emit)."""
    if X.dim() != 2 or X.shape[1] != STEPS or X.dtype != torch.float32:
        raise ValueError(f"X must be [nseq, 256] fp32, got {tuple(X.shape)} {X.dtype}")
    X = X.contiguous()
    nseq = X.shape[0]
    dev = select_device(X)
    out = torch.empty(nseq, STEPS, dtype=torch.int32, device=X.device)
    if nseq == 0:
        return out
    ws_bytes = lib().exl3b_tailbite_workspace_bytes(nseq, int(K))
    ws = torch.empty(max(ws_bytes, 1), dtype=torch.uint8, device=X.device)
    call("exl3b_tailbite", X.data_ptr(), nseq, int(K), code_id(code), int(pivot),
         int(margin), out.data_ptr(), ws.data_ptr(), ws_bytes, stream_handle(dev))
    return out
