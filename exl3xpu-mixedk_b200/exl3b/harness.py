"""Inputs of the reference's harness entry point quantize() built from a
weight and its captured input Gram, as the reference's per-tensor check does
(check_tensor_bitexact.py:45-66 build_inputs).

quantize(W_transformed, U_upper, ...) takes the weight already in the inner
(post-incoherence) domain and the GPTQ-convention factor U (upper
triangular, U^T U = G^-1) of the rotated, damped Gram G.  build_inputs()
produces both from W [out, in] and H [in, in]:

  * W_inner = to_inner(W^T, suh, svh) on the library's rotation kernel,
    returned transposed ([out, in]);
  * G = rotate_hessian(H, suh) with dead diagonal entries set to 1 and
    percdamp x mean(diag) added (the library's kernels: exactly quantize_linear's
    damped G);
  * U = cholesky(cholesky_inverse(cholesky(G in fp64)), upper) -- the
    reference builds this factor with torch.linalg in fp64, and so does this
    helper (on the device holding the tensors).  It is input preparation for
    the harness, not part of the quantizer: quantize() converts U back to G
    and factors it with the library's block LDL.

With seed = 128 (the pivot) and margin = 0, quantize(*build_inputs(W, H))
encodes the same problem as quantize_linear(W, H), up to the fp64 round trip
of G through U.
"""
from __future__ import annotations

import torch

from . import api
from .native import call

SU_SEED = 20261011
PERCDAMP = 0.01


def damped_gram(H: torch.Tensor, suh: torch.Tensor, percdamp: float = PERCDAMP,
                device=None) -> torch.Tensor:
    """Rotated, damped Gram G (fp32, on the CUDA device) exactly as
    quantize_linear builds it (quantize.py:809-814)."""
    dev = api._cuda_device(device if device is not None else H.device)
    G = api.rotate_hessian(H, suh, device=dev)
    call("exl3b_damp_hessian", G.data_ptr(), G.shape[0], float(percdamp), None,
         api._stream(dev))
    return G


def build_inputs(W: torch.Tensor, H: torch.Tensor, su_seed: int = SU_SEED,
                 percdamp: float = PERCDAMP, device=None):
    """(W_transformed [out, in] fp32, U [in, in] fp32 upper triangular with
    U^T U = G^-1) for quantize(); tensors on the CUDA device."""
    m_out, k_in = W.shape
    dev = api._cuda_device(device if device is not None else W.device)
    suh = api.sign_vec(k_in, su_seed).half()
    svh = api.sign_vec(m_out, su_seed + 1).half()
    W_inner = api.to_inner(W.detach().to(dev).float().t(), suh, svh, device=dev)
    G = damped_gram(H, suh, percdamp, dev).double()
    Gi = torch.cholesky_inverse(torch.linalg.cholesky(G))
    U = torch.linalg.cholesky(Gi, upper=True)
    return W_inner.t().contiguous(), U.float().contiguous()
