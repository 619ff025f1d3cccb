"""Drop-in replacement for the reference's ``quantize/quantize.py`` module
(SergiioB/exl3xpu-mixedk): ``import quantize as xq`` with this directory on
``sys.path`` gives the same public API, computed by the B200 CUDA kernels of
``exl3b`` (see exl3b/api.py)."""
from exl3b.api import (  # noqa: F401
    CODES,
    block_LDL,
    decode_trellis,
    from_inner,
    get_lut,
    had_left,
    had_right,
    hadamard128,
    hessian_weighted_err,
    ldlq_viterbi,
    pack_states,
    prepare_incoherence,
    quantize,
    quantize_linear,
    quantize_linear_fused,
    quantize_seq_tailbite,
    rel_mse,
    rotate_hessian,
    sign_vec,
    tensor_core_perm,
    to_inner,
    unpack_states,
    verify_trellis,
    viterbi,
)
