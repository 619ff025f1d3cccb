"""exl3b -- B200-native EXL3 trellis quantizer (host side).

Layers:
  native  ctypes binding of the C ABI (libexl3b200.so, include/exl3b200.h)
  ops     torch-tensor wrappers: device pointers + the current CUDA stream
  api     the reference-compatible Python API (quantize_linear, quantize,
          ldlq_viterbi, prepare_incoherence, ...)
"""
