// exl3b_common.cuh -- shared definitions for the B200 EXL3 trellis quantizer.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace exl3b {

// Return codes of the C ABI.  1..7 keep the meaning of the reference's
// xtq_vit_* codes (viterbi_esimd.cpp:945-1003); 8+ are new.
enum Rc : int {
    RC_OK = 0,
    RC_NO_DEVICE = 1,      // no CUDA device / runtime failure at init
    RC_ALLOC = 2,          // device allocation failed
    RC_BAD_DEVICE = 3,     // bad device index
    RC_DEVICE_ERROR = 4,   // CUDA error during a launch or copy
    RC_TOO_MANY_BYTES = 5, // request exceeds the configured device-byte cap
    RC_BAD_NSEQ = 6,       // sequence count out of range
    RC_BAD_REQUEST = 7,    // malformed request (bad code / argument)
    RC_BAD_K = 8,          // K outside 2..7
    RC_NOT_SPD = 9,        // Cholesky met a non-positive pivot
    RC_NONFINITE = 10,     // non-finite input where a finite one is required
    RC_WORKSPACE = 11,     // caller workspace too small / misaligned
};

// Code ids for the V=1 decode tables (quantize.py:56-87).
enum CodeId : int { CODE_MUL1 = 0, CODE_3INST = 1, CODE_MCG = 2 };

constexpr int kSteps = 256;   // trellis steps per 16x16 tile
constexpr int kL = 16;        // shift-register state bits

// Records the last error text for exl3b_last_error() (host side).
void set_error(const char* fmt, ...);
int check_cuda(cudaError_t e, const char* what);

}  // namespace exl3b
