// exl3b_internal.h -- host-side declarations shared by the .cu files.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "exl3b_common.cuh"

namespace exl3b {

constexpr int kMaxDevices = 64;

// Per-device state owned by the library (decode tables, grow-only scratch).
struct DeviceState {
    bool ready = false;
    int sms = 0;
    __half* lut16[3] = {nullptr, nullptr, nullptr};   // per CodeId, [65536]
    float* lut32[3] = {nullptr, nullptr, nullptr};
    uint4* f2tab[3][8] = {};          // per (CodeId, K): pre-paired decode words
    uint8_t* scratch = nullptr;       // library-owned workspace (grow-only)
    size_t scratch_bytes = 0;
    float* stageX = nullptr;          // xtq_vit_run staging (grow-only)
    int32_t* stageS = nullptr;
    size_t stage_seqs = 0;
};

// Current device's state, initialised on first use (rc != 0 on failure).
int device_state(DeviceState** out);
int device_sms();

// Host-side decode table (fp32, fp16-exact values) for a code id.
int build_code_lut(int code, float* out65536);

// Bytes of one CTA's backpointer slot for K.
size_t bp_slot_bytes(int K);

// Pre-paired decode-word table ([16][512] uint4) of code/K, built on first use.
int f2tab_get(DeviceState* st, int code, int K, const uint4** out);
int build_f2tab(int K, const __half* lut16, uint4* tab, cudaStream_t stream);

// Tail-biting encode of nseq sequences X [nseq][256] -> states [nseq][256].
// ws must hold grid * bp_slot_bytes(K) bytes.
int launch_tailbite(const float* dX, int nseq, int K, int pivot, int margin,
                    int32_t* dStates, uint8_t* ws, int grid,
                    const uint4* f2tab, cudaStream_t stream);

}  // namespace exl3b
