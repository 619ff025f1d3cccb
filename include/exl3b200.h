/* exl3b200.h -- C ABI of libexl3b200.so, the B200 EXL3 trellis quantizer.
 *
 * Plain pointers and sizes; no framework types.  Every function returns an
 * int status (0 = success; codes below) and never aborts the process;
 * exl3b_last_error() returns a text description of the calling thread's last
 * failure.  "d" pointers are CUDA device pointers on the current device;
 * `stream` is a cudaStream_t (NULL = legacy default stream).  Entry points
 * that take a stream are asynchronous with respect to the host.
 *
 * Reference interfaces replaced (SergiioB/exl3xpu-mixedk):
 *   quantize/viterbi_esimd.cpp:935-968   xtq_vit_init
 *   quantize/viterbi_esimd.cpp:970-1005  xtq_vit_run
 *   quantize/quantize.py:611-628         _esimd_tailbite  (exl3b_tailbite)
 *   quantize/quantize.py:323-354         quantize_seq_tailbite
 */
#ifndef EXL3B200_H
#define EXL3B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define EXL3B_ABI_VERSION 1

/* Status codes.  1..7 keep the meanings of the reference's xtq_vit_* codes. */
#define EXL3B_OK              0
#define EXL3B_NO_DEVICE       1   /* no CUDA device / init failure            */
#define EXL3B_ALLOC           2   /* device allocation failed                 */
#define EXL3B_BAD_DEVICE      3   /* device index out of range                */
#define EXL3B_DEVICE_ERROR    4   /* CUDA error in a launch or copy           */
#define EXL3B_TOO_MANY_BYTES  5   /* over XTQ_VIT_MAXBYTES                    */
#define EXL3B_BAD_NSEQ        6   /* sequence count out of range              */
#define EXL3B_BAD_REQUEST     7   /* malformed request / unsupported code     */
#define EXL3B_BAD_K           8   /* K outside 2..7                           */
#define EXL3B_NOT_SPD         9   /* factorisation met a non-positive pivot   */
#define EXL3B_NONFINITE      10   /* non-finite input                         */
#define EXL3B_WORKSPACE      11   /* caller workspace too small / misaligned  */

/* Code ids of the V=1 decode tables (quantize.py:56-87). */
#define EXL3B_CODE_MUL1   0       /* "exl3_mul1"  */
#define EXL3B_CODE_3INST  1       /* "exl3_3inst" */
#define EXL3B_CODE_MCG    2       /* "exl3_mcg"   */

/* Text of the calling thread's last error ("" if none). */
const char* exl3b_last_error(void);

/* EXL3B_ABI_VERSION of the loaded library. */
int exl3b_abi_version(void);

/* Host-only: fp32 [65536] decode table of a code id (quantize.py:90-97
 * get_lut).  Needs no GPU. */
int exl3b_code_lut(int code, float* out65536);

/* Select `device` and build its decode tables (optional; first use of any
 * entry point initialises the current device). */
int exl3b_device_init(int device);

/* Workspace bytes exl3b_tailbite needs for (nseq, K) on the current device
 * (0 for invalid arguments). */
size_t exl3b_tailbite_workspace_bytes(int nseq, int K);

/* Tail-biting Viterbi encode (quantize_seq_tailbite, quantize.py:323-354,
 * bit-exact with its fp32 "sq" emit), K = 2..7, V = 1.
 *   dX       [nseq][256] fp32 targets, 16-byte aligned (one tile per row,
 *            element t = tile position perm[t])
 *   pivot    pass-1 boundary step, 0 <= pivot < 256
 *   margin   0 = full pass 1; > 0 = pass 1 runs pivot+margin steps
 *   dStates  [nseq][256] int32 full 16-bit states
 *   workspace/workspace_bytes: caller scratch (256-byte aligned, at least
 *            exl3b_tailbite_workspace_bytes) or NULL for library scratch. */
int exl3b_tailbite(const float* dX, int nseq, int K, int code, int pivot,
                   int margin, int32_t* dStates, void* workspace,
                   size_t workspace_bytes, void* stream);

/* Drop-in for the reference's native Viterbi (viterbi_esimd.cpp:935-1005):
 * same signatures, argument meaning and return codes.  Host X [nseq][256]
 * fp32 in, host int32 states [nseq][256] out, synchronous, mul1 code at
 * K = 4 ("mul1p", "mul1", "mul1t").  Env: XTQ_VIT_DEVIDX, XTQ_VIT_MAXSEQ,
 * XTQ_VIT_MAXBYTES. */
int xtq_vit_init(void);
int xtq_vit_run(const float* X, int nseq, const char* code, int margin,
                int pivot, int32_t* out);

#ifdef __cplusplus
}
#endif
#endif /* EXL3B200_H */
