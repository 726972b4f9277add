// common.cuh -- shared definitions for the sm_100a kernels and the C ABI.
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "../../include/bread_b200.h"

namespace bread {

constexpr int QK = 256;          // weights per Q4_K / Q6_K super-block
constexpr int Q4K_BYTES = 144;   // fp16 d, fp16 dmin, 12 B scales, 128 B nibbles
constexpr int Q6K_BYTES = 210;   // 128 B ql, 64 B qh, 16 int8 scales, fp16 d
constexpr int Q80_BYTES = 34;    // fp16 d, 32 int8
constexpr int Q80_ELEMS = 32;
constexpr int XGROUP = 32;       // activation quantisation group (one Q4_K sub-block)

// Device error word bits (read by bread_device_error).
constexpr unsigned DEVERR_TIMEOUT = 1u;
constexpr unsigned DEVERR_ROUTE = 2u;   // expert index out of range reached a kernel

// Bounded spin budget for every device-side wait (mbarrier, peer flags).
// 1<<26 polls with a nanosleep back-off is several seconds at most.
constexpr long long SPIN_LIMIT = 1ll << 26;

// ---- host-side error reporting (errors.cu) ----
int set_error(int status, const char *fmt, ...);
int cuda_status(cudaError_t e, const char *what);

inline int block_bytes(int qtype)
{
    return qtype == BREAD_QTYPE_Q4_K ? Q4K_BYTES : qtype == BREAD_QTYPE_Q6_K ? Q6K_BYTES
         : qtype == BREAD_QTYPE_Q8_0 ? Q80_BYTES : 0;
}
inline int block_elems(int qtype) { return qtype == BREAD_QTYPE_Q8_0 ? Q80_ELEMS : QK; }

// Number of SMs of the current device (cached per device).
int sm_count();

}  // namespace bread

#define BREAD_TRY(...)                    \
    do {                                  \
        int _st = (__VA_ARGS__);          \
        if (_st != BREAD_OK) return _st;  \
    } while (0)

#define BREAD_CUDA(expr, what)                                      \
    do {                                                            \
        cudaError_t _e = (expr);                                    \
        if (_e != cudaSuccess) return bread::cuda_status(_e, what); \
    } while (0)
