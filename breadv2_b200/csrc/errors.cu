// errors.cu -- status strings, per-thread last-error text, device error word.
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <atomic>

#include "common.cuh"
#include "ptx.cuh"

namespace bread {

__device__ unsigned g_dev_error = 0;

static thread_local char t_last_error[512] = "";

int set_error(int status, const char *fmt, ...)
{
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(t_last_error, sizeof t_last_error, fmt, ap);
    va_end(ap);
    return status;
}

int cuda_status(cudaError_t e, const char *what)
{
    return set_error(BREAD_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

int sm_count()
{
    // per-device cache; atomics because host threads may make their first
    // calls at the same time (both would store the same value)
    static std::atomic<int> cached[64];
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    int n = cached[dev].load(std::memory_order_relaxed);
    if (!n) {
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        cached[dev].store(n, std::memory_order_relaxed);
    }
    return n;
}

}  // namespace bread

extern "C" const char *bread_status_string(int s)
{
    switch (s) {
    case BREAD_OK: return "ok";
    case BREAD_ERR_ARG: return "invalid argument";
    case BREAD_ERR_QTYPE: return "unsupported qtype";
    case BREAD_ERR_ALIGN: return "misaligned pointer";
    case BREAD_ERR_CUDA: return "CUDA error";
    case BREAD_ERR_WORKSPACE: return "workspace too small";
    case BREAD_ERR_TIMEOUT: return "device wait timed out";
    case BREAD_ERR_STATE: return "invalid state";
    default: return "unknown status";
    }
}

extern "C" const char *bread_last_error(void) { return bread::t_last_error; }

extern "C" int bread_device_error(unsigned *word_out, int clear)
{
    unsigned w = 0;
    BREAD_CUDA(cudaMemcpyFromSymbol(&w, bread::g_dev_error, sizeof w), "read device error word");
    if (clear) {
        const unsigned z = 0;
        BREAD_CUDA(cudaMemcpyToSymbol(bread::g_dev_error, &z, sizeof z), "clear device error word");
    }
    if (word_out) *word_out = w;
    return BREAD_OK;
}
