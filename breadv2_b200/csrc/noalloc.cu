// noalloc.cu -- bread_moe_ffn_noalloc: the MoE FFN block for callers that
// cannot allocate device memory.
//
// Who needs it: an engine that hands every free byte of HBM to its resident
// expert weights and caches at start-up has nothing left for cudaMalloc to
// return, and some host loops may not call cudaMalloc on the decode path at
// all because it can synchronise the whole device and stall other streams.
// Such callers still own their inputs and outputs; only the scratch of
// bread_moe_ffn (router logits, int16 activations, expert token lists, the
// SiLU*mul intermediate) moves into a fixed array compiled into this library.
//
// Properties of that array (g_moe_scratch below):
//   * NOALLOC_SCRATCH_BYTES (256 KiB) on every GPU that loads the library, held
//     until the process exits;
//   * shared by every call on a device and keeping the previous call's
//     contents: each call clears the part that must start at zero (the
//     router's completion counter, via bread_moe_ffn) and writes everything
//     else before reading it;
//   * calls whose kernels overlap on the GPU (different streams, or host
//     threads without ordering) race on it and give wrong results: order them.
#include <mutex>

#include "common.cuh"
#include "moe.cuh"

namespace bread {

constexpr size_t NOALLOC_SCRATCH_BYTES = 256 * 1024;

// Device storage.  In host code `g_moe_scratch` is only a host-side stand-in
// for the symbol, never a device address: the kernels get the address that
// cudaGetSymbolAddress returns for the current device.
static __device__ __align__(256) uint8_t g_moe_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int NOALLOC_MAX_DEVICES = 64;
static std::mutex g_scratch_mu;
static void *g_scratch_addr[NOALLOC_MAX_DEVICES] = {};

// Device address of g_moe_scratch on the current device.  The first call on
// a device looks it up, so that call should come before any stream capture.
// Every later call made outside capture looks it up again (no allocation,
// cheap), so an address from before a cudaDeviceReset -- which reloads the
// module and moves the array -- is never handed to a kernel; a call on a
// capturing stream cannot make the lookup and takes the last address found.
static int scratch_address(cudaStream_t stream, void **out)
{
    int dev = 0;
    BREAD_CUDA(cudaGetDevice(&dev), "moe_ffn_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= NOALLOC_MAX_DEVICES)
        return set_error(BREAD_ERR_STATE, "moe_ffn_noalloc: device %d beyond %d", dev, NOALLOC_MAX_DEVICES);
    cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
    BREAD_CUDA(cudaStreamIsCapturing(stream, &cap), "moe_ffn_noalloc: cudaStreamIsCapturing");
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    if (cap == cudaStreamCaptureStatusNone) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_scratch);
        if (e != cudaSuccess) return cuda_status(e, "moe_ffn_noalloc: cudaGetSymbolAddress");
        if (!p) return set_error(BREAD_ERR_CUDA, "moe_ffn_noalloc: no device address for the scratch array");
        g_scratch_addr[dev] = p;
    } else if (!g_scratch_addr[dev]) {
        return set_error(BREAD_ERR_STATE,
                         "moe_ffn_noalloc: first call on device %d is inside stream capture; make one call outside "
                         "capture first",
                         dev);
    }
    *out = g_scratch_addr[dev];
    return BREAD_OK;
}

}  // namespace bread

using namespace bread;

extern "C" int bread_moe_ffn_noalloc(const void *const *gate_ptrs, const void *const *up_ptrs,
                                     const void *const *down_ptrs, const float *W_r, const void *w_sg,
                                     const void *sh_gate, const void *sh_up, const void *sh_down, const float *x,
                                     float *out, int T, int H, int I, int E, int top_k, int *idx_out, float *w_out,
                                     float *sg_out, cudaStream_t stream)
{
    BREAD_TRY(moe_check_shapes(T, H, I, E, top_k, true));
    const size_t need = StepWs::make(T, H, I, E, top_k, false).total;
    if (need > NOALLOC_SCRATCH_BYTES)
        return set_error(BREAD_ERR_WORKSPACE,
                         "moe_ffn_noalloc: T=%d H=%d I=%d E=%d top_k=%d need %zu bytes of scratch, the fixed array "
                         "holds %zu; use bread_moe_ffn with a workspace",
                         T, H, I, E, top_k, need, NOALLOC_SCRATCH_BYTES);
    void *scratch = nullptr;
    BREAD_TRY(scratch_address(stream, &scratch));
    return bread_moe_ffn(gate_ptrs, up_ptrs, down_ptrs, W_r, w_sg, sh_gate, sh_up, sh_down, x, out, T, H, I, E, top_k,
                         idx_out, w_out, sg_out, scratch, NOALLOC_SCRATCH_BYTES, stream);
}
