// ref_gpu_shim.cu -- TEST / MEASUREMENT INFRASTRUCTURE ONLY.
//
// C entry points around the reference's OWN GPU GEMV (bread_matvec,
// kernels.cu:289-308, compiled for sm_100a from the reference sources by
// oracle/Makefile into _ref/libbread_refgpu.so) so that bench.py can time the
// reference's GPU path on the B200 beside this library: one matvec launch,
// and the per-expert serial launch loop of expert_bench.cu:182-194 (gate,
// up, silu_mul, down, scale_accum for each routed expert on one stream).
// Nothing in breadv2_b200 links or loads this.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

// the reference's dispatcher (C++ linkage, defined in kernels.cu)
void bread_matvec(void *w, half *x, half *y, int rows, int cols, int qtype, cudaStream_t stream);

// The two elementwise kernels of the loop, restated from
// expert_bench.cu:21-37 (static there, so they cannot be linked).
static __global__ void refgpu_silu_mul(half *gate, const half *up, int n)
{
    const int i = (int)(blockIdx.x * blockDim.x + threadIdx.x);
    if (i < n) {
        const float g = __half2float(gate[i]);
        const float u = __half2float(up[i]);
        gate[i] = __float2half((g / (1.0f + expf(-g))) * u);
    }
}

static __global__ void refgpu_scale_accum(half *dst, const half *src, float scale, int n)
{
    const int i = (int)(blockIdx.x * blockDim.x + threadIdx.x);
    if (i < n) dst[i] = __float2half(__half2float(dst[i]) + scale * __half2float(src[i]));
}

extern "C" int refgpu_matvec(void *w, void *x, void *y, int rows, int cols, int qtype, void *stream)
{
    bread_matvec(w, static_cast<half *>(x), static_cast<half *>(y), rows, cols, qtype,
                 static_cast<cudaStream_t>(stream));
    return (int)cudaGetLastError();
}

// expert_bench.cu:182-194 for n experts: hidden = sum_k w[k] * down_k(silu(gate_k x) * (up_k x)),
// fp16 x/hidden, host arrays of device pointers and weights.
extern "C" int refgpu_expert_loop(void *const *gate, void *const *up, void *const *down, const float *w, int n,
                                  void *x, void *hidden, void *eg, void *eu, void *eo, int H, int I, void *stream)
{
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    cudaMemsetAsync(hidden, 0, (size_t)H * sizeof(half), s);
    for (int k = 0; k < n; ++k) {
        bread_matvec(gate[k], static_cast<half *>(x), static_cast<half *>(eg), I, H, 12, s);
        bread_matvec(up[k], static_cast<half *>(x), static_cast<half *>(eu), I, H, 12, s);
        refgpu_silu_mul<<<(I + 255) / 256, 256, 0, s>>>(static_cast<half *>(eg), static_cast<const half *>(eu), I);
        bread_matvec(down[k], static_cast<half *>(eg), static_cast<half *>(eo), H, I, 14, s);
        refgpu_scale_accum<<<(H + 255) / 256, 256, 0, s>>>(static_cast<half *>(hidden), static_cast<const half *>(eo),
                                                           w[k], H);
    }
    return (int)cudaGetLastError();
}
