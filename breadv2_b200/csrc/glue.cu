// glue.cu -- the four fp16 launchers reference layer_logic.cu:28-31 declares
// (and never defines), with the semantics of one_layer.cu's kernels.
#include <stdio.h>
#include <stdlib.h>

#include "common.cuh"

namespace bread {

// one_layer.cu:158-180 rmsnorm_inplace: one CTA of 256 threads; per-thread
// strided sum of squares (nvcc contracts the reference's acc += v*v into a
// fused multiply-add), then the same halving tree, rsqrtf(ss/n + eps), and
// x[i] = half((x[i]*rms)*w[i]).  Reduction order matches the reference kernel.
__global__ void rmsnorm_half_kernel(__half *x, const float *w, int n, float eps)
{
    __shared__ float sdata[256];
    const int tid = threadIdx.x;
    float acc = 0.0f;
    for (int i = tid; i < n; i += 256) {
        const float v = __half2float(x[i]);
        acc = __fmaf_rn(v, v, acc);
    }
    sdata[tid] = acc;
    __syncthreads();
    for (int s = 128; s > 0; s >>= 1) {
        if (tid < s) sdata[tid] = __fadd_rn(sdata[tid], sdata[tid + s]);
        __syncthreads();
    }
    const float rms = rsqrtf(sdata[0] / (float)n + eps);
    for (int i = tid; i < n; i += 256) x[i] = __float2half(__fmul_rn(__fmul_rn(__half2float(x[i]), rms), w[i]));
}

// one_layer.cu:190-197 silu_mul_inplace: gate = half(g/(1+expf(-g))*u)
__global__ void silu_mul_half_kernel(__half *gate, const __half *up, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const float g = __half2float(gate[i]);
    const float u = __half2float(up[i]);
    gate[i] = __float2half(g / (1.0f + expf(-g)) * u);
}

// one_layer.cu:203-208 scale_accum: dst = half(dst + scale*src); nvcc contracts
// the reference expression into one fused multiply-add, written out here.
__global__ void scale_accum_half_kernel(__half *dst, const __half *src, float scale, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    dst[i] = __float2half(__fmaf_rn(scale, __half2float(src[i]), __half2float(dst[i])));
}

// one_layer.cu:214-218 copy_half
__global__ void copy_half_kernel(__half *dst, const __half *src, int n)
{
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) dst[i] = src[i];
}

static int grid_for(int n) { return (n + 255) / 256; }

}  // namespace bread

using namespace bread;

extern "C" int bread_rmsnorm_half_c(void *x, const float *w, int n, float eps, cudaStream_t s)
{
    if (!x || !w || n <= 0) return set_error(BREAD_ERR_ARG, "rmsnorm_half: bad argument");
    rmsnorm_half_kernel<<<1, 256, 0, s>>>(static_cast<__half *>(x), w, n, eps);
    BREAD_CUDA(cudaGetLastError(), "rmsnorm_half launch");
    return BREAD_OK;
}

extern "C" int bread_silu_mul_c(void *gate, const void *up, int n, cudaStream_t s)
{
    if (!gate || !up || n <= 0) return set_error(BREAD_ERR_ARG, "silu_mul: bad argument");
    silu_mul_half_kernel<<<grid_for(n), 256, 0, s>>>(static_cast<__half *>(gate), static_cast<const __half *>(up), n);
    BREAD_CUDA(cudaGetLastError(), "silu_mul launch");
    return BREAD_OK;
}

extern "C" int bread_scale_accum_c(void *dst, const void *src, float scale, int n, cudaStream_t s)
{
    if (!dst || !src || n <= 0) return set_error(BREAD_ERR_ARG, "scale_accum: bad argument");
    scale_accum_half_kernel<<<grid_for(n), 256, 0, s>>>(static_cast<__half *>(dst), static_cast<const __half *>(src),
                                                        scale, n);
    BREAD_CUDA(cudaGetLastError(), "scale_accum launch");
    return BREAD_OK;
}

extern "C" int bread_copy_half_c(void *dst, const void *src, int n, cudaStream_t s)
{
    if (!dst || !src || n <= 0) return set_error(BREAD_ERR_ARG, "copy_half: bad argument");
    copy_half_kernel<<<grid_for(n), 256, 0, s>>>(static_cast<__half *>(dst), static_cast<const __half *>(src), n);
    BREAD_CUDA(cudaGetLastError(), "copy_half launch");
    return BREAD_OK;
}

static void die_on(int st, const char *what)
{
    if (st != BREAD_OK) {
        fprintf(stderr, "%s: %s (%s)\n", what, bread_status_string(st), bread_last_error());
        exit(1);
    }
}

// C++-linkage drop-ins with the layer_logic.cu:28-31 signatures.
void bread_rmsnorm_half(half *x, const float *w, int n, float eps, cudaStream_t s)
{
    die_on(bread_rmsnorm_half_c(x, w, n, eps, s), "bread_rmsnorm_half");
}
void bread_silu_mul(half *gate, const half *up, int n, cudaStream_t s)
{
    die_on(bread_silu_mul_c(gate, up, n, s), "bread_silu_mul");
}
void bread_scale_accum(half *dst, const half *src, float scale, int n, cudaStream_t s)
{
    die_on(bread_scale_accum_c(dst, src, scale, n, s), "bread_scale_accum");
}
void bread_copy_half(half *dst, const half *src, int n, cudaStream_t s)
{
    die_on(bread_copy_half_c(dst, src, n, s), "bread_copy_half");
}
