// synth.cu -- seeded synthetic weights and activations with the value
// distributions of the reference path's benchmark configurations, produced
// bit-identically on the host and on the device (integer hashing, one
// correctly rounded fp32 multiply per value, integer fp32 -> fp16 rounding).
//
//   Q4_K: d, dmin = fp16(|N(0,1)| * 1e-3); the 12 scale bytes and 128 nibble
//         bytes uniform (any byte pattern decodes to 6-bit (scale, min) pairs
//         uniform in [0, 63], dequant_q4k_cpu.c:70-79).
//   Q6_K: ql, qh uniform; int8 scales uniform in [-32, 31];
//         d = fp16(+-|N(0,1)| * 1e-3).
//   Q8_0: d = fp16(|N(0,1)| * 1e-2), int8 quants uniform.
//   N(0,1): Irwin-Hall sum of four uniform 16-bit integers, centred and scaled.
#include "common.cuh"

namespace bread {

__host__ __device__ inline uint64_t mix64(uint64_t z)
{
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
// hash(seed, stream, ctr) = mix64(key(seed, stream) + ctr)
__host__ __device__ inline uint64_t hash_key(uint64_t seed, uint64_t stream)
{
    return mix64(seed ^ mix64(stream + 0x632BE59BD9B4E019ull));
}
__host__ __device__ inline uint64_t hash3(uint64_t key, uint64_t ctr) { return mix64(key + ctr); }
// Irwin-Hall(4) of the four 16-bit fields of h, minus its mean: |value| < 131071.
__host__ __device__ inline int ih4(uint64_t h)
{
    return (int)(h & 0xFFFF) + (int)((h >> 16) & 0xFFFF) + (int)((h >> 32) & 0xFFFF) + (int)(h >> 48) - 131070;
}
// 1 / std of ih4 = sqrt(3) / 65536
#define BREAD_IH4_INV ((float)(1.7320508075688772 / 65536.0))

// fp32 -> fp16 bits, round to nearest even, integer only.
__host__ __device__ inline uint16_t f32_to_f16_bits(float f)
{
    union {
        float f;
        uint32_t u;
    } c;
    c.f = f;
    const uint32_t x = c.u;
    const uint32_t sign = (x >> 16) & 0x8000u;
    const uint32_t ex = (x >> 23) & 0xFFu;
    uint32_t man = x & 0x7FFFFFu;
    if (ex == 0xFF) return (uint16_t)(sign | 0x7C00u | (man ? 0x200u : 0u));
    const int e = (int)ex - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7C00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        const int shift = 14 - e;
        const uint32_t halfb = 1u << (shift - 1);
        const uint32_t rest = man & ((1u << shift) - 1u);
        uint32_t r = man >> shift;
        if (rest > halfb || (rest == halfb && (r & 1u))) r++;
        return (uint16_t)(sign | r);
    }
    uint32_t r = ((uint32_t)e << 10) | (man >> 13);
    const uint32_t rest = man & 0x1FFFu;
    if (rest > 0x1000u || (rest == 0x1000u && (r & 1u))) r++;
    return (uint16_t)(sign | r);
}

// |N(0,1)| * scale as fp32 (one rounding: int -> float is exact)
__host__ __device__ inline float abs_normal(uint64_t h, float scale_times_inv)
{
    int v = ih4(h);
    if (v < 0) v = -v;
    return (float)v * scale_times_inv;
}

// Block b of a synthetic tensor, written to dst (block-sized buffer).
__host__ __device__ inline void synth_block(uint8_t *dst, int qtype, uint64_t key, long long b)
{
    const uint64_t base = (uint64_t)b * 32u;
    if (qtype == BREAD_QTYPE_Q4_K) {
        for (int i = 0; i < 18; ++i) {
            const uint64_t h = hash3(key, base + i);
            for (int k = 0; k < 8; ++k) dst[8 * i + k] = (uint8_t)(h >> (8 * k));
        }
        const uint16_t d = f32_to_f16_bits(abs_normal(hash3(key, base + 20), (float)(1e-3 * 1.7320508075688772 / 65536.0)));
        const uint16_t m = f32_to_f16_bits(abs_normal(hash3(key, base + 21), (float)(1e-3 * 1.7320508075688772 / 65536.0)));
        dst[0] = (uint8_t)d;
        dst[1] = (uint8_t)(d >> 8);
        dst[2] = (uint8_t)m;
        dst[3] = (uint8_t)(m >> 8);
    } else if (qtype == BREAD_QTYPE_Q6_K) {
        for (int i = 0; i < 24; ++i) {
            const uint64_t h = hash3(key, base + i);
            for (int k = 0; k < 8; ++k) dst[8 * i + k] = (uint8_t)(h >> (8 * k));
        }
        const uint64_t hs0 = hash3(key, base + 24), hs1 = hash3(key, base + 25);
        for (int k = 0; k < 16; ++k) {
            const uint8_t byte = (uint8_t)((k < 8 ? hs0 : hs1) >> (8 * (k & 7)));
            dst[192 + k] = (uint8_t)(int8_t)((int)(byte & 63) - 32);
        }
        const uint64_t hd = hash3(key, base + 26);
        uint16_t d = f32_to_f16_bits(abs_normal(hd, (float)(1e-3 * 1.7320508075688772 / 65536.0)));
        if (hash3(key, base + 27) & 1) d |= 0x8000u;
        dst[208] = (uint8_t)d;
        dst[209] = (uint8_t)(d >> 8);
    } else {  // Q8_0
        for (int i = 0; i < 5; ++i) {
            const uint64_t h = hash3(key, base + i);
            for (int k = 0; k < 8 && 8 * i + k < Q80_BYTES; ++k) dst[8 * i + k] = (uint8_t)(h >> (8 * k));
        }
        const uint16_t d = f32_to_f16_bits(abs_normal(hash3(key, base + 6), (float)(1e-2 * 1.7320508075688772 / 65536.0)));
        dst[0] = (uint8_t)d;
        dst[1] = (uint8_t)(d >> 8);
    }
}

__host__ __device__ inline float synth_normal(uint64_t key, long long i, float stddev)
{
    return ((float)ih4(hash3(key, (uint64_t)i)) * BREAD_IH4_INV) * stddev;
}

__global__ void synth_blocks_kernel(uint8_t *dst, long long n, int qtype, int bb, uint64_t key)
{
    __align__(16) uint8_t buf[Q6K_BYTES + 14];
    for (long long b = blockIdx.x * (long long)blockDim.x + threadIdx.x; b < n; b += (long long)gridDim.x * blockDim.x) {
        synth_block(buf, qtype, key, b);
        uint8_t *o = dst + b * bb;
        const uintptr_t al = reinterpret_cast<uintptr_t>(o);
        if ((al & 15) == 0 && (bb & 15) == 0) {
            for (int i = 0; i < bb; i += 16) *reinterpret_cast<uint4 *>(o + i) = *reinterpret_cast<const uint4 *>(buf + i);
        } else if ((al & 1) == 0 && (bb & 1) == 0) {
            for (int i = 0; i < bb; i += 2) *reinterpret_cast<uint16_t *>(o + i) = *reinterpret_cast<const uint16_t *>(buf + i);
        } else {
            for (int i = 0; i < bb; ++i) o[i] = buf[i];
        }
    }
}

__global__ void synth_normal_kernel(void *dst, long long n, float stddev, uint64_t key, int half_out)
{
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
        const float v = synth_normal(key, i, stddev);
        if (half_out)
            static_cast<uint16_t *>(dst)[i] = f32_to_f16_bits(v);
        else
            static_cast<float *>(dst)[i] = v;
    }
}

static int grid_of(long long n) { long long g = (n + 255) / 256; const long long cap = (long long)sm_count() * 32; return (int)(g < cap ? (g > 0 ? g : 1) : cap); }

}  // namespace bread

using namespace bread;

extern "C" int bread_synth_blocks(void *dst, long long n_blocks, int qtype, uint64_t seed, uint64_t stream_id,
                                  cudaStream_t stream)
{
    const int bb = block_bytes(qtype);
    if (!bb) return set_error(BREAD_ERR_QTYPE, "synth: unknown qtype %d", qtype);
    if (!dst || n_blocks < 0) return set_error(BREAD_ERR_ARG, "synth: bad argument");
    if (!n_blocks) return BREAD_OK;
    synth_blocks_kernel<<<grid_of(n_blocks), 256, 0, stream>>>(static_cast<uint8_t *>(dst), n_blocks, qtype, bb,
                                                               hash_key(seed, stream_id));
    BREAD_CUDA(cudaGetLastError(), "synth blocks launch");
    return BREAD_OK;
}

extern "C" int bread_synth_normal_f32(float *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id,
                                      cudaStream_t stream)
{
    if (!dst || n < 0) return set_error(BREAD_ERR_ARG, "synth: bad argument");
    if (!n) return BREAD_OK;
    synth_normal_kernel<<<grid_of(n), 256, 0, stream>>>(dst, n, stddev, hash_key(seed, stream_id), 0);
    BREAD_CUDA(cudaGetLastError(), "synth normal launch");
    return BREAD_OK;
}

extern "C" int bread_synth_normal_f16(void *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id,
                                      cudaStream_t stream)
{
    if (!dst || n < 0) return set_error(BREAD_ERR_ARG, "synth: bad argument");
    if (!n) return BREAD_OK;
    synth_normal_kernel<<<grid_of(n), 256, 0, stream>>>(dst, n, stddev, hash_key(seed, stream_id), 1);
    BREAD_CUDA(cudaGetLastError(), "synth normal launch");
    return BREAD_OK;
}

extern "C" int bread_synth_blocks_host(void *dst, long long n_blocks, int qtype, uint64_t seed, uint64_t stream_id)
{
    const int bb = block_bytes(qtype);
    if (!bb) return set_error(BREAD_ERR_QTYPE, "synth: unknown qtype %d", qtype);
    if (!dst || n_blocks < 0) return set_error(BREAD_ERR_ARG, "synth: bad argument");
    const uint64_t key = hash_key(seed, stream_id);
    for (long long b = 0; b < n_blocks; ++b) synth_block(static_cast<uint8_t *>(dst) + b * bb, qtype, key, b);
    return BREAD_OK;
}

extern "C" int bread_synth_normal_f32_host(float *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id)
{
    if (!dst || n < 0) return set_error(BREAD_ERR_ARG, "synth: bad argument");
    const uint64_t key = hash_key(seed, stream_id);
    for (long long i = 0; i < n; ++i) dst[i] = synth_normal(key, i, stddev);
    return BREAD_OK;
}

extern "C" int bread_synth_normal_f16_host(void *dst, long long n, float stddev, uint64_t seed, uint64_t stream_id)
{
    if (!dst || n < 0) return set_error(BREAD_ERR_ARG, "synth: bad argument");
    const uint64_t key = hash_key(seed, stream_id);
    for (long long i = 0; i < n; ++i) static_cast<uint16_t *>(dst)[i] = f32_to_f16_bits(synth_normal(key, i, stddev));
    return BREAD_OK;
}
