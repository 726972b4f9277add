// gemv.cu -- Q4_K / Q6_K / Q8_0 dequantise-and-multiply GEMV for sm_100a and
// the bread_matvec family of entry points (reference kernels.cu:150-308).
//
// Fast path (Q4_K / Q6_K, 16-byte aligned weights, cols/256 in {1,2,4,8,16}):
//   * every warp owns a contiguous range of rows and streams them through its
//     own ring of shared-memory stages with 1-D bulk copies (TMA engine,
//     completion on an mbarrier), so no registers are tied up by loads in
//     flight and each weight byte crosses HBM once;
//   * 4 lanes share a super-block (each lane decodes 64 weights), so a warp
//     covers 32/(4*cols/256) rows per step;
//   * the activation is quantised once per CTA to int16 per 32 values and
//     each lane keeps its 64-value slice in registers (one token) or reloads
//     it from shared memory per token (several tokens); a group whose largest
//     value dwarfs the rest also gets a second int16 level (the first level's
//     error, quant32_r_n), and when any group of the launch has one, every row
//     takes a second dot pass over that residual (exact by linearity);
//   * weight x activation products are exact int32 dp2a sums per sub-block,
//     scaled in fp32 (qdot.cuh).
// Generic path (any alignment, any cols multiple of the block, Q8_0): one warp
// per row, exact fp32 dequantisation per element, fp32 FMA.
#include <stdio.h>
#include <stdlib.h>

#include <type_traits>

#include "common.cuh"
#include "ptx.cuh"
#include "qdot.cuh"

namespace bread {

template <int QT, int NB>
struct Geo {
    static constexpr int BB = QT == BREAD_QTYPE_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    static constexpr int LANES_ALL = 4 * NB;  // 4 lanes per super-block
    static constexpr int CP = LANES_ALL > 32 ? LANES_ALL / 32 : 1;  // column passes per lane
    static constexpr int LPR = LANES_ALL > 32 ? 32 : LANES_ALL;      // lanes per row
    static constexpr int RPW = 32 / LPR;                              // rows per warp step
    static constexpr int ROWB = BB * NB;
    static constexpr int STEPB = ROWB * RPW;  // a multiple of 16 for every NB above
    static constexpr int COLS = QK * NB;
};

constexpr int GEMV_WARPS = 8;
// shared-memory stages per warp: two for one token at 2048 columns (2 x 8 x
// 3.4 KB, so three CTAs fit an SM: 24 warps hide the decode latency better
// than a third stage does), three otherwise
__host__ __device__ constexpr int gemv_stages(int nb, bool one) { return one && nb == 8 ? 2 : 3; }
constexpr int GEMV_TMAX = 8;     // tokens per launch on the fast path
// tokens per launch at NB super-blocks per row: at 4096 columns eight tokens'
// two activation levels would not fit in shared memory beside the stages
__host__ __device__ constexpr int gemv_tmax(int nb) { return nb >= 16 ? 4 : GEMV_TMAX; }

// warp steps per bulk copy: copies of about 2.3 - 3.5 KB
template <int STEPB>
struct Chunk {
    static constexpr int CH = STEPB >= 3000 ? 1 : (STEPB >= 1500 ? 2 : 3);
};

__host__ __device__ constexpr size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Shared-memory offsets of a launch of T tokens: per level (first, then the
// residual) int16 values [T x cols] in the xq_pos layout, fp32 scales per 32
// and int sums per 16; then the per-warp stages and their mbarriers.
struct GemvLayout {
    size_t xs, xs16, xr, xs2, xr16, st;
    __host__ __device__ GemvLayout(int T, int cols)
    {
        const size_t q = align_up((size_t)T * cols * 2, 16), s = align_up((size_t)T * cols / 32 * 4, 16),
                     s16 = align_up((size_t)T * cols / 16 * 4, 16);
        xs = q;
        xs16 = xs + s;
        xr = xs16 + s16;
        xs2 = xr + q;
        xr16 = xs2 + s;
        st = xr16 + s16;
    }
};

template <int QT, int NB>
struct GemvSmem {
    static constexpr int CH = Chunk<Geo<QT, NB>::STEPB>::CH;
    static constexpr size_t chunk = (size_t)Geo<QT, NB>::STEPB * CH;
    // prow: rows per warp of the two-pass row values
    static size_t bytes(int T, int prow)
    {
        size_t b = GemvLayout(T, Geo<QT, NB>::COLS).st;
        const int ns = gemv_stages(NB, T == 1);
        b += (size_t)GEMV_WARPS * ns * chunk + 16;                             // stages + tail pad
        b = align_up(b, 8) + GEMV_WARPS * ns * 8;                              // mbarriers
        b = align_up(b, 16) + (size_t)GEMV_WARPS * prow * T * 4;               // row values
        return b;
    }
};

// Quantise T x cols activations (fp32 or fp16) into shared memory, both
// levels, four groups per warp at a time (their reductions interleaved);
// returns nonzero on the lanes of a warp that gave some group a second level.
template <bool IN_HALF>
__device__ __forceinline__ int quantise_to_smem(const void *x, int T, int cols, int16_t *xq, float *xs, int *xs16,
                                                int16_t *xr, float *xs2, int *xr16, int warp, int nwarps, int lane)
{
    constexpr int N = 4;
    const int groups = T * cols / 32;
    int two = 0;
    for (int g0 = warp; g0 < groups; g0 += N * nwarps) {
        float v[N];
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const int gi = g0 + k * nwarps;
            const int idx = gi * 32 + lane;
            v[k] = gi >= groups ? 0.0f
                   : IN_HALF    ? __half2float(reinterpret_cast<const __half *>(x)[idx])
                                : reinterpret_cast<const float *>(x)[idx];
        }
        int q[N], r[N];
        float sc[N], s2[N];
        quant32_r_n<N>(v, q, r, sc, s2);
#pragma unroll
        for (int k = 0; k < N; ++k) {
            const int gi = g0 + k * nwarps;
            if (gi >= groups) break;  // (warp-uniform)
            const int idx = gi * 32 + lane;
            const int t = idx / cols, e = idx - t * cols;
            xq[(size_t)t * cols + xq_pos(e)] = (int16_t)q[k];
            const int s16 = sum16(q[k]);
            if (lane == 0) {
                xs[gi] = sc[k];
                xs2[gi] = s2[k];
            }
            if ((lane & 15) == 0) xs16[2 * gi + (lane >> 4)] = s16;
            // (a group without a second level leaves its residual values
            // unwritten: they enter every dot product times its s2 = 0)
            if (s2[k] > 0.0f) {  // (warp-uniform)
                xr[(size_t)t * cols + xq_pos(e)] = (int16_t)r[k];
                const int r16 = sum16(r[k]);
                if ((lane & 15) == 0) xr16[2 * gi + (lane >> 4)] = r16;
                two = 1;
            }
        }
    }
    return two;
}

// Fused greedy sampling (the argmax after the lm-head GEMV that
// greedy_sample, main.cu:324-337, runs on the host over fp16 logits): every
// lane that finishes a row folds it into a running 64-bit key
// {order-preserving value bits, ~row}, so the largest value wins and, among
// equal values, the lowest row (the reference's strict `>` scan).  Each warp
// then posts its best key with one atomicMax; the last warp to arrive (ticket)
// decodes the winner into token/value and re-zeroes the state for the next
// call.  NaN logits never win (the reference's `v > best` skips them).
struct ArgmaxArgs {
    unsigned long long *key;  // state[0]; state[1] low word: arrival ticket
    unsigned *ticket;
    int *token;
    float *value;
    int round_half;           // 1: compare fp16-rounded logits (what greedy_sample sees)
    int finalize;             // 0: another launch arrives after this one and finalises
};
__device__ __forceinline__ unsigned long long am_key(float v, long long row, int round_half)
{
    if (round_half) v = __half2float(__float2half_rn(v));
    if (v != v) return 0ull;
    const uint32_t b = __float_as_uint(v);
    const uint32_t k = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
    return ((unsigned long long)k << 32) | (unsigned long long)(0xFFFFFFFFu - (uint32_t)row);
}
// One warp's arrival (all 32 lanes, each with its best key); n_arrive: warps
// of this launch.
__device__ __forceinline__ void am_arrive(const ArgmaxArgs &am, unsigned long long best, unsigned n_arrive)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const unsigned long long other = __shfl_xor_sync(0xffffffffu, best, o);
        best = other > best ? other : best;
    }
    if ((threadIdx.x & 31) == 0) {
        if (best) atomicMax(am.key, best);
        __threadfence();
        if (am.finalize && atomicAdd(am.ticket, 1u) == n_arrive - 1) {
            __threadfence();
            const unsigned long long k = atomicExch(am.key, 0ull);
            atomicExch(am.ticket, 0u);
            const uint32_t kv = (uint32_t)(k >> 32);
            const uint32_t b = (kv & 0x80000000u) ? (kv & 0x7FFFFFFFu) : ~kv;
            *am.token = k ? (int)(0xFFFFFFFFu - (uint32_t)k) : 0;
            if (am.value) *am.value = k ? __uint_as_float(b) : __int_as_float(0x7fc00000);
        }
    }
}

// One launch: the CTA quantises the activations (both levels) into shared
// memory while its warps' first weight stages are in flight, then every warp
// streams its rows.  A launch in which some group has a second level makes
// two passes over its rows (the weights streamed twice): the first with the
// first level, its row values kept in shared memory (part, `prow` rows per
// warp), the second with the residual level, adding them -- the same loop
// code either way, so the one-level launch runs as without outliers.
template <int QT, int NB, bool ONE_TOKEN, bool IN_HALF, bool OUT_HALF, bool AM = false>
__global__ void __launch_bounds__(GEMV_WARPS * 32, ONE_TOKEN && NB == 8 ? 3 : 1)
gemv_tma_kernel(const uint8_t *__restrict__ W, long long nsteps, const void *__restrict__ x, int T,
                void *__restrict__ y, int rows_total, long long row0, int prow, const ArgmaxArgs am)
{
    using G = Geo<QT, NB>;
    constexpr size_t CHUNK = GemvSmem<QT, NB>::chunk;
    constexpr int GEMV_CH = GemvSmem<QT, NB>::CH;
    constexpr int GEMV_STAGES = gemv_stages(NB, ONE_TOKEN);
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLayout lay(T, G::COLS);
    int16_t *xq = reinterpret_cast<int16_t *>(smem);
    float *xs = reinterpret_cast<float *>(smem + lay.xs);
    int *xs16 = reinterpret_cast<int *>(smem + lay.xs16);
    int16_t *xr = reinterpret_cast<int16_t *>(smem + lay.xr);
    float *xs2 = reinterpret_cast<float *>(smem + lay.xs2);
    int *xr16 = reinterpret_cast<int *>(smem + lay.xr16);
    uint8_t *stages = smem + lay.st;
    const size_t o_bars = align_up(lay.st + (size_t)GEMV_WARPS * GEMV_STAGES * CHUNK + 16, 8);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + o_bars);
    float *parts = reinterpret_cast<float *>(smem + align_up(o_bars + GEMV_WARPS * GEMV_STAGES * 8, 16));

    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint8_t *my_stage = stages + (size_t)warp * GEMV_STAGES * CHUNK;
    uint64_t *my_bar = bars + warp * GEMV_STAGES;
    float *part = parts + (size_t)warp * prow * T;  // [row of the warp][token]

    // this warp's step range
    const long long wtot = (long long)gridDim.x * GEMV_WARPS;
    const long long wid = (long long)blockIdx.x * GEMV_WARPS + warp;
    const long long s0 = wid * nsteps / wtot, s1 = (wid + 1) * nsteps / wtot;
    const int nst = (int)(s1 - s0);
    const int nchunks = (nst + GEMV_CH - 1) / GEMV_CH;

    if (lane == 0) {
        for (int s = 0; s < GEMV_STAGES; ++s) mbar_init(my_bar + s, 1);
        fence_mbar_init();
    }
    __syncwarp();
    // stage sequence position cc (passes one after another): weight chunk cc mod nchunks
    auto issue = [&](int cc) {
        const int c = cc < nchunks ? cc : cc - nchunks;
        const int first = c * GEMV_CH;
        const int n = min(GEMV_CH, nst - first);
        const unsigned bytes = (unsigned)(n * G::STEPB);
        uint64_t *bar = my_bar + (cc % GEMV_STAGES);
        mbar_arrive_expect_tx(bar, bytes);
        bulk_g2s(my_stage + (size_t)(cc % GEMV_STAGES) * CHUNK, W + (s0 + first) * (long long)G::STEPB, bytes, bar);
    };
    if (lane == 0)
        for (int c = 0; c < min(GEMV_STAGES, nchunks); ++c) issue(c);

    // two: some group of the launch has a second level (CTA-uniform)
    const bool two = __syncthreads_or(
        quantise_to_smem<IN_HALF>(x, T, G::COLS, xq, xs, xs16, xr, xs2, xr16, warp, GEMV_WARPS, lane));
    if (two && lane == 0)
        for (int cc = min(GEMV_STAGES, nchunks); cc < min(GEMV_STAGES, 2 * nchunks); ++cc) issue(cc);

    // lane geometry
    const int rho = lane / G::LPR;        // row within the warp step
    const int lr = lane % G::LPR;         // lane within the row
    const int bb = lr >> 2;               // block within the pass
    const int sub = lr & 3;               // Q4_K: pair g; Q6_K: (h, g) = (sub >> 1, sub & 1)
    Q6Lane L6;
    if (QT == BREAD_QTYPE_Q6_K) {
        // byte offset of this lane's block inside a 16-aligned step: 210*k, k = rho*NB + bb (+8 per pass)
        L6 = q6_lane(((rho * NB + bb) & 1) ? 2 : 0, sub & 1);
    }
    auto slice_of = [&](XSlice &X, const int16_t *vq, const float *vs, int t, int cp) {
        const int b = cp * 8 + bb;
        if (QT == BREAD_QTYPE_Q4_K)
            load_slice_q4k(X, vq + (size_t)t * G::COLS, vs + (size_t)t * G::COLS / 32, QK * b + 64 * sub);
        else
            load_slice_q6k(X, vq + (size_t)t * G::COLS, vs + (size_t)t * G::COLS / 32, QK * b + 128 * (sub >> 1),
                           sub & 1);
    };

    unsigned long long best = 0ull;  // AM: this lane's best key
    // The row loop over one activation level.  MODE 0: the only pass (writes
    // the outputs); 1: first of two passes (keeps the row values); 2: second
    // of two (adds the kept values, writes the outputs).  cc0: stage sequence
    // position of the pass's first chunk.
    auto rows = [&](auto mode_c, const int16_t *vq, const float *vs, const int *v16, int cc0) -> bool {
        constexpr int MODE = decltype(mode_c)::value;
        XSlice X1[ONE_TOKEN ? G::CP : 1];
        if (ONE_TOKEN) {
#pragma unroll
            for (int cp = 0; cp < G::CP; ++cp) slice_of(X1[cp], vq, vs, 0, cp);
        }
        for (int c = 0; c < nchunks; ++c) {
            const int cc = MODE == 2 ? c + cc0 : c;
            const int slot = cc % GEMV_STAGES;
            if (!mbar_wait(my_bar + slot, (unsigned)((cc / GEMV_STAGES) & 1))) return false;
            const uint8_t *buf = my_stage + (size_t)slot * CHUNK;
            const int n = min(GEMV_CH, nst - c * GEMV_CH);
            for (int st = 0; st < n; ++st) {
                const int rw = (c * GEMV_CH + st) * G::RPW + rho;  // row within the warp's range
                const long long row = row0 + s0 * G::RPW + rw;
                const uint8_t *rowp = buf + (size_t)st * G::STEPB + (size_t)rho * G::ROWB;
                float acc[ONE_TOKEN ? 1 : GEMV_TMAX];
#pragma unroll
                for (int t = 0; t < (ONE_TOKEN ? 1 : GEMV_TMAX); ++t) acc[t] = 0.0f;
#pragma unroll
                for (int cp = 0; cp < G::CP; ++cp) {
                    const uint8_t *blk = rowp + (size_t)(cp * 8 + bb) * G::BB;
                    if (ONE_TOKEN) {
                        acc[0] += QT == BREAD_QTYPE_Q4_K ? q4k_lane_dot(blk, sub, X1[cp])
                                                         : q6k_lane_dot(blk, sub >> 1, sub & 1, L6, X1[cp]);
                    } else if (QT == BREAD_QTYPE_Q4_K) {
                        // several tokens: decode the lane's weights once, then one
                        // dot per token from its slice in shared memory
                        Q4W Wd;
                        q4k_lane_w(Wd, blk, sub);
                        const int e0 = QK * (cp * 8 + bb) + 64 * sub;
#pragma unroll
                        for (int t = 0; t < GEMV_TMAX; ++t)
                            if (t < T)
                                acc[t] += q4k_dot_w(Wd, vq + (size_t)t * G::COLS, vs + (size_t)t * G::COLS / 32,
                                                    v16 + (size_t)t * G::COLS / 16, e0, 1.0f);
                    } else {
                        Q6W Wd;
                        q6k_lane_w(Wd, blk, sub >> 1, sub & 1, L6);
                        const int base = QK * (cp * 8 + bb) + 128 * (sub >> 1);
#pragma unroll
                        for (int t = 0; t < GEMV_TMAX; ++t)
                            if (t < T)
                                acc[t] += q6k_dot_w(Wd, vq + (size_t)t * G::COLS, vs + (size_t)t * G::COLS / 32,
                                                    v16 + (size_t)t * G::COLS / 16, base, sub & 1, 1.0f);
                    }
                }
#pragma unroll
                for (int t = 0; t < (ONE_TOKEN ? 1 : GEMV_TMAX); ++t) {
                    if (ONE_TOKEN || t < T) {
                        float v = acc[t];
#pragma unroll
                        for (int o = G::LPR / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                        if (lr == 0) {
                            if (MODE == 1) {
                                part[(size_t)rw * T + t] = v;
                                continue;
                            }
                            if (MODE == 2) v += part[(size_t)rw * T + t];
                            const size_t oi = (size_t)t * rows_total + row;
                            if (AM) {
                                const unsigned long long k = am_key(v, row, am.round_half);
                                best = k > best ? k : best;
                                if (y) reinterpret_cast<float *>(y)[oi] = v;
                            } else if (OUT_HALF) {
                                reinterpret_cast<__half *>(y)[oi] = __float2half_rn(v);
                            } else {
                                reinterpret_cast<float *>(y)[oi] = v;
                            }
                        }
                    }
                }
            }
            __syncwarp();
            if (lane == 0 && cc + GEMV_STAGES < (MODE == 0 ? nchunks : 2 * nchunks)) {
                fence_proxy_async_smem();
                issue(cc + GEMV_STAGES);
            }
        }
        return true;
    };
    if (!two) {
        if (!rows(std::integral_constant<int, 0>{}, xq, xs, xs16, 0)) return;
    } else {
        if (!rows(std::integral_constant<int, 1>{}, xq, xs, xs16, 0)) return;
        if (!rows(std::integral_constant<int, 2>{}, xr, xs2, xr16, nchunks)) return;
    }
    if (AM) am_arrive(am, best, gridDim.x * GEMV_WARPS);
}

// One warp per row; exact element dequantisation; any alignment.
template <int QT, bool IN_HALF, bool OUT_HALF, bool AM = false>
__global__ void gemv_generic_kernel(const uint8_t *__restrict__ W, int row0, int rows, int cols, const void *x, int T,
                                    void *y, int rows_total, const ArgmaxArgs am)
{
    constexpr int BE = QT == BREAD_QTYPE_Q8_0 ? Q80_ELEMS : QK;
    constexpr int BBY = QT == BREAD_QTYPE_Q4_K ? Q4K_BYTES : QT == BREAD_QTYPE_Q6_K ? Q6K_BYTES : Q80_BYTES;
    const int lane = threadIdx.x & 31;
    const int wpb = blockDim.x >> 5;
    const int nb = cols / BE;
    unsigned long long best = 0ull;  // AM: lane 0's best key
    for (int r = blockIdx.x * wpb + (threadIdx.x >> 5); r < rows; r += gridDim.x * wpb) {
        const int row = row0 + r;
        const uint8_t *rp = W + (size_t)row * nb * BBY;
        for (int t = 0; t < T; ++t) {
            float acc = 0.0f;
            for (int e = lane; e < cols; e += 32) {
                const float w = elem_exact<QT>(rp + (size_t)(e / BE) * BBY, e % BE);
                const size_t xi = (size_t)t * cols + e;
                const float xv = IN_HALF ? __half2float(reinterpret_cast<const __half *>(x)[xi])
                                         : reinterpret_cast<const float *>(x)[xi];
                acc = fmaf(w, xv, acc);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
            if (lane == 0) {
                const size_t oi = (size_t)t * rows_total + row;
                if (AM) {
                    const unsigned long long k = am_key(acc, row, am.round_half);
                    best = k > best ? k : best;
                    if (y) reinterpret_cast<float *>(y)[oi] = acc;
                } else if (OUT_HALF) {
                    reinterpret_cast<__half *>(y)[oi] = __float2half_rn(acc);
                } else {
                    reinterpret_cast<float *>(y)[oi] = acc;
                }
            }
        }
    }
    if (AM) am_arrive(am, best, gridDim.x * wpb);
}

// Bit-exact block dequantisation: one warp per block.
template <int QT>
__global__ void dequant_kernel(const uint8_t *__restrict__ W, float *__restrict__ out, long long n_blocks)
{
    constexpr int BE = QT == BREAD_QTYPE_Q8_0 ? Q80_ELEMS : QK;
    constexpr int BBY = QT == BREAD_QTYPE_Q4_K ? Q4K_BYTES : QT == BREAD_QTYPE_Q6_K ? Q6K_BYTES : Q80_BYTES;
    const int lane = threadIdx.x & 31;
    const long long wpb = blockDim.x >> 5;
    for (long long b = blockIdx.x * wpb + (threadIdx.x >> 5); b < n_blocks; b += (long long)gridDim.x * wpb) {
        const uint8_t *blk = W + b * BBY;
        for (int e = lane; e < BE; e += 32) out[b * BE + e] = elem_exact<QT>(blk, e);
    }
}

// ---------------------------------------------------------------------------
// host dispatch
// ---------------------------------------------------------------------------
constexpr size_t GEMV_SMEM_MAX = 232448;  // dynamic shared memory per CTA (227 KB)

// One matrix, in pieces of rows when the two-pass row values of a piece
// would not fit in shared memory (only for very tall matrices); with AM only
// the last piece finalises.
template <int QT, int NB, bool ONE, bool IH, bool OH, bool AM = false>
static int launch_fast(const uint8_t *W, long long nsteps, const void *x, int T, void *y, int rows_total,
                       cudaStream_t stream, const ArgmaxArgs &am = ArgmaxArgs{})
{
    using G = Geo<QT, NB>;
    auto kern = gemv_tma_kernel<QT, NB, ONE, IH, OH, AM>;
    if (T > (ONE ? 1 : gemv_tmax(NB))) return set_error(BREAD_ERR_ARG, "gemv: %d tokens in one launch at %d columns", T, NB * QK);
    static int per_sm = 0;  // per instantiation: CTAs per SM without the row values
    if (!per_sm) {
        BREAD_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)GEMV_SMEM_MAX),
                   "gemv: set smem attribute");
        int n = 1;
        BREAD_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, GEMV_WARPS * 32,
                                                                 GemvSmem<QT, NB>::bytes(ONE ? 1 : gemv_tmax(NB), 0)),
                   "gemv occupancy");
        per_sm = n < 1 ? 1 : n;
    }
    const size_t base = GemvSmem<QT, NB>::bytes(T, 0) + 16;
    const long long steps_fit = base < GEMV_SMEM_MAX ? (long long)((GEMV_SMEM_MAX - base) / ((size_t)GEMV_WARPS * T * 4)) / G::RPW : 0;
    if (steps_fit < 1) return set_error(BREAD_ERR_ARG, "gemv: %d tokens at %d columns exceed shared memory", T, NB * QK);
    const long long cap = (long long)sm_count() * per_sm;
    for (long long done = 0; done < nsteps;) {
        long long ns = nsteps - done;
        const long long want = (ns + GEMV_WARPS - 1) / GEMV_WARPS;
        const int grid = (int)(want < cap ? want : cap);
        const long long wtot = (long long)grid * GEMV_WARPS;
        long long per_warp = (ns + wtot - 1) / wtot;  // steps of the busiest warp
        if (per_warp > steps_fit) {
            per_warp = steps_fit;
            ns = per_warp * wtot;
        }
        ArgmaxArgs piece = am;
        if (done + ns < nsteps) piece.finalize = 0;
        const int prow = (int)(per_warp * G::RPW);
        kern<<<grid, GEMV_WARPS * 32, GemvSmem<QT, NB>::bytes(T, prow), stream>>>(
            W + done * G::STEPB, ns, x, T, y, rows_total, done * G::RPW, prow, piece);
        BREAD_CUDA(cudaGetLastError(), "gemv fast launch");
        done += ns;
    }
    return BREAD_OK;
}

template <int QT, bool IH, bool OH, bool AM = false>
static int launch_generic(const uint8_t *W, int row0, int rows, int cols, const void *x, int T, void *y,
                          int rows_total, cudaStream_t stream, const ArgmaxArgs &am = ArgmaxArgs{})
{
    if (rows <= 0) return BREAD_OK;
    const int warps = 8;
    long long want = ((long long)rows + warps - 1) / warps;
    const long long cap = (long long)sm_count() * 8;
    const int grid = (int)(want < cap ? want : cap);
    gemv_generic_kernel<QT, IH, OH, AM><<<grid, warps * 32, 0, stream>>>(W, row0, rows, cols, x, T, y, rows_total, am);
    BREAD_CUDA(cudaGetLastError(), "gemv generic launch");
    return BREAD_OK;
}

// AM (argmax, one fp32 token): the launch that runs last finalises.
template <int QT, bool IH, bool OH, bool AM = false>
static int gemv_dispatch_q(const uint8_t *W, int rows, int cols, const void *x, int T, void *y, cudaStream_t stream,
                           const ArgmaxArgs &am = ArgmaxArgs{})
{
    const int nb = cols / QK;
    const bool aligned = (reinterpret_cast<uintptr_t>(W) & 15) == 0;
    int rpw = 0;
    if (aligned && (nb == 1 || nb == 2 || nb == 4 || nb == 8 || nb == 16)) rpw = nb >= 8 ? 1 : 8 / nb;
    if (!rpw) return launch_generic<QT, IH, OH, AM>(W, 0, rows, cols, x, T, y, rows, stream, am);
    const long long nsteps = rows / rpw;
    const int rows_main = (int)(nsteps * rpw);
    ArgmaxArgs am_fast = am;
    if (rows_main < rows) am_fast.finalize = 0;  // the generic tail launch finalises
    if (nsteps > 0) {
        int st = BREAD_OK;
        const bool one = T == 1;
#define BREAD_FAST(NB_)                                                                                         \
    case NB_:                                                                                                   \
        st = AM    ? launch_fast<QT, NB_, true, IH, OH, AM>(W, nsteps, x, T, y, rows, stream, am_fast)          \
             : one ? launch_fast<QT, NB_, true, IH, OH>(W, nsteps, x, T, y, rows, stream)                       \
                   : launch_fast<QT, NB_, false, IH, OH>(W, nsteps, x, T, y, rows, stream);                    \
        break;
        switch (nb) {
            BREAD_FAST(1)
            BREAD_FAST(2)
            BREAD_FAST(4)
            BREAD_FAST(8)
            BREAD_FAST(16)
        default: break;
        }
#undef BREAD_FAST
        if (st != BREAD_OK) return st;
    }
    return launch_generic<QT, IH, OH, AM>(W, rows_main, rows - rows_main, cols, x, T, y, rows, stream, am);
}

// y[T x rows] = x[T x cols] * W^T for T <= GEMV_TMAX.
template <bool IH, bool OH>
static int gemv_any(const void *w, int qtype, int rows, int cols, const void *x, int T, void *y, cudaStream_t stream)
{
    const uint8_t *W = static_cast<const uint8_t *>(w);
    switch (qtype) {
    case BREAD_QTYPE_Q4_K: return gemv_dispatch_q<BREAD_QTYPE_Q4_K, IH, OH>(W, rows, cols, x, T, y, stream);
    case BREAD_QTYPE_Q6_K: return gemv_dispatch_q<BREAD_QTYPE_Q6_K, IH, OH>(W, rows, cols, x, T, y, stream);
    case BREAD_QTYPE_Q8_0: return launch_generic<BREAD_QTYPE_Q8_0, IH, OH>(W, 0, rows, cols, x, T, y, rows, stream);
    default: return set_error(BREAD_ERR_QTYPE, "unknown qtype %d", qtype);
    }
}

static int check_gemv_args(const void *w, const void *x, const void *y, int rows, int cols, int qtype, int T)
{
    if (!w || !x || !y) return set_error(BREAD_ERR_ARG, "matvec: NULL pointer");
    const int be = block_elems(qtype);
    if (!block_bytes(qtype)) return set_error(BREAD_ERR_QTYPE, "matvec: unknown qtype %d", qtype);
    if (rows <= 0 || cols <= 0 || cols % be) return set_error(BREAD_ERR_ARG, "matvec: rows=%d cols=%d (cols must be a positive multiple of %d)", rows, cols, be);
    if (T < 1 || T > 64) return set_error(BREAD_ERR_ARG, "matvec: T=%d outside 1..64", T);
    if (reinterpret_cast<uintptr_t>(x) & 3) return set_error(BREAD_ERR_ALIGN, "matvec: x not 4-byte aligned");
    return BREAD_OK;
}

}  // namespace bread

using namespace bread;

extern "C" int bread_matvec_f32(const void *w, const float *x, float *y, int rows, int cols, int qtype,
                                cudaStream_t stream)
{
    BREAD_TRY(check_gemv_args(w, x, y, rows, cols, qtype, 1));
    return gemv_any<false, false>(w, qtype, rows, cols, x, 1, y, stream);
}

extern "C" int bread_matvec_f16(const void *w, const void *x, void *y, int rows, int cols, int qtype,
                                cudaStream_t stream)
{
    if (!w || !x || !y) return set_error(BREAD_ERR_ARG, "matvec: NULL pointer");
    if (!block_bytes(qtype)) return set_error(BREAD_ERR_QTYPE, "unknown qtype %d", qtype);
    if (rows <= 0 || cols <= 0 || cols % block_elems(qtype)) return set_error(BREAD_ERR_ARG, "matvec: rows=%d cols=%d", rows, cols);
    if (reinterpret_cast<uintptr_t>(x) & 1) return set_error(BREAD_ERR_ALIGN, "matvec: x not 2-byte aligned");
    return gemv_any<true, true>(w, qtype, rows, cols, x, 1, y, stream);
}

extern "C" int bread_matvec_batch_f32(const void *w, const float *x, float *y, int rows, int cols, int qtype, int T,
                                      cudaStream_t stream)
{
    BREAD_TRY(check_gemv_args(w, x, y, rows, cols, qtype, T));
    // token chunks (8, or 4 at 4096 columns): each chunk streams the weights once
    const int tc = gemv_tmax(cols / QK);
    for (int t0 = 0; t0 < T; t0 += tc) {
        const int n = T - t0 < tc ? T - t0 : tc;
        BREAD_TRY(gemv_any<false, false>(w, qtype, rows, cols, x + (size_t)t0 * cols, n, y + (size_t)t0 * rows,
                                         stream));
    }
    return BREAD_OK;
}

extern "C" int bread_lm_head_argmax(const void *w, const float *x, int rows, int cols, int qtype, int round_half,
                                    float *logits, int *token, float *value, void *state, cudaStream_t stream)
{
    if (!w || !x || !token || !state) return set_error(BREAD_ERR_ARG, "lm_head_argmax: NULL pointer");
    if (qtype != BREAD_QTYPE_Q4_K && qtype != BREAD_QTYPE_Q6_K && qtype != BREAD_QTYPE_Q8_0)
        return set_error(BREAD_ERR_QTYPE, "lm_head_argmax: unknown qtype %d", qtype);
    if (rows <= 0 || cols <= 0 || cols % block_elems(qtype))
        return set_error(BREAD_ERR_ARG, "lm_head_argmax: rows=%d cols=%d", rows, cols);
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(state)) & 7)
        return set_error(BREAD_ERR_ALIGN, "lm_head_argmax: x and state must be 8-byte aligned");
    ArgmaxArgs am;
    am.key = static_cast<unsigned long long *>(state);
    am.ticket = reinterpret_cast<unsigned *>(am.key + 1);
    am.token = token;
    am.value = value;
    am.round_half = round_half ? 1 : 0;
    am.finalize = 1;
    const uint8_t *W = static_cast<const uint8_t *>(w);
    switch (qtype) {
    case BREAD_QTYPE_Q4_K:
        return gemv_dispatch_q<BREAD_QTYPE_Q4_K, false, false, true>(W, rows, cols, x, 1, logits, stream, am);
    case BREAD_QTYPE_Q6_K:
        return gemv_dispatch_q<BREAD_QTYPE_Q6_K, false, false, true>(W, rows, cols, x, 1, logits, stream, am);
    default:
        return launch_generic<BREAD_QTYPE_Q8_0, false, false, true>(W, 0, rows, cols, x, 1, logits, rows, stream, am);
    }
}

extern "C" int bread_dequant(const void *w, float *out, long long n_blocks, int qtype, cudaStream_t stream)
{
    if (!w || !out || n_blocks < 0) return set_error(BREAD_ERR_ARG, "dequant: bad argument");
    if (n_blocks == 0) return BREAD_OK;
    const long long want = (n_blocks + 7) / 8;
    const long long cap = (long long)sm_count() * 16;
    const int grid = (int)(want < cap ? want : cap);
    const uint8_t *W = static_cast<const uint8_t *>(w);
    switch (qtype) {
    case BREAD_QTYPE_Q4_K: dequant_kernel<BREAD_QTYPE_Q4_K><<<grid, 256, 0, stream>>>(W, out, n_blocks); break;
    case BREAD_QTYPE_Q6_K: dequant_kernel<BREAD_QTYPE_Q6_K><<<grid, 256, 0, stream>>>(W, out, n_blocks); break;
    case BREAD_QTYPE_Q8_0: dequant_kernel<BREAD_QTYPE_Q8_0><<<grid, 256, 0, stream>>>(W, out, n_blocks); break;
    default: return set_error(BREAD_ERR_QTYPE, "dequant: unknown qtype %d", qtype);
    }
    BREAD_CUDA(cudaGetLastError(), "dequant launch");
    return BREAD_OK;
}

// Drop-in for kernels.cu:289 (C++ linkage, same signature): aborts on error
// like the reference's CUDA_CHECK / unknown-qtype exit.
void bread_matvec(void *w, half *x, half *y, int rows, int cols, int qtype, cudaStream_t stream)
{
    const int st = bread_matvec_f16(w, x, y, rows, cols, qtype, stream);
    if (st != BREAD_OK) {
        fprintf(stderr, "bread_matvec: %s (%s)\n", bread_status_string(st), bread_last_error());
        exit(1);
    }
}
