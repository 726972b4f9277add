// moe.cu -- the MoE FFN block on sm_100a: device router with top-k (K1), one
// grouped gate/up + SiLU*mul launch over every active expert (K2), one grouped
// down launch fused with the router-weighted combine (K3), and the
// expert-parallel combine.
//
// Reference path replaced: route_layer (one_layer.cu:937-992, with
// cpu_softmax/cpu_topk layer_ops.cu:222-250), the shared expert
// (one_layer.cu:1840-1894) and the serial expert loop (one_layer.cu:1931-1983:
// per expert bread_matvec gate, up, silu_mul_inplace, bread_matvec down,
// scale_accum).
//
// Data flow for T tokens (all in the caller's workspace):
//   K1  CTAs of 2 router rows x 4 tokens: quantise a slice of x to int16 (+ per
//       group sums of squares) and compute their logits (fp32, fixed-order
//       reduction).  The last CTA to finish (atomic ticket) does softmax and
//       top-k per token, groups the (token, slot) pairs by expert -- group 0
//       is the shared expert, then routed experts by ascending id -- and
//       writes a table of chunks (<= 8 pairs of one expert) holding resolved
//       weight pointers, tokens and weights, so the expert kernels start
//       their copies after a single table read.
//   K2  persistent CTAs walk items (chunk, 32-row tile): a producer warp bulk
//       copies the chunk record and its tokens' int16 activations, and the 32
//       gate + 32 up rows in sub-stages; 8 consumer warps compute silu(g)*u
//       and quantise the 32 results (one activation group) to int16.
//   K3  CTAs own 16 output rows: the producer streams, per chunk, those rows
//       of the chunk's down matrix together with the chunk's intermediate;
//       consumers accumulate w * result per (token, row) in per-warp shared
//       memory, summed in fixed warp order at the end: deterministic, no
//       atomics.
// All kernels are launched with programmatic dependent launch: each one
// issues the work that does not depend on its predecessor (router rows in K1,
// shared-expert rows in K2, down rows in K3) before griddepcontrol.wait.
#include <math.h>

#include <utility>

#include "common.cuh"
#include "moe.cuh"
#include "ptx.cuh"
#include "qdot.cuh"

namespace bread {

template <int QT, int NB>
struct MGeo {
    static constexpr int BB = QT == BREAD_QTYPE_Q4_K ? Q4K_BYTES : Q6K_BYTES;
    static constexpr int LANES_ALL = 4 * NB;
    static constexpr int CP = LANES_ALL > 32 ? LANES_ALL / 32 : 1;
    static constexpr int LPR = LANES_ALL > 32 ? 32 : LANES_ALL;
    static constexpr int RPW = 32 / LPR;
    static constexpr int ROWB = BB * NB;
    static constexpr int STEPB = ROWB * RPW;
};

constexpr size_t CHUNK_HDR = 128;  // chunk record at the head of a staged slot

__host__ __device__ constexpr size_t al16(size_t v) { return (v + 15) / 16 * 16; }

__device__ __forceinline__ float warp_sum(float v)
{
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// ---------------------------------------------------------------------------
// K1: router + finalize
// ---------------------------------------------------------------------------
constexpr int K1_ROWS = 2;                  // router rows per CTA (4 warps per row)
constexpr int K1_MAXV = MOE_HMAX / 4 / 64;  // float2 per lane of a quarter row

// Runs in the last K1 CTA to finish (256 threads).  It sits between the router
// GEMV and the expert kernels, so global inputs are read in one round of
// independent loads and all intermediate state stays in shared memory.
__device__ void moe_finalize(const MoeArgs &a)
{
    __shared__ int s_cnt[MOE_EMAX], s_run[MOE_EMAX], s_off[MOE_EMAX];
    __shared__ int s_gexp[MOE_EMAX + 1], s_goff[MOE_EMAX + 1], s_gcnt[MOE_EMAX + 1], s_gcpre[MOE_EMAX + 2];
    __shared__ float s_rinv[MOE_TMAX], s_sgw[MOE_TMAX];
    __shared__ int s_idx[MOE_TMAX * MOE_KMAX];
    __shared__ float s_w[MOE_TMAX * MOE_KMAX];
    __shared__ int s_ptok[MOE_TMAX * (MOE_KMAX + 1)];
    __shared__ float s_pw[MOE_TMAX * (MOE_KMAX + 1)];
    __shared__ int s_ng, s_nch, s_np;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = a.T, H = a.H, E = a.E, K = a.top_k, HG = H / 32;
    for (int i = tid; i < MOE_EMAX; i += blockDim.x) {
        s_cnt[i] = 0;
        s_run[i] = 0;
    }

    // (a) per token (one warp each): RMS factor, softmax, top-k
    //     (layer_ops.cu:222-250), renormalised weights, shared-gate sigmoid
    constexpr int PER = MOE_EMAX / 32;
    for (int t = warp; t < T; t += 8) {
        float p[PER];
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int e = lane + 32 * j;
            p[j] = e < E ? __ldcg(a.logits + (size_t)t * E + e) : -INFINITY;
        }
        float ss = 0.0f;
        for (int g = lane; g < HG; g += 32) ss += __ldcg(a.ssq + t * HG + g);
        const float score = __ldcg(a.score + t);
        ss = warp_sum(ss);
        const float r = a.norm_eps >= 0.0f ? rsqrtf(ss / (float)H + a.norm_eps) : 1.0f;
        float m = -INFINITY;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            p[j] *= r;
            m = fmaxf(m, p[j]);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
        float s = 0.0f;
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            p[j] = (lane + 32 * j) < E ? expf(p[j] - m) : 0.0f;
            s += p[j];
        }
        s = warp_sum(s);
#pragma unroll
        for (int j = 0; j < PER; ++j) p[j] = (lane + 32 * j) < E ? p[j] / s : -1.0f;
        unsigned used = 0;
        float wsum = 0.0f, my_w = 0.0f;
        int my_i = 0;
        for (int k = 0; k < K; ++k) {
            float bv = -1e30f;
            int bi = 0x7fffffff;
#pragma unroll
            for (int j = 0; j < PER; ++j)
                if (!((used >> j) & 1u) && p[j] > bv) {
                    bv = p[j];
                    bi = lane + 32 * j;
                }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
                const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
                if (ov > bv || (ov == bv && oi < bi)) {
                    bv = ov;
                    bi = oi;
                }
            }
            if ((bi & 31) == lane) used |= 1u << (bi >> 5);
            if (lane == k) {
                my_w = bv;
                my_i = bi;
            }
            wsum += bv;
        }
        if (lane < K) {
            const float w = wsum > 0.0f ? my_w / wsum : my_w;
            s_idx[t * K + lane] = my_i;
            s_w[t * K + lane] = w;
            a.ridx[t * K + lane] = my_i;
            a.rw[t * K + lane] = w;
            if (a.idx_out) a.idx_out[t * K + lane] = my_i;
            if (a.w_out) a.w_out[t * K + lane] = w;
        }
        if (lane == 0) {
            const float sg = a.w_sg ? 1.0f / (1.0f + expf(-(score * r))) : 0.5f;
            s_rinv[t] = r;
            s_sgw[t] = sg;
            a.sgw[t] = sg;
            if (a.sg_out) a.sg_out[t] = sg;
        }
    }
    __syncthreads();

    // (b) scales of the normalised activations; pairs per local expert
    if (a.norm_eps >= 0.0f)
        for (int i = tid; i < T * HG; i += blockDim.x) a.xs[i] = __ldcg(a.xs + i) * s_rinv[i / HG];
    const int P = T * K;
    for (int q = tid; q < P; q += blockDim.x) {
        const int e = s_idx[q];
        if (e >= a.lo && e < a.hi) atomicAdd(&s_cnt[e - a.lo], 1);
    }
    __syncthreads();

    // (c) one warp: groups (shared expert first, then routed experts by id),
    //     chunk prefix, pair placement (token-major inside each expert)
    if (warp == 0) {
        const int NL = a.hi - a.lo;
        const int hs = a.shared_here ? 1 : 0;
        int gbase = hs, pbase = hs ? T : 0;
        if (hs && lane == 0) {
            s_gexp[0] = E;
            s_goff[0] = 0;
            s_gcnt[0] = T;
        }
        for (int c0 = 0; c0 < NL; c0 += 32) {
            const int el = c0 + lane;
            const int cnt = el < NL ? s_cnt[el] : 0;
            const int flag = cnt > 0 ? 1 : 0;
            int fi = flag, ci = cnt;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int f = __shfl_up_sync(0xffffffffu, fi, o);
                const int c = __shfl_up_sync(0xffffffffu, ci, o);
                if (lane >= o) {
                    fi += f;
                    ci += c;
                }
            }
            const int gid = gbase + fi - flag, off = pbase + ci - cnt;
            if (flag) {
                s_gexp[gid] = a.lo + el;
                s_goff[gid] = off;
                s_gcnt[gid] = cnt;
            }
            if (el < NL) s_off[el] = off;
            gbase += __shfl_sync(0xffffffffu, fi, 31);
            pbase += __shfl_sync(0xffffffffu, ci, 31);
        }
        __syncwarp();
        const int ng = gbase;
        int cbase = 0;
        for (int g0 = 0; g0 < ng; g0 += 32) {
            const int g = g0 + lane;
            const int ch = g < ng ? (s_gcnt[g] + MOE_TC - 1) / MOE_TC : 0;
            int ci = ch;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int c = __shfl_up_sync(0xffffffffu, ci, o);
                if (lane >= o) ci += c;
            }
            if (g < ng) s_gcpre[g] = cbase + ci - ch;
            cbase += __shfl_sync(0xffffffffu, ci, 31);
        }
        for (int q0 = 0; q0 < P; q0 += 32) {
            const int q = q0 + lane;
            int e = -1;
            bool loc = false;
            if (q < P) {
                e = s_idx[q];
                loc = e >= a.lo && e < a.hi;
            }
            const unsigned act = __ballot_sync(0xffffffffu, loc);
            if (loc) {
                const unsigned peers = __match_any_sync(act, e);
                const int rank = __popc(peers & ((1u << lane) - 1u));
                const int el = e - a.lo;
                const int pos = s_off[el] + s_run[el] + rank;
                s_ptok[pos] = q / K;
                s_pw[pos] = s_w[q];
                if (__ffs(peers) - 1 == lane) s_run[el] += __popc(peers);
            }
            __syncwarp();
        }
        if (hs)
            for (int t = lane; t < T; t += 32) {
                s_ptok[t] = t;
                s_pw[t] = s_sgw[t];
            }
        if (lane == 0) {
            s_gcpre[ng] = cbase;
            s_ng = ng;
            s_nch = cbase;
            s_np = pbase;
        }
    }
    __syncthreads();

    // (d) all threads: pair lists and the chunk table
    const int ng = s_ng, nch = s_nch, np_tot = s_np;
    for (int p = tid; p < np_tot; p += blockDim.x) {
        a.p_token[p] = s_ptok[p];
        a.p_w[p] = s_pw[p];
    }
    // (route-only calls have no expert tables and need no chunk table)
    for (int c = tid; a.gate && c < nch; c += blockDim.x) {
        int lo = 0, hi = ng - 1;
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (s_gcpre[mid] <= c)
                lo = mid;
            else
                hi = mid - 1;
        }
        const int g = lo, ci = c - s_gcpre[g], e = s_gexp[g];
        MoeChunk ch;
        ch.gate = e >= E ? a.sh_gate : a.gate[e];
        ch.up = e >= E ? a.sh_up : a.up[e];
        ch.down = e >= E ? a.sh_down : a.down[e];
        ch.p0 = s_goff[g] + MOE_TC * ci;
        ch.np = min(MOE_TC, s_gcnt[g] - MOE_TC * ci);
        ch.group = g;
        ch.pad = 0;
#pragma unroll
        for (int j = 0; j < MOE_TC; ++j) {
            ch.tok[j] = (uint8_t)(j < ch.np ? s_ptok[ch.p0 + j] : 0);
            ch.w[j] = j < ch.np ? s_pw[ch.p0 + j] : 0.0f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) ch.pad2[j] = 0;
        const uint4 *src = reinterpret_cast<const uint4 *>(&ch);
        uint4 *dst = reinterpret_cast<uint4 *>(a.chunks + c);
#pragma unroll
        for (int j = 0; j < (int)(sizeof(MoeChunk) / 16); ++j) dst[j] = src[j];
    }
    if (tid == 0) {
        a.hdr[HDR_NGROUPS] = ng;
        a.hdr[HDR_NCHUNKS] = nch;
        a.hdr[HDR_NPAIRS] = np_tot;
        if (a.stats) {
            a.stats[0] = ng;
            a.stats[1] = np_tot;
        }
        a.hdr[HDR_TICKET] = 0;  // re-armed for the next launch
    }
}

__global__ void __launch_bounds__(256) moe_route_kernel(MoeArgs a)
{
    __shared__ float s_part[K1_ROWS][4][K1_TG];
    __shared__ int s_last;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = a.T, H = a.H, E = a.E;
    const int nrows = E + (a.w_sg ? 1 : 0);
    const int rl = warp >> 2, qt = warp & 3;
    const int row = blockIdx.x * K1_ROWS + rl;
    const int seg = H >> 2, nv = seg >> 6;  // float2 per lane
    const int c0 = qt * seg + 2 * lane;

    // The router row does not depend on the previous kernel: load it first.
    float2 wv[K1_MAXV];
#pragma unroll
    for (int j = 0; j < K1_MAXV; ++j) {
        wv[j] = make_float2(0.0f, 0.0f);
        if (j < nv && row < nrows) {
            const int c = c0 + 64 * j;
            if (row < E)
                wv[j] = *reinterpret_cast<const float2 *>(a.W_r + (size_t)row * H + c);
            else
                wv[j] = __half22float2(*reinterpret_cast<const __half2 *>(a.w_sg + c));
        }
    }
    pdl_wait();
    pdl_launch_dependents();

    // quantise x: T*H/32 groups over all warps of the grid
    {
        const int groups = T * (H / 32);
        const int nw = gridDim.x * gridDim.y * 8;
        for (int gi = (blockIdx.y * gridDim.x + blockIdx.x) * 8 + warp; gi < groups; gi += nw) {
            const float v = a.x[(size_t)gi * 32 + lane];
            const float ss = warp_sum(v * v);
            if (lane == 0) a.ssq[gi] = ss;
            const int q = quant32(v, a.xs + gi, lane);
            a.xq[(size_t)gi * 32 + lane] = (int16_t)q;
        }
    }
    // logits of this CTA's rows for its tokens, two tokens per pass
    const int t0 = blockIdx.y * K1_TG;
    const int tn = min(K1_TG, T - t0);
    if (row < nrows) {
        for (int tl = 0; tl < tn; tl += 2) {
            const bool two = tl + 1 < tn;
            const float *x0 = a.x + (size_t)(t0 + tl) * H;
            const float *x1 = two ? x0 + H : x0;
            float2 xa[K1_MAXV], xb[K1_MAXV];
#pragma unroll
            for (int j = 0; j < K1_MAXV; ++j)
                if (j < nv) {
                    xa[j] = *reinterpret_cast<const float2 *>(x0 + c0 + 64 * j);
                    xb[j] = *reinterpret_cast<const float2 *>(x1 + c0 + 64 * j);
                }
            float s0 = 0.0f, s1 = 0.0f;
#pragma unroll
            for (int j = 0; j < K1_MAXV; ++j)
                if (j < nv) {
                    s0 = fmaf(wv[j].x, xa[j].x, s0);
                    s0 = fmaf(wv[j].y, xa[j].y, s0);
                    s1 = fmaf(wv[j].x, xb[j].x, s1);
                    s1 = fmaf(wv[j].y, xb[j].y, s1);
                }
            s0 = warp_sum(s0);
            s1 = warp_sum(s1);
            if (lane == 0) {
                s_part[rl][qt][tl] = s0;
                if (two) s_part[rl][qt][tl + 1] = s1;
            }
        }
    }
    __syncthreads();
    for (int i = tid; i < K1_ROWS * tn; i += blockDim.x) {
        const int r_l = i / tn, tl = i % tn;
        const int rr = blockIdx.x * K1_ROWS + r_l;
        if (rr < nrows) {
            const float v = ((s_part[r_l][0][tl] + s_part[r_l][1][tl]) + s_part[r_l][2][tl]) + s_part[r_l][3][tl];
            if (rr < E)
                a.logits[(size_t)(t0 + tl) * E + rr] = v;
            else
                a.score[t0 + tl] = v;
        }
    }
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const unsigned total = gridDim.x * gridDim.y;
        const unsigned prev = atomicAdd(reinterpret_cast<unsigned *>(a.hdr + HDR_TICKET), 1u);
        s_last = prev == total - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    moe_finalize(a);
}

// ---------------------------------------------------------------------------
// K2: gate/up + SiLU*mul
// ---------------------------------------------------------------------------
template <int NB>
struct K2Cfg {
    using G = MGeo<BREAD_QTYPE_Q4_K, NB>;
    static constexpr int H = QK * NB;
    static constexpr int SR = 8 * G::RPW < MOE_ROWTILE ? 8 * G::RPW : MOE_ROWTILE;  // rows per sub-stage
    static constexpr int SPI = MOE_ROWTILE / SR;                                      // sub-stages per item
    static constexpr int STB = 2 * SR * G::ROWB;                                      // gate rows + up rows
    static constexpr int NS = NB >= 16 ? 2 : 4;                                       // weight sub-stage ring
    static constexpr size_t X_OFF = (size_t)NS * STB;
    // activation slot: chunk record, then up to 8 token rows of int16, then their scales
    __host__ __device__ static int tc(int T) { return T < MOE_TC ? T : MOE_TC; }
    __host__ __device__ static size_t xslot(int T) { return al16(CHUNK_HDR + (size_t)tc(T) * (H * 2 + H / 8)); }
    __host__ __device__ static size_t bar_off(int T) { return X_OFF + 2 * xslot(T) + 16; }
    __host__ __device__ static size_t abuf_off(int T) { return bar_off(T) + (size_t)(2 * NS + 4) * 8; }
    __host__ __device__ static size_t smem(int T) { return abuf_off(T) + MOE_TC * MOE_ROWTILE * 4; }
};

template <int NB>
__global__ void __launch_bounds__(288) moe_gateup_kernel(MoeArgs a)
{
    using C = K2Cfg<NB>;
    using G = typename C::G;
    constexpr int H = C::H;
    extern __shared__ __align__(128) uint8_t smem[];
    const int T = a.T;
    const int TC = C::tc(T);
    const size_t XSLOT = C::xslot(T);
    uint8_t *wst = smem;
    uint8_t *xst = smem + C::X_OFF;
    uint64_t *wfull = reinterpret_cast<uint64_t *>(smem + C::bar_off(T));
    uint64_t *wempty = wfull + C::NS;
    uint64_t *xfull = wempty + C::NS;
    uint64_t *xempty = xfull + 2;
    float *abuf = reinterpret_cast<float *>(smem + C::abuf_off(T));
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int R = a.I / MOE_ROWTILE;
    if (tid == 0) {
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(wfull + s, 1);
            mbar_init(wempty + s, 8);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(xfull + s, 1);
            mbar_init(xempty + s, 8);
        }
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == 8) {  // producer
        if (lane != 0) return;
        // The shared expert's chunks come first (chunks 0 .. ceil(T/8)-1 are
        // group 0), so the first item's weight rows are known before the
        // router has finished: stream them before waiting on it.
        const long long sh_items = a.shared_here ? (long long)((T + MOE_TC - 1) / MOE_TC) * R : 0;
        const long long it0 = blockIdx.x;
        const bool pre = it0 < sh_items;
        constexpr int NPRE = C::SPI < C::NS ? C::SPI : C::NS;  // sub-stages that fit the ring
        if (pre) {
            const size_t r0 = (size_t)(it0 % R) * MOE_ROWTILE;
            for (int s = 0; s < NPRE; ++s) {
                const unsigned bytes = (unsigned)(C::SR * G::ROWB);
                mbar_arrive_expect_tx(wfull + s, 2 * bytes);
                bulk_g2s(wst + (size_t)s * C::STB, a.sh_gate + (r0 + (size_t)s * C::SR) * G::ROWB, bytes, wfull + s);
                bulk_g2s(wst + (size_t)s * C::STB + bytes, a.sh_up + (r0 + (size_t)s * C::SR) * G::ROWB, bytes,
                         wfull + s);
            }
        }
        pdl_wait();
        pdl_launch_dependents();
        const long long n_items = (long long)__ldcg(a.hdr + HDR_NCHUNKS) * R;
        int n = 0, i = 0;
        for (long long it = it0; it < n_items; it += gridDim.x, ++i) {
            const int c = (int)(it / R), rt = (int)(it % R);
            const MoeChunk *cp = a.chunks + c;
            const uint8_t *gb =
                reinterpret_cast<const uint8_t *>(__ldcg(reinterpret_cast<const unsigned long long *>(&cp->gate)));
            const uint8_t *ub =
                reinterpret_cast<const uint8_t *>(__ldcg(reinterpret_cast<const unsigned long long *>(&cp->up)));
            const int np = __ldcg(&cp->np);
            const uint2 tk = __ldcg(reinterpret_cast<const uint2 *>(cp->tok));
            // activations of the chunk's tokens
            const int xsl = i & 1;
            if (i >= 2 && !mbar_wait(xempty + xsl, (unsigned)(((i >> 1) - 1) & 1))) return;
            uint8_t *xb = xst + (size_t)xsl * XSLOT;
            mbar_arrive_expect_tx(xfull + xsl, (unsigned)(sizeof(MoeChunk) + (size_t)np * (H * 2 + H / 8)));
            bulk_g2s(xb, cp, sizeof(MoeChunk), xfull + xsl);
            for (int j = 0; j < np; ++j) {
                const int t = (int)(((j < 4 ? tk.x : tk.y) >> (8 * (j & 3))) & 0xFFu);
                bulk_g2s(xb + CHUNK_HDR + (size_t)j * H * 2, a.xq + (size_t)t * H, H * 2, xfull + xsl);
                bulk_g2s(xb + CHUNK_HDR + (size_t)TC * H * 2 + (size_t)j * (H / 8), a.xs + (size_t)t * (H / 32), H / 8,
                         xfull + xsl);
            }
            // weights, in sub-stages
            const bool ok = gb && ub && !((reinterpret_cast<uintptr_t>(gb) | reinterpret_cast<uintptr_t>(ub)) & 15);
            if (!ok) flag_error(DEVERR_ROUTE);
            for (int s = 0; s < C::SPI; ++s, ++n) {
                if (pre && it == it0 && s < NPRE) continue;  // already streaming since before the wait
                const int slot = n % C::NS;
                if (n >= C::NS && !mbar_wait(wempty + slot, (unsigned)(((n / C::NS) - 1) & 1))) return;
                const size_t r0 = (size_t)rt * MOE_ROWTILE + (size_t)s * C::SR;
                const unsigned bytes = (unsigned)(C::SR * G::ROWB);
                if (ok) {
                    mbar_arrive_expect_tx(wfull + slot, 2 * bytes);
                    bulk_g2s(wst + (size_t)slot * C::STB, gb + r0 * G::ROWB, bytes, wfull + slot);
                    bulk_g2s(wst + (size_t)slot * C::STB + bytes, ub + r0 * G::ROWB, bytes, wfull + slot);
                } else {
                    mbar_arrive(wfull + slot);
                }
            }
        }
        return;
    }

    // consumers: warps 0..7
    pdl_wait();
    const long long n_items = (long long)__ldcg(a.hdr + HDR_NCHUNKS) * R;
    const int rho = lane / G::LPR, lr = lane % G::LPR, bb = lr >> 2, sub = lr & 3;
    const int rs = warp * G::RPW + rho;           // row inside a sub-stage
    const bool has_rows = warp * G::RPW < C::SR;  // H = 256: only warps 0..3 have rows
    XSlice X[G::CP];
    int n = 0, i = 0;
    for (long long it = blockIdx.x; it < n_items; it += gridDim.x, ++i) {
        const int rt = (int)(it % R);
        const int xsl = i & 1;
        if (!mbar_wait(xfull + xsl, (unsigned)((i >> 1) & 1))) return;
        const uint8_t *xb = xst + (size_t)xsl * XSLOT;
        const MoeChunk *ch = reinterpret_cast<const MoeChunk *>(xb);
        const int np = ch->np, p0 = ch->p0;
        const int16_t *xq = reinterpret_cast<const int16_t *>(xb + CHUNK_HDR);
        const float *xsc = reinterpret_cast<const float *>(xb + CHUNK_HDR + (size_t)TC * H * 2);
        for (int s = 0; s < C::SPI; ++s, ++n) {
            const int slot = n % C::NS;
            if (!mbar_wait(wfull + slot, (unsigned)((n / C::NS) & 1))) return;
            const uint8_t *grow = wst + (size_t)slot * C::STB + (size_t)rs * G::ROWB;
            const uint8_t *urow = grow + (size_t)C::SR * G::ROWB;
            for (int j = 0; has_rows && j < np; ++j) {
                if (np > 1 || s == 0) {  // one token: its slice stays in registers across sub-stages
#pragma unroll
                    for (int cp = 0; cp < G::CP; ++cp)
                        load_slice_q4k(X[cp], xq + (size_t)j * H, xsc + (size_t)j * (H / 32),
                                       QK * (cp * 8 + bb) + 64 * sub);
                }
                float gs = 0.0f, us = 0.0f;
#pragma unroll
                for (int cp = 0; cp < G::CP; ++cp) {
                    gs += q4k_lane_dot(grow + (size_t)(cp * 8 + bb) * Q4K_BYTES, sub, X[cp]);
                    us += q4k_lane_dot(urow + (size_t)(cp * 8 + bb) * Q4K_BYTES, sub, X[cp]);
                }
#pragma unroll
                for (int o = G::LPR / 2; o; o >>= 1) {
                    gs += __shfl_xor_sync(0xffffffffu, gs, o);
                    us += __shfl_xor_sync(0xffffffffu, us, o);
                }
                if (lr == 0) abuf[j * MOE_ROWTILE + s * C::SR + rs] = gs / (1.0f + expf(-gs)) * us;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(wempty + slot);
        }
        named_sync(1, 256);
        if (lane == 0) mbar_arrive(xempty + xsl);
        for (int j = warp; j < np; j += 8) {
            const size_t p = (size_t)(p0 + j);
            const int q = quant32(abuf[j * MOE_ROWTILE + lane], a.as + p * (a.I / 32) + rt, lane);
            a.aq[p * a.I + (size_t)rt * MOE_ROWTILE + lane] = (int16_t)q;
        }
        named_sync(1, 256);
    }
}

// ---------------------------------------------------------------------------
// K3: down + weighted combine
// ---------------------------------------------------------------------------
template <int NB>
struct K3Cfg {
    using G = MGeo<BREAD_QTYPE_Q6_K, NB>;
    static constexpr int I = QK * NB;
    static constexpr int WS = MOE_RT3 / G::RPW;              // warp steps per stage
    static constexpr size_t WB = (size_t)MOE_RT3 * G::ROWB;  // weight bytes per stage
    static constexpr size_t ABY = (size_t)I * 2 + I / 8;     // one pair's intermediate + its scales
    static constexpr size_t STB = al16(CHUNK_HDR + WB + MOE_TC * ABY);
    static constexpr int NS0 = (int)((96 * 1024) / STB);
    static constexpr int NS = NS0 < 2 ? 2 : (NS0 > 16 ? 16 : NS0);
    static constexpr size_t BAR_OFF = (size_t)NS * STB + 16;
    static constexpr size_t ACC_OFF = BAR_OFF + 2 * NS * 8;
    __host__ __device__ static size_t smem(int T) { return ACC_OFF + (size_t)8 * T * MOE_RT3 * 4; }
};

template <int NB>
__global__ void __launch_bounds__(288) moe_down_kernel(MoeArgs a)
{
    using C = K3Cfg<NB>;
    using G = typename C::G;
    constexpr int I = C::I;
    extern __shared__ __align__(128) uint8_t smem[];
    uint8_t *stages = smem;
    uint64_t *full = reinterpret_cast<uint64_t *>(smem + C::BAR_OFF);
    uint64_t *empty = full + C::NS;
    float *accs = reinterpret_cast<float *>(smem + C::ACC_OFF);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = a.T;
    if (tid == 0) {
        for (int s = 0; s < C::NS; ++s) {
            mbar_init(full + s, 1);
            mbar_init(empty + s, C::WS);
        }
        fence_mbar_init();
    }
    for (int i = tid; i < 8 * T * MOE_RT3; i += blockDim.x) accs[i] = 0.0f;
    __syncthreads();
    const int n_items = a.H / MOE_RT3;
    // This kernel starts once every gate/up CTA has passed its own wait on the
    // router, so the chunk table is complete and is read before this kernel's
    // wait -- through L2, since the previous layer's table may sit in L1.
    const int nch = __ldcg(a.hdr + HDR_NCHUNKS);
    const int my_items = (int)blockIdx.x < n_items ? (n_items - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int n_stages = my_items * nch;

    if (warp == 8) {  // producer: lane j feeds stage base + j of each batch of NS stages
        if (n_stages == 0) {
            pdl_wait();
            pdl_launch_dependents();
            return;
        }
        for (int base = 0; base < n_stages; base += C::NS) {
            const int n = base + lane;
            const bool act = lane < C::NS && n < n_stages;
            const int slot = n % C::NS;
            const MoeChunk *cp = nullptr;
            int np = 0, p0 = 0;
            if (act) {
                if (n >= C::NS && !mbar_wait(empty + slot, (unsigned)(((n / C::NS) - 1) & 1))) return;
                const int it = (int)blockIdx.x + (n / nch) * (int)gridDim.x;
                cp = a.chunks + (n % nch);
                const uint8_t *db =
                    reinterpret_cast<const uint8_t *>(__ldcg(reinterpret_cast<const unsigned long long *>(&cp->down)));
                np = __ldcg(&cp->np);
                p0 = __ldcg(&cp->p0);
                const bool ok = db && !(reinterpret_cast<uintptr_t>(db) & 15);
                if (!ok) flag_error(DEVERR_ROUTE);
                uint8_t *st = stages + (size_t)slot * C::STB;
                mbar_arrive_expect_tx(full + slot,
                                      (unsigned)(sizeof(MoeChunk) + (ok ? C::WB : 0) + (size_t)np * (I * 2 + I / 8)));
                bulk_g2s(st, cp, sizeof(MoeChunk), full + slot);
                if (ok) bulk_g2s(st + CHUNK_HDR, db + (size_t)it * MOE_RT3 * G::ROWB, (unsigned)C::WB, full + slot);
            }
            if (base == 0) {
                pdl_wait();  // the intermediate comes from the gate/up kernel
                pdl_launch_dependents();
            }
            if (act && np > 0) {
                uint8_t *st = stages + (size_t)slot * C::STB;
                bulk_g2s(st + CHUNK_HDR + C::WB, a.aq + (size_t)p0 * I, (unsigned)(np * I * 2), full + slot);
                bulk_g2s(st + CHUNK_HDR + C::WB + (size_t)MOE_TC * I * 2, a.as + (size_t)p0 * (I / 32),
                         (unsigned)(np * (I / 8)), full + slot);
            }
        }
        return;
    }

    pdl_wait();
    const int rho = lane / G::LPR, lr = lane % G::LPR, bb = lr >> 2, sub = lr & 3;
    const Q6Lane L6 = q6_lane(((rho * NB + bb) & 1) ? 2 : 0, sub & 1);
    float *my_acc = accs + (size_t)warp * T * MOE_RT3;
    int n = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
        for (int c = 0; c < nch; ++c, ++n) {
            const int slot = n % C::NS;
            const uint8_t *st = stages + (size_t)slot * C::STB;
            bool waited = false;
            for (int ws = 0; ws < C::WS; ++ws) {
                if (((c * C::WS + ws) & 7) != warp) continue;
                if (!waited) {
                    if (!mbar_wait(full + slot, (unsigned)((n / C::NS) & 1))) return;
                    waited = true;
                }
                const MoeChunk *ch = reinterpret_cast<const MoeChunk *>(st);
                const int np = ch->np;
                const uint8_t *rowp = st + CHUNK_HDR + (size_t)ws * G::STEPB + (size_t)rho * G::ROWB;
                const int16_t *aqs = reinterpret_cast<const int16_t *>(st + CHUNK_HDR + C::WB);
                const float *ass = reinterpret_cast<const float *>(st + CHUNK_HDR + C::WB + (size_t)MOE_TC * I * 2);
                for (int j = 0; j < np; ++j) {
                    const int t = ch->tok[j];
                    const float wgt = ch->w[j];
                    float v = 0.0f;
#pragma unroll
                    for (int cp = 0; cp < G::CP; ++cp) {
                        XSlice X;
                        load_slice_q6k(X, aqs + (size_t)j * I, ass + (size_t)j * (I / 32),
                                       QK * (cp * 8 + bb) + 128 * (sub >> 1), sub & 1);
                        v += q6k_lane_dot(rowp + (size_t)(cp * 8 + bb) * Q6K_BYTES, sub >> 1, sub & 1, L6, X);
                    }
#pragma unroll
                    for (int o = G::LPR / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                    if (lr == 0) my_acc[t * MOE_RT3 + ws * G::RPW + rho] += wgt * v;
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(empty + slot);
            }
        }
        named_sync(1, 256);
        for (int i = tid; i < T * MOE_RT3; i += 256) {
            const int t = i / MOE_RT3, r = i % MOE_RT3;
            float s = 0.0f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                s += accs[(size_t)w * T * MOE_RT3 + i];
                accs[(size_t)w * T * MOE_RT3 + i] = 0.0f;
            }
            const size_t oi = (size_t)t * a.H + (size_t)it * MOE_RT3 + r;
            if (a.ep_world > 1) {
                // this rank's partial -> slot [ep_slot][ep_rank] of every rank's mailbox (NVLink stores)
                const size_t off = MoeMailbox::data_off(a.ep_slot, a.ep_rank, a.ep_world, a.ep_tmax, a.H) / 4 + oi;
                for (int p = 0; p < a.ep_world; ++p) a.ep_mb[p][off] = s;
            } else {
                a.out[oi] = a.out[oi] + s;
            }
        }
        named_sync(1, 256);
    }
    if (a.ep_world > 1) {
        // one arrival per CTA at every rank, after all of this CTA's stores
        __threadfence_system();
        named_sync(1, 256);
        if (tid == 0) {
            const MoeMailbox L = MoeMailbox::make(a.ep_world, a.ep_tmax, a.H);
            for (int p = 0; p < a.ep_world; ++p) {
                unsigned *f = reinterpret_cast<unsigned *>(reinterpret_cast<uint8_t *>(a.ep_mb[p]) + L.flag_off) +
                              a.ep_slot * 8 + a.ep_rank;
                atomicAdd_system(f, 1u);
            }
        }
    }
}

// Expert-parallel combine (one per layer, after the down kernel on every
// rank): wait, bounded, until every rank's down-kernel CTAs have arrived in
// this rank's mailbox slot, then h += sum over ranks (rank order, so every
// rank gets the same bits); the last CTA re-arms the slot's counters.
__global__ void __launch_bounds__(256) ep_combine_kernel(float *h, MoeArgs a, int n_signals)
{
    pdl_wait();
    pdl_launch_dependents();
    uint8_t *own = reinterpret_cast<uint8_t *>(a.ep_mb[a.ep_rank]);
    const MoeMailbox L = MoeMailbox::make(a.ep_world, a.ep_tmax, a.H);
    volatile unsigned *flags = reinterpret_cast<volatile unsigned *>(own + L.flag_off) + a.ep_slot * 8;
    __shared__ int s_ok;
    if (threadIdx.x == 0) {
        int ok = 1;
        for (int r = 0; r < a.ep_world && ok; ++r) {
            long long i = 0;
            while (flags[r] < (unsigned)n_signals) {
                if (++i > SPIN_LIMIT) {
                    ok = 0;
                    flag_error(DEVERR_TIMEOUT);
                    break;
                }
                if (i > 64) __nanosleep(128);
            }
        }
        __threadfence_system();
        s_ok = ok;
    }
    __syncthreads();
    if (s_ok) {
        const float *mb = reinterpret_cast<const float *>(own);
        const size_t n = (size_t)a.T * a.H;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
            float v = h[i];
            for (int r = 0; r < a.ep_world; ++r)
                v += __ldcv(mb + MoeMailbox::data_off(a.ep_slot, r, a.ep_world, a.ep_tmax, a.H) / 4 + i);
            h[i] = v;
        }
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        unsigned *ticket = reinterpret_cast<unsigned *>(own + L.ticket_off) + a.ep_slot;
        __threadfence();
        if (atomicAdd(ticket, 1u) == gridDim.x - 1) {
            for (int r = 0; r < a.ep_world; ++r) flags[r] = 0;
            *ticket = 0;
            __threadfence_system();
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <typename... KArgs, typename... Args>
static cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args &&...args)
{
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, std::forward<Args>(args)...);
}

void moe_bind_workspace(MoeArgs &a, void *ws, const MoeWs &L)
{
    uint8_t *b = static_cast<uint8_t *>(ws);
    a.hdr = reinterpret_cast<int *>(b + L.hdr);
    a.logits = reinterpret_cast<float *>(b + L.logits);
    a.ssq = reinterpret_cast<float *>(b + L.ssq);
    a.score = reinterpret_cast<float *>(b + L.score);
    a.ridx = reinterpret_cast<int *>(b + L.ridx);
    a.rw = reinterpret_cast<float *>(b + L.rw);
    a.sgw = reinterpret_cast<float *>(b + L.sgw);
    a.xq = reinterpret_cast<int16_t *>(b + L.xq);
    a.xs = reinterpret_cast<float *>(b + L.xs);
    a.p_token = reinterpret_cast<int *>(b + L.p_token);
    a.p_w = reinterpret_cast<float *>(b + L.p_w);
    a.chunks = reinterpret_cast<MoeChunk *>(b + L.chunks);
    a.aq = reinterpret_cast<int16_t *>(b + L.aq);
    a.as = reinterpret_cast<float *>(b + L.as);
}

static bool nb_ok_h(int nb) { return nb == 1 || nb == 2 || nb == 4 || nb == 8 || nb == 16; }
static bool nb_ok_i(int nb) { return nb == 1 || nb == 2 || nb == 4 || nb == 8; }

int moe_check_shapes(int T, int H, int I, int E, int top_k, bool need_experts)
{
    if (T < 1 || T > MOE_TMAX) return set_error(BREAD_ERR_ARG, "moe: T=%d outside 1..%d", T, MOE_TMAX);
    if (top_k < 1 || top_k > MOE_KMAX || E < top_k || E > MOE_EMAX)
        return set_error(BREAD_ERR_ARG, "moe: E=%d top_k=%d (need 1 <= top_k <= %d, top_k <= E <= %d)", E, top_k,
                         MOE_KMAX, MOE_EMAX);
    if (H < 256 || H > MOE_HMAX || H % 256 || !nb_ok_h(H / 256))
        return set_error(BREAD_ERR_ARG, "moe: H=%d (need H/256 in {1,2,4,8,16})", H);
    if (need_experts && (I < 256 || I > MOE_IMAX || I % 256 || !nb_ok_i(I / 256)))
        return set_error(BREAD_ERR_ARG, "moe: I=%d (need I/256 in {1,2,4,8})", I);
    return BREAD_OK;
}

int moe_launch_route(const MoeArgs &a, cudaStream_t s)
{
    const dim3 grid((a.E + (a.w_sg ? 1 : 0) + K1_ROWS - 1) / K1_ROWS, (a.T + K1_TG - 1) / K1_TG);
    BREAD_CUDA(launch_pdl(moe_route_kernel, grid, dim3(256), 0, s, a), "moe route launch");
    return BREAD_OK;
}

template <int NB>
static int setup_gateup_nb()
{
    static bool done = false;
    if (!done) {
        BREAD_CUDA(cudaFuncSetAttribute(moe_gateup_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        (int)K2Cfg<NB>::smem(MOE_TMAX)),
                   "moe gate/up smem attribute");
        done = true;
    }
    return BREAD_OK;
}

template <int NB>
static int launch_gateup_nb(const MoeArgs &a, cudaStream_t s)
{
    BREAD_TRY(setup_gateup_nb<NB>());
    BREAD_CUDA(launch_pdl(moe_gateup_kernel<NB>, dim3(sm_count()), dim3(288), K2Cfg<NB>::smem(a.T), s, a),
               "moe gate/up launch");
    return BREAD_OK;
}

int moe_launch_gateup(const MoeArgs &a, cudaStream_t s)
{
    switch (a.H / 256) {
    case 1: return launch_gateup_nb<1>(a, s);
    case 2: return launch_gateup_nb<2>(a, s);
    case 4: return launch_gateup_nb<4>(a, s);
    case 8: return launch_gateup_nb<8>(a, s);
    case 16: return launch_gateup_nb<16>(a, s);
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported H=%d", a.H);
    }
}

// Grid of the down kernel (also the number of arrivals each rank's combine
// waits for).  The smem attribute and occupancy are set up once.
template <int NB>
static int down_grid_nb(const MoeArgs &a)
{
    using C = K3Cfg<NB>;
    static int per_sm = 0;
    if (!per_sm) {
        if (cudaFuncSetAttribute(moe_down_kernel<NB>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)C::smem(MOE_TMAX)) != cudaSuccess)
            return -1;
        int n = 1;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, moe_down_kernel<NB>, 288, C::smem(1)) != cudaSuccess)
            return -1;
        per_sm = n < 1 ? 1 : n;
    }
    const int items = a.H / MOE_RT3;
    const int cap = sm_count() * (a.T <= 8 ? per_sm : 1);
    return items < cap ? items : cap;
}

template <int NB>
static int launch_down_nb(const MoeArgs &a, cudaStream_t s)
{
    const int grid = down_grid_nb<NB>(a);
    if (grid < 1) return set_error(BREAD_ERR_CUDA, "moe down: kernel set-up failed");
    BREAD_CUDA(launch_pdl(moe_down_kernel<NB>, dim3(grid), dim3(288), K3Cfg<NB>::smem(a.T), s, a), "moe down launch");
    return BREAD_OK;
}

int moe_down_grid(const MoeArgs &a)
{
    switch (a.I / 256) {
    case 1: return down_grid_nb<1>(a);
    case 2: return down_grid_nb<2>(a);
    case 4: return down_grid_nb<4>(a);
    default: return down_grid_nb<8>(a);
    }
}

int moe_launch_down(const MoeArgs &a, cudaStream_t s)
{
    switch (a.I / 256) {
    case 1: return launch_down_nb<1>(a, s);
    case 2: return launch_down_nb<2>(a, s);
    case 4: return launch_down_nb<4>(a, s);
    case 8: return launch_down_nb<8>(a, s);
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported I=%d", a.I);
    }
}

// One-time kernel attribute set-up for these shapes (before any graph capture).
int moe_setup_kernels(int H, int I)
{
    int st = BREAD_OK;
    switch (H / 256) {
    case 1: st = setup_gateup_nb<1>(); break;
    case 2: st = setup_gateup_nb<2>(); break;
    case 4: st = setup_gateup_nb<4>(); break;
    case 8: st = setup_gateup_nb<8>(); break;
    case 16: st = setup_gateup_nb<16>(); break;
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported H=%d", H);
    }
    if (st) return st;
    MoeArgs a{};
    a.H = H;
    a.I = I;
    a.T = 1;
    return moe_down_grid(a) > 0 ? BREAD_OK : set_error(BREAD_ERR_CUDA, "moe down: kernel set-up failed");
}

int moe_launch_combine(const MoeArgs &a, float *h, cudaStream_t s)
{
    const int n = a.T * a.H;
    int grid = (n + 255) / 256;
    if (grid > sm_count()) grid = sm_count();
    BREAD_CUDA(launch_pdl(ep_combine_kernel, dim3(grid), dim3(256), 0, s, h, a, moe_down_grid(a)),
               "ep combine launch");
    return BREAD_OK;
}

}  // namespace bread

using namespace bread;

extern "C" size_t bread_moe_workspace_bytes(int T, int H, int I, int E, int top_k)
{
    if (T < 1 || H < 32 || E < 1 || top_k < 1) return 0;
    return MoeWs::make(T, H, I, E, top_k).total;
}

static int moe_prepare(MoeArgs &a, const float *x, const float *W_r, const void *w_sg, int T, int H, int I, int E,
                       int top_k, void *workspace, size_t workspace_bytes, bool need_experts)
{
    BREAD_TRY(moe_check_shapes(T, H, I, E, top_k, need_experts));
    if (!x || !W_r) return set_error(BREAD_ERR_ARG, "moe: NULL x or W_r");
    const MoeWs L = MoeWs::make(T, H, need_experts ? I : 0, E, top_k);
    if (!workspace || workspace_bytes < L.total)
        return set_error(BREAD_ERR_WORKSPACE, "moe: workspace %zu bytes, need %zu", workspace_bytes, L.total);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return set_error(BREAD_ERR_ALIGN, "moe: workspace not 256-byte aligned");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W_r)) & 7)
        return set_error(BREAD_ERR_ALIGN, "moe: x / W_r not 8-byte aligned");
    if (reinterpret_cast<uintptr_t>(w_sg) & 3) return set_error(BREAD_ERR_ALIGN, "moe: w_sg not 4-byte aligned");
    a = MoeArgs{};
    a.W_r = W_r;
    a.w_sg = static_cast<const __half *>(w_sg);
    a.T = T;
    a.H = H;
    a.I = I;
    a.E = E;
    a.top_k = top_k;
    a.lo = 0;
    a.hi = E;
    a.norm_eps = -1.0f;
    a.x = x;
    moe_bind_workspace(a, workspace, L);
    return BREAD_OK;
}

extern "C" int bread_moe_route(const float *x, const float *W_r, const void *w_sg, int T, int H, int E, int top_k,
                               int *idx, float *w, float *sg_weight, void *workspace, size_t workspace_bytes,
                               cudaStream_t stream)
{
    MoeArgs a;
    BREAD_TRY(moe_prepare(a, x, W_r, w_sg, T, H, 0, E, top_k, workspace, workspace_bytes, false));
    if (!idx || !w) return set_error(BREAD_ERR_ARG, "moe_route: NULL idx or w");
    a.idx_out = idx;
    a.w_out = w;
    a.sg_out = sg_weight;
    a.shared_here = 0;
    BREAD_CUDA(cudaMemsetAsync(a.hdr, 0, 64, stream), "moe_route: reset ticket");
    return moe_launch_route(a, stream);
}

extern "C" int bread_moe_ffn(const void *const *gate_ptrs, const void *const *up_ptrs, const void *const *down_ptrs,
                             const float *W_r, const void *w_sg, const void *sh_gate, const void *sh_up,
                             const void *sh_down, const float *x, float *out, int T, int H, int I, int E, int top_k,
                             int *idx_out, float *w_out, float *sg_out, void *workspace, size_t workspace_bytes,
                             cudaStream_t stream)
{
    MoeArgs a;
    BREAD_TRY(moe_prepare(a, x, W_r, w_sg, T, H, I, E, top_k, workspace, workspace_bytes, true));
    if (!gate_ptrs || !up_ptrs || !down_ptrs || !out) return set_error(BREAD_ERR_ARG, "moe_ffn: NULL pointer table or out");
    const int nsh = (sh_gate != nullptr) + (sh_up != nullptr) + (sh_down != nullptr);
    if (nsh != 0 && nsh != 3) return set_error(BREAD_ERR_ARG, "moe_ffn: give all three shared-expert matrices or none");
    if (nsh == 3 && ((reinterpret_cast<uintptr_t>(sh_gate) | reinterpret_cast<uintptr_t>(sh_up) |
                      reinterpret_cast<uintptr_t>(sh_down)) & 15))
        return set_error(BREAD_ERR_ALIGN, "moe_ffn: shared-expert matrices must be 16-byte aligned");
    BREAD_TRY(moe_setup_kernels(H, I));
    a.gate = reinterpret_cast<const uint8_t *const *>(gate_ptrs);
    a.up = reinterpret_cast<const uint8_t *const *>(up_ptrs);
    a.down = reinterpret_cast<const uint8_t *const *>(down_ptrs);
    a.sh_gate = static_cast<const uint8_t *>(sh_gate);
    a.sh_up = static_cast<const uint8_t *>(sh_up);
    a.sh_down = static_cast<const uint8_t *>(sh_down);
    a.shared_here = nsh == 3;
    a.out = out;
    a.idx_out = idx_out;
    a.w_out = w_out;
    a.sg_out = sg_out;
    BREAD_CUDA(cudaMemsetAsync(a.hdr, 0, 64, stream), "moe_ffn: reset ticket");
    BREAD_TRY(moe_launch_route(a, stream));
    BREAD_TRY(moe_launch_gateup(a, stream));
    return moe_launch_down(a, stream);
}
