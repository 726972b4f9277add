// moe_kernel.cuh -- the MoE FFN on sm_100a as ONE persistent, cooperative
// kernel per call (device code and per-shape host templates; instantiated by
// one translation unit per hidden size, moe_h*.cu, so they compile in
// parallel): a whole decode step of L MoE layers (or one MoE block) runs in a
// single launch of one CTA per SM, with grid-wide barriers between phases
// instead of kernel boundaries.
//
// Reference path replaced: route_layer (one_layer.cu:937-992, with
// cpu_softmax/cpu_topk layer_ops.cu:222-250), the shared expert
// (one_layer.cu:1840-1894) and the serial expert loop (one_layer.cu:1931-1983:
// per expert bread_matvec gate, up, silu_mul_inplace, bread_matvec down,
// scale_accum), for each of the 40 layers of the decode loop (main.cu:683-687).
//
// Per layer, for T tokens (CTA = 8 consumer warps + 1 producer warp):
//   A  every CTA quantises a share of the layer input to int16 per 32 values
//      (plus per-group sums of squares for the RMS norm) and computes its
//      router rows (fp32 weights already in shared memory, loaded during the
//      previous layer) -> logits.                          grid barrier
//   B  every CTA routes all tokens itself from the logits (softmax, top-k
//      with lowest index winning ties, renormalisation, sigmoid of the shared
//      gate) and groups the (token, expert) pairs by expert -- the same
//      deterministic tables in every CTA, no extra barrier.  The producer
//      then issues, at once, the bulk copies of this CTA's gate/up rows AND
//      of its down rows (which do not depend on the intermediate), so a
//      whole layer's expert weights are in flight together.  Consumers
//      compute silu(g)*u for 32-row items and store it quantised to int16.
//                                                          grid barrier
//   C  each CTA owns 16 output columns of h: it adds the router-weighted
//      down projections of every active expert for them, in fixed order
//      (deterministic, no atomics), h_out = h_in + sum.     grid barrier
// Work that does not depend on the routing -- the next layer's router rows
// and the first shared-expert gate/up rows -- is copied during the previous
// layer.  With expert parallelism (ep_world > 1) phase C writes the rank's
// partial columns into every rank's mailbox over NVLink and counts one
// arrival per column tile there; the next phase A waits (bounded) for all
// ranks' arrivals and reads h = h_prev + sum of partials in rank order, so
// every rank holds the same bits and routes identically.
#pragma once
#include <math.h>
#include <stdlib.h>

#include <mutex>

#include "common.cuh"
#include "moe.cuh"
#include "ptx.cuh"
#include "qdot.cuh"

namespace bread {

constexpr int ST_THREADS = 288;  // 8 consumer warps + 1 producer warp
constexpr int ST_CONS = 256;
constexpr int BAR_CONS = 1;      // named barrier of the consumer warps
constexpr int BAR_ALL = 2;       // consumers + producer: routing tables ready
constexpr size_t SMEM_LIMIT = 232448;  // dynamic shared memory per CTA (227 KB)
constexpr unsigned long long GRID_WAIT_NS = 2000000000ull;  // 2 s
constexpr int ROUTE_DIST_T = 16;  // above this many tokens the grid routes them (one warp each)
constexpr int ROUTER_TILE_T = 8;  // above this many tokens the router works in 16-row x 8-token units

template <int NBH, int NBI>
struct SCfg {
    using GH = MGeo<BREAD_QTYPE_Q4_K, NBH>;
    using GI = MGeo<BREAD_QTYPE_Q6_K, NBI>;
    static constexpr int H = QK * NBH;
    static constexpr int I = QK * NBI;
    static constexpr int SR = 8 * GH::RPW < MOE_ROWTILE ? 8 * GH::RPW : MOE_ROWTILE;  // rows per gate/up sub-stage
    static constexpr int SPI = MOE_ROWTILE / SR;                                      // sub-stages per item
    static constexpr int STB = 2 * SR * GH::ROWB;                                     // gate rows + up rows
    static constexpr int WS = MOE_RT3 / GI::RPW;                                      // warp steps per down stage
    static constexpr int WB = MOE_RT3 * GI::ROWB;                                     // down weight bytes per stage
    static constexpr int XTOK = H * 2 + H / 8;  // one token: int16 activations + group scales
    static constexpr int ATOK = I * 2 + I / 8;  // one pair: int16 intermediate + group scales
};

// ---------------------------------------------------------------------------
// device helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ bool dev_failed() { return *reinterpret_cast<volatile unsigned *>(&g_dev_error) != 0; }

// Bounded wait until *p >= target (acquire at gpu or system scope).  Gives up
// at once when a wait anywhere on the device has already failed, so a lost
// peer costs one timeout, not one per remaining barrier.
static __device__ bool wait_counter(const unsigned long long *p, unsigned long long target, bool sys,
                                    unsigned long long limit_ns)
{
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        const unsigned long long v = sys ? ld_acquire_sys(p) : ld_acquire_gpu(p);
        if (v >= target) return true;
        if ((i & 63) == 63) {
            if (dev_failed()) return false;
            const unsigned long long now = globaltimer();
            if (!t0) {
                t0 = now;
            } else if (now - t0 > limit_ns) {
                flag_error(DEVERR_TIMEOUT);
                return false;
            }
        }
        if (i > 16) __nanosleep(20);
    }
}

// Bounded mbarrier wait that also gives up once the device error word is set.
// The spin loop is out of line: the waits are many and mostly succeed at
// once, and the persistent kernel's instruction footprint is on its critical
// path (every phase of every layer re-fetches its code).
static __device__ __noinline__ void swait_slow(uint64_t *bar, unsigned parity)
{
    for (long long i = 0; i < SPIN_LIMIT; ++i) {
        if (mbar_try_wait(bar, parity)) return;
        if ((i & 1023) == 1023 && dev_failed()) return;
        if (i > 64) __nanosleep(32);
    }
    flag_error(DEVERR_TIMEOUT);
}
__device__ __forceinline__ void swait(uint64_t *bar, unsigned parity)
{
    if (!mbar_try_wait(bar, parity)) swait_slow(bar, parity);
}

// Flagged word *p once its tag equals `tag`: bounded poll (the grid-barrier
// limit), giving up at once when a wait elsewhere on the device has failed.
// Returns the payload (0 after a timeout, with the device error set).
static __device__ __noinline__ uint32_t flagged_wait(const unsigned long long *p, uint32_t tag, unsigned long long limit_ns)
{
    unsigned long long t0 = 0;
    for (unsigned i = 0;; ++i) {
        const unsigned long long v = ld_flagged(p);
        if ((uint32_t)(v >> 32) == tag) return (uint32_t)v;
        if ((i & 31) == 31) {
            if (dev_failed()) return 0u;
            const unsigned long long now = globaltimer();
            if (!t0) {
                t0 = now;
            } else if (now - t0 > limit_ns) {
                flag_error(DEVERR_TIMEOUT);
                return 0u;
            }
        }
        if (i > 8) __nanosleep(32);
    }
}
// Payload of an already loaded word, polling again only when its tag is not
// the expected one (so a batch of loads is in flight together first).
__device__ __forceinline__ uint32_t flagged_take(unsigned long long v, const unsigned long long *p, uint32_t tag,
                                                  unsigned long long limit_ns)
{
    return (uint32_t)(v >> 32) == tag ? (uint32_t)v : flagged_wait(p, tag, limit_ns);
}
// The words addr(k), k < N with bit k of `valid` set, polled as one batch --
// every word still carrying an old tag is loaded again in the same round --
// until all tags equal `tag` (bounded like flagged_wait).  r[k]: the words.
template <int N, class Addr, bool SYS = false>
__device__ __forceinline__ void flagged_poll(unsigned long long (&r)[N], unsigned valid, const Addr &addr, uint32_t tag,
                                             unsigned long long limit_ns = GRID_WAIT_NS)
{
#pragma unroll
    for (int k = 0; k < N; ++k) r[k] = 0ull;
    unsigned pend = valid;
    unsigned long long t0 = 0;
    // one copy of the loads: the first round loads every valid word, later
    // rounds only those still carrying an old tag
    for (unsigned it = 0;; ++it) {
#pragma unroll
        for (int k = 0; k < N; ++k)
            if ((pend >> k) & 1u) r[k] = SYS ? ld_flagged_sys(addr(k)) : ld_flagged(addr(k));
        unsigned np = 0;
#pragma unroll
        for (int k = 0; k < N; ++k)
            if (((pend >> k) & 1u) && (uint32_t)(r[k] >> 32) != tag) np |= 1u << k;
        pend = np;
        if (!pend) return;
        if (it > 2) __nanosleep(40);
        if ((it & 31) == 31) {
            if (dev_failed()) return;
            const unsigned long long now = globaltimer();
            if (!t0) {
                t0 = now;
            } else if (now - t0 > limit_ns) {
                flag_error(DEVERR_TIMEOUT);
                return;
            }
        }
    }
}

// Sums V values per lane over groups of LPR consecutive lanes (LPR a power
// of two, V a power of two <= LPR) with a transposed butterfly: each halving
// step trades half of the lane's values with its partner, so V values take
// V - 1 + log2(LPR / V) + ... shuffles instead of V * log2(LPR).  Returns the
// fully reduced value of index q(lane) = the top log2(V) bits of
// (lane % LPR) (lane bit log2(LPR)-1 is the most significant); every lane of
// the group whose top bits equal q holds it.
template <int V, int LPR>
__device__ __forceinline__ float tr_reduce(float (&v)[V])
{
    const int lane = threadIdx.x & 31;
    int n = V;
#pragma unroll
    for (int off = LPR / 2; off >= 1; off >>= 1) {
        if (n > 1) {
            const bool hi = (lane & off) != 0;
            const int h = n / 2;
#pragma unroll
            for (int i = 0; i < V / 2; ++i) {
                if (i < h) {
                    const float keep = hi ? v[h + i] : v[i];
                    const float give = hi ? v[i] : v[h + i];
                    v[i] = keep + __shfl_xor_sync(0xffffffffu, give, off);
                }
            }
            n = h;
        } else {
            v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
        }
    }
    return v[0];
}

// Bound of the waits inside one GPU.  With expert parallelism every wait
// depends, through the layers before it, on the other ranks' progress (a rank
// may start its launch late), so all waits take the peer bound.
__device__ __forceinline__ unsigned long long wait_bound(const StepArgs &a)
{
    return a.ep_world > 1 ? a.ep_wait_ns : GRID_WAIT_NS;
}

// Grid-wide barrier number `idx` of this launch (all 256 consumer threads).
__device__ __forceinline__ void grid_barrier(const StepArgs &a, int idx, int tid)
{
    named_sync(BAR_CONS, ST_CONS);
    if (tid == 0) {
        // release at gpu scope, cumulative over the CTA's writes ordered by the
        // barrier above; the poll acquires
        red_release_gpu(a.ctrl + CTRL_GRID, 1ull);
        wait_counter(a.ctrl + CTRL_GRID, (unsigned long long)(idx + 1) * gridDim.x, false, wait_bound(a));
    }
    named_sync(BAR_CONS, ST_CONS);
}

// Layer l's descriptor: the kernel's shared-memory copy of StepArgs::layers
// (made at launch: a global load here would sit right after each layer's
// routing, on the critical path), else l0.
__device__ __forceinline__ StepLayer layer_desc(const StepArgs &a, int l)
{
    extern __shared__ __align__(128) uint8_t smem[];
    return a.layers ? reinterpret_cast<const StepLayer *>(smem + a.sm.ldesc)[l] : a.l0;
}
__device__ __forceinline__ const float *in_of(const StepArgs &a, int l) { return l == 0 ? a.x : a.buf[l & 1]; }
__device__ __forceinline__ float *out_of(const StepArgs &a, int l) { return l == a.L - 1 ? a.y : a.buf[(l + 1) & 1]; }

// Mailbox slot of layer l's partials.  Consecutive layers, and the last layer
// of a step and the first of the next, always use different slots; with the
// chained waits that makes a slot safe to rewrite.
__device__ __forceinline__ int ep_slot(int L, int l) { return ((L & 1) && l == L - 1) ? 2 : (l & 1); }
// Arrival count that completes layer l's partials in launch `epoch`.
__device__ __forceinline__ unsigned long long ep_target(const StepArgs &a, int l, unsigned long long epoch, int NT)
{
    const int s = ep_slot(a.L, l);
    const unsigned long long uses = s == 2 ? 1ull : (unsigned long long)(a.L / 2);
    const unsigned long long u = s == 2 ? 0ull : (unsigned long long)(l >> 1);
    return (epoch * uses + u + 1) * (unsigned long long)a.ep_world * (unsigned long long)NT;
}
// Float offset of a mailbox slot's partials (rank r's start r * ep_tmax * H later).
__device__ __forceinline__ size_t mb_slot_off(int slot, const StepArgs &a)
{
    return StepMailbox::data_off(slot, 0, a.ep_world, a.ep_tmax, a.H) / 4;
}
__device__ __forceinline__ unsigned long long *ep_counter(const StepArgs &a, int rank, int slot)
{
    const StepMailbox M = StepMailbox::make(a.ep_world, a.ep_tmax, a.H);
    return reinterpret_cast<unsigned long long *>(reinterpret_cast<uint8_t *>(a.ep_mb[rank]) + M.ctr_off) + slot;
}

// Decode mode, expert parallel: the flagged word of element oi (t * H + col)
// of source rank `src`'s partial for mailbox slot `slot` in rank `dst`'s
// mailbox.
__device__ __forceinline__ unsigned long long *ep_ll_word(const StepArgs &a, int dst, int slot, int src, size_t oi)
{
    const StepMailbox M = StepMailbox::make(a.ep_world, a.ep_tmax, a.H);
    unsigned long long *w = reinterpret_cast<unsigned long long *>(reinterpret_cast<uint8_t *>(a.ep_mb[dst]) + M.ll_off);
    return w + ((size_t)slot * a.ep_world + src) * (size_t)M.llT * a.H + oi;
}

__device__ __forceinline__ const uint8_t *expert_ptr(const uint8_t *const *tab, const uint8_t *sh, int e, int E)
{
    if (e >= E) return sh;
    return reinterpret_cast<const uint8_t *>(__ldg(reinterpret_cast<const unsigned long long *>(tab + e)));
}

// Routing tables of one layer, in shared memory (identical in every CTA).
struct RouteTabs {
    int *idx;
    float *w, *rinv, *sgw;
    int *cnt, *run, *off, *gexp, *goff, *gcnt, *gcpre, *ptok;
    float *pw;
    int *scal;             // [0] groups, [1] chunks, [2] pairs
    const uint8_t **ptr;   // [EL][3]: gate, up, down of each routed expert used here
    int4 *chunk;           // [chunks]: expert, first pair, pairs
};

struct ChunkInfo {
    int e, p0, np;
};

// Cursor of a ring of `ns` shared-memory stages: the slot, the parity of its
// current use, and whether the slot was used before (then its "empty" barrier
// of the previous use is awaited before refilling).  Advanced incrementally:
// no division on the per-copy path of the single producer thread.
struct Ring {
    int slot = 0, phase = 0, used = 0;
    __device__ __forceinline__ void next(int ns)
    {
        if (++slot == ns) {
            slot = 0;
            phase ^= 1;
            used = 1;
        }
    }
    // Cursor k positions ahead (0 <= k <= ns): at most one wrap.
    __device__ __forceinline__ Ring ahead(int k, int ns) const
    {
        Ring r = *this;
        r.slot += k;
        if (r.slot >= ns) {
            r.slot -= ns;
            r.phase ^= 1;
            r.used = 1;
        }
        return r;
    }
};

// Matrix k (0 gate, 1 up, 2 down) of expert e (E = the shared expert).
__device__ __forceinline__ const uint8_t *mat_ptr(const RouteTabs &R, const StepLayer &Ld, const StepArgs &a, int e,
                                                  int k)
{
    if (e >= a.E) return k == 0 ? Ld.sh_gate : k == 1 ? Ld.sh_up : Ld.sh_down;
    if (Ld.gate_base) {
        const size_t j = (size_t)(e - a.lo);
        return k == 0 ? Ld.gate_base + j * Ld.gu_stride : k == 1 ? Ld.up_base + j * Ld.gu_stride
                                                                 : Ld.down_base + j * Ld.d_stride;
    }
    return R.ptr[3 * (e - a.lo) + k];
}

// Chunk c: up to MOE_TC consecutive pairs of one expert group (from the
// table built with the routing).
__device__ __forceinline__ ChunkInfo chunk_info(const RouteTabs &R, int c)
{
    const int4 v = R.chunk[c];
    ChunkInfo ci;
    ci.e = v.x;
    ci.p0 = v.y;
    ci.np = v.z;
    return ci;
}

// Chunk c looked up from the group tables (binary search over groups).
__device__ __forceinline__ ChunkInfo chunk_search(const RouteTabs &R, int c)
{
    int lo = 0, hi = R.scal[0] - 1;
    while (lo < hi) {
        const int mid = (lo + hi + 1) >> 1;
        if (R.gcpre[mid] <= c)
            lo = mid;
        else
            hi = mid - 1;
    }
    const int k = c - R.gcpre[lo];
    ChunkInfo ci;
    ci.e = R.gexp[lo];
    ci.p0 = R.goff[lo] + MOE_TC * k;
    ci.np = min(MOE_TC, R.gcnt[lo] - MOE_TC * k);
    return ci;
}

// Phase B routing, run by the 256 consumer threads of every CTA from the
// logits in global memory: softmax + top-k (layer_ops.cu:222-250) with the
// RMS factor of the token applied to the logits, renormalised weights, the
// shared gate's sigmoid (0.5 without a gate vector, one_layer.cu:944,1889),
// then the (token, expert) pairs grouped by expert: group 0 is the shared
// expert (all T tokens), then the routed experts held here by ascending id,
// pairs token-major inside each group.
// Routes token t (one warp): RMS factor from the group sums of squares, top-k
// of the scaled logits (see below), renormalised weights, the shared gate's
// sigmoid (0.5 without a gate vector, one_layer.cu:944,1889).  Writes
// idx/w [t*K + k], rinv/sgw [t]; `outputs` also writes the caller's copies.
// LLM (flagged-exchange mode): the logits (row E = the shared-gate score) are
// flagged words at llg [t * (E + 1) + row] with tag `tag`, and the group sums
// of squares sit in shared memory (ssq_l), computed by this CTA.
struct NoEarly {
    __device__ void operator()(int) const {}
};
// `early(e)` runs (all lanes) as soon as pick number `kw` is known; with
// EVERY, `early(k, e)` runs at every pick k instead.
template <int PER, bool LLM = false, class Early = NoEarly, bool EVERY = false>
__device__ void route_token(const StepArgs &a, const StepLayer &Ld, int t, int *idx, float *w, float *rinv,
                            float *sgw, bool outputs, unsigned long long *st, int l, int *pick_i = nullptr,
                            float *pick_w = nullptr, float *pick_sg = nullptr,
                            const unsigned long long *llg = nullptr, const float *ssq_l = nullptr, uint32_t tag = 0,
                            int kw = -1, const Early &early = Early{})
{
    const int lane = threadIdx.x & 31;
    const int H = a.H, E = a.E, K = a.top_k, HG = H / 32;
    float p[PER];
    float ss = 0.0f, score = 0.0f;
    if constexpr (LLM) {
        // lane's logits e = lane + 32 j and, as entry PER, the score (row E)
        const unsigned long long *row = llg + (size_t)t * (E + 1);
        unsigned valid = Ld.w_sg ? 1u << PER : 0u;
#pragma unroll
        for (int j = 0; j < PER; ++j)
            if (lane + 32 * j < E) valid |= 1u << j;
        unsigned long long raw[PER + 1];
        flagged_poll(raw, valid, [&](int k) { return k < PER ? row + lane + 32 * k : row + E; }, tag, wait_bound(a));
        for (int g = lane; g < HG; g += 32) ss += ssq_l[t * HG + g];
#pragma unroll
        for (int j = 0; j < PER; ++j) p[j] = lane + 32 * j < E ? __uint_as_float((uint32_t)raw[j]) : -INFINITY;
        if (Ld.w_sg) score = __uint_as_float((uint32_t)raw[PER]);
    } else {
#pragma unroll
        for (int j = 0; j < PER; ++j) {
            const int e = lane + 32 * j;
            p[j] = e < E ? __ldcg(a.logits + (size_t)t * E + e) : -INFINITY;
        }
        for (int g = lane; g < HG; g += 32) ss += __ldcg(a.ssq + t * HG + g);
        score = Ld.w_sg ? __ldcg(a.score + t) : 0.0f;
    }
    ss = warp_sum(ss);
    const float r = a.norm_eps >= 0.0f ? rsqrtf(ss / (float)H + a.norm_eps) : 1.0f;
    if (st) st[19] = globaltimer();
    // top-k by repeated argmax over the RMS-scaled logits.  The softmax is
    // monotonic, so this selects what cpu_topk selects on the probabilities
    // (strict >: the lowest index wins ties); and the renormalised weights
    // p_k / sum(p_top) = exp(l_k - l_max) / sum exp(l_top - l_max) need no
    // full softmax.  Keys: the float bits made order-preserving as unsigned
    // (0 = taken or no expert); one warp max finds the value, one warp min the
    // lowest index holding it.
    unsigned key[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
        const unsigned b = __float_as_uint(p[j] * r);
        key[j] = (lane + 32 * j) < E ? (b & 0x80000000u ? ~b : b | 0x80000000u) : 0u;
    }
    float my_l = 0.0f, lmax = 0.0f;
    int my_i = 0;
    for (int k = 0; k < K; ++k) {
        unsigned best = 0;
#pragma unroll
        for (int j = 0; j < PER; ++j) best = key[j] > best ? key[j] : best;
        const unsigned mk = __reduce_max_sync(0xffffffffu, best);
        unsigned cand = 0xffffffffu;
#pragma unroll
        for (int j = PER - 1; j >= 0; --j)
            if (key[j] == mk) cand = (unsigned)(lane + 32 * j);
        const unsigned bi = __reduce_min_sync(0xffffffffu, cand);
        if constexpr (EVERY)
            early(k, (int)bi);
        else if (k == kw)
            early((int)bi);
        if ((int)(bi & 31) == lane) {
#pragma unroll
            for (int j = 0; j < PER; ++j)
                if (j == (int)(bi >> 5)) key[j] = 0;
        }
        const float lv = __uint_as_float(mk & 0x80000000u ? mk & 0x7fffffffu : ~mk);
        if (k == 0) lmax = lv;
        if (lane == k) {
            my_l = lv;
            my_i = (int)bi;
        }
    }
    const float my_e = lane < K ? expf(my_l - lmax) : 0.0f;
    const float wsum = warp_sum(my_e);
    const float my_w = my_e / wsum;
    if (st) st[20] = globaltimer();
    if (pick_i) {
        *pick_i = my_i;
        *pick_w = my_w;
        *pick_sg = Ld.w_sg ? 1.0f / (1.0f + expf(-(score * r))) : 0.5f;
    }
    // caller's copies: [T x K] of the launch's layer, or [L][T x K] when
    // every layer is recorded (out_per_layer)
    const size_t ob = a.out_per_layer ? (size_t)l * a.T : 0;
    if (lane < K) {
        idx[t * K + lane] = my_i;
        w[t * K + lane] = my_w;
        if (outputs && a.idx_out) a.idx_out[(ob + t) * K + lane] = my_i;
        if (outputs && a.w_out) a.w_out[(ob + t) * K + lane] = my_w;
    }
    if (lane == 0) {
        const float sg = Ld.w_sg ? 1.0f / (1.0f + expf(-(score * r))) : 0.5f;
        rinv[t] = r;
        sgw[t] = sg;
        if (outputs && a.sg_out) a.sg_out[ob + t] = sg;
    }
}

// Phase B routing tables, run by the 256 consumer threads of every CTA.
// Local (dist = false): the CTA routes every token itself.  Distributed: the
// grid routed the tokens into global memory (route_token, then a grid
// barrier) and the CTA copies them.  Then the (token, expert) pairs are
// grouped by expert: group 0 is the shared expert (all T tokens), then the
// routed experts held here, pairs token-major inside each group.
// LLM: the logits come as flagged words (llg, tag) and, before anything else,
// warp 0 waits for the presence word of every CTA for this layer (pres).
template <int PER, bool BIG, bool LLM = false, bool T1 = false, class Early = NoEarly, bool EVERY = false>
__device__ void route_tables(const StepArgs &a, const StepLayer &Ld, const RouteTabs &R, int l, bool cta0,
                             unsigned long long *st, bool dist, const unsigned long long *llg = nullptr,
                             const unsigned long long *pres = nullptr, const float *ssq_l = nullptr,
                             uint32_t tag = 0, int kw = -1, const Early &early = Early{})
{
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int T = T1 ? 1 : a.T, E = a.E, K = a.top_k;
    const int EL = a.hi - a.lo;
    if constexpr (LLM) {
        if (warp == 0 && pres) {
            const int G = gridDim.x;
            unsigned valid = 0;
#pragma unroll
            for (int k = 0; k < LL_GMAX / 32; ++k)
                if (lane + 32 * k < G) valid |= 1u << k;
            unsigned long long raw[LL_GMAX / 32];
            flagged_poll(raw, valid, [&](int k) { return pres + lane + 32 * k; }, tag, wait_bound(a));
        }
    }
    for (int i = tid; i < EL; i += ST_CONS) {
        R.cnt[i] = 0;
        R.run[i] = 0;
    }
    if (BIG && dist) {
        for (int i = tid; i < T * K; i += ST_CONS) {
            R.idx[i] = __ldcg(a.ridx + i);
            R.w[i] = __ldcg(a.rw + i);
        }
        for (int i = tid; i < T; i += ST_CONS) {
            R.rinv[i] = __ldcg(a.rinv + i);
            R.sgw[i] = __ldcg(a.rsgw + i);
        }
    } else if (!BIG && T == 1 && !a.route_only) {
        // One token (decode): the routing warp builds the tables from its
        // registers -- one pair per picked expert held here, shared expert
        // first, then the picks in top-k order.
        if (warp == 0) {
            int e;
            float w, sg;
            route_token<PER, LLM, Early, EVERY>(a, Ld, 0, R.idx, R.w, R.rinv, R.sgw, cta0, (st && lane == 0) ? st : nullptr,
                                         l, &e, &w, &sg, llg, ssq_l, tag, kw, early);
            const int hs = Ld.sh_gate ? 1 : 0;
            const bool loc = lane < K && e >= a.lo && e < a.hi;
            const unsigned locs = __ballot_sync(0xffffffffu, loc);
            const int g = hs + __popc(locs & ((1u << lane) - 1u));
            if (loc) {
                R.ptok[g] = 0;
                R.pw[g] = w;
                R.gexp[g] = e;
                R.goff[g] = g;
                R.gcnt[g] = 1;
                R.gcpre[g] = g;
                R.chunk[g] = make_int4(e, g, 1, 0);
                if (!Ld.gate_base) {
                    R.ptr[3 * (e - a.lo) + 0] = expert_ptr(Ld.gate, nullptr, e, E);
                    R.ptr[3 * (e - a.lo) + 1] = expert_ptr(Ld.up, nullptr, e, E);
                    R.ptr[3 * (e - a.lo) + 2] = expert_ptr(Ld.down, nullptr, e, E);
                }
            }
            if (lane == 0) {
                if (hs) {
                    R.ptok[0] = 0;
                    R.pw[0] = sg;
                    R.gexp[0] = E;
                    R.goff[0] = 0;
                    R.gcnt[0] = 1;
                    R.gcpre[0] = 0;
                    R.chunk[0] = make_int4(E, 0, 1, 0);
                }
                const int ng = hs + __popc(locs);
                R.gcpre[ng] = ng;
                R.scal[0] = ng;
                R.scal[1] = ng;
                R.scal[2] = ng;
                if (cta0 && a.stats) {
                    a.stats[2 * l] = ng;
                    a.stats[2 * l + 1] = ng;
                }
            }
            if (st && lane == 0) st[21] = globaltimer();
        }
        named_sync(BAR_CONS, ST_CONS);
        return;
    } else {
        for (int t = warp; t < T; t += 8)
            route_token<PER, LLM>(a, Ld, t, R.idx, R.w, R.rinv, R.sgw, cta0, (st && tid == 0) ? st : nullptr, l,
                                  nullptr, nullptr, nullptr, llg, ssq_l, tag);
    }
    named_sync(BAR_CONS, ST_CONS);
    if (a.route_only) return;

    const int P = T * K;
    if (!BIG && P <= 32) {
        // Few pairs (decode): one warp builds the tables with a handful of
        // warp-wide operations.  Lane q holds pair q = (token q / K, slot
        // q % K).  Groups: the shared expert first, then the routed experts in
        // order of their first pair (a fixed order, so every CTA and every
        // rank builds the same tables); pairs token-major inside each group.
        if (warp == 0) {
            const int hs = Ld.sh_gate ? 1 : 0;
            const int hsc = hs ? (T + MOE_TC - 1) / MOE_TC : 0;
            const int pb = hs ? T : 0;
            int e = -1 - lane;  // distinct dummies for lanes without a local pair
            float w = 0.0f;
            bool loc = false;
            if (lane < P) {
                const int ee = R.idx[lane];
                if (ee >= a.lo && ee < a.hi) {
                    e = ee;
                    w = R.w[lane];
                    loc = true;
                }
            }
            const unsigned lt = (1u << lane) - 1u;
            const unsigned peers = __match_any_sync(0xffffffffu, e);
            const int before = __popc(peers & lt), same = __popc(peers);
            const bool first = loc && before == 0;
            const unsigned firsts = __ballot_sync(0xffffffffu, first);
            const int g = hs + __popc(firsts & lt);  // group of this lane's expert (valid on first lanes)
            // exclusive prefix over first lanes of (pairs, chunks) of their group
            int vp = first ? same : 0, vc = first ? (same + MOE_TC - 1) / MOE_TC : 0;
            int ip = vp, ic = vc;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int tp = __shfl_up_sync(0xffffffffu, ip, o);
                const int tc = __shfl_up_sync(0xffffffffu, ic, o);
                if (lane >= o) {
                    ip += tp;
                    ic += tc;
                }
            }
            const int xp = ip - vp, xc = ic - vc;
            const int f = __ffs(peers) - 1;  // first lane of this lane's expert
            const int goff = pb + __shfl_sync(0xffffffffu, xp, f);
            if (loc) {
                R.ptok[goff + before] = lane / K;
                R.pw[goff + before] = w;
            }
            if (first) {
                R.gexp[g] = e;
                R.goff[g] = goff;
                R.gcnt[g] = same;
                R.gcpre[g] = hsc + xc;
                for (int k = 0; k < vc; ++k)
                    R.chunk[hsc + xc + k] = make_int4(e, goff + MOE_TC * k, min(MOE_TC, same - MOE_TC * k), 0);
                if (!Ld.gate_base) {
                    R.ptr[3 * (e - a.lo) + 0] = expert_ptr(Ld.gate, nullptr, e, E);
                    R.ptr[3 * (e - a.lo) + 1] = expert_ptr(Ld.up, nullptr, e, E);
                    R.ptr[3 * (e - a.lo) + 2] = expert_ptr(Ld.down, nullptr, e, E);
                }
            }
            const int ngr = __popc(firsts);
            const int npl = __shfl_sync(0xffffffffu, ip, 31);
            const int nchr = __shfl_sync(0xffffffffu, ic, 31);
            if (hs) {
                for (int t = lane; t < T; t += 32) {
                    R.ptok[t] = t;
                    R.pw[t] = R.sgw[t];
                }
                for (int k = lane; k < hsc; k += 32) R.chunk[k] = make_int4(E, MOE_TC * k, min(MOE_TC, T - MOE_TC * k), 0);
            }
            if (lane == 0) {
                if (hs) {
                    R.gexp[0] = E;
                    R.goff[0] = 0;
                    R.gcnt[0] = T;
                    R.gcpre[0] = 0;
                }
                const int ng = hs + ngr;
                R.gcpre[ng] = hsc + nchr;
                R.scal[0] = ng;
                R.scal[1] = hsc + nchr;
                R.scal[2] = pb + npl;
                if (cta0 && a.stats) {
                    a.stats[2 * l] = ng;
                    a.stats[2 * l + 1] = pb + npl;
                }
            }
        }
        if (st && tid == 0) st[21] = globaltimer();
        named_sync(BAR_CONS, ST_CONS);
        return;
    }

    for (int q = tid; q < P; q += ST_CONS) {
        const int e = R.idx[q];
        if (e >= a.lo && e < a.hi) atomicAdd(&R.cnt[e - a.lo], 1);
    }
    named_sync(BAR_CONS, ST_CONS);

    // warps 1..7: weight pointers of every expert used here, all loads in
    // flight together (the producer would otherwise chase them one by one)
    if (warp > 0 && !Ld.gate_base)
        for (int el = tid - 32; el < EL; el += ST_CONS - 32)
            if (R.cnt[el]) {
                const int e = a.lo + el;
                const uint8_t *g = expert_ptr(Ld.gate, nullptr, e, E);
                const uint8_t *u = expert_ptr(Ld.up, nullptr, e, E);
                const uint8_t *d = expert_ptr(Ld.down, nullptr, e, E);
                R.ptr[3 * el + 0] = g;
                R.ptr[3 * el + 1] = u;
                R.ptr[3 * el + 2] = d;
            }
    if (warp == 0) {
        const int hs = Ld.sh_gate ? 1 : 0;
        int gbase = hs, pbase = hs ? T : 0;
        if (hs && lane == 0) {
            R.gexp[0] = E;
            R.goff[0] = 0;
            R.gcnt[0] = T;
        }
        for (int c0 = 0; c0 < EL; c0 += 32) {
            const int el = c0 + lane;
            const int cnt = el < EL ? R.cnt[el] : 0;
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
                R.gexp[gid] = a.lo + el;
                R.goff[gid] = off;
                R.gcnt[gid] = cnt;
            }
            if (el < EL) R.off[el] = off;
            gbase += __shfl_sync(0xffffffffu, fi, 31);
            pbase += __shfl_sync(0xffffffffu, ci, 31);
        }
        __syncwarp();
        const int ng = gbase;
        int cbase = 0;
        for (int g0 = 0; g0 < ng; g0 += 32) {
            const int g = g0 + lane;
            const int ch = g < ng ? (R.gcnt[g] + MOE_TC - 1) / MOE_TC : 0;
            int ci = ch;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int c = __shfl_up_sync(0xffffffffu, ci, o);
                if (lane >= o) ci += c;
            }
            if (g < ng) R.gcpre[g] = cbase + ci - ch;
            cbase += __shfl_sync(0xffffffffu, ci, 31);
        }
        for (int q0 = 0; q0 < P; q0 += 32) {
            const int q = q0 + lane;
            int e = -1;
            bool loc = false;
            if (q < P) {
                e = R.idx[q];
                loc = e >= a.lo && e < a.hi;
            }
            const unsigned act = __ballot_sync(0xffffffffu, loc);
            if (loc) {
                const unsigned peers = __match_any_sync(act, e);
                const int rank = __popc(peers & ((1u << lane) - 1u));
                const int el = e - a.lo;
                const int pos = R.off[el] + R.run[el] + rank;
                R.ptok[pos] = q / K;
                R.pw[pos] = R.w[q];
                if (__ffs(peers) - 1 == lane) R.run[el] += __popc(peers);
            }
            __syncwarp();
        }
        if (hs)
            for (int t = lane; t < T; t += 32) {
                R.ptok[t] = t;
                R.pw[t] = R.sgw[t];
            }
        if (lane == 0) {
            R.gcpre[ng] = cbase;
            R.scal[0] = ng;
            R.scal[1] = cbase;
            R.scal[2] = pbase;
            if (cta0 && a.stats) {
                a.stats[2 * l] = ng;
                a.stats[2 * l + 1] = pbase;
            }
        }
    }
    named_sync(BAR_CONS, ST_CONS);
    for (int c = tid; c < R.scal[1]; c += ST_CONS) {
        const ChunkInfo ci = chunk_search(R, c);
        R.chunk[c] = make_int4(ci.e, ci.p0, ci.np, 0);
    }
    named_sync(BAR_CONS, ST_CONS);
}

// ---------------------------------------------------------------------------
// the step kernel
// ---------------------------------------------------------------------------
// MODE_BIG: more than ROUTER_TILE_T tokens (tiled router, shared ring arena,
// grid routing above ROUTE_DIST_T).  MODE_SMALL: up to ROUTER_TILE_T tokens
// with grid barriers (expert parallel, routing only).  MODE_LL: decode on one
// GPU, up to LL_TMAX tokens, CTAs exchanging flagged words instead of meeting
// at grid barriers (every CTA quantises the layer input itself).  Each
// instantiation carries only its own paths, which keeps the decode
// instruction footprint small.
// MODE_LLEP: the decode mode with expert parallelism -- every rank runs the
// flagged-word decode step on its own experts, and each column tile's owner
// stores its partial sums as flagged words into every rank's mailbox over
// NVLink, then polls the N partials of its tile in its own mailbox and adds
// them in rank order (so every rank holds the same bits and routes the same):
// no arrival counters, no system-scope release, no grid barrier.
constexpr int MODE_LL = 0, MODE_SMALL = 1, MODE_BIG = 2, MODE_LLEP = 3;
// T1: the decode modes compiled for exactly one token (the batch-1 decode
// step): every per-token loop and the batch paths of the routing drop out of
// the instruction stream, which is on this latency-bound step's critical path.
template <int NBH, int NBI, int MODE, bool T1 = false>
__global__ void __launch_bounds__(ST_THREADS, 1) moe_step_kernel(const __grid_constant__ StepArgs a)
{
    constexpr bool BIG = MODE == MODE_BIG;
    constexpr bool LL = MODE == MODE_LL || MODE == MODE_LLEP;
    constexpr bool LLEP = MODE == MODE_LLEP;
    static_assert(!T1 || LL, "the one-token instantiation is a decode mode");
    using C = SCfg<NBH, NBI>;
    using GH = typename C::GH;
    using GI = typename C::GI;
    constexpr int H = C::H, I = C::I;
    extern __shared__ __align__(128) uint8_t smem[];
    const StepSmem &m = a.sm;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, bx = blockIdx.x;
    const int T = T1 ? 1 : a.T, E = a.E;
    const int TC = T < MOE_TC ? T : MOE_TC;
    const int R = I / MOE_ROWTILE;  // gate/up row tiles per expert
    const int NT = H / MOE_RT3;     // 16-column tiles of h (down output)
    const bool ep = !LL && a.ep_world > 1;
    const bool norm = a.norm_eps >= 0.0f;
    const int NS_G = m.NS_G, NS_D = m.NS_D;
    const bool dist = BIG && T > ROUTE_DIST_T;        // routing spread over the grid (+1 barrier)
    constexpr bool arena = BIG;                       // gate/up and down rings share shared memory
    const int nbl = (ep ? 2 : 3) + (dist ? 1 : 0);    // grid barriers per layer

    float *rbuf = reinterpret_cast<float *>(smem + m.rbuf);
    float *part = reinterpret_cast<float *>(smem + m.part);
    RouteTabs RT;
    RT.idx = reinterpret_cast<int *>(smem + m.r_idx);
    RT.w = reinterpret_cast<float *>(smem + m.r_w);
    RT.rinv = reinterpret_cast<float *>(smem + m.r_rinv);
    RT.sgw = reinterpret_cast<float *>(smem + m.r_sgw);
    RT.cnt = reinterpret_cast<int *>(smem + m.r_cnt);
    RT.run = reinterpret_cast<int *>(smem + m.r_run);
    RT.off = reinterpret_cast<int *>(smem + m.r_off);
    RT.gexp = reinterpret_cast<int *>(smem + m.r_gexp);
    RT.goff = reinterpret_cast<int *>(smem + m.r_goff);
    RT.gcnt = reinterpret_cast<int *>(smem + m.r_gcnt);
    RT.gcpre = reinterpret_cast<int *>(smem + m.r_gcpre);
    RT.ptok = reinterpret_cast<int *>(smem + m.r_ptok);
    RT.pw = reinterpret_cast<float *>(smem + m.r_pw);
    RT.scal = reinterpret_cast<int *>(smem + m.r_scal);
    RT.ptr = reinterpret_cast<const uint8_t **>(smem + m.r_ptr);
    RT.chunk = reinterpret_cast<int4 *>(smem + m.r_chunk);
    // chunk c of the routing tables (one token: always one pair)
    auto cinfo = [&](int c) {
        ChunkInfo ci = chunk_info(RT, c);
        if (T1) ci.np = 1;
        return ci;
    };
    uint8_t *xsl = smem + m.xsl;
    uint8_t *gring = smem + m.gring;
    float *abuf = reinterpret_cast<float *>(smem + m.abuf);
    uint8_t *dring = smem + m.dring;
    float *acc = reinterpret_cast<float *>(smem + m.acc);
    // flagged-exchange mode: this CTA's quantised copy of the layer input,
    // the input itself (phase A) sharing bytes with the gathered intermediate
    // (phase C), and the input's per-32 sums of squares
    int16_t *xlq = reinterpret_cast<int16_t *>(smem + m.xloc);
    float *xls = reinterpret_cast<float *>(smem + m.xloc + (size_t)T * H * 2);
    float *xf = reinterpret_cast<float *>(smem + m.xf);
    int16_t *alq = reinterpret_cast<int16_t *>(smem + m.xf);
    float *als = reinterpret_cast<float *>(smem + m.xf + (size_t)T * (a.top_k + 1) * I * 2);
    float *ssql = reinterpret_cast<float *>(smem + m.ssql);
    uint64_t *bars = reinterpret_cast<uint64_t *>(smem + m.bars);
    uint64_t *rbar = bars;
    uint64_t *gfull = bars + 1, *gempty = gfull + NS_G;
    uint64_t *xfull = gempty + NS_G, *xempty = xfull + 2;
    uint64_t *dw = xempty + 2, *da = dw + NS_D, *dempty = da + NS_D;

    if (tid == 0) {
        mbar_init(rbar, 1);
        for (int s = 0; s < NS_G; ++s) {
            mbar_init(gfull + s, 1);
            mbar_init(gempty + s, 8);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(xfull + s, 1);
            mbar_init(xempty + s, 8);
        }
        for (int s = 0; s < NS_D; ++s) {
            mbar_init(dw + s, 1);
            mbar_init(da + s, 1);
            mbar_init(dempty + s, C::WS);
        }
        fence_mbar_init();
    }
    for (int i = tid; i < 8 * T * MOE_RT3; i += ST_THREADS) acc[i] = 0.0f;
    if (a.layers) {
        const unsigned long long *src = reinterpret_cast<const unsigned long long *>(a.layers);
        unsigned long long *dst = reinterpret_cast<unsigned long long *>(smem + m.ldesc);
        for (int i = tid; i < a.L * (int)(sizeof(StepLayer) / 8); i += ST_THREADS) dst[i] = __ldg(src + i);
    }
    __syncthreads();
    const unsigned long long epoch = __ldcg(a.ctrl + CTRL_EPOCH);
    const unsigned long long seq0 = __ldcg(a.ctrl + CTRL_SEQ);
    auto tag_of = [&](int l) { return (uint32_t)(seq0 + (unsigned long long)l + 1ull); };
    auto par_of = [&](int l) { return (size_t)(l & 1); };

    if (warp == 8) {
        // ================================================================ producer
        // All 32 lanes run the same control flow; the copies of different
        // ring slots are issued by different lanes in parallel (a single
        // thread's dependent address arithmetic costs several hundred ns per
        // copy).
        Ring gR, dR;   // gate/up and down rings, continued across layers
        int nX = 0;    // activation slots used (2 slots)
        auto pstamp = [&](int l, int k) {
            if (a.stamps && lane == 0) a.stamps[((size_t)l * G + bx) * STAMPS + k] = globaltimer();
        };
        // Router rows of layer l (and the shared-gate vector as row E) -> rbuf.
        auto issue_router = [&](int l) {
            const StepLayer Ld = layer_desc(a, l);
            if constexpr (BIG) {
                // tiled router: warm L2 with the rows of this CTA's units
                const int nrows = E + (Ld.w_sg ? 1 : 0);
                const int nrb = (nrows + 15) / 16;
                for (int u = bx + G * lane; u < nrb * ((T + 7) / 8); u += G * 32) {
                    const int r0 = (u % nrb) * 16, r1 = r0 + 16 < E ? r0 + 16 : E;
                    if (r1 > r0) prefetch_l2(Ld.W_r + (size_t)r0 * H, (unsigned)((r1 - r0) * H * 4));
                }
                if (lane == 0) mbar_arrive(rbar);
                return;
            }
            unsigned bytes = 0;
            for (int rl = 0; rl < m.RR; ++rl) {
                const int r = bx + rl * G;
                bytes += r < E ? H * 4 : (r == E && Ld.w_sg ? H * 2 : 0);
            }
            // the RMSNorm weight travels with the rows (needed first in phase A)
            const bool nwc = Ld.norm_w && a.norm_eps >= 0.0f && !(reinterpret_cast<uintptr_t>(Ld.norm_w) & 15);
            if (nwc) bytes += H * 4;
            if (lane == 0) {
                if (bytes)
                    mbar_arrive_expect_tx(rbar, bytes);
                else
                    mbar_arrive(rbar);
            }
            __syncwarp();
            const int r = bx + lane * G;
            if (lane < m.RR) {
                if (r < E)
                    bulk_g2s(rbuf + (size_t)lane * H, Ld.W_r + (size_t)r * H, H * 4, rbar);
                else if (r == E && Ld.w_sg)
                    bulk_g2s(rbuf + (size_t)lane * H, Ld.w_sg, H * 2, rbar);
            }
            if (nwc && lane == 31) bulk_g2s(smem + m.nwb, Ld.norm_w, H * 4, rbar);
        };
        // One gate/up sub-stage (SR gate rows + SR up rows from row r0) at ring
        // cursor g (called by the issuing lane).
        auto issue_gu = [&](const Ring &g, const uint8_t *gb, const uint8_t *ub, size_t r0) {
            if (g.used) swait(gempty + g.slot, (unsigned)(g.phase ^ 1));
            const unsigned bytes = (unsigned)(C::SR * GH::ROWB);
            uint8_t *dst = gring + (size_t)g.slot * C::STB;
            if (gb && ub && !((reinterpret_cast<uintptr_t>(gb) | reinterpret_cast<uintptr_t>(ub)) & 15)) {
                mbar_arrive_expect_tx(gfull + g.slot, 2 * bytes);
                bulk_g2s(dst, gb + r0 * GH::ROWB, bytes, gfull + g.slot);
                bulk_g2s(dst + bytes, ub + r0 * GH::ROWB, bytes, gfull + g.slot);
            } else {
                flag_error(DEVERR_ROUTE);
                mbar_arrive(gfull + g.slot);
            }
        };
        // The shared expert's pairs are the first chunks of every layer, so a
        // CTA whose first item is a shared one knows its rows before routing:
        // copy its first sub-stages at the next ring positions (ring drained).
        auto preissue_shared = [&](int l) -> int {
            const StepLayer Ld = layer_desc(a, l);
            if (arena || a.route_only || !Ld.sh_gate || bx >= ((T + MOE_TC - 1) / MOE_TC) * R) return 0;
            const int npre = C::SPI < NS_G ? C::SPI : NS_G;
            if (lane < npre)
                issue_gu(gR.ahead(lane, NS_G), Ld.sh_gate, Ld.sh_up,
                         (size_t)(bx % R) * MOE_ROWTILE + (size_t)lane * C::SR);
            __syncwarp();
            return npre;
        };
        issue_router(0);
        int npre = preissue_shared(0);
        for (int l = 0; l < a.L; ++l) {
            named_sync(BAR_ALL, ST_THREADS);  // routing tables of layer l are ready
            if (a.route_only) break;
            if (T1 && RT.scal[3] > 0) npre = RT.scal[3];  // issued by the routing warp at its pick
            pstamp(l, 10);
            const StepLayer Ld = layer_desc(a, l);
            // (the copies below read data other CTAs wrote only in barrier modes)
            if constexpr (!LL) fence_proxy_async_global();
            const int nch = RT.scal[1];
            // gate/up items (chunk c, row tile rt): activations of the chunk's
            // tokens + 32 gate and up rows in sub-stages
            for (int it = bx; it < nch * R; it += G, ++nX) {
                const int c = it / R, rt = it % R;  // R: a power of two
                const ChunkInfo ci = cinfo(c);
                if constexpr (!LL) {  // (flagged mode: every CTA quantised the input itself)
                    const int xs_ = nX & 1;
                    if (lane == 0) {
                        if (nX >= 2) swait(xempty + xs_, (unsigned)(((nX >> 1) - 1) & 1));
                        mbar_arrive_expect_tx(xfull + xs_, (unsigned)(ci.np * C::XTOK));
                    }
                    __syncwarp();
                    if (lane < ci.np) {
                        uint8_t *xb = xsl + (size_t)xs_ * m.xslot;
                        const int t = RT.ptok[ci.p0 + lane];
                        bulk_g2s(xb + (size_t)lane * H * 2, a.xq + (size_t)t * H, H * 2, xfull + xs_);
                        bulk_g2s(xb + (size_t)TC * H * 2 + (size_t)lane * (H / 8), a.xs + (size_t)t * (H / 32), H / 8,
                                 xfull + xs_);
                    }
                }
                const uint8_t *gb = mat_ptr(RT, Ld, a, ci.e, 0);
                const uint8_t *ub = mat_ptr(RT, Ld, a, ci.e, 1);
                for (int s0 = 0; s0 < C::SPI; s0 += NS_G) {  // batches of distinct slots
                    const int nb = C::SPI - s0 < NS_G ? C::SPI - s0 : NS_G;
                    const int s = s0 + lane;
                    if (lane < nb && !(it == bx && s < npre))  // (else copied during the previous layer)
                        issue_gu(gR.ahead(lane, NS_G), gb, ub, (size_t)rt * MOE_ROWTILE + (size_t)s * C::SR);
                    gR = gR.ahead(nb, NS_G);
                    __syncwarp();
                }
            }
            npre = 0;
            pstamp(l, 11);
            // down stages n = (tile, chunk), tile-major: the weights depend only
            // on the routing, so the first NS_D go out now and are in flight
            // while the gate/up items compute; the intermediate follows after
            // the grid barrier
            const int my_tiles = bx < NT ? (NT - 1 - bx) / G + 1 : 0;
            const int nds = my_tiles * nch;
            const int dpre = arena ? 0 : (nds < NS_D ? nds : NS_D);
            auto issue_dw = [&](const Ring &d, int n) {
                if (d.used) swait(dempty + d.slot, (unsigned)(d.phase ^ 1));
                const ChunkInfo ci = cinfo(n % nch);
                const int it3 = bx + (n / nch) * G;
                const uint8_t *db = mat_ptr(RT, Ld, a, ci.e, 2);
                if (db && !(reinterpret_cast<uintptr_t>(db) & 15)) {
                    mbar_arrive_expect_tx(dw + d.slot, (unsigned)C::WB);
                    bulk_g2s(dring + (size_t)d.slot * m.dslot, db + (size_t)it3 * MOE_RT3 * GI::ROWB, (unsigned)C::WB,
                             dw + d.slot);
                } else {
                    flag_error(DEVERR_ROUTE);
                    mbar_arrive(dw + d.slot);
                }
            };
            auto issue_da = [&](const Ring &d, int n) {
                const ChunkInfo ci = cinfo(n % nch);
                uint8_t *st = dring + (size_t)d.slot * m.dslot + C::WB;
                mbar_arrive_expect_tx(da + d.slot, (unsigned)(ci.np * C::ATOK));
                bulk_g2s(st, a.aq + (size_t)ci.p0 * I, (unsigned)(ci.np * I * 2), da + d.slot);
                bulk_g2s(st + (size_t)TC * I * 2, a.as + (size_t)ci.p0 * (I / 32), (unsigned)(ci.np * (I / 8)),
                         da + d.slot);
            };
            // The down weights are needed only after the next grid barrier:
            // request them once this CTA's gate/up stages have landed, so they
            // do not compete with them for HBM (nor do the next layer's router
            // rows, issued with them).
            if (dpre > 0 && nch * R > bx) {
                if (lane < C::SPI && lane < NS_G) {
                    // stage issued `lane + 1` positions before the cursor: its slot
                    // is that of NS_G - 1 - lane positions ahead, one lap earlier
                    const Ring g = gR.ahead(NS_G - 1 - lane, NS_G);
                    swait(gfull + g.slot, (unsigned)(g.phase ^ 1));
                }
                __syncwarp();
            }
            if (lane < dpre) issue_dw(dR.ahead(lane, NS_D), lane);
            __syncwarp();
            pstamp(l, 12);
            if (l + 1 < a.L) issue_router(l + 1);  // consumers are past phase A
            pstamp(l, 13);
            // the intermediate of every CTA is complete after grid barrier (phase
            // B); flagged mode: the consumers gather it themselves
            if constexpr (!LL) {
                if (lane == 0) {
                    const int bidx = l * nbl + (dist ? 2 : 1);
                    wait_counter(a.ctrl + CTRL_GRID, (unsigned long long)(bidx + 1) * G, false, wait_bound(a));
                }
                __syncwarp();
                fence_proxy_async_global();
            }
            pstamp(l, 14);
            for (int n0 = 0; n0 < nds; n0 += NS_D) {  // batches of distinct slots
                const int nb = nds - n0 < NS_D ? nds - n0 : NS_D;
                if (lane < nb) {
                    const Ring d = dR.ahead(lane, NS_D);
                    if (n0 + lane >= dpre) issue_dw(d, n0 + lane);
                    if constexpr (!LL) issue_da(d, n0 + lane);
                }
                dR = dR.ahead(nb, NS_D);
                __syncwarp();
            }
            pstamp(l, 15);
            if (l + 1 < a.L) npre = preissue_shared(l + 1);
        }
        return;
    }

    // ==================================================================== consumers
    Ring gR, dR;
    int nX = 0;
    int bar = 0;
    const bool stamp = a.stamps && tid == 0;
    auto stamp_at = [&](int l, int k) { a.stamps[((size_t)l * G + bx) * STAMPS + k] = globaltimer(); };
    for (int l = 0; l < a.L; ++l) {
        const StepLayer Ld = layer_desc(a, l);
        // ------------------------------------------------------------ phase A
        const float *src = in_of(a, l);
        const float *pmb = nullptr;  // layer l-1's partials in this rank's mailbox (EP)
        if (ep && l > 0) {
            const int s = ep_slot(a.L, l - 1);
            if (tid == 0) wait_counter(ep_counter(a, a.ep_rank, s), ep_target(a, l - 1, epoch, NT), true, a.ep_wait_ns);
            named_sync(BAR_CONS, ST_CONS);
            src = in_of(a, l - 1);
            pmb = a.ep_mb[a.ep_rank] + mb_slot_off(s, a);
        }
        if (stamp) stamp_at(l, 0);
        const size_t TH = (size_t)a.ep_tmax * H;
        const uint32_t tg = tag_of(l);
        auto xin = [&](size_t i) -> float {
            if constexpr (LL) return xf[i];
            float v = __ldcg(src + i);
            if (pmb)
                for (int r = 0; r < a.ep_world; ++r) v += __ldcg(pmb + (size_t)r * TH + i);
            return v;
        };
        auto xin4 = [&](size_t i) -> float4 {  // i: a multiple of 4
            if constexpr (LL) return *reinterpret_cast<const float4 *>(xf + i);
            float4 v = __ldcg(reinterpret_cast<const float4 *>(src + i));
            if (pmb)
                for (int r = 0; r < a.ep_world; ++r) {
                    const float4 q = __ldcg(reinterpret_cast<const float4 *>(pmb + (size_t)r * TH + i));
                    v.x += q.x;
                    v.y += q.y;
                    v.z += q.z;
                    v.w += q.w;
                }
            return v;
        };
        // the layer input times the RMSNorm weight (rmsnorm_inplace,
        // one_layer.cu:158-180: x * rms * w; the rms factor is applied later
        // to the logits and to the activations' group scales)
        // (one-GPU and small-batch modes: the copy in shared memory, landed
        // with the router rows -- so that wait comes first; a misaligned
        // weight vector is read from global memory)
        const float *nw = norm ? Ld.norm_w : nullptr;
        if (!BIG && nw) {
            swait(rbar, (unsigned)(l & 1));
            if (!(reinterpret_cast<uintptr_t>(Ld.norm_w) & 15)) nw = reinterpret_cast<const float *>(smem + m.nwb);
        }
        // (decode mode: xf already holds the weighted input, see below)
        auto xinw = [&](size_t i) -> float {
            if constexpr (LL) return xin(i);
            const float v = xin(i);
            return nw ? v * nw[i & (size_t)(H - 1)] : v;  // H: a power of two
        };
        auto xin4w = [&](size_t i) -> float4 {  // i: a multiple of 4
            if constexpr (LL) return xin4(i);
            float4 v = xin4(i);
            if (nw) {
                const float4 w = *reinterpret_cast<const float4 *>(nw + (i & (size_t)(H - 1)));
                v.x *= w.x;
                v.y *= w.y;
                v.z *= w.z;
                v.w *= w.w;
            }
            return v;
        };
        if constexpr (LL) {
            // (1) the whole layer input into shared memory: the caller's x for
            // layer 0, else the previous layer's flagged output words
            const int n = T * H;
            if (l == 0) {
                for (int i = 4 * tid; i < n; i += 4 * ST_CONS)
                    *reinterpret_cast<float4 *>(xf + i) = __ldcg(reinterpret_cast<const float4 *>(src + i));
            } else {
                const unsigned long long *hin = a.ll_h + par_of(l - 1) * a.ll_h_n;
                const uint32_t tgp = tag_of(l - 1);
                for (int i0 = tid; i0 < n; i0 += 8 * ST_CONS) {
                    unsigned valid = 0;
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if (i0 + k * ST_CONS < n) valid |= 1u << k;
                    unsigned long long r[8];
                    flagged_poll(r, valid, [&](int k) { return hin + i0 + k * ST_CONS; }, tgp, wait_bound(a));
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        if ((valid >> k) & 1u) xf[i0 + k * ST_CONS] = __uint_as_float((uint32_t)r[k]);
                }
            }
            named_sync(BAR_CONS, ST_CONS);
            // (2) per-32 sums of squares (all that routing needs), four groups
            // at a time so their reductions interleave; the int16 quantisation
            // follows the router rows, below.  (Published to the routing warps
            // by the consumer barrier after the router dots.)
            const int ngr = T * (H / 32);
            for (int g0 = warp; g0 < ngr; g0 += 32) {
                float v[4];
#pragma unroll
                for (int k = 0; k < 4; ++k) {
                    const int gi = g0 + 8 * k;
                    const float x = gi < ngr ? xf[gi * 32 + lane] : 0.0f;
                    v[k] = x * x;
                    // RMSNorm weight: the lane rewrites the value it read
                    if (nw && gi < ngr) xf[gi * 32 + lane] = x * nw[(gi * 32 + lane) & (H - 1)];
                }
#pragma unroll
                for (int o = 16; o; o >>= 1)
#pragma unroll
                    for (int k = 0; k < 4; ++k) v[k] += __shfl_xor_sync(0xffffffffu, v[k], o);
                if (lane == 0)
#pragma unroll
                    for (int k = 0; k < 4; ++k)
                        if (g0 + 8 * k < ngr) ssql[g0 + 8 * k] = v[k];
            }
            if (nw) named_sync(BAR_CONS, ST_CONS);  // the weighted input, read by every warp below
        } else {
            // (1) this CTA's share of the int16 quantisation (+ group sums of squares)
            const int ngr = T * (H / 32);
            for (int gi = (G - 1 - bx) * 8 + warp; gi < ngr; gi += G * 8) {
                const float v = xin((size_t)gi * 32 + lane);
                const float ss = warp_sum(v * v);
                if (lane == 0) a.ssq[gi] = ss;
                const int q = quant32(nw ? v * nw[((size_t)gi * 32 + lane) & (size_t)(H - 1)] : v, a.xs + gi,
                                      lane);
                const int e = gi * 32 + lane, t = e / H;  // H: a power of two
                a.xq[(size_t)t * H + xq_pos(e - t * H)] = (int16_t)q;
            }
        }
        if (stamp) stamp_at(l, 16);
        // (2) EP: the owner of each column tile materialises this layer's input
        if (pmb) {
            float *dst = const_cast<float *>(in_of(a, l));
            for (int it3 = bx; it3 < NT; it3 += G)
                for (int i = tid; i < T * MOE_RT3; i += ST_CONS) {
                    const size_t o = (size_t)(i / MOE_RT3) * H + (size_t)it3 * MOE_RT3 + i % MOE_RT3;
                    dst[o] = xin(o);
                }
        }
        // (3) router rows of this CTA (row E = fp16 shared-gate vector)
        swait(rbar, (unsigned)(l & 1));
        if (stamp) stamp_at(l, 17);
        if constexpr (BIG) {
            // Many tokens: units of 16 router rows x 8 tokens.  The unit's
            // tokens are staged in shared memory (the activation slots are idle
            // in this phase); each warp computes two whole rows for them, with
            // the rows read from L2 (prefetched during the previous layer).
            const int nrows = E + (Ld.w_sg ? 1 : 0);
            const int nrb = (nrows + 15) / 16, ntb = (T + 7) / 8;
            float *xst = reinterpret_cast<float *>(xsl);
            for (int u = bx; u < nrb * ntb; u += G) {
                const int rb = u % nrb, t0 = (u / nrb) * 8;
                const int tn = T - t0 < 8 ? T - t0 : 8;
                for (int i = tid; i < tn * (H / 4); i += ST_CONS) {
                    const int t = i / (H / 4), c4 = i % (H / 4);
                    reinterpret_cast<float4 *>(xst)[i] = xin4w((size_t)(t0 + t) * H + 4 * c4);
                }
                named_sync(BAR_CONS, ST_CONS);
                for (int rr = 0; rr < 2; ++rr) {
                    const int row = rb * 16 + 2 * warp + rr;
                    if (row >= nrows) break;
                    float acc8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
                    for (int cb = 0; cb < H; cb += 1024) {  // 8 loads per lane in flight per round
                        float4 w4[8];
#pragma unroll
                        for (int j = 0; j < 8; ++j) {
                            const int c = cb + 4 * lane + 128 * j;
                            if (c >= H) {
                                w4[j] = make_float4(0.f, 0.f, 0.f, 0.f);
                            } else if (row < E) {
                                w4[j] = __ldcg(reinterpret_cast<const float4 *>(Ld.W_r + (size_t)row * H + c));
                            } else {
                                const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(Ld.w_sg + c));
                                const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(Ld.w_sg + c + 2));
                                w4[j] = make_float4(lo.x, lo.y, hi.x, hi.y);
                            }
                        }
#pragma unroll
                        for (int t = 0; t < 8; ++t)
                            if (t < tn) {
#pragma unroll
                                for (int j = 0; j < 8; ++j) {
                                    const int c = cb + 4 * lane + 128 * j;
                                    if (c < H) {
                                        const float4 x4 = reinterpret_cast<const float4 *>(xst)[((size_t)t * H + c) >> 2];
                                        acc8[t] = fmaf(w4[j].x, x4.x,
                                                       fmaf(w4[j].y, x4.y, fmaf(w4[j].z, x4.z, fmaf(w4[j].w, x4.w, acc8[t]))));
                                    }
                                }
                            }
                    }
#pragma unroll
                    for (int t = 0; t < 8; ++t)
                        if (t < tn) {
                            const float v = warp_sum(acc8[t]);
                            if (lane == 0) {
                                if (row < E)
                                    a.logits[(size_t)(t0 + t) * E + row] = v;
                                else
                                    a.score[t0 + t] = v;
                            }
                        }
                }
                // the staging area is refilled next (generic writes) and later by
                // bulk copies (async proxy)
                fence_proxy_async_smem();
                named_sync(BAR_CONS, ST_CONS);
            }
            if (stamp) stamp_at(l, 18);
        } else {
            const int rl = warp / m.WPR, qt = warp % m.WPR;
            const int row = bx + rl * G;
            const int nrows = E + (Ld.w_sg ? 1 : 0);
            const int seg = H / m.WPR, c0 = qt * seg;
            if (row < nrows) {
                const float *wr = rbuf + (size_t)rl * H;
                const __half *wh = reinterpret_cast<const __half *>(wr);
                if ((seg & 127) == 0) {
                    // float4 per lane, 4 per 512 columns: 2 tokens per pass,
                    // every load in flight before the first use
                    const float4 *w4 = reinterpret_cast<const float4 *>(wr);
                    for (int t0 = 0; t0 < T; t0 += 2) {
                        const bool two = t0 + 1 < T;
                        float s0 = 0.0f, s1 = 0.0f;
                        for (int cb = c0; cb < c0 + seg; cb += 512) {
                            float4 x0[4], x1[4];
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const int c = cb + 4 * lane + 128 * j;
                                const bool in = c < c0 + seg;
                                x0[j] = in ? xin4w((size_t)t0 * H + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                                x1[j] = (in && two) ? xin4w((size_t)(t0 + 1) * H + c) : make_float4(0.f, 0.f, 0.f, 0.f);
                            }
#pragma unroll
                            for (int j = 0; j < 4; ++j) {
                                const int c = cb + 4 * lane + 128 * j;
                                if (c < c0 + seg) {
                                    float4 w;
                                    if (row < E) {
                                        w = w4[c >> 2];
                                    } else {
                                        const float2 lo = __half22float2(*reinterpret_cast<const __half2 *>(wh + c));
                                        const float2 hi = __half22float2(*reinterpret_cast<const __half2 *>(wh + c + 2));
                                        w = make_float4(lo.x, lo.y, hi.x, hi.y);
                                    }
                                    s0 = fmaf(w.x, x0[j].x, fmaf(w.y, x0[j].y, fmaf(w.z, x0[j].z, fmaf(w.w, x0[j].w, s0))));
                                    s1 = fmaf(w.x, x1[j].x, fmaf(w.y, x1[j].y, fmaf(w.z, x1[j].z, fmaf(w.w, x1[j].w, s1))));
                                }
                            }
                        }
                        s0 = warp_sum(s0);
                        s1 = warp_sum(s1);
                        if (lane == 0) {
                            part[(rl * m.WPR + qt) * T + t0] = s0;
                            if (two) part[(rl * m.WPR + qt) * T + t0 + 1] = s1;
                        }
                    }
                } else {
                    // narrow segments (H / warps-per-row < 128): scalar loads
                    for (int t = 0; t < T; ++t) {
                        float s0 = 0.0f;
                        for (int c = c0 + lane; c < c0 + seg; c += 32) {
                            const float w = row < E ? wr[c] : __half2float(wh[c]);
                            s0 = fmaf(w, xinw((size_t)t * H + c), s0);
                        }
                        s0 = warp_sum(s0);
                        if (lane == 0) part[(rl * m.WPR + qt) * T + t] = s0;
                    }
                }
            }
            if (stamp) stamp_at(l, 18);
            named_sync(BAR_CONS, ST_CONS);
            for (int i = tid; i < m.RR * T; i += ST_CONS) {
                const int r_l = i / T, t = i % T, rr = bx + r_l * G;
                if (rr < nrows) {
                    float v = 0.0f;
                    for (int q = 0; q < m.WPR; ++q) v += part[(r_l * m.WPR + q) * T + t];
                    if constexpr (LL)
                        st_flagged(a.ll_lg + par_of(l) * a.ll_lg_n + (size_t)t * (E + 1) + rr, __float_as_uint(v), tg);
                    else if (rr < E)
                        a.logits[(size_t)t * E + rr] = v;
                    else
                        a.score[t] = v;
                }
            }
            // flagged mode: this CTA is done with the layer input (and with
            // everything of layer l-1).  With a router row in every CTA (rows
            // r -> CTA r mod G) its logits say so; else its presence word does
            if (LL && nrows < G && tid == 0) st_flagged(a.ll_pres + par_of(l) * a.ll_pres_n + bx, 0u, tg);
        }
        if constexpr (LL) {
            // the whole input quantised to int16 per 32, after the logits are
            // out: it overlaps the wait for the other CTAs' logits.  One token:
            // warp 0 routes meanwhile (warps 1..7 quantise); the routing's
            // consumer barriers publish the values before any gate/up item.
            const int w0 = T == 1 ? 1 : 0, nw = 8 - w0, ngq = T * (H / 32);
            if (warp >= w0) {
                // four groups per round (groups warp - w0 + nw * m), their
                // reductions interleaved
                for (int m0 = 0; warp - w0 + nw * m0 < ngq; m0 += 4) {
                    float v[4], sc[4];
                    int q[4];
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int gi = warp - w0 + nw * (m0 + k);
                        v[k] = gi < ngq ? xf[gi * 32 + lane] : 0.0f;
                    }
                    quant32_n<4>(v, q, sc);
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        const int gi = warp - w0 + nw * (m0 + k);
                        if (gi < ngq) {
                            const int e = gi * 32 + lane, t = e / H;  // H: a power of two
                            xlq[(size_t)t * H + xq_pos(e - t * H)] = (int16_t)q[k];
                            if (lane == 0) xls[gi] = sc[k];
                        }
                    }
                }
            }
        }
        if (stamp) stamp_at(l, 1);
        if constexpr (!LL) grid_barrier(a, bar++, tid);
        if (stamp) stamp_at(l, 2);

        // ------------------------------------------------------------ phase B
        unsigned long long *st_l = stamp ? a.stamps + ((size_t)l * G + bx) * STAMPS : nullptr;
        if (BIG && dist) {
            // one warp of the grid per token, then every CTA reads the result
            for (int t = bx * 8 + warp; t < T; t += G * 8) {
                if (E <= 256)
                    route_token<8>(a, Ld, t, a.ridx, a.rw, a.rinv, a.rsgw, true, nullptr, l);
                else
                    route_token<MOE_EMAX / 32>(a, Ld, t, a.ridx, a.rw, a.rinv, a.rsgw, true, nullptr, l);
            }
            grid_barrier(a, bar++, tid);
        }
        {
            const unsigned long long *llg = LL ? a.ll_lg + par_of(l) * a.ll_lg_n : nullptr;
            const unsigned long long *pres =
                (LL && E + (Ld.w_sg ? 1 : 0) < G) ? a.ll_pres + par_of(l) * a.ll_pres_n : nullptr;
            if constexpr (T1 && MODE == MODE_LLEP) {
                // One token with expert parallelism: the same early request
                // as below, but a rank's chunks are its own picks in top-k
                // order, so the routing warp counts the local picks as they
                // come and requests this CTA's item at the local pick of its
                // chunk.
                const int hs = Ld.sh_gate ? 1 : 0, c0 = bx / R;
                const int kw = (Ld.gate_base && c0 >= hs && c0 < hs + a.top_k) ? c0 - hs : -1;
                if (warp == 0 && lane == 0) RT.scal[3] = 0;
                int nloc = 0;  // local picks so far (the same on every lane)
                auto early = [&](int, int e) {
                    if (e < a.lo || e >= a.hi) return;
                    if (nloc++ != kw) return;
                    const int n = C::SPI < NS_G ? C::SPI : NS_G;
                    const size_t j = (size_t)(e - a.lo);
                    const uint8_t *gb = Ld.gate_base + j * Ld.gu_stride, *ub = Ld.up_base + j * Ld.gu_stride;
                    if (lane < n) {
                        const Ring g = gR.ahead(lane, NS_G);
                        const unsigned bytes = (unsigned)(C::SR * GH::ROWB);
                        const size_t r0 = (size_t)(bx % R) * MOE_ROWTILE + (size_t)lane * C::SR;
                        uint8_t *dst = gring + (size_t)g.slot * C::STB;
                        if (!((reinterpret_cast<uintptr_t>(gb) | reinterpret_cast<uintptr_t>(ub)) & 15)) {
                            mbar_arrive_expect_tx(gfull + g.slot, 2 * bytes);
                            bulk_g2s(dst, gb + r0 * GH::ROWB, bytes, gfull + g.slot);
                            bulk_g2s(dst + bytes, ub + r0 * GH::ROWB, bytes, gfull + g.slot);
                        } else {
                            flag_error(DEVERR_ROUTE);
                            mbar_arrive(gfull + g.slot);
                        }
                    }
                    if (lane == 0) RT.scal[3] = n;
                };
                route_tables<8, BIG, LL, T1, decltype(early), true>(a, Ld, RT, l, bx == 0, st_l, dist, llg, pres, ssql,
                                                                    tg, -1, early);
            } else if constexpr (T1) {
                // One token: the routing warp requests this CTA's first gate/up
                // item itself as soon as the item's expert is picked (pick
                // bx / R - shared, in top-k order: the order of the chunks),
                // into the ring positions the producer would use next (the
                // consumers' cursor mirrors it; the slots' previous uses ended
                // in the last layer's item loop, which every consumer warp has
                // left), and tells the producer how many sub-stages to skip.
                const int hs = Ld.sh_gate ? 1 : 0, c0 = bx / R;
                // (one GPU: with expert parallelism the chunks follow the
                // rank's own picks -- the instantiation above)
                const int kw = (Ld.gate_base && a.ep_world == 1 && c0 >= hs && c0 < hs + a.top_k) ? c0 - hs : -1;
                if (warp == 0 && lane == 0) RT.scal[3] = 0;
                auto early = [&](int e) {
                    if (e < a.lo || e >= a.hi) return;
                    const int n = C::SPI < NS_G ? C::SPI : NS_G;
                    const size_t j = (size_t)(e - a.lo);
                    const uint8_t *gb = Ld.gate_base + j * Ld.gu_stride, *ub = Ld.up_base + j * Ld.gu_stride;
                    if (lane < n) {
                        const Ring g = gR.ahead(lane, NS_G);
                        const unsigned bytes = (unsigned)(C::SR * GH::ROWB);
                        const size_t r0 = (size_t)(bx % R) * MOE_ROWTILE + (size_t)lane * C::SR;
                        uint8_t *dst = gring + (size_t)g.slot * C::STB;
                        if (!((reinterpret_cast<uintptr_t>(gb) | reinterpret_cast<uintptr_t>(ub)) & 15)) {
                            mbar_arrive_expect_tx(gfull + g.slot, 2 * bytes);
                            bulk_g2s(dst, gb + r0 * GH::ROWB, bytes, gfull + g.slot);
                            bulk_g2s(dst + bytes, ub + r0 * GH::ROWB, bytes, gfull + g.slot);
                        } else {
                            flag_error(DEVERR_ROUTE);
                            mbar_arrive(gfull + g.slot);
                        }
                    }
                    if (lane == 0) RT.scal[3] = n;
                };
                route_tables<8, BIG, LL, T1>(a, Ld, RT, l, bx == 0, st_l, dist, llg, pres, ssql, tg, kw, early);
            } else if (LL || E <= 256)  // (decode mode is used only with E <= 256)
                route_tables<8, BIG, LL, T1>(a, Ld, RT, l, bx == 0, st_l, dist, llg, pres, ssql, tg);
            else
                route_tables<MOE_EMAX / 32, BIG, LL>(a, Ld, RT, l, bx == 0, st_l, dist, llg, pres, ssql, tg);
        }
        if (stamp) stamp_at(l, 3);
        named_sync(BAR_ALL, ST_THREADS);
        if (a.route_only) break;
        const int nch = RT.scal[1];
        {
            const int rho = lane / GH::LPR, lr = lane % GH::LPR, bb = lr >> 2, sub = lr & 3;
            const int rs = warp * GH::RPW + rho;            // row inside a sub-stage
            const bool has_rows = warp * GH::RPW < C::SR;   // H = 256: only warps 0..3 have rows
            XSlice X[GH::CP];
            for (int it = bx; it < nch * R; it += G, ++nX) {
                const int c = it / R, rt = it % R;  // R: a power of two
                const ChunkInfo ci = cinfo(c);
                const int xs_ = nX & 1;
                if constexpr (!LL) swait(xfull + xs_, (unsigned)((nX >> 1) & 1));
                if (stamp && it == bx) stamp_at(l, 4);
                const uint8_t *xb = xsl + (size_t)xs_ * m.xslot;
                // the chunk's token j (token t): its int16 activations and group
                // scales (flagged mode: this CTA's own copy of every token)
                auto xq_of = [&](int j, int t) -> const int16_t * {
                    if constexpr (LL) return xlq + (size_t)t * H;
                    return reinterpret_cast<const int16_t *>(xb) + (size_t)j * H;
                };
                auto xs_of = [&](int j, int t) -> const float * {
                    if constexpr (LL) return xls + (size_t)t * (H / 32);
                    return reinterpret_cast<const float *>(xb + (size_t)TC * H * 2) + (size_t)j * (H / 32);
                };
                if (C::SPI <= NS_G) {
                    // The item's sub-stages are in flight together: wait for all,
                    // then per token one activation slice feeds the item's
                    // 2 x SPI row dot products (independent chains).
#pragma unroll
                    for (int s = 0; s < C::SPI; ++s) {
                        const Ring g = gR.ahead(s, NS_G);
                        swait(gfull + g.slot, (unsigned)g.phase);
                    }
                    for (int j = 0; has_rows && j < ci.np; ++j) {
                        {
                            const int t = RT.ptok[ci.p0 + j];
                            const float rsc = norm ? RT.rinv[t] : 1.0f;
#pragma unroll
                            for (int cp = 0; cp < GH::CP; ++cp)
                                load_slice_q4k(X[cp], xq_of(j, t), xs_of(j, t), QK * (cp * 8 + bb) + 64 * sub, rsc);
                        }
                        // v[2s] = gate row dot, v[2s+1] = up row dot of sub-stage s
                        constexpr int NV = 2 * C::SPI;
                        float v[NV];
#pragma unroll
                        for (int s = 0; s < C::SPI; ++s) {
                            const uint8_t *grow =
                                gring + (size_t)gR.ahead(s, NS_G).slot * C::STB + (size_t)rs * GH::ROWB;
                            const uint8_t *urow = grow + (size_t)C::SR * GH::ROWB;
                            v[2 * s] = 0.0f;
                            v[2 * s + 1] = 0.0f;
#pragma unroll
                            for (int cp = 0; cp < GH::CP; ++cp) {
                                v[2 * s] += q4k_lane_dot(grow + (size_t)(cp * 8 + bb) * Q4K_BYTES, sub, X[cp]);
                                v[2 * s + 1] += q4k_lane_dot(urow + (size_t)(cp * 8 + bb) * Q4K_BYTES, sub, X[cp]);
                            }
                        }
                        // transposed reduction over the row's lanes: lane group
                        // q = top bits of lr holds value q (gate of sub-stage
                        // q/2 when q is even); its up value sits LPR/NV lanes up
                        static_assert(NV <= GH::LPR, "gate/up values per lane exceed the row's lanes");
                        const float r = tr_reduce<NV, GH::LPR>(v);
                        const float u = __shfl_xor_sync(0xffffffffu, r, GH::LPR / NV);
                        if ((lr & (2 * GH::LPR / NV - 1)) == 0) {
                            const int sidx = (lr / (GH::LPR / NV)) >> 1;
                            abuf[j * MOE_ROWTILE + sidx * C::SR + rs] = r / (1.0f + expf(-r)) * u;
                        }
                    }
                    __syncwarp();
                    if (lane == 0)
#pragma unroll
                        for (int s = 0; s < C::SPI; ++s) mbar_arrive(gempty + gR.ahead(s, NS_G).slot);
                    gR = gR.ahead(C::SPI, NS_G);
                } else {
                    for (int s = 0; s < C::SPI; ++s, gR.next(NS_G)) {
                        const int slot = gR.slot;
                        swait(gfull + slot, (unsigned)gR.phase);
                        const uint8_t *grow = gring + (size_t)slot * C::STB + (size_t)rs * GH::ROWB;
                        const uint8_t *urow = grow + (size_t)C::SR * GH::ROWB;
                        for (int j = 0; has_rows && j < ci.np; ++j) {
                            if (ci.np > 1 || s == 0) {  // one token: its slice stays in registers across sub-stages
                                const int t = RT.ptok[ci.p0 + j];
                                const float rsc = norm ? RT.rinv[t] : 1.0f;
#pragma unroll
                                for (int cp = 0; cp < GH::CP; ++cp)
                                    load_slice_q4k(X[cp], xq_of(j, t), xs_of(j, t), QK * (cp * 8 + bb) + 64 * sub, rsc);
                            }
                            float gs = 0.0f, us = 0.0f;
#pragma unroll
                            for (int cp = 0; cp < GH::CP; ++cp) {
                                gs += q4k_lane_dot(grow + (size_t)(cp * 8 + bb) * Q4K_BYTES, sub, X[cp]);
                                us += q4k_lane_dot(urow + (size_t)(cp * 8 + bb) * Q4K_BYTES, sub, X[cp]);
                            }
#pragma unroll
                            for (int o = GH::LPR / 2; o; o >>= 1) {
                                gs += __shfl_xor_sync(0xffffffffu, gs, o);
                                us += __shfl_xor_sync(0xffffffffu, us, o);
                            }
                            if (lr == 0) abuf[j * MOE_ROWTILE + s * C::SR + rs] = gs / (1.0f + expf(-gs)) * us;
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive(gempty + slot);
                    }
                }
                named_sync(BAR_CONS, ST_CONS);
                if (!LL && lane == 0) mbar_arrive(xempty + xs_);
                for (int j = warp; j < ci.np; j += 8) {
                    const size_t p = (size_t)(ci.p0 + j);
                    if constexpr (LL) {
                        // flagged words: two int16 (positions 2i, 2i+1 of the
                        // xq_pos layout, one 8-value piece) per word, and the scale
                        float sc;
                        const int q = quant32(abuf[j * MOE_ROWTILE + lane], &sc, lane);
                        const int qn = __shfl_down_sync(0xffffffffu, q, 1);
                        const uint32_t tgl = tag_of(l);
                        if (!(lane & 1))
                            st_flagged(a.ll_a + par_of(l) * a.ll_a_n + p * (I / 2) +
                                           (xq_pos(rt * MOE_ROWTILE + lane) >> 1),
                                       ((uint32_t)q & 0xffffu) | ((uint32_t)qn << 16), tgl);
                        if (lane == 0)
                            st_flagged(a.ll_as + par_of(l) * a.ll_as_n + p * (I / 32) + rt, __float_as_uint(sc), tgl);
                    } else {
                        const int q = quant32(abuf[j * MOE_ROWTILE + lane], a.as + p * (I / 32) + rt, lane);
                        a.aq[p * I + xq_pos(rt * MOE_ROWTILE + lane)] = (int16_t)q;
                    }
                }
                named_sync(BAR_CONS, ST_CONS);
            }
        }
        if (stamp) stamp_at(l, 5);
        if (arena) fence_proxy_async_smem();  // the down copies reuse the gate/up stages' bytes
        if constexpr (!LL) grid_barrier(a, bar++, tid);
        if (stamp) stamp_at(l, 6);

        // ------------------------------------------------------------ phase C
        {
            float *out = out_of(a, l);
            const float *res = a.res_is_out ? out : in_of(a, l);
            const int slot_l = ep_slot(a.L, l);
            const int rho = lane / GI::LPR, lr = lane % GI::LPR, bb = lr >> 2, sub = lr & 3;
            const Q6Lane L6 = q6_lane(((rho * NBI + bb) & 1) ? 2 : 0, sub & 1);
            float *my_acc = acc + (size_t)warp * T * MOE_RT3;
            // Work units: a chunk's 16 rows (WS warp steps), or half of them
            // when the chunks are too few to keep the 8 warps busy.  A unit's
            // warp loads each token's activation slice once and runs the
            // unit's row dot products from it (independent chains).
            const int WG = (nch >= 8 || C::WS < 2) ? C::WS : C::WS / 2;
            const int UPC = C::WS / WG;
            const uint32_t tg = tag_of(l);
            if (LL && bx < NT) {
                // flagged mode: gather the whole intermediate (every pair's
                // int16 values and group scales) from the flagged words
                const int P = RT.scal[2];
                const unsigned long long *fa = a.ll_a + par_of(l) * a.ll_a_n;
                const unsigned long long *fs = a.ll_as + par_of(l) * a.ll_as_n;
                uint32_t *alq32 = reinterpret_cast<uint32_t *>(alq);
                const int na = P * (I / 2), ns = P * (I / 32);
                for (int i0 = tid; i0 < na + ns; i0 += 16 * ST_CONS) {
                    unsigned valid = 0;
#pragma unroll
                    for (int k = 0; k < 16; ++k)
                        if (i0 + k * ST_CONS < na + ns) valid |= 1u << k;
                    unsigned long long r[16];
                    flagged_poll(r, valid, [&](int k) {
                        const int i = i0 + k * ST_CONS;
                        return i < na ? fa + i : fs + (i - na);
                    }, tg, wait_bound(a));
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const int i = i0 + k * ST_CONS;
                        if (i < na)
                            alq32[i] = (uint32_t)r[k];
                        else if (i < na + ns)
                            als[i - na] = __uint_as_float((uint32_t)r[k]);
                    }
                }
                named_sync(BAR_CONS, ST_CONS);
            }
            for (int it3 = bx; it3 < NT; it3 += G) {
                // residual of this tile's columns, loaded before the stages
                // (flagged mode, l > 0: the previous layer's output words)
                float rv[MOE_TMAX * MOE_RT3 / ST_CONS];
                const unsigned long long *fres = (LL && l > 0) ? a.ll_h + par_of(l - 1) * a.ll_h_n : nullptr;
#pragma unroll
                for (int k = 0; k < MOE_TMAX * MOE_RT3 / ST_CONS; ++k) {
                    const int i = tid + k * ST_CONS;
                    const size_t o = (size_t)(i / MOE_RT3) * H + (size_t)it3 * MOE_RT3 + i % MOE_RT3;
                    if (ep || i >= T * MOE_RT3)
                        rv[k] = 0.0f;
                    else if (fres)
                        rv[k] = __uint_as_float(flagged_take(ld_flagged(fres + o), fres + o, tag_of(l - 1), wait_bound(a)));
                    else
                        rv[k] = __ldcg(res + o);
                }
                // Every chunk of the tile in its own ring slot: the tile's
                // nch x WS warp steps are split into 8 contiguous, equal ranges
                // (a range spans at most a few chunks; each chunk's activation
                // slice is loaded once per range).  The slots' previous uses all
                // finished before the tile's last consumer barrier, so no wait
                // looks two phases ahead.
                if (nch <= NS_D) {
                    const int S = nch * C::WS;
                    const int s1 = (warp + 1) * S / 8;
                    for (int s = warp * S / 8; s < s1;) {
                        const int c = s / C::WS;
                        const int wlo = s - c * C::WS;
                        const int whi = s1 - c * C::WS < C::WS ? s1 - c * C::WS : C::WS;
                        const int pos = dR.slot + c;
                        const int slot = pos % NS_D;
                        const unsigned par = (unsigned)(dR.phase ^ ((pos / NS_D) & 1));
                        const uint8_t *st = dring + (size_t)slot * m.dslot;
                        swait(dw + slot, par);
                        if constexpr (!LL) swait(da + slot, par);
                        if (stamp && s == 0 && it3 == bx) stamp_at(l, 7);
                        const ChunkInfo ci = cinfo(c);
                        const int16_t *aqs = LL ? alq + (size_t)ci.p0 * I : reinterpret_cast<const int16_t *>(st + C::WB);
                        const float *ass = LL ? als + (size_t)ci.p0 * (I / 32)
                                              : reinterpret_cast<const float *>(st + C::WB + (size_t)TC * I * 2);
                        for (int j = 0; j < ci.np; ++j) {
                            const int t = RT.ptok[ci.p0 + j];
                            const float wgt = RT.pw[ci.p0 + j];
                            XSlice X[GI::CP];
#pragma unroll
                            for (int cp = 0; cp < GI::CP; ++cp)
                                load_slice_q6k(X[cp], aqs + (size_t)j * I, ass + (size_t)j * (I / 32),
                                               QK * (cp * 8 + bb) + 128 * (sub >> 1), sub & 1);
                            // up to DB steps at a time: their dot chains and
                            // shuffle reductions interleave
                            constexpr int DB = C::WS < 4 ? C::WS : 4;
                            for (int wb = wlo; wb < whi; wb += DB) {
                                float v[DB];
#pragma unroll
                                for (int wi = 0; wi < DB; ++wi) {
                                    v[wi] = 0.0f;
                                    if (wb + wi < whi) {
                                        const uint8_t *rowp =
                                            st + (size_t)(wb + wi) * GI::STEPB + (size_t)rho * GI::ROWB;
#pragma unroll
                                        for (int cp = 0; cp < GI::CP; ++cp)
                                            v[wi] += q6k_lane_dot(rowp + (size_t)(cp * 8 + bb) * Q6K_BYTES, sub >> 1,
                                                                  sub & 1, L6, X[cp]);
                                    }
                                }
                                // transposed reduction: lane group q of the
                                // row's lanes holds step wb + q
                                static_assert(DB <= GI::LPR, "down values per lane exceed the row's lanes");
                                const float r = tr_reduce<DB, GI::LPR>(v);
                                const int q = lr / (GI::LPR / DB);
                                if ((lr & (GI::LPR / DB - 1)) == 0 && wb + q < whi)
                                    my_acc[t * MOE_RT3 + (wb + q) * GI::RPW + rho] += wgt * r;
                            }
                        }
                        __syncwarp();
                        if (lane == 0) mbar_arrive_cnt(dempty + slot, (unsigned)(whi - wlo));
                        s = c * C::WS + whi;
                    }
                }
                // Otherwise rounds of RSU units whose chunks sit in distinct ring
                // slots, with a consumer barrier between rounds: a slot's previous
                // use is then finished before any warp waits on it again, so the
                // parity wait below never looks two phases ahead.
                const int RSU = 8 < NS_D * UPC ? 8 : NS_D * UPC;
                for (int r0 = 0; nch > NS_D && r0 < nch * UPC; r0 += RSU) {
                    const int u = r0 + warp;
                    if (warp >= RSU || u >= nch * UPC) {
                        named_sync(BAR_CONS, ST_CONS);
                        continue;
                    }
                    const int c = u / UPC, ws0 = (u - c * UPC) * WG;
                    const int pos = dR.slot + c;  // ring position of chunk c from the tile's first stage
                    const int slot = pos % NS_D;
                    const unsigned par = (unsigned)(dR.phase ^ ((pos / NS_D) & 1));
                    const uint8_t *st = dring + (size_t)slot * m.dslot;
                    swait(dw + slot, par);
                    if constexpr (!LL) swait(da + slot, par);
                    if (stamp && r0 == 0 && it3 == bx) stamp_at(l, 7);
                    const ChunkInfo ci = cinfo(c);
                    const int16_t *aqs = LL ? alq + (size_t)ci.p0 * I : reinterpret_cast<const int16_t *>(st + C::WB);
                    const float *ass = LL ? als + (size_t)ci.p0 * (I / 32)
                                          : reinterpret_cast<const float *>(st + C::WB + (size_t)TC * I * 2);
                    for (int j = 0; j < ci.np; ++j) {
                        const int t = RT.ptok[ci.p0 + j];
                        const float wgt = RT.pw[ci.p0 + j];
                        XSlice X[GI::CP];
#pragma unroll
                        for (int cp = 0; cp < GI::CP; ++cp)
                            load_slice_q6k(X[cp], aqs + (size_t)j * I, ass + (size_t)j * (I / 32),
                                           QK * (cp * 8 + bb) + 128 * (sub >> 1), sub & 1);
#pragma unroll
                        for (int wi = 0; wi < C::WS; ++wi) {
                            if (wi >= WG) continue;
                            const int ws = ws0 + wi;
                            const uint8_t *rowp = st + (size_t)ws * GI::STEPB + (size_t)rho * GI::ROWB;
                            float v = 0.0f;
#pragma unroll
                            for (int cp = 0; cp < GI::CP; ++cp)
                                v += q6k_lane_dot(rowp + (size_t)(cp * 8 + bb) * Q6K_BYTES, sub >> 1, sub & 1, L6, X[cp]);
#pragma unroll
                            for (int o = GI::LPR / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
                            if (lr == 0) my_acc[t * MOE_RT3 + ws * GI::RPW + rho] += wgt * v;
                        }
                    }
                    __syncwarp();
                    if (lane == 0) mbar_arrive_cnt(dempty + slot, (unsigned)WG);
                    named_sync(BAR_CONS, ST_CONS);
                }
                for (int c = 0; c < nch; ++c) dR.next(NS_D);
                if (stamp) stamp_at(l, 22);
                named_sync(BAR_CONS, ST_CONS);
#pragma unroll
                for (int k = 0; k < MOE_TMAX * MOE_RT3 / ST_CONS; ++k) {
                    const int i = tid + k * ST_CONS;
                    if (i >= T * MOE_RT3) continue;
                    const int t = i / MOE_RT3, r = i % MOE_RT3;
                    float s = 0.0f;
#pragma unroll
                    for (int w = 0; w < 8; ++w) {  // warps in order: a fixed summation order
                        s += acc[(size_t)w * T * MOE_RT3 + i];
                        acc[(size_t)w * T * MOE_RT3 + i] = 0.0f;
                    }
                    const size_t oi = (size_t)t * H + (size_t)it3 * MOE_RT3 + r;
                    if (ep) {
                        // this rank's partial -> slot [slot_l][ep_rank] of every rank's mailbox (NVLink stores)
                        const size_t off = mb_slot_off(slot_l, a) + (size_t)a.ep_rank * TH + oi;
                        for (int p = 0; p < a.ep_world; ++p) a.ep_mb[p][off] = s;
                    } else if (LLEP) {
                        // this rank's partial -> word [slot_l][ep_rank] of every
                        // rank's mailbox (system-scope 64-bit stores over NVLink),
                        // then every rank's partial of the element from this
                        // rank's own mailbox, polled as one batch, added in rank
                        // order after the residual
                        for (int p = 0; p < a.ep_world; ++p)
                            st_flagged_sys(ep_ll_word(a, p, slot_l, a.ep_rank, oi), __float_as_uint(s), tg);
                        unsigned long long pw[EP_MAXW];
                        const unsigned valid = (1u << a.ep_world) - 1u;
                        auto pa = [&](int src) -> const unsigned long long * {
                            return ep_ll_word(a, a.ep_rank, slot_l, src, oi);
                        };
                        flagged_poll<EP_MAXW, decltype(pa), true>(pw, valid, pa, tg, a.ep_wait_ns);
                        float h = rv[k];
#pragma unroll
                        for (int src = 0; src < EP_MAXW; ++src)
                            if (src < a.ep_world) h += __uint_as_float((uint32_t)pw[src]);
                        if (l < a.L - 1)
                            st_flagged(a.ll_h + par_of(l) * a.ll_h_n + oi, __float_as_uint(h), tg);
                        else
                            out[oi] = h;
                    } else if (LL && l < a.L - 1) {
                        st_flagged(a.ll_h + par_of(l) * a.ll_h_n + oi, __float_as_uint(rv[k] + s), tg);
                    } else {
                        out[oi] = rv[k] + s;
                    }
                }
                if (stamp) stamp_at(l, 23);
                if (ep) {
                    // system-scope releases, one rank per thread (in parallel:
                    // each release waits for the CTA's stores in flight), after
                    // the CTA barrier that orders every thread's partial stores
                    // before them (a release is cumulative over what its
                    // thread has observed)
                    named_sync(BAR_CONS, ST_CONS);
                    if (tid < a.ep_world) red_release_sys(ep_counter(a, tid, slot_l), 1ull);
                }
                named_sync(BAR_CONS, ST_CONS);
            }
        }
        if (stamp) stamp_at(l, 8);
        if (arena) fence_proxy_async_smem();  // the next gate/up copies reuse the down stages' bytes
        if (!ep && !LL) grid_barrier(a, bar++, tid);
        if (stamp) stamp_at(l, 9);
    }

    // EP: the last layer's partials -> output columns owned by this CTA
    if (ep && !a.route_only) {
        const int s = ep_slot(a.L, a.L - 1);
        if (tid == 0) wait_counter(ep_counter(a, a.ep_rank, s), ep_target(a, a.L - 1, epoch, NT), true, a.ep_wait_ns);
        named_sync(BAR_CONS, ST_CONS);
        const float *src = in_of(a, a.L - 1);
        const float *pmb = a.ep_mb[a.ep_rank] + mb_slot_off(s, a);
        const size_t TH = (size_t)a.ep_tmax * H;
        for (int it3 = bx; it3 < NT; it3 += G)
            for (int i = tid; i < T * MOE_RT3; i += ST_CONS) {
                const size_t o = (size_t)(i / MOE_RT3) * H + (size_t)it3 * MOE_RT3 + i % MOE_RT3;
                float v = __ldcg(src + o);
                for (int r = 0; r < a.ep_world; ++r) v += __ldcg(pmb + (size_t)r * TH + o);
                a.y[o] = v;
            }
    }

    // exit ticket: the last CTA re-arms the barrier counter, advances the epoch
    // (counter-mode launches) and the layer sequence
    named_sync(BAR_CONS, ST_CONS);
    if (tid == 0) {
        __threadfence();
        const unsigned long long prev = atomicAdd(a.ctrl + CTRL_EXIT, 1ull);
        if (prev == (unsigned long long)G - 1) {
            a.ctrl[CTRL_GRID] = 0;
            a.ctrl[CTRL_EXIT] = 0;
            // the epoch counts the launches that add arrivals to the mailbox
            // counters (the targets derive from it); decode launches with
            // expert parallelism exchange tagged words and add none
            a.ctrl[CTRL_EPOCH] = ep ? epoch + 1 : epoch;
            a.ctrl[CTRL_SEQ] = seq0 + (unsigned long long)a.L;
            __threadfence();
        }
    }
}

// ---------------------------------------------------------------------------
// host side
// ---------------------------------------------------------------------------
template <int NBH, int NBI>
static int step_layout(StepSmem &m, int T, int K, int E, int EL, int G, int mode, int ndesc)
{
    using C = SCfg<NBH, NBI>;
    size_t o = 0;
    auto take = [&](size_t n, size_t al) {
        o = (o + al - 1) / al * al;
        const size_t at = o;
        o += n;
        return (uint32_t)at;
    };
    const int need = (E + 1 + G - 1) / G;
    int rr = 1;
    while (rr < need) rr <<= 1;
    if (rr > 8) return -1;
    m.RR = rr;
    m.WPR = 8 / rr;
    m.ldesc = take((size_t)ndesc * sizeof(StepLayer), 16);
    const bool arena = mode == MODE_BIG;  // tiled router (no rows in smem), rings share one arena
    const bool ll = mode == MODE_LL;
    m.rbuf = take(arena ? 16 : (size_t)rr * C::H * 4, 128);
    m.nwb = take(arena ? 16 : (size_t)C::H * 4, 128);
    m.part = take((size_t)8 * T * 4, 16);
    const int GM = (EL < T * K ? EL : T * K) + 1, PM = T * (K + 1);
    m.r_idx = take((size_t)T * K * 4, 16);
    m.r_w = take((size_t)T * K * 4, 16);
    m.r_rinv = take((size_t)T * 4, 16);
    m.r_sgw = take((size_t)T * 4, 16);
    m.r_cnt = take((size_t)(EL > 0 ? EL : 1) * 4, 16);
    m.r_run = take((size_t)(EL > 0 ? EL : 1) * 4, 16);
    m.r_off = take((size_t)(EL > 0 ? EL : 1) * 4, 16);
    m.r_gexp = take((size_t)GM * 4, 16);
    m.r_goff = take((size_t)GM * 4, 16);
    m.r_gcnt = take((size_t)GM * 4, 16);
    m.r_gcpre = take((size_t)(GM + 1) * 4, 16);
    m.r_ptok = take((size_t)PM * 4, 16);
    m.r_pw = take((size_t)PM * 4, 16);
    m.r_scal = take(16, 16);
    m.r_ptr = take((size_t)(EL > 0 ? EL : 1) * 3 * sizeof(void *), 16);
    m.r_chunk = take((size_t)(GM + (PM + MOE_TC - 1) / MOE_TC) * sizeof(int4), 16);
    const int TC = T < MOE_TC ? T : MOE_TC;
    if (ll) {
        // no activation slots: every token quantised locally (xloc), the layer
        // input (phase A) and the gathered intermediate (phase C) in one area
        m.xslot = 0;
        m.xsl = take(16, 128);
        m.xloc = take((size_t)T * C::XTOK, 128);
        const size_t xfb = (size_t)T * C::H * 4, alb = (size_t)T * (K + 1) * C::ATOK;
        m.xf = take(xfb > alb ? xfb : alb, 128);
        m.ssql = take((size_t)T * (C::H / 32) * 4, 16);
    } else {
        m.xslot = (uint32_t)al16((size_t)TC * C::XTOK);
        m.xsl = take(2 * (size_t)m.xslot, 128);
        m.xloc = m.xf = m.ssql = 0;
    }
    m.abuf = take((size_t)TC * MOE_ROWTILE * 4, 16);
    m.acc = take((size_t)8 * T * MOE_RT3 * 4, 16);
    m.dslot = (uint32_t)al16((size_t)C::WB + (ll ? 0 : (size_t)TC * C::ATOK));
    const size_t bars_max = (size_t)(1 + 2 * 16 + 4 + 3 * 16) * 8 + 8;
    int nsg, nsd;
    if (!arena) {
        // few tokens: separate rings, so the down weights can be in flight
        // during the gate/up phase
        // (flagged mode: fewer gate/up stages when the down ring would
        // otherwise be shallow)
        int nsg0 = 4;
        while (nsg0 > 2 && (size_t)nsg0 * C::STB > 80 * 1024) --nsg0;
        const size_t g0 = (o + 127) / 128 * 128;
        for (nsg = nsg0;; --nsg) {
            const size_t d0 = (g0 + (size_t)nsg * C::STB + 127) / 128 * 128;
            const size_t avail = SMEM_LIMIT > d0 + bars_max ? SMEM_LIMIT - d0 - bars_max : 0;
            nsd = (int)(avail / m.dslot);
            if (nsd > 16) nsd = 16;
            if (!ll || nsd >= 6 || nsg == 2) break;
        }
        m.gring = take((size_t)nsg * C::STB, 128);
        m.dring = take((size_t)(nsd > 0 ? nsd : 0) * m.dslot, 128);
    } else {
        // many tokens: both rings in one arena (the down phase starts after
        // every gate/up stage of the CTA is consumed), as deep as it allows
        const size_t a0 = (o + 127) / 128 * 128;
        const size_t avail = SMEM_LIMIT > a0 + bars_max ? SMEM_LIMIT - a0 - bars_max : 0;
        nsg = (int)(avail / C::STB);
        nsd = (int)(avail / m.dslot);
        if (nsg > 16) nsg = 16;
        if (nsd > 16) nsd = 16;
        m.gring = m.dring = (uint32_t)a0;
        const size_t gb = (size_t)(nsg > 0 ? nsg : 0) * C::STB, db = (size_t)(nsd > 0 ? nsd : 0) * m.dslot;
        o = a0 + (gb > db ? gb : db);
    }
    if (nsg < 2 || nsd < 2) return -1;
    m.NS_G = nsg;
    m.NS_D = nsd;
    m.bars = take((size_t)(1 + 2 * nsg + 4 + 3 * nsd) * 8, 8);
    m.total = (uint32_t)o;
    return o <= SMEM_LIMIT ? 0 : -1;
}

constexpr int MAX_DEVICES = 64;

template <int NBH, int NBI>
static int setup_nb()
{
    static std::mutex mu;
    static bool done[MAX_DEVICES] = {};
    int dev = 0;
    BREAD_CUDA(cudaGetDevice(&dev), "moe step: cudaGetDevice");
    if (dev < 0 || dev >= MAX_DEVICES) return set_error(BREAD_ERR_STATE, "moe step: device %d", dev);
    std::lock_guard<std::mutex> lock(mu);
    if (!done[dev]) {
        for (int mode = 0; mode < 6; ++mode) {
            auto kern = mode == MODE_LL      ? moe_step_kernel<NBH, NBI, MODE_LL>
                        : mode == MODE_SMALL ? moe_step_kernel<NBH, NBI, MODE_SMALL>
                        : mode == MODE_BIG   ? moe_step_kernel<NBH, NBI, MODE_BIG>
                        : mode == MODE_LLEP  ? moe_step_kernel<NBH, NBI, MODE_LLEP>
                        : mode == 4          ? moe_step_kernel<NBH, NBI, MODE_LL, true>
                                             : moe_step_kernel<NBH, NBI, MODE_LLEP, true>;
            BREAD_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_LIMIT),
                       "moe step: shared-memory attribute");
            int n = 0;
            BREAD_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, ST_THREADS, SMEM_LIMIT),
                       "moe step: occupancy");
            if (n < 1) return set_error(BREAD_ERR_CUDA, "moe step: kernel does not fit on an SM");
        }
        done[dev] = true;
    }
    return BREAD_OK;
}

template <int NBH, int NBI>
static int launch_nb(StepArgs &a, cudaStream_t s)
{
    BREAD_TRY(setup_nb<NBH, NBI>());
    const int G = sm_count();
    // decode on one GPU: flagged-word exchange when its buffers are there and
    // its layout fits (BREAD_NO_FLAGGED=1 forces the grid-barrier path)
    static const bool no_flagged = [] {
        const char *e = getenv("BREAD_NO_FLAGGED");
        return e && e[0] == '1';
    }();
    int mode = a.T > ROUTER_TILE_T ? MODE_BIG : MODE_SMALL;
    const int ndesc = a.layers ? a.L : 0;
    // expert-parallel decode needs the inter-layer words and its mailbox words
    const bool ll_ep_ok = a.ep_world == 1 || (a.ll_h && a.T <= StepMailbox::make(a.ep_world, a.ep_tmax, a.H).llT);
    if (mode == MODE_SMALL && !no_flagged && a.ll_pres && ll_ep_ok && !a.route_only && a.T <= LL_TMAX &&
        a.E <= 256 && G <= LL_GMAX && (a.L == 1 || a.ll_h) &&
        step_layout<NBH, NBI>(a.sm, a.T, a.top_k, a.E, a.hi - a.lo, G, MODE_LL, ndesc) == 0)
        mode = a.ep_world > 1 ? MODE_LLEP : MODE_LL;
    else if (step_layout<NBH, NBI>(a.sm, a.T, a.top_k, a.E, a.hi - a.lo, G, mode, ndesc))
        return set_error(BREAD_ERR_ARG, "moe step: T=%d H=%d I=%d does not fit in shared memory", a.T, a.H, a.I);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(G);
    cfg.blockDim = dim3(ST_THREADS);
    cfg.dynamicSmemBytes = a.sm.total;
    cfg.stream = s;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeCooperative;
    at[0].val.cooperative = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    if (mode == MODE_BIG)
        BREAD_CUDA(cudaLaunchKernelEx(&cfg, moe_step_kernel<NBH, NBI, MODE_BIG>, a), "moe step launch");
    else if (mode == MODE_SMALL)
        BREAD_CUDA(cudaLaunchKernelEx(&cfg, moe_step_kernel<NBH, NBI, MODE_SMALL>, a), "moe step launch");
    else if (mode == MODE_LLEP && a.T == 1)
        BREAD_CUDA(cudaLaunchKernelEx(&cfg, moe_step_kernel<NBH, NBI, MODE_LLEP, true>, a), "moe step launch");
    else if (mode == MODE_LLEP)
        BREAD_CUDA(cudaLaunchKernelEx(&cfg, moe_step_kernel<NBH, NBI, MODE_LLEP>, a), "moe step launch");
    else if (a.T == 1)
        BREAD_CUDA(cudaLaunchKernelEx(&cfg, moe_step_kernel<NBH, NBI, MODE_LL, true>, a), "moe step launch");
    else
        BREAD_CUDA(cudaLaunchKernelEx(&cfg, moe_step_kernel<NBH, NBI, MODE_LL>, a), "moe step launch");
    return BREAD_OK;
}

template <int NBH>
int step_launch_h(StepArgs &a, cudaStream_t s, int nbi)
{
    switch (nbi) {
    case 1: return launch_nb<NBH, 1>(a, s);
    case 2: return launch_nb<NBH, 2>(a, s);
    case 4: return launch_nb<NBH, 4>(a, s);
    case 8: return launch_nb<NBH, 8>(a, s);
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported I=%d", a.I);
    }
}

template <int NBH>
int step_setup_h(int nbi)
{
    switch (nbi) {
    case 1: return setup_nb<NBH, 1>();
    case 2: return setup_nb<NBH, 2>();
    case 4: return setup_nb<NBH, 4>();
    case 8: return setup_nb<NBH, 8>();
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported I=%d", nbi * QK);
    }
}

}  // namespace bread
