// moe.cuh -- shared definitions of the persistent MoE step kernel (moe_kernel.cuh)
// and its callers (the MoE block entry points in moe.cu, the stack executor
// in stack.cu, the no-alloc entry point in noalloc.cu).
#pragma once
#include "common.cuh"

namespace bread {

constexpr int MOE_TMAX = 64;     // tokens per call
constexpr int MOE_EMAX = 512;    // routed experts
constexpr int MOE_KMAX = 16;     // top-k
constexpr int MOE_HMAX = 4096;   // hidden size
constexpr int MOE_IMAX = 2048;   // expert intermediate size
constexpr int MOE_TC = 8;        // (token, expert) pairs per chunk
constexpr int MOE_ROWTILE = 32;  // gate/up rows per work item (one activation group)
constexpr int MOE_RT3 = 16;      // down rows (= output columns of h) per tile
constexpr int EP_MAXW = 8;       // expert-parallel ranks
constexpr unsigned long long EP_WAIT_NS = 20000000000ull;  // default bound of a wait on another rank: 20 s

__host__ __device__ constexpr size_t al16(size_t v) { return (v + 15) / 16 * 16; }

// Lane geometry of the quantised lane dots (qdot.cuh): 4 lanes per
// super-block, so one row of NB blocks takes 4*NB lanes; wider rows take
// several column passes (CP), narrower ones share a warp (RPW rows per step).
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

// Weights of one MoE layer as the step kernel reads them.  Routed experts
// come either from per-expert pointer tables (the reference's
// weight_cache_t gate_ptrs[e] etc., loader.h:79-84) or, when *_base is set,
// from contiguous arrays holding experts [lo, hi) at a fixed stride (no
// pointer loads on the critical path).
struct StepLayer {
    const uint8_t *const *gate;  // device tables [E] of per-expert matrices;
    const uint8_t *const *up;    // NULL entries: expert not held here
    const uint8_t *const *down;
    const uint8_t *gate_base, *up_base, *down_base;  // or contiguous experts [lo, hi)
    size_t gu_stride, d_stride;                      // bytes between consecutive experts
    const uint8_t *sh_gate, *sh_up, *sh_down;        // shared expert, or NULL
    const float *W_r;                                // [E x H] fp32 router
    const __half *w_sg;                              // [H] fp16 shared-gate vector, or NULL
    const float *norm_w;                             // [H] fp32 weight of the layer's pre-MoE RMSNorm
                                                     // (post_attention_norm.weight), or NULL for 1
};
static_assert(sizeof(StepLayer) % 8 == 0, "layer descriptors are copied to shared memory in 8-byte words");

// Control words at the head of the workspace (u64 each): the grid-barrier
// counter, the exit ticket, the launch epoch and the layer sequence (tags of
// the flagged exchange words, below).  Zero before the first launch; the last
// CTA of every launch resets the first two, advances the epoch by one if the
// launch counted expert-parallel arrivals in the mailbox counters, and the
// layer sequence by the launch's layers.
enum { CTRL_GRID = 0, CTRL_EXIT = 1, CTRL_EPOCH = 2, CTRL_SEQ = 3 };

// Flagged exchange (decode launches of a few tokens on one GPU): the values
// CTAs hand to one another inside a launch -- router logits, the quantised
// gate/up intermediate, the residual stream between layers -- travel as 8-byte
// words {payload (low 32 bits), tag (high 32 bits)}, stored and loaded as
// single 64-bit accesses at gpu scope.  The tag of layer l of a launch is
// layer sequence + l + 1, so a reader that polls a word until its tag matches
// has waited for exactly that value: no grid barrier, and the wait and the
// read are one load.  Buffers alternate by layer parity; every CTA also posts
// one presence word per layer, awaited by all, which keeps any CTA from
// running two layers ahead of another (the double buffering is then enough).
constexpr int LL_TMAX = 8;    // tokens per launch of the flagged-exchange decode mode
constexpr int LL_GMAX = 256;  // CTAs of such a launch (presence words)

// Phase points recorded per layer and CTA by a profiled launch
// (StepArgs::stamps, %globaltimer ns).  Consumer thread 0: 0 layer start,
// 1 logits written, 2 after the router barrier, 3 routing tables built, 4 first
// activation slot landed, 5 gate/up done, 6 after the gate/up barrier, 7 first
// down stage landed, 8 down done, 9 layer end.  Producer: 10 routing tables
// seen, 11 gate/up copies issued, 12 down weight copies issued, 13 next
// layer's router rows issued, 14 gate/up barrier seen, 15 all down copies
// issued.  Consumer thread 0 again: 16 quantisation share done (flagged
// mode: layer input read), 17 router rows landed, 18 router dots done, 19
// routing inputs read, 20 top-k done, 21 tables built (= 3 before the chunk
// table), 22 down stages done, 23 down columns stored.
constexpr int STAMPS = 24;
constexpr size_t CTRL_BYTES = 256;

// Global scratch of one step launch (byte offsets, each 256-byte aligned).
// The flagged-exchange words (LL_TMAX tokens at most) follow the control
// words.  A stack workspace (inter_layer_buffers) holds them beside the other
// pieces, two parities; a one-block workspace holds one parity in the same
// bytes as the barrier-mode pieces (a launch uses one mode) and the caller
// zeroes [0, ll_end) before every launch.
struct StepWs {
    size_t ctrl, logits, score, ssq, xq, xs, aq, as, ridx, rw, rinv, rsgw, buf0, buf1, total;
    size_t ll_pres, ll_lg, ll_a, ll_as, ll_h, ll_end;  // ll_end == 0: no flagged-exchange words
    int PM, ll_T, ll_par;
    __host__ static StepWs make(int T, int H, int I, int E, int K, bool inter_layer_buffers)
    {
        StepWs w;
        size_t o = 0;
        auto take = [&](size_t bytes) {
            const size_t at = o;
            o += (bytes + 255) / 256 * 256;
            return at;
        };
        w.PM = T * (K + 1);
        w.ctrl = take(CTRL_BYTES);
        w.ll_T = T < LL_TMAX ? T : LL_TMAX;
        w.ll_par = inter_layer_buffers ? 2 : 1;
        w.ll_pres = w.ll_lg = w.ll_a = w.ll_as = w.ll_h = w.ll_end = 0;
        if (I > 0 && (inter_layer_buffers || T <= LL_TMAX)) {
            const size_t pm = (size_t)w.ll_T * (K + 1), par = (size_t)w.ll_par;
            w.ll_pres = take(par * LL_GMAX * 8);
            w.ll_lg = take(par * w.ll_T * (E + 1) * 8);
            w.ll_a = take(par * pm * (I / 2) * 8);
            w.ll_as = take(par * pm * (I / 32) * 8);
            w.ll_h = inter_layer_buffers ? take(par * w.ll_T * H * 8) : 0;
            w.ll_end = o;
            if (!inter_layer_buffers) o = w.ctrl + CTRL_BYTES;  // the barrier-mode pieces share these bytes
        }
        w.logits = take((size_t)T * E * 4);
        w.score = take((size_t)T * 4);
        w.ssq = take((size_t)T * (H / 32) * 4);
        w.xq = take((size_t)T * H * 2);
        w.xs = take((size_t)T * (H / 32) * 4);
        w.aq = take((size_t)w.PM * (I > 0 ? I : 32) * 2);
        w.as = take((size_t)w.PM * (I > 0 ? I / 32 : 1) * 4);
        w.ridx = take((size_t)T * K * 4);
        w.rw = take((size_t)T * K * 4);
        w.rinv = take((size_t)T * 4);
        w.rsgw = take((size_t)T * 4);
        w.buf0 = inter_layer_buffers ? take((size_t)T * H * 4) : 0;
        w.buf1 = inter_layer_buffers ? take((size_t)T * H * 4) : 0;
        w.total = o > w.ll_end ? o : w.ll_end;
        return w;
    }
};

// Shared-memory layout of one launch (byte offsets), computed on the host.
struct StepSmem {
    uint32_t rbuf, part, xsl, gring, abuf, dring, acc, bars, total;
    uint32_t xloc, xf, ssql;  // flagged-exchange mode: quantised tokens, layer input / intermediate, group sums
    uint32_t ldesc;           // copies of the L layer descriptors (StepArgs::layers)
    uint32_t nwb;             // the layer's RMSNorm weight [H] (copied with the router rows)
    uint32_t r_idx, r_w, r_rinv, r_sgw, r_cnt, r_run, r_off, r_gexp, r_goff, r_gcnt, r_gcpre, r_ptok, r_pw, r_scal, r_ptr, r_chunk;
    uint32_t xslot, dslot;
    int NS_G, NS_D, RR, WPR;
};

// Expert-parallel mailbox of one rank: [3 slots][world][Tmax x H] fp32
// partials written by every rank over NVLink, then one u64 arrival counter
// per slot (monotonic; targets derive from the launch epoch) -- the
// grid-barrier instantiations' exchange -- and, for decode launches of at
// most LL_TMAX tokens, [3 slots][world][llT x H] flagged words {partial,
// layer tag} that every rank stores into every rank's mailbox and polls in
// its own (llT = min(Tmax, LL_TMAX)).
constexpr int MB_SLOTS = 3;
struct StepMailbox {
    size_t ctr_off, ll_off, total;
    int llT;
    __host__ __device__ static StepMailbox make(int world, int Tmax, int H)
    {
        StepMailbox m;
        const size_t data = (size_t)MB_SLOTS * world * Tmax * H * 4;
        m.ctr_off = (data + 255) / 256 * 256;
        m.ll_off = m.ctr_off + 256;
        m.llT = Tmax < LL_TMAX ? Tmax : LL_TMAX;
        m.total = m.ll_off + (size_t)MB_SLOTS * world * m.llT * H * 8;
        return m;
    }
    __host__ __device__ static size_t data_off(int slot, int src, int world, int Tmax, int H)
    {
        return ((size_t)slot * world + src) * Tmax * H * 4;
    }
};

// Everything the step kernel reads (passed by value).
struct StepArgs {
    StepLayer l0;               // layer 0 when `layers` is NULL
    const StepLayer *layers;    // device array [L], or NULL (L == 1)
    int L, T, H, I, E, top_k;
    int lo, hi;                 // routed experts computed here: [lo, hi)
    float norm_eps;             // >= 0: each layer's input is RMS-normalised first
    int route_only;             // 1: routing outputs only (no expert work)
    int res_is_out;             // 1: y += moe(x) (one block);  0: h <- h + moe(norm(h)) per layer
    const float *x;             // input of layer 0 [T x H]
    float *y;                   // output of the last layer [T x H]
    float *buf[2];              // inter-layer buffers [T x H] (L > 1)
    // workspace
    unsigned long long *ctrl;
    float *logits, *score, *ssq;
    int16_t *xq;
    float *xs;
    int16_t *aq;
    float *as;
    int *ridx;                  // routing of the grid (large T): [T x k] experts and weights,
    float *rw, *rinv, *rsgw;    // [T] RMS factors and shared-gate weights
    // flagged-exchange words [parity][...] (NULL: the workspace has none)
    unsigned long long *ll_pres, *ll_lg, *ll_a, *ll_as, *ll_h;
    size_t ll_pres_n, ll_lg_n, ll_a_n, ll_as_n, ll_h_n;  // words per parity
    size_t ll_reset;            // host only: bytes from ctrl zeroed before a one-block launch
    // optional outputs (written by CTA 0): the routing of the launch's layer
    // [T x K], or of every layer [L][T x K] when out_per_layer is set
    int *idx_out;
    float *w_out, *sg_out;
    int out_per_layer;
    int *stats;                 // [L][2]: expert groups, pairs computed here
    unsigned long long *stamps; // [L][grid][STAMPS] %globaltimer at phase points of every CTA, or NULL
    // expert parallel
    float *ep_mb[EP_MAXW];
    int ep_world, ep_rank, ep_tmax;
    unsigned long long ep_wait_ns;  // bound of every wait on another rank (then DEVERR_TIMEOUT)
    StepSmem sm;
};

int moe_check_shapes(int T, int H, int I, int E, int top_k, bool need_experts);
// Binds the workspace pieces of StepWs::make(...) at `ws` into `a`.
void step_bind_workspace(StepArgs &a, void *ws, const StepWs &L);
// Computes the shared-memory layout for the current device, sets the kernel
// attributes once per device and launches the cooperative step kernel.
int step_launch(StepArgs &a, cudaStream_t s);
// One-time per-device kernel set-up (call before any stream capture).
int step_setup(int H, int I);

}  // namespace bread
