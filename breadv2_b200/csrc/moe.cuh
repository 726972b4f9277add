// moe.cuh -- shared definitions of the MoE FFN kernels (moe.cu) and the stack
// executor (stack.cu).
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
constexpr int MOE_RT3 = 16;      // down rows (= output rows) per work item
constexpr int K1_TG = 4;         // tokens per router CTA

// One chunk of up to MOE_TC pairs of one expert group, with everything the
// expert kernels need to start their bulk copies: resolved weight pointers,
// the pairs' first index (pairs of a group are contiguous), their tokens and
// routing weights.  Written by the router's finalize step; 16-byte aligned so
// that it can itself be bulk-copied into shared memory.
struct __align__(16) MoeChunk {
    const uint8_t *gate, *up, *down;
    int p0, np, group, pad;
    uint8_t tok[MOE_TC];
    float w[MOE_TC];
    uint8_t pad2[8];
};
static_assert(sizeof(MoeChunk) == 96, "MoeChunk layout");

// Byte offsets of the pieces of a MoE workspace (all 256-byte aligned).
struct MoeWs {
    size_t hdr, logits, ssq, score, ridx, rw, sgw, xq, xs, p_token, p_w, chunks, aq, as, total;
    int GM, PM, CM;
    static MoeWs make(int T, int H, int I, int E, int k)
    {
        MoeWs w;
        size_t o = 0;
        auto take = [&](size_t bytes) {
            const size_t at = o;
            o += (bytes + 255) / 256 * 256;
            return at;
        };
        w.GM = (E < T * k ? E : T * k) + 1;
        w.PM = T * (k + 1);
        w.CM = w.GM + (w.PM + MOE_TC - 1) / MOE_TC;
        w.hdr = take(64);
        w.logits = take((size_t)T * E * 4);
        w.ssq = take((size_t)T * (H / 32) * 4);
        w.score = take((size_t)T * 4);
        w.ridx = take((size_t)T * k * 4);
        w.rw = take((size_t)T * k * 4);
        w.sgw = take((size_t)T * 4);
        w.xq = take((size_t)T * H * 2);
        w.xs = take((size_t)T * (H / 32) * 4);
        w.p_token = take((size_t)w.PM * 4);
        w.p_w = take((size_t)w.PM * 4);
        w.chunks = take((size_t)w.CM * sizeof(MoeChunk));
        w.aq = take((size_t)w.PM * (I > 0 ? I : 1) * 2);
        w.as = take((size_t)w.PM * (I > 0 ? I / 32 : 1) * 4);
        w.total = o;
        return w;
    }
};

// Header words at MoeWs::hdr.
enum { HDR_TICKET = 0, HDR_NGROUPS = 1, HDR_NCHUNKS = 2, HDR_NPAIRS = 3 };

// Everything the MoE kernels read or write (passed by value).
struct MoeArgs {
    const uint8_t *const *gate;  // device tables [E] (routed experts)
    const uint8_t *const *up;
    const uint8_t *const *down;
    const float *W_r;            // [E x H] fp32
    const __half *w_sg;          // [H] fp16 or NULL
    const uint8_t *sh_gate, *sh_up, *sh_down;  // shared expert or NULL
    int T, H, I, E, top_k;
    int lo, hi;                  // experts computed here: [lo, hi)
    int shared_here;             // 1: the shared expert is computed here
    float norm_eps;              // >= 0: inputs are RMS-normalised first
    const float *x;              // router / expert input [T x H]
    float *out;                  // [T x H] accumulated into
    // workspace
    int *hdr;
    float *logits, *ssq, *score;
    int *ridx;
    float *rw, *sgw;
    int16_t *xq;
    float *xs;
    int *p_token;
    float *p_w;
    MoeChunk *chunks;
    int16_t *aq;
    float *as;
    // optional routing copies
    int *idx_out;
    float *w_out, *sg_out;
    int *stats;  // optional: [groups, pairs] computed here (written by the router)
    // expert parallel (ep_world > 1): the down kernel stores its partial rows
    // into every rank's mailbox instead of accumulating into `out`, then
    // counts one arrival per CTA at every rank (MoeMailbox layout)
    float *ep_mb[8];
    int ep_world, ep_rank, ep_slot, ep_tmax;
};

// Mailbox of one rank (expert parallel): [MB_SLOTS][world][Tmax x H] fp32
// partials, arrival counters [MB_SLOTS][8], combine tickets [MB_SLOTS].
constexpr int MB_SLOTS = 3;
struct MoeMailbox {
    size_t flag_off, ticket_off, total;
    __host__ __device__ static MoeMailbox make(int world, int Tmax, int H)
    {
        MoeMailbox m;
        const size_t data = (size_t)MB_SLOTS * world * Tmax * H * 4;
        m.flag_off = (data + 255) / 256 * 256;
        m.ticket_off = m.flag_off + 256;
        m.total = m.ticket_off + 256;
        return m;
    }
    __host__ __device__ static size_t data_off(int slot, int src, int world, int Tmax, int H)
    {
        return ((size_t)slot * world + src) * Tmax * H * 4;
    }
};

void moe_bind_workspace(MoeArgs &a, void *ws, const MoeWs &L);
int moe_check_shapes(int T, int H, int I, int E, int top_k, bool need_experts);
// Router + finalize, gate/up + SiLU*mul, down + combine, expert-parallel
// combine.  All are launched with programmatic dependent launch allowed.
int moe_launch_route(const MoeArgs &a, cudaStream_t s);
int moe_launch_gateup(const MoeArgs &a, cudaStream_t s);
int moe_launch_down(const MoeArgs &a, cudaStream_t s);
int moe_down_grid(const MoeArgs &a);
int moe_launch_combine(const MoeArgs &a, float *h, cudaStream_t s);
int moe_setup_kernels(int H, int I);

}  // namespace bread
