// stack.cu -- the expert-stack executor: the MoE part of the decode loop
// (reference main.cu:683-687 -> one_layer_forward -> one_layer.cu:1820-1985)
// for n_layers layers with every expert resident in HBM (no loader.c LRU, no
// host->device expert streaming).
//
// One decode step for T tokens, per layer l:
//   K1 route (RMS-normalises h on the fly) -> K2 gate/up -> K3 down + combine
//   and, with world > 1 (expert parallel), K3 stores its partial rows into
//   every rank's mailbox over NVLink and signals with system-scope atomics;
//   a combine kernel on each rank then waits (bounded) for all ranks and adds
//   the partials in rank order, so every rank holds the same bits.
// The whole step is captured once per (T, h) into a CUDA graph and replayed.
//
// Expert parallelism: rank r holds routed experts [r*E/world, (r+1)*E/world)
// of every layer plus the shared expert of layers l with l % world == r; the
// router (2 MB per layer) is replicated, so all ranks route identically and no
// dispatch exchange is needed.
#include <string.h>

#include <map>
#include <utility>
#include <vector>

#include "common.cuh"
#include "moe.cuh"
#include "ptx.cuh"

namespace bread {

// stream ids of the synthetic tensors: (layer, kind, expert)
static uint64_t sid(int layer, int kind, int e) { return ((uint64_t)layer << 32) | ((uint64_t)kind << 24) | (uint64_t)e; }
enum { K_GATE = 0, K_UP = 1, K_DOWN = 2, K_SH_GATE = 3, K_SH_UP = 4, K_SH_DOWN = 5, K_ROUTER = 6, K_SGVEC = 7 };

constexpr int EP_MAXW = 8;

struct LayerW {
    uint8_t *gate, *up, *down;           // local experts, contiguous [n_local x ...]
    uint8_t *sh_gate, *sh_up, *sh_down;  // NULL when another rank owns the shared expert
    float *W_r;
    __half *w_sg;
    const uint8_t **tab;                 // device: gate[E], up[E], down[E] pointer tables
};

}  // namespace bread

struct bread_stack {
    bread_stack_config_t cfg;
    int dev = 0;
    int lo = 0, hi = 0, n_local = 0;
    size_t bytes = 0;
    std::vector<void *> allocs;
    std::vector<bread::LayerW> layers;
    void *ws = nullptr;
    bread::MoeWs wsl;
    float *h_dev = nullptr;  // staging buffer of bread_stack_step_host
    // expert parallel
    uint8_t *mailbox = nullptr;
    bread::MoeMailbox mbl;
    bool peers_set = false;
    cudaStream_t cap = nullptr;  // private stream graphs are captured on
    float *peer_mb[bread::EP_MAXW] = {};
    std::map<std::pair<int, float *>, cudaGraphExec_t> graphs;
    int *stats_dev = nullptr;  // [n_layers][2]: groups, pairs of the last step
    // instrumented replay: events around every kernel of every layer
    std::vector<cudaEvent_t> ev;
    std::map<std::pair<int, float *>, cudaGraphExec_t> prof_graphs;
};

using namespace bread;

static int stack_alloc(bread_stack *st, void **p, size_t bytes, const char *what)
{
    cudaError_t e = cudaMalloc(p, bytes);
    if (e != cudaSuccess) return cuda_status(e, what);
    st->allocs.push_back(*p);
    st->bytes += bytes;
    return BREAD_OK;
}

extern "C" int bread_stack_destroy(bread_stack_t *st)
{
    if (!st) return BREAD_OK;
    for (auto &kv : st->graphs) cudaGraphExecDestroy(kv.second);
    for (auto &kv : st->prof_graphs) cudaGraphExecDestroy(kv.second);
    for (cudaEvent_t e : st->ev) cudaEventDestroy(e);
    if (st->cap) cudaStreamDestroy(st->cap);
    for (void *p : st->allocs) cudaFree(p);
    delete st;
    return BREAD_OK;
}

extern "C" int bread_stack_create(bread_stack_t **out, const bread_stack_config_t *cfg)
{
    if (!out || !cfg) return set_error(BREAD_ERR_ARG, "stack_create: NULL argument");
    *out = nullptr;
    const bread_stack_config_t c = *cfg;
    if (c.n_layers < 1) return set_error(BREAD_ERR_ARG, "stack_create: n_layers=%d", c.n_layers);
    BREAD_TRY(moe_check_shapes(c.max_tokens, c.hidden, c.inter, c.n_experts, c.top_k, true));
    if (c.world < 1 || c.world > EP_MAXW || c.rank < 0 || c.rank >= c.world || c.n_experts % c.world)
        return set_error(BREAD_ERR_ARG, "stack_create: rank=%d world=%d E=%d (E must divide by world <= %d)", c.rank,
                         c.world, c.n_experts, EP_MAXW);
    bread_stack *st = new bread_stack();
    st->cfg = c;
    cudaGetDevice(&st->dev);
    const int E = c.n_experts, H = c.hidden, I = c.inter;
    st->n_local = E / c.world;
    st->lo = c.rank * st->n_local;
    st->hi = st->lo + st->n_local;
    const size_t gate_b = (size_t)I * (H / QK) * Q4K_BYTES;  // one expert's gate (= up)
    const size_t down_b = (size_t)H * (I / QK) * Q6K_BYTES;
    int rc = BREAD_OK;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        delete st;
        return set_error(BREAD_ERR_CUDA, "stack_create: stream");
    }
    st->layers.resize(c.n_layers);
    for (int l = 0; l < c.n_layers && rc == BREAD_OK; ++l) {
        LayerW &L = st->layers[l];
        L = LayerW{};
        void *p;
        if ((rc = stack_alloc(st, &p, gate_b * st->n_local, "stack: gate"))) break;
        L.gate = (uint8_t *)p;
        if ((rc = stack_alloc(st, &p, gate_b * st->n_local, "stack: up"))) break;
        L.up = (uint8_t *)p;
        if ((rc = stack_alloc(st, &p, down_b * st->n_local, "stack: down"))) break;
        L.down = (uint8_t *)p;
        for (int j = 0; j < st->n_local && rc == BREAD_OK; ++j) {
            const int e = st->lo + j;
            rc = bread_synth_blocks(L.gate + j * gate_b, (long long)(gate_b / Q4K_BYTES), BREAD_QTYPE_Q4_K, c.seed, sid(l, K_GATE, e), s);
            if (!rc) rc = bread_synth_blocks(L.up + j * gate_b, (long long)(gate_b / Q4K_BYTES), BREAD_QTYPE_Q4_K, c.seed, sid(l, K_UP, e), s);
            if (!rc) rc = bread_synth_blocks(L.down + j * down_b, (long long)(down_b / Q6K_BYTES), BREAD_QTYPE_Q6_K, c.seed, sid(l, K_DOWN, e), s);
        }
        if (rc) break;
        if (c.shared_expert && l % c.world == c.rank) {
            if ((rc = stack_alloc(st, &p, 2 * gate_b + down_b, "stack: shared expert"))) break;
            L.sh_gate = (uint8_t *)p;
            L.sh_up = L.sh_gate + gate_b;
            L.sh_down = L.sh_up + gate_b;
            rc = bread_synth_blocks(L.sh_gate, (long long)(gate_b / Q4K_BYTES), BREAD_QTYPE_Q4_K, c.seed, sid(l, K_SH_GATE, 0), s);
            if (!rc) rc = bread_synth_blocks(L.sh_up, (long long)(gate_b / Q4K_BYTES), BREAD_QTYPE_Q4_K, c.seed, sid(l, K_SH_UP, 0), s);
            if (!rc) rc = bread_synth_blocks(L.sh_down, (long long)(down_b / Q6K_BYTES), BREAD_QTYPE_Q6_K, c.seed, sid(l, K_SH_DOWN, 0), s);
            if (rc) break;
        }
        if ((rc = stack_alloc(st, &p, (size_t)E * H * 4 + (size_t)H * 2 + 256, "stack: router"))) break;
        L.W_r = (float *)p;
        L.w_sg = reinterpret_cast<__half *>((uint8_t *)p + (size_t)E * H * 4);
        rc = bread_synth_normal_f32(L.W_r, (long long)E * H, 0.02f, c.seed, sid(l, K_ROUTER, 0), s);
        if (!rc && c.shared_expert) rc = bread_synth_normal_f16(L.w_sg, H, 0.02f, c.seed, sid(l, K_SGVEC, 0), s);
        if (!c.shared_expert) L.w_sg = nullptr;
        if (rc) break;
        // pointer tables gate[E], up[E], down[E]; experts of other ranks are NULL
        std::vector<const uint8_t *> tab(3 * (size_t)E, nullptr);
        for (int j = 0; j < st->n_local; ++j) {
            tab[st->lo + j] = L.gate + j * gate_b;
            tab[E + st->lo + j] = L.up + j * gate_b;
            tab[2 * E + st->lo + j] = L.down + j * down_b;
        }
        if ((rc = stack_alloc(st, &p, tab.size() * sizeof(void *), "stack: tables"))) break;
        L.tab = (const uint8_t **)p;
        if (cudaMemcpyAsync(p, tab.data(), tab.size() * sizeof(void *), cudaMemcpyHostToDevice, s) != cudaSuccess ||
            cudaStreamSynchronize(s) != cudaSuccess)
            rc = set_error(BREAD_ERR_CUDA, "stack: upload tables");
    }
    if (!rc) {
        st->wsl = MoeWs::make(c.max_tokens, H, I, E, c.top_k);
        rc = stack_alloc(st, &st->ws, st->wsl.total, "stack: workspace");
        if (!rc && cudaMemsetAsync(st->ws, 0, st->wsl.total, s) != cudaSuccess) rc = set_error(BREAD_ERR_CUDA, "stack: clear workspace");
        void *p = nullptr;
        if (!rc) rc = stack_alloc(st, &p, (size_t)c.max_tokens * H * 4, "stack: h staging");
        st->h_dev = (float *)p;
        if (!rc) rc = stack_alloc(st, &p, (size_t)c.n_layers * 2 * sizeof(int), "stack: stats");
        st->stats_dev = (int *)p;
    }
    if (!rc && cudaStreamCreateWithFlags(&st->cap, cudaStreamNonBlocking) != cudaSuccess)
        rc = set_error(BREAD_ERR_CUDA, "stack: capture stream");
    if (!rc) rc = moe_setup_kernels(H, I);
    if (!rc && c.world > 1) {
        st->mbl = MoeMailbox::make(c.world, c.max_tokens, H);
        void *p = nullptr;
        rc = stack_alloc(st, &p, st->mbl.total, "stack: mailbox");
        st->mailbox = (uint8_t *)p;
        if (!rc && cudaMemsetAsync(p, 0, st->mbl.total, s) != cudaSuccess) rc = set_error(BREAD_ERR_CUDA, "stack: clear mailbox");
    }
    if (!rc && cudaStreamSynchronize(s) != cudaSuccess) rc = set_error(BREAD_ERR_CUDA, "stack: synth");
    cudaStreamDestroy(s);
    if (rc) {
        bread_stack_destroy(st);
        return rc;
    }
    *out = st;
    return BREAD_OK;
}

extern "C" size_t bread_stack_device_bytes(const bread_stack_t *st) { return st ? st->bytes : 0; }

extern "C" int bread_stack_layer(const bread_stack_t *st, int layer, const void **gate_base, const void **up_base,
                                 const void **down_base, const float **W_r, const void **w_sg, const void **sh_gate,
                                 const void **sh_up, const void **sh_down, int *expert_lo, int *expert_hi)
{
    if (!st || layer < 0 || layer >= st->cfg.n_layers) return set_error(BREAD_ERR_ARG, "stack_layer: bad layer");
    const LayerW &L = st->layers[layer];
    if (gate_base) *gate_base = L.gate;
    if (up_base) *up_base = L.up;
    if (down_base) *down_base = L.down;
    if (W_r) *W_r = L.W_r;
    if (w_sg) *w_sg = L.w_sg;
    if (sh_gate) *sh_gate = L.sh_gate;
    if (sh_up) *sh_up = L.sh_up;
    if (sh_down) *sh_down = L.sh_down;
    if (expert_lo) *expert_lo = st->lo;
    if (expert_hi) *expert_hi = st->hi;
    return BREAD_OK;
}

extern "C" int bread_stack_mailbox(bread_stack_t *st, void **ptr, size_t *bytes)
{
    if (!st) return set_error(BREAD_ERR_ARG, "stack_mailbox: NULL stack");
    if (ptr) *ptr = st->mailbox;
    if (bytes) *bytes = st->mailbox ? st->mbl.total : 0;
    return BREAD_OK;
}

extern "C" int bread_stack_set_peers(bread_stack_t *st, void *const *peer_mailboxes, int world)
{
    if (!st || !peer_mailboxes || world != st->cfg.world || world < 2)
        return set_error(BREAD_ERR_ARG, "stack_set_peers: need world=%d peer pointers", st ? st->cfg.world : 0);
    for (int r = 0; r < world; ++r) {
        if (!peer_mailboxes[r]) return set_error(BREAD_ERR_ARG, "stack_set_peers: NULL mailbox of rank %d", r);
        st->peer_mb[r] = static_cast<float *>(peer_mailboxes[r]);
    }
    st->peers_set = true;
    for (auto &kv : st->graphs) cudaGraphExecDestroy(kv.second);
    st->graphs.clear();
    for (auto &kv : st->prof_graphs) cudaGraphExecDestroy(kv.second);
    st->prof_graphs.clear();
    return BREAD_OK;
}

extern "C" int bread_ipc_get_handle(const void *dev_ptr, void *handle_out)
{
    if (!dev_ptr || !handle_out) return set_error(BREAD_ERR_ARG, "ipc_get_handle: NULL argument");
    cudaIpcMemHandle_t h;
    BREAD_CUDA(cudaIpcGetMemHandle(&h, const_cast<void *>(dev_ptr)), "cudaIpcGetMemHandle");
    memcpy(handle_out, &h, sizeof h);
    return BREAD_OK;
}

extern "C" int bread_ipc_open_handle(const void *handle, void **dev_ptr)
{
    if (!handle || !dev_ptr) return set_error(BREAD_ERR_ARG, "ipc_open_handle: NULL argument");
    cudaIpcMemHandle_t h;
    memcpy(&h, handle, sizeof h);
    BREAD_CUDA(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess), "cudaIpcOpenMemHandle");
    return BREAD_OK;
}

extern "C" int bread_ipc_close_handle(void *dev_ptr)
{
    if (!dev_ptr) return set_error(BREAD_ERR_ARG, "ipc_close_handle: NULL argument");
    BREAD_CUDA(cudaIpcCloseMemHandle(dev_ptr), "cudaIpcCloseMemHandle");
    return BREAD_OK;
}

extern "C" int bread_stack_launches_per_step(const bread_stack_t *st, int T)
{
    (void)T;
    if (!st) return 0;
    return st->cfg.n_layers * (st->cfg.world > 1 ? 4 : 3);
}

// Mailbox slot of layer l: consecutive layers (also the last and the first
// of the next step) always use different slots, which is what makes a slot
// safe to overwrite (see ep_combine_kernel).
static int mailbox_slot(int l, int L) { return (L & 1) && l == L - 1 ? 2 : (l & 1); }

// ev: NULL, or 5 events per layer recorded before K1, K2, K3, the combine,
// and at the end of the layer.
static int stack_enqueue(bread_stack_t *st, float *h, int T, cudaStream_t s, const cudaEvent_t *ev = nullptr)
{
    const bread_stack_config_t &c = st->cfg;
    for (int l = 0; l < c.n_layers; ++l) {
        const LayerW &L = st->layers[l];
        MoeArgs a{};
        a.gate = L.tab;
        a.up = L.tab + c.n_experts;
        a.down = L.tab + 2 * c.n_experts;
        a.W_r = L.W_r;
        a.w_sg = L.w_sg;
        a.sh_gate = L.sh_gate;
        a.sh_up = L.sh_up;
        a.sh_down = L.sh_down;
        a.T = T;
        a.H = c.hidden;
        a.I = c.inter;
        a.E = c.n_experts;
        a.top_k = c.top_k;
        a.lo = st->lo;
        a.hi = st->hi;
        a.shared_here = L.sh_gate != nullptr;
        a.norm_eps = c.norm_eps;
        a.x = h;
        a.out = h;
        a.stats = st->stats_dev + 2 * l;
        if (c.world > 1) {
            a.ep_world = c.world;
            a.ep_rank = c.rank;
            a.ep_slot = mailbox_slot(l, c.n_layers);
            a.ep_tmax = c.max_tokens;
            for (int r = 0; r < c.world; ++r) a.ep_mb[r] = st->peer_mb[r];
        }
        moe_bind_workspace(a, st->ws, st->wsl);
        if (ev) BREAD_CUDA(cudaEventRecordWithFlags(ev[5 * l + 0], s, cudaEventRecordExternal), "stack: event");
        BREAD_TRY(moe_launch_route(a, s));
        if (ev) BREAD_CUDA(cudaEventRecordWithFlags(ev[5 * l + 1], s, cudaEventRecordExternal), "stack: event");
        BREAD_TRY(moe_launch_gateup(a, s));
        if (ev) BREAD_CUDA(cudaEventRecordWithFlags(ev[5 * l + 2], s, cudaEventRecordExternal), "stack: event");
        BREAD_TRY(moe_launch_down(a, s));
        if (ev) BREAD_CUDA(cudaEventRecordWithFlags(ev[5 * l + 3], s, cudaEventRecordExternal), "stack: event");
        if (c.world > 1) BREAD_TRY(moe_launch_combine(a, h, s));
        if (ev) BREAD_CUDA(cudaEventRecordWithFlags(ev[5 * l + 4], s, cudaEventRecordExternal), "stack: event");
    }
    return BREAD_OK;
}

// Captures one step into a graph on the stack's private stream (capture is
// not allowed on the legacy default stream a caller may use).
static int capture(bread_stack_t *st, float *h, int T, const cudaEvent_t *ev, cudaGraphExec_t *out)
{
    cudaGraph_t g = nullptr;
    BREAD_CUDA(cudaStreamBeginCapture(st->cap, cudaStreamCaptureModeThreadLocal), "stack: begin capture");
    const int rc = stack_enqueue(st, h, T, st->cap, ev);
    const cudaError_t ce = cudaStreamEndCapture(st->cap, &g);
    if (rc != BREAD_OK) {
        if (g) cudaGraphDestroy(g);
        return rc;
    }
    if (ce != cudaSuccess) return cuda_status(ce, "stack: end capture");
    const cudaError_t ie = cudaGraphInstantiate(out, g, 0);
    cudaGraphDestroy(g);
    if (ie != cudaSuccess) return cuda_status(ie, "stack: instantiate graph");
    return BREAD_OK;
}

static int ready(const bread_stack_t *st, const float *h, int T)
{
    if (!st || !h) return set_error(BREAD_ERR_ARG, "stack: NULL argument");
    if (T < 1 || T > st->cfg.max_tokens) return set_error(BREAD_ERR_ARG, "stack: T=%d outside 1..%d", T, st->cfg.max_tokens);
    if (st->cfg.world > 1 && !st->peers_set)
        return set_error(BREAD_ERR_STATE, "stack: expert-parallel stack needs bread_stack_set_peers first");
    return BREAD_OK;
}

extern "C" int bread_stack_step(bread_stack_t *st, float *h, int T, cudaStream_t stream)
{
    BREAD_TRY(ready(st, h, T));
    const auto key = std::make_pair(T, h);
    auto it = st->graphs.find(key);
    if (it == st->graphs.end()) {
        cudaGraphExec_t ge = nullptr;
        BREAD_TRY(capture(st, h, T, nullptr, &ge));
        it = st->graphs.emplace(key, ge).first;
    }
    BREAD_CUDA(cudaGraphLaunch(it->second, stream), "stack: graph launch");
    return BREAD_OK;
}

extern "C" int bread_stack_profile_step(bread_stack_t *st, float *h, int T, cudaStream_t stream, float *kernel_ms)
{
    BREAD_TRY(ready(st, h, T));
    if (!kernel_ms) return set_error(BREAD_ERR_ARG, "stack_profile_step: NULL kernel_ms");
    const int L = st->cfg.n_layers;
    if (st->ev.empty()) {
        st->ev.resize((size_t)5 * L);
        for (auto &e : st->ev) BREAD_CUDA(cudaEventCreate(&e), "stack: create event");
    }
    const auto key = std::make_pair(T, h);
    auto it = st->prof_graphs.find(key);
    if (it == st->prof_graphs.end()) {
        cudaGraphExec_t ge = nullptr;
        BREAD_TRY(capture(st, h, T, st->ev.data(), &ge));
        it = st->prof_graphs.emplace(key, ge).first;
    }
    BREAD_CUDA(cudaGraphLaunch(it->second, stream), "stack: graph launch");
    BREAD_CUDA(cudaStreamSynchronize(stream), "stack: profile sync");
    for (int l = 0; l < L; ++l)
        for (int k = 0; k < 4; ++k)
            BREAD_CUDA(cudaEventElapsedTime(kernel_ms + 4 * l + k, st->ev[5 * l + k], st->ev[5 * l + k + 1]),
                       "stack: elapsed time");
    return BREAD_OK;
}

extern "C" int bread_stack_routing_stats(const bread_stack_t *st, int *groups, int *pairs)
{
    if (!st || !groups || !pairs) return set_error(BREAD_ERR_ARG, "stack_routing_stats: NULL argument");
    std::vector<int> v((size_t)2 * st->cfg.n_layers);
    BREAD_CUDA(cudaMemcpy(v.data(), st->stats_dev, v.size() * sizeof(int), cudaMemcpyDeviceToHost), "stack: stats");
    for (int l = 0; l < st->cfg.n_layers; ++l) {
        groups[l] = v[2 * l];
        pairs[l] = v[2 * l + 1];
    }
    return BREAD_OK;
}

extern "C" int bread_stack_step_host(bread_stack_t *st, const float *h_in, float *h_out, int T, cudaStream_t stream)
{
    if (!st || !h_in || !h_out) return set_error(BREAD_ERR_ARG, "stack_step_host: NULL argument");
    if (T < 1 || T > st->cfg.max_tokens) return set_error(BREAD_ERR_ARG, "stack_step_host: T=%d", T);
    const size_t bytes = (size_t)T * st->cfg.hidden * 4;
    BREAD_CUDA(cudaMemcpyAsync(st->h_dev, h_in, bytes, cudaMemcpyHostToDevice, stream), "stack: h to device");
    BREAD_TRY(bread_stack_step(st, st->h_dev, T, stream));
    BREAD_CUDA(cudaMemcpyAsync(h_out, st->h_dev, bytes, cudaMemcpyDeviceToHost, stream), "stack: h to host");
    return BREAD_OK;
}
