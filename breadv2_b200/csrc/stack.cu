// stack.cu -- the expert-stack executor: the MoE part of the decode loop
// (reference main.cu:683-687 -> one_layer_forward -> one_layer.cu:1820-1985)
// for n_layers layers with every expert resident in HBM (no loader.c LRU, no
// host->device expert streaming).
//
// One decode step for T tokens is ONE launch of the persistent step kernel
// (moe.cu): per layer l, h <- h + moe_l(rmsnorm(h)) with grid-wide barriers
// between the router, gate/up and down phases.  With world > 1 (expert
// parallel) the down phase stores the rank's partial columns into every
// rank's mailbox over NVLink and counts arrivals there; the next layer's
// first phase waits (bounded) for all ranks and adds the partials in rank
// order, so every rank holds the same bits.
//
// Expert parallelism: rank r holds routed experts [r*E/world, (r+1)*E/world)
// of every layer plus the shared expert of layers l with l % world == r; the
// router (2 MB per layer) is replicated, so all ranks route identically and no
// dispatch exchange is needed.
#include <stdio.h>
#include <string.h>

#include <string>
#include <vector>

#include "common.cuh"
#include "moe.cuh"
#include "ptx.cuh"

namespace bread {

// stream ids of the synthetic tensors: (layer, kind, expert)
static uint64_t sid(int layer, int kind, int e) { return ((uint64_t)layer << 32) | ((uint64_t)kind << 24) | (uint64_t)e; }
enum { K_GATE = 0, K_UP = 1, K_DOWN = 2, K_SH_GATE = 3, K_SH_UP = 4, K_SH_DOWN = 5, K_ROUTER = 6, K_SGVEC = 7, K_NORM = 8 };

struct LayerW {
    uint8_t *gate, *up, *down;           // local experts, contiguous [n_local x ...]
    uint8_t *sh_gate, *sh_up, *sh_down;  // NULL when another rank owns the shared expert
    float *W_r;
    __half *w_sg;
    float *norm_w;                       // pre-MoE RMSNorm weight [H], or NULL (unit weight)
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
    bread::StepLayer *layer_desc = nullptr;  // device array [n_layers] the step kernel reads
    void *ws = nullptr;
    bread::StepWs wsl;
    float *h_dev = nullptr;  // staging buffer of bread_stack_step_host
    // expert parallel
    uint8_t *mailbox = nullptr;
    bread::StepMailbox mbl;
    bool peers_set = false;
    float *peer_mb[bread::EP_MAXW] = {};
    int *stats_dev = nullptr;                   // [n_layers][2]: groups, pairs of the last step
    int *rec_idx = nullptr;                     // [n_layers][max_tokens][top_k]: routing of the last step
    float *rec_w = nullptr;                     // [n_layers][max_tokens][top_k]
    float *rec_sg = nullptr;                    // [n_layers][max_tokens]
    int rec_T = 0;                              // tokens of the last step
    unsigned long long *stamps_dev = nullptr;   // [n_layers][ctas][STAMPS]: phase points of the last profiled step
    int ctas = 0;                               // grid of the step kernel (one CTA per SM)
    unsigned long long ep_wait_ns = bread::EP_WAIT_NS;  // bound of each wait on another rank
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
    for (void *p : st->allocs) cudaFree(p);
    delete st;
    return BREAD_OK;
}

namespace bread {

// Where a stack's weights come from: the seeded generator (bread_stack_create)
// or a GGUF model file (bread_stack_create_gguf).  Every call fills device
// memory on stream s.
struct WeightSource {
    virtual ~WeightSource() {}
    // experts [lo, lo + n) of matrix kind (K_GATE / K_UP / K_DOWN) of layer l
    virtual int experts(int l, int kind, int lo, int n, uint8_t *dst, size_t expert_bytes, cudaStream_t s) = 0;
    virtual bool has_shared(int l) = 0;
    virtual int shared(int l, int kind, uint8_t *dst, size_t bytes, cudaStream_t s) = 0;
    virtual int router(int l, float *dst, size_t n, cudaStream_t s) = 0;
    virtual bool has_shared_gate(int l) = 0;
    virtual int shared_gate(int l, __half *dst, int H, cudaStream_t s) = 0;
    virtual bool has_norm(int l) = 0;
    virtual int norm(int l, float *dst, int H, cudaStream_t s) = 0;
};

struct SynthSource : WeightSource {
    const bread_stack_config_t &c;
    explicit SynthSource(const bread_stack_config_t &cfg) : c(cfg) {}
    int experts(int l, int kind, int lo, int n, uint8_t *dst, size_t eb, cudaStream_t s) override
    {
        const int qt = kind == K_DOWN ? BREAD_QTYPE_Q6_K : BREAD_QTYPE_Q4_K;
        const size_t bb = kind == K_DOWN ? Q6K_BYTES : Q4K_BYTES;
        for (int j = 0; j < n; ++j)
            BREAD_TRY(bread_synth_blocks(dst + j * eb, (long long)(eb / bb), qt, c.seed, sid(l, kind, lo + j), s));
        return BREAD_OK;
    }
    bool has_shared(int) override { return c.shared_expert != 0; }
    int shared(int l, int kind, uint8_t *dst, size_t bytes, cudaStream_t s) override
    {
        const int qt = kind == K_SH_DOWN ? BREAD_QTYPE_Q6_K : BREAD_QTYPE_Q4_K;
        const size_t bb = kind == K_SH_DOWN ? Q6K_BYTES : Q4K_BYTES;
        return bread_synth_blocks(dst, (long long)(bytes / bb), qt, c.seed, sid(l, kind, 0), s);
    }
    int router(int l, float *dst, size_t n, cudaStream_t s) override
    {
        return bread_synth_normal_f32(dst, (long long)n, 0.02f, c.seed, sid(l, K_ROUTER, 0), s);
    }
    bool has_shared_gate(int) override { return c.shared_expert != 0; }
    int shared_gate(int l, __half *dst, int H, cudaStream_t s) override
    {
        return bread_synth_normal_f16(dst, H, 0.02f, c.seed, sid(l, K_SGVEC, 0), s);
    }
    bool has_norm(int) override { return c.norm_weight != 0; }
    int norm(int l, float *dst, int H, cudaStream_t s) override
    {
        // post_attention_norm.weight stand-in: 1 + 0.1 * N(0,1), seeded
        std::vector<float> w((size_t)H);
        bread_synth_normal_f32_host(w.data(), H, 0.1f, c.seed, sid(l, K_NORM, 0));
        for (float &v : w) v += 1.0f;
        BREAD_CUDA(cudaMemcpyAsync(dst, w.data(), (size_t)H * 4, cudaMemcpyHostToDevice, s), "stack: upload norm weight");
        BREAD_CUDA(cudaStreamSynchronize(s), "stack: upload norm weight");
        return BREAD_OK;
    }
};

// GGUF model file: byte ranges of the named tensors copied through a pinned
// staging buffer (loader.c:156-206 names and expert byte ranges: expert k of
// a *_exps tensor starts at k * size / n_experts).
struct GgufSource : WeightSource {
    bread_gguf_t *g = nullptr;
    void *stage = nullptr;
    static constexpr size_t STAGE = 32u << 20;
    ~GgufSource() override
    {
        if (stage) cudaFreeHost(stage);
        bread_gguf_close(g);
    }
    static std::string name(int l, const char *what)
    {
        char b[96];
        snprintf(b, sizeof b, "blk.%d.%s.weight", l, what);
        return b;
    }
    bool find(int l, const char *what, bread_gguf_tensor_t *t)
    {
        char saved[512];
        snprintf(saved, sizeof saved, "%s", bread_last_error());
        const bool ok = bread_gguf_find(g, name(l, what).c_str(), t) == BREAD_OK;
        set_error(BREAD_OK, "%s", saved);  // absence of an optional tensor is not an error
        return ok;
    }
    int need(int l, const char *what, uint32_t type, bread_gguf_tensor_t *t)
    {
        if (bread_gguf_find(g, name(l, what).c_str(), t) != BREAD_OK)
            return set_error(BREAD_ERR_ARG, "stack_create_gguf: no tensor %s", name(l, what).c_str());
        if (t->type != type)
            return set_error(BREAD_ERR_QTYPE, "stack_create_gguf: %s has ggml type %u, expected %u", name(l, what).c_str(),
                             t->type, type);
        return BREAD_OK;
    }
    // bytes [off, off + n) of the data section -> device dst
    int copy(uint64_t off, void *dst, size_t n, cudaStream_t s)
    {
        uint8_t *d = static_cast<uint8_t *>(dst);
        for (size_t done = 0; done < n;) {
            const size_t k = n - done < STAGE ? n - done : STAGE;
            BREAD_CUDA(cudaStreamSynchronize(s), "stack: gguf staging");
            BREAD_TRY(bread_gguf_read(g, off + done, stage, k));
            BREAD_CUDA(cudaMemcpyAsync(d + done, stage, k, cudaMemcpyHostToDevice, s), "stack: gguf upload");
            done += k;
        }
        BREAD_CUDA(cudaStreamSynchronize(s), "stack: gguf upload");
        return BREAD_OK;
    }
    int experts(int l, int kind, int lo, int n, uint8_t *dst, size_t eb, cudaStream_t s) override
    {
        const char *what = kind == K_GATE ? "ffn_gate_exps" : kind == K_UP ? "ffn_up_exps" : "ffn_down_exps";
        bread_gguf_tensor_t t;
        BREAD_TRY(need(l, what, kind == K_DOWN ? BREAD_QTYPE_Q6_K : BREAD_QTYPE_Q4_K, &t));
        const uint64_t ne = t.n_dims ? t.dims[t.n_dims - 1] : 0;
        if (!ne || t.size / ne != eb || (uint64_t)lo + n > ne)
            return set_error(BREAD_ERR_ARG, "stack_create_gguf: %s holds %llu experts of %llu bytes, need %zu-byte experts "
                             "[%d, %d)", name(l, what).c_str(), (unsigned long long)ne,
                             (unsigned long long)(ne ? t.size / ne : 0), eb, lo, lo + n);
        return copy(t.offset + (uint64_t)lo * eb, dst, (size_t)n * eb, s);
    }
    bool has_shared(int l) override
    {
        bread_gguf_tensor_t t;
        return find(l, "ffn_gate_shexp", &t);
    }
    int shared(int l, int kind, uint8_t *dst, size_t bytes, cudaStream_t s) override
    {
        const char *what = kind == K_SH_GATE ? "ffn_gate_shexp" : kind == K_SH_UP ? "ffn_up_shexp" : "ffn_down_shexp";
        bread_gguf_tensor_t t;
        BREAD_TRY(need(l, what, kind == K_SH_DOWN ? BREAD_QTYPE_Q6_K : BREAD_QTYPE_Q4_K, &t));
        if (t.size != bytes)
            return set_error(BREAD_ERR_ARG, "stack_create_gguf: %s is %llu bytes, expected %zu", name(l, what).c_str(),
                             (unsigned long long)t.size, bytes);
        return copy(t.offset, dst, bytes, s);
    }
    int router(int l, float *dst, size_t n, cudaStream_t s) override
    {
        bread_gguf_tensor_t t;
        BREAD_TRY(need(l, "ffn_gate_inp", 0, &t));  // F32 (one_layer.cu:246-251)
        if (t.size != n * 4) return set_error(BREAD_ERR_ARG, "stack_create_gguf: %s has the wrong size", name(l, "ffn_gate_inp").c_str());
        return copy(t.offset, dst, n * 4, s);
    }
    bool has_shared_gate(int l) override
    {
        bread_gguf_tensor_t t;
        return find(l, "ffn_gate_inp_shexp", &t);
    }
    int shared_gate(int l, __half *dst, int H, cudaStream_t s) override
    {
        bread_gguf_tensor_t t;
        BREAD_TRY(need(l, "ffn_gate_inp_shexp", 1, &t));  // F16 (one_layer.cu:258-263)
        if (t.size != (uint64_t)H * 2)
            return set_error(BREAD_ERR_ARG, "stack_create_gguf: %s has the wrong size", name(l, "ffn_gate_inp_shexp").c_str());
        return copy(t.offset, dst, (size_t)H * 2, s);
    }
    bool has_norm(int l) override
    {
        bread_gguf_tensor_t t;
        return find(l, "post_attention_norm", &t);
    }
    int norm(int l, float *dst, int H, cudaStream_t s) override
    {
        bread_gguf_tensor_t t;
        BREAD_TRY(need(l, "post_attention_norm", 0, &t));
        if (t.size != (uint64_t)H * 4)
            return set_error(BREAD_ERR_ARG, "stack_create_gguf: %s has the wrong size", name(l, "post_attention_norm").c_str());
        return copy(t.offset, dst, (size_t)H * 4, s);
    }
};

}  // namespace bread

// Allocates every buffer of a stack and fills the weights from `src`.
static int stack_build(bread_stack_t **out, const bread_stack_config_t &c, WeightSource &src)
{
    *out = nullptr;
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
        if ((rc = src.experts(l, K_GATE, st->lo, st->n_local, L.gate, gate_b, s))) break;
        if ((rc = src.experts(l, K_UP, st->lo, st->n_local, L.up, gate_b, s))) break;
        if ((rc = src.experts(l, K_DOWN, st->lo, st->n_local, L.down, down_b, s))) break;
        if (src.has_shared(l) && l % c.world == c.rank) {
            if ((rc = stack_alloc(st, &p, 2 * gate_b + down_b, "stack: shared expert"))) break;
            L.sh_gate = (uint8_t *)p;
            L.sh_up = L.sh_gate + gate_b;
            L.sh_down = L.sh_up + gate_b;
            if ((rc = src.shared(l, K_SH_GATE, L.sh_gate, gate_b, s))) break;
            if ((rc = src.shared(l, K_SH_UP, L.sh_up, gate_b, s))) break;
            if ((rc = src.shared(l, K_SH_DOWN, L.sh_down, down_b, s))) break;
        }
        if ((rc = stack_alloc(st, &p, (size_t)E * H * 4 + (size_t)H * 2 + 256, "stack: router"))) break;
        L.W_r = (float *)p;
        L.w_sg = reinterpret_cast<__half *>((uint8_t *)p + (size_t)E * H * 4);
        if ((rc = src.router(l, L.W_r, (size_t)E * H, s))) break;
        if (src.has_shared_gate(l)) {
            if ((rc = src.shared_gate(l, L.w_sg, H, s))) break;
        } else {
            L.w_sg = nullptr;
        }
        if (src.has_norm(l)) {
            if ((rc = stack_alloc(st, &p, (size_t)H * 4, "stack: norm weight"))) break;
            L.norm_w = (float *)p;
            if ((rc = src.norm(l, L.norm_w, H, s))) break;
        }
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
        st->wsl = StepWs::make(c.max_tokens, H, I, E, c.top_k, true);
        rc = stack_alloc(st, &st->ws, st->wsl.total, "stack: workspace");
        if (!rc && cudaMemsetAsync(st->ws, 0, st->wsl.total, s) != cudaSuccess) rc = set_error(BREAD_ERR_CUDA, "stack: clear workspace");
        void *p = nullptr;
        if (!rc) rc = stack_alloc(st, &p, (size_t)c.max_tokens * H * 4, "stack: h staging");
        st->h_dev = (float *)p;
        if (!rc) rc = stack_alloc(st, &p, (size_t)c.n_layers * 2 * sizeof(int), "stack: stats");
        st->stats_dev = (int *)p;
        const size_t nrec = (size_t)c.n_layers * c.max_tokens;
        if (!rc) rc = stack_alloc(st, &p, nrec * (2 * c.top_k + 1) * 4, "stack: routing record");
        st->rec_idx = (int *)p;
        st->rec_w = reinterpret_cast<float *>(st->rec_idx + nrec * c.top_k);
        st->rec_sg = st->rec_w + nrec * c.top_k;
        st->ctas = sm_count();
        if (!rc) rc = stack_alloc(st, &p, (size_t)c.n_layers * st->ctas * STAMPS * sizeof(unsigned long long), "stack: stamps");
        st->stamps_dev = (unsigned long long *)p;
    }
    if (!rc) {
        // per-layer descriptors the step kernel reads
        std::vector<StepLayer> d((size_t)c.n_layers);
        for (int l = 0; l < c.n_layers; ++l) {
            const LayerW &L = st->layers[l];
            d[l].gate = L.tab;
            d[l].up = L.tab + E;
            d[l].down = L.tab + 2 * E;
            d[l].gate_base = L.gate;  // local experts are contiguous: no pointer loads
            d[l].up_base = L.up;
            d[l].down_base = L.down;
            d[l].gu_stride = gate_b;
            d[l].d_stride = down_b;
            d[l].sh_gate = L.sh_gate;
            d[l].sh_up = L.sh_up;
            d[l].sh_down = L.sh_down;
            d[l].W_r = L.W_r;
            d[l].w_sg = L.w_sg;
            d[l].norm_w = L.norm_w;
        }
        void *p = nullptr;
        rc = stack_alloc(st, &p, d.size() * sizeof(StepLayer), "stack: layer descriptors");
        st->layer_desc = (StepLayer *)p;
        if (!rc && (cudaMemcpyAsync(p, d.data(), d.size() * sizeof(StepLayer), cudaMemcpyHostToDevice, s) != cudaSuccess ||
                    cudaStreamSynchronize(s) != cudaSuccess))
            rc = set_error(BREAD_ERR_CUDA, "stack: upload layer descriptors");
    }
    if (!rc) rc = step_setup(H, I);
    if (!rc && c.world > 1) {
        st->mbl = StepMailbox::make(c.world, c.max_tokens, H);
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

extern "C" int bread_stack_create(bread_stack_t **out, const bread_stack_config_t *cfg)
{
    if (!out || !cfg) return set_error(BREAD_ERR_ARG, "stack_create: NULL argument");
    SynthSource src(*cfg);
    return stack_build(out, *cfg, src);
}

extern "C" int bread_stack_create_gguf(bread_stack_t **out, const char *path, const bread_stack_config_t *cfg)
{
    if (!out || !path || !cfg) return set_error(BREAD_ERR_ARG, "stack_create_gguf: NULL argument");
    *out = nullptr;
    GgufSource src;
    BREAD_TRY(bread_gguf_open(path, &src.g));
    // shapes from layer 0's tensors: gate_exps [H, I, E] (dims[0] innermost), down_exps [I, H, E]
    bread_gguf_tensor_t tg, td;
    BREAD_TRY(src.need(0, "ffn_gate_exps", BREAD_QTYPE_Q4_K, &tg));
    BREAD_TRY(src.need(0, "ffn_down_exps", BREAD_QTYPE_Q6_K, &td));
    if (tg.n_dims != 3 || td.n_dims != 3 || td.dims[0] != tg.dims[1] || td.dims[1] != tg.dims[0] || td.dims[2] != tg.dims[2])
        return set_error(BREAD_ERR_ARG, "stack_create_gguf: expert tensors of layer 0 have unexpected shapes");
    bread_stack_config_t c = *cfg;
    const int H = (int)tg.dims[0], I = (int)tg.dims[1], E = (int)tg.dims[2];
    if ((c.hidden && c.hidden != H) || (c.inter && c.inter != I) || (c.n_experts && c.n_experts != E))
        return set_error(BREAD_ERR_ARG, "stack_create_gguf: file has H=%d I=%d E=%d, config asks %d/%d/%d", H, I, E,
                         c.hidden, c.inter, c.n_experts);
    c.hidden = H;
    c.inter = I;
    c.n_experts = E;
    c.shared_expert = src.has_shared(0) ? 1 : 0;
    c.norm_weight = src.has_norm(0) ? 1 : 0;
    if (cudaHostAlloc(&src.stage, GgufSource::STAGE, cudaHostAllocDefault) != cudaSuccess)
        return set_error(BREAD_ERR_CUDA, "stack_create_gguf: pinned staging buffer");
    return stack_build(out, c, src);
}

extern "C" size_t bread_stack_device_bytes(const bread_stack_t *st) { return st ? st->bytes : 0; }

extern "C" int bread_stack_get_config(const bread_stack_t *st, bread_stack_config_t *out)
{
    if (!st || !out) return set_error(BREAD_ERR_ARG, "stack_get_config: NULL argument");
    *out = st->cfg;
    return BREAD_OK;
}

extern "C" int bread_stack_norm_weight(const bread_stack_t *st, int layer, float *host_out, int *has_weight)
{
    if (!st || layer < 0 || layer >= st->cfg.n_layers || !host_out || !has_weight)
        return set_error(BREAD_ERR_ARG, "stack_norm_weight: bad argument");
    const float *w = st->layers[layer].norm_w;
    *has_weight = w ? 1 : 0;
    if (w)
        BREAD_CUDA(cudaMemcpy(host_out, w, (size_t)st->cfg.hidden * 4, cudaMemcpyDeviceToHost),
                   "stack: read norm weight");
    return BREAD_OK;
}

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
    return BREAD_OK;
}

extern "C" int bread_stack_set_peer_timeout(bread_stack_t *st, double seconds)
{
    if (!st || !(seconds > 0.0) || seconds > 3600.0)
        return set_error(BREAD_ERR_ARG, "stack_set_peer_timeout: seconds must be in (0, 3600]");
    st->ep_wait_ns = (unsigned long long)(seconds * 1e9);
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
    return st ? 1 : 0;  // one cooperative launch of the step kernel per decode step
}

static int ready(const bread_stack_t *st, const float *h, int T)
{
    if (!st || !h) return set_error(BREAD_ERR_ARG, "stack: NULL argument");
    if (T < 1 || T > st->cfg.max_tokens) return set_error(BREAD_ERR_ARG, "stack: T=%d outside 1..%d", T, st->cfg.max_tokens);
    if (st->cfg.world > 1 && !st->peers_set)
        return set_error(BREAD_ERR_STATE, "stack: expert-parallel stack needs bread_stack_set_peers first");
    if (reinterpret_cast<uintptr_t>(h) & 15) return set_error(BREAD_ERR_ALIGN, "stack: h must be 16-byte aligned");
    return BREAD_OK;
}

// One decode step: all layers in one launch of the step kernel.
static int stack_launch(bread_stack_t *st, float *h, int T, cudaStream_t s, unsigned long long *stamps)
{
    const bread_stack_config_t &c = st->cfg;
    StepArgs a{};
    a.layers = st->layer_desc;
    a.L = c.n_layers;
    a.T = T;
    a.H = c.hidden;
    a.I = c.inter;
    a.E = c.n_experts;
    a.top_k = c.top_k;
    a.lo = st->lo;
    a.hi = st->hi;
    a.norm_eps = c.norm_eps;
    a.res_is_out = 0;
    a.x = h;
    a.y = h;
    a.stats = st->stats_dev;
    a.stamps = stamps;
    // every layer's routing [L][T x K] (CTA 0 writes a few words per layer)
    a.idx_out = st->rec_idx;
    a.w_out = st->rec_w;
    a.sg_out = st->rec_sg;
    a.out_per_layer = 1;
    st->rec_T = T;
    a.ep_world = c.world;
    a.ep_wait_ns = st->ep_wait_ns;
    a.ep_rank = c.rank;
    a.ep_tmax = c.max_tokens;
    if (c.world > 1)
        for (int r = 0; r < c.world; ++r) a.ep_mb[r] = st->peer_mb[r];
    step_bind_workspace(a, st->ws, st->wsl);
    return step_launch(a, s);
}

extern "C" int bread_stack_step(bread_stack_t *st, float *h, int T, cudaStream_t stream)
{
    BREAD_TRY(ready(st, h, T));
    return stack_launch(st, h, T, stream, nullptr);
}

extern "C" int bread_stack_profile_step(bread_stack_t *st, float *h, int T, cudaStream_t stream, float *kernel_ms)
{
    BREAD_TRY(ready(st, h, T));
    if (!kernel_ms) return set_error(BREAD_ERR_ARG, "stack_profile_step: NULL kernel_ms");
    const int L = st->cfg.n_layers;
    const size_t n = (size_t)L * st->ctas * STAMPS;
    // points a CTA never reaches (no work of that kind) read 0
    BREAD_CUDA(cudaMemsetAsync(st->stamps_dev, 0, n * sizeof(unsigned long long), stream), "stack: clear stamps");
    BREAD_TRY(stack_launch(st, h, T, stream, st->stamps_dev));
    std::vector<unsigned long long> t(n);
    BREAD_CUDA(cudaMemcpyAsync(t.data(), st->stamps_dev, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost, stream),
               "stack: read phase stamps");
    BREAD_CUDA(cudaStreamSynchronize(stream), "stack: profile sync");
    // CTA 0's view of layer l: router phase [0,2), gate/up [2,6), down [6,9),
    // then the gap until the next layer starts (the expert-parallel wait)
    for (int l = 0; l < L; ++l) {
        const unsigned long long *p = t.data() + (size_t)l * st->ctas * STAMPS;
        kernel_ms[4 * l + 0] = (float)(p[2] - p[0]) * 1e-6f;
        kernel_ms[4 * l + 1] = (float)(p[6] - p[2]) * 1e-6f;
        kernel_ms[4 * l + 2] = (float)(p[9] - p[6]) * 1e-6f;
        kernel_ms[4 * l + 3] =
            l + 1 < L ? (float)(p[(size_t)st->ctas * STAMPS] - p[9]) * 1e-6f : 0.0f;
    }
    return BREAD_OK;
}

extern "C" int bread_stack_profile_stamps(const bread_stack_t *st, unsigned long long *out, size_t n_words, int *ctas)
{
    if (!st || !out) return set_error(BREAD_ERR_ARG, "stack_profile_stamps: NULL argument");
    const size_t n = (size_t)st->cfg.n_layers * st->ctas * STAMPS;
    if (n_words < n) return set_error(BREAD_ERR_ARG, "stack_profile_stamps: need %zu words", n);
    BREAD_CUDA(cudaMemcpy(out, st->stamps_dev, n * sizeof(unsigned long long), cudaMemcpyDeviceToHost),
               "stack: read phase stamps");
    if (ctas) *ctas = st->ctas;
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

extern "C" int bread_stack_routing(const bread_stack_t *st, int *idx, float *w, float *sg_weight, int *T_out)
{
    if (!st || !idx || !w || !sg_weight) return set_error(BREAD_ERR_ARG, "stack_routing: NULL argument");
    const int T = st->rec_T, K = st->cfg.top_k, L = st->cfg.n_layers;
    if (T_out) *T_out = T;
    if (!T) return set_error(BREAD_ERR_STATE, "stack_routing: no step has run");
    // the record is [L][T x K] packed for the last step's T
    BREAD_CUDA(cudaMemcpy(idx, st->rec_idx, (size_t)L * T * K * 4, cudaMemcpyDeviceToHost), "stack: routing idx");
    BREAD_CUDA(cudaMemcpy(w, st->rec_w, (size_t)L * T * K * 4, cudaMemcpyDeviceToHost), "stack: routing w");
    BREAD_CUDA(cudaMemcpy(sg_weight, st->rec_sg, (size_t)L * T * 4, cudaMemcpyDeviceToHost), "stack: routing sg");
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
