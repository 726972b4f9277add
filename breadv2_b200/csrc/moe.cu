// moe.cu -- the MoE block entry points (bread_moe_route, bread_moe_ffn) and
// the shape dispatch of the persistent step kernel, whose device code lives in
// moe_kernel.cuh and is instantiated per hidden size in moe_h*.cu.
//
// Reference path replaced: route_layer (one_layer.cu:937-992) and the MoE
// block of one_layer_forward (one_layer.cu:1840-1983).
#include "common.cuh"
#include "moe.cuh"

namespace bread {

// Defined in moe_h<NBH>.cu for NBH = H / 256.
template <int NBH>
int step_launch_h(StepArgs &a, cudaStream_t s, int nbi);
template <int NBH>
int step_setup_h(int nbi);

int step_launch(StepArgs &a, cudaStream_t s)
{
    const int nbi = a.route_only ? 1 : a.I / QK;
    switch (a.H / QK) {
    case 1: return step_launch_h<1>(a, s, nbi);
    case 2: return step_launch_h<2>(a, s, nbi);
    case 4: return step_launch_h<4>(a, s, nbi);
    case 8: return step_launch_h<8>(a, s, nbi);
    case 16: return step_launch_h<16>(a, s, nbi);
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported H=%d", a.H);
    }
}

int step_setup(int H, int I)
{
    const int nbi = I > 0 ? I / QK : 1;
    switch (H / QK) {
    case 1: return step_setup_h<1>(nbi);
    case 2: return step_setup_h<2>(nbi);
    case 4: return step_setup_h<4>(nbi);
    case 8: return step_setup_h<8>(nbi);
    case 16: return step_setup_h<16>(nbi);
    default: return set_error(BREAD_ERR_ARG, "moe: unsupported H=%d", H);
    }
}

void step_bind_workspace(StepArgs &a, void *ws, const StepWs &L)
{
    uint8_t *b = static_cast<uint8_t *>(ws);
    a.ctrl = reinterpret_cast<unsigned long long *>(b + L.ctrl);
    a.logits = reinterpret_cast<float *>(b + L.logits);
    a.score = reinterpret_cast<float *>(b + L.score);
    a.ssq = reinterpret_cast<float *>(b + L.ssq);
    a.xq = reinterpret_cast<int16_t *>(b + L.xq);
    a.xs = reinterpret_cast<float *>(b + L.xs);
    a.aq = reinterpret_cast<int16_t *>(b + L.aq);
    a.as = reinterpret_cast<float *>(b + L.as);
    a.ridx = reinterpret_cast<int *>(b + L.ridx);
    a.rw = reinterpret_cast<float *>(b + L.rw);
    a.rinv = reinterpret_cast<float *>(b + L.rinv);
    a.rsgw = reinterpret_cast<float *>(b + L.rsgw);
    a.buf[0] = L.buf0 ? reinterpret_cast<float *>(b + L.buf0) : nullptr;
    a.buf[1] = L.buf1 ? reinterpret_cast<float *>(b + L.buf1) : nullptr;
    auto ll = [&](size_t off) { return L.ll_end ? reinterpret_cast<unsigned long long *>(b + off) : nullptr; };
    a.ll_pres = ll(L.ll_pres);
    a.ll_lg = ll(L.ll_lg);
    a.ll_a = ll(L.ll_a);
    a.ll_as = ll(L.ll_as);
    a.ll_h = L.ll_h ? ll(L.ll_h) : nullptr;
    a.ll_pres_n = LL_GMAX;
    a.ll_lg_n = (size_t)L.ll_T * (a.E + 1);
    a.ll_a_n = (size_t)L.ll_T * (a.top_k + 1) * (a.I / 2);
    a.ll_as_n = (size_t)L.ll_T * (a.top_k + 1) * (a.I / 32);
    a.ll_h_n = (size_t)L.ll_T * a.H;
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

}  // namespace bread

using namespace bread;

extern "C" size_t bread_moe_workspace_bytes(int T, int H, int I, int E, int top_k)
{
    if (T < 1 || H < 32 || E < 1 || top_k < 1) return 0;
    return StepWs::make(T, H, I, E, top_k, false).total;
}

// One MoE block (L = 1): shared argument checks of the route / FFN entries.
static int moe_prepare(StepArgs &a, const float *x, const float *W_r, const void *w_sg, int T, int H, int I, int E,
                       int top_k, void *workspace, size_t workspace_bytes, bool need_experts)
{
    BREAD_TRY(moe_check_shapes(T, H, I, E, top_k, need_experts));
    if (!x || !W_r) return set_error(BREAD_ERR_ARG, "moe: NULL x or W_r");
    const StepWs L = StepWs::make(T, H, need_experts ? I : 0, E, top_k, false);
    if (!workspace || workspace_bytes < L.total)
        return set_error(BREAD_ERR_WORKSPACE, "moe: workspace %zu bytes, need %zu", workspace_bytes, L.total);
    if (reinterpret_cast<uintptr_t>(workspace) & 255)
        return set_error(BREAD_ERR_ALIGN, "moe: workspace not 256-byte aligned");
    if ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(W_r) | reinterpret_cast<uintptr_t>(w_sg)) & 15)
        return set_error(BREAD_ERR_ALIGN, "moe: x, W_r and w_sg must be 16-byte aligned");
    a = StepArgs{};
    a.l0.W_r = W_r;
    a.l0.w_sg = static_cast<const __half *>(w_sg);
    a.L = 1;
    a.T = T;
    a.H = H;
    a.I = I;
    a.E = E;
    a.top_k = top_k;
    a.lo = 0;
    a.hi = E;
    a.norm_eps = -1.0f;
    a.x = x;
    a.ep_world = 1;
    a.ep_tmax = T;
    a.ep_wait_ns = EP_WAIT_NS;
    step_bind_workspace(a, workspace, L);
    a.ll_reset = L.ll_end;
    return BREAD_OK;
}

extern "C" int bread_moe_route(const float *x, const float *W_r, const void *w_sg, int T, int H, int E, int top_k,
                               int *idx, float *w, float *sg_weight, void *workspace, size_t workspace_bytes,
                               cudaStream_t stream)
{
    StepArgs a;
    BREAD_TRY(moe_prepare(a, x, W_r, w_sg, T, H, 0, E, top_k, workspace, workspace_bytes, false));
    if (!idx || !w) return set_error(BREAD_ERR_ARG, "moe_route: NULL idx or w");
    a.route_only = 1;
    a.idx_out = idx;
    a.w_out = w;
    a.sg_out = sg_weight;
    BREAD_CUDA(cudaMemsetAsync(a.ctrl, 0, CTRL_BYTES, stream), "moe_route: reset control words");
    return step_launch(a, stream);
}

extern "C" int bread_moe_ffn(const void *const *gate_ptrs, const void *const *up_ptrs, const void *const *down_ptrs,
                             const float *W_r, const void *w_sg, const void *sh_gate, const void *sh_up,
                             const void *sh_down, const float *x, float *out, int T, int H, int I, int E, int top_k,
                             int *idx_out, float *w_out, float *sg_out, void *workspace, size_t workspace_bytes,
                             cudaStream_t stream)
{
    StepArgs a;
    BREAD_TRY(moe_prepare(a, x, W_r, w_sg, T, H, I, E, top_k, workspace, workspace_bytes, true));
    if (!gate_ptrs || !up_ptrs || !down_ptrs || !out)
        return set_error(BREAD_ERR_ARG, "moe_ffn: NULL pointer table or out");
    const int nsh = (sh_gate != nullptr) + (sh_up != nullptr) + (sh_down != nullptr);
    if (nsh != 0 && nsh != 3) return set_error(BREAD_ERR_ARG, "moe_ffn: give all three shared-expert matrices or none");
    if (nsh == 3 && ((reinterpret_cast<uintptr_t>(sh_gate) | reinterpret_cast<uintptr_t>(sh_up) |
                      reinterpret_cast<uintptr_t>(sh_down)) & 15))
        return set_error(BREAD_ERR_ALIGN, "moe_ffn: shared-expert matrices must be 16-byte aligned");
    a.l0.gate = reinterpret_cast<const uint8_t *const *>(gate_ptrs);
    a.l0.up = reinterpret_cast<const uint8_t *const *>(up_ptrs);
    a.l0.down = reinterpret_cast<const uint8_t *const *>(down_ptrs);
    a.l0.sh_gate = static_cast<const uint8_t *>(sh_gate);
    a.l0.sh_up = static_cast<const uint8_t *>(sh_up);
    a.l0.sh_down = static_cast<const uint8_t *>(sh_down);
    a.res_is_out = 1;
    a.y = out;
    a.idx_out = idx_out;
    a.w_out = w_out;
    a.sg_out = sg_out;
    // control words (and the flagged-exchange words, whose tags restart at 1)
    BREAD_CUDA(cudaMemsetAsync(a.ctrl, 0, a.ll_reset > CTRL_BYTES ? a.ll_reset : CTRL_BYTES, stream),
               "moe_ffn: reset control words");
    return step_launch(a, stream);
}
