"""GPU: the expert-stack executor (graph-captured multi-layer decode step) and
the synthetic-data generator it uses."""
import numpy as np
import pytest
import torch

import breadv2_b200 as bb

pytestmark = pytest.mark.gpu
TOL = 1e-3


def sid(layer, kind, e):
    return (layer << 32) | (kind << 24) | e


@pytest.mark.parametrize("qt", [12, 14, 8])
def test_synth_device_equals_host(cuda, qt):
    d = bb.synth_blocks(3001, qt, 7, 3, device=cuda).cpu().numpy()
    assert np.array_equal(d, bb.synth_blocks_host(3001, qt, 7, 3))


def test_synth_normal_device_equals_host(cuda):
    a = bb.synth_normal(10007, 0.02, 5, 6, device=cuda).cpu().numpy()
    assert np.array_equal(a.view(np.uint32), bb.synth_normal_host(10007, 0.02, 5, 6).view(np.uint32))
    b = bb.synth_normal(10007, 0.02, 5, 6, half=True, device=cuda).cpu().numpy()
    assert np.array_equal(b.view(np.uint16), bb.synth_normal_host(10007, 0.02, 5, 6, half=True))


MARGIN = 1e-4  # top-k gaps below this are inside fp32 summation noise


def norm_weight(orc, cfg, l):
    """Layer l's pre-MoE RMSNorm weight as the stack generates it (1 + 0.1 N(0,1),
    fp32), as fp64; 1 when the stack was built without norm weights."""
    if not cfg.get("norm_weight", True):
        return 1.0
    w = orc.synth_normal(cfg["hidden"], 0.1, cfg["seed"], sid(l, 8, 0)) + np.float32(1.0)
    return w.astype(np.float64)


def oracle_chain(orc, cfg, h0, n_layers, gpu_routing=None, xs_out=None):
    """fp64 decode step: h <- h + moe_l(rmsnorm(h)) per layer, weights rebuilt
    on the host from the same seeded generator the stack used.

    Without gpu_routing the oracle routes every token itself and every
    token's top-k gap must exceed MARGIN (the seed is chosen for that).
    gpu_routing = (idx [L,T,K], w [L,T,K], sg [L,T]) of the stack's own step:
    every layer then uses the GPU's expert choices and weights, so the chain
    checks all expert arithmetic along the GPU's own path even where a near-tie
    in the router logits let the two sides pick differently (a long chain
    drifts by fp32 noise); check_routing() checks the choices themselves.
    xs_out: list that receives each layer's normalised input (fp32 [T,H])."""
    L, H, I, E, K, seed, eps = n_layers, cfg["hidden"], cfg["inter"], cfg["n_experts"], cfg["top_k"], cfg["seed"], cfg["eps"]
    nb_g, nb_d = I * H // 256, H * I // 256
    h = h0.astype(np.float64)
    for l in range(L):
        rinv = 1.0 / np.sqrt((h * h).mean(axis=1, keepdims=True) + eps)
        x = (h * rinv * norm_weight(orc, cfg, l)).astype(np.float32)
        if xs_out is not None:
            xs_out.append(x)
        if gpu_routing is None:
            W_r = orc.synth_normal(E * H, 0.02, seed, sid(l, 6, 0)).reshape(E, H)
            w_sg = orc.synth_normal(H, 0.02, seed, sid(l, 7, 0), half=True)
            idx, w, sg, _ = orc.route(x, W_r, w_sg, K)
            assert orc.routing_margin(x, W_r, K).min() > MARGIN, "pick a seed whose routing is well separated"
        else:
            idx, w, sg = (a[l] for a in gpu_routing)
        used = sorted(set(idx.ravel().tolist()))
        gate = [np.zeros(1, np.uint8)] * E
        up, down = list(gate), list(gate)
        for e in used:
            gate[e] = orc.synth_blocks(nb_g, 12, seed, sid(l, 0, e))
            up[e] = orc.synth_blocks(nb_g, 12, seed, sid(l, 1, e))
            down[e] = orc.synth_blocks(nb_d, 14, seed, sid(l, 2, e))
        sh = (orc.synth_blocks(nb_g, 12, seed, sid(l, 3, 0)), orc.synth_blocks(nb_g, 12, seed, sid(l, 4, 0)),
              orc.synth_blocks(nb_d, 14, seed, sid(l, 5, 0)))
        es = orc.ExpertSet(gate, up, down, *sh)
        h = h + orc.moe_f64(es, x, idx, w, sg, H, I)
    return h


def check_routing(orc, cfg, xs, gpu_routing, drift):
    """The GPU's routing of every layer against the oracle's routing of the
    oracle chain's own layer inputs xs.  The two inputs differ by the chain's
    fp32 drift (relative L2 `drift` of the residual stream; a unit-RMS x moves
    by |dx| = drift * sqrt(H)), which moves a logit gap by ~0.02 * sqrt(2) *
    |dx| rms (router weights N(0, 0.02)).  Tokens whose k-th / (k+1)-th gap
    exceeds 10 such sigmas (and MARGIN) must pick the same experts with the
    same renormalised weights (1e-3) and shared-gate weight; returns the
    fraction of token-layers left as near-ties."""
    H, E, K, seed = cfg["hidden"], cfg["n_experts"], cfg["top_k"], cfg["seed"]
    tol = max(MARGIN, 10 * 0.02 * np.sqrt(2.0) * drift * np.sqrt(H))
    gi, gw, gs = gpu_routing
    close_n = total = 0
    for l, x in enumerate(xs):
        W_r = orc.synth_normal(E * H, 0.02, seed, sid(l, 6, 0)).reshape(E, H)
        w_sg = orc.synth_normal(H, 0.02, seed, sid(l, 7, 0), half=True)
        idx, w, sg, _ = orc.route(x, W_r, w_sg, K)
        srt = -np.sort(-orc.router_logits_f64(x, W_r), axis=1)
        sep = (srt[:, K - 1] - srt[:, K]) > tol
        close_n += int((~sep).sum())
        total += sep.size
        a = np.argsort(gi[l][sep], axis=1)
        b = np.argsort(idx[sep], axis=1)
        assert np.array_equal(np.take_along_axis(gi[l][sep], a, 1), np.take_along_axis(idx[sep], b, 1)), \
            f"layer {l}: expert sets differ on a well-separated token (tol {tol:.2e})"
        # a weight moves relatively by about the logit perturbation, the
        # shared-gate sigmoid by at most a quarter of its score's; the drift
        # of single tokens exceeds the all-token rel-L2, hence the factor 4
        # (a wrong weight or token is off by tens of percent)
        rt = max(2e-3, 4 * tol)
        np.testing.assert_allclose(np.take_along_axis(gw[l][sep], a, 1), np.take_along_axis(w[sep], b, 1),
                                   rtol=rt, atol=1e-5, err_msg=f"layer {l}: routing weights")
        np.testing.assert_allclose(gs[l][sep], sg[sep], rtol=rt, atol=rt, err_msg=f"layer {l}: shared gate")
    return close_n / max(total, 1)


@pytest.mark.parametrize("T,seed", [(1, 11), (3, 11), (12, 18), (24, 18)])
def test_stack_small_vs_oracle(cuda, orc, T, seed):
    """3 layers chained through the residual; T > 8 takes the tiled router and
    the shared ring arena, T > 16 the grid-distributed top-k (seeds picked so
    every token's routing is separated by more than fp32 noise)."""
    cfg = dict(hidden=512, inter=256, n_experts=16, top_k=4, seed=seed, eps=1e-6)
    st = bb.ExpertStack(n_layers=3, hidden=512, inter=256, n_experts=16, top_k=4, max_tokens=max(4, T),
                        shared_expert=True, norm_eps=1e-6, seed=seed)
    h0 = bb.synth_normal(T * 512, 1.0, seed, 1000 + T, device=cuda).view(T, 512)
    h = h0.clone()
    st.step(h)
    torch.cuda.synchronize()
    ref = oracle_chain(orc, cfg, h0.cpu().numpy(), 3)
    assert orc.rel_l2(h.cpu().numpy(), ref) < TOL
    assert bb.device_error() == 0
    st.close()


@pytest.mark.parametrize("T", [1, 64])
def test_stack_config_size_two_layers(cuda, orc, T):
    """Full layer shapes (H=2048, I=512, 256 experts, top-8 + shared), 2 layers,
    T=1 and the bench's batch of 64: the fp64 chain along the GPU's routing,
    then the routing itself against the oracle's."""
    cfg = dict(hidden=2048, inter=512, n_experts=256, top_k=8, seed=3, eps=1e-6)
    st = bb.ExpertStack(n_layers=2, max_tokens=T, seed=3)
    h0 = bb.synth_normal(T * 2048, 1.0, 3, 43, device=cuda).view(T, 2048)
    h = h0.clone()
    st.step(h)
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    rec = st.routing()
    st.close()
    xs = []
    ref = oracle_chain(orc, cfg, h0.cpu().numpy(), 2, gpu_routing=rec, xs_out=xs)
    err = orc.rel_l2(h.cpu().numpy(), ref)
    assert err < TOL
    check_routing(orc, cfg, xs, rec, err)


def test_stack_from_gguf_equals_synthetic(cuda, orc, tmp_path):
    """Row f2: a GGUF model file holding the synthetic stack's weights, loaded
    by bread_stack_create_gguf, steps bit-identically to the synthetic stack
    (decode kernel at T = 1 and 5, large-batch kernel at T = 12)."""
    import gguf_file as G

    path = str(tmp_path / "model.gguf")
    G.write_synthetic_model(orc, path, 3, 1024, 256, 16, seed=13)
    a = bb.ExpertStack(n_layers=3, hidden=1024, inter=256, n_experts=16, top_k=4, max_tokens=12, seed=13)
    b = bb.ExpertStack.from_gguf(path, n_layers=3, top_k=4, max_tokens=12)
    assert (b.cfg.hidden, b.cfg.inter, b.cfg.n_experts, b.cfg.shared_expert, b.cfg.norm_weight) == (1024, 256, 16, 1, 1)
    for T in (1, 5, 12):
        h0 = bb.synth_normal(T * 1024, 1.0, 13, 50 + T, device=cuda).view(T, 1024)
        ha, hb = h0.clone(), h0.clone()
        a.step(ha)
        b.step(hb)
        torch.cuda.synchronize()
        assert torch.equal(ha, hb), f"T={T}"
    assert bb.device_error() == 0
    a.close()
    b.close()


def test_stack_norm_weight_matches_generator(cuda, orc):
    """The stack's per-layer RMSNorm weights (post_attention_norm.weight
    stand-ins) are the seeded vectors the oracle chain uses; a stack built
    without them reports none."""
    cfg = dict(hidden=512, seed=7)
    st = bb.ExpertStack(n_layers=2, hidden=512, inter=256, n_experts=16, top_k=4, max_tokens=2, seed=7)
    for l in range(2):
        w = st.norm_weight(l)
        assert w is not None
        assert np.array_equal(w.astype(np.float64), norm_weight(orc, cfg, l))
    st.close()
    st = bb.ExpertStack(n_layers=1, hidden=512, inter=256, n_experts=16, top_k=4, max_tokens=2, seed=7,
                        norm_weight=False)
    assert st.norm_weight(0) is None
    st.close()


def test_stack_host_step_and_determinism(cuda):
    st = bb.ExpertStack(n_layers=4, hidden=1024, inter=512, n_experts=32, top_k=4, max_tokens=8, seed=5)
    T = 8
    h0 = bb.synth_normal(T * 1024, 1.0, 5, 1, device=cuda).view(T, 1024)
    a = h0.clone()
    st.step(a)
    b = h0.clone()
    st.step(b)  # graph replay
    hin = h0.cpu().pin_memory()
    hout = torch.empty_like(hin).pin_memory()
    st.step_host(hin, hout)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    assert torch.equal(a.cpu(), hout)
    assert st.launches_per_step(T) == 1  # the whole step is one cooperative launch
    st.close()


@pytest.mark.parametrize("T", [1, 64])
def test_stack_bench_config_40_layers(cuda, orc, T):
    """The benchmark's own workload at full size: 40 layers x (256 + 1)
    experts resident (21 GB), H=2048, I=512, top-8 + shared expert, one decode
    step at T=1 (the flagged-word decode kernel) and T=64 (the large-batch
    kernel) against the fp64 oracle chain over all 40 layers, then every
    layer's routing against the oracle's."""
    cfg = dict(hidden=2048, inter=512, n_experts=256, top_k=8, seed=1234, eps=1e-6)
    st = bb.ExpertStack(n_layers=40, max_tokens=T, seed=1234)
    h0 = bb.synth_normal(T * 2048, 1.0, 1234, 900, device=cuda).view(T, 2048)
    h = h0.clone()
    st.step(h)
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    rec = st.routing()
    st.close()
    xs = []
    ref = oracle_chain(orc, cfg, h0.cpu().numpy(), 40, gpu_routing=rec, xs_out=xs)
    err = orc.rel_l2(h.cpu().numpy(), ref)
    assert err < TOL
    near = check_routing(orc, cfg, xs, rec, err)
    assert near < 0.25, f"near-tie fraction {near:.3f} (rel-L2 {err:.2e})"
