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


def oracle_chain(orc, cfg, h0, n_layers, gpu_routing=None, stats=None):
    """fp64 decode step: h <- h + moe_l(rmsnorm(h)) per layer, weights rebuilt
    on the host from the same seeded generator the stack used.

    gpu_routing: (idx [L,T,K], w [L,T,K], sg [L,T]) of the stack's own step.
    Without it every token's top-k gap must exceed MARGIN (the seed is chosen
    for that).  With it, a token whose k-th / (k+1)-th logit gap is below
    MARGIN -- where fp32 summation order alone may flip the pick -- takes the
    GPU's routing for that layer only; every other token's experts must equal
    the oracle's (checked here)."""
    L, H, I, E, K, seed, eps = n_layers, cfg["hidden"], cfg["inter"], cfg["n_experts"], cfg["top_k"], cfg["seed"], cfg["eps"]
    nb_g, nb_d = I * H // 256, H * I // 256
    h = h0.astype(np.float64)
    injected = 0
    for l in range(L):
        rinv = 1.0 / np.sqrt((h * h).mean(axis=1, keepdims=True) + eps)
        x = (h * rinv).astype(np.float32)
        W_r = orc.synth_normal(E * H, 0.02, seed, sid(l, 6, 0)).reshape(E, H)
        w_sg = orc.synth_normal(H, 0.02, seed, sid(l, 7, 0), half=True)
        idx, w, sg, _ = orc.route(x, W_r, w_sg, K)
        margin = orc.routing_margin(x, W_r, K)
        if gpu_routing is None:
            assert margin.min() > MARGIN, "pick a seed whose routing is well separated"
        else:
            gi, gw, gs = gpu_routing
            close = margin <= MARGIN
            sep = ~close
            assert np.array_equal(np.sort(gi[l][sep], axis=1), np.sort(idx[sep], axis=1)), f"layer {l}: routing differs"
            idx, w, sg = idx.copy(), w.copy(), sg.copy()
            idx[close], w[close], sg[close] = gi[l][close], gw[l][close], gs[l][close]
            injected += int(close.sum())
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
    if stats is not None:
        stats["injected"] = injected
    return h


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


def test_stack_config_size_two_layers(cuda, orc):
    """Full layer shapes (H=2048, I=512, 256 experts, top-8 + shared), 2 layers, T=1."""
    cfg = dict(hidden=2048, inter=512, n_experts=256, top_k=8, seed=3, eps=1e-6)
    st = bb.ExpertStack(n_layers=2, max_tokens=2, seed=3)
    h0 = bb.synth_normal(2048, 1.0, 3, 43, device=cuda).view(1, 2048)
    h = h0.clone()
    st.step(h)
    torch.cuda.synchronize()
    ref = oracle_chain(orc, cfg, h0.cpu().numpy(), 2)
    assert orc.rel_l2(h.cpu().numpy(), ref) < TOL
    st.close()


def test_stack_config_size_batch64(cuda, orc):
    """The bench's batched workload: full layer shapes, T=64, 2 layers."""
    cfg = dict(hidden=2048, inter=512, n_experts=256, top_k=8, seed=3, eps=1e-6)
    st = bb.ExpertStack(n_layers=2, max_tokens=64, seed=3)
    h0 = bb.synth_normal(64 * 2048, 1.0, 3, 43, device=cuda).view(64, 2048)
    h = h0.clone()
    st.step(h)
    torch.cuda.synchronize()
    ref = oracle_chain(orc, cfg, h0.cpu().numpy(), 2)
    assert orc.rel_l2(h.cpu().numpy(), ref) < TOL
    assert bb.device_error() == 0
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
    kernel) against the fp64 oracle chain over all 40 layers."""
    cfg = dict(hidden=2048, inter=512, n_experts=256, top_k=8, seed=1234, eps=1e-6)
    st = bb.ExpertStack(n_layers=40, max_tokens=T, seed=1234)
    h0 = bb.synth_normal(T * 2048, 1.0, 1234, 900, device=cuda).view(T, 2048)
    h = h0.clone()
    st.step(h)
    torch.cuda.synchronize()
    assert bb.device_error() == 0
    rec = st.routing()
    st.close()
    info = {}
    ref = oracle_chain(orc, cfg, h0.cpu().numpy(), 40, gpu_routing=rec, stats=info)
    assert info["injected"] <= max(2, T * 40 // 50), info  # near-ties are rare
    assert orc.rel_l2(h.cpu().numpy(), ref) < TOL
