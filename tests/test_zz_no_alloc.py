"""GPU: bread_moe_ffn_noalloc, the MoE block for callers that cannot allocate
device memory (an engine that gave all free HBM to its weights and caches, or a
decode loop that must not call cudaMalloc because it can synchronise the
device).  Its scratch is a fixed array inside the library instead of a caller
workspace; the results must match bread_moe_ffn's within the MoE tolerance
(relative L2 1e-3), on two calls in a row (the second one finds the first
call's leftovers in the shared array).  Kept in the last-collected file so a
run that stops at the first failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

import breadv2_b200 as bb

pytestmark = pytest.mark.gpu
TOL = 1e-3


def _rel(a, b):
    return float((a - b).norm() / b.norm())


def _layer(dev, H, I, E, seed):
    nb_g, nb_d = I * H // 256, H * I // 256
    gate = [bb.synth_blocks(nb_g, 12, seed, 10 + e, device=dev) for e in range(E)]
    up = [bb.synth_blocks(nb_g, 12, seed, 1000 + e, device=dev) for e in range(E)]
    down = [bb.synth_blocks(nb_d, 14, seed, 2000 + e, device=dev) for e in range(E)]
    shared = (bb.synth_blocks(nb_g, 12, seed, 3000, device=dev), bb.synth_blocks(nb_g, 12, seed, 3001, device=dev),
              bb.synth_blocks(nb_d, 14, seed, 3002, device=dev))
    W_r = bb.synth_normal(E * H, 0.02, seed, 3003, device=dev).view(E, H)
    w_sg = bb.synth_normal(H, 0.02, seed, 3004, half=True, device=dev)
    tabs = [bb.pointer_table(t, dev) for t in (gate, up, down)]
    return tabs, W_r, w_sg, shared, (gate, up, down)


def _noalloc(tabs, W_r, w_sg, shared, x, out, I, K, idx, w, sg, stream=None):
    T, H = x.shape
    E = W_r.shape[0]
    p = bb._p
    return bb.lib().bread_moe_ffn_noalloc(p(tabs[0]), p(tabs[1]), p(tabs[2]), p(W_r), p(w_sg), p(shared[0]),
                                          p(shared[1]), p(shared[2]), p(x), p(out), T, H, I, E, K, p(idx), p(w),
                                          p(sg), bb._s(stream))


@pytest.mark.parametrize("T", [1, 8, 16])
def test_noalloc_matches_workspace_entry(cuda, T):
    H, I, E, K = 2048, 512, 256, 8
    tabs, W_r, w_sg, shared, _keep = _layer(cuda, H, I, E, seed=17)
    x = bb.synth_normal(T * H, 1.0, 17, 4000 + T, device=cuda).view(T, H)
    base = bb.synth_normal(T * H, 3.0, 17, 5000 + T, device=cuda).view(T, H)
    ref = base.clone()
    ridx, rw, rsg = bb.moe_ffn(*tabs, W_r, w_sg, shared, x, ref, I, K, want_routing=True)
    for call in range(2):
        out = base.clone()
        idx = torch.empty(T, K, dtype=torch.int32, device=cuda)
        w = torch.empty(T, K, dtype=torch.float32, device=cuda)
        sg = torch.empty(T, dtype=torch.float32, device=cuda)
        st = _noalloc(tabs, W_r, w_sg, shared, x, out, I, K, idx, w, sg)
        assert st == 0, bb.last_error()
        torch.cuda.synchronize()
        assert torch.equal(idx, ridx), f"call {call}: routing differs"
        assert _rel(out - base, ref - base) < TOL, f"call {call}"
    assert bb.device_error() == 0


def test_noalloc_t16_on_a_side_stream(cuda):
    """The largest accepted shape at the config sizes (T = 16), two calls
    ordered on a non-default stream, both equal to the workspace entry point."""
    H, I, E, K, T = 2048, 512, 256, 8, 16
    tabs, W_r, w_sg, shared, _keep = _layer(cuda, H, I, E, seed=23)
    x = bb.synth_normal(T * H, 1.0, 23, 4100, device=cuda).view(T, H)
    base = bb.synth_normal(T * H, 3.0, 23, 5100, device=cuda).view(T, H)
    ref = base.clone()
    bb.moe_ffn(*tabs, W_r, w_sg, shared, x, ref, I, K)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    outs = [base.clone(), base.clone()]
    idx = torch.empty(T, K, dtype=torch.int32, device=cuda)
    w = torch.empty(T, K, dtype=torch.float32, device=cuda)
    sg = torch.empty(T, dtype=torch.float32, device=cuda)
    side.wait_stream(torch.cuda.current_stream())
    for out in outs:  # back to back on the side stream: ordered, so they do not race on the array
        assert _noalloc(tabs, W_r, w_sg, shared, x, out, I, K, idx, w, sg, stream=side) == 0, bb.last_error()
    side.synchronize()
    for call, out in enumerate(outs):
        assert _rel(out - base, ref - base) < TOL, f"call {call}"
    assert bb.device_error() == 0


@pytest.mark.parametrize("T", [17, 64])
def test_noalloc_rejects_oversized_shapes(cuda, T):
    """Shapes whose scratch exceeds the fixed array are refused before any GPU
    work: at the config sizes T = 16 is the largest accepted, 17 is refused."""
    H, I, E, K = 2048, 512, 256, 8
    dummy = torch.zeros(16, dtype=torch.int64, device=cuda)
    x = torch.zeros(T, H, device=cuda)
    st = bb.lib().bread_moe_ffn_noalloc(bb._p(dummy), bb._p(dummy), bb._p(dummy), bb._p(x), None, None, None, None,
                                        bb._p(x), bb._p(x), T, H, I, E, K, None, None, None, bb._s(None))
    assert st == 5  # BREAD_ERR_WORKSPACE
    assert "scratch" in bb.last_error()
