"""GPU: the MoE FFN block (router top-k, grouped gate/up + SiLU*mul, grouped
down + weighted combine) against the oracle.

Routing: indices must equal the oracle's (route_layer semantics, lowest index
wins ties) for every token whose k-th/(k+1)-th logit gap exceeds fp32
summation noise; weights within 1e-5 relative.  MoE outputs: relative L2 <=
1e-3 against the fp64 oracle given the same routing."""
import numpy as np
import pytest
import torch

import breadv2_b200 as bb
from oracle import blocks as B

pytestmark = pytest.mark.gpu
TOL = 1e-3
MARGIN = 1e-4  # logit gap below which fp32 summation order may legally reorder


class Layer:
    """Synthetic MoE layer on the device (bread_synth_*), pointer tables included."""

    def __init__(self, cuda, H, I, E, shared=True, sg_vec=True, seed=5, stack_layer=0, router_std=0.02):
        self.H, self.I, self.E = H, I, E
        sid = lambda kind, e: (stack_layer << 32) | (kind << 24) | e  # noqa: E731
        nb_g, nb_d = I * H // 256, H * I // 256
        self.gate = [bb.synth_blocks(nb_g, 12, seed, sid(0, e), device=cuda) for e in range(E)]
        self.up = [bb.synth_blocks(nb_g, 12, seed, sid(1, e), device=cuda) for e in range(E)]
        self.down = [bb.synth_blocks(nb_d, 14, seed, sid(2, e), device=cuda) for e in range(E)]
        self.shared = None
        if shared:
            self.shared = (bb.synth_blocks(nb_g, 12, seed, sid(3, 0), device=cuda),
                           bb.synth_blocks(nb_g, 12, seed, sid(4, 0), device=cuda),
                           bb.synth_blocks(nb_d, 14, seed, sid(5, 0), device=cuda))
        self.W_r = bb.synth_normal(E * H, router_std, seed, sid(6, 0), device=cuda).view(E, H)
        self.w_sg = bb.synth_normal(H, 0.02, seed, sid(7, 0), half=True, device=cuda) if sg_vec else None
        self.tabs = [bb.pointer_table(t, cuda) for t in (self.gate, self.up, self.down)]

    def host_set(self, orc, experts):
        """oracle.ExpertSet holding host copies of the given experts (others empty)."""
        gate = [np.zeros(1, np.uint8)] * self.E
        up, down = list(gate), list(gate)
        for e in set(int(v) for v in experts):
            gate[e] = self.gate[e].cpu().numpy()
            up[e] = self.up[e].cpu().numpy()
            down[e] = self.down[e].cpu().numpy()
        sh = [t.cpu().numpy() for t in self.shared] if self.shared else [None] * 3
        return orc.ExpertSet(gate, up, down, *sh)

    def ffn(self, x, top_k, out=None):
        if out is None:
            out = torch.zeros_like(x)
        r = bb.moe_ffn(*self.tabs, self.W_r, self.w_sg, self.shared, x, out, self.I, top_k, want_routing=True)
        return out, r


def check_routing(orc, x, W_r, w_sg, top_k, idx, w, sg, w_rtol=1e-5):
    """w_rtol: a softmax weight's relative error is its logit's absolute error,
    and fp32 summation noise in a logit grows with the logit's magnitude, so
    routers with larger weights get a proportionally larger tolerance."""
    xi = x.cpu().numpy()
    ridx, rw, rsg, _ = orc.route(xi, W_r.cpu().numpy(), None if w_sg is None else w_sg.cpu().numpy().view(np.uint16),
                                 top_k)
    margin = orc.routing_margin(xi, W_r.cpu().numpy(), top_k)
    ok = margin > MARGIN
    assert ok.mean() > 0.9, "seeded inputs should be mostly well separated"
    gi, gw = idx.cpu().numpy(), w.cpu().numpy()
    assert np.array_equal(gi[ok], ridx[ok])
    np.testing.assert_allclose(gw[ok], rw[ok], rtol=w_rtol, atol=1e-7)
    np.testing.assert_allclose(sg.cpu().numpy(), rsg, rtol=1e-5)
    return ridx, rw, rsg


@pytest.mark.parametrize("T", [1, 8, 64])
def test_route_config(cuda, orc, T):
    H, E, K = 2048, 256, 8
    W_r = bb.synth_normal(E * H, 0.02, 3, 1, device=cuda).view(E, H)
    w_sg = bb.synth_normal(H, 0.02, 3, 2, half=True, device=cuda)
    x = bb.synth_normal(T * H, 1.0, 3, 10 + T, device=cuda).view(T, H)
    idx, w, sg = bb.moe_route(x, W_r, w_sg, K)
    check_routing(orc, x, W_r, w_sg, K, idx, w, sg)
    assert torch.allclose(w.sum(1), torch.ones(T, device=cuda), atol=1e-5)


def test_route_golden(cuda, golden):
    g = golden["route"]
    x = torch.from_numpy(g["x"]).to(cuda)
    W = torch.from_numpy(g["W_r"]).to(cuda)
    sg = torch.from_numpy(g["w_sg"].view(np.float16)).to(cuda)
    idx, w, s = bb.moe_route(x, W, sg, int(g["top_k"]))
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    np.testing.assert_allclose(w.cpu().numpy(), g["w"], rtol=1e-5)
    np.testing.assert_allclose(s.cpu().numpy(), g["sg_weight"], rtol=1e-5)


def test_route_no_shared_gate_is_half(cuda):
    W = bb.synth_normal(64 * 256, 0.02, 1, 1, device=cuda).view(64, 256)
    x = bb.synth_normal(3 * 256, 1.0, 1, 2, device=cuda).view(3, 256)
    _, _, sg = bb.moe_route(x, W, None, 4)
    assert torch.all(sg == 0.5)  # one_layer.cu:944,1889


def test_route_ties_lowest_index(cuda):
    """Equal logits: the lowest expert index wins (layer_ops.cu:241 strict >)."""
    E, H = 32, 256
    W = torch.zeros(E, H, device=cuda)
    W[[3, 7, 9, 20], 0] = 1.0  # four equal winners
    x = torch.zeros(1, H, device=cuda)
    x[0, 0] = 1.0
    idx, w, _ = bb.moe_route(x, W, None, 6)
    assert idx[0, :4].tolist() == [3, 7, 9, 20]
    assert idx[0, 4:].tolist() == [0, 1]


def test_moe_ffn_golden(cuda, orc, golden):
    """The reference's own fp32 expert block (expert_bench.cu:158-179 + shared)."""
    g = golden["moe"]
    T, H, I, E, K = (int(v) for v in g["dims"])
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(cuda)  # noqa: E731
    gate, up, down = [d(a) for a in g["gate"]], [d(a) for a in g["up"]], [d(a) for a in g["down"]]
    tabs = [bb.pointer_table(t, cuda) for t in (gate, up, down)]
    shared = (d(g["sh_gate"]), d(g["sh_up"]), d(g["sh_down"]))
    x = d(g["x"])
    out = torch.zeros_like(x)
    idx, w, sg = bb.moe_ffn(*tabs, d(g["W_r"]), d(g["w_sg"].view(np.float16)), shared, x, out, I, K,
                            want_routing=True)
    assert np.array_equal(idx.cpu().numpy(), g["idx"])
    es = orc.ExpertSet(list(g["gate"]), list(g["up"]), list(g["down"]), g["sh_gate"], g["sh_up"], g["sh_down"])
    ref64 = orc.moe_f64(es, g["x"], g["idx"], g["w"], g["sg_weight"], H, I)
    assert orc.rel_l2(out.cpu().numpy(), ref64) < TOL
    assert orc.rel_l2(out.cpu().numpy(), g["out"]) < TOL


@pytest.mark.parametrize("T", [1, 2, 4, 8, 16, 32, 64])
def test_moe_ffn_config(cuda, orc, T):
    """Config 3 (T=1) and config 4's sweep: H=2048, 256 experts, top-8 + shared.
    T <= 8 routes from router rows held in shared memory; T > 8 tiles the
    router over the grid and shares one ring arena between gate/up and down;
    T > 16 also spreads the top-k selection over the grid."""
    H, I, E, K = 2048, 512, 256, 8
    L = getattr(test_moe_ffn_config, "_layer", None)
    if L is None:
        L = test_moe_ffn_config._layer = Layer(cuda, H, I, E)
    x = bb.synth_normal(T * H, 1.0, 77, T, device=cuda).view(T, H)
    out, (idx, w, sg) = L.ffn(x, K)
    ridx, rw, rsg = check_routing(orc, x, L.W_r, L.w_sg, K, idx, w, sg)
    gi, gw, gs = idx.cpu().numpy(), w.cpu().numpy(), sg.cpu().numpy()
    es = L.host_set(orc, gi.ravel())
    ref = orc.moe_f64(es, x.cpu().numpy(), gi, gw, gs, H, I)
    assert orc.rel_l2(out.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("T", [1, 5, 24])
def test_moe_ffn_wide_router(cuda, orc, T):
    """512 experts, top-16 (the kernel's largest router): per-lane key arrays
    twice as long as at 256 experts, on every routing path (one token, a few
    tokens, grid-distributed selection)."""
    H, I, E, K = 1024, 256, 512, 16
    L = getattr(test_moe_ffn_wide_router, "_layer", None)
    if L is None:
        L = test_moe_ffn_wide_router._layer = Layer(cuda, H, I, E, seed=31, router_std=0.1)
    x = bb.synth_normal(T * H, 1.0, 31, 100 + T, device=cuda).view(T, H)
    out, (idx, w, sg) = L.ffn(x, K)
    # router std 0.1 (logits ~3, five times the 0.02 router's): weights to 5e-5
    check_routing(orc, x, L.W_r, L.w_sg, K, idx, w, sg, w_rtol=5e-5)
    gi = idx.cpu().numpy()
    assert all(len(set(r)) == K for r in gi.tolist())
    es = L.host_set(orc, gi.ravel())
    ref = orc.moe_f64(es, x.cpu().numpy(), gi, w.cpu().numpy(), sg.cpu().numpy(), H, I)
    assert orc.rel_l2(out.cpu().numpy(), ref) < TOL


def test_moe_ffn_accumulates_and_no_shared(cuda, orc):
    H, I, E, K, T = 512, 256, 16, 4, 3
    L = Layer(cuda, H, I, E, shared=False, sg_vec=False, seed=9)
    x = bb.synth_normal(T * H, 1.0, 9, 1, device=cuda).view(T, H)
    base = bb.synth_normal(T * H, 5.0, 9, 2, device=cuda).view(T, H)
    out, (idx, w, sg) = L.ffn(x, K, out=base.clone())
    es = L.host_set(orc, idx.cpu().numpy().ravel())
    ref = orc.moe_f64(es, x.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), sg.cpu().numpy(), H, I)
    assert orc.rel_l2(out.cpu().numpy() - base.cpu().numpy(), ref) < TOL


@pytest.mark.parametrize("H,I", [(256, 256), (1024, 1024), (4096, 512), (512, 2048)])
def test_moe_ffn_shapes(cuda, orc, H, I):
    E, K, T = 32, 4, 5
    L = Layer(cuda, H, I, E, seed=H + I)
    x = bb.synth_normal(T * H, 1.0, 3, 3, device=cuda).view(T, H)
    out, (idx, w, sg) = L.ffn(x, K)
    es = L.host_set(orc, idx.cpu().numpy().ravel())
    ref = orc.moe_f64(es, x.cpu().numpy(), idx.cpu().numpy(), w.cpu().numpy(), sg.cpu().numpy(), H, I)
    assert orc.rel_l2(out.cpu().numpy(), ref) < TOL


def test_moe_ffn_deterministic(cuda):
    H, I, E, K, T = 1024, 512, 64, 8, 16
    L = Layer(cuda, H, I, E, seed=1)
    x = bb.synth_normal(T * H, 1.0, 4, 4, device=cuda).view(T, H)
    a, _ = L.ffn(x, K)
    b, _ = L.ffn(x, K)
    assert torch.equal(a, b)
