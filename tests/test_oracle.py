"""CPU: the oracle restatement (oracle/oracle.c) pinned against the reference.

Pins: the reference's known-answer blocks (dequant_q4k_cpu.c:181-283,
kernels.cu:411-446), fixtures produced by the reference's own CPU code
(tests/golden, see make_golden.py), and -- where the reference was compiled
here (oracle/_ref) -- fresh seeded inputs run through both.
"""
import numpy as np
import pytest

from oracle import blocks as B

Q4_K, Q6_K = 12, 14


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


def test_kat_q4k(orc):
    # dequant_q4k_cpu.c:212-234: elements 64g+0..31 = 9.0, 64g+32..63 = 5.0
    out = orc.dequant(B.kat_q4k_block(), Q4_K, 1)
    exp = np.tile(np.r_[np.full(32, 9.0), np.full(32, 5.0)], 4).astype(np.float32)
    assert np.array_equal(out, exp)


def test_kat_q6k(orc):
    # dequant_q4k_cpu.c:253-283: all 256 = 8.0
    assert np.array_equal(orc.dequant(B.kat_q6k_block(), Q6_K, 1), np.full(256, 8.0, np.float32))


def test_kat_rowsum(orc):
    # kernels.cu:451-579 self-test shape: 8 rows x 1 block, x = 1 -> 1792 (Q4_K), 2048 (Q6_K)
    x = np.ones(256, np.float32)
    y4 = orc.matvec_f32(np.tile(B.kat_q4k_block(), 8), Q4_K, x, 8, 256)
    y6 = orc.matvec_f32(np.tile(B.kat_q6k_block(), 8), Q6_K, x, 8, 256)
    assert np.all(y4 == 1792.0) and np.all(y6 == 2048.0)


@pytest.mark.parametrize("name,qt", [("q4k", Q4_K), ("q6k", Q6_K)])
def test_dequant_golden(orc, golden, name, qt):
    g = golden["dequant"]
    blk = g[f"{name}_blocks"]
    n = blk.shape[0]
    assert np.array_equal(bits(orc.dequant(blk.reshape(-1), qt, n, ftz=False)), bits(g[f"{name}_exact"]))
    assert np.array_equal(bits(orc.dequant(blk.reshape(-1), qt, n, ftz=True)), bits(g[f"{name}_ftz"]))


def test_subnormal_divergence_is_only_on_subnormal_scales(orc, golden):
    """The two reference decoders (layer_ops.cu exact, dequant_q4k_cpu.c FTZ)
    disagree exactly on blocks whose fp16 scales are subnormal."""
    g = golden["dequant"]
    blk = g["q4k_blocks"]
    ex, ftz = g["q4k_exact"].reshape(-1, 256), g["q4k_ftz"].reshape(-1, 256)
    d = blk[:, 0].astype(np.uint16) | (blk[:, 1].astype(np.uint16) << 8)
    m = blk[:, 2].astype(np.uint16) | (blk[:, 3].astype(np.uint16) << 8)
    sub = (((d >> 10) & 31) == 0) & ((d & 0x3FF) != 0) | (((m >> 10) & 31) == 0) & ((m & 0x3FF) != 0)
    differs = np.any(bits(ex) != bits(ftz), axis=1)
    assert np.all(differs <= sub) and differs.any()


def test_matvec_golden(orc, golden):
    g = golden["matvec"]
    assert np.array_equal(orc.matvec_f32(g["q4k_w"], Q4_K, g["q4k_x"], 64, 2048), g["q4k_y"])
    assert np.array_equal(orc.matvec_f32(g["q6k_w"], Q6_K, g["q6k_x"], 128, 512), g["q6k_y"])


def test_matvec_f64_close(orc, golden):
    g = golden["matvec"]
    y64 = orc.matvec_f64(g["q4k_w"], Q4_K, g["q4k_x"], 64, 2048)
    assert orc.rel_l2(g["q4k_y"], y64) < 1e-5


def test_route_golden(orc, golden):
    g = golden["route"]
    idx, w, sg, _ = orc.route(g["x"], g["W_r"], g["w_sg"], int(g["top_k"]))
    assert np.array_equal(idx, g["idx"])
    assert np.array_equal(w, g["w"])
    assert np.array_equal(sg, g["sg_weight"])


def test_swiglu_golden(orc, golden):
    g = golden["swiglu"]
    assert np.array_equal(orc.swiglu(g["g"], g["u"]), g["out"])


def _moe_set(orc, g):
    return orc.ExpertSet(list(g["gate"]), list(g["up"]), list(g["down"]), g["sh_gate"], g["sh_up"], g["sh_down"])


def test_moe_golden(orc, golden):
    g = golden["moe"]
    T, H, I, E, K = (int(v) for v in g["dims"])
    es = _moe_set(orc, g)
    out32 = orc.moe_f32(es, g["x"], g["idx"], g["w"], g["sg_weight"], H, I)
    assert np.array_equal(out32, g["out"])
    out64 = orc.moe_f64(es, g["x"], g["idx"], g["w"], g["sg_weight"], H, I)
    assert orc.rel_l2(g["out"], out64) < 1e-5


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference not compiled here")
def test_reference_kat_main(orc):
    assert orc.ref_kat() == 0  # the reference's own main(): "Overall: PASS"


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference not compiled here")
@pytest.mark.parametrize("mode", ["baseline", "subnormal", "zero_scale", "large", "mixed"])
def test_dequant_vs_reference_fresh(orc, mode):
    rng = np.random.default_rng(7)
    for qt, gen in ((Q4_K, B.q4k_blocks), (Q6_K, B.q6k_blocks)):
        w = gen(rng, 200, mode).reshape(-1)
        for ftz in (False, True):
            assert np.array_equal(bits(orc.dequant(w, qt, 200, ftz)), bits(orc.ref_dequant(w, qt, 200, ftz)))


@pytest.mark.skipif(not __import__("oracle").ref_available(), reason="reference not compiled here")
def test_route_vs_reference_fresh(orc):
    rng = np.random.default_rng(8)
    x = rng.standard_normal((6, 2048)).astype(np.float32)
    W = (rng.standard_normal((256, 2048)) * 0.02).astype(np.float32)
    sg = (rng.standard_normal(2048) * 0.02).astype(np.float16).view(np.uint16)
    a = orc.route(x, W, sg, 8)
    b = orc.ref_route(x, W, sg, 8)
    for u, v in zip(a[:3], b):
        assert np.array_equal(u, v)
