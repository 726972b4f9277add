"""GPU: Q4_K / Q6_K / Q8_0 GEMV parity.  Bar: relative L2 error <= 1e-3
against an fp64-accumulated product of the exactly dequantised weights
(oracle.matvec_f64)."""
import numpy as np
import pytest
import torch

import breadv2_b200 as bb
from oracle import blocks as B

pytestmark = pytest.mark.gpu
TOL = 1e-3


def dev(a, cuda):
    return torch.from_numpy(np.ascontiguousarray(a)).to(cuda)


SHAPES = [
    (12, 512, 2048),   # config 1: one expert gate_proj
    (14, 2048, 512),   # config 2: one expert down_proj
    (12, 64, 256), (12, 130, 512), (12, 37, 1024), (12, 100, 4096),   # cols/256 = 1, 2 (ragged), 4, 16
    (14, 96, 256), (14, 33, 1024), (14, 64, 2048), (14, 50, 4096),
    (12, 16, 768), (14, 9, 1536),                                     # cols/256 = 3, 6: generic path
    (8, 64, 2048), (8, 5, 96),                                        # Q8_0
    (12, 1, 2048), (14, 1, 512),                                      # one row
]


@pytest.mark.parametrize("qt,rows,cols", SHAPES)
def test_matvec_f32(cuda, orc, qt, rows, cols):
    rng = np.random.default_rng(rows * 7 + cols + qt)
    w = B.matrix(qt, rng, rows, cols)
    x = rng.standard_normal(cols).astype(np.float32)
    y = bb.matvec_f32(dev(w, cuda), dev(x, cuda), rows, cols, qt).cpu().numpy()
    ref = orc.matvec_f64(w, qt, x, rows, cols)
    assert orc.rel_l2(y, ref) < TOL


@pytest.mark.parametrize("qt", [12, 14])
@pytest.mark.parametrize("mode", ["subnormal", "zero_scale", "large", "mixed"])
def test_matvec_weight_modes(cuda, orc, qt, mode):
    rng = np.random.default_rng(31)
    rows, cols = 256, 2048
    w = B.matrix(qt, rng, rows, cols, mode)
    x = rng.standard_normal(cols).astype(np.float32)
    y = bb.matvec_f32(dev(w, cuda), dev(x, cuda), rows, cols, qt).cpu().numpy()
    ref = orc.matvec_f64(w, qt, x, rows, cols)
    if mode == "zero_scale" and qt == 12:
        assert np.all(y == 0)
    else:
        assert orc.rel_l2(y, ref) < TOL


@pytest.mark.parametrize("qt", [12, 14])
def test_matvec_activation_edges(cuda, orc, qt):
    rng = np.random.default_rng(3)
    rows, cols = 128, 2048
    w = B.matrix(qt, rng, rows, cols)
    wd = dev(w, cuda)
    x0 = np.zeros(cols, np.float32)
    assert np.all(bb.matvec_f32(wd, dev(x0, cuda), rows, cols, qt).cpu().numpy() == 0)
    x = rng.standard_normal(cols).astype(np.float32)
    x[17] = 3e4          # one outlier: its 32-value group keeps ~16 bits around it
    x[100:132] = 1e-30   # a group of tiny values
    y = bb.matvec_f32(wd, dev(x, cuda), rows, cols, qt).cpu().numpy()
    assert orc.rel_l2(y, orc.matvec_f64(w, qt, x, rows, cols)) < TOL
    xn = x.copy()
    xn[5] = np.nan
    yn = bb.matvec_f32(wd, dev(xn, cuda), rows, cols, qt).cpu().numpy()
    assert np.all(np.isnan(yn))


def _zero_column(w, qt, rows, cols, c):
    """Give column c zero weight in every row, keeping the other columns of
    its 32-value group: Q4_K with dmin = 0 and that element's nibble 0;
    Q6_K with that element's 6-bit value 32 (dequant_q4k_cpu.c:146-172)."""
    blk = w.reshape(rows, cols // 256, -1)
    b, e = divmod(c, 256)
    if qt == 12:
        blk[:, b, 2:4] = 0
        g, within = divmod(e, 64)
        i = 16 + 32 * g + within % 32
        blk[:, b, i] &= np.uint8(0xF0 if within < 32 else 0x0F)
    else:
        h, e2 = divmod(e, 128)
        r, l = divmod(e2, 32)
        i = 64 * h + l + 32 * (r & 1)
        blk[:, b, i] &= np.uint8(0xF0 if r < 2 else 0x0F)
        j = 128 + 32 * h + l
        blk[:, b, j] = (blk[:, b, j] & np.uint8(0xFF ^ (3 << (2 * r)))) | np.uint8(2 << (2 * r))


@pytest.mark.parametrize("qt", [12, 14])
@pytest.mark.parametrize("T,cols", [(1, 2048), (3, 2048), (1, 4096), (6, 4096), (8, 512)])
def test_matvec_outlier_groups(cuda, orc, qt, T, cols):
    """Massive activations (3e4, -2e4 among N(0,1) values) in two columns of
    one 32-value group, which every row weights by zero: the output is made
    of the other values only -- the 30 that share the outliers' quantisation
    group included -- so their precision is what the check sees.  (One int16
    level per group would leave those 30 values ~5 bits; the group's second
    level restores them.)  Plus a group of tiny values in the last token."""
    rng = np.random.default_rng(41 + qt + 10 * T + cols)
    rows = 256
    w = B.matrix(qt, rng, rows, cols)
    c1, c2 = 32 * 5 + 17, 32 * 5 + 3
    _zero_column(w, qt, rows, cols, c1)
    _zero_column(w, qt, rows, cols, c2)
    wf = orc.dequant(w, qt, rows * cols // 256).reshape(rows, cols)
    assert np.all(wf[:, [c1, c2]] == 0) and np.count_nonzero(wf[:, 32 * 5:32 * 6]) > rows * 20
    x = rng.standard_normal((T, cols)).astype(np.float32)
    x[:, c1] = 3e4
    x[:, c2] = -2e4
    x[-1, 64:96] = 1e-30
    y = bb.matvec_f32(dev(w, cuda), dev(x[0] if T == 1 else x, cuda), rows, cols, qt).cpu().numpy().reshape(T, rows)
    ref = orc.matvec_f64(w, qt, x, rows, cols).reshape(T, rows)
    for t in range(T):
        assert orc.rel_l2(y[t], ref[t]) < TOL
    # the fp16 drop-in (fp16 x and y): within its output rounding
    xh = x[0].astype(np.float16)
    yh = torch.empty(rows, dtype=torch.float16, device=cuda)
    bb.matvec(dev(w, cuda), dev(xh, cuda), yh, rows, cols, qt)
    assert orc.rel_l2(yh.float().cpu().numpy(), orc.matvec_f64(w, qt, xh.astype(np.float32), rows, cols)) < 2e-3


@pytest.mark.parametrize("qt,rows,cols", [(12, 512, 2048), (14, 2048, 512), (12, 33, 512)])
def test_matvec_unaligned_weights(cuda, orc, qt, rows, cols):
    """Weights at a 2-byte offset take the alignment-agnostic path."""
    rng = np.random.default_rng(11)
    w = B.matrix(qt, rng, rows, cols)
    buf = torch.zeros(w.size + 16, dtype=torch.uint8, device=cuda)
    buf[2:2 + w.size] = dev(w, cuda)
    x = rng.standard_normal(cols).astype(np.float32)
    y = torch.empty(rows, dtype=torch.float32, device=cuda)
    bb.check(bb.lib().bread_matvec_f32(bb._p(buf.data_ptr() + 2), bb._p(dev(x, cuda)), bb._p(y), rows, cols, qt,
                                       bb._s(None)), "matvec")
    assert orc.rel_l2(y.cpu().numpy(), orc.matvec_f64(w, qt, x, rows, cols)) < TOL


@pytest.mark.parametrize("qt,rows,cols", [(12, 512, 2048), (14, 2048, 512), (12, 8, 256)])
def test_matvec_f16_dropin(cuda, orc, qt, rows, cols):
    """bread_matvec (kernels.cu:289): fp16 x, fp16 y."""
    rng = np.random.default_rng(21)
    w = B.matrix(qt, rng, rows, cols)
    xh = rng.standard_normal(cols).astype(np.float16)
    y = torch.empty(rows, dtype=torch.float16, device=cuda)
    bb.matvec(dev(w, cuda), dev(xh, cuda), y, rows, cols, qt)
    ref = orc.matvec_f64(w, qt, xh.astype(np.float32), rows, cols)
    # fp16 output rounding alone is ~2.9e-4 relative (rms)
    assert orc.rel_l2(y.float().cpu().numpy(), ref) < 2e-3


def test_matvec_kat_selftest(cuda):
    """The reference self-test shape (kernels.cu:451-579): 8 rows x 1 block, x = 1."""
    x = torch.ones(256, dtype=torch.float16, device=cuda)
    for blk, qt, exp in ((B.kat_q4k_block(), 12, 1792.0), (B.kat_q6k_block(), 14, 2048.0)):
        y = torch.empty(8, dtype=torch.float16, device=cuda)
        bb.matvec(dev(np.tile(blk, 8), cuda), x, y, 8, 256, qt)
        assert torch.all(y.float() == exp)


@pytest.mark.parametrize("T", [2, 5, 8, 16])
@pytest.mark.parametrize("qt,rows,cols", [(12, 512, 2048), (14, 2048, 512)])
def test_matvec_batch(cuda, orc, T, qt, rows, cols):
    rng = np.random.default_rng(T)
    w = B.matrix(qt, rng, rows, cols)
    x = rng.standard_normal((T, cols)).astype(np.float32)
    y = bb.matvec_f32(dev(w, cuda), dev(x, cuda), rows, cols, qt).cpu().numpy()
    ref = orc.matvec_f64(w, qt, x, rows, cols)
    for t in range(T):
        assert orc.rel_l2(y[t], ref[t]) < TOL


def test_lm_head_q6k_full_size(cuda, orc):
    """Config 2's 248320 x 2048 Q6_K output head (417 MB): synthetic weights on
    the device; 512 random rows checked against the oracle, plus linearity of
    the whole product."""
    rows, cols = 248320, 2048
    nb = rows * cols // 256
    w = bb.synth_blocks(nb, 14, 99, 1, device=cuda)
    rng = np.random.default_rng(4)
    x1 = rng.standard_normal(cols).astype(np.float32)
    x2 = rng.standard_normal(cols).astype(np.float32)
    y1 = bb.matvec_f32(w, dev(x1, cuda), rows, cols, 14)
    y2 = bb.matvec_f32(w, dev(x2, cuda), rows, cols, 14)
    y12 = bb.matvec_f32(w, dev(x1 + 2 * x2, cuda), rows, cols, 14)
    torch.cuda.synchronize()
    lin = (y12 - (y1 + 2 * y2)).norm() / y12.norm()
    assert lin.item() < 2 * TOL
    pick = np.sort(rng.choice(rows, 512, replace=False))
    rb = 8 * 210
    wr = w.view(rows, rb)[torch.from_numpy(pick).to(cuda)].cpu().numpy().reshape(-1)
    ref = orc.matvec_f64(wr, 14, x1, 512, cols)
    assert orc.rel_l2(y1.cpu().numpy()[pick], ref) < TOL


# ---- f1: lm head + greedy sample on the device ------------------------------
def _expected_token(orc, ref64, gpu_logits, round_half):
    """The oracle's greedy token (fp64 logits), accepting any row whose logit is
    within fp32-summation noise of the top (then the GPU's own order decides)."""
    top = float(ref64.max())
    tol = 1e-4 * max(1.0, abs(top)) + (abs(top) * 2.0 ** -10 if round_half else 0.0)
    return set(np.nonzero(ref64 >= top - tol)[0].tolist())


@pytest.mark.parametrize("qt,rows,cols", [(14, 8192, 2048), (12, 4097, 512), (12, 3000, 2048), (8, 1000, 1024)])
@pytest.mark.parametrize("round_half", [1, 0])
def test_lm_head_argmax(cuda, orc, qt, rows, cols, round_half):
    """bread_lm_head_argmax against the oracle's logits and against its own
    logits output (which must be bit-equal to bread_matvec_f32's).  4097 rows
    of Q4_K with cols=512 run a fast launch plus a generic tail launch; Q8_0 the
    generic kernel only.  Two calls in a row share the state."""
    rng = np.random.default_rng(rows + qt)
    w = B.matrix(qt, rng, rows, cols)
    wd = dev(w, cuda)
    state = torch.zeros(2, dtype=torch.int64, device=cuda)
    for call in range(2):
        x = rng.standard_normal(cols).astype(np.float32)
        xd = dev(x, cuda)
        logits = torch.empty(rows, device=cuda)
        tok, val = bb.lm_head_argmax(wd, xd, rows, cols, qt, round_half=bool(round_half), state=state, logits=logits)
        y = bb.matvec_f32(wd, xd, rows, cols, qt)
        torch.cuda.synchronize()
        assert torch.equal(logits, y), "fused logits differ from bread_matvec_f32"
        yl = y.cpu().numpy()
        cmp = yl.astype(np.float16).astype(np.float32) if round_half else yl
        assert int(tok.item()) == int(np.argmax(cmp)), f"call {call}"  # np.argmax: first of the maxima
        assert float(val.item()) == float(cmp.max())
        assert int(tok.item()) in _expected_token(orc, orc.matvec_f64(w, qt, x, rows, cols), yl, round_half)
        assert torch.all(state == 0), "state re-zeroed for the next call"


def test_lm_head_argmax_ties_lowest_row(cuda):
    """Identical top rows: the lowest index wins (greedy_sample's strict `>`)."""
    rng = np.random.default_rng(5)
    rows, cols = 2048, 2048
    w = B.matrix(14, rng, rows, cols).reshape(rows, -1)
    x = rng.standard_normal(cols).astype(np.float32)
    y = bb.matvec_f32(dev(w.reshape(-1), cuda), dev(x, cuda), rows, cols, 14).cpu().numpy()
    top = int(np.argmax(y))
    for r in (1500, 777, 1999):
        w[r] = w[top]
    tok, _ = bb.lm_head_argmax(dev(w.reshape(-1), cuda), dev(x, cuda), rows, cols, 14, round_half=False)
    torch.cuda.synchronize()
    assert int(tok.item()) == min(top, 777)


def test_lm_head_argmax_full_head(cuda, orc):
    """Config 2's 248320 x 2048 Q6_K output head: the fused argmax equals the
    first maximum of the GPU's own logits and is the oracle's top token up to
    fp32 noise."""
    rows, cols = 248320, 2048
    w = bb.synth_blocks(rows * cols // 256, 14, 99, 1, device=cuda)
    x = bb.synth_normal(cols, 1.0, 99, 2, device=cuda)
    tok, val = bb.lm_head_argmax(w, x, rows, cols, 14, round_half=True)
    y = bb.matvec_f32(w, x, rows, cols, 14)
    torch.cuda.synchronize()
    yh = y.half().float().cpu().numpy()
    assert int(tok.item()) == int(np.argmax(yh)) and float(val.item()) == float(yh.max())
    ref = orc.matvec_f64(w.cpu().numpy(), 14, x.cpu().numpy(), rows, cols)
    assert int(tok.item()) in _expected_token(orc, ref, y.cpu().numpy(), True)


# ---- f4: the attention / SSM projection GEMVs of one_layer_forward ----------
# (rows, cols, qtype) as one_layer.cu calls bread_matvec with the model's
# dimensions (bread.h:32-52): q_proj 8192 x 2048 and k/v_proj 512 x 2048
# (:1527-1532), SSM qkv 8192 x 2048, z 4096 x 2048, alpha/beta 32 x 2048
# (:1639-1646), o_proj and ssm_out 2048 x 4096 (:1763, :1784).
PROJ = [(12, 8192, 2048), (12, 512, 2048), (14, 512, 2048), (12, 4096, 2048), (12, 32, 2048), (12, 2048, 4096)]


@pytest.mark.parametrize("qt,rows,cols", PROJ)
def test_projection_shapes(cuda, orc, qt, rows, cols):
    rng = np.random.default_rng(rows ^ cols ^ qt)
    w = B.matrix(qt, rng, rows, cols)
    wd = dev(w, cuda)
    x = rng.standard_normal(cols).astype(np.float32)
    y = bb.matvec_f32(wd, dev(x, cuda), rows, cols, qt).cpu().numpy()
    assert orc.rel_l2(y, orc.matvec_f64(w, qt, x, rows, cols)) < TOL
    # the fp16 form the reference calls (d_normed half in, half out)
    xh = x.astype(np.float16)
    yh = torch.empty(rows, dtype=torch.float16, device=cuda)
    bb.matvec(wd, dev(xh, cuda), yh, rows, cols, qt)
    ref = orc.matvec_f64(w, qt, xh.astype(np.float32), rows, cols)
    assert orc.rel_l2(yh.float().cpu().numpy(), ref) < TOL
