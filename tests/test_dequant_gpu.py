"""GPU: bread_dequant is bit-exact against the oracle (the reference CPU
decoders, layer_ops.cu:44-105) on seeded blocks of every edge-case mode and on
the golden fixtures of the reference's own code."""
import numpy as np
import pytest
import torch

import breadv2_b200 as bb
from oracle import blocks as B

pytestmark = pytest.mark.gpu


def bits(a):
    return np.asarray(a, dtype=np.float32).view(np.uint32)


@pytest.mark.parametrize("qt", [12, 14])
@pytest.mark.parametrize("mode", ["baseline", "subnormal", "zero_scale", "large", "mixed"])
def test_dequant_bitexact(cuda, orc, qt, mode):
    rng = np.random.default_rng(100 + qt)
    n = 4096
    w = (B.q4k_blocks if qt == 12 else B.q6k_blocks)(rng, n, mode).reshape(-1)
    out = bb.dequant(torch.from_numpy(w).to(cuda), n, qt).cpu().numpy()
    assert np.array_equal(bits(out), bits(orc.dequant(w, qt, n)))


def test_dequant_q8_0(cuda, orc):
    rng = np.random.default_rng(5)
    w = B.q8_0_blocks(rng, 1000).reshape(-1)
    out = bb.dequant(torch.from_numpy(w).to(cuda), 1000, 8).cpu().numpy()
    assert np.array_equal(bits(out), bits(orc.dequant(w, 8, 1000)))


@pytest.mark.parametrize("name,qt", [("q4k", 12), ("q6k", 14)])
def test_dequant_golden(cuda, golden, name, qt):
    g = golden["dequant"]
    blk = g[f"{name}_blocks"]
    n = blk.shape[0]
    out = bb.dequant(torch.from_numpy(blk.reshape(-1).copy()).to(cuda), n, qt).cpu().numpy()
    # exact fp16 decode (layer_ops.cu): every block
    assert np.array_equal(bits(out), bits(g[f"{name}_exact"]))
    # flush-to-zero decode (dequant_q4k_cpu.c): every block whose scales are normal or zero
    ftz = g[f"{name}_ftz"].reshape(n, 256)
    same = np.all(bits(out.reshape(n, 256)) == bits(ftz), axis=1)
    hdr = blk[:, 0:4] if qt == 12 else blk[:, 208:210]
    h16 = hdr.copy().view(np.uint16).reshape(n, -1)
    sub = np.any(((h16 >> 10) & 31 == 0) & (h16 & 0x3FF != 0), axis=1)
    assert np.all(same | sub)


def test_dequant_kat(cuda):
    out = bb.dequant(torch.from_numpy(B.kat_q4k_block()).to(cuda), 1, 12).cpu().numpy()
    assert np.array_equal(out[:64], np.r_[np.full(32, 9.0), np.full(32, 5.0)].astype(np.float32))
    out = bb.dequant(torch.from_numpy(B.kat_q6k_block()).to(cuda), 1, 14).cpu().numpy()
    assert np.all(out == 8.0)


def test_dequant_unaligned_and_empty(cuda, orc):
    rng = np.random.default_rng(9)
    w = B.q6k_blocks(rng, 33).reshape(-1)
    buf = torch.zeros(w.size + 3, dtype=torch.uint8, device=cuda)
    buf[1:1 + w.size] = torch.from_numpy(w).to(cuda)
    out = torch.empty(33 * 256, dtype=torch.float32, device=cuda)
    bb.check(bb.lib().bread_dequant(bb._p(buf.data_ptr() + 1), bb._p(out), 33, 14, bb._s(None)), "dequant")
    assert np.array_equal(bits(out.cpu().numpy()), bits(orc.dequant(w, 14, 33)))
    bb.check(bb.lib().bread_dequant(bb._p(buf), bb._p(out), 0, 14, bb._s(None)), "dequant empty")
