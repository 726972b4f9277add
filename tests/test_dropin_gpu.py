"""GPU: the C++-linkage drop-ins executed through the symbols the reference's
callers link against (the mangled names of kernels.cu:289 `bread_matvec` and
of the four launchers layer_logic.cu:28-31 declares), not through the
status-returning C forms.  Checked against the oracle (GEMV) and a torch fp32
restatement of one_layer.cu:158-218 (glue launchers)."""
import ctypes

import numpy as np
import pytest
import torch

import breadv2_b200 as bb
from breadv2_b200 import _lib
from oracle import blocks as B

pytestmark = pytest.mark.gpu
P = ctypes.c_void_p


def _sym(name):
    fn = getattr(bb.lib(), _lib.MANGLED[name])
    fn.restype = None
    return fn


def _ulp_close(a, b, ulps):
    a, b = a.float(), b.float()
    return bool(torch.all((a - b).abs() <= ulps * torch.clamp(b.abs(), min=6.1e-5) * 2.0 ** -10))


@pytest.mark.parametrize("qt,rows,cols", [(12, 512, 2048), (14, 2048, 512), (8, 300, 1024), (14, 1000, 4096)])
def test_mangled_bread_matvec(cuda, orc, qt, rows, cols):
    """bread_matvec(void*, half*, half*, int, int, int, cudaStream_t), fp16 x
    and y: rel-L2 <= 1e-3 against the fp64 product of the exactly decoded
    weights with the fp16-rounded x (the fp16 output alone costs ~3e-4)."""
    rng = np.random.default_rng(rows + cols + qt)
    w = B.matrix(qt, rng, rows, cols)
    xh = rng.standard_normal(cols).astype(np.float16)
    wd = torch.from_numpy(w).to(cuda)
    xd = torch.from_numpy(xh).to(cuda)
    yd = torch.full((rows,), float("nan"), dtype=torch.float16, device=cuda)
    s = torch.cuda.current_stream()
    _sym("bread_matvec")(P(wd.data_ptr()), P(xd.data_ptr()), P(yd.data_ptr()), rows, cols, qt, P(s.cuda_stream))
    torch.cuda.synchronize()
    ref = orc.matvec_f64(w, qt, xh.astype(np.float32), rows, cols)
    assert orc.rel_l2(yd.float().cpu().numpy(), ref) < 1e-3
    assert bb.device_error() == 0


def test_mangled_glue_launchers(cuda):
    s = P(torch.cuda.current_stream().cuda_stream)
    g = (torch.randn(4096, device=cuda) * 4).half()
    u = (torch.randn(4096, device=cuda) * 4).half()
    ref = (g.float() / (1 + torch.exp(-g.float())) * u.float()).half()
    out = g.clone()
    _sym("bread_silu_mul")(P(out.data_ptr()), P(u.data_ptr()), 4096, s)
    torch.cuda.synchronize()
    assert _ulp_close(out, ref, 1)

    d = torch.randn(2048, device=cuda).half()
    src = torch.randn(2048, device=cuda).half()
    # the kernel (like the reference's nvcc build) fuses the multiply-add: one
    # fp32 rounding of the exact d + c*s (exact in fp64), then fp16
    c = torch.tensor(0.37, dtype=torch.float32).double()
    ref = (d.double() + c * src.double()).float().half()
    out = d.clone()
    _sym("bread_scale_accum")(P(out.data_ptr()), P(src.data_ptr()), ctypes.c_float(0.37), 2048, s)
    torch.cuda.synchronize()
    assert _ulp_close(out, ref, 1)

    x = (torch.randn(2048, device=cuda) * 3).half()
    wn = torch.rand(2048, device=cuda) + 0.5
    xf = x.float()
    ref = (xf * torch.rsqrt((xf * xf).mean() + 1e-6) * wn).half()
    out = x.clone()
    _sym("bread_rmsnorm_half")(P(out.data_ptr()), P(wn.data_ptr()), 2048, ctypes.c_float(1e-6), s)
    torch.cuda.synchronize()
    assert _ulp_close(out, ref, 2)

    y = torch.empty(3000, dtype=torch.float16, device=cuda)
    x = torch.randn(3000, device=cuda).half()
    _sym("bread_copy_half")(P(y.data_ptr()), P(x.data_ptr()), 3000, s)
    torch.cuda.synchronize()
    assert torch.equal(x, y)
