"""GPU: the fp16 launchers of layer_logic.cu:28-31 against a torch fp32
reference of the same operation (one_layer.cu:158-218 semantics)."""
import pytest
import torch

import breadv2_b200 as bb

pytestmark = pytest.mark.gpu


def ulp_close(a, b, ulps=1):
    a, b = a.float(), b.float()
    tol = ulps * torch.clamp(b.abs(), min=6.1e-5) * 2.0 ** -10
    return bool(torch.all((a - b).abs() <= tol))


def test_silu_mul(cuda):
    g = (torch.randn(4096, device=cuda) * 4).half()
    u = (torch.randn(4096, device=cuda) * 4).half()
    ref = (g.float() / (1 + torch.exp(-g.float())) * u.float()).half()
    out = g.clone()
    bb.silu_mul(out, u)
    assert ulp_close(out, ref)


def test_scale_accum(cuda):
    d = torch.randn(2048, device=cuda).half()
    s = torch.randn(2048, device=cuda).half()
    # fused multiply-add as the kernel (and the reference's nvcc build): one fp32
    # rounding of the exact d + c*s (exact in fp64), then fp16
    c = torch.tensor(0.37, dtype=torch.float32).double()
    ref = (d.double() + c * s.double()).float().half()
    out = d.clone()
    bb.scale_accum(out, s, 0.37)
    assert ulp_close(out, ref)


def test_rmsnorm_half(cuda):
    x = (torch.randn(2048, device=cuda) * 3).half()
    w = torch.rand(2048, device=cuda) + 0.5
    xf = x.float()
    ref = (xf * torch.rsqrt((xf * xf).mean() + 1e-6) * w).half()
    out = x.clone()
    bb.rmsnorm_half(out, w, 1e-6)
    assert ulp_close(out, ref, ulps=2)


def test_copy_half(cuda):
    x = torch.randn(3000, device=cuda).half()
    y = torch.empty_like(x)
    bb.copy_half(y, x)
    assert torch.equal(x, y)
