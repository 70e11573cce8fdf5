"""MSAR kernels (temporal augmentation, depth-read gate) against the torch modules on the GPU."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _both(module, x, monkeypatch, dout):
    from nexttransformer_b200.ops import msar as K
    outs = []
    for fused in (True, False):
        if not fused:
            monkeypatch.setattr(K, "supported", lambda t: False)
        module.zero_grad()
        xi = x.detach().clone().requires_grad_()
        y = module(xi)
        y.backward(dout)
        outs.append((y.detach().float(), xi.grad.float(), [p.grad.float().clone() if p.grad is not None else torch.zeros_like(p, dtype=torch.float32)
                                                            for p in module.parameters()]))
    return outs


@pytest.mark.parametrize("dtype,T", [(torch.float32, 100), (torch.bfloat16, 300), (torch.float32, 5)])
def test_temporal(dtype, T, monkeypatch):
    from nexttransformer_b200.methods.msar.ops import TemporalAugmentation
    torch.manual_seed(0)
    C = 192
    m = TemporalAugmentation(C).cuda()
    with torch.no_grad():
        for t in m.taps:
            t.normal_(std=0.3)
    x = torch.randn(2, T, C, device="cuda", dtype=dtype)
    dout = torch.randn(2, T, 4, C, device="cuda", dtype=dtype)
    (y, dx, dp), (ry, rdx, rdp) = _both(m, x, monkeypatch, dout)
    tol = dict(rtol=1e-4, atol=1e-4) if dtype == torch.float32 else dict(rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(y, ry, **tol)
    torch.testing.assert_close(dx, rdx, **tol)
    for a, b in zip(dp, rdp):
        assert ((a - b).norm() / b.norm()) < (1e-4 if dtype == torch.float32 else 2e-2)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_depth_read(dtype, monkeypatch):
    from nexttransformer_b200.methods.msar.ops import DepthRead
    torch.manual_seed(1)
    C = 256
    m = DepthRead(C).cuda()
    with torch.no_grad():
        m.query.normal_()
        m.alpha_pre.fill_(0.7)
        m.bias_pre.normal_(std=0.5)
    x = torch.randn(3, 50, 4, C, device="cuda", dtype=dtype)
    x[0, 3] = 0          # an all-zero token (rms 1)
    dout = torch.randn(3, 50, C, device="cuda", dtype=dtype)
    (y, dx, dp), (ry, rdx, rdp) = _both(m, x, monkeypatch, dout)
    tol = dict(rtol=2e-4, atol=2e-4) if dtype == torch.float32 else dict(rtol=3e-2, atol=3e-2)
    torch.testing.assert_close(y, ry, **tol)
    torch.testing.assert_close(dx, rdx, **tol)
    names = [n for n, _ in m.named_parameters()]
    for n, a, b in zip(names, dp, rdp):
        if n == "query":
            continue                      # the gate does not use the query
        assert ((a - b).norm() / b.norm().clamp_min(1e-12)) < (2e-4 if dtype == torch.float32 else 3e-2), n
