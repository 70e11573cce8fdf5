"""Plugin heads on CUDA (gated attention, XSA, Canon) against fp32 PyTorch expressions of the same ops."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("per_head", [False, True])
def test_gate_mul(per_head):
    from nexttransformer_b200.ops.plugins import gate_mul
    torch.manual_seed(0)
    B, T, H, D = 2, 77, 6, 128
    y = torch.randn(B, T, H, D, device="cuda").bfloat16().requires_grad_()
    g = (torch.randn(B, T, H, 1 if per_head else D, device="cuda") * 2).bfloat16().requires_grad_()
    z = gate_mul(y, g)
    dz = torch.randn_like(z)
    z.backward(dz)
    yr, gr = (t.detach().float().requires_grad_() for t in (y, g))
    zr = yr * torch.sigmoid(gr)
    zr.backward(dz.float())
    torch.testing.assert_close(z.float(), zr, rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(y.grad.float(), yr.grad, rtol=1e-2, atol=1e-2)
    assert _rel(g.grad, gr.grad) < 1e-2


@pytest.mark.parametrize("H,Hk", [(4, 4), (6, 2)])
def test_exclusive_projection(H, Hk):
    from nexttransformer_b200.methods.xsa import exclusive_projection as reference
    from nexttransformer_b200.ops.plugins import exclusive_projection
    torch.manual_seed(1)
    B, T, D = 2, 50, 128
    y = torch.randn(B, T, H, D, device="cuda").bfloat16().requires_grad_()
    v = torch.randn(B, T, Hk, D, device="cuda")
    v[0, 3] = 0.0  # a zero value: u = 0 (F.normalize's clamp)
    v = v.bfloat16().requires_grad_()
    z = exclusive_projection(y, v)
    dz = torch.randn_like(z)
    z.backward(dz)
    yr, vr = (t.detach().float().requires_grad_() for t in (y, v))
    zr = reference(yr, vr.repeat_interleave(H // Hk, dim=2))
    zr.backward(dz.float())
    torch.testing.assert_close(z.float(), zr, rtol=1e-2, atol=2e-2)
    assert _rel(y.grad, yr.grad) < 1e-2
    assert _rel(v.grad, vr.grad) < 1e-2


@pytest.mark.parametrize("C,T", [(256, 100), (1024, 33)])
def test_canon(C, T):
    from nexttransformer_b200.ops.plugins import canon
    torch.manual_seed(2)
    B, K = 2, 4
    x = torch.randn(B, T, C, device="cuda").bfloat16().requires_grad_()
    w = (torch.randn(C, 1, K, device="cuda") * 0.3).requires_grad_()
    y = canon(x, w)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().clone().requires_grad_()
    yr = xr + F.conv1d(F.pad(xr.transpose(1, 2), (K - 1, 0)), wr, groups=C).transpose(1, 2)
    yr.backward(dy.float())
    torch.testing.assert_close(y.float(), yr, rtol=1e-2, atol=2e-2)
    assert _rel(x.grad, xr.grad) < 1e-2
    assert _rel(w.grad, wr.grad) < 1e-3


@pytest.mark.parametrize("method", ["gated_attention", "gated_attention_headwise", "xsa", "attnres_full_canon_abcd"])
def test_plugin_models_match_torch_path(method, monkeypatch):
    """A small model of each plugin on CUDA: loss and gradients with the kernels equal those with the
    PyTorch expressions of the same heads (both bf16), so the wiring is right."""
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.ops import plugins
    cfg = debug_config(method, width=256, sequence_len=64)
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randint(0, cfg.vocab_size, (2, cfg.sequence_len), device="cuda", generator=g)
    y = torch.randint(0, cfg.vocab_size, (2, cfg.sequence_len), device="cuda", generator=g)
    results = []
    for use_kernels in (True, False):
        if not use_kernels:
            monkeypatch.setattr(plugins, "supported", lambda *a, **k: False)
        model = build_model(cfg, "cuda", seed=3)
        gp = torch.Generator(device="cuda").manual_seed(7)
        with torch.no_grad():  # non-trivial plugin parameters (Canon taps start at zero)
            for n, p in model.named_parameters():
                if "canon" in n:
                    p.normal_(std=0.2, generator=gp)
        loss = model(x, y)
        loss.backward()
        results.append((loss.detach().float(), {n: p.grad.float().clone() for n, p in model.named_parameters()
                                                 if p.grad is not None}))
    (l1, g1), (l2, g2) = results
    assert abs(l1.item() - l2.item()) <= 1e-2 * abs(l2.item()), (l1.item(), l2.item())
    assert g1.keys() == g2.keys()
    for n in g2:
        if g2[n].norm() > 0:
            assert _rel(g1[n], g2[n]) < 5e-2, (n, _rel(g1[n], g2[n]))
