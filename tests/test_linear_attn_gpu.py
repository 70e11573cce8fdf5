"""sm_100a linear-attention kernels against fp32 PyTorch references of the same ops."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _conv_ref(x, w):
    y = F.conv1d(F.pad(x.transpose(1, 2), (w.shape[-1] - 1, 0)), w, groups=x.shape[-1])
    return F.silu(y.transpose(1, 2))


@pytest.mark.parametrize("B,T,C,K", [(2, 77, 64, 4), (1, 300, 1280, 4), (3, 5, 24, 3), (2, 130, 256, 2)])
def test_causal_conv_silu(B, T, C, K):
    from nexttransformer_b200.ops.linear_attention import causal_conv_silu
    torch.manual_seed(0)
    x = torch.randn(B, T, C, device="cuda").to(torch.bfloat16).requires_grad_()
    w = (torch.randn(C, 1, K, device="cuda") * K ** -.5).requires_grad_()
    y = causal_conv_silu(x, w)
    dy = torch.randn_like(y)
    y.backward(dy)
    xr, wr = x.detach().float().requires_grad_(), w.detach().clone().requires_grad_()
    yr = _conv_ref(xr, wr)
    yr.backward(dy.float())
    torch.testing.assert_close(y.float(), yr, atol=2e-2, rtol=2e-2)
    torch.testing.assert_close(x.grad.float(), xr.grad, atol=3e-2, rtol=3e-2)
    torch.testing.assert_close(w.grad, wr.grad, atol=0.2, rtol=2e-2)


@pytest.mark.parametrize("rows,D", [(1, 128), (333, 128), (4096, 64)])
def test_gated_rmsnorm(rows, D):
    from nexttransformer_b200.ops.linear_attention import gated_rms_norm
    torch.manual_seed(1)
    y = torch.randn(rows, 3, D, device="cuda").to(torch.bfloat16).requires_grad_()
    g = torch.randn(rows, 3, D, device="cuda").to(torch.bfloat16).requires_grad_()
    gain = (1 + 0.1 * torch.randn(D, device="cuda")).requires_grad_()
    out = gated_rms_norm(y, g, gain)
    do = torch.randn_like(out)
    out.backward(do)
    yr, gr, gainr = (t.detach().float().requires_grad_() for t in (y, g, gain))
    ref = yr * torch.rsqrt(yr.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps) * gainr * F.silu(gr)
    ref.backward(do.float())
    torch.testing.assert_close(out.float(), ref, atol=3e-2, rtol=2e-2)
    torch.testing.assert_close(y.grad.float(), yr.grad, atol=5e-2, rtol=3e-2)
    torch.testing.assert_close(g.grad.float(), gr.grad, atol=5e-2, rtol=3e-2)
    torch.testing.assert_close(gain.grad, gainr.grad, atol=0.5, rtol=2e-2)


@pytest.mark.parametrize("kind", ["gdn", "kda", "deltanet"])
def test_linear_mixer_cuda_matches_cpu(kind):
    """The CUDA path of a chunked delta-rule model (conv, chunk scan, gated norm) against the CPU path."""
    from nexttransformer_b200.models import build_model
    from nexttransformer_b200.models.config import debug_config
    c = debug_config(kind, width=256, sequence_len=128)
    torch.manual_seed(2)
    tok = torch.randint(0, c.vocab_size, (2, 129))
    x, y = tok[:, :-1], tok[:, 1:]
    cpu = build_model(c, "cpu", seed=3)
    gpu = build_model(c, "cuda", seed=3)
    lc = cpu(x, y)
    lg = gpu(x.cuda(), y.cuda())
    lc.backward()
    lg.backward()
    assert abs(lc.item() - lg.item()) < 0.05
    for (n, pc), pg in zip(cpu.named_parameters(), gpu.parameters()):
        if pc.grad is None:
            continue
        rel = (pc.grad - pg.grad.float().cpu()).norm() / pc.grad.norm().clamp_min(1e-12)
        assert rel < 0.1, (n, rel.item())
