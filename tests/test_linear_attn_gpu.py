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


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("kind,T", [("gdn", 64), ("gdn", 300), ("kda", 256), ("deltanet", 192)])
def test_delta_chunk_scan_matches_fp32(kind, T):
    """The sm_100a chunk scan (bf16 operands, fp32 state) against the fp32 torch chunk form."""
    from nexttransformer_b200.models.linear import chunk_scan
    from nexttransformer_b200.ops.linear_attention import delta_chunk_cuda
    torch.manual_seed(4)
    B, H, D = 2, 3, 128
    q = torch.randn(B, T, H, D, device="cuda")
    k = torch.randn(B, T, H, D, device="cuda")
    v = torch.randn(B, T, H, D, device="cuda")
    if kind != "gdn":
        q, k = F.normalize(q, dim=-1), F.normalize(k, dim=-1)
    beta = torch.rand(B, T, H, device="cuda")
    g = None
    if kind == "gdn":
        g = -F.softplus(torch.randn(B, T, H, device="cuda")) * 0.2
    elif kind == "kda":
        g = -F.softplus(torch.randn(B, T, H, D, device="cuda")) * 0.05
    scale = D ** -.5 if kind == "gdn" else None
    leaves = [t.clone().requires_grad_() for t in (q, k, v, beta)] + ([g.clone().requires_grad_()] if g is not None else [])
    gl = leaves[4] if g is not None else None
    y = delta_chunk_cuda(*leaves[:3], kind=kind, g=gl, beta=leaves[3], chunk=64, qk_l2norm_scale=scale)
    dy = torch.randn_like(y)
    y.backward(dy)
    ref = [t.clone().requires_grad_() for t in (q, k, v, beta)] + ([g.clone().requires_grad_()] if g is not None else [])
    qr, kr = ref[0], ref[1]
    if scale is not None:
        qr, kr = F.normalize(qr, dim=-1) * scale, F.normalize(kr, dim=-1)
    torch.backends.cuda.matmul.allow_tf32 = False
    yr = chunk_scan(qr, kr, ref[2], kind=kind, g=ref[4] if g is not None else None, beta=ref[3], chunk=64)
    yr.backward(dy)
    assert _rel(y, yr) < 2e-2
    for a, b in zip(leaves, ref):
        assert _rel(a.grad, b.grad) < 5e-2


@pytest.mark.parametrize("T", [64, 200])
def test_retnet_chunk_scan_matches_fp32(T):
    """RetNet's scalar-decay chunk form on the scan kernels (w = 0) against the fp32 torch chunk form."""
    from nexttransformer_b200.models.linear import chunk_scan
    from nexttransformer_b200.ops.linear_attention import scalar_chunk_cuda
    torch.manual_seed(6)
    B, H, D = 2, 3, 128
    q = torch.randn(B, T, H, D, device="cuda") * D ** -.5
    k = torch.randn(B, T, H, D, device="cuda")
    v = torch.randn(B, T, H, D, device="cuda")
    gamma = 1 - 2. ** (-5 - torch.arange(H, device="cuda", dtype=torch.float32))
    g = gamma.log()[None, None].expand(B, T, H)
    leaves = [t.clone().requires_grad_() for t in (q, k, v)]
    y = scalar_chunk_cuda(*leaves, g, 64)
    dy = torch.randn_like(y)
    y.backward(dy)
    ref = [t.clone().requires_grad_() for t in (q, k, v)]
    torch.backends.cuda.matmul.allow_tf32 = False
    yr = chunk_scan(*ref, kind="retnet", g=g, chunk=64)
    yr.backward(dy)
    assert _rel(y, yr) < 2e-2
    for a, b in zip(leaves, ref):
        assert _rel(a.grad, b.grad) < 5e-2


@pytest.mark.parametrize("method", ["retnet", "gla"])
def test_scan_kernel_mixers_match_recurrence(method, monkeypatch):
    """RetNet and GLA models on CUDA: the chunk form on the scan kernels against the token recurrence
    of the same mixer (both bf16 activations), loss and every gradient."""
    import nexttransformer_b200.models.linear as L
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.lm import build_model
    cfg = debug_config(method, width=256, sequence_len=128)
    g = torch.Generator(device="cuda").manual_seed(0)
    x = torch.randint(0, cfg.vocab_size, (2, cfg.sequence_len), device="cuda", generator=g)
    y = torch.randint(0, cfg.vocab_size, (2, cfg.sequence_len), device="cuda", generator=g)
    res = []
    for kernels in (True, False):
        if not kernels:
            monkeypatch.setattr(L, "_gla_kernel_ok", lambda q, v: False)
        model = build_model(cfg, "cuda", seed=5)
        loss = model(x, y)
        loss.backward()
        res.append((loss.detach().float(), {n: p.grad.float().clone() for n, p in model.named_parameters()
                                             if p.grad is not None}))
    (l1, g1), (l2, g2) = res
    assert abs(l1.item() - l2.item()) <= 1e-2 * abs(l2.item()), (l1.item(), l2.item())
    for n in g2:
        if g2[n].norm() > 0:
            assert _rel(g1[n], g2[n]) < 5e-2, (n, _rel(g1[n], g2[n]))
