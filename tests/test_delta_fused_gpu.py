"""The fused chunked delta rule (chunk-term kernels + inter-chunk scan, bf16 inputs) against the
chunk form of ``models/linear.py`` evaluated in float64 on the same inputs: outputs within 1e-2 and
every gradient within 3e-2 in relative norm (the FLA numerics bar), plus an elementwise bound of
5 % of each tensor's largest entry."""
import pytest
import torch
import torch.nn.functional as F

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.double() - b.double()).norm() / b.double().norm().clamp_min(1e-30)).item()


def _inputs(kind, B, T, H, seed):
    D = 128
    g = torch.Generator(device="cuda").manual_seed(seed)
    q = torch.randn(B, T, H, D, device="cuda", generator=g)
    k = torch.randn(B, T, H, D, device="cuda", generator=g)
    v = torch.randn(B, T, H, D, device="cuda", generator=g)
    if kind != "gdn":
        q, k = F.normalize(q, dim=-1) * D ** -.5, F.normalize(k, dim=-1)
    beta = torch.rand(B, T, H, device="cuda", generator=g)
    gate = None
    if kind == "gdn":
        gate = -F.softplus(torch.randn(B, T, H, device="cuda", generator=g)) * 0.3
    elif kind == "kda":
        gate = -F.softplus(torch.randn(B, T, H, D, device="cuda", generator=g)) * 0.05
    return q.bfloat16(), k.bfloat16(), v.bfloat16(), beta, gate


@pytest.mark.parametrize("kind,B,T,H", [("gdn", 2, 200, 3), ("kda", 2, 256, 2), ("deltanet", 1, 192, 3),
                                        ("gdn", 1, 1024, 2), ("kda", 1, 700, 1)])
def test_fused_delta_chunk_matches_fp64(kind, B, T, H, monkeypatch):
    import nexttransformer_b200.ops.linear_attention as LA
    monkeypatch.setattr(LA, "FUSED_DELTA", True)
    from nexttransformer_b200.models.linear import chunk_scan
    from nexttransformer_b200.ops._ext import check_errors
    from nexttransformer_b200.ops.linear_attention import delta_chunk_cuda, fused_chunk_supported
    D = 128
    q, k, v, beta, gate = _inputs(kind, B, T, H, seed=T + H)
    assert fused_chunk_supported(q, k, v, 64)
    scale = D ** -.5 if kind == "gdn" else None
    leaves = [t.clone().requires_grad_() for t in (q, k, v, beta)] + ([gate.clone().requires_grad_()] if gate is not None else [])
    y = delta_chunk_cuda(*leaves[:3], kind=kind, g=leaves[4] if gate is not None else None, beta=leaves[3], chunk=64,
                         qk_l2norm_scale=scale)
    assert "DeltaChunk" in type(y.grad_fn).__name__ or "DeltaChunk" in str(y.grad_fn.next_functions)
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    torch.cuda.synchronize()
    check_errors()
    ref = [t.detach().double().requires_grad_() for t in (q, k, v, beta)]
    if gate is not None:
        ref.append(gate.detach().double().requires_grad_())
    qr, kr = ref[0], ref[1]
    if scale is not None:
        qr, kr = F.normalize(qr, dim=-1) * scale, F.normalize(kr, dim=-1)
    yr = chunk_scan(qr, kr, ref[2], kind=kind, g=ref[4] if gate is not None else None, beta=ref[3], chunk=64)
    yr.backward(dy.double())
    assert _rel(y, yr) < 1e-2, _rel(y, yr)
    for name, a, b in zip(("q", "k", "v", "beta", "g"), leaves, ref):
        err = _rel(a.grad, b.grad)
        assert err < 3e-2, (name, err)
        worst = (a.grad.double() - b.grad).abs().max().item()
        assert worst <= 5e-2 * b.grad.abs().max().item(), (name, worst)


def test_gla_chunk_kernels_match_recurrence():
    """GLA through the chunk form on the scan kernels equals the token recurrence (fp64 oracle)."""
    import torch.nn.functional as F
    from nexttransformer_b200.models.linear import recurrent_scan
    from nexttransformer_b200.ops.linear_attention import gla_chunk_cuda
    g = torch.Generator(device="cuda").manual_seed(3)
    B, T, H, D = 2, 200, 3, 128
    q = (torch.randn(B, T, H, D, device="cuda", generator=g) * D ** -.5).requires_grad_()
    k = torch.randn(B, T, H, D, device="cuda", generator=g).requires_grad_()
    v = torch.randn(B, T, H, D, device="cuda", generator=g).requires_grad_()
    gate = torch.randn(B, T, H, D, device="cuda", generator=g).requires_grad_()
    logd = F.logsigmoid(gate) / 16
    y = gla_chunk_cuda(q, k, v, logd)
    dy = torch.randn_like(y)
    grads = torch.autograd.grad(y, (q, k, v, gate), dy)
    leaves = [x.detach().double().requires_grad_() for x in (q, k, v, gate)]
    ref, _ = recurrent_scan(leaves[0], leaves[1], leaves[2], kind="gla",
                            decay=(F.logsigmoid(leaves[3]) / 16).exp())
    rgrads = torch.autograd.grad(ref, leaves, dy.double())
    assert ((y.double() - ref).norm() / ref.norm()) < 1e-2
    for a, r in zip(grads, rgrads):
        assert ((a.double() - r).norm() / r.norm()) < 3e-2


@pytest.mark.parametrize("B,T,H,norm", [(2, 256, 2, True), (1, 700, 3, True), (1, 320, 2, False)])
def test_kda_gate_from_preactivation_matches_fp64(B, T, H, norm):
    """KDA with the gate formed in the kernel, g = -exp(g_log) softplus(g_raw + g_bias), and the q / k
    normalisation there too, against the fp64 chunk form of the same expression."""
    from nexttransformer_b200.models.linear import chunk_scan
    from nexttransformer_b200.ops._ext import check_errors
    from nexttransformer_b200.ops.linear_attention import kda_chunk_cuda
    D = 128
    g = torch.Generator(device="cuda").manual_seed(T + H)
    q = torch.randn(B, T, H, D, device="cuda", generator=g)
    k = torch.randn(B, T, H, D, device="cuda", generator=g)
    if not norm:
        q, k = F.normalize(q, dim=-1) * D ** -.5, F.normalize(k, dim=-1)
    v = torch.randn(B, T, H, D, device="cuda", generator=g)
    raw = torch.randn(B, T, H, D, device="cuda", generator=g)
    beta = torch.rand(B, T, H, device="cuda", generator=g)
    g_log = (torch.randn(H, D, device="cuda", generator=g) * 0.5 - 1.0)
    g_bias = torch.full((H, D), -3.0, device="cuda") + torch.randn(H, D, device="cuda", generator=g)
    q, k, v, raw = (t.bfloat16() for t in (q, k, v, raw))
    leaves = [t.clone().requires_grad_() for t in (q, k, v, raw, g_log, g_bias, beta)]
    y = kda_chunk_cuda(leaves[0], leaves[1], leaves[2], leaves[3], leaves[4], leaves[5], leaves[6],
                       qk_l2norm_scale=D ** -.5 if norm else None)
    assert "KdaChunk" in type(y.grad_fn).__name__
    dy = torch.randn_like(y.float())
    y.float().backward(dy)
    torch.cuda.synchronize()
    check_errors()
    ref = [t.detach().double().requires_grad_() for t in (q, k, v, raw, g_log, g_bias, beta)]
    qr, kr = ref[0], ref[1]
    if norm:
        qr, kr = F.normalize(qr, dim=-1) * D ** -.5, F.normalize(kr, dim=-1)
    decay = -ref[4].exp() * F.softplus(ref[3] + ref[5])
    yr = chunk_scan(qr, kr, ref[2], kind="kda", g=decay, beta=ref[6], chunk=64)
    yr.backward(dy.double())
    assert _rel(y, yr) < 1e-2, _rel(y, yr)
    for name, a, b in zip(("q", "k", "v", "g_raw", "g_log", "g_bias", "beta"), leaves, ref):
        err = _rel(a.grad, b.grad)
        assert err < 3e-2, (name, err)
        worst = (a.grad.double() - b.grad).abs().max().item()
        assert worst <= 5e-2 * b.grad.abs().max().item(), (name, worst)
