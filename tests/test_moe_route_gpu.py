"""Fused MoE routing kernels (csrc/moe_route.cu) against the unfused torch routing and plan."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _oracle(logits, bias, k):
    probs = logits.softmax(-1)
    choice = (probs + bias).topk(k, dim=-1).indices
    w = probs.gather(-1, choice)
    return choice, w / w.sum(-1, keepdim=True), probs


@pytest.mark.parametrize("N,E,k", [(4096, 64, 8), (1000, 32, 2), (777, 128, 6), (300, 256, 16)])
def test_route_plan_matches_torch(N, E, k):
    from nexttransformer_b200.ops._ext import ext
    from nexttransformer_b200.ops.moe import plan
    torch.manual_seed(0)
    logits = torch.randn(N, E, device="cuda") * 2
    bias = torch.randn(E, device="cuda") * 0.05
    load = torch.zeros(E, device="cuda")
    choice, w, lse, row_of, src_of, grp_m, grp_k, counts, aux_grad, aux = ext().moe_route(logits, bias, k, 0.01, 1e-3,
                                                                                          load)
    c_ref, w_ref, probs = _oracle(logits, bias, k)
    assert torch.equal(choice.long(), c_ref)
    torch.testing.assert_close(w, w_ref, rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(lse, torch.logsumexp(logits, -1), rtol=1e-5, atol=1e-5)
    ref = plan(c_ref, E)
    assert torch.equal(row_of, ref["row_of"]) and torch.equal(src_of, ref["src_of"])
    assert torch.equal(grp_m, ref["grp_m"]) and torch.equal(grp_k, ref["grp_k"])
    assert torch.equal(counts.long(), ref["counts"]) and torch.equal(load, ref["counts"].float())
    frac = ref["counts"].float() / (N * k)
    bal = 0.01 * E * (frac * probs.mean(0)).sum()
    z = 1e-3 * torch.logsumexp(logits, -1).square().mean()
    torch.testing.assert_close(aux, torch.stack((bal, z)), rtol=1e-4, atol=1e-7)
    torch.testing.assert_close(aux_grad, 0.01 * E * frac / N, rtol=1e-6, atol=0)


@pytest.mark.parametrize("E,k", [(64, 8), (32, 2), (256, 16)])
def test_route_backward_matches_autograd(E, k):
    from nexttransformer_b200.ops._ext import ext
    torch.manual_seed(1)
    N = 999
    logits = (torch.randn(N, E, device="cuda") * 2).requires_grad_()
    bias = torch.randn(E, device="cuda") * 0.05
    choice, w, lse, *_, aux_grad, aux = ext().moe_route(logits.detach(), bias, k, 0.01, 1e-3, None)
    dw = torch.randn(N, k, device="cuda")
    daux = 0.7
    got = ext().moe_route_bwd(logits.detach(), lse, choice, w, dw, aux_grad, torch.tensor([daux], device="cuda"), 1e-3)
    probs = logits.softmax(-1)
    wr = probs.gather(-1, choice.long())
    wr = wr / wr.sum(-1, keepdim=True)
    frac = torch.bincount(choice.flatten().long(), minlength=E).float() / (N * k)
    loss = (wr * dw).sum() + daux * (0.01 * E * (frac * probs.mean(0)).sum()
                                     + 1e-3 * torch.logsumexp(logits, -1).square().mean())
    (ref,) = torch.autograd.grad(loss, logits)
    torch.testing.assert_close(got, ref, rtol=1e-4, atol=1e-6)


def test_moe_layer_uses_fused_route():
    """The MoE layer's forward / backward through the fused routing equals the unfused routing."""
    from nexttransformer_b200.models import moe as M
    torch.manual_seed(2)
    layer = M.MoEFFN(256, 64, 8, 512, aux_loss_coeff=0.01, z_loss_coeff=1e-3).cuda()
    x = torch.randn(2, 200, 256, device="cuda", requires_grad=True)
    outs = []
    for fused in (True, False):
        layer.zero_grad()
        x.grad = None
        layer.fused_route = fused
        y = layer(x)
        (y.square().mean() + layer.last_aux).backward()
        outs.append((y.detach(), x.grad.clone(), layer.router.weight.grad.clone(), layer.last_aux.detach()))
    # the weights differ in the last fp32 bits (summation order), which can flip a bf16 rounding
    for a, b in zip(*outs):
        torch.testing.assert_close(a, b, rtol=1e-2, atol=1e-3)
