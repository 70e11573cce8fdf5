"""Grouped-expert MoE on the sm_100a kernels against the fp32 per-expert PyTorch path."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


@pytest.mark.parametrize("T,E,k,d,F", [(100, 8, 2, 128, 128), (1000, 16, 4, 256, 192), (37, 64, 8, 128, 64)])
def test_grouped_experts_match_fp32(T, E, k, d, F):
    from nexttransformer_b200.models.moe import MoEFFN
    torch.manual_seed(0)
    cpu = MoEFFN(d, E, k, F, shared=1)
    for p in cpu.parameters():
        torch.nn.init.normal_(p, std=0.05)
    gpu = MoEFFN(d, E, k, F, shared=1).cuda()
    gpu.load_state_dict(cpu.state_dict())
    x = torch.randn(2, T, d)
    xg = x.cuda().to(torch.bfloat16).requires_grad_()
    xc = x.clone().requires_grad_()
    yc = cpu(xc)
    yg = gpu(xg)
    dy = torch.randn_like(yc)
    yc.backward(dy)
    yg.backward(dy.cuda().to(torch.bfloat16))
    assert _rel(yg.cpu(), yc) < 2e-2
    assert _rel(xg.grad.cpu(), xc.grad) < 3e-2
    for (n, pc), pg in zip(cpu.named_parameters(), gpu.parameters()):
        if pc.grad is None or pc.grad.norm() == 0:
            continue
        # bf16 activations against fp32: experts with few rows see the largest relative error
        assert _rel(pg.grad.cpu(), pc.grad) < 6e-2, n


def test_plan_layout():
    from nexttransformer_b200.ops.moe import plan
    torch.manual_seed(1)
    choice = torch.randint(0, 5, (50, 3), device="cuda")
    pl = plan(choice, 5)
    row_of, src_of, grp_m, grp_k = (pl[k].cpu().long() for k in ("row_of", "src_of", "grp_m", "grp_k"))
    flat = choice.flatten().cpu()
    assert len(set(row_of.tolist())) == flat.numel()
    assert (src_of[row_of] == torch.arange(150) // 3).all()
    for j, r in enumerate(row_of.tolist()):
        e = int(flat[j])
        assert grp_k[e] <= r < grp_k[e + 1]
        assert grp_m[r // 128] == e
    assert (grp_k % 128 == 0).all()
