"""Residual-stream kernels (mHC Sinkhorn-Knopp) against the PyTorch log-domain form in fp64."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,iterations", [(1, 1), (1000, 20), (4097, 7)])
def test_sinkhorn_kernel_matches_reference(rows, iterations):
    from nexttransformer_b200.models import residual
    torch.manual_seed(0)
    logits = torch.randn(rows, 4, 4, dtype=torch.float64) * 2
    ref_in = logits.clone().requires_grad_()
    ref = residual.sinkhorn_knopp(ref_in, iterations)            # CPU: the PyTorch form
    g = torch.randn_like(ref)
    ref.backward(g)
    dev_in = logits.float().cuda().requires_grad_()
    out = residual.sinkhorn_knopp(dev_in, iterations)            # CUDA: the fused kernel
    out.backward(g.float().cuda())
    torch.testing.assert_close(out.double().cpu(), ref.detach(), atol=2e-5, rtol=2e-4)
    torch.testing.assert_close(dev_in.grad.double().cpu(), ref_in.grad, atol=2e-4, rtol=2e-3)
