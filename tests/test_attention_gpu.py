"""sm_100a flash attention (forward + backward) against an fp32 PyTorch reference."""
import math

import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(qkv, B, T, H, Hk, D, window):
    from nexttransformer_b200.models.shell import window_mask
    v4 = qkv.float().view(B, T, H + 2 * Hk, D)
    q = v4[:, :, :H].transpose(1, 2)
    k = v4[:, :, H:H + Hk].transpose(1, 2).repeat_interleave(H // Hk, 1)
    v = v4[:, :, H + Hk:].transpose(1, 2).repeat_interleave(H // Hk, 1)
    s = (q @ k.transpose(-1, -2)) / math.sqrt(D)
    s = s.masked_fill(~window_mask(T, window if window >= 0 else T, qkv.device), float("-inf"))
    p = torch.softmax(s, -1)
    return (p @ v).transpose(1, 2).reshape(B * T, H * D)


@pytest.mark.parametrize("B,T,H,Hk,window", [(1, 128, 1, 1, -1), (2, 256, 2, 1, -1), (1, 384, 4, 2, -1),
                                             (1, 512, 2, 2, 200), (1, 200, 2, 1, -1), (2, 1024, 4, 1, 300),
                                             (1, 2048, 10, 5, -1)])
def test_attention_forward_backward(B, T, H, Hk, window):
    from nexttransformer_b200.ops import attention as A
    from nexttransformer_b200.ops._ext import check_errors
    torch.manual_seed(0)
    D = 128
    M = B * T
    qkv = (torch.randn(M, (H + 2 * Hk) * D, device="cuda") * 0.5).bfloat16()
    ref_in = qkv.float().requires_grad_()
    ref = _ref(ref_in, B, T, H, Hk, D, window)
    dout = torch.randn_like(ref)
    ref.backward(dout)
    inp = qkv.clone().requires_grad_()
    out = A._KernelAttn.apply(inp, B, T, H, Hk, D, window)
    out.backward(dout.bfloat16())
    torch.cuda.synchronize()
    check_errors()
    err = (out.float() - ref).abs().max().item()
    assert err < 2e-2, f"forward max err {err}"
    g, rg = inp.grad.float(), ref_in.grad
    for name, sl in (("dq", slice(0, H * D)), ("dk", slice(H * D, (H + Hk) * D)), ("dv", slice((H + Hk) * D, None))):
        e = (g[:, sl] - rg[:, sl]).abs().max().item()
        scale = rg[:, sl].abs().max().item()
        assert e <= 2e-2 + 2e-2 * scale, f"{name} max err {e} (scale {scale})"


@pytest.mark.parametrize("B,T,H,Hk,window", [(2, 512, 4, 2, -1), (1, 700, 2, 1, 300)])
def test_deterministic_backward_is_bitwise_reproducible(B, T, H, Hk, window):
    """Deterministic mode: the same gradients bit for bit on every run, equal to the default mode's
    within fp32 summation-order noise, and within the fp32 oracle's tolerance."""
    from nexttransformer_b200.ops import attention as A
    from nexttransformer_b200.ops._ext import check_errors
    torch.manual_seed(3)
    D = 128
    M = B * T
    qkv = (torch.randn(M, (H + 2 * Hk) * D, device="cuda") * 0.5).bfloat16()
    dout = torch.randn(M, H * D, device="cuda").bfloat16()

    def grads():
        inp = qkv.clone().requires_grad_()
        A._KernelAttn.apply(inp, B, T, H, Hk, D, window).backward(dout)
        torch.cuda.synchronize()
        return inp.grad.clone()
    try:
        A.set_deterministic(True)
        first, second = grads(), grads()
    finally:
        A.set_deterministic(False)
    default = grads()
    check_errors()
    assert torch.equal(first, second)
    assert (first.float() - default.float()).abs().max().item() <= 1e-2 * default.float().abs().max().item()
    ref_in = qkv.float().requires_grad_()
    _ref(ref_in, B, T, H, Hk, D, window).backward(dout.float())
    e = (first.float() - ref_in.grad).abs().max().item()
    assert e <= 2e-2 + 2e-2 * ref_in.grad.abs().max().item()
