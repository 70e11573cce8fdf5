"""NSA compressed-branch kernels against the fp32 torch expression of models/sparse.py."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _reference(q, ck, cv, cstride, csize, ssize, scale):
    """fp32 oracle: output [B, T, H, D], importance [B, H, T, nsel], visibility [T, Nc]."""
    B, T, H, D = q.shape
    Nc, Hk = ck.shape[1], ck.shape[2]
    rep = H // Hk
    qh = q.float().transpose(1, 2)                                   # B H T D
    kh = ck.float().transpose(1, 2).repeat_interleave(rep, 1)        # B H Nc D
    vh = cv.float().transpose(1, 2).repeat_interleave(rep, 1)
    ends = torch.arange(Nc, device=q.device) * cstride + csize - 1
    pos = torch.arange(T, device=q.device)
    vis = ends[None, :] <= pos[:, None]                              # T Nc
    sc = (qh @ kh.transpose(-1, -2)) * scale
    sc = sc.masked_fill(~vis, -torch.inf)
    nonempty = vis.any(-1)[:, None]
    p = torch.where(nonempty, sc, torch.zeros_like(sc)).softmax(-1) * vis
    out = (p @ vh).transpose(1, 2)
    nsel = (T + ssize - 1) // ssize
    starts = torch.arange(Nc, device=q.device) * cstride
    sb = torch.arange(nsel, device=q.device)
    overlap = (starts[:, None] < (sb[None, :] + 1) * ssize) & (ends[:, None] >= sb[None, :] * ssize)
    return out, p @ overlap.float(), vis


@pytest.mark.parametrize("B,T,H,Hk,cstride,csize,ssize,topk", [(1, 1024, 4, 1, 16, 32, 64, 4),
                                                                (2, 700, 2, 2, 32, 32, 32, 3),
                                                                (1, 2048, 16, 1, 16, 32, 64, 16)])
def test_compressed_branch(B, T, H, Hk, cstride, csize, ssize, topk):
    from nexttransformer_b200.ops.nsa_compress import nsa_compressed
    g = torch.Generator(device="cuda").manual_seed(0)
    Nc = (T - csize) // cstride + 1
    q = (torch.randn(B, T, H, 128, device="cuda", generator=g)).bfloat16().requires_grad_()
    ck = (torch.randn(B, Nc, Hk, 128, device="cuda", generator=g) * 0.3).bfloat16().requires_grad_()
    cv = torch.randn(B, Nc, Hk, 128, device="cuda", generator=g).bfloat16().requires_grad_()
    scale = 128 ** -.5
    out, sel = nsa_compressed(q, ck, cv, cstride, csize, ssize, topk, scale)
    dout = torch.randn_like(out)
    grads = torch.autograd.grad(out, (q, ck, cv), dout)
    leaves = [x.detach().float().requires_grad_() for x in (q, ck, cv)]
    ref, imp, vis = _reference(*leaves, cstride, csize, ssize, scale)
    rgrads = torch.autograd.grad(ref, leaves, dout.float())
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)
    for gk, gr in zip(grads, rgrads):
        err = (gk.float() - gr).norm() / gr.norm()
        assert err < 2e-2, err
    # selection: own block always; the others are top-k complete blocks (importance within 1e-3 of
    # the oracle's k-th largest, as bf16 scores can reorder near-ties)
    nsel = (T + ssize - 1) // ssize
    pos = torch.arange(T, device="cuda")
    cur = pos // ssize
    full = (torch.arange(nsel, device="cuda")[None, :] + 1) * ssize - 1 <= pos[:, None]
    eligible = full & (torch.arange(nsel, device="cuda")[None, :] != cur[:, None])
    assert sel.shape == (B, H, T, nsel) and sel.dtype == torch.bool
    assert sel.gather(-1, cur[None, None, :, None].expand(B, H, T, 1)).all()
    others = sel & eligible[None, None]
    n_elig = eligible.sum(-1)
    assert torch.equal(others.sum(-1), n_elig.clamp_max(topk)[None, None].expand(B, H, T))
    masked = imp.masked_fill(~eligible[None, None], -1.0)
    kth = masked.topk(min(topk, nsel), -1).values[..., -1:]
    chosen_min = masked.masked_fill(~others, 2.0).amin(-1, keepdim=True)
    has = others.any(-1, keepdim=True)
    assert ((chosen_min >= kth - 1e-3) | ~has).all()
