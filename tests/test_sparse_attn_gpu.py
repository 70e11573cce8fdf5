"""Block-sparse attention kernels against a dense fp32 masked-softmax reference."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def _reference(q, k, v, blocks, scale):
    B, T, H, D = q.shape
    Hk, G = k.shape[2], blocks.shape[1]
    keys = torch.arange(T, device=q.device)
    sel = blocks.repeat_interleave(64, -1)[..., :T]                     # [B, G, T, T]
    vis = sel & (keys[None, :] <= keys[:, None])
    vis = vis.repeat_interleave(H // G, 1)                               # [B, H, T, T]
    kk = k.float().repeat_interleave(H // Hk, 2).transpose(1, 2)
    vv = v.float().repeat_interleave(H // Hk, 2).transpose(1, 2)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float().transpose(1, 2), kk) * scale
    s = s.masked_fill(~vis, -torch.inf)
    p = torch.where(vis.any(-1, keepdim=True), s.softmax(-1).nan_to_num(0.0), torch.zeros_like(s))
    return torch.einsum("bhqk,bhkd->bhqd", p, vv).transpose(1, 2)


@pytest.mark.parametrize("B,T,H,Hk,G,nsel", [(1, 256, 2, 1, 1, 2), (2, 700, 4, 1, 1, 3), (1, 1024, 4, 2, 4, 4),
                                              (2, 384, 16, 1, 1, 16)])
def test_block_sparse_attention(B, T, H, Hk, G, nsel):
    from nexttransformer_b200.ops.sparse_attention import block_lists, block_sparse_attention
    torch.manual_seed(0)
    D = 128
    NB = (T + 63) // 64
    score = torch.rand(B, G, T, NB, device="cuda")
    pos_blk = torch.arange(T, device="cuda") // 64
    score = score.masked_fill(torch.arange(NB, device="cuda")[None, :] > pos_blk[:, None], -1.0)
    top = score.topk(min(nsel, NB), -1).indices
    blocks = torch.zeros(B, G, T, NB, dtype=torch.bool, device="cuda").scatter_(-1, top, True)
    blocks &= torch.arange(NB, device="cuda")[None, :] <= pos_blk[:, None]
    lists, masks = block_lists(blocks)
    q = torch.randn(B, T, H, D, device="cuda").to(torch.bfloat16).requires_grad_()
    k = torch.randn(B, T, Hk, D, device="cuda").to(torch.bfloat16).requires_grad_()
    v = torch.randn(B, T, Hk, D, device="cuda").to(torch.bfloat16).requires_grad_()
    scale = D ** -.5
    y = block_sparse_attention(q, k, v, lists, masks, scale)
    dy = torch.randn_like(y)
    y.backward(dy)
    qr, kr, vr = (t.detach().float().requires_grad_() for t in (q, k, v))
    yr = _reference(qr, kr, vr, blocks, scale)
    yr.backward(dy.float())
    from nexttransformer_b200.ops._ext import check_errors
    check_errors()
    assert _rel(y, yr) < 2e-2
    assert _rel(q.grad, qr.grad) < 3e-2
    assert _rel(k.grad, kr.grad) < 3e-2
    assert _rel(v.grad, vr.grad) < 3e-2


def test_block_lists_layout():
    from nexttransformer_b200.ops.sparse_attention import block_lists
    torch.manual_seed(1)
    blocks = torch.rand(1, 2, 300, 5, device="cuda") > 0.6
    lists, masks = block_lists(blocks)
    L, M = lists.cpu(), masks.cpu().to(torch.int64) & 0xFFFFFFFF
    for g in range(2):
        for t in range(3):
            rows = blocks[0, g, t * 128:(t + 1) * 128].cpu()
            want = sorted(set(torch.nonzero(rows.any(0)).flatten().tolist()))
            got = [x for x in L[0, g, t].tolist() if x >= 0]
            assert got == want
            for li, j in enumerate(got):
                for r in range(rows.shape[0]):
                    assert bool((M[0, g, t, li, r // 32] >> (r % 32)) & 1) == bool(rows[r, j])


@pytest.mark.parametrize("kind", ["moba", "nsa"])
def test_sparse_mixer_kernel_matches_reference(kind):
    """A sparse mixer's block-sparse kernel path against its gathered-key reference path."""
    from dataclasses import replace
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.sparse import SparseMixer
    c = debug_config(kind, width=256, sequence_len=512)
    extra = dict(block_size=128, sparse_topk=256) if kind == "moba" else \
        dict(compression_size=64, compression_stride=0, block_size=64, sparse_topk=128, local_window=96)
    c = replace(c, heads=2, **extra)
    torch.manual_seed(3)
    mix = SparseMixer(c, 1).cuda().to(torch.bfloat16)
    x = torch.randn(2, 512, 256, device="cuda").to(torch.bfloat16)
    t = torch.arange(512, dtype=torch.float32, device="cuda")
    f = torch.outer(t, 1.0 / (100000 ** (torch.arange(0, 128, 2, device="cuda").float() / 128)))
    cos_sin = (f.cos().to(torch.bfloat16)[None, :, None, :], f.sin().to(torch.bfloat16)[None, :, None, :])
    outs, grads = [], []
    for backend in ("reference", "kernel"):
        mix.backend = backend
        xi = x.clone().requires_grad_()
        y = mix(xi, None, cos_sin, None)
        y.float().square().mean().backward()
        outs.append(y.detach())
        grads.append(xi.grad.detach())
        mix.zero_grad()
    assert _rel(outs[1], outs[0]) < 3e-2
    assert _rel(grads[1], grads[0]) < 5e-2


@pytest.mark.parametrize("kind", ["moba", "nsa"])
def test_sparse_mixer_kernel_matches_reference_bench_shape(kind):
    """The benchmark's selection shapes (MoBA 512-key blocks top-3, NSA stride-16 compression with
    64-key selection, 12 query heads / 1 KV head) at T 2048: kernel path against the reference path."""
    from dataclasses import replace
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.sparse import SparseMixer
    T = 2048
    c = debug_config(kind, width=1536, sequence_len=T)
    extra = dict(block_size=512, sparse_topk=1536) if kind == "moba" else \
        dict(compression_size=32, compression_stride=16, block_size=64, sparse_topk=1024, local_window=512)
    c = replace(c, heads=12, kv_heads=1, **extra)
    torch.manual_seed(5)
    mix = SparseMixer(c, 1).cuda().to(torch.bfloat16)
    x = torch.randn(1, T, 1536, device="cuda").to(torch.bfloat16)
    t = torch.arange(T, dtype=torch.float32, device="cuda")
    f = torch.outer(t, 1.0 / (100000 ** (torch.arange(0, 128, 2, device="cuda").float() / 128)))
    cos_sin = (f.cos().to(torch.bfloat16)[None, :, None, :], f.sin().to(torch.bfloat16)[None, :, None, :])
    outs, grads = [], []
    for backend in ("reference", "kernel"):
        mix.backend = backend
        xi = x.clone().requires_grad_()
        y = mix(xi, None, cos_sin, None)
        y.float().square().mean().backward()
        outs.append(y.detach())
        grads.append(xi.grad.detach())
        mix.zero_grad()
    assert _rel(outs[1], outs[0]) < 3e-2
    assert _rel(grads[1], grads[0]) < 5e-2


@pytest.mark.parametrize("B,T,H", [(1, 256, 2), (2, 300, 3)])
def test_rel_attention_matches_oracle(B, T, H):
    """Inkling REL (relative bias r @ E) on the block-sparse kernels against the dense fp32 oracle."""
    from nexttransformer_b200.methods.inkling_rel.reference import dense_oracle
    from nexttransformer_b200.ops.sparse_attention import block_sparse_attention, causal_lists
    torch.manual_seed(7)
    D, d_rel, extent = 128, 16, T + 5
    q = (torch.randn(B, T, H, D, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    k = (torch.randn(B, T, H, D, device="cuda") * 0.5).to(torch.bfloat16).requires_grad_()
    v = torch.randn(B, T, H, D, device="cuda").to(torch.bfloat16).requires_grad_()
    r = torch.randn(B, T, H, d_rel, device="cuda").requires_grad_()
    table = (torch.randn(d_rel, extent, device="cuda") * 0.3).requires_grad_()
    lists, masks = causal_lists(B, T, q.device)
    rel = (r @ table).transpose(1, 2).contiguous()
    y = block_sparse_attention(q, k, v, lists, masks, D ** -0.5, rel)
    dy = torch.randn_like(y)
    y.backward(dy)
    leaves = [t.detach().float().requires_grad_() for t in (q, k, v, r, table)]
    yr = dense_oracle(*leaves)
    yr.backward(dy.float())
    assert _rel(y, yr) < 2e-2
    for a, b in zip((q, k, v, r, table), leaves):
        assert _rel(a.grad, b.grad) < 4e-2
