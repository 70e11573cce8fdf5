"""Attention over selected key blocks for the sparse mixers (NSA selected blocks, MoBA).

``block_lists(blocks)`` turns a per-row selection of 64-key blocks (``blocks`` bool [B, G, T, NB]:
row t of list group g selects keys [64 j, 64 j + 64)) into what the sm_100a kernels walk: per
128-row query tile the sorted union of the selected blocks (int32 lists [B, G, n_qt, Lmax], -1
padded) and per listed block a 128-bit row mask (int32 [B, G, n_qt, Lmax, 4]).

``block_sparse_attention(q, k, v, lists, masks, scale)`` (q [B, T, H, 128], k / v [B, T, Hk, 128],
bf16) runs ``csrc/sparse_attn.cu``: row t of head h attends to the keys j <= t of the blocks its
list group h / (H / G) selected; rows that see no key give 0, as the reference's safe softmax.

``masked_attention(q, k, v, mask)`` keeps the explicit-mask interface of the "kernel" backend for
selections that are not made of 64-key blocks (PyTorch's memory-efficient attention, a library
kernel).
"""
import torch
from torch.autograd import Function
import torch.nn.functional as F

from nexttransformer_b200.ops._ext import ext

QT, KB = 128, 64


def block_lists(blocks):
    B, G, T, NB = blocks.shape
    n_qt = (T + QT - 1) // QT
    pad = n_qt * QT - T
    mem = F.pad(blocks, (0, 0, 0, pad)) if pad else blocks
    mem = mem.view(B, G, n_qt, QT, NB)
    union = mem.any(3)
    Lmax = max(1, int(union.sum(-1).max()))
    key = (~union).to(torch.int64) * NB + torch.arange(NB, device=blocks.device)
    order = key.argsort(-1)[..., :Lmax]
    valid = union.gather(-1, order)
    lists = torch.where(valid, order, torch.full_like(order, -1)).to(torch.int32).contiguous()
    rows = mem.permute(0, 1, 2, 4, 3).gather(3, order[..., None].expand(-1, -1, -1, -1, QT))
    rows = rows & valid[..., None]
    bits = rows.view(B, G, n_qt, Lmax, 4, 32).to(torch.int64) << torch.arange(32, device=blocks.device)
    words = bits.sum(-1)
    words = torch.where(words >= 2 ** 31, words - 2 ** 32, words)
    return lists, words.to(torch.int32).contiguous()


class _BlockSparseAttention(Function):
    @staticmethod
    def forward(ctx, q, k, v, lists, masks, scale, rel):
        B, T, H, D = q.shape
        Hk = k.shape[2]
        qf = q.reshape(B * T, H * D).contiguous()
        kf = k.reshape(B * T, Hk * D).contiguous()
        vf = v.reshape(B * T, Hk * D).contiguous()
        o = torch.empty_like(qf)
        lse = torch.empty(B, H, T, device=q.device, dtype=torch.float32)
        relf = None if rel is None else rel.float().contiguous()
        ext().sparse_attn_fwd(qf, kf, vf, lists, masks, o, lse, B, T, H, Hk, float(scale), relf)
        ctx.save_for_backward(qf, kf, vf, lists, masks, o, lse, relf)
        ctx.dims = (B, T, H, Hk, D, float(scale))
        ctx.rel_dtype = None if rel is None else rel.dtype
        return o.view(B, T, H, D)

    @staticmethod
    def backward(ctx, do):
        qf, kf, vf, lists, masks, o, lse, relf = ctx.saved_tensors
        B, T, H, Hk, D, scale = ctx.dims
        dof = do.reshape(B * T, H * D).to(torch.bfloat16).contiguous()
        delta = (dof.float() * o.float()).view(B, T, H, D).sum(-1).permute(0, 2, 1).contiguous()
        dq = torch.empty_like(qf)
        dk = torch.zeros(B * T, Hk * D, device=qf.device, dtype=torch.float32)
        dv = torch.zeros_like(dk)
        drel = None if relf is None else torch.zeros_like(relf)
        ext().sparse_attn_bwd(qf, kf, vf, lists, masks, lse, dof, delta, dq, dk, dv, B, T, H, Hk, scale, relf, drel)
        return (dq.view(B, T, H, D), dk.to(torch.bfloat16).view(B, T, Hk, D), dv.to(torch.bfloat16).view(B, T, Hk, D),
                None, None, None, None if drel is None else drel.to(ctx.rel_dtype))


def visibility(lists, masks, T):
    """Dense [B, G, T, T] key visibility of block lists (row t sees key j of its selected blocks, j <= t)."""
    B, G, n_qt, Lmax = lists.shape
    bits = ((masks.to(torch.int64) & 0xFFFFFFFF)[..., None] >> torch.arange(32, device=masks.device)) & 1
    rows = bits.reshape(B, G, n_qt, Lmax, QT).bool()                     # [B, G, n_qt, L, 128]
    nb = (T + KB - 1) // KB
    # padding entries (-1) scatter into an extra column that is dropped
    sel = torch.zeros(B, G, n_qt, QT, nb + 1, dtype=torch.bool, device=lists.device)
    idx = torch.where(lists >= 0, lists, torch.full_like(lists, nb)).long()[..., None, :].expand(-1, -1, -1, QT, -1)
    sel.scatter_(-1, idx, rows.transpose(-1, -2))
    sel = sel[..., :nb].reshape(B, G, n_qt * QT, nb)[:, :, :T].repeat_interleave(KB, -1)[..., :T]
    pos = torch.arange(T, device=lists.device)
    return sel & (pos[None, :] <= pos[:, None])


def block_sparse_reference(q, k, v, lists, masks, scale, rel=None):
    """The same attention in fp32 PyTorch (dense masked softmax), the oracle of the kernels."""
    B, T, H, D = q.shape
    Hk, G = k.shape[2], lists.shape[1]
    vis = visibility(lists, masks, T).repeat_interleave(H // G, 1)
    kk = k.float().repeat_interleave(H // Hk, 2).transpose(1, 2)
    vv = v.float().repeat_interleave(H // Hk, 2).transpose(1, 2)
    s = torch.einsum("bhqd,bhkd->bhqk", q.float().transpose(1, 2), kk) * scale
    if rel is not None:
        pos = torch.arange(T, device=q.device)
        dist = (pos[:, None] - pos[None, :]).clamp_min(0)
        s = s + rel.float().gather(-1, dist[None, None].expand(B, H, T, T))
    s = s.masked_fill(~vis, -torch.inf)
    p = torch.where(vis.any(-1, keepdim=True), s.softmax(-1).nan_to_num(0.0), torch.zeros_like(s))
    return torch.einsum("bhqk,bhkd->bhqd", p, vv).transpose(1, 2).to(q.dtype)


def block_sparse_attention(q, k, v, lists, masks, scale=None, rel=None):
    """``rel`` (optional, [B, H, T, extent >= T]): additive bias, logit(i, j) += rel[b, h, i, i - j]."""
    scale = q.shape[-1] ** -.5 if scale is None else scale
    if not q.is_cuda:
        return block_sparse_reference(q, k, v, lists, masks, scale, rel)
    return _BlockSparseAttention.apply(q, k, v, lists, masks, scale, rel)


def causal_lists(B, T, device):
    """Lists of every 64-key block at or before each query tile (dense causal attention), one group."""
    nb = (T + KB - 1) // KB
    pos_blk = torch.arange(T, device=device) // KB
    blocks = (torch.arange(nb, device=device)[None, :] <= pos_blk[:, None])[None, None].expand(B, 1, T, nb)
    return block_lists(blocks.contiguous())


def masked_attention(q, k, v, mask):
    """q [B, H, Q, D], k / v [B, H, T, D], mask [B, H, Q, T] (nonzero = visible)."""
    keep = mask > 0
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=keep)
    return torch.where(keep.any(-1, keepdim=True), out, torch.zeros_like(out))
