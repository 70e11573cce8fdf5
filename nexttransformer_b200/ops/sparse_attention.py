"""Attention under an explicit key mask for the sparse mixers' "kernel" backend.

``masked_attention(q, k, v, mask)``: q [B, H, Q, D], k / v [B, H, T, D], mask [B, H, Q, T]
(nonzero = key visible).  Rows with no visible key return zeros, as the reference's safe softmax
does.  This runs PyTorch's memory-efficient attention with a boolean mask (a library kernel);
the "reference" backend (gathered keys, ``models.sparse.indexed_attention``) is the default of
every admitted sparse configuration.
"""
import torch
import torch.nn.functional as F


def masked_attention(q, k, v, mask):
    keep = mask > 0
    out = F.scaled_dot_product_attention(q, k, v, attn_mask=keep)
    return torch.where(keep.any(-1, keepdim=True), out, torch.zeros_like(out))
