"""Causal-edge formulation of REL attention (CPU oracle and the graph the FLOP ledger audits).

Only the causal (query, key) pairs are formed: scores and value products are computed per edge
(packed in row order), the edge scores are scattered into a ``-inf``-padded square for the row
softmax, and outputs are accumulated by scatter-add over query rows.  The cost ledger charges these
operators, so this is the path whose arithmetic the method's FLOPs per token are defined by.
"""
import torch


def relative_attention_edges(q, k, v, r, table):
    """``[B, T, H, D]`` q/k/v (MHA), ``r [B, T, H, d_rel]``, ``table [d_rel, extent]``."""
    B, T, H, D = q.shape
    if k.shape != q.shape or v.shape != q.shape:
        raise ValueError("REL needs full-sequence MHA with equal q/k/v shapes")
    extent = table.shape[1]
    if T > extent:
        raise ValueError("the relative table must cover the sequence")
    rel = r @ table                                               # [B, T, H, extent]
    qi, kj = torch.tril_indices(T, T, device=q.device)            # causal edges, row order
    E = qi.numel()
    q_idx = qi[None, :, None, None].expand(B, E, H, D)
    k_idx = kj[None, :, None, None].expand(B, E, H, D)
    k_e = k.gather(1, k_idx)
    s = (q.gather(1, q_idx) * k_e).sum(-1) * D ** -0.5            # [B, E, H]
    flat = (qi[:, None] * H + torch.arange(H, device=q.device)[None, :]) * extent + (qi - kj)[:, None]
    s = s + rel.reshape(B, -1).gather(1, flat.reshape(1, -1).expand(B, -1)).reshape(B, E, H)
    square = torch.full((B, H, T, T), -torch.inf, dtype=s.dtype, device=s.device)
    square[:, :, qi, kj] = s.transpose(1, 2)
    p = square.softmax(-1)[:, :, qi, kj].transpose(1, 2)          # [B, E, H]
    contrib = p.unsqueeze(-1) * v.gather(1, k_idx)
    return torch.zeros_like(q).scatter_add(1, q_idx, contrib)


def dense_oracle(q, k, v, r, table):
    """Independent dense formulation (``[B, H, T, T]`` scores) for validation."""
    B, T, H, D = q.shape
    dist = torch.arange(T, device=q.device)[:, None] - torch.arange(T, device=q.device)[None, :]
    rel = (r @ table).transpose(1, 2)                             # [B, H, T, extent]
    bias = rel.gather(-1, dist.clamp_min(0)[None, None].expand(B, H, T, T))
    s = q.transpose(1, 2) @ k.transpose(1, 2).transpose(-1, -2) * D ** -0.5 + bias
    s = s.masked_fill(dist[None, None] < 0, -torch.inf)
    return (s.softmax(-1) @ v.transpose(1, 2)).transpose(1, 2)
