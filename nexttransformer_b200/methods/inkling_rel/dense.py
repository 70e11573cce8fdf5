"""REL attention on the GPU: the dense formulation, processed in query blocks.

Each block of ``BLOCK`` query rows forms its ``[B, H, BLOCK, T]`` scores, adds the relative bias
gathered from ``r @ table`` and applies the causal mask, so peak memory is ``B*H*BLOCK*T`` floats
per block instead of the full square.  Autograd differentiates through every block (scores and
bias are recomputed by autograd's saved tensors, not re-derived).
"""
import torch

BLOCK = 512


def relative_attention_dense(q, k, v, r, table):
    B, T, H, D = q.shape
    rel = (r @ table).transpose(1, 2)                             # [B, H, T, extent]
    qt, kt, vt = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    keys = torch.arange(T, device=q.device)
    outs = []
    for s0 in range(0, T, BLOCK):
        s1 = min(T, s0 + BLOCK)
        rows = torch.arange(s0, s1, device=q.device)
        dist = rows[:, None] - keys[None, :s1]
        bias = rel[:, :, s0:s1].gather(-1, dist.clamp_min(0)[None, None].expand(B, H, s1 - s0, s1))
        s = (qt[:, :, s0:s1].float() @ kt[:, :, :s1].float().transpose(-1, -2)) * D ** -0.5 + bias.float()
        s = s.masked_fill(dist[None, None] < 0, -torch.inf)
        outs.append((s.softmax(-1) @ vt[:, :, :s1].float()).to(q.dtype))
    return torch.cat(outs, 2).transpose(1, 2)
