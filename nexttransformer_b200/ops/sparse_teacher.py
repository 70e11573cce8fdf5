"""Head-mean distillation teacher of the learned sparse indexers.

``head_mean_teacher(q, k, mask, q_start, scale)`` returns ``safe_softmax(q k^T scale, domain).mean(1)``
as ``[B, Q, T]`` fp32, the domain being keys at or before each query's absolute position
``q_start + i`` that ``mask`` ([B, Q, T] bool, shared by every head; None for the causal burn-in
domain) allows.  On CUDA with bf16 operands and head dim 128 it runs the two sm_100a kernels of
``csrc/sparse_teacher.cu`` (a per-head log-sum-exp pass, then the head-summed probabilities tile by
tile), so the ``[B, H, Q, T]`` scores are never stored; elsewhere it is the torch expression above.
The result carries no gradient (the teacher is a distillation target).
"""
import torch

from nexttransformer_b200.ops._ext import ext


def _reference(q, k, mask, q_start, scale):
    from nexttransformer_b200.models.sparse import safe_softmax
    B, H, Q, _ = q.shape
    T = k.shape[2]
    if k.shape[1] != H:
        k = k.repeat_interleave(H // k.shape[1], dim=1)
    pos = torch.arange(q_start, q_start + Q, device=q.device)
    domain = (torch.arange(T, device=q.device)[None, :] <= pos[:, None])[None]
    if mask is not None:
        domain = domain & mask
    raw = torch.matmul(q.float(), k.float().transpose(-2, -1)) * scale
    return safe_softmax(raw, domain[:, None].expand(B, H, Q, T)).mean(1)


def kernel_supported(q, k):
    return (q.is_cuda and q.dtype == k.dtype == torch.bfloat16 and q.shape[-1] == 128 and q.stride(-1) == 1
            and k.stride(-1) == 1 and q.shape[1] % k.shape[1] == 0 and getattr(ext(), "sparse_teacher", None))


@torch.no_grad()
def head_mean_teacher(q, k, mask, q_start, scale):
    if kernel_supported(q, k):
        return ext().sparse_teacher(q, k, mask, int(q_start), float(scale))
    return _reference(q, k, mask, q_start, scale)
