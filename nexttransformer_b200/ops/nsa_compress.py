"""NSA compressed branch and block selection on the sm_100a kernels (``csrc/nsa_compress.cu``).

``nsa_compressed(q, ck, cv, cstride, csize, ssize, topk, scale)`` takes q ``[B, T, H, 128]`` and the
compressed keys / values ``[B, Nc, Hk, 128]`` (bf16) and returns the compressed-branch output
``[B, T, H, 128]`` (softmax over the complete compressed blocks of each query) and the selection
membership ``[B, H, T, ceil(T / ssize)]`` (bool): the ``topk`` complete selection blocks of highest
importance (the probability mass of the compressed blocks overlapping them), the row's own block
excluded from the choice and then added.  The output is differentiable in q, ck and cv; the
membership is not.  It is the same computation as the torch compressed branch of
``models/sparse.py`` with the [B, H, T, Nc] scores, probabilities and importance never stored.
"""
import torch
from torch.autograd import Function

from nexttransformer_b200.ops._ext import ext


class _Compressed(Function):
    @staticmethod
    def forward(ctx, q, ck, cv, cstride, csize, ssize, topk, scale):
        o, lse, sel = ext().nsa_compressed_fwd(q, ck, cv, cstride, csize, ssize, topk, scale)
        ctx.save_for_backward(q, ck, cv, o, lse)
        ctx.meta = (cstride, csize, scale)
        ctx.mark_non_differentiable(sel)
        return o, sel.view(torch.bool)

    @staticmethod
    def backward(ctx, do, _sel):
        q, ck, cv, o, lse = ctx.saved_tensors
        cstride, csize, scale = ctx.meta
        do = do.contiguous().to(torch.bfloat16)
        delta = (do.float() * o.float()).sum(-1).transpose(1, 2).contiguous()   # [B, H, T]
        dq, dk, dv = ext().nsa_compressed_bwd(q, ck, cv, lse, do, delta, cstride, csize, scale)
        return dq.to(q.dtype), dk.to(ck.dtype), dv.to(cv.dtype), None, None, None, None, None


def supported(q, ck):
    T = q.shape[1]
    return (q.is_cuda and q.dtype == ck.dtype == torch.bfloat16 and q.shape[-1] == 128 and ck.shape[-1] == 128
            and q.shape[2] % ck.shape[2] == 0 and getattr(ext(), "nsa_compressed_fwd", None) is not None
            and (T + 63) // 64 <= 256)


def nsa_compressed(q, ck, cv, cstride, csize, ssize, topk, scale):
    return _Compressed.apply(q.contiguous(), ck.contiguous(), cv.contiguous(), int(cstride), int(csize), int(ssize),
                             int(topk), float(scale))
