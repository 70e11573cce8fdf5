"""CUDA entry points of the linear-attention mixers (DeltaNet / GDN / KDA).

* ``causal_conv_silu(x, w)``: the short causal depthwise convolution (width 4) with SiLU on
  ``[B, T, C]``, one sm_100a kernel each way (``csrc/linear_attn.cu``); the convolution output
  is kept for the backward.
* ``gated_rms_norm(y, gate, gain)``: ``RMSNorm(y) * gain * SiLU(gate)`` over the head dimension,
  one kernel each way.
* ``delta_chunk_cuda(...)``: the chunked (gated) delta rule.  With bf16 q / k / v of head size 128
  and chunk 64 it is two kernels each way: the per-chunk terms (``csrc/delta_prep.cu``: q / k L2
  normalisation for GDN, cumulative gates, the WY solve, qt / kc / aqk / carry) and the inter-chunk
  scan (``csrc/delta_scan.cu``); the backward runs the scan's reverse pass, four batched GEMMs for
  the chain-free products and the terms' backward kernel.  Other shapes keep the fp32 PyTorch chunk
  form of ``models/linear.py``.
"""
import torch
from torch.autograd import Function
import torch.nn.functional as F

from nexttransformer_b200.ops._ext import ext


class _ConvSiLU(Function):
    @staticmethod
    def forward(ctx, x, w):
        x = x.contiguous()
        B, T, C = x.shape
        wf = w.reshape(C, -1).float().contiguous()
        y = torch.empty_like(x)
        pre = torch.empty_like(x)
        ext().conv_silu_fwd(x, wf, y, pre)
        ctx.save_for_backward(x, pre, wf)
        ctx.wshape, ctx.wdtype = w.shape, w.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, pre, wf = ctx.saved_tensors
        dx = torch.empty_like(x)
        dw = torch.zeros_like(wf)
        ext().conv_silu_bwd(x, pre, dy.contiguous().to(x.dtype), wf, dx, dw)
        return dx, dw.reshape(ctx.wshape).to(ctx.wdtype)


def causal_conv_silu(x, w):
    if x.dtype != torch.bfloat16 or x.shape[-1] % 8:
        y = F.conv1d(F.pad(x.transpose(1, 2), (w.shape[-1] - 1, 0)), w.to(x.dtype), groups=x.shape[-1])
        return F.silu(y.transpose(1, 2))
    return _ConvSiLU.apply(x, w)


class _GatedRMSNorm(Function):
    @staticmethod
    def forward(ctx, y, gate, gain):
        y, gate = y.contiguous(), gate.contiguous()
        D = y.shape[-1]
        g32 = gain.float().contiguous()
        out = torch.empty_like(y)
        rstd = torch.empty(y.numel() // D, device=y.device, dtype=torch.float32)
        ext().gated_rmsnorm_fwd(y, gate, g32, out, rstd)
        ctx.save_for_backward(y, gate, g32, rstd)
        ctx.gdtype = gain.dtype
        return out

    @staticmethod
    def backward(ctx, dout):
        y, gate, g32, rstd = ctx.saved_tensors
        dy, dg = torch.empty_like(y), torch.empty_like(gate)
        dgain = torch.zeros_like(g32)
        ext().gated_rmsnorm_bwd(y, gate, g32, rstd, dout.contiguous().to(y.dtype), dy, dg, dgain)
        return dy, dg, dgain.to(ctx.gdtype)


def gated_rms_norm(y, gate, gain):
    if y.dtype != torch.bfloat16 or gate.dtype != torch.bfloat16 or y.shape[-1] not in (64, 128):
        from nexttransformer_b200.models.linear import gated_rms_norm as reference
        return reference(y, gate, gain)
    return _GatedRMSNorm.apply(y, gate, gain)


class _DeltaScan(Function):
    """The inter-chunk scan on the sm_100a kernels; inputs [B, H, N, 64, 128|64] (fp32 or bf16),
    carry [B, H, N, 128].  The per-chunk gradient products run as batched GEMMs on the engine."""

    @staticmethod
    def forward(ctx, w, u0, qt, kc, aqk, carry):
        B, H, N = w.shape[:3]
        BH = B * H

        def bf(t):
            return t.reshape(BH, N, *t.shape[3:]).to(torch.bfloat16).contiguous()
        wb, u0b, qtb, kcb, aqkb = bf(w), bf(u0), bf(qt), bf(kc), bf(aqk)
        cb = carry.reshape(BH, N, 128).float().contiguous()
        o = torch.empty_like(u0b)
        u = torch.empty_like(u0b)
        states = torch.empty(BH, N, 128, 128, device=w.device, dtype=torch.bfloat16)
        ext().delta_scan_fwd(wb, qtb, kcb, aqkb, u0b, cb, o, states, u)
        ctx.save_for_backward(wb, qtb, kcb, aqkb, cb, states, u)
        ctx.shape = (B, H, N)
        return o.reshape(B, H, N, 64, 128)

    @staticmethod
    def backward(ctx, do):
        from nexttransformer_b200.ops.gemm import EPI_F32, gemm
        wb, qtb, kcb, aqkb, cb, states, u = ctx.saved_tensors
        B, H, N = ctx.shape
        BH = B * H
        dob = do.reshape(BH, N, 64, 128).to(torch.bfloat16).contiguous()
        ds = torch.empty_like(states)
        dut = torch.empty(BH, N, 128, 64, device=do.device, dtype=torch.bfloat16)
        dcarry = torch.empty_like(cb)
        ext().delta_scan_bwd(dob, wb, qtb, kcb, aqkb, cb, states, ds, dut, dcarry)
        M = BH * N

        def f32(rows, cols):
            return torch.empty(M, rows, cols, device=do.device, dtype=torch.float32)
        flat = lambda t: t.reshape(M, *t.shape[2:])
        dqt = gemm(flat(dob), flat(states), f32(64, 128), epi=EPI_F32)                # do S^T
        dw = gemm(flat(dut), flat(states), f32(64, 128), a_mn=True, epi=EPI_F32, s_acc=-1.0)   # -du S^T
        daqk = gemm(flat(dob), flat(u), f32(64, 64), epi=EPI_F32)                     # do u^T
        dkc = gemm(flat(u), flat(ds), f32(64, 128), epi=EPI_F32)                      # u dS^T
        du0 = dut.transpose(-1, -2).float()
        shp = (B, H, N, 64)
        return (dw.reshape(*shp, 128), du0.reshape(*shp, 128), dqt.reshape(*shp, 128), dkc.reshape(*shp, 128),
                daqk.reshape(*shp, 64), dcarry.reshape(B, H, N, 128))


GATE_MODE = {"deltanet": 0, "gdn": 1, "kda": 2}
# The fused chunk-term kernels; NT_FUSED_DELTA=0 keeps the fp32 PyTorch chunk terms.
import os as _os
FUSED_DELTA = _os.environ.get("NT_FUSED_DELTA", "1") == "1"


def _chunk_scan_forward(prep, q):
    """Chunk terms (``prep`` fills w, u0, qt, kc, aqk, carry) and the inter-chunk scan; returns the
    output [B, T, H, 128] (a view of the chunk-major result) and the tensors the backward needs."""
    lib = ext()
    B, T, H, D = q.shape
    N = (T + 63) // 64
    BH = B * H
    dev = q.device
    bf = torch.bfloat16
    w, u0, qt, kc = (torch.empty(BH, N, 64, 128, device=dev, dtype=bf) for _ in range(4))
    aqk = torch.empty(BH, N, 64, 64, device=dev, dtype=bf)
    carry = torch.empty(BH, N, 128, device=dev, dtype=torch.float32)
    prep(w, u0, qt, kc, aqk, carry)
    o = torch.empty_like(u0)
    u = torch.empty_like(u0)
    states = torch.empty(BH, N, 128, 128, device=dev, dtype=bf)
    lib.delta_scan_fwd(w, qt, kc, aqk, u0, carry, o, states, u)
    return o.view(B, H, N * 64, 128)[:, :, :T].transpose(1, 2), (w, u0, qt, kc, aqk, carry, states, u)


def _chunk_scan_backward(dout, saved, shape):
    """The scan's reverse pass and the four chain-free products: dw, du0, dqt, dkc, daqk, dcarry."""
    from nexttransformer_b200.ops.gemm import EPI_F32, gemm
    lib = ext()
    w, u0, qt, kc, aqk, carry, states, u = saved
    B, T, H = shape
    N = (T + 63) // 64
    BH = B * H
    M = BH * N
    dev = dout.device
    do = torch.zeros(B, H, N * 64, 128, device=dev, dtype=torch.bfloat16)
    do[:, :, :T] = dout.transpose(1, 2)
    do = do.view(BH, N, 64, 128)
    ds = torch.empty_like(states)
    dut = torch.empty(BH, N, 128, 64, device=dev, dtype=torch.bfloat16)
    dcarry = torch.empty_like(carry)
    lib.delta_scan_bwd(do, w, qt, kc, aqk, carry, states, ds, dut, dcarry)

    def f32(rows, cols):
        return torch.empty(M, rows, cols, device=dev, dtype=torch.float32)
    flat = lambda t: t.view(M, *t.shape[2:])
    dqt = gemm(flat(do), flat(states), f32(64, 128), epi=EPI_F32)                      # do S^T
    dw = gemm(flat(dut), flat(states), f32(64, 128), a_mn=True, epi=EPI_F32, s_acc=-1.0)  # -du S^T
    daqk = gemm(flat(do), flat(u), f32(64, 64), epi=EPI_F32)                           # do u^T
    dkc = gemm(flat(u), flat(ds), f32(64, 128), epi=EPI_F32)                           # u dS^T
    du0 = dut.transpose(-1, -2).float().contiguous()
    return dw, du0, dqt, dkc, daqk, dcarry


class _DeltaChunk(Function):
    """Fused chunked delta rule: chunk terms (delta_prep) + inter-chunk scan (delta_scan)."""

    @staticmethod
    def forward(ctx, q, k, v, g, beta, gate, scale):
        lib = ext()
        out, saved = _chunk_scan_forward(
            lambda *o: lib.delta_prep_fwd(q, k, v, g, beta, gate, scale, *o), q)
        ctx.save_for_backward(q, k, v, g, beta, *saved)
        ctx.meta = (gate, scale)
        return out

    @staticmethod
    def backward(ctx, dout):
        lib = ext()
        q, k, v, g, beta, *saved = ctx.saved_tensors
        gate, scale = ctx.meta
        B, T, H, D = q.shape
        w, u0 = saved[0], saved[1]
        dw, du0, dqt, dkc, daqk, dcarry = _chunk_scan_backward(dout, saved, (B, T, H))
        dq, dk, dv = (torch.empty(q.shape, device=q.device, dtype=torch.float32) for _ in range(3))
        dbeta = torch.empty_like(beta)
        dg = torch.empty_like(g) if g is not None else None
        lib.delta_prep_bwd(q, k, v, g, beta, gate, scale, w, u0, dw, du0, dqt, dkc, daqk, dcarry, dq, dk, dv, dg,
                           dbeta)
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg, dbeta, None, None


class _KdaChunk(Function):
    """KDA with the per-feature gate formed in the chunk-term kernel from its pre-activation,
    g = -exp(g_log) softplus(g_raw + g_bias), and (qk_norm) the q / k L2 normalisation there too:
    the fp32 [B, T, H, 128] gate and the normalised q / k never reach global memory."""

    @staticmethod
    def forward(ctx, q, k, v, g_raw, g_log, g_bias, beta, scale, qk_norm):
        lib = ext()
        gl, gb = g_log.float().contiguous(), g_bias.float().contiguous()
        out, saved = _chunk_scan_forward(
            lambda *o: lib.delta_prep_kda_fwd(q, k, v, g_raw, gl, gb, beta, scale, qk_norm, *o), q)
        ctx.save_for_backward(q, k, v, g_raw, gl, gb, beta, *saved)
        ctx.meta = (scale, qk_norm, g_log.dtype, g_bias.dtype)
        return out

    @staticmethod
    def backward(ctx, dout):
        lib = ext()
        q, k, v, g_raw, gl, gb, beta, *saved = ctx.saved_tensors
        scale, qk_norm, log_dt, bias_dt = ctx.meta
        B, T, H, D = q.shape
        N = (T + 63) // 64
        w, u0 = saved[0], saved[1]
        dw, du0, dqt, dkc, daqk, dcarry = _chunk_scan_backward(dout, saved, (B, T, H))
        dq, dk, dv = (torch.empty(q.shape, device=q.device, dtype=torch.float32) for _ in range(3))
        dbeta = torch.empty_like(beta)
        dg_raw = torch.empty_like(g_raw)
        parts = torch.empty(2, B, N, H, 128, device=q.device, dtype=torch.float32)
        lib.delta_prep_kda_bwd(q, k, v, g_raw, gl, gb, beta, scale, qk_norm, w, u0, dw, du0, dqt, dkc, daqk, dcarry,
                               dq, dk, dv, dg_raw, parts[0], parts[1], dbeta)
        sums = parts.sum((1, 2))
        return (dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), dg_raw, sums[0].to(log_dt), sums[1].to(bias_dt),
                dbeta, None, None)


def kda_chunk_cuda(q, k, v, g_raw, g_log, g_bias, beta, *, qk_l2norm_scale=None):
    """KDA on the fused kernels from the gate's pre-activation (bf16 [B, T, H, 128]) and its per-head,
    per-feature parameters g_log / g_bias [H, 128]; q / k raw when ``qk_l2norm_scale`` is given (the
    kernel normalises them: q <- s q / |q|, k <- k / |k|), else already normalised."""
    norm = qk_l2norm_scale is not None
    return _KdaChunk.apply(q.contiguous(), k.contiguous(), v.contiguous(), g_raw.contiguous(), g_log, g_bias,
                           beta.float().contiguous(), float(qk_l2norm_scale) if norm else 1.0, norm)


def fused_chunk_supported(q, k, v, chunk):
    return (FUSED_DELTA and q.is_cuda and chunk == 64 and q.shape[-1] == 128 and v.shape[-1] == 128 and
            q.dtype == k.dtype == v.dtype == torch.bfloat16 and q.shape == k.shape == v.shape)


def scan_supported(q, v, chunk):
    return q.is_cuda and chunk == 64 and q.shape[-1] == 128 and v.shape[-1] == 128


def delta_chunk_cuda(q, k, v, *, kind, g=None, beta=None, chunk, qk_l2norm_scale=None):
    """Chunked (gated) delta rule on CUDA: q, k, v [B, T, H, 128]; g log decay (GDN [B, T, H],
    KDA [B, T, H, 128]); beta [B, T, H].  The per-chunk WY terms are formed in fp32 with torch
    (triangular solve included), the scan runs on the sm_100a kernels."""
    from nexttransformer_b200.models.linear import _chunked, _delta_scan, _delta_terms
    if fused_chunk_supported(q, k, v, chunk) and kind in GATE_MODE:
        gate = GATE_MODE[kind]
        gf = None if gate == 0 else g.float().contiguous()
        return _DeltaChunk.apply(q.contiguous(), k.contiguous(), v.contiguous(), gf, beta.float().contiguous(), gate,
                                 float(qk_l2norm_scale) if qk_l2norm_scale is not None else 1.0)
    dt = q.dtype
    T = q.shape[1]
    q, k, v = q.float(), k.float(), v.float()
    if qk_l2norm_scale is not None:
        q, k = F.normalize(q, dim=-1) * qk_l2norm_scale, F.normalize(k, dim=-1)
    qc, kc_, vc = (_chunked(x, chunk) for x in (q, k, v))
    gc = None if g is None else _chunked(g.float(), chunk)
    w, u0, qt, kc, aqk, carry = _delta_terms(qc, kc_, vc, gc, _chunked(beta.float(), chunk), chunk,
                                             per_feature=(kind == "kda"))
    if scan_supported(q, v, chunk):
        B, H, N = w.shape[:3]
        if carry is None:
            carry = w.new_ones(B, H, N, 128)
        else:
            carry = carry.squeeze(-1).expand(B, H, N, 128)
        out = _DeltaScan.apply(w, u0, qt, kc, aqk, carry)
    else:
        out = _delta_scan(w, u0, qt, kc, aqk, carry)
    return out.movedim(1, 3).flatten(1, 2)[:, :T].to(dt)


def scalar_chunk_cuda(q, k, v, g, chunk):
    """Linear attention with a per-head scalar log decay g [B, T, H] (RetNet) on the scan kernels:
    the delta-rule scan with w = 0 and u0 = v is S <- c S + k_c^T v, o = q~ S + aqk v, the chunk
    form of ``models/linear.py`` ``_scalar_decay_chunks``."""
    import math
    from nexttransformer_b200.models.linear import _chunked, _scalar_decay_chunks, _tril
    dt = q.dtype
    T = q.shape[1]
    qc, kc_, vc = (_chunked(x.float(), chunk) for x in (q, k, v))
    if not scan_supported(q, v, chunk):
        out = _scalar_decay_chunks(qc, kc_, vc, None if g is None else _chunked(g.float(), chunk), chunk)
        return out.movedim(1, 3).flatten(1, 2)[:, :T].to(dt)
    causal = _tril(chunk, q.device)
    B, H, N = qc.shape[:3]
    if g is None:
        aqk = (qc @ kc_.transpose(-1, -2)).masked_fill(~causal, 0)
        qt, kc, carry = qc, kc_, qc.new_ones(B, H, N, 128)
    else:
        b = _chunked(g.float(), chunk).cumsum(-1)
        pair = (b[..., :, None] - b[..., None, :]).masked_fill(~causal, -math.inf).exp()
        aqk = (qc @ kc_.transpose(-1, -2)) * pair
        qt = qc * b.exp()[..., None]
        kc = kc_ * (b[..., -1:] - b).exp()[..., None]
        carry = b[..., -1].exp()[..., None].expand(B, H, N, 128)
    w = torch.zeros_like(qt)
    out = _DeltaScan.apply(w, vc, qt, kc, aqk, carry)
    return out.movedim(1, 3).flatten(1, 2)[:, :T].to(dt)


def gla_supported(q, v):
    return q.is_cuda and q.shape[-1] == 128 and v.shape[-1] == 128


def gla_chunk_cuda(q, k, v, log_decay, chunk=64):
    """GLA, S <- diag(e^{g_t}) S + k_t v_t^T and o_t = q_t S_t with a per-feature log decay
    g [B, T, H, 128], in the chunk form on the scan kernels: the delta-rule scan with w = 0 and
    u0 = v, qt = q e^{b}, kc = k e^{b_last - b}, aqk = tril(qt (k e^{-b})^T) and carry e^{b_last}
    (b the within-chunk cumulative log decay), so the recurrence over T tokens becomes one scan over
    T / 64 chunks."""
    from nexttransformer_b200.models.linear import _chunked, _tril
    dt, T = q.dtype, q.shape[1]
    qc, kc_, vc = (_chunked(x.float(), chunk) for x in (q, k, v))
    b = _chunked(log_decay.float(), chunk).cumsum(-2)
    causal = _tril(chunk, q.device)
    qt = qc * b.exp()
    aqk = (qt @ (kc_ * (-b).exp()).transpose(-1, -2)).masked_fill(~causal, 0)
    last = b[..., -1:, :]
    kc = kc_ * (last - b).exp()
    carry = last.squeeze(-2).exp().contiguous()
    out = _DeltaScan.apply(torch.zeros_like(qt), vc, qt, kc, aqk, carry)
    return out.movedim(1, 3).flatten(1, 2)[:, :T].to(dt)
