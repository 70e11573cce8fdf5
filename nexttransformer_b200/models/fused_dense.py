"""CUDA execution of the dense shell with the sm_100a kernels.

Per layer the forward is five launches of our own kernels plus attention:
  mix+RMSNorm -> packed QKV GEMM -> RoPE+QK-norm+VE gate (in place) -> attention
  -> O-projection GEMM with residual-add epilogue -> RMSNorm -> c_fc GEMM with ReLU^2 epilogue
  -> c_proj GEMM with residual-add epilogue.
The head is one GEMM whose epilogue evaluates the soft-capped cross-entropy: it stores the
unnormalised logit gradient G = exp(z - cap) (1 - tanh^2) instead of the logits, plus per-row partial
sums of exp(z - cap) and the target's z; a row kernel turns those into loss, 1 / sum and the target
correction.  The backward folds the row normalisation and the one-hot term into the input-gradient
GEMM's epilogue and into a row-scaled weight-gradient operand, so no logits pass exists.

Gradients of parameters never go through autograd: each Function writes (first micro-batch)
or accumulates (later micro-batches) fp32 gradients straight into ``param.main_grad`` with
the GEMM epilogue.  Autograd only carries activation gradients between the Functions.
"""
import torch
from torch.autograd import Function

from nexttransformer_b200.ops import gemm as G
from nexttransformer_b200.ops._ext import ext
from nexttransformer_b200.ops.attention import attention_fn

# Cross-entropy kernel variant (0: automatic, 1: two-pass); kept selectable for numerics checks.
CE_VARIANT = 0
# True: the cross-entropy runs in the head GEMM's epilogue; False: GEMM + separate CE kernel.
FUSED_HEAD_CE = True


class GradSlot:
    """An fp32 gradient buffer that the next GEMM overwrites instead of accumulating into."""

    __slots__ = ("buf", "fresh")

    def __init__(self, buf):
        self.buf = buf
        self.fresh = True

    def take(self):
        """(buffer, accumulate?) for a GEMM epilogue; marks the buffer as holding data."""
        acc = not self.fresh
        self.fresh = False
        return self.buf, acc


class FusedState:
    """bf16 weight shadows and fp32 gradient buffers of a ``GPTShell`` on CUDA.

    ``c_q | c_k | c_v`` of a layer share one packed shadow (one QKV GEMM) and one packed
    gradient buffer; every parameter's ``main_grad`` is a view into these buffers.
    """

    def __init__(self, model, grad_alloc=None, plan_only=False):
        """``grad_alloc(shape)`` (optional) supplies the fp32 gradient buffers in a fixed order (a
        flat arena, e.g. in symmetric memory); ``plan_only`` only walks that order so the caller
        can size the arena, touching no parameter."""
        self.model = model
        dev = model.get_device()
        f32, bf = torch.float32, torch.bfloat16
        self.slots = []        # GEMM-written gradients (fresh / accumulate)
        self.zeroed = []       # gradients accumulated with atomics or torch ops
        self.casts = []        # (fp32 master, bf16 shadow)
        self.arena = None

        def grad(shape):
            if grad_alloc is not None:
                return grad_alloc(tuple(shape))
            return torch.zeros(tuple(shape), device=dev, dtype=f32)

        if plan_only:
            for blk in model.transformer.h:
                a = blk.attn
                grad((a.c_q.weight.shape[0] + 2 * a.c_k.weight.shape[0], a.c_q.weight.shape[1]))
                for lin in (a.c_proj, blk.mlp.c_fc, blk.mlp.c_proj):
                    grad(lin.weight.shape)
                if a.ve_gate is not None:
                    grad(a.ve_gate.weight.shape)
            grad(model.lm_head.weight.shape)
            for p in self._loose(model):
                grad(p.shape)
            return

        def shadow(p, out=None):
            out = out if out is not None else torch.empty(p.shape, device=dev, dtype=bf)
            self.casts.append((p, out))
            return out

        for blk in model.transformer.h:
            a = blk.attn
            nq, nk, d = a.c_q.weight.shape[0], a.c_k.weight.shape[0], a.c_q.weight.shape[1]
            a._w_qkv = torch.empty(nq + 2 * nk, d, device=dev, dtype=bf)
            g = grad((nq + 2 * nk, d))
            a._g_qkv = GradSlot(g)
            self.slots.append(a._g_qkv)
            for lin, lo, hi in ((a.c_q, 0, nq), (a.c_k, nq, nq + nk), (a.c_v, nq + nk, nq + 2 * nk)):
                lin.weight.main_grad = g[lo:hi]
                shadow(lin.weight, a._w_qkv[lo:hi])
            for lin in (a.c_proj, blk.mlp.c_fc, blk.mlp.c_proj):
                lin._w = shadow(lin.weight)
                lin.weight.main_grad = grad(lin.weight.shape)
                lin._g = GradSlot(lin.weight.main_grad)
                self.slots.append(lin._g)
            if a.ve_gate is not None:
                a.ve_gate._w = shadow(a.ve_gate.weight)
                a.ve_gate.weight.main_grad = grad(a.ve_gate.weight.shape)
                self.zeroed.append(a.ve_gate.weight.main_grad)
        head = model.lm_head
        head._w = shadow(head.weight)
        head.weight.main_grad = grad(head.weight.shape)
        head._g = GradSlot(head.weight.main_grad)
        self.slots.append(head._g)
        model.smear_gate._w = shadow(model.smear_gate.weight)
        for p in self._loose(model):
            p.main_grad = grad(p.shape)
            self.zeroed.append(p.main_grad)
        self.refresh_shadows()

    @staticmethod
    def _loose(model):
        """Parameters whose gradients are accumulated by atomics or torch ops (zeroed per update)."""
        return (model.transformer.wte.weight, *[e.weight for e in model.value_embeds.values()],
                model.resid_lambdas, model.x0_lambdas, model.smear_gate.weight, model.smear_lambda,
                model.backout_lambda)

    @torch.no_grad()
    def refresh_shadows(self):
        lib = ext()
        for p, s in self.casts:
            if p.is_contiguous() and s.is_contiguous():
                lib.cast_bf16(p.detach(), s)
            else:
                s.copy_(p.detach())

    def zero_grads(self):
        for s in self.slots:
            s.fresh = True
        for z in self.zeroed:
            z.zero_()


class StepScratch:
    """Per-forward shared state: the fp32 accumulator of d(x0) over all layers."""

    def __init__(self, M, d, device):
        self.dx0 = torch.zeros(M, d, device=device, dtype=torch.float32)


# ---------------------------------------------------------------------------------- embedding
class EmbedFn(Function):
    @staticmethod
    def forward(ctx, idx, wte, model, scratch, T):
        lib = ext()
        M, d = idx.numel(), wte.shape[1]
        n = torch.empty(M, d, device=wte.device, dtype=torch.bfloat16)
        x = torch.empty_like(n)
        sig = torch.empty(M, device=wte.device, dtype=torch.float32)
        lib.embed_smear(wte, idx, model.smear_gate._w, model.smear_lambda.detach(), n, x, sig, T)
        ctx.save_for_backward(idx, n, sig)
        ctx.model, ctx.scratch, ctx.T = model, scratch, T
        return x

    @staticmethod
    def backward(ctx, dx):
        idx, n, sig = ctx.saved_tensors
        model, T = ctx.model, ctx.T
        lib = ext()
        M, d = n.shape
        B = M // T
        tot = (dx.float() + ctx.scratch.dx0).view(B, T, d)
        nf = n.float().view(B, T, d)
        lam = model.smear_lambda.detach().to(torch.bfloat16).float()
        s = sig.view(B, T)[:, 1:]
        gate = lam * s
        dn = tot.clone()
        dn[:, :-1] += gate[..., None] * tot[:, 1:]
        dg = (tot[:, 1:] * nf[:, :-1]).sum(-1)
        dz = dg * lam * s * (1 - s)
        w = model.smear_gate.weight.detach().view(-1)
        G_ = w.numel()
        dn[:, 1:, :G_] += dz[..., None] * w
        model.smear_lambda.main_grad += (dg * s).sum().view(1)
        model.smear_gate.weight.main_grad += (dz[..., None] * nf[:, 1:, :G_]).sum((0, 1)).view(1, -1)
        e = model.transformer.wte.weight.detach().index_select(0, idx)
        de = torch.empty_like(e)
        lib.norm_bwd(e, dn.view(M, d).to(torch.bfloat16), None, de)
        lib.embed_scatter(de, idx, model.transformer.wte.weight.main_grad)
        return None, None, None, None, None


# ---------------------------------------------------------------------------------- attention sublayer
class PreAttnFn(Function):
    """xm = a x + b x0;  qkv = rope/qk-norm/VE(norm(xm) Wqkv^T)."""

    @staticmethod
    def forward(ctx, x, x0, ab, attn, model, scratch, idx, layer, T, cos, sin):
        lib = ext()
        M, d = x.shape
        H, Hk, D = attn.n_head, attn.n_kv_head, attn.head_dim
        xm = torch.empty_like(x)
        h = torch.empty_like(x)
        lib.mix_norm_fwd(x, x0, ab, xm, h, None, 1.0)
        qkv = G.linear(h, attn._w_qkv)
        rstd = torch.empty(M, H + Hk, device=x.device, dtype=torch.float32)
        ve_table = model.value_embeds[str(layer)].weight.detach() if str(layer) in model.value_embeds else None
        gate = None
        if ve_table is not None and attn.ve_gate is not None:
            gate = torch.empty(M, Hk, device=x.device, dtype=torch.float32)
            lib.rope_norm_fwd(qkv, cos, sin, rstd, T, H, Hk, D, 1.2, ve_table, idx, h, attn.ve_gate._w, gate)
        else:
            ve_table = None
            lib.rope_norm_fwd(qkv, cos, sin, rstd, T, H, Hk, D, 1.2, None, None, None, None, None)
        ctx.save_for_backward(x, x0, ab, xm, h, qkv, rstd, idx, *(() if gate is None else (gate,)))
        ctx.attn, ctx.model, ctx.scratch, ctx.layer, ctx.T = attn, model, scratch, layer, T
        ctx.cos, ctx.sin, ctx.has_ve = cos, sin, gate is not None
        return xm, qkv

    @staticmethod
    def backward(ctx, dxm, dqkv):
        saved = ctx.saved_tensors
        x, x0, ab, xm, h, qkv, rstd, idx = saved[:8]
        gate = saved[8] if ctx.has_ve else None
        attn, model, layer = ctx.attn, ctx.model, ctx.layer
        lib = ext()
        H, Hk, D = attn.n_head, attn.n_kv_head, attn.head_dim
        dqkv = dqkv.contiguous().clone()
        if gate is not None:
            ve = model.value_embeds[str(layer)].weight
            dz = torch.empty_like(gate)
            lib.rope_norm_bwd(dqkv, qkv, ctx.cos, ctx.sin, rstd, ctx.T, H, Hk, D, 1.2, ve.detach(), idx, gate, dz,
                              ve.main_grad)
        else:
            lib.rope_norm_bwd(dqkv, qkv, ctx.cos, ctx.sin, rstd, ctx.T, H, Hk, D, 1.2, None, None, None, None, None)
        dh = G.dgrad(dqkv, attn._w_qkv)
        buf, acc = attn._g_qkv.take()
        G.wgrad(dqkv, h, buf, accumulate=acc)
        if gate is not None:
            gw = attn.ve_gate.weight
            C = gw.shape[1]
            hc = h[:, :C].float()
            gw.main_grad += dz.t() @ hc
            dh[:, :C] += (dz @ gw.detach().to(torch.bfloat16).float()).to(torch.bfloat16)
        if dxm is None:
            dxm = torch.zeros_like(x)
        dx = torch.empty_like(x)
        part = torch.empty(x.shape[0], 2, device=x.device, dtype=torch.float32)
        lib.mix_norm_bwd(x, x0, xm, dh, dxm.contiguous(), ab, dx, ctx.scratch.dx0, part)
        dab = part.sum(0)
        model.resid_lambdas.main_grad[layer:layer + 1] += dab[0:1]
        model.x0_lambdas.main_grad[layer:layer + 1] += dab[1:2]
        return dx, None, None, None, None, None, None, None, None, None, None


class OutProjFn(Function):
    """x1 = xm + y Wo^T."""

    @staticmethod
    def forward(ctx, y, xm, lin):
        x1 = G.linear_residual(y, lin._w, xm)
        ctx.save_for_backward(y)
        ctx.lin = lin
        return x1

    @staticmethod
    def backward(ctx, dx1):
        (y,) = ctx.saved_tensors
        lin = ctx.lin
        dx1 = dx1.contiguous()
        dy = G.dgrad(dx1, lin._w)
        buf, acc = lin._g.take()
        G.wgrad(dx1, y, buf, accumulate=acc)
        return dy, dx1, None


class MLPFn(Function):
    """x2 = x1 + relu(norm(x1) Wfc^T)^2 Wpr^T."""

    @staticmethod
    def forward(ctx, x1, mlp):
        lib = ext()
        h2 = torch.empty_like(x1)
        lib.mix_norm_fwd(x1, None, None, None, h2, None, 1.0)
        pre, u = G.linear_relu2(h2, mlp.c_fc._w)
        x2 = G.linear_residual(u, mlp.c_proj._w, x1)
        ctx.save_for_backward(x1, h2, pre, u)
        ctx.mlp = mlp
        return x2

    @staticmethod
    def backward(ctx, dx2):
        x1, h2, pre, u = ctx.saved_tensors
        mlp = ctx.mlp
        lib = ext()
        dx2 = dx2.contiguous()
        dpre = G.dgrad_relu2(dx2, mlp.c_proj._w, pre)
        buf, acc = mlp.c_proj._g.take()
        G.wgrad(dx2, u, buf, accumulate=acc)
        dh2 = G.dgrad(dpre, mlp.c_fc._w)
        buf, acc = mlp.c_fc._g.take()
        G.wgrad(dpre, h2, buf, accumulate=acc)
        dx1 = torch.empty_like(x1)
        lib.norm_bwd(x1, dh2, dx2, dx1)
        return dx1, None


# ---------------------------------------------------------------------------------- head + loss
class HeadLossFn(Function):
    """loss = CE(cap tanh(norm(x - lambda xb) Wh^T / cap), targets), mean over valid targets or sum."""

    @staticmethod
    def forward(ctx, x, xb, model, tgt, reduction):
        lib = ext()
        cfg = model.shell
        lam = model.backout_lambda.detach().to(torch.bfloat16)
        xo = x - lam * xb if xb is not None else x
        xo = xo.contiguous()
        hf = torch.empty_like(xo)
        lib.mix_norm_fwd(xo, None, None, None, hf, None, 1.0)
        M = hf.shape[0]
        if FUSED_HEAD_CE:
            W = model.lm_head._w
            Vp = W.shape[0]
            Gm = torch.empty(M, Vp, device=x.device, dtype=torch.bfloat16)
            part = torch.empty(M, (Vp + 127) // 128, device=x.device, dtype=torch.float32)
            ztgt = torch.zeros(M, device=x.device, dtype=torch.float32)
            rows = torch.empty(M, device=x.device, dtype=torch.float32)
            rscale = torch.empty_like(rows)
            rcorr = torch.empty_like(rows)
            lib.gemm_ce_fwd(hf, W, Gm, tgt, part, ztgt, rows, rscale, rcorr, cfg.vocab_size, cfg.softcap)
            del part
            saved = (Gm, rscale, rcorr)
        else:
            logits = G.linear(hf, model.lm_head._w)
            rows = torch.empty(M, device=x.device, dtype=torch.float32)
            lib.softcap_ce(logits, tgt, rows, None, cfg.vocab_size, cfg.softcap, CE_VARIANT)
            saved = (logits,)
        total = rows.sum()
        if reduction == "mean":
            count = (tgt != -1).sum().clamp_min(1).float()
            loss = total / count
            inv = (1.0 / count).reshape(1)
        else:
            loss = total
            inv = torch.ones(1, device=x.device, dtype=torch.float32)
        ctx.save_for_backward(hf, xo, xb if xb is not None else xo, inv, tgt, *saved)
        ctx.model, ctx.has_xb, ctx.fused = model, xb is not None, FUSED_HEAD_CE
        return loss

    @staticmethod
    def backward(ctx, g):
        hf, xo, xb, inv, tgt, *saved = ctx.saved_tensors
        model = ctx.model
        lib = ext()
        scale = (g.float().reshape(1) * inv).contiguous()
        W = model.lm_head._w
        buf, acc = model.lm_head._g.take()
        if ctx.fused:
            Gm, rscale, rcorr = saved
            # dlogits = scale (rscale G - rcorr onehot(target)); both terms go into the GEMMs
            dh = torch.empty_like(hf)
            lib.gemm_ce_dgrad(Gm, W, dh, tgt, rscale, rcorr, scale)
            hf_s = (hf.float() * rscale[:, None]).to(torch.bfloat16)
            G.wgrad(Gm, hf_s, buf, accumulate=acc, s_dev=scale)
            corr = hf.float() * (-(scale * rcorr))[:, None]
            lib.embed_scatter(corr, tgt.clamp_min(0), buf)
        else:
            (dlogits,) = saved
            dh = G.dgrad(dlogits, W, s_dev=scale)
            G.wgrad(dlogits, hf, buf, accumulate=acc, s_dev=scale)
        dxo = torch.empty_like(xo)
        lib.norm_bwd(xo, dh, None, dxo)
        dxb = None
        if ctx.has_xb:
            lam = model.backout_lambda.detach().to(torch.bfloat16)
            dxb = -(lam * dxo)
            model.backout_lambda.main_grad -= (dxo.float() * xb.float()).sum().view(1)
        return dxo, dxb, None, None, None


def fused_forward(model, idx, targets, reduction="mean"):
    """Training loss of the dense shell on CUDA (fp32 parameter gradients land in ``main_grad``)."""
    cfg = model.shell
    B, T = idx.shape
    st = model.fused_state()
    idx_f = idx.reshape(-1).contiguous()
    tgt_f = targets.reshape(-1).contiguous()
    d = cfg.n_embd
    scratch = StepScratch(B * T, d, idx.device)
    cos = model.cos[0, :T, 0].contiguous()
    sin = model.sin[0, :T, 0].contiguous()
    x0 = EmbedFn.apply(idx_f, model.transformer.wte.weight, model, scratch, T)
    x = x0
    n = cfg.n_layer
    backout = None
    for i, blk in enumerate(model.transformer.h):
        a = blk.attn
        with torch.no_grad():
            ab = torch.stack((model.resid_lambdas[i], model.x0_lambdas[i])).float().contiguous()
        xm, qkv = PreAttnFn.apply(x, x0, ab, a, model, scratch, idx_f, i, T, cos, sin)
        y = attention_fn(qkv, B, T, a.n_head, a.n_kv_head, a.head_dim, model.window_sizes[i][0])
        x = OutProjFn.apply(y, xm, a.c_proj)
        x = MLPFn.apply(x, blk.mlp)
        if i == n // 2:
            backout = x
    return HeadLossFn.apply(x, backout, model, tgt_f, reduction)
