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
from nexttransformer_b200.utils.trace import nvtx_range

# Cross-entropy kernel variant (0: automatic, 1: two-pass); kept selectable for numerics checks.
CE_VARIANT = 0
# True: the cross-entropy runs in the head GEMM's epilogue; False: GEMM + separate CE kernel.
FUSED_HEAD_CE = True
# Grouped expert GEMMs need the expert width and the model width in multiples of 64.
MIN_EXPERT_DIM = 64


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
    """bf16 weight shadows and fp32 gradient buffers of a shell model on CUDA.

    Two registrations, chosen by ``model.fused_supported()``:
      * trunk mode (the model's trunk runs ``fused_forward``): ``c_q | c_k | c_v`` of every
        shell attention share one packed shadow (one QKV GEMM) and one packed gradient buffer,
        the shell MLPs, the head and the embedding-side parameters get gradient buffers written
        by the fused Functions below;
      * in both modes every other eligible ``Linear`` of the model (linear / sparse / MLA mixers,
        looped-block adapters, plugin projections) gets a shadow and a gradient slot and runs on
        the GEMM engine through ``ops.dense.KernelLinear`` when it is called.
    Every registered parameter's ``main_grad`` is a view into these buffers.
    """

    def __init__(self, model, grad_alloc=None, plan_only=False):
        """``grad_alloc(shape)`` (optional) supplies the fp32 gradient buffers in a fixed order (a
        flat arena, e.g. in symmetric memory); ``plan_only`` only walks that order so the caller
        can size the arena, touching no parameter."""
        self.model = model
        self.trunk = bool(model.fused_supported())
        dev = model.get_device()
        f32, bf = torch.float32, torch.bfloat16
        self.slots = []        # GEMM-written gradients (fresh / accumulate)
        self.zeroed = []       # gradients accumulated with atomics or torch ops
        self.casts = []        # (fp32 master, bf16 shadow)
        self.kernel_linears = []
        self.arena = None
        self._plan = plan_only
        self._seen = set()
        # data-parallel overlap (optim.muon_adamw.MuonAdamW.overlap_with): the optimizer that
        # reduces each layer's gradients as soon as the last micro-batch's backward has produced
        # them, and whose parameter gathers each layer's forward waits for
        self.optimizer = None
        self.final_micro = False
        self._groups = None

        def grad(shape):
            if grad_alloc is not None:
                return grad_alloc(tuple(shape))
            return torch.zeros(tuple(shape), device=dev, dtype=f32)

        def shadow(p, out=None):
            out = out if out is not None else torch.empty(p.shape, device=dev, dtype=bf)
            self.casts.append((p, out))
            return out

        self._grad, self._shadow = grad, shadow
        self._register(model)
        if not plan_only:
            self.refresh_shadows()

    # ------------------------------------------------------------------ registration
    def _register(self, model):
        from nexttransformer_b200.models.moe import MoEFFN
        from nexttransformer_b200.models.shell import MLP, Block, CausalSelfAttention
        grad, shadow, plan = self._grad, self._shadow, self._plan
        dev = model.get_device()
        for blk in model.transformer.h:
            a, m = getattr(blk, "attn", None), getattr(blk, "mlp", None)
            if self.trunk and type(blk) is Block and type(a) is CausalSelfAttention:
                nq, nk, d = a.c_q.weight.shape[0], a.c_k.weight.shape[0], a.c_q.weight.shape[1]
                g = grad((nq + 2 * nk, d))
                if not plan:
                    a._w_qkv = torch.empty(nq + 2 * nk, d, device=dev, dtype=torch.bfloat16)
                    a._g_qkv = GradSlot(g)
                    self.slots.append(a._g_qkv)
                    for lin, lo, hi in ((a.c_q, 0, nq), (a.c_k, nq, nq + nk), (a.c_v, nq + nk, nq + 2 * nk)):
                        lin.weight.main_grad = g[lo:hi]
                        shadow(lin.weight, a._w_qkv[lo:hi])
                self._fused_linear(a.c_proj)
                if a.ve_gate is not None:
                    g = grad(a.ve_gate.weight.shape)
                    if not plan:
                        a.ve_gate._w = shadow(a.ve_gate.weight)
                        a.ve_gate.weight.main_grad = g
                        self.zeroed.append(g)
                self._seen.update(id(x) for x in (a.c_q, a.c_k, a.c_v, a.ve_gate))
            if self.trunk and type(blk) is Block and type(m) is MLP:
                self._fused_linear(m.c_fc)
                self._fused_linear(m.c_proj)
            if isinstance(m, MoEFFN):
                self._experts(m)
            self._generic(blk)
        if self.trunk:
            self._fused_linear(model.lm_head)
            if not plan:
                model.smear_gate._w = shadow(model.smear_gate.weight)
            for p in self._loose(model):
                g = grad(p.shape)
                if not plan:
                    p.main_grad = g
                    self.zeroed.append(g)
        self._generic(model)

    def _experts(self, moe):
        """Routed experts run as grouped GEMMs (``ops.moe``) on stacked bf16 shadows; each expert
        weight's ``main_grad`` is one slice of a stacked fp32 buffer the grouped weight-gradient
        GEMMs accumulate into (zeroed once per update).  The router stays on F.linear (fp32
        logits) and the shared expert runs through the generic kernel linears."""
        local = moe.local_experts()
        self._seen.add(id(moe.router))
        F_, d_ = local[0].c_fc.weight.shape
        if F_ % MIN_EXPERT_DIM or d_ % MIN_EXPERT_DIM:
            return
        for e in local:
            self._seen.update((id(e), id(e.c_fc), id(e.c_proj)))
        E = len(local)
        gf, gp = self._grad((E, F_, d_)), self._grad((E, d_, F_))
        if self._plan:
            return
        dev = local[0].c_fc.weight.device
        moe._w_fc = torch.empty(E, F_, d_, device=dev, dtype=torch.bfloat16)
        moe._w_proj = torch.empty(E, d_, F_, device=dev, dtype=torch.bfloat16)
        moe._g_fc, moe._g_proj = gf, gp
        for j, e in enumerate(local):
            e.c_fc.weight.main_grad = gf[j]
            e.c_proj.weight.main_grad = gp[j]
            self._shadow(e.c_fc.weight, moe._w_fc[j])
            self._shadow(e.c_proj.weight, moe._w_proj[j])
        self.zeroed += [gf, gp]

    def _fused_linear(self, lin):
        """A Linear whose GEMMs are issued by the fused trunk Functions."""
        g = self._grad(lin.weight.shape)
        self._seen.add(id(lin))
        if self._plan:
            return
        lin._w = self._shadow(lin.weight)
        lin.weight.main_grad = g
        lin._g = GradSlot(g)
        self.slots.append(lin._g)

    def _generic(self, module):
        """Every not yet registered, eligible ``Linear`` under ``module`` runs on the GEMM engine."""
        from nexttransformer_b200.models.shell import Linear
        from nexttransformer_b200.ops.dense import linear_eligible
        for lin in module.modules():
            if not isinstance(lin, Linear) or id(lin) in self._seen or not linear_eligible(lin.weight):
                continue
            self._seen.add(id(lin))
            g = self._grad(lin.weight.shape)
            if self._plan:
                continue
            lin._w = self._shadow(lin.weight)
            lin.weight.main_grad = g
            lin._g = GradSlot(g)
            lin.weight._nt_slot = lin._g
            lin._kernel = True
            self.slots.append(lin._g)
            self.kernel_linears.append(lin)

    # ------------------------------------------------------------------ overlap hooks
    def use_groups(self):
        """Forward-use groups: -1 the embedding side and every shared scalar, i the parameters of
        layer i (with its value-embedding table), n_layer the head."""
        if self._groups is None:
            model = self.model
            n = len(model.transformer.h)
            groups = {}
            taken = set()
            for i, blk in enumerate(model.transformer.h):
                ps = list(blk.parameters())
                if str(i) in model.value_embeds:
                    ps.append(model.value_embeds[str(i)].weight)
                groups[i] = ps
                taken.update(id(p) for p in ps)
            groups[n] = [model.lm_head.weight]
            taken.add(id(model.lm_head.weight))
            groups[-1] = [p for p in model.parameters() if id(p) not in taken]
            self._groups = groups
        return self._groups

    def grads_ready(self, group, tables=True):
        """Called by the backward once group ``group``'s kernel-written gradients are final
        (``tables``: the layer's value-embedding table included)."""
        if self.final_micro and self.optimizer is not None:
            with nvtx_range(f"group{group}.reduce_issue"):
                self._issue(group, tables)

    def _issue(self, group, tables):
        model = self.model
        skip = set() if tables or str(group) not in model.value_embeds else \
            {id(model.value_embeds[str(group)].weight)}
        self.optimizer.issue_reduce([p for p in self.use_groups()[group] if getattr(p, "main_grad", None)
                                     is not None and p.requires_grad and id(p) not in skip])

    def params_needed(self, group):
        """Called by the forward before it reads group ``group``'s parameters."""
        if self.optimizer is not None:
            with nvtx_range(f"group{group}.gather_wait"):
                self.optimizer.wait_gathers(group)

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
        model._fused.grads_ready(layer)
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
        model._fused.grads_ready(len(model.transformer.h))
        return dxo, dxb, None, None, None


def fused_forward(model, idx, targets, reduction="mean"):
    """Training loss of a shell model on CUDA: ``(lm_loss, aux)`` with ``aux`` the sum of the
    mixers' auxiliary losses (None when no mixer has one).

    Per layer the shell's own attention and MLP run the fused Functions above; any other mixer
    (linear, sparse, MLA) or FFN (MoE) runs its own forward between the kernel mix+RMSNorm and
    a residual add, with its projections on the GEMM engine (``ops.dense``).  fp32 parameter
    gradients land in ``main_grad``."""
    cfg = model.shell
    B, T = idx.shape
    model.fused_state()
    idx_f = idx.reshape(-1).contiguous()
    tgt_f = targets.reshape(-1).contiguous()
    scratch = StepScratch(B * T, cfg.n_embd, idx.device)
    cos = model.cos[0, :T, 0].contiguous()
    sin = model.sin[0, :T, 0].contiguous()
    cos_sin = (model.cos[:, :T], model.sin[:, :T])
    st = model._fused
    st.params_needed(-1)
    x0 = EmbedFn.apply(idx_f, model.transformer.wte.weight, model, scratch, T)
    x = x0
    n = cfg.n_layer
    backout = aux = None
    for i, blk in enumerate(model.transformer.h):
        with nvtx_range(f"layer{i}.forward"):
            x, aux = _layer_forward(model, st, i, blk, x, x0, aux, idx_f, B, T, cos, sin, cos_sin, scratch)
        if i == n // 2:
            backout = x
    st.params_needed(n)
    with nvtx_range("head.forward"):
        return HeadLossFn.apply(x, backout, model, tgt_f, reduction), aux


def _layer_forward(model, st, i, blk, x, x0, aux, idx_f, B, T, cos, sin, cos_sin, scratch):
    """One layer of ``fused_forward``: (new state, running auxiliary loss)."""
    from nexttransformer_b200.models.shell import MLP
    from nexttransformer_b200.ops.dense import MixNormFn, rms_norm, table_lookup
    M, d = x.shape
    a, mlp = blk.attn, blk.mlp
    st.params_needed(i)
    window = model.layer_window(i)
    with torch.no_grad():
        ab = torch.stack((model.resid_lambdas[i], model.x0_lambdas[i])).float().contiguous()
    if getattr(a, "_w_qkv", None) is not None:
        xm, qkv = PreAttnFn.apply(x, x0, ab, a, model, scratch, idx_f, i, T, cos, sin)
        y = attention_fn(qkv, B, T, a.n_head, a.n_kv_head, a.head_dim, window)
        x = OutProjFn.apply(y, xm, a.c_proj)
    else:
        xm, h = MixNormFn.apply(x, x0, ab, model, scratch, i)
        key = str(i)
        ve = table_lookup(idx_f, model.value_embeds[key].weight).view(B, T, -1) \
            if key in model.value_embeds else None
        y = a(h.view(B, T, d), ve, cos_sin, (window, 0), None)
        x = xm + y.reshape(M, d).to(xm.dtype)
        part = getattr(a, "last_aux", None)
        if torch.is_tensor(part):
            aux = part if aux is None else aux + part
    if type(mlp) is MLP and getattr(mlp.c_fc, "_g", None) is not None and not mlp.c_fc._kernel:
        x = MLPFn.apply(x, mlp)
    else:
        h2 = rms_norm(x)
        x = x + mlp(h2.view(B, T, d)).reshape(M, d).to(x.dtype)
        part = getattr(mlp, "last_aux", None)
        if torch.is_tensor(part):
            aux = part if aux is None else aux + part
    return x, aux
