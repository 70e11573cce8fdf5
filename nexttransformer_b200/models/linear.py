"""Linear-attention mixers: DeltaNet, GLA, KDA, RetNet, ELU+1 (plain / norm / qknorm), Gated DeltaNet.

Behaviour and parameter names follow ``nexttransformer/models/linear.py`` of the reference:
q/k/v projections (short causal depthwise conv + SiLU for the delta-rule family), value
embeddings gated per head, method feature maps (ELU+1, L2-normalised q/k, xPos-style
retention rotation), per-token gates (GLA low-rank sigmoid gate, KDA per-feature decay,
GDN per-head Mamba-2 decay), output RMSNorm x gain and SiLU output gate.

Two mathematically equal forms of every recurrence are provided:
  * ``recurrent_scan`` - the token-by-token recurrence (the oracle);
  * ``chunk_scan`` - the chunked WY / UT form used for training (chunk 64): within a chunk the
    delta-rule corrections are solved as one unit-lower-triangular system, and one state
    update is carried per chunk.  ``ops.linear_attention`` runs it on CUDA.
"""
from contextlib import contextmanager
import math

import torch
from torch import nn
from torch.nn import functional as F

from nexttransformer_b200.models.shell import Linear, has_ve, norm

ELU_QK_TEMPERATURE = 8.
GDN_A_RANGE, GDN_DT_RANGE, GDN_DT_FLOOR = (0., 16.), (1e-3, 1e-1), 1e-4
CHUNK_BACKENDS = {"fla_chunk64": 64}


def acc_dtype(x):
    return torch.float32 if x.dtype in (torch.float16, torch.bfloat16) else x.dtype


@torch.no_grad()
def init_gdn_gate(log_decay, dt_bias):
    """A ~ U(0, 16) stored as log A; dt log-uniform in [1e-3, 1e-1] (floor 1e-4) stored as softplus^-1(dt)."""
    log_decay.copy_(torch.empty_like(log_decay).uniform_(*GDN_A_RANGE).log())
    lo, hi = math.log(GDN_DT_RANGE[0]), math.log(GDN_DT_RANGE[1])
    dt = (torch.rand_like(dt_bias) * (hi - lo) + lo).exp().clamp_min(GDN_DT_FLOOR)
    dt_bias.copy_(dt + torch.log(-torch.expm1(-dt)))


def elu_feature_map(x):
    """ELU(x) + 1 evaluated without cancellation; the unused exp branch is clamped."""
    x = x.to(acc_dtype(x))
    return torch.where(x > 0, x + 1, x.clamp_max(0).exp())


# ---------------------------------------------------------------------------- recurrence
def recurrent_scan(q, k, v, *, kind, decay=None, beta=None, initial_state=None, eps=1e-6):
    """Token recurrence on [B, T, H, D]; ``decay`` is multiplicative (not log).

    deltanet / kda / gdn:  S <- diag(decay) S;  S <- S + k (beta (v - k^T S))^T;  o = q^T S
    gla / retnet:          S <- diag(decay) S + k v^T;                           o = q^T S
    elu_*:                 S <- S + k v^T (and z <- z + k for elu_linear: o = q^T S / (q.z + eps))
    Returns (outputs, final state).
    """
    dtype = q.dtype
    q, k, v = (x.to(acc_dtype(x)) for x in (q, k, v))
    B, T, H, D = q.shape
    if kind == "gdn":
        kind, decay = "kda", decay.expand(B, T, H, D)
    S = q.new_zeros(B, H, D, v.shape[-1])
    z = q.new_zeros(B, H, D)
    if initial_state is not None:
        if kind == "elu_linear":
            S, z = initial_state
        else:
            S = initial_state
    outs = []
    # per-token views through unbind: its backward stacks the token gradients once (indexing
    # q[:, t] would add T full-size gradient buffers, a cost quadratic in T)
    qs, ks, vs = q.unbind(1), k.unbind(1), v.unbind(1)
    ds = decay.unbind(1) if decay is not None else None
    bs = beta.unbind(1) if beta is not None else None
    for t in range(T):
        qt, kt, vt = qs[t], ks[t], vs[t]
        if decay is not None:
            S = S * ds[t].to(q).unsqueeze(-1)
        if kind in ("deltanet", "kda"):
            pred = torch.einsum("bhd,bhde->bhe", kt, S)
            S = S + kt.unsqueeze(-1) * ((vt - pred) * bs[t].to(q).unsqueeze(-1)).unsqueeze(-2)
        else:
            S = S + kt.unsqueeze(-1) * vt.unsqueeze(-2)
        o = torch.einsum("bhd,bhde->bhe", qt, S)
        if kind == "elu_linear":
            z = z + kt
            o = o / ((qt * z).sum(-1, keepdim=True) + eps)
        outs.append(o)
    final = (S, z) if kind == "elu_linear" else S
    return torch.stack(outs, 1).to(dtype), final


# ---------------------------------------------------------------------------- chunk form
def _chunked(x, C):
    """[B, T, H, ...] -> [B, H, N, C, ...] with zero padding of the last chunk."""
    pad = -x.shape[1] % C
    if pad:
        x = F.pad(x, (0, 0) * (x.dim() - 2) + (0, pad))
    return x.unflatten(1, (x.shape[1] // C, C)).movedim(3, 1)


def _tril(C, device, strict=False):
    return torch.ones(C, C, dtype=torch.bool, device=device).tril(-1 if strict else 0)


def _delta_terms(q, k, v, g, beta, C, per_feature):
    """Per-chunk terms of the gated delta rule.  g: log decay per token (per head [..,C] or per
    feature [..,C,D]).

    Inside chunk n with cumulative log decay b_i (<= 0 increments):
      (I + strict_tril(beta_i k~_i . k^_j)) [w | u0] = beta [k~ | v],   k~ = k e^{b}, k^ = k e^{-b}
    and the scan below runs
      u = u0 - w S,   o = (q e^{b}) S + tril((q e^{b}) . k^) u,   S <- e^{b_C} S + (k e^{b_C - b})^T u
    (per-head gates use pairwise e^{b_i - b_j} <= 1 directly, so no factor can overflow).
    Returns (w, u0, qt, kc, aqk, carry) with carry None (no decay), [..,N,1,1] or [..,N,D,1].
    """
    causal = _tril(C, q.device)
    wgt = beta[..., None]
    if g is None:
        akk = k @ k.transpose(-1, -2)
        aqk = (q @ k.transpose(-1, -2)).masked_fill(~causal, 0)
        kt, qt, kc = k, q, k
        carry = None
    elif per_feature:
        b = g.cumsum(-2)
        kt, qt, kinv = k * b.exp(), q * b.exp(), k * (-b).exp()
        akk = kt @ kinv.transpose(-1, -2)
        aqk = (qt @ kinv.transpose(-1, -2)).masked_fill(~causal, 0)
        last = b[..., -1:, :]
        kc = k * (last - b).exp()
        carry = last.squeeze(-2).exp()[..., :, None]                  # [B,H,N,D,1]
    else:
        b = g.cumsum(-1)
        pair = (b[..., :, None] - b[..., None, :]).masked_fill(~causal, -math.inf).exp()
        akk = (k @ k.transpose(-1, -2)) * pair
        aqk = (q @ k.transpose(-1, -2)) * pair
        kt, qt = k * b.exp()[..., None], q * b.exp()[..., None]
        last = b[..., -1:]
        kc = k * (last - b).exp()[..., None]
        carry = last.exp()[..., None]                                 # [B,H,N,1,1]
    rhs = torch.cat((wgt * kt, wgt * v), -1)
    sol = torch.linalg.solve_triangular(wgt * akk, rhs, upper=False, unitriangular=True)
    w, u0 = sol.split((k.shape[-1], v.shape[-1]), -1)
    return w, u0, qt, kc, aqk, carry


def _delta_scan(w, u0, qt, kc, aqk, carry):
    """The sequential part over chunks (state S [Dk, Dv] carried in the input dtype)."""
    N = qt.shape[2]
    S = None
    outs = []
    for n in range(N):
        if S is None:
            u = u0[:, :, n]
            outs.append(aqk[:, :, n] @ u)
        else:
            u = u0[:, :, n] - w[:, :, n] @ S
            outs.append(qt[:, :, n] @ S + aqk[:, :, n] @ u)
        if n == N - 1:
            break
        upd = kc[:, :, n].transpose(-1, -2) @ u
        if S is None:
            S = upd
        else:
            S = (S if carry is None else S * carry[:, :, n]) + upd
    return torch.stack(outs, 2)


def _delta_chunks(q, k, v, g, beta, C, per_feature):
    """Gated delta rule over chunks: the per-chunk terms, then the scan."""
    return _delta_scan(*_delta_terms(q, k, v, g, beta, C, per_feature))


def _scalar_decay_chunks(q, k, v, g, C):
    """Linear attention with an optional per-head scalar log decay (RetNet, ELU+1 numerator)."""
    causal = _tril(C, q.device)
    sc = q @ k.transpose(-1, -2)
    if g is None:
        sc = sc.masked_fill(~causal, 0)
        carry = None
    else:
        b = g.cumsum(-1)
        sc = sc * (b[..., :, None] - b[..., None, :]).masked_fill(~causal, -math.inf).exp()
        q = q * b[..., None].exp()
        k = k * (b[..., -1:] - b)[..., None].exp()
        carry = b[..., -1].exp()
    out = sc @ v
    N = q.shape[2]
    S, inter = None, []
    for n in range(N):
        inter.append(q.new_zeros(*q[:, :, n].shape[:-1], v.shape[-1]) if S is None else q[:, :, n] @ S)
        if n == N - 1:
            break
        upd = k[:, :, n].transpose(-1, -2) @ v[:, :, n]
        S = upd if S is None else (S if carry is None else S * carry[:, :, n][..., None, None]) + upd
    return out + torch.stack(inter, 2)


def _kda_kernel_ok(q, k, v):
    """The fused KDA chunk kernels take these operands (CUDA, bf16, head size 128, chunk 64)."""
    if not q.is_cuda:
        return False
    from nexttransformer_b200.ops.linear_attention import fused_chunk_supported
    return fused_chunk_supported(q, k, v, 64)


def _gla_kernel_ok(q, v):
    from nexttransformer_b200.ops.linear_attention import gla_supported
    return gla_supported(q, v)


def chunk_scan(q, k, v, *, kind, g=None, beta=None, chunk):
    """Chunked training form; g is a log decay (KDA [B,T,H,D], GDN/RetNet [B,T,H], None otherwise)."""
    T = q.shape[1]
    q, k, v = (_chunked(x, chunk) for x in (q, k, v))
    if kind == "kda":
        out = _delta_chunks(q, k, v, _chunked(g, chunk), _chunked(beta, chunk), chunk, per_feature=True)
    elif kind in ("gdn", "deltanet"):
        out = _delta_chunks(q, k, v, None if g is None else _chunked(g, chunk), _chunked(beta, chunk), chunk,
                            per_feature=False)
    else:
        out = _scalar_decay_chunks(q, k, v, None if g is None else _chunked(g, chunk), chunk)
    return out.movedim(1, 3).flatten(1, 2)[:, :T]


@contextmanager
def ieee_fp32():
    prev = torch.get_float32_matmul_precision()
    torch.set_float32_matmul_precision("highest")
    try:
        yield
    finally:
        torch.set_float32_matmul_precision(prev)


def _elu_numerator(q, k, v, C):
    """sum_{j<=i} (q_i . k_j) v_j with the chunk loop batched (one cumsum of chunk states)."""
    T = q.shape[1]
    q, k, v = (_chunked(x, C) for x in (q, k, v))
    out = (q @ k.transpose(-1, -2)).masked_fill(~_tril(C, q.device), 0) @ v
    if q.shape[2] > 1:
        states = (k[:, :, :-1].transpose(-1, -2) @ v[:, :, :-1]).cumsum(2)
        out = torch.cat((out[:, :, :1], out[:, :, 1:] + q[:, :, 1:] @ states), 2)
    return out.movedim(1, 3).flatten(1, 2)[:, :T]


class _ELUChunk(torch.autograd.Function):
    """ELU+1 chunk forms with forward and backward in IEEE fp32 (TF32 off): the q/k gradients are
    small differences of large terms once the feature sums grow."""

    @staticmethod
    def forward(ctx, q, k, v, chunk, kind):
        acc = torch.float64 if q.dtype == torch.float64 else torch.float32
        leaves = [x.detach().to(acc).requires_grad_(x.requires_grad) for x in (q, k, v)]
        with ieee_fp32(), torch.enable_grad():
            num = _elu_numerator(*leaves, chunk)
            y = num / ((leaves[0] * leaves[1].cumsum(1)).sum(-1, keepdim=True) + 1e-6) if kind == "elu_linear" else num
        ctx.graph, ctx.dtypes = (leaves, y), (q.dtype, k.dtype, v.dtype)
        return y.detach().to(q.dtype)

    @staticmethod
    def backward(ctx, grad):
        leaves, y = ctx.graph
        need = [x for x in leaves if x.requires_grad]
        with ieee_fp32():
            got = iter(torch.autograd.grad(y, need, grad.to(y.dtype)))
        ctx.graph = None
        return (*(next(got).to(d) if x.requires_grad else None for x, d in zip(leaves, ctx.dtypes)), None, None)


def chunk_attention(q, k, v, *, kind, g=None, beta=None, chunk, qk_l2norm_scale=None):
    """Chunked mixing entry point.  GDN passes raw q/k: q <- scale q/|q|, k <- k/|k| happen here."""
    if (kind == "gdn") != (qk_l2norm_scale is not None):
        raise ValueError("GDN, and only GDN, normalises q/k inside chunk_attention")
    if kind in ("elu_linear", "elu_norm", "elu_qknorm"):
        return _ELUChunk.apply(q, k, v, chunk, kind)
    if q.is_cuda and kind in ("gdn", "kda", "deltanet"):
        from nexttransformer_b200.ops.linear_attention import delta_chunk_cuda
        return delta_chunk_cuda(q, k, v, kind=kind, g=g, beta=beta, chunk=chunk, qk_l2norm_scale=qk_l2norm_scale)
    if kind == "retnet":
        g = g.expand(*q.shape[:2], -1)
        if q.is_cuda:
            from nexttransformer_b200.ops.linear_attention import scalar_chunk_cuda
            return scalar_chunk_cuda(q, k, v, g, chunk)
    if qk_l2norm_scale is not None:
        q, k = F.normalize(q, dim=-1) * qk_l2norm_scale, F.normalize(k, dim=-1)
    return chunk_scan(q, k, v, kind=kind, g=g, beta=beta, chunk=chunk)


def gated_rms_norm(y, gate, gain):
    """RMSNorm(y) * gain * SiLU(gate) with fp32 internals (eps: fp32 machine epsilon)."""
    yf = y.float()
    out = yf * torch.rsqrt(yf.pow(2).mean(-1, keepdim=True) + torch.finfo(torch.float32).eps)
    return (out * gain.float() * F.silu(gate.float())).to(y.dtype)


class CausalDepthwise(nn.Module):
    """Causal depthwise conv (width `size`) + SiLU on [B, T, D]."""

    def __init__(self, width, size, fused=False):
        super().__init__()
        self.weight = nn.Parameter(torch.empty(width, 1, size))
        nn.init.normal_(self.weight, std=size ** -.5)
        self.size = size
        self.fused = fused

    def forward(self, x):
        if x.is_cuda and self.fused:
            from nexttransformer_b200.ops.linear_attention import causal_conv_silu
            return causal_conv_silu(x, self.weight)
        y = F.conv1d(F.pad(x.transpose(1, 2), (self.size - 1, 0)), self.weight.to(x.dtype), groups=x.shape[-1])
        return F.silu(y.transpose(1, 2))


class LinearMixer(nn.Module):
    """Linear-attention mixer inside the shared block (called as (x, ve, cos_sin, window, kv_cache))."""

    def __init__(self, config, layer_idx, kind=None):
        super().__init__()
        self.config = config
        self.kind = kind or ("kda" if config.method == "kda_no_ve" else config.method)
        d, h = config.width, config.heads
        self.c_q = Linear(d, d, bias=False)
        self.c_k = Linear(d, d, bias=False)
        self.c_v = Linear(d, d, bias=False)
        self.c_proj = Linear(d, d, bias=False)
        self.ve_gate = Linear(12, h, bias=False) if has_ve(layer_idx, config.n_layer) else None
        self.last_aux = None
        self.last_stats = {}
        if self.kind in ("deltanet", "kda", "gdn"):
            fused = config.backend in CHUNK_BACKENDS
            self.q_conv = CausalDepthwise(d, config.conv_size, fused)
            self.k_conv = CausalDepthwise(d, config.conv_size, fused)
            self.v_conv = CausalDepthwise(d, config.conv_size, fused)
            self.beta_proj = Linear(d, h, bias=False)
        if self.kind in ("gla", "kda"):
            self.gate_down = Linear(d, config.gate_rank, bias=False)
            self.gate_up = Linear(config.gate_rank, d, bias=False)
        if self.kind == "kda":
            self.log_decay = nn.Parameter(torch.zeros(h, config.head_dim))
            self.dt_bias = nn.Parameter(torch.full((h, config.head_dim), -3.))
        if self.kind == "gdn":
            self.decay_proj = Linear(d, h, bias=False)
            self.log_decay = nn.Parameter(torch.empty(h))
            self.dt_bias = nn.Parameter(torch.empty(h))
            init_gdn_gate(self.log_decay, self.dt_bias)
        if self.kind in ("gla", "kda", "gdn", "retnet"):
            self.output_gate = Linear(d, d, bias=False)
        if self.kind != "elu_linear":
            self.output_gain = nn.Parameter(torch.ones(config.head_dim))

    @staticmethod
    def _retention_rotation(x):
        d = x.shape[-1]
        inv = 10000. ** (-torch.arange(0, d, 2, device=x.device, dtype=torch.float32) / d)
        ang = torch.arange(x.shape[1], device=x.device)[:, None] * inv[None]
        cos, sin = ang.cos().to(x)[None, :, None], ang.sin().to(x)[None, :, None]
        ev, od = x[..., 0::2], x[..., 1::2]
        return torch.stack((ev * cos - od * sin, ev * sin + od * cos), -1).flatten(-2)

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise NotImplementedError("linear mixers carry their own recurrent state; no KV cache")
        c = self.config
        chunked = c.backend in CHUNK_BACKENDS
        B, T, d = x.shape
        H, D = c.heads, c.head_dim
        q, k, v = self.c_q(x), self.c_k(x), self.c_v(x)
        if self.kind in ("deltanet", "kda", "gdn"):
            q, k, v = self.q_conv(q), self.k_conv(k), self.v_conv(v)
        q, k, v = (z.reshape(B, T, H, D) for z in (q, k, v))
        if ve is not None and self.ve_gate is not None:
            v = v + (3 * torch.sigmoid(self.ve_gate(x[..., :12]))).unsqueeze(-1) * ve.reshape_as(v)
        beta = decay = None
        # KDA on the fused kernels: the gate and the q / k normalisation are formed inside them
        kda_fused = self.kind == "kda" and chunked and x.dtype == torch.bfloat16 and _kda_kernel_ok(q, k, v)
        if self.kind in ("elu_linear", "elu_norm", "elu_qknorm"):
            if self.kind == "elu_qknorm":
                q, k = (norm(z.to(acc_dtype(z))) * ELU_QK_TEMPERATURE for z in (q, k))
            q, k = elu_feature_map(q), elu_feature_map(k)
        elif self.kind in ("deltanet", "kda", "gdn"):
            if not (self.kind == "gdn" and chunked) and not kda_fused:
                q, k = F.normalize(q, dim=-1), F.normalize(k, dim=-1)
                q = q * D ** -.5
            beta = torch.sigmoid(self.beta_proj(x))
        elif self.kind == "retnet":
            q, k = self._retention_rotation(q), self._retention_rotation(k)
            q = q * D ** -.5
            gamma = 1 - 2. ** (-5 - torch.arange(H, device=x.device, dtype=torch.float32))
            decay = gamma.log() if chunked else gamma[None, None, :, None].expand(B, T, -1, 1)
        elif self.kind == "gla":
            q = q * D ** -.5
        if self.kind in ("gla", "kda"):
            gate = self.gate_up(self.gate_down(x)).reshape(B, T, H, D)
            if self.kind == "gla":
                decay = (F.logsigmoid(gate.float()) / 16).exp()
            elif not kda_fused:
                decay = -self.log_decay.exp() * F.softplus(gate.float() + self.dt_bias)
                if not chunked:
                    decay = decay.exp()
        elif self.kind == "gdn":
            decay = -self.log_decay.exp() * F.softplus(self.decay_proj(x).float() + self.dt_bias)
            if not chunked:
                decay = decay.exp().unsqueeze(-1)
        if kda_fused:
            from nexttransformer_b200.ops.linear_attention import kda_chunk_cuda
            y = kda_chunk_cuda(q, k, v, gate, self.log_decay, self.dt_bias, beta, qk_l2norm_scale=D ** -.5)
        elif chunked:
            y = chunk_attention(q, k, v, kind=self.kind, g=decay, beta=beta, chunk=CHUNK_BACKENDS[c.backend],
                                qk_l2norm_scale=D ** -.5 if self.kind == "gdn" else None)
        elif self.kind == "gla" and x.is_cuda and _gla_kernel_ok(q, v):
            # the same recurrence in the chunk form on the scan kernels (log decay, not its exp)
            from nexttransformer_b200.ops.linear_attention import gla_chunk_cuda
            y = gla_chunk_cuda(q, k, v, F.logsigmoid(gate.float()) / 16)
        elif self.kind == "retnet" and x.is_cuda and _gla_kernel_ok(q, v):
            # the retention recurrence in the chunk form on the scan kernels (per-head log decay)
            from nexttransformer_b200.ops.linear_attention import scalar_chunk_cuda
            y = scalar_chunk_cuda(q, k, v, gamma.log()[None, None].expand(B, T, -1), 64)
        else:
            y, _ = recurrent_scan(q, k, v, kind=self.kind, decay=decay, beta=beta)
        gated = self.kind in ("gdn", "kda") and chunked and y.is_cuda
        if self.kind in ("elu_norm", "elu_qknorm"):
            y = F.rms_norm(y, (D,), eps=torch.finfo(x.dtype).eps)
            y = (y * self.output_gain.to(x.dtype)).to(x.dtype)
        elif self.kind == "elu_linear":
            y = y.to(x.dtype)
        elif gated:
            # one kernel each way (ops.linear_attention), the fp32 torch expression elsewhere
            from nexttransformer_b200.ops.linear_attention import gated_rms_norm as gated_rms_norm_cuda
            y = gated_rms_norm_cuda(y, self.output_gate(x).reshape(B, T, H, D), self.output_gain)
        else:
            y = norm(y) * self.output_gain.to(y.dtype)
        y = y.reshape(B, T, d)
        if hasattr(self, "output_gate") and not gated:
            y = y * F.silu(self.output_gate(x))
        self.last_aux = x.new_zeros(())
        self.last_stats = {"state_precision": "fp32-carry" if chunked else str(acc_dtype(x)),
                           "backend": c.backend, "sequence_length": T}
        return self.c_proj(y)
