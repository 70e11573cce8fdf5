"""The shared decoder shell (nanochat-style d24 backbone) and its dense attention / MLP blocks.

Behaviour follows the reference backbone (``nexttransformer/models/backbone.py``): token
embedding -> RMSNorm -> smear gate -> blocks on ``resid_lambda * x + x0_lambda * x0`` ->
backout of the mid-depth residual -> RMSNorm -> LM head -> soft-cap 15 -> cross entropy.
Attention uses QK-norm x 1.2, RoPE (base 1e5, rotation by -theta), value embeddings on
alternating layers gated by ``3 sigmoid(W x[:12])``, GQA and SSSL windows; the MLP is ReLU^2.
Parameter names and shapes are the reference's, so checkpoints load in both directions.

Two execution paths compute the same function:
  * ``forward_eager`` - plain PyTorch ops on any device.  It is the CPU path, the numerical
    oracle of the kernels and the graph the FLOP ledger audits.
  * ``models.fused_dense`` - CUDA tensors: the sm_100a kernels with fused epilogues
    (``csrc/``), fp32 gradients accumulated straight into ``main_grad`` buffers.
"""
from dataclasses import dataclass
import math

import torch
from torch import nn
import torch.nn.functional as F

from nexttransformer_b200.utils.dtype import COMPUTE_DTYPE


@dataclass(frozen=True)
class ShellConfig:
    sequence_len: int = 2048
    vocab_size: int = 32768
    n_layer: int = 12
    n_head: int = 6
    n_kv_head: int = 6
    n_embd: int = 768
    mlp_width: int = 0          # 0: 4 * n_embd
    window_pattern: str = "SSSL"
    value_embeddings: bool = True
    softcap: float = 15.0
    pad_vocab_to: int = 64
    attn_head_dim: int = 0      # 0: n_embd / n_head

    @property
    def head_dim(self):
        return self.attn_head_dim or self.n_embd // self.n_head

    @property
    def ffn(self):
        return self.mlp_width or 4 * self.n_embd

    @property
    def padded_vocab(self):
        p = self.pad_vocab_to
        return (self.vocab_size + p - 1) // p * p


def norm(x):
    """RMSNorm without weight (eps: torch's default for the input dtype)."""
    return F.rms_norm(x, (x.size(-1),))


class Linear(nn.Linear):
    """Linear with fp32 master weight, cast to the activation dtype at use (no autocast).

    Once the kernel state of a model on CUDA has registered the layer (``_kernel``: a bf16
    shadow ``_w`` written by the optimizer and an fp32 gradient slot ``_g``), bf16 inputs run
    on the sm_100a GEMM engine (``ops.dense.KernelLinear``); everything else uses ``F.linear``."""

    _kernel = False

    def forward(self, x):
        if self._kernel and x.is_cuda and x.dtype == torch.bfloat16:
            from nexttransformer_b200.ops.dense import kernel_linear
            return kernel_linear(x, self)
        return F.linear(x, self.weight.to(dtype=x.dtype))


def has_ve(layer, n_layer):
    """Value embeddings on alternating layers; the last layer always has one."""
    return layer % 2 == (n_layer - 1) % 2


def apply_rotary_emb(x, cos, sin):
    """Rotate (x1, x2) halves by -theta: y1 = x1 c + x2 s, y2 = -x1 s + x2 c."""
    half = x.shape[-1] // 2
    x1, x2 = x[..., :half], x[..., half:]
    return torch.cat((x1 * cos + x2 * sin, x1 * (-sin) + x2 * cos), -1)


def window_mask(T, window, device):
    """Boolean [T, T] mask of keys a query may see: causal and, if window >= 0, at most `window` back."""
    i = torch.arange(T, device=device)[:, None]
    j = torch.arange(T, device=device)[None, :]
    m = j <= i
    if 0 <= window < T - 1:
        m = m & (i - j <= window)
    return m


def sdpa(q, k, v, window):
    """Causal attention on [B, T, H, D] tensors with an optional left window (GQA by repetition).

    CUDA bf16 tensors of a supported head dim run the sm_100a flash-attention kernels; everything else
    (CPU, fp32 oracles, FakeTensor audits) runs PyTorch's SDPA.
    """
    if q.is_cuda:
        from nexttransformer_b200.ops import attention as _attn
        if _attn.kernel_supports(q, k, v):
            return _attn.attention_bthd(q, k, v, window)
    B, T, H, D = q.shape
    q, k, v = q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2)
    gqa = k.shape[1] != H
    if window < 0 or window >= T - 1:
        y = F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=gqa)
    else:
        y = F.scaled_dot_product_attention(q, k, v, attn_mask=window_mask(T, window, q.device), enable_gqa=gqa)
    return y.transpose(1, 2)


class CausalSelfAttention(nn.Module):
    def __init__(self, cfg: ShellConfig, layer: int):
        super().__init__()
        self.layer_idx = layer
        self.n_head, self.n_kv_head, self.head_dim = cfg.n_head, cfg.n_kv_head, cfg.head_dim
        d = cfg.n_embd
        if (d % cfg.n_head and not cfg.attn_head_dim) or cfg.n_head % cfg.n_kv_head:
            raise ValueError("heads must divide width and kv heads must divide heads")
        self.c_q = Linear(d, cfg.n_head * self.head_dim, bias=False)
        self.c_k = Linear(d, cfg.n_kv_head * self.head_dim, bias=False)
        self.c_v = Linear(d, cfg.n_kv_head * self.head_dim, bias=False)
        self.c_proj = Linear(cfg.n_head * self.head_dim, d, bias=False)
        self.ve_gate_channels = 12
        self.ve_gate = Linear(12, cfg.n_kv_head, bias=False) if (cfg.value_embeddings and has_ve(layer, cfg.n_layer)) \
            else None

    def projections(self, x):
        """The raw q, k, v projections ``[B, T, heads * head_dim]`` (a hook for variants that
        transform them before the heads are split)."""
        return self.c_q(x), self.c_k(x), self.c_v(x)

    def project(self, x, ve, cos_sin):
        """q, k, v after value-embedding mixing, RoPE and QK-norm (shared by the mixers that reuse it)."""
        B, T, _ = x.shape
        q, k, v = self.projections(x)
        q = q.view(B, T, self.n_head, self.head_dim)
        k = k.view(B, T, self.n_kv_head, self.head_dim)
        v = v.view(B, T, self.n_kv_head, self.head_dim)
        if ve is not None and self.ve_gate is not None:
            ve = ve.view(B, T, self.n_kv_head, self.head_dim)
            gate = 3 * torch.sigmoid(self.ve_gate(x[..., :self.ve_gate_channels]))
            v = v + gate.unsqueeze(-1) * ve
        cos, sin = cos_sin
        q, k = apply_rotary_emb(q, cos, sin), apply_rotary_emb(k, cos, sin)
        q, k = norm(q) * 1.2, norm(k) * 1.2
        return q, k, v

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise NotImplementedError("KV-cache decoding goes through nexttransformer_b200.inference")
        B, T, _ = x.shape
        q, k, v = self.project(x, ve, cos_sin)
        y = sdpa(q, k, v, window_size[0])
        return self.c_proj(y.contiguous().view(B, T, -1))


class MLP(nn.Module):
    def __init__(self, cfg: ShellConfig):
        super().__init__()
        self.c_fc = Linear(cfg.n_embd, cfg.ffn, bias=False)
        self.c_proj = Linear(cfg.ffn, cfg.n_embd, bias=False)

    def hidden(self, x):
        """The pre-activation hidden layer (a hook for variants that transform it)."""
        return self.c_fc(x)

    def forward(self, x):
        return self.c_proj(F.relu(self.hidden(x)).square())


class Block(nn.Module):
    def __init__(self, cfg: ShellConfig, layer: int):
        super().__init__()
        self.attn = CausalSelfAttention(cfg, layer)
        self.mlp = MLP(cfg)

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        x = x + self.attn(norm(x), ve, cos_sin, window_size, kv_cache)
        return x + self.mlp(norm(x))


def short_window(T):
    """Quarter context in 128-token tiles, as the reference computes it (2048 -> 512)."""
    return -(-T // 4 // 128) * 128


class GPTShell(nn.Module):
    """The shared shell.  Construct under ``torch.device('meta')`` and call ``init_weights``."""

    def __init__(self, cfg: ShellConfig):
        super().__init__()
        self.shell = cfg
        self.window_sizes = self._compute_window_sizes(cfg)
        V, d = cfg.padded_vocab, cfg.n_embd
        self.transformer = nn.ModuleDict({
            "wte": nn.Embedding(V, d),
            "h": nn.ModuleList([Block(cfg, i) for i in range(cfg.n_layer)]),
        })
        self.lm_head = Linear(d, V, bias=False)
        self.resid_lambdas = nn.Parameter(torch.ones(cfg.n_layer))
        self.x0_lambdas = nn.Parameter(torch.zeros(cfg.n_layer))
        self.smear_gate = Linear(24, 1, bias=False)
        self.smear_lambda = nn.Parameter(torch.zeros(1))
        self.backout_lambda = nn.Parameter(0.2 * torch.ones(1))
        kvd = cfg.n_kv_head * cfg.head_dim
        self.value_embeds = nn.ModuleDict({str(i): nn.Embedding(V, kvd) for i in range(cfg.n_layer)
                                           if cfg.value_embeddings and has_ve(i, cfg.n_layer)})
        self.rotary_seq_len = cfg.sequence_len * 10
        cos, sin = self._rotary(self.rotary_seq_len, cfg.head_dim)
        self.register_buffer("cos", cos, persistent=False)
        self.register_buffer("sin", sin, persistent=False)
        self._fused = None

    # ------------------------------------------------------------------ construction
    @staticmethod
    def _compute_window_sizes(cfg):
        pat = cfg.window_pattern.upper()
        if not pat or set(pat) - set("SL"):
            raise ValueError(f"invalid window_pattern {pat!r}")
        long, short = cfg.sequence_len, short_window(cfg.sequence_len)
        sizes = [((long if pat[i % len(pat)] == "L" else short), 0) for i in range(cfg.n_layer)]
        sizes[-1] = (long, 0)
        return sizes

    def _rotary(self, seq_len, head_dim, base=100000, device=None):
        if device is None:
            device = self.transformer.wte.weight.device
        ch = torch.arange(0, head_dim, 2, dtype=torch.float32, device=device)
        inv = 1.0 / (base ** (ch / head_dim))
        t = torch.arange(seq_len, dtype=torch.float32, device=device)
        f = torch.outer(t, inv)
        cos, sin = f.cos().to(COMPUTE_DTYPE), f.sin().to(COMPUTE_DTYPE)
        return cos[None, :, None, :], sin[None, :, None, :]

    @torch.no_grad()
    def init_weights(self):
        """Initialisation of the reference shell (same distributions, same RNG draw order)."""
        cfg = self.shell
        nn.init.normal_(self.transformer.wte.weight, mean=0.0, std=0.8)
        nn.init.normal_(self.lm_head.weight, mean=0.0, std=0.001)
        s = 3 ** 0.5 * cfg.n_embd ** -0.5
        for blk in self.transformer.h:
            a, m = blk.attn, blk.mlp
            if hasattr(a, "c_q"):
                nn.init.uniform_(a.c_q.weight, -s, s)
                nn.init.uniform_(a.c_k.weight, -s, s)
                nn.init.uniform_(a.c_v.weight, -s, s)
                nn.init.zeros_(a.c_proj.weight)
            if hasattr(m, "c_fc"):
                nn.init.uniform_(m.c_fc.weight, -s * 0.4, s * 0.4)
                nn.init.zeros_(m.c_proj.weight)
        n = cfg.n_layer
        for i in range(n):
            self.resid_lambdas.data[i] = 1.15 - 0.10 * i / max(n - 1, 1)
            self.x0_lambdas.data[i] = 0.20 - 0.15 * i / max(n - 1, 1)
        nn.init.zeros_(self.smear_lambda)
        nn.init.constant_(self.backout_lambda, 0.2)
        nn.init.uniform_(self.smear_gate.weight, 0.0, 0.02)
        for ve in self.value_embeds.values():
            nn.init.uniform_(ve.weight, -s, s)
        for blk in self.transformer.h:
            g = getattr(blk.attn, "ve_gate", None)
            if g is not None:
                nn.init.uniform_(g.weight, 0.0, 0.02)
        self.cos, self.sin = self._rotary(self.rotary_seq_len, cfg.head_dim)
        if COMPUTE_DTYPE != torch.float16:
            for emb in (self.transformer.wte, *self.value_embeds.values()):
                if emb.weight.dtype != COMPUTE_DTYPE:
                    emb.to(dtype=COMPUTE_DTYPE)

    def get_device(self):
        return self.transformer.wte.weight.device

    # ------------------------------------------------------------------ accounting
    def num_matmul_params(self):
        return sum(m.weight.numel() for m in self.modules() if isinstance(m, Linear))

    def estimate_flops(self):
        """Training FLOPs per token: 6 x matmul params + 12 h q T_eff per layer (PaLM convention)."""
        cfg = self.shell
        h, q, t = cfg.n_head, cfg.head_dim, cfg.sequence_len
        attn = sum(12 * h * q * (t if w < 0 else min(w, t)) for w, _ in self.window_sizes)
        return 6 * self.num_matmul_params() + attn

    def num_scaling_params(self):
        wte = self.transformer.wte.weight.numel()
        ve = sum(p.numel() for p in self.value_embeds.parameters())
        head = self.lm_head.weight.numel()
        blocks = sum(p.numel() for p in self.transformer.h.parameters())
        scalars = sum(p.numel() for p in (self.resid_lambdas, self.x0_lambdas, self.smear_gate.weight,
                                          self.smear_lambda, self.backout_lambda))
        return dict(wte=wte, value_embeds=ve, lm_head=head, transformer_matrices=blocks, scalars=scalars,
                    total=wte + ve + head + blocks + scalars)

    # ------------------------------------------------------------------ forward
    def embed(self, idx):
        x = norm(self.transformer.wte(idx).to(COMPUTE_DTYPE))
        if x.shape[1] > 1:
            gate = self.smear_lambda.to(x.dtype) * torch.sigmoid(self.smear_gate(x[:, 1:, :24]))
            x = torch.cat((x[:, :1], x[:, 1:] + gate * x[:, :-1]), 1)
        return x

    def readout(self, x, backout):
        if backout is not None:
            x = x - self.backout_lambda.to(x.dtype) * backout
        logits = self.lm_head(norm(x))[..., :self.shell.vocab_size].float()
        cap = self.shell.softcap
        return cap * torch.tanh(logits / cap)

    def forward_eager(self, idx, targets=None, loss_reduction="mean"):
        B, T = idx.shape
        if T > self.cos.size(1):
            raise ValueError("sequence longer than the rotary cache")
        cos_sin = self.cos[:, :T], self.sin[:, :T]
        x = self.embed(idx)
        x0 = x
        n = self.shell.n_layer
        backout = None
        for i, blk in enumerate(self.transformer.h):
            x = self.resid_lambdas[i] * x + self.x0_lambdas[i] * x0
            ve = self.value_embeds[str(i)](idx).to(x.dtype) if str(i) in self.value_embeds else None
            x = blk(x, ve, cos_sin, self.window_sizes[i], None)
            if i == n // 2:
                backout = x
        logits = self.readout(x, backout)
        if targets is None:
            return logits
        return F.cross_entropy(logits.view(-1, logits.size(-1)), targets.reshape(-1), ignore_index=-1,
                               reduction=loss_reduction)

    def fused_supported(self):
        """True when every block is the shell's own dense attention + ReLU^2 MLP."""
        return all(type(b) is Block and type(b.attn) is CausalSelfAttention and type(b.mlp) is MLP
                   for b in self.transformer.h)

    def layer_window(self, i):
        """Left attention window of layer ``i`` (a window >= T - 1 is plain causal attention)."""
        return self.window_sizes[i][0]

    def forward(self, idx, targets=None, loss_reduction="mean"):
        if idx.is_cuda and self.fused_supported() and targets is not None and loss_reduction in ("mean", "sum"):
            from nexttransformer_b200.models.fused_dense import fused_forward
            return fused_forward(self, idx, targets, loss_reduction)[0]
        return self.forward_eager(idx, targets, loss_reduction)

    # ------------------------------------------------------------------ fused-path state
    def fused_state(self):
        """The kernel state (bf16 shadows, fp32 gradient slots) of this model on CUDA."""
        if self._fused is None:
            from nexttransformer_b200.models.fused_dense import FusedState
            self._fused = FusedState(self)
        return self._fused

    def refresh_shadows(self):
        """Re-cast the bf16 copies of the fp32 matrices after an optimizer step."""
        if self._fused is not None:
            self._fused.refresh_shadows()

    def zero_main_grads(self):
        if self._fused is not None:
            self._fused.zero_grads()


def build_shell(cfg: ShellConfig, device="cpu", seed=42):
    """Meta construction, materialisation on `device`, reference-order initialisation."""
    torch.manual_seed(seed)
    with torch.device("meta"):
        model = GPTShell(cfg)
    model.to_empty(device=device)
    for m in model.modules():
        if isinstance(m, nn.Linear):
            m.reset_parameters()
    model.init_weights()
    return model
