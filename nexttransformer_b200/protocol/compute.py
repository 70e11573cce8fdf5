"""Shape-only FLOP ledger: forward, backward and optimizer arithmetic of one training update.

A ``TorchDispatchMode`` executes the model's eager path under ``FakeTensorMode`` (no storage,
no GPU) and charges every ATen operator by a fixed cost table.  Attention is charged by
explicit edge rules (causal / sliding-window / selected-key edges) instead of the dense score
matrix; chunked linear attention charges C x C intra-chunk tiles for causal pairs only; unknown
floating-point operators are reported so admission can fail closed.

The cost table, the attention edge rules and the optimizer operator sequence are those of the
reference ledger (``nexttransformer/protocol/compute.py``, formula "reference-aten-math-v2"):
the FLOPs-per-token every run is charged must agree with the reference within 1 %, so the
counting conventions are reproduced exactly rather than redesigned.
"""
from collections import Counter, defaultdict
from contextlib import contextmanager
import math

import torch
from torch._subclasses.fake_tensor import FakeTensorMode
from torch.utils._python_dispatch import TorchDispatchMode

from nexttransformer_b200.models import sparse as sparse_mod
from nexttransformer_b200.models import shell as shell_mod
from nexttransformer_b200.models.config import CHUNK_BACKENDS
from nexttransformer_b200.models.registry import PLUGIN_METHODS
from nexttransformer_b200.protocol.spec import Protocol

FORMULA_VERSION = "reference-aten-math-v2"


def causal_edges(length, left):
    """(query, key) pairs of causal attention with a left window of `left` previous keys (-1: all)."""
    width = length if left < 0 else min(length, left + 1)
    return width * (width + 1) // 2 + (length - width) * width


def selected_edges(config, start, stop, stage, branch=0, kind=None):
    kind = kind or config.method
    if stage == "burnin" and kind in ("dsa", "qsa", "seer"):
        return sum(i + 1 for i in range(start, stop))
    if kind == "dsa":
        return sum(min(config.sparse_topk, i + 1) for i in range(start, stop))
    if kind == "qsa":
        s = config.compression_size
        return sum(min(config.sparse_topk, (i + 1) // s * s) + (i + 1) % s for i in range(start, stop))
    if kind == "nsa" and branch == 1:
        return sum(min(config.local_window, i + 1) for i in range(start, stop))
    size = config.compression_size if kind in ("qsa", "nsa") else config.block_size
    top = max(0, config.sparse_topk // size - 1) if kind == "moba" else max(1, (config.sparse_topk + size - 1) // size)
    return sum(min(top, i // size) * size + i % size + 1 for i in range(start, stop))


def _tensors(v):
    if isinstance(v, torch.Tensor):
        yield v
    elif isinstance(v, (list, tuple)):
        for x in v:
            yield from _tensors(x)
    elif isinstance(v, dict):
        for x in v.values():
            yield from _tensors(x)


class Ledger(TorchDispatchMode):
    FREE = {"_to_copy", "_unsafe_view", "alias", "arange", "as_strided", "as_strided_", "cat", "clone",
            "constant_pad_nd", "contiguous", "copy_", "detach", "detach_", "empty", "empty_like", "empty_strided",
            "expand", "fill_", "flip", "full", "full_like", "gather", "index", "index_put", "index_put_",
            "lift_fresh", "masked_fill", "masked_fill_", "new_empty", "new_empty_strided", "new_zeros", "ones",
            "ones_like", "permute", "randn", "randint", "scalar_tensor", "select", "select_backward", "slice",
            "slice_backward", "split", "split_with_sizes", "squeeze", "stack", "t", "transpose", "unbind",
            "uniform_", "unsqueeze", "view", "view_as", "where", "zero_", "zeros", "zeros_like", "any", "all", "eq",
            "ne", "lt", "le", "gt", "ge", "bitwise_and", "bitwise_or", "bitwise_not", "topk", "floor_divide",
            "remainder", "isfinite", "normal_", "tril", "tril_", "triu", "triu_", "eye", "sort", "argsort",
            "index_select", "bincount", "unfold"}
    PAIR_EXACT = {"linalg_solve_triangular"}
    PER_ELEMENT = {"add": 1, "add_": 1, "sub": 1, "sub_": 1, "rsub": 1, "mul": 1, "mul_": 1, "div": 1, "div_": 1,
                   "neg": 1, "exp": 1, "log": 1, "sqrt": 1, "rsqrt": 1, "reciprocal": 1, "sin": 1, "cos": 1,
                   "tanh": 1, "clamp_min": 1, "clamp_max": 1, "clamp": 1, "relu": 1, "abs": 1, "sign": 1,
                   "signbit": 1, "pow": 1, "sigmoid": 4, "silu": 5, "softplus": 4, "elu": 3, "lerp": 3, "lerp_": 3,
                   "sigmoid_backward": 3, "tanh_backward": 3, "threshold_backward": 1, "silu_backward": 8,
                   "softplus_backward": 5, "elu_backward": 3}

    def __init__(self, pair_block=None):
        super().__init__()
        self.phase = "forward"
        self.ops = defaultdict(lambda: dict(calls=0, theory=0, padded_envelope=0, matrix=0))
        self.unknown = Counter()
        self.scalars_ignored = 0
        self.pair_block = pair_block

    def _pair(self, v):
        c = self.pair_block
        return c is not None and v.dim() >= 2 and tuple(v.shape[-2:]) == (c, c)

    def _pairs(self, v):
        c = self.pair_block
        return v.numel() // (c * c) * (c * (c + 1) // 2) if self._pair(v) else v.numel()

    def add(self, name, count, matrix=0, padded=None):
        it = self.ops[self.phase + "/" + name]
        it["calls"] += 1
        it["theory"] += int(count)
        it["matrix"] += int(matrix)
        it["padded_envelope"] += int(count if padded is None else padded)

    def _cost(self, name, func, args, kwargs, outs):
        n = sum(v.numel() for v in outs if v.is_floating_point())
        if name in ("mm", "bmm", "addmm", "baddbmm"):
            a, b = args[-2:] if name in ("mm", "bmm") else args[1:3]
            m = 2 * math.prod(a.shape[:-2]) * a.shape[-2] * a.shape[-1] * b.shape[-1]
            return m + (outs[0].numel() if name in ("addmm", "baddbmm") else 0), m
        if name in self.PER_ELEMENT:
            c = n * self.PER_ELEMENT[name]
            if name in ("add", "add_", "sub", "sub_") and kwargs.get("alpha", 1) != 1:
                c += n
            return c, 0
        if name in ("sum", "mean", "amax"):
            c = max(0, args[0].numel() - outs[0].numel())
            return c + (outs[0].numel() if name == "mean" else 0), 0
        if name in ("_softmax", "_log_softmax"):
            return 5 * args[0].numel(), 0
        if name in ("_softmax_backward_data", "_log_softmax_backward_data"):
            return 4 * args[0].numel(), 0
        if name == "log_sigmoid_forward":
            return 4 * args[0].numel(), 0
        if name == "log_sigmoid_backward":
            return 5 * args[0].numel(), 0
        if name == "linalg_vector_norm":
            return 2 * args[0].numel() + outs[0].numel(), 0
        if name == "embedding":
            return 0, 0
        if name == "embedding_dense_backward":
            return args[0].numel(), 0
        if name in ("scatter_add", "scatter_add_"):
            return args[3].numel(), 0
        if name == "index_add":
            return args[3].numel(), 0
        if name == "unfold_backward":
            # overlapping windows (strided compression): one addition per gradient element
            return args[0].numel(), 0
        if name == "native_layer_norm":
            return 7 * args[0].numel() + 5 * outs[1].numel(), 0
        if name == "native_layer_norm_backward":
            c = 10 * args[1].numel() if args[-1][0] else 0
            return c + sum(2 * args[1].numel() for on in args[-1][1:] if on), 0
        if name == "nll_loss_forward":
            return 2 * args[1].numel() + (1 if args[3] == 1 else 0), 0
        if name == "nll_loss_backward":
            return 2 * args[2].numel(), 0
        if name == "binary_cross_entropy_with_logits":
            return 10 * args[0].numel(), 0
        if name == "convolution":
            w = args[1]
            m = 2 * outs[0].numel() * math.prod(w.shape[1:])
            return m + (outs[0].numel() if args[2] is not None else 0), m
        if name == "convolution_backward":
            dy, _, w = args[:3]
            mask = args[-1]
            one = 2 * dy.numel() * math.prod(w.shape[1:])
            m = one * (int(mask[0]) + int(mask[1]))
            return m + (dy.numel() if mask[2] else 0), m
        if name == "cumsum":
            L = args[0].shape[args[1]] if args[0].dim() else 1
            return args[0].numel() - args[0].numel() // max(L, 1), 0
        if name == "linalg_solve_triangular":
            a = args[0]
            nn_ = a.shape[-1]
            cols = outs[0].numel() // nn_
            m = cols * nn_ * (nn_ - 1)
            return m + (0 if kwargs.get("unitriangular", False) else cols * nn_), m
        self.unknown[str(func)] += 1
        return 0, 0

    def __torch_dispatch__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        name = func._schema.name.split("::")[-1]
        if name == "_local_scalar_dense":
            self.scalars_ignored += 1
            return 0
        out = func(*args, **kwargs)
        ins, outs = list(_tensors(args)), list(_tensors(out))
        floats = [v for v in outs if v.is_floating_point()]
        if name in self.FREE or not floats:
            return out
        cost, matrix = self._cost(name, func, args, kwargs, floats)
        padded = None
        if cost and name not in self.PAIR_EXACT and any(self._pair(v) for v in ins + outs):
            padded = cost
            c = self.pair_block
            pairs = c * (c + 1) // 2
            if name in ("sum", "mean", "amax"):
                i_, o_ = self._pairs(args[0]), self._pairs(floats[0])
                cost, matrix = max(0, i_ - o_) + (o_ if name == "mean" else 0), 0
            else:
                if (cost * pairs) % (c * c) or (matrix * pairs) % (c * c):
                    raise RuntimeError(f"non-tile operator on a chunk tile: {func}")
                cost, matrix = cost * pairs // (c * c), matrix * pairs // (c * c)
        if cost:
            self.add(str(func), cost, matrix, padded)
        return out

    def report(self):
        tot = {ph: sum(v["theory"] for k, v in self.ops.items() if k.startswith(ph + "/"))
               for ph in ("forward", "backward", "optimizer")}
        return dict(formula_version=FORMULA_VERSION, phases=tot, pair_block=self.pair_block, total=sum(tot.values()),
                    matrix_total=sum(v["matrix"] for v in self.ops.values()),
                    padded_envelope=sum(v["padded_envelope"] for v in self.ops.values()),
                    operators=dict(sorted(self.ops.items())), unknown=dict(self.unknown),
                    diagnostic_scalar_reads=self.scalars_ignored)


class _AttentionCost(torch.autograd.Function):
    """Stand-in for attention: charges 2 E (d + dv) + 6 E forward and the matching backward."""

    @staticmethod
    def forward(ctx, q, k, v, edges, padded, ledger, label):
        ctx.save_for_backward(q, k, v)
        ctx.cost = (edges, padded, ledger, label)
        d, dv = q.shape[-1], v.shape[-1]
        m = 2 * edges * (d + dv)
        ledger.add(label, m + 6 * edges, m, 2 * padded * (d + dv) + 6 * padded)
        return q.new_empty(*q.shape[:-1], dv)

    @staticmethod
    def backward(ctx, g):
        q, k, v = ctx.saved_tensors
        edges, padded, ledger, label = ctx.cost
        nq, nk, nv = ctx.needs_input_grad[:3]
        d, dv = q.shape[-1], v.shape[-1]
        f = 2 * d * (int(nq) + int(nk)) + 2 * dv * (int(nq or nk) + int(nv))
        soft = 5 if nq or nk else 0
        ledger.add(label, edges * (f + soft), edges * f, padded * (f + soft))
        return (torch.empty_like(q) if nq else None, torch.empty_like(k) if nk else None,
                torch.empty_like(v) if nv else None, None, None, None, None)


@contextmanager
def attention_rules(model, ledger, stage):
    """Swap the attention numerics for edge-rule charges during a shape-only audit."""
    orig_sdpa, orig_idx = shell_mod.sdpa, sparse_mod.indexed_attention
    active, handles = {}, []

    def enter(module, args):
        active.update(config=module.config, kind=module.kind, calls=0)
    for m in model.modules():
        if isinstance(m, sparse_mod.SparseMixer):
            handles.append(m.register_forward_pre_hook(enter))

    def native(q, k, v, window):
        B, T, H, _ = q.shape
        rep = H // k.shape[2]
        kk, vv = k.transpose(1, 2), v.transpose(1, 2)
        edges = B * H * causal_edges(T, window)
        y = _AttentionCost.apply(q.transpose(1, 2), kk, vv, edges, B * H * T * T, ledger, "native_attention")
        return y.transpose(1, 2)

    def indexed(q, k, v, idx, valid):
        c, calls = active["config"], active["calls"]
        active["calls"] += 1
        branches = 2 if active["kind"] == "nsa" else 1
        start = (calls // branches) * c.reference_chunk
        stop = start + q.shape[-2]
        edges = q.shape[0] * q.shape[1] * selected_edges(c, start, stop, stage, calls % branches, kind=active["kind"])
        return _AttentionCost.apply(q, k, v, edges, idx.numel(), ledger, "indexed_attention")
    shell_mod.sdpa, sparse_mod.indexed_attention = native, indexed
    try:
        yield
    finally:
        shell_mod.sdpa, sparse_mod.indexed_attention = orig_sdpa, orig_idx
        for h in handles:
            h.remove()


# ------------------------------------------------------------------ optimizer cost model
def _adamw_ops(p, grad, exp_avg, exp_avg_sq, step_t, lr_t, b1_t, b2_t, eps_t, wd_t):
    """The ATen operator sequence of one fused AdamW update (fp32 math), run only for counting."""
    p32, m32, v32, g32 = p.float(), exp_avg.float(), exp_avg_sq.float(), grad.float()
    p32.mul_(1 - lr_t * wd_t)
    m32.lerp_(g32, 1 - b1_t)
    v32.lerp_(g32.square(), 1 - b2_t)
    bias1, bias2 = 1 - b1_t ** step_t, 1 - b2_t ** step_t
    denom = (v32 / bias2).sqrt() + eps_t
    p32.add_(m32 / denom, alpha=-(lr_t / bias1))
    p.copy_(p32)
    exp_avg.copy_(m32)
    exp_avg_sq.copy_(v32)


def _muon_ops(grads, params, mom, second, mom_t, lr_t, wd_t, b2_t, ns_steps, red_dim):
    """The ATen operator sequence of one fused Muon update, run only for counting."""
    from nexttransformer_b200.optim.muon_adamw import POLAR_EXPRESS
    mu = mom_t.to(grads.dtype)
    mom.lerp_(grads, 1 - mu)
    g = grads.lerp_(mom, mu)
    X = g.bfloat16()
    target = X.float().norm(dim=(-2, -1), keepdim=True) / (X.size(-2) ** 0.5)
    rown = X.float().norm(dim=-1, keepdim=True).clamp_min(1e-6)
    X = X * (target / rown).to(X.dtype)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)
    if g.size(-2) > g.size(-1):
        for a, b, c in POLAR_EXPRESS[:ns_steps]:
            A = X.mT @ X
            X = a * X + X @ (b * A + c * (A @ A))
    else:
        for a, b, c in POLAR_EXPRESS[:ns_steps]:
            A = X @ X.mT
            X = a * X + (b * A + c * (A @ A)) @ X
    g = X.to(params.dtype)
    g = g * (min(g.size(-2), g.size(-1)) ** 0.5 / g.float().norm(dim=(-2, -1), keepdim=True).clamp_min(1e-6)).to(g.dtype)
    b2 = b2_t.to(g.dtype)
    vmean = g.float().square().mean(dim=red_dim, keepdim=True)
    rs = g.size(red_dim)
    vnorm = (vmean.sum(dim=(-2, -1), keepdim=True) * rs).sqrt()
    second.lerp_(vmean.to(second.dtype), 1 - b2)
    step = second.clamp_min(1e-10).rsqrt()
    vnew = ((vmean * rs) * step.float().square()).sum(dim=(-2, -1), keepdim=True).sqrt()
    g = g * (step * (vnorm / vnew.clamp_min(1e-10))).to(g.dtype)
    lr, wd = lr_t.to(g.dtype), wd_t.to(g.dtype)
    mask = (g * params) >= 0
    params.sub_(lr * g + lr * wd * params * mask)


def count_optimizer(model, ledger, train=None):
    """One logical optimizer update (no communication, no padded ranks)."""
    from nexttransformer_b200.optim.groups import protocol_groups
    scalar = lambda v: torch.tensor(float(v))
    ledger.phase = "optimizer"
    with torch.no_grad(), ledger:
        for g in protocol_groups(model, train):
            if g["kind"] == "adamw":
                for p in g["params"]:
                    _adamw_ops(p, torch.empty_like(p), torch.empty_like(p), torch.empty_like(p),
                               *[scalar(x) for x in (1, g["lr"], *g["betas"], g["eps"], g["weight_decay"])])
            else:
                ps = g["params"]
                m, n = ps[0].shape
                stack = torch.empty((len(ps), m, n))
                red = -1 if m >= n else -2
                second = torch.empty((len(ps), m, 1) if red == -1 else (len(ps), 1, n))
                _muon_ops(torch.empty_like(stack), stack, torch.empty_like(stack), second,
                          *[scalar(x) for x in (g["momentum"], g["lr"], g["weight_decay"], g["beta2"])],
                          g["ns_steps"], red)


def audit_graph(config, *, sequence_len=None, batch=1, stage="joint", depth=None, optimizer=True):
    """A complete fake execution of one update: no storage, no GPU."""
    from nexttransformer_b200.models.lm import construct, materialize
    T = sequence_len or config.sequence_len
    pair = CHUNK_BACKENDS.get(config.backend)
    if pair in (config.width, config.heads, config.head_dim, config.mlp_width, config.vocab_size,
                config.gate_rank, config.conv_size):
        raise ValueError("a model dimension equals the chunk length; C x C tiles would be ambiguous")
    ledger = Ledger(pair)
    torch.manual_seed(42)
    meta = construct(config)  # built outside the fake mode: fake tensors then replace plain meta tensors
    with FakeTensorMode(allow_non_fake_inputs=True):
        model = materialize(meta, "cpu")
        p = Protocol()
        if config.method in PLUGIN_METHODS:
            from nexttransformer_b200.models.plugins import stages
            start, step = 0, 0
            for name, count in stages(config):
                if name == stage:
                    step = start
                start += count
        else:
            step = 0 if stage == "burnin" else p.steps - config.ouro_gate_steps if stage == "gate_only" \
                else config.burnin_steps + 1
        model.set_training_stage(step)
        if config.method == "huginn":
            if depth is None:
                raise ValueError("Huginn cost needs an explicit sampled depth")
            model.accounting_depth = depth
        x = torch.zeros((batch, T), dtype=torch.long)
        with attention_rules(model, ledger, stage), ledger:
            loss = model(x, x)
            ledger.phase = "backward"
            loss.backward()
        if optimizer:
            count_optimizer(model, ledger)
        params = sum(q.numel() for q in model.parameters())
    rep = ledger.report()
    rep.update(method=config.method, model_hash=config.fingerprint, sequence_len=T, batch=batch, stage=stage,
               depth=depth, parameters=params)
    return rep


def flops_per_token(config, batch=512, stage="joint", depth=None):
    """Audited training FLOPs per input token of one update at the protocol batch."""
    r = audit_graph(config, batch=batch, stage=stage, depth=depth)
    return r["total"] / (batch * (config.sequence_len))
