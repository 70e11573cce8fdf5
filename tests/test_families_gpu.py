"""Every model family on the generic sm_100a path against an fp64 oracle of the same weights.

The kernel model is built on CUDA (bf16 activations, fp32 masters) and trained through its kernel
state: the shell's attention / MLP as fused Functions, every other projection on the tcgen05 GEMM
engine (``ops.dense.KernelLinear``), RMSNorms on the row kernels, linear mixers on the scan /
conv / gated-norm kernels, sparse mixers on the block-sparse kernels, routed experts as grouped
GEMMs, the head as the fused soft-capped cross-entropy GEMM.  The oracle is the same model,
same weights, run eagerly on the CPU in float64.  The loss and every parameter gradient must
agree elementwise, per tensor: ``max |g - g_ref|`` within 5 % of the tensor's largest entry (10 %
for routed experts, whose router may break near-ties differently), or within twice the error of
the same model run on the plain bf16 PyTorch graph (which calibrates what bf16 activations alone
cost), plus 1e-4 of the model's largest gradient; the shell's scalar gains, whose gradients are
one sum of bf16 products over every token with cancellation, get 25 % or four times the baseline's
error plus 2e-4 of the largest gradient (a gradient that is exactly zero in the
oracle, like the backout gain's when the backout point is the last layer, is bf16 noise).
"""
from contextlib import contextmanager
from dataclasses import replace

import pytest
import torch

pytestmark = pytest.mark.gpu

BASE = dict(width=256, heads=2, vocab_size=512, sequence_len=256, mlp_width=1024, scale="custom",
            window_pattern="L")
CASES = {
    "dense": dict(layers=2, window_pattern="SL", kv_heads=1),
    "gdn_hybrid_swa": dict(layers=4, backend="fla_chunk64", sliding_window=128),
    "kda_hybrid": dict(layers=4, backend="fla_chunk64", q_rank=128, kv_rank=128, qk_nope_dim=128, qk_rope_dim=0,
                       v_head_dim=128),
    "gdn": dict(layers=2, backend="fla_chunk64"),
    "kda": dict(layers=2, backend="fla_chunk64"),
    "deltanet": dict(layers=2, backend="fla_chunk64"),
    "nsa": dict(layers=2, heads=4, kv_heads=1, attn_head_dim=128, compression_size=32, compression_stride=16,
                block_size=64, sparse_topk=128, local_window=64),
    "moba": dict(layers=2, kv_heads=1, block_size=64, sparse_topk=128),
    "moe": dict(layers=2, kv_heads=1, moe_experts=8, moe_topk=2, moe_ffn=128, moe_shared=1),
}


@contextmanager
def compute_dtype(dtype):
    """Build and run models with activations in ``dtype`` (the module-level compute dtype)."""
    import nexttransformer_b200.models.lm as lm
    import nexttransformer_b200.models.shell as shell
    import nexttransformer_b200.utils.dtype as ud
    mods = (lm, shell, ud)
    old = [m.COMPUTE_DTYPE for m in mods]
    for m in mods:
        m.COMPUTE_DTYPE = dtype
    try:
        yield
    finally:
        for m, o in zip(mods, old):
            m.COMPUTE_DTYPE = o


def _config(method):
    from nexttransformer_b200.models.config import candidate_config
    return replace(candidate_config(method), **{**BASE, **CASES[method]})


def _grads(model):
    from nexttransformer_b200.optim.muon_adamw import grad_of
    out = {}
    for n, p in model.named_parameters():
        g = grad_of(p)
        if g is not None:
            out[n] = g.detach().double().cpu()
    return out


@pytest.mark.parametrize("method", sorted(CASES))
def test_family_matches_fp64_oracle(method):
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.ops._ext import check_errors
    cfg = _config(method)
    model = build_model(cfg, "cuda", seed=5)
    # the zero-initialised output projections would hide most of the backward: give them signal
    with torch.no_grad():
        for n, p in model.named_parameters():
            if p.ndim == 2 and float(p.abs().max()) == 0.0:
                p.normal_(0, 0.02)
    if method in ("nsa", "moba"):
        model.set_sparse_backend("kernel")
    model.train()
    st = model.fused_state()
    st.refresh_shadows()
    st.zero_grads()
    g = torch.Generator().manual_seed(11)
    tok = torch.randint(0, cfg.vocab_size, (2, cfg.sequence_len + 1), generator=g)
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    loss = model(x.cuda(), y.cuda())
    loss.backward()
    torch.cuda.synchronize()
    check_errors()
    # the generic path really ran: every eligible projection was a kernel linear that wrote its slot
    if method != "dense":
        assert st.kernel_linears, "no projection ran on the GEMM engine"
        idle = [n for n, m in model.named_modules() if m in st.kernel_linears and m._g.fresh]
        assert not idle, f"registered projections that never ran: {idle}"
    got = _grads(model)

    # bf16 baseline: the same model on the plain PyTorch graph (no kernel state), whose error against
    # the fp64 oracle calibrates what bf16 activations alone cost
    eager = build_model(cfg, "cuda", seed=5)
    eager.kernel_path = False
    eager.load_state_dict(model.state_dict())
    if method in ("nsa", "moba"):
        eager.set_sparse_backend("reference")
    eager.train()
    eager(x.cuda(), y.cuda()).backward()
    base = {n: p.grad.detach().double().cpu() for n, p in eager.named_parameters() if p.grad is not None}

    with compute_dtype(torch.float64):
        oracle = build_model(cfg, "cpu", seed=5)
        oracle.load_state_dict({k: v.detach().cpu() for k, v in model.state_dict().items()})
        oracle.train()
        ref_loss = oracle(x, y)
        ref_loss.backward()
    ref = {n: p.grad.detach().double() for n, p in oracle.named_parameters() if p.grad is not None}

    assert abs(loss.item() - ref_loss.item()) <= 1e-2 * abs(ref_loss.item()), (loss.item(), ref_loss.item())
    top = max(float(r.abs().max()) for r in ref.values())
    checked = 0
    for name, r in ref.items():
        scale = float(r.abs().max())
        if scale == 0.0:
            continue
        assert name in got, f"{name}: no gradient on the kernel path"
        err = float((got[name] - r).abs().max())
        bf16 = float((base[name] - r).abs().max()) if name in base else 0.0
        # within 5 % of the tensor's largest entry (10 % for routed experts), or at most twice the
        # bf16 baseline's own error; entries far below the model's largest gradient are bf16 noise
        if r.numel() <= 64:      # scalar gains: one fp32 sum of bf16 products over every token
            assert err <= max(0.25 * scale, 4.0 * bf16) + 2e-4 * top, (name, err, scale, bf16)
        else:
            tol = 0.1 if ("experts" in name or "router" in name) else 0.05
            assert err <= max(tol * scale, 2.0 * bf16) + 1e-4 * top, (name, err, scale, bf16)
        checked += 1
    assert checked >= 8
