"""Numerics, determinism and timing of the sm_100a kernels against PyTorch references (one GPU).

    python -m nexttransformer_b200.checks.kernels [--only gemm attention ce adamw muon] [--output k.json]

For each kernel family and a set of shapes: the kernel's result against a plain-PyTorch fp32
restatement of the same op (max abs / relative error with the family's tolerance), a bitwise
run-twice comparison for the kernels that promise determinism (GEMM incl. split-K, attention
forward, CE, AdamW, Muon), and CUDA-event timings of the kernel and of the PyTorch/cuBLAS path
for the same op.  Exits non-zero when a tolerance or a determinism promise is broken.
This is the B200 counterpart of the reference's ``checks/speedups.py`` and ``checks/fla.py``.
"""
import argparse
import json
import math
from pathlib import Path

import torch
import torch.nn.functional as F


def _time(fn, iters=5):
    fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _err(x, ref):
    d = (x.float() - ref.float()).abs().max().item()
    return d, d / max(ref.float().abs().max().item(), 1e-30)


def check_gemm(rows):
    from nexttransformer_b200.ops import gemm as G
    out = []
    for M, N, K in ((rows, 1280, 1280), (rows, 5120, 1280), (rows, 1280, 5120), (1000, 264, 328)):
        a = torch.randn(M, K, device="cuda").bfloat16()
        w = torch.randn(N, K, device="cuda").bfloat16()
        c = torch.empty(M, N, device="cuda", dtype=torch.bfloat16)
        G.gemm(a, w, c)
        ref = a.float() @ w.float().t()
        _, rel = _err(c, ref)
        c2 = torch.empty_like(c)
        G.gemm(a, w, c2)
        g1 = torch.zeros(N, K, device="cuda")
        g2 = torch.zeros(N, K, device="cuda")
        dy = torch.randn(M, N, device="cuda").bfloat16()
        G.wgrad(dy, a, g1, accumulate=True)
        G.wgrad(dy, a, g2, accumulate=True)
        _, wrel = _err(g1, dy.float().t() @ a.float())
        out.append(dict(op="gemm", shape=[M, N, K], rel_err=rel, wgrad_rel_err=wrel, ok=rel < 2e-2 and wrel < 2e-2,
                        deterministic=bool(torch.equal(c, c2) and torch.equal(g1, g2)),
                        ms=_time(lambda: G.gemm(a, w, c)), ms_torch=_time(lambda: a @ w.t())))
    return out


def check_attention(rows):
    from nexttransformer_b200.ops.attention import attention_fn
    out = []
    for B, T, H, Hk, window in ((max(1, rows // 2048), 2048, 10, 5, -1), (2, 1024, 4, 4, 255), (1, 384, 2, 1, -1)):
        D = 128
        qkv = (torch.randn(B * T, (H + 2 * Hk) * D, device="cuda") * 0.5).bfloat16().requires_grad_()
        y = attention_fn(qkv, B, T, H, Hk, D, window)
        y2 = attention_fn(qkv, B, T, H, Hk, D, window)
        dy = torch.randn_like(y)
        (g,) = torch.autograd.grad(y, qkv, dy)
        ref_in = qkv.detach().float().requires_grad_()
        v4 = ref_in.view(B, T, H + 2 * Hk, D).transpose(1, 2)
        q, k, v = v4[:, :H], v4[:, H:H + Hk].repeat_interleave(H // Hk, 1), v4[:, H + Hk:].repeat_interleave(H // Hk, 1)
        i = torch.arange(T, device="cuda")
        mask = (i[None, :] <= i[:, None]) & ((window < 0) | (i[:, None] - i[None, :] <= window))
        ref = F.scaled_dot_product_attention(q, k, v, attn_mask=mask).transpose(1, 2).reshape(B * T, H * D)
        (rg,) = torch.autograd.grad(ref, ref_in, dy.float())
        _, rel = _err(y, ref)
        _, grel = _err(g, rg)
        qt = qkv.detach().view(B, T, H + 2 * Hk, D).transpose(1, 2)
        lib = lambda: F.scaled_dot_product_attention(qt[:, :H], qt[:, H:H + Hk], qt[:, H + Hk:], is_causal=True,
                                                     enable_gqa=True)
        out.append(dict(op="attention", shape=[B, T, H, Hk, D], window=window, rel_err=rel, grad_rel_err=grel,
                        ok=rel < 2e-2 and grel < 5e-2, deterministic_forward=bool(torch.equal(y, y2)),
                        ms=_time(lambda: attention_fn(qkv, B, T, H, Hk, D, window)),
                        ms_torch=_time(lib) if window < 0 else None))
    return out


def check_ce(rows):
    from nexttransformer_b200.ops._ext import ext
    out = []
    for M, V in ((min(rows, 8192), 65536), (1000, 1000)):
        logits = (torch.randn(M, V, device="cuda") * 4).bfloat16()
        tgt = torch.randint(0, V, (M,), device="cuda")
        work = logits.clone()
        loss = torch.empty(M, device="cuda")
        lse = torch.empty(M, device="cuda")
        ext().softcap_ce(work, tgt, loss, lse, V, 15.0)
        lf = logits.float().requires_grad_()
        capped = 15 * torch.tanh(lf / 15)
        ref = F.cross_entropy(capped, tgt, reduction="none")
        (rg,) = torch.autograd.grad(ref.sum(), lf)
        work2 = logits.clone()
        loss2 = torch.empty_like(loss)
        ext().softcap_ce(work2, tgt, loss2, torch.empty_like(lse), V, 15.0)
        _, rel = _err(loss, ref)
        _, grel = _err(work, rg)
        out.append(dict(op="softcap_ce", shape=[M, V], rel_err=rel, grad_rel_err=grel, ok=rel < 1e-3 and grel < 2e-2,
                        deterministic=bool(torch.equal(loss, loss2) and torch.equal(work, work2))))
    return out


def check_adamw(rows):
    from nexttransformer_b200.ops._ext import ext
    from nexttransformer_b200.optim.muon_adamw import adamw_reference
    p = torch.randn(rows // 16, 1280, device="cuda")
    g = torch.randn_like(p)
    st = [torch.zeros_like(p), torch.zeros_like(p)]
    ref = [p.clone(), torch.zeros_like(p), torch.zeros_like(p)]
    for step in (1, 2, 3):
        ext().adamw(p, g, st[0], st[1], None, 1e-2, .8, .95, 1e-10, .01, step)
        adamw_reference(ref[0], g, ref[1], ref[2], step, 1e-2, .8, .95, 1e-10, .01)
    _, rel = _err(p, ref[0])
    return [dict(op="adamw", shape=list(p.shape), rel_err=rel, ok=rel < 1e-5)]


def check_muon(rows):
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW, muon_reference
    out = []
    for m, n in ((1280, 1280), (5120, 1280), (1280, 5120)):
        torch.manual_seed(0)
        params = [torch.nn.Parameter(torch.randn(m, n, device="cuda") * .02) for _ in range(4)]
        grads = [torch.randn(m, n, device="cuda") for _ in params]
        for q, gr in zip(params, grads):
            q.grad = gr.clone()
        ref_p = torch.stack([q.detach().clone() for q in params])
        mom = torch.zeros_like(ref_p)
        smb = torch.zeros(4, *((m, 1) if m >= n else (1, n)), device="cuda")
        opt = MuonAdamW([dict(kind="muon", params=params, lr=.02, momentum=.95, ns_steps=5, beta2=.9,
                              weight_decay=.1)])
        opt.step()
        lr = .02 * max(1.0, m / n) ** .5
        muon_reference(torch.stack(grads), ref_p, mom, smb, .95, lr, .1, .9, 5, torch.bfloat16)
        got = torch.stack([q.detach() for q in params])
        d, _ = _err(got, ref_p)
        out.append(dict(op="muon", shape=[4, m, n], max_abs_err=d, ok=d < 1e-3))
    return out


FAMILIES = dict(gemm=check_gemm, attention=check_attention, ce=check_ce, adamw=check_adamw, muon=check_muon)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--only", nargs="+", choices=sorted(FAMILIES), default=sorted(FAMILIES))
    ap.add_argument("--rows", type=int, default=16384)
    ap.add_argument("--output", type=Path)
    a = ap.parse_args(argv)
    if not torch.cuda.is_available():
        raise SystemExit("checks.kernels needs a CUDA device")
    torch.manual_seed(0)
    results = []
    for name in a.only:
        for r in FAMILIES[name](a.rows):
            print(json.dumps(r), flush=True)
            results.append(r)
    from nexttransformer_b200.ops._ext import check_errors
    check_errors()
    if a.output:
        a.output.write_text(json.dumps(results, indent=1) + "\n")
    bad = [r for r in results if not r["ok"] or r.get("deterministic") is False
           or r.get("deterministic_forward") is False]
    if bad:
        raise SystemExit(f"{len(bad)} kernel check(s) failed")
    return results


if __name__ == "__main__":
    main()
