"""Per-kernel timing harness for the sm_100a kernels (one GPU).

    python -m nexttransformer_b200.ops.microbench <case> [--rows M] [--iters N] [--warmup W]

Cases time one kernel family with CUDA events on the launching stream (warm-up first, a
synchronize on both sides) and print one JSON line: milliseconds per launch, the algorithmic
FLOPs or bytes, the achieved rate and its fraction of the measured peaks of this machine when
``MEASURED_PEAKS.json`` sits at the repository root.  Operands are larger than L2 for the default
sizes, so no flush is needed between launches.  The same command with small ``--rows`` and
``--iters 1`` is the small case to capture under a profiler.

Cases (shapes of the benchmark model: width 1280, 10/5 heads of 128, FFN 5120, vocab 65536):
  gemm_qkv, gemm_fc, gemm_proj, gemm_wgrad, gemm_head - the GEMM engine with its epilogues
  gemm_head_ce                                         - the LM head with the soft-capped CE epilogue
  gemm_wgrad_qkv, gemm_wgrad_o                         - weight gradients of the QKV / output projections
  attn_fwd, attn_bwd                                   - flash attention, rows = B*T (T 2048, or --seq)
  sdpa_fwd, sdpa_bwd                                   - the same shape through torch SDPA with one backend
                                                         (--sdpa cudnn | flash | efficient): the library bar
  ce                                                   - soft-capped cross-entropy over 65536 logits
  mix_norm_fwd/bwd, rope_norm_fwd/bwd                  - the shell's row kernels (bytes they must move)
  adamw                                                - AdamW over a [rows, 1280] table
  muon                                                 - the Muon chain on 20 matrices [5120, 1280]
  step                                                 - one fused training micro-step (all kernels)
  attn_bwd_trace, attn_fwd_trace                       - clock stamps of the first backward / forward CTA
  mma_rate                                             - tcgen05.mma issue rate of one thread per SM (probe
                                                         kernel): rolled vs unrolled k-steps, N 128 / 256, TS
  delta_scan_fwd, delta_scan_bwd                       - chunked delta-rule scan, B*H = rows/4096*12, T 4096
  delta_gdn, delta_kda                                 - the fused chunked delta rule (chunk terms + scan),
                                                         forward + backward, bf16, T 4096, B*H = rows/4096*12
  fla_gdn, fla_kda                                     - FLA's chunk_kda on the same inputs (the library bar;
                                                         GDN through chunk_kda with a broadcast gate)
  sparse_fwd, sparse_bwd                               - block-sparse attention (NSA shape: 16 / 1 heads,
                                                         16 selected 64-key blocks per row), T 8192
  moe_fwd, moe_fwd_bwd                                 - grouped experts: 64 x (2048 -> 1024 -> 2048), top-8
  sinkhorn                                             - mHC Sinkhorn-Knopp (20 iterations) fwd + bwd
"""
import argparse
import json
import math
from pathlib import Path

import torch

WIDTH, HEADS, KV_HEADS, HEAD_DIM, FFN, VOCAB, SEQ = 1280, 10, 5, 128, 5120, 65536, 2048


def peaks():
    path = Path(__file__).resolve().parents[2] / "MEASURED_PEAKS.json"
    if not path.is_file():
        return {}
    raw = json.loads(path.read_text())
    flat = {}

    def walk(d):
        for k, v in d.items():
            if isinstance(v, dict):
                walk(v)
            elif isinstance(v, (int, float)):
                flat.setdefault(k, v)
    walk(raw)
    return flat


def timed(fn, iters, warmup):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for _ in range(iters):
        fn()
    b.record()
    torch.cuda.synchronize()
    return a.elapsed_time(b) / iters


def _bf16(*shape):
    return torch.randn(*shape, device="cuda").to(torch.bfloat16)


def case_gemm(kind, rows):
    from nexttransformer_b200.ops import gemm as G
    if kind == "gemm_qkv":
        a, w = _bf16(rows, WIDTH), _bf16(WIDTH + 2 * KV_HEADS * HEAD_DIM, WIDTH)
        out = torch.empty(rows, w.shape[0], device="cuda", dtype=torch.bfloat16)
        return (lambda: G.gemm(a, w, out)), 2 * rows * w.shape[0] * WIDTH
    if kind == "gemm_fc":
        a, w = _bf16(rows, WIDTH), _bf16(FFN, WIDTH)
        pre = torch.empty(rows, FFN, device="cuda", dtype=torch.bfloat16)
        act = torch.empty_like(pre)
        return (lambda: G.gemm(a, w, act, epi=G.EPI_RELU2, p=pre)), 2 * rows * FFN * WIDTH
    if kind == "gemm_proj":
        a, w, r = _bf16(rows, FFN), _bf16(WIDTH, FFN), _bf16(rows, WIDTH)
        out = torch.empty(rows, WIDTH, device="cuda", dtype=torch.bfloat16)
        return (lambda: G.gemm(a, w, out, epi=G.EPI_BF16_AXPBY, r=r)), 2 * rows * WIDTH * FFN
    if kind in ("gemm_wgrad", "gemm_wgrad_qkv", "gemm_wgrad_o"):
        # weight gradients of the MLP up-projection, the QKV projection and the output projection
        out_f = {"gemm_wgrad": FFN, "gemm_wgrad_qkv": (HEADS + 2 * KV_HEADS) * HEAD_DIM, "gemm_wgrad_o": WIDTH}[kind]
        dy, x = _bf16(rows, out_f), _bf16(rows, WIDTH)
        grad = torch.zeros(out_f, WIDTH, device="cuda")
        return (lambda: G.wgrad(dy, x, grad, accumulate=True)), 2 * rows * out_f * WIDTH
    if kind == "gemm_head":
        a, w = _bf16(rows, WIDTH), _bf16(VOCAB, WIDTH)
        out = torch.empty(rows, VOCAB, device="cuda", dtype=torch.bfloat16)
        return (lambda: G.gemm(a, w, out)), 2 * rows * VOCAB * WIDTH
    if kind == "gemm_head_ce":
        # the LM head with the soft-capped cross-entropy in its epilogue (the training path)
        from nexttransformer_b200.ops._ext import ext
        a, w = _bf16(rows, WIDTH), _bf16(VOCAB, WIDTH).mul_(0.2)
        out = torch.empty(rows, VOCAB, device="cuda", dtype=torch.bfloat16)
        tgt = torch.randint(0, VOCAB, (rows,), device="cuda")
        part = torch.empty(rows, (VOCAB + 127) // 128, device="cuda")
        ztgt, loss, rscale, rcorr = (torch.empty(rows, device="cuda") for _ in range(4))
        return (lambda: ext().gemm_ce_fwd(a, w, out, tgt, part, ztgt, loss, rscale, rcorr, VOCAB, 15.0)), \
            2 * rows * VOCAB * WIDTH
    raise ValueError(kind)


def _attn_flops(B, causal_pairs, fwd):
    per_pair = 4 * HEAD_DIM * HEADS      # QK^T and PV
    return B * causal_pairs * per_pair * (1 if fwd else 2.5)


def case_sdpa(kind, rows, backend):
    """torch SDPA (one backend forced) on the attention benchmark shape, [B, H, T, D] layout."""
    import torch.nn.functional as F
    from torch.nn.attention import SDPBackend, sdpa_kernel
    chosen = {"cudnn": SDPBackend.CUDNN_ATTENTION, "flash": SDPBackend.FLASH_ATTENTION,
              "efficient": SDPBackend.EFFICIENT_ATTENTION}[backend]
    B = max(1, rows // SEQ)
    q = _bf16(B, HEADS, SEQ, HEAD_DIM).mul_(0.3).requires_grad_(kind == "sdpa_bwd")
    k = _bf16(B, KV_HEADS, SEQ, HEAD_DIM).mul_(0.3).requires_grad_(kind == "sdpa_bwd")
    v = _bf16(B, KV_HEADS, SEQ, HEAD_DIM).mul_(0.3).requires_grad_(kind == "sdpa_bwd")
    pairs = SEQ * (SEQ + 1) // 2

    def run():
        with sdpa_kernel([chosen]):
            return F.scaled_dot_product_attention(q, k, v, is_causal=True, enable_gqa=True)
    if kind == "sdpa_fwd":
        return run, _attn_flops(B, pairs, True)
    y = run()
    dy = torch.randn_like(y)

    def bwd():
        with sdpa_kernel([chosen]):
            torch.autograd.grad(y, (q, k, v), dy, retain_graph=True)
    return bwd, _attn_flops(B, pairs, False)


def case_attn(kind, rows):
    from nexttransformer_b200.ops.attention import attention_fn
    B = max(1, rows // SEQ)
    M = B * SEQ
    qkv = _bf16(M, (HEADS + 2 * KV_HEADS) * HEAD_DIM).mul_(0.3).requires_grad_(kind == "attn_bwd")
    pairs = SEQ * (SEQ + 1) // 2
    if kind == "attn_fwd":
        return (lambda: attention_fn(qkv, B, SEQ, HEADS, KV_HEADS, HEAD_DIM, -1)), _attn_flops(B, pairs, True)
    y = attention_fn(qkv, B, SEQ, HEADS, KV_HEADS, HEAD_DIM, -1)
    dy = torch.randn_like(y)

    def bwd():
        torch.autograd.grad(y, qkv, dy, retain_graph=True)
    return bwd, _attn_flops(B, pairs, False)


def attn_bwd_trace(rows):
    """Pipeline stamps of the first backward CTA: per (role, pair) the SM-clock offsets of its events."""
    from nexttransformer_b200.ops._ext import ext
    lib = ext()
    B = max(1, rows // SEQ)
    M, H, Hk, D = B * SEQ, HEADS, KV_HEADS, HEAD_DIM
    qkv = _bf16(M, (H + 2 * Hk) * D).mul_(0.3)
    q, k, v = qkv[:, :H * D], qkv[:, H * D:(H + Hk) * D], qkv[:, (H + Hk) * D:]
    o = torch.empty(M, H * D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, H, SEQ, device="cuda")
    sc = 1.0 / math.sqrt(D)
    lib.attn_fwd(q, k, v, o, lse, B, SEQ, H, Hk, D, -1, sc)
    do = torch.randn_like(o)
    dqkv = torch.empty_like(qkv)
    trace = torch.zeros(4, 64, 8, dtype=torch.int64, device="cuda")
    for _ in range(2):
        trace.zero_()
        lib.attn_bwd(q, k, v, o, lse, do, dqkv[:, :H * D], dqkv[:, H * D:(H + Hk) * D], dqkv[:, (H + Hk) * D:],
                     torch.zeros(M, H * D, device="cuda"), torch.empty(B, H, SEQ, device="cuda"), B, SEQ, H, Hk, D, -1,
                     sc, trace)
    torch.cuda.synchronize()
    t = trace.cpu()
    base = int(t[t > 0].min())
    names = {0: "producer: q_empty do_empty", 1: "mma: - dP_issued p_full ds_full dq_issued",
             2: "softmax: stat s_full p_arrive dp_full prev_dq_full ds_arrive", 3: "drain: dq_full staged0 issued3"}
    out = {}
    for role in range(4):
        rows_ = []
        for it in range(16):
            ev = [int(x) - base if int(x) else None for x in t[role, it]]
            if any(e is not None for e in ev):
                rows_.append(ev)
        out[names[role]] = rows_
    return out


def attn_fwd_trace(rows):
    """Pipeline stamps of the first forward CTA: per (role, key tile) the SM-clock offsets of its events."""
    from nexttransformer_b200.ops._ext import ext
    B = max(1, rows // SEQ)
    M, H, Hk, D = B * SEQ, HEADS, KV_HEADS, HEAD_DIM
    qkv = _bf16(M, (H + 2 * Hk) * D).mul_(0.3)
    q, k, v = qkv[:, :H * D], qkv[:, H * D:(H + Hk) * D], qkv[:, (H + Hk) * D:]
    o = torch.empty(M, H * D, device="cuda", dtype=torch.bfloat16)
    lse = torch.empty(B, H, SEQ, device="cuda")
    trace = torch.zeros(4, 64, 8, dtype=torch.int64, device="cuda")
    for _ in range(2):
        trace.zero_()
        ext().attn_fwd_trace(q, k, v, o, lse, B, SEQ, H, Hk, D, -1, 1.0 / math.sqrt(D), trace)
    torch.cuda.synchronize()
    t = trace.cpu()
    base = int(t[t > 0].min())
    # MMA role: the four issues (stamped after their commit), then the four wait exits before them
    names = {1: "mma: S_A S_B PV_A PV_B issued, then ready S_A S_B PV_A PV_B",
             2: "softmax A: s_full loaded max rescaled p_arrive",
             3: "softmax B: s_full loaded max rescaled p_arrive"}
    out = {}
    for role, name in names.items():
        width = 8 if role == 1 else 5
        out[name] = [[int(x) - base if int(x) else None for x in t[role, it][:width]] for it in range(16)
                     if (t[role, it] > 0).any()]
    return out


def mma_rate(groups=4096):
    """tcgen05 issue rate: per probe variant, SM clocks per MMA of the issue loop and to completion (median
    over one CTA per SM) and the aggregate TFLOP/s from CUDA events."""
    from nexttransformer_b200.ops._ext import ext
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    variants = {0: ("rolled loop, run-time descriptors, SS 128x128x16", 128),
                1: ("unrolled, SS 128x128x16", 128), 2: ("unrolled, SS 128x256x16", 256),
                3: ("unrolled, TS (A from TMEM) 128x128x16", 128)}
    res = {}
    for v, (name, n) in variants.items():
        out = torch.zeros(sms, 3, dtype=torch.int64, device="cuda")
        ext().mma_rate(v, groups, out)              # warm-up
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        ext().mma_rate(v, groups, out)
        e1.record()
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        o = out.cpu()
        mmas = groups * 8
        res[name] = {"issue_clk_per_mma": float(o[:, 0].median()) / mmas,
                     "total_clk_per_mma": float(o[:, 1].median()) / mmas, "waits_ok": int(o[:, 2].sum()),
                     "tflops": sms * mmas * 2 * 128 * n * 16 / (ms * 1e-3) / 1e12}
    return res


def case_delta_fused(kind, rows):
    """Forward + backward of the whole chunked delta rule on [B, 4096, 12, 128] bf16 inputs."""
    import torch.nn.functional as F
    T, H, D = 4096, 12, 128
    B = max(1, rows // T)
    g = torch.Generator(device="cuda").manual_seed(0)
    q = torch.randn(B, T, H, D, device="cuda", generator=g)
    k = torch.randn(B, T, H, D, device="cuda", generator=g)
    v = torch.randn(B, T, H, D, device="cuda", generator=g).bfloat16().requires_grad_()
    beta = torch.rand(B, T, H, device="cuda", generator=g).requires_grad_()
    gdn = kind.endswith("gdn")
    if gdn:
        gate = (-F.softplus(torch.randn(B, T, H, device="cuda", generator=g)) * 0.3).requires_grad_()
    else:
        gate = (-F.softplus(torch.randn(B, T, H, D, device="cuda", generator=g)) * 0.05).requires_grad_()
        q, k = F.normalize(q, dim=-1) * D ** -.5, F.normalize(k, dim=-1)
    q, k = q.bfloat16().requires_grad_(), k.bfloat16().requires_grad_()
    if kind.startswith("fla_"):
        from fla.ops.kda import chunk_kda

        def run():
            gk = gate[..., None].expand(-1, -1, -1, D).contiguous() if gdn else gate
            y, _ = chunk_kda(q, k, v, gk, beta.bfloat16(), scale=D ** -.5 if gdn else 1.0,
                             use_qk_l2norm_in_kernel=gdn)
            return y
    else:
        from nexttransformer_b200.ops.linear_attention import delta_chunk_cuda

        def run():
            return delta_chunk_cuda(q, k, v, kind="gdn" if gdn else "kda", g=gate, beta=beta, chunk=64,
                                    qk_l2norm_scale=D ** -.5 if gdn else None)
    dy = torch.randn(B, T, H, D, device="cuda").bfloat16()

    def step():
        y = run()
        torch.autograd.grad(y, (q, k, v, beta, gate), dy.to(y.dtype))
    # 4 D^2 per token and head for the WY terms, 4 D^2 for the state products, 2 x for the backward
    flops = 3 * 8 * D * D * B * T * H
    return step, flops


def case_delta(kind, rows):
    from nexttransformer_b200.ops.linear_attention import _DeltaScan
    T, H = 4096, 12
    B = max(1, rows // T)
    N = T // 64
    g = torch.Generator(device="cuda").manual_seed(0)

    def r(*s):
        return (torch.randn(*s, device="cuda", generator=g) * 0.05).to(torch.bfloat16)
    w, u0, qt, kc, aqk = r(B, H, N, 64, 128), r(B, H, N, 64, 128), r(B, H, N, 64, 128), r(B, H, N, 64, 128), \
        r(B, H, N, 64, 64)
    carry = torch.full((B, H, N, 128), 0.97, device="cuda")
    flops_fwd = B * H * N * 2 * (128 * 128 * 128 + 2 * 64 * 64 * 128 + 128 * 64 * 128)
    if kind == "delta_scan_fwd":
        return (lambda: _DeltaScan.apply(w, u0, qt, kc, aqk, carry)), flops_fwd
    ins = [t.clone().requires_grad_() for t in (w, u0, qt, kc, aqk)] + [carry.clone().requires_grad_()]
    o = _DeltaScan.apply(*ins)
    do = torch.randn_like(o)
    return (lambda: torch.autograd.grad(o, ins, do, retain_graph=True)), 2 * flops_fwd


def case_sparse(kind, rows):
    from nexttransformer_b200.ops.sparse_attention import block_lists, block_sparse_attention
    T, H, Hk, D, nsel = 8192, 16, 1, 128, 16
    B = max(1, rows // T)
    NB = T // 64
    g = torch.Generator(device="cuda").manual_seed(0)
    score = torch.rand(B, 1, T, NB, device="cuda", generator=g)
    pos_blk = torch.arange(T, device="cuda") // 64
    allowed = torch.arange(NB, device="cuda")[None, :] <= pos_blk[:, None]
    top = score.masked_fill(~allowed, -1.0).topk(nsel, -1).indices
    blocks = torch.zeros(B, 1, T, NB, dtype=torch.bool, device="cuda").scatter_(-1, top, True) & allowed
    lists, masks = block_lists(blocks)
    q = _bf16(B, T, H, D).mul_(0.3).requires_grad_(kind == "sparse_bwd")
    k = _bf16(B, T, Hk, D).mul_(0.3).requires_grad_(kind == "sparse_bwd")
    v = _bf16(B, T, Hk, D).requires_grad_(kind == "sparse_bwd")
    pairs = int((blocks.repeat_interleave(64, -1)[..., :T] &
                 (torch.arange(T, device="cuda")[None, :] <= torch.arange(T, device="cuda")[:, None])).sum()) * H
    flops = 4 * D * pairs
    if kind == "sparse_fwd":
        return (lambda: block_sparse_attention(q, k, v, lists, masks)), flops
    y = block_sparse_attention(q, k, v, lists, masks)
    dy = torch.randn_like(y)
    return (lambda: torch.autograd.grad(y, (q, k, v), dy, retain_graph=True)), 2.5 * flops


def case_moe(kind, rows):
    from nexttransformer_b200.ops.moe import grouped_experts
    E, k, d, F = 64, 8, 2048, 1024
    T = rows // 4
    g = torch.Generator(device="cuda").manual_seed(0)
    x = _bf16(T, d).requires_grad_(kind == "moe_fwd_bwd")
    choice = torch.rand(T, E, device="cuda", generator=g).topk(k, -1).indices
    w = torch.full((T, k), 1.0 / k, device="cuda")
    wf = (torch.randn(E, F, d, device="cuda") * 0.02).requires_grad_(kind == "moe_fwd_bwd")
    wp = (torch.randn(E, d, F, device="cuda") * 0.02).requires_grad_(kind == "moe_fwd_bwd")
    flops = 2 * T * k * 2 * d * F
    if kind == "moe_fwd":
        return (lambda: grouped_experts(x, choice, w, wf, wp)), flops

    def run():
        y = grouped_experts(x, choice, w, wf, wp)
        torch.autograd.grad(y, (x, wf, wp), torch.ones_like(y))
    return run, 3 * flops


def case_sinkhorn(rows):
    from nexttransformer_b200.models.residual import sinkhorn_knopp
    z = torch.randn(rows, 4, 4, device="cuda").requires_grad_()
    g = torch.randn(rows, 4, 4, device="cuda")

    def run():
        torch.autograd.grad(sinkhorn_knopp(z, 20), z, g)
    return run, None, rows * 16 * 4 * 5


def case_ce(rows):
    from nexttransformer_b200.ops._ext import ext
    logits = _bf16(rows, VOCAB)
    tgt = torch.randint(0, VOCAB, (rows,), device="cuda")
    loss = torch.empty(rows, device="cuda")
    lse = torch.empty(rows, device="cuda")
    keep = logits.clone()

    def run():
        logits.copy_(keep)
        ext().softcap_ce(logits, tgt, loss, lse, VOCAB, 15.0)
    # the kernel reads the logits twice and writes the gradient once (the restore copy is extra)
    return run, None, 3 * logits.numel() * 2


def case_norm(kind, rows):
    """The shell's memory-bound row kernels on [rows, 1280] / the QKV rows (bytes: what each must move)."""
    from nexttransformer_b200.ops._ext import ext
    if kind == "mix_norm_fwd":
        x, x0 = _bf16(rows, WIDTH), _bf16(rows, WIDTH)
        ab = torch.tensor([0.9, 0.1], device="cuda")
        xm, h = torch.empty_like(x), torch.empty_like(x)
        return (lambda: ext().mix_norm_fwd(x, x0, ab, xm, h, None, 1.0)), None, 4 * x.numel() * 2
    if kind == "mix_norm_bwd":
        x, x0, xm, dh, dres = (_bf16(rows, WIDTH) for _ in range(5))
        ab = torch.tensor([0.9, 0.1], device="cuda")
        dx = torch.empty_like(x)
        dx0 = torch.zeros(rows, WIDTH, device="cuda")
        part = torch.empty(rows, 2, device="cuda")
        # reads x, x0, xm, dh, dres (bf16) and dx0 (fp32), writes dx (bf16) and dx0 (fp32)
        return (lambda: ext().mix_norm_bwd(x, x0, xm, dh, dres, ab, dx, dx0, part)), None, \
            x.numel() * (6 * 2 + 2 * 4)
    if kind in ("rope_norm_fwd", "rope_norm_bwd"):
        cols = (HEADS + 2 * KV_HEADS) * HEAD_DIM
        qkv = _bf16(rows, cols)
        ang = torch.arange(SEQ, device="cuda")[:, None] * torch.rand(HEAD_DIM // 2, device="cuda")[None]
        cosb, sinb = ang.cos().bfloat16().contiguous(), ang.sin().bfloat16().contiguous()
        rstd = torch.empty(rows * (HEADS + KV_HEADS), device="cuda")
        ext().rope_norm_fwd(qkv, cosb, sinb, rstd, SEQ, HEADS, KV_HEADS, HEAD_DIM, 1.2, None, None, None, None, None)
        qk = rows * (HEADS + KV_HEADS) * HEAD_DIM
        if kind == "rope_norm_fwd":
            # q / k rows read and written in place (v untouched without value embeddings)
            return (lambda: ext().rope_norm_fwd(qkv, cosb, sinb, rstd, SEQ, HEADS, KV_HEADS, HEAD_DIM, 1.2, None, None,
                                                None, None, None)), None, 2 * qk * 2
        dqkv = _bf16(rows, cols)
        return (lambda: ext().rope_norm_bwd(dqkv, qkv, cosb, sinb, rstd, SEQ, HEADS, KV_HEADS, HEAD_DIM, 1.2, None,
                                            None, None, None, None)), None, 3 * qk * 2
    raise ValueError(kind)


def case_adamw(rows):
    from nexttransformer_b200.ops._ext import ext
    p = torch.randn(rows, WIDTH, device="cuda")
    g, m, v = torch.randn_like(p), torch.zeros_like(p), torch.zeros_like(p)
    sh = torch.empty(rows, WIDTH, device="cuda", dtype=torch.bfloat16)
    step = [0]

    def run():
        step[0] += 1
        ext().adamw(p, g, m, v, sh, 1e-3, 0.8, 0.95, 1e-10, 0.01, step[0])
    # read p, g, m, v; write p, m, v (fp32) and the bf16 shadow
    return run, None, p.numel() * (7 * 4 + 2)


def case_muon(rows):
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    params = [torch.nn.Parameter(torch.randn(FFN, WIDTH, device="cuda") * 0.02) for _ in range(20)]
    for p in params:
        p.grad = torch.randn_like(p)
    opt = MuonAdamW([dict(kind="muon", params=params, lr=0.02, momentum=0.95, ns_steps=5, beta2=0.9,
                          weight_decay=0.0)])
    # 5 Polar-Express iterations x 3 GEMMs on tall [m, n] = [5120, 1280] matrices
    m, n = FFN, WIDTH
    flops = 20 * 5 * (2 * m * n * n + 2 * n * n * n + 2 * m * n * n)
    return (lambda: opt.step()), flops


def case_step(rows, layers):
    from nexttransformer_b200.models.shell import ShellConfig, build_shell
    B = max(1, rows // SEQ)
    model = build_shell(ShellConfig(sequence_len=SEQ, vocab_size=VOCAB, n_layer=layers, n_head=HEADS,
                                    n_kv_head=KV_HEADS, n_embd=WIDTH, window_pattern="L"), "cuda", seed=1)
    model.fused_state()
    model.train()
    tok = torch.randint(0, VOCAB, (B, SEQ + 1), device="cuda")
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()

    def run():
        model(x, y).backward()
    return run, model.estimate_flops() * B * SEQ


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("case")
    ap.add_argument("--rows", type=int, default=65536)
    ap.add_argument("--iters", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--layers", type=int, default=2)
    ap.add_argument("--seq", type=int, default=0, help="sequence length of the attention cases (default 2048)")
    ap.add_argument("--sdpa", choices=("cudnn", "flash", "efficient"), default="cudnn")
    a = ap.parse_args(argv)
    global SEQ
    if a.seq:
        SEQ = a.seq
    torch.manual_seed(0)
    byts = None
    if a.case == "attn_bwd_trace":
        print(json.dumps(attn_bwd_trace(a.rows)), flush=True)
        return
    if a.case == "mma_rate":
        print(json.dumps(mma_rate()), flush=True)
        return
    if a.case == "attn_fwd_trace":
        print(json.dumps(attn_fwd_trace(a.rows)), flush=True)
        return
    if a.case.startswith("gemm_"):
        fn, flops = case_gemm(a.case, a.rows)
    elif a.case.startswith("attn_"):
        fn, flops = case_attn(a.case, a.rows)
    elif a.case.startswith("sdpa_"):
        fn, flops = case_sdpa(a.case, a.rows, a.sdpa)
    elif a.case.startswith("delta_scan"):
        fn, flops = case_delta(a.case, a.rows)
    elif a.case in ("delta_gdn", "delta_kda", "fla_gdn", "fla_kda"):
        fn, flops = case_delta_fused(a.case, a.rows)
    elif a.case.startswith("sparse_"):
        fn, flops = case_sparse(a.case, a.rows)
    elif a.case.startswith("moe_"):
        fn, flops = case_moe(a.case, a.rows)
    elif a.case == "sinkhorn":
        fn, flops, byts = case_sinkhorn(a.rows)
    elif a.case == "ce":
        fn, flops, byts = case_ce(a.rows)
    elif a.case in ("mix_norm_fwd", "mix_norm_bwd", "rope_norm_fwd", "rope_norm_bwd"):
        fn, flops, byts = case_norm(a.case, a.rows)
    elif a.case == "adamw":
        fn, flops, byts = case_adamw(a.rows)
    elif a.case == "muon":
        fn, flops = case_muon(a.rows)
    elif a.case == "step":
        fn, flops = case_step(a.rows, a.layers)
    else:
        raise SystemExit(f"unknown case {a.case}")
    ms = timed(fn, a.iters, a.warmup)
    from nexttransformer_b200.ops._ext import check_errors
    check_errors()
    pk = peaks()
    out = {"case": a.case, "rows": a.rows, "seq": SEQ, "ms": ms, **({"sdpa": a.sdpa} if a.case.startswith("sdpa_") else {})}
    if flops:
        tf = flops / ms / 1e9
        out.update(tflops=tf)
        if "bf16_tflops" in pk:
            out.update(frac_of_measured_bf16=tf / pk["bf16_tflops"])
    if byts:
        gbs = byts / ms / 1e6
        out.update(gbps=gbs)
        if "hbm_gbs" in pk:
            out.update(frac_of_measured_hbm=gbs / pk["hbm_gbs"])
    print(json.dumps(out), flush=True)


if __name__ == "__main__":
    main()
