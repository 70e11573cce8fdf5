"""Expert-parallel MoE exchange over NVLink peer memory against the NCCL all-to-all path.

    torchrun --nproc-per-node 2 -m nexttransformer_b200.checks.moe_ep [--tokens 4096] [--iters 5]

Every rank builds the same MoE layer (same seed), shards its experts over the world, routes its
own tokens and runs forward + backward once with the peer-memory exchange (``parallel.expert.
PeerExpertExchange``: pull rows from the peers' send buffers, grouped expert GEMMs, push rows
back) and once with the NCCL all-to-all exchange.  Outputs, input gradients and the local
experts' weight gradients must agree to bf16 rounding.  Then both are timed with CUDA events on
the benchmark shape (d 2048, 64 experts of FFN 1024, top-8), maximum over ranks, and the bytes
that cross NVLink per rank are reported with the achieved fraction of the measured peer
bandwidth of this pool (770 GB/s per direction).
"""
import argparse
import json

import torch
import torch.distributed as dist

PEER_GBS = 770.0


def _layer(d, E, k, F, device, seed=7):
    from nexttransformer_b200.models.moe import MoEFFN
    torch.manual_seed(seed)
    m = MoEFFN(d, E, k, F, shared=1)
    for p in m.parameters():
        torch.nn.init.normal_(p, std=0.03)
    return m.to(device)


def _run(m, x, dy, mode):
    m.ep_exchange = mode
    for p in m.parameters():
        p.grad = None
    xi = x.clone().requires_grad_()
    y = m(xi)
    y.backward(dy)
    return y.detach(), xi.grad.detach(), [p.grad.detach().clone() if p.grad is not None else None for p in m.parameters()]


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-12)).item()


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--tokens", type=int, default=4096, help="tokens per rank for the timing")
    ap.add_argument("--iters", type=int, default=5)
    a = ap.parse_args(argv)
    from nexttransformer_b200.ops._ext import check_errors
    from nexttransformer_b200.parallel.expert import enable_expert_parallel
    from nexttransformer_b200.runtime.process import initialize, shutdown
    rank, world, device = initialize(0, timeout_s=120)

    # correctness on a small layer
    m = _layer(256, 8 * world, 2, 128, device)
    enable_expert_parallel(m)
    g = torch.Generator(device=device).manual_seed(100 + rank)
    x = torch.randn(333, 256, device=device, generator=g).to(torch.bfloat16)
    dy = torch.randn(333, 256, device=device, generator=g).to(torch.bfloat16)
    yp, gp, wp = _run(m, x, dy, "peer")
    yn, gn, wn = _run(m, x, dy, "nccl")
    torch.cuda.synchronize()
    check_errors()
    errs = dict(out=_rel(yp, yn), dx=_rel(gp, gn),
                dw=max((_rel(p, q) for p, q in zip(wp, wn) if p is not None and q is not None and q.norm() > 0),
                       default=0.0))
    worst = torch.tensor([max(errs.values())], device=device)
    dist.all_reduce(worst, op=dist.ReduceOp.MAX)

    # timing on the benchmark shape
    d, E, k, F = 2048, 64, 8, 1024
    big = _layer(d, E, k, F, device).to(torch.bfloat16)
    enable_expert_parallel(big)
    xb = torch.randn(a.tokens, d, device=device, generator=g).to(torch.bfloat16)
    dyb = torch.randn_like(xb)

    def step(mode):
        big.ep_exchange = mode
        xi = xb.clone().requires_grad_()
        big(xi).backward(dyb)

    def timed(mode):
        for _ in range(2):
            step(mode)
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            step(mode)
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    ms_peer = timed("peer")
    ms_nccl = timed("nccl")
    check_errors()
    # rows that leave this rank per step: forward dispatch + combine, backward dispatch + combine
    cross = 4 * a.tokens * k * d * 2 * (world - 1) / world
    res = dict(world=world, tokens_per_rank=a.tokens, rel_err=errs, max_rel_err=float(worst),
               ms_layer_fwd_bwd_peer=ms_peer, ms_layer_fwd_bwd_nccl=ms_nccl,
               nvlink_bytes_per_rank=cross, nvlink_floor_ms=cross / PEER_GBS / 1e6)
    if rank == 0:
        print(json.dumps(res), flush=True)
    shutdown()
    if float(worst) > 2e-2:
        raise SystemExit(f"peer exchange differs from the all-to-all path by {float(worst)}")
    return res


if __name__ == "__main__":
    main()
