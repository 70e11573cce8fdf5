"""Peer-memory reduce-scatter against NCCL on the GPUs of one node (one process per GPU).

    torchrun --nproc-per-node 2 -m nexttransformer_b200.checks.comm [--mib 256] [--iters 10]

Each rank fills a symmetric-memory gradient arena with rank-dependent values; the peer kernel
averages every rank's owned segment in place; the result must match NCCL's average of the same
data to fp32 rounding (NCCL adds in its own order).  Then both are timed with CUDA events, the
maximum over ranks is taken, and the achieved bus bandwidth ((N-1)/N x bytes / time) is printed
with its fraction of the measured per-direction peer bandwidth of this pool (770 GB/s).
"""
import argparse
import json
import os

import torch
import torch.distributed as dist

PEER_GBS = 770.0


def check_gather(rank, world, device):
    """Parameter all-gather through peer memory: every rank owns row shards and whole matrices of a
    synthetic layout, writes its own values, and after the gather every rank must hold every owner's
    values exactly (fp32 masters) and their bf16 casts (shadows)."""
    import types
    from nexttransformer_b200.parallel.symmetric import GradArena, ParamArena, PeerParamGather
    shapes = [(1024, 256), (640, 128), (2048, 64)]
    arena = GradArena(shapes, device, group=dist.group.WORLD)
    grads = [arena.alloc(s) for s in shapes]
    params = [torch.nn.Parameter(torch.zeros(s, device=device)) for s in shapes]
    segs = []
    for i, (p, g) in enumerate(zip(params, grads)):
        base = arena.offset_of(g)
        if i == 1:                                      # a whole matrix owned by one rank
            segs.append((base, p.numel(), i % world, p, base))
        else:                                           # equal row shards
            per = p.numel() // world
            segs.extend((base + r * per, per, r, p, base) for r in range(world))
    pa = ParamArena(arena, segs, dist.group.WORLD)
    shadows = {p: torch.zeros(p.shape, device=device, dtype=torch.bfloat16) for p in params}
    gather = PeerParamGather(pa, segs, shadows, rank, world)
    flat = {id(p): p.data.view(-1) for p in params}
    for off, n, owner, p, base in segs:
        if owner == rank:
            idx = torch.arange(n, device=device, dtype=torch.float32)
            flat[id(p)][off - base:off - base + n] = (owner + 1) * 1000.0 + idx % 977
    torch.cuda.synchronize()
    dist.barrier()
    gather()
    torch.cuda.synchronize()
    err = 0.0
    for off, n, owner, p, base in segs:
        idx = torch.arange(n, device=device, dtype=torch.float32)
        want = (owner + 1) * 1000.0 + idx % 977
        got = flat[id(p)][off - base:off - base + n]
        err = max(err, (got - want).abs().max().item())
        sh = shadows[p].view(-1)[off - base:off - base + n].float()
        err = max(err, (sh - want.to(torch.bfloat16).float()).abs().max().item())
    t = torch.tensor([err], device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    del gather, pa, arena
    return float(t)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--mib", type=int, default=256, help="arena size in MiB of fp32")
    ap.add_argument("--iters", type=int, default=10)
    a = ap.parse_args(argv)
    from nexttransformer_b200.parallel.symmetric import GradArena, PeerReduceScatter
    from nexttransformer_b200.runtime.process import initialize, shutdown
    rank, world, device = initialize(0, timeout_s=120)
    n = a.mib * (1 << 20) // 4
    n -= n % (64 * world)
    arena = GradArena([(n,)], device, group=dist.group.WORLD)
    buf = arena.alloc((n,))
    per = n // world
    segs = [(r * per, per, r) for r in range(world)]
    red = PeerReduceScatter(arena, segs, rank, world)
    g = torch.Generator(device=device).manual_seed(1234 + rank)
    data = torch.randn(n, device=device, generator=g)
    buf.copy_(data)
    ref = data.clone()
    dist.all_reduce(ref)
    ref /= world
    torch.cuda.synchronize()
    red()
    torch.cuda.synchronize()
    red.check_errors()
    mine = buf[rank * per:(rank + 1) * per]
    err = (mine - ref[rank * per:(rank + 1) * per]).abs().max().item()

    def timed(fn):
        for _ in range(2):
            fn()
        dist.barrier()
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(a.iters):
            fn()
        e.record()
        torch.cuda.synchronize()
        t = torch.tensor([s.elapsed_time(e) / a.iters], device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t)

    out = torch.empty(per, device=device)
    ms_p2p = timed(red)
    ms_nccl = timed(lambda: dist.reduce_scatter_tensor(out, data, op=dist.ReduceOp.AVG))
    red.check_errors()
    bytes_ = n * 4 * (world - 1) / world
    res = dict(world=world, mib=a.mib, max_abs_err=err, ms_p2p=ms_p2p, ms_nccl=ms_nccl,
               busbw_p2p_gbs=bytes_ / ms_p2p / 1e6, busbw_nccl_gbs=bytes_ / ms_nccl / 1e6,
               frac_of_peer_peak_p2p=bytes_ / ms_p2p / 1e6 / PEER_GBS)
    if rank == 0:
        print(json.dumps(res), flush=True)
    gather_err = check_gather(rank, world, device)
    res["gather_max_abs_err"] = gather_err
    if rank == 0:
        print(json.dumps({"param_gather_max_abs_err": gather_err}), flush=True)
    del red, arena, buf
    shutdown()
    if gather_err > 0:
        raise SystemExit(f"peer parameter gather differs from the owners' values by {gather_err}")
    if err > 1e-5:
        raise SystemExit(f"peer reduce-scatter differs from NCCL by {err}")
    return res


if __name__ == "__main__":
    main()
