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
    del red, arena, buf
    shutdown()
    if err > 1e-5:
        raise SystemExit(f"peer reduce-scatter differs from NCCL by {err}")
    return res


if __name__ == "__main__":
    main()
