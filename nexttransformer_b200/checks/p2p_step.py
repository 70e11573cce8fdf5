"""Training steps with the peer-memory gradient reduce-scatter (K8) and parameter gather (K9),
checked update by update on the GPUs of one node (one process per GPU).

    RS=1 GATHER=1 torchrun --nproc-per-node 2 -m nexttransformer_b200.checks.p2p_step
    RS=0 GATHER=0 torchrun --nproc-per-node 2 -m nexttransformer_b200.checks.p2p_step   # NCCL only

The benchmark's dense GQA model at LAYERS layers (default 4) runs four updates of two micro-batches
of rank-dependent random tokens.  After every update rank 0 prints the mean loss over ranks, the
parameters whose sums differ between ranks or are not finite, and the bf16 shadows that differ from
the casts of their fp32 masters; a correct peer path prints no parameter and no shadow, and the same
loss curve as the NCCL-only run.
"""
from datetime import timedelta
import os

import torch
import torch.distributed as dist

MODEL = dict(sequence_len=2048, vocab_size=65536, n_layer=20, n_head=10, n_kv_head=5, n_embd=1280, window_pattern="L")


def main():
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    dev = torch.device("cuda", int(os.environ["LOCAL_RANK"]))
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from nexttransformer_b200.models.shell import ShellConfig, build_shell
    from nexttransformer_b200.optim.groups import shell_groups
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    from nexttransformer_b200.parallel.symmetric import (ParamArena, PeerParamGather, PeerReduceScatter,
                                                         fused_state_with_arena, ownership_segments, param_segments)
    cfg = dict(MODEL, n_layer=int(os.environ.get("LAYERS", "4")))
    model = build_shell(ShellConfig(**cfg), dev, seed=42)
    rs_on, gather_on = os.environ.get("RS", "1") == "1", os.environ.get("GATHER", "1") == "1"
    st = fused_state_with_arena(model, dist.group.WORLD) if rs_on or gather_on else model.fused_state()
    opt = MuonAdamW(shell_groups(model), shadows={p: s for p, s in st.casts})
    if rs_on:
        segs, covered = ownership_segments(opt, st.arena, world)
        opt.use_peer_reduce_scatter(PeerReduceScatter(st.arena, segs, rank, world), covered)
    if gather_on:
        psegs = param_segments(opt, st.arena, world)
        gather = PeerParamGather(ParamArena(st.arena, psegs, dist.group.WORLD), psegs,
                                 {p: s for p, s in st.casts}, rank, world)
        opt.use_peer_gather(gather, gather.covered)
    names = {p: n for n, p in model.named_parameters()}
    T, B = cfg["sequence_len"], 4
    for step in range(4):
        model.zero_main_grads()
        for p in model.parameters():
            p.grad = None
        tot = 0.0
        for m in range(2):
            g = torch.Generator(device="cpu").manual_seed(1000 * step + 10 * m + rank)
            x = torch.randint(0, cfg["vocab_size"], (B, T + 1), generator=g).to(dev)
            loss = model(x[:, :-1], x[:, 1:])
            (loss / 2).backward()
            tot += loss.item() / 2
        mean = torch.tensor([tot], device=dev)
        dist.all_reduce(mean, op=dist.ReduceOp.AVG)
        opt.step()
        torch.cuda.synchronize()
        bad = []
        for p in model.parameters():
            s = torch.tensor([p.data.double().sum().item(), p.data.double().abs().sum().item()], device=dev)
            every = [torch.zeros_like(s) for _ in range(world)]
            dist.all_gather(every, s)
            if not all(torch.equal(every[0], v) for v in every) or not torch.isfinite(s).all():
                bad.append(names[p])
        stale = [names[p] for p, s in st.casts if not torch.equal(s, p.data.to(torch.bfloat16))]
        if rank == 0:
            print(f"rs={rs_on} gather={gather_on} step {step} mean loss {mean.item():.5f} "
                  f"differing/nonfinite {len(bad)} {bad[:3]} stale shadows {len(stale)}", flush=True)
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
