"""Expert- and tensor-parallel algorithms on gloo ranks (CPU) against single-process references."""
import os

import pytest
import torch
import torch.multiprocessing as mp

from tests.conftest import free_port


def _init(rank, world, port):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), CUDA_VISIBLE_DEVICES="")
    dist.init_process_group("gloo", rank=rank, world_size=world)
    return dist


def _ep_worker(rank, world, port, q):
    dist = _init(rank, world, port)
    from nexttransformer_b200.models.moe import MoEFFN
    from nexttransformer_b200.parallel.expert import enable_expert_parallel
    torch.manual_seed(0)
    ref = MoEFFN(16, num_experts=4, top_k=2, expert_width=8)
    with torch.no_grad():
        for p in ref.parameters():
            p.normal_(0, 0.3)
    ep = MoEFFN(16, num_experts=4, top_k=2, expert_width=8)
    ep.load_state_dict(ref.state_dict())
    enable_expert_parallel(ep)
    torch.manual_seed(1)
    x_all = torch.randn(world, 12, 16)
    x = x_all[rank].clone().requires_grad_()
    y = ep(x)
    xr = x_all[rank].clone().requires_grad_()
    yr = ref(xr)
    fwd = (y - yr).abs().max().item()
    y.square().sum().backward()
    yr.square().sum().backward()
    dx = (x.grad - xr.grad).abs().max().item()
    # expert weights: the owner's gradient equals the sum of the reference gradients over ranks
    own = [i for i in range(4) if i // 2 == rank]
    g_all = torch.stack([ref.experts[i].c_fc.weight.grad for i in range(4)])
    dist.all_reduce(g_all)
    assert len(ep.local_experts()) == 2     # only this rank's experts are held
    g_ep = torch.cat([ep.expert(i).c_fc.weight.grad.flatten() for i in own])
    g_ref = torch.cat([g_all[i].flatten() for i in own])
    q.put((rank, fwd, dx, (g_ep - g_ref).abs().max().item()))
    dist.destroy_process_group()


def _tp_worker(rank, world, port, q):
    dist = _init(rank, world, port)
    from nexttransformer_b200.models.shell import MLP, ShellConfig
    from nexttransformer_b200.parallel.tensor import MLPTP
    torch.manual_seed(0)
    dense = MLP(ShellConfig(n_embd=16, n_head=2, n_kv_head=2, mlp_width=32))
    with torch.no_grad():
        for p in dense.parameters():
            p.normal_(0, .2)
    tp = MLPTP.from_dense(dense)
    torch.manual_seed(2)
    x = torch.randn(8, 16)
    rows = x.shape[0] // world
    y_shard = tp(x[rank * rows:(rank + 1) * rows])
    ref = dense(x)[rank * rows:(rank + 1) * rows]
    q.put((rank, (y_shard - ref).abs().max().item()))
    dist.destroy_process_group()


def _tp_model_worker(rank, world, port, q):
    dist = _init(rank, world, port)
    import copy
    from nexttransformer_b200.models.shell import ShellConfig, build_shell
    from nexttransformer_b200.parallel.tensor import enable_tensor_parallel
    cfg = ShellConfig(sequence_len=16, vocab_size=64, n_layer=2, n_head=2, n_kv_head=2, n_embd=32, mlp_width=64)
    dense = build_shell(cfg, "cpu", seed=3)
    with torch.no_grad():  # signal through the zero-initialised output projections
        for blk in dense.transformer.h:
            blk.attn.c_proj.weight.normal_(0, 0.1)
            blk.mlp.c_proj.weight.normal_(0, 0.1)
    tp = copy.deepcopy(dense)
    assert enable_tensor_parallel(tp) == cfg.n_layer
    g = torch.Generator().manual_seed(5)
    idx = torch.randint(0, 64, (2, 16), generator=g)
    tgt = torch.randint(0, 64, (2, 16), generator=g)
    ld, lt = dense(idx, tgt), tp(idx, tgt)
    ld.backward()
    lt.backward()
    err = abs(ld.item() - lt.item())
    dg = dict(dense.named_parameters())
    size = dist.get_world_size()
    for name, p in tp.named_parameters():
        if ".mlp.tp." in name:
            full = dg[name.replace(".mlp.tp.", ".mlp.")].grad
            if name.endswith("c_fc.weight"):
                n = full.shape[0] // size
                ref = full[rank * n:(rank + 1) * n]
            else:
                n = full.shape[1] // size
                ref = full[:, rank * n:(rank + 1) * n]
        else:
            ref = dg[name].grad
        err = max(err, (p.grad - ref).abs().max().item())
    q.put((rank, err))
    dist.destroy_process_group()


@pytest.mark.parametrize("worker", ["ep", "tp", "tp_model"])
def test_parallel_matches_reference(worker):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = free_port()
    fn = {"ep": _ep_worker, "tp": _tp_worker, "tp_model": _tp_model_worker}[worker]
    procs = [ctx.Process(target=fn, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=300)
        assert p.exitcode == 0
    for _ in range(2):
        vals = q.get()
        assert max(vals[1:]) < 1e-4, vals


def _sharded_worker(rank, port, results):
    import os
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    from nexttransformer_b200.training.sharded import ExperimentOptimizer

    def make():
        torch.manual_seed(0)
        ps = [torch.nn.Parameter(torch.randn(64, 32)), torch.nn.Parameter(torch.randn(3)),
              torch.nn.Parameter(torch.randn(32, 32)), torch.nn.Parameter(torch.randn(32, 32))]
        groups = [dict(kind="adamw", params=ps[:2], lr=1e-2, betas=(0.9, 0.95), eps=1e-10, weight_decay=0.01),
                  dict(kind="muon", params=ps[2:], lr=2e-2, momentum=0.95, ns_steps=5, beta2=0.9, weight_decay=0.1)]
        return ps, groups
    ref_p, ref_g = make()
    sh_p, sh_g = make()
    ref, sharded = MuonAdamW(ref_g), ExperimentOptimizer(sh_g)
    for step in range(2):
        g = torch.Generator().manual_seed(100 * step + rank)
        local = [torch.randn(p.shape, generator=g) for p in ref_p]
        for p, x in zip(ref_p, local):
            p.grad = x.clone()
        for p, x in zip(sh_p, local):          # what DDP would hand over: the average
            avg = x.clone()
            dist.all_reduce(avg)
            p.grad = avg / 2
        ref.step()
        sharded.step()
    results[rank] = max(float((a - b).abs().max()) for a, b in zip(ref_p, sh_p))
    dist.destroy_process_group()


def test_experiment_optimizer_matches_owner_reduction():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        results = m.dict()
        mp.start_processes(_sharded_worker, args=(port, results), nprocs=2, start_method="spawn")
        assert results[0] < 1e-5 and results[1] < 1e-5, dict(results)


def test_param_segments_keep_bf16_tables_out():
    """The fp32 parameter arena of the peer gather never takes a bf16 table (its kernels read bf16)."""
    import torch
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    from nexttransformer_b200.parallel.symmetric import GradArena, ownership_segments, param_segments
    table = torch.nn.Parameter(torch.zeros(64, 32, dtype=torch.bfloat16))
    head = torch.nn.Parameter(torch.zeros(64, 32))
    mats = [torch.nn.Parameter(torch.zeros(32, 32)) for _ in range(2)]
    params = [table, head, *mats]
    arena = GradArena([tuple(p.shape) for p in params], "cpu")
    for p in params:
        p.main_grad = arena.alloc(p.shape)
    opt = MuonAdamW([dict(kind="adamw", params=[table, head], lr=1e-3, betas=(0.9, 0.95), eps=1e-10,
                          weight_decay=0.0),
                     dict(kind="muon", params=mats, lr=1e-2, momentum=0.95, ns_steps=5, beta2=0.9,
                          weight_decay=0.0)])
    segs, covered = ownership_segments(opt, arena, 2)
    assert table in covered and head in covered            # gradients are fp32 either way
    psegs = param_segments(opt, arena, 2)
    got = {id(p) for *_, p, _ in psegs}
    assert id(table) not in got and {id(head), id(mats[0]), id(mats[1])} <= got
    assert len([s for s in psegs if s[3] is head]) == 2    # one row shard per owner


def _overlap_worker(rank, port, results):
    """Early per-group reductions and deferred, use-ordered gathers give the same update."""
    import os
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=2)
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW

    def make():
        torch.manual_seed(0)
        ps = [torch.nn.Parameter(torch.randn(64, 32)), torch.nn.Parameter(torch.randn(3)),
              *[torch.nn.Parameter(torch.randn(32, 32)) for _ in range(3)], torch.nn.Parameter(torch.randn(48, 32))]
        groups = [dict(kind="adamw", params=[ps[0], ps[1], ps[5]], lr=1e-2, betas=(0.9, 0.95), eps=1e-10,
                       weight_decay=0.01),
                  dict(kind="muon", params=ps[2:5], lr=2e-2, momentum=0.95, ns_steps=5, beta2=0.9, weight_decay=0.1)]
        return ps, groups
    ref_p, ref_g = make()
    ov_p, ov_g = make()
    ref, ov = MuonAdamW(ref_g), MuonAdamW(ov_g)
    # forward-use groups: -1 the small vector, 0 two matrices and the table, 1 the rest
    ov.use_group = {ov_p[1]: -1, ov_p[0]: 0, ov_p[2]: 0, ov_p[3]: 0, ov_p[4]: 1, ov_p[5]: 1}
    ov.defer_gathers = True
    for step in range(3):
        g = torch.Generator().manual_seed(100 * step + rank)
        local = [torch.randn(p.shape, generator=g) for p in ref_p]
        for p, x in zip(ref_p, local):
            p.grad = x.clone()
        for p, x in zip(ov_p, local):
            p.grad = x.clone()
        ov.issue_reduce([ov_p[4], ov_p[0]])      # as the backward would, layer by layer
        ov.issue_reduce([ov_p[2], ov_p[3]])
        ref.step()
        ov.step()
        assert set(ov._pending) <= {-1, 0, 1}
        for group in (-1, 0, 1):                 # as the next forward would
            ov.wait_gathers(group)
        assert not ov._pending
    results[rank] = max(float((a - b).abs().max()) for a, b in zip(ref_p, ov_p))
    dist.destroy_process_group()


def test_overlapped_reduce_and_deferred_gathers_match():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        results = m.dict()
        mp.start_processes(_overlap_worker, args=(port, results), nprocs=2, start_method="spawn")
        assert results[0] == 0.0 and results[1] == 0.0, dict(results)


def _stacked_worker(rank, world, port, results):
    """Stacked Muon reduce-scatter / all-gather equals the per-matrix reduce / broadcast at several
    world sizes, shape groups with fewer matrices than ranks included."""
    import os
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW

    def make():
        torch.manual_seed(0)
        ps = [*[torch.nn.Parameter(torch.randn(32, 16)) for _ in range(5)], torch.nn.Parameter(torch.randn(24, 40)),
              *[torch.nn.Parameter(torch.randn(16, 16)) for _ in range(2)]]
        return ps, [dict(kind="muon", params=ps[:5], lr=2e-2, momentum=0.95, ns_steps=5, beta2=0.9, weight_decay=0.1),
                    dict(kind="muon", params=ps[5:6], lr=2e-2, momentum=0.95, ns_steps=5, beta2=0.9, weight_decay=0.1),
                    dict(kind="muon", params=ps[6:], lr=2e-2, momentum=0.95, ns_steps=5, beta2=0.9, weight_decay=0.1)]
    ref_p, ref_g = make()
    st_p, st_g = make()
    ref, st = MuonAdamW(ref_g), MuonAdamW(st_g)
    ref.stack_muon, st.stack_muon = False, "always"
    for step in range(3):
        g = torch.Generator().manual_seed(100 * step + rank)
        for a, b in zip(ref_p, st_p):
            a.grad = torch.randn(a.shape, generator=g)
            b.grad = a.grad.clone()
        ref.step()
        st.step()
    diff = max(float((a - b).abs().max()) for a, b in zip(ref_p, st_p))
    gathered = [torch.zeros(1) for _ in range(world)]
    dist.all_gather(gathered, torch.tensor([float(sum(p.sum() for p in st_p))]))
    results[rank] = (diff, max(float(x) for x in gathered) - min(float(x) for x in gathered))
    dist.destroy_process_group()


@pytest.mark.parametrize("world", [3, 4])
def test_stacked_muon_matches_per_matrix(world):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    with mp.Manager() as m:
        results = m.dict()
        mp.start_processes(_stacked_worker, args=(world, port, results), nprocs=world, start_method="spawn")
        for r in range(world):
            diff, spread = results[r]
            assert diff < 1e-5 and spread == 0.0, dict(results)
