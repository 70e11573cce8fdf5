"""Owner-sharded Muon/AdamW for gradients that arrive already averaged (``ExperimentOptimizer`` of
``nexttransformer/training/sharded.py`` in the reference, which runs under DDP).

``MuonAdamW`` reduces every gradient to its owner itself (reduce-scatter / reduce, never a full
all-reduce).  When something else has already averaged the gradients on every rank - DDP's bucketed
all-reduce, or a caller's own collective - this subclass skips that reduce phase: each rank takes
its own rows of the large AdamW tables and its own Muon matrices straight from the averaged local
gradients, updates them, and the all-gathers / broadcasts of the updated parameters run as in
``MuonAdamW``.  Small AdamW tensors (fewer than 1024 elements or rows not divisible by the world)
are updated whole on every rank, as in ``MuonAdamW``.
"""
from nexttransformer_b200.optim.muon_adamw import MuonAdamW, grad_of


class ExperimentOptimizer(MuonAdamW):
    def __init__(self, param_groups, shadows=None):
        super().__init__(param_groups, shadows=shadows)
        # every gradient is already the average: the Muon owners must not divide again
        self.p2p_params = frozenset(p for g in self.param_groups for p in g["params"])

    def _adamw_plan(self, group, rank, world):
        plans = []
        for p in group["params"]:
            g = grad_of(p)
            if g is None:
                raise RuntimeError("missing gradient in the fixed training graph")
            if world == 1 or p.numel() < 1024 or p.shape[0] % world:
                plans.append((p, None, None, g))
            else:
                n = p.shape[0] // world
                rows = slice(rank * n, (rank + 1) * n)
                plans.append((p, rows, None, g[rows]))
        return plans

    def _muon_reduce(self, group, rank, world):
        return []
