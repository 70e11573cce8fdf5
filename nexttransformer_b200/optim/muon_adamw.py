"""Muon + AdamW with ZeRO-style ownership, on the sm_100a kernels.

The update rules are the reference's (``nanochat/optim.py``):
  * AdamW: decoupled decay ``p *= 1 - lr wd``, moments by lerp, bias correction, ``eps`` outside
    the square root.  Moments are kept in fp32 (the reference keeps them in the parameter's
    dtype, bf16 for embeddings).
  * Muon: Nesterov momentum by lerp -> bf16 -> MuonEq row equilibration -> Frobenius normalise
    (x 1.01) -> 5 Polar-Express quintic iterations with per-step coefficients (tall/wide
    forms) -> Muon+ renormalisation to sqrt(min(m, n)) -> NorMuon factored second moment
    (beta2) -> cautious weight decay; learning rate scaled by sqrt(max(1, m / n)).

Distribution (world > 1): each rank owns whole Muon matrices (``ceil(K / world)`` of every
same-shape group, in group order) and row slices of the large AdamW tensors.  Gradients are
reduced to their owner (averaged), the owner updates, and updated parameters are sent back
to every rank - reduce-scatter + all-gather volume, never a full all-reduce of gradients.
By default each Muon shape group moves as ONE stacked reduce-scatter and ONE all-gather (the
group's gradients copied into a persistent ``[chunk x world, m, n]`` buffer, the owner's chunk
reduced into a second one), the reference DistMuon's layout: 12 collectives for the six shape
groups of a dense model instead of two per matrix, whose per-call latency dominated the
exposed communication.  The per-matrix path serves the overlap mode, whose reductions start
layer by layer during the backward.

Gradients are read from ``p.main_grad`` when a fused path produced one, else ``p.grad``.

Overlap (``overlap_with(model)``, world > 1): the model's kernel state calls ``issue_reduce``
with each layer's parameters as soon as the last micro-batch's backward has finished that layer,
so their reductions run on NCCL's stream under the rest of the backward; ``step`` then only waits
for them.  After the update the parameter gathers are issued in the order the next forward
uses the parameters (embedding side, layer 0, 1, ..., head) and are not waited: the forward
waits for each layer's gathers right before the layer (``wait_gathers``), so the gathers run
under the preceding layers' compute.  ``flush()`` waits for every outstanding gather (before a
checkpoint, an evaluation or the end of a timed region).  This is the reference's DDP bucket
overlap (``nexttransformer/train.py:353-357``) and DistMuon's asynchronous phases
(``nanochat/optim.py:428-459``) arranged for a step whose forward waits per layer.
"""
import math

import torch
import torch.distributed as dist

POLAR_EXPRESS = (
    (8.156554524902461, -22.48329292557795, 15.878769915207462),
    (4.042929935166739, -2.808917465908714, 0.5000178451051316),
    (3.8916678022926607, -2.772484153217685, 0.5060648178503393),
    (3.285753657755655, -2.3681294933425376, 0.46449024233003106),
    (2.3465413258596377, -1.7097828382687081, 0.42323551169305323),
)


def grad_of(p):
    """The parameter's gradient for this update: ``main_grad`` where a kernel path owns one.

    A weight run through ``ops.dense.KernelLinear`` carries a gradient slot whose GEMM writes
    ``main_grad``; if that slot was never written this update (the layer did not run) its
    stale contents are replaced, and any gradient autograd produced for the same weight (a use
    outside the kernel path) is folded in.  Idempotent within one update."""
    g = getattr(p, "main_grad", None)
    if g is None:
        return p.grad
    slot = getattr(p, "_nt_slot", None)
    if slot is not None and slot.fresh:
        if p.grad is not None:
            g.copy_(p.grad)
        else:
            g.zero_()
        slot.fresh = False
        p.grad = None
    elif p.grad is not None and slot is not None:
        g.add_(p.grad)
        p.grad = None
    return g


# ------------------------------------------------------------------ reference math (any device)
@torch.no_grad()
def adamw_reference(p, g, m, v, step, lr, b1, b2, eps, wd):
    p32 = p.float()
    p32.mul_(1 - lr * wd)
    m.lerp_(g.float(), 1 - b1)
    v.lerp_(g.float().square(), 1 - b2)
    denom = (v / (1 - b2 ** step)).sqrt() + eps
    p32.add_(m / denom, alpha=-lr / (1 - b1 ** step))
    p.copy_(p32)


@torch.no_grad()
def muon_reference(grads, params, mom, smb, momentum, lr, wd, beta2, ns_steps, compute_dtype=torch.bfloat16):
    """One Muon step on stacked [K, m, n] tensors (grads are consumed)."""
    mom.lerp_(grads, 1 - momentum)
    g = grads.lerp_(mom, momentum)
    X = g.to(compute_dtype)
    target = X.float().norm(dim=(-2, -1), keepdim=True) / X.size(-2) ** 0.5
    rown = X.float().norm(dim=-1, keepdim=True).clamp_min(1e-6)
    X = X * (target / rown).to(X.dtype)
    X = X / (X.norm(dim=(-2, -1), keepdim=True) * 1.01 + 1e-6)
    tall = g.size(-2) > g.size(-1)
    for a, b, c in POLAR_EXPRESS[:ns_steps]:
        if tall:
            A = X.mT @ X
            X = a * X + X @ (b * A + c * (A @ A))
        else:
            A = X @ X.mT
            X = a * X + (b * A + c * (A @ A)) @ X
    g = X.to(params.dtype)
    g = g * (min(g.size(-2), g.size(-1)) ** 0.5 / g.float().norm(dim=(-2, -1), keepdim=True).clamp_min(1e-6)).to(g.dtype)
    red = -1 if g.size(-2) >= g.size(-1) else -2
    vmean = g.float().square().mean(dim=red, keepdim=True)
    rsize = g.size(red)
    vnorm = (vmean.sum(dim=(-2, -1), keepdim=True) * rsize).sqrt()
    smb.lerp_(vmean.to(smb.dtype), 1 - beta2)
    step = smb.clamp_min(1e-10).rsqrt()
    vnew = ((vmean * rsize) * step.float().square()).sum(dim=(-2, -1), keepdim=True).sqrt()
    g = g * (step * (vnorm / vnew.clamp_min(1e-10))).to(g.dtype)
    mask = (g * params) >= 0
    params.sub_(lr * g + lr * wd * params * mask)


# ------------------------------------------------------------------ optimizer
class MuonAdamW(torch.optim.Optimizer):
    """param_groups: dicts with ``kind`` 'adamw' (lr, betas, eps, weight_decay) or 'muon'
    (lr, momentum, ns_steps, beta2, weight_decay); every Muon group holds same-shape matrices."""

    def __init__(self, param_groups, shadows=None):
        super().__init__(param_groups, defaults={})
        # fp32 master -> bf16 shadow written by the update (the fused forward reads shadows)
        self.shadows = shadows or {}
        self._work = {}
        # Optional peer-memory reduce-scatter (parallel.symmetric.PeerReduceScatter) and the set of
        # parameters whose gradients it averages in place; the others use NCCL collectives.
        self.p2p, self.p2p_params = None, frozenset()
        self.gather, self.gather_params = None, frozenset()
        # overlap state: parameter -> forward-use group, early-issued reductions, deferred gathers
        self.use_group = {}
        self.defer_gathers = False
        # grouped reduce-scatter / all-gather of Muon matrices: True on CUDA, "always" on any device
        # (gloo supports both collectives; the CPU tests use it), False: per-matrix reduce / broadcast
        self.stack_muon = True
        self._stacks = {}
        self._stack_finish = []
        self._early = {}
        self._pending = {}
        self._meta = None

    def use_peer_reduce_scatter(self, reducer, covered):
        self.p2p, self.p2p_params = reducer, frozenset(covered)

    # -------------------------------------------------------------- overlap
    def overlap_with(self, model):
        """Reduce each layer's gradients during the backward and let the next forward wait for each
        layer's gathered parameters (no effect on one rank).  Needs the model's fused trunk."""
        st = model.fused_state()
        self.use_group = {p: g for g, ps in st.use_groups().items() for p in ps}
        self.defer_gathers = True
        st.optimizer = self
        self._overlap_state = st

    def overlap_off(self):
        """Suspend the overlap (returns what ``overlap_restore`` needs)."""
        state = getattr(self, "_overlap_state", None)
        saved = (self.defer_gathers, state.optimizer if state is not None else None)
        self.defer_gathers = False
        if state is not None:
            state.optimizer = None
        return saved

    def overlap_restore(self, saved):
        self.defer_gathers = saved[0]
        state = getattr(self, "_overlap_state", None)
        if state is not None:
            state.optimizer = saved[1]

    def _param_meta(self):
        """parameter -> ('adamw', group) or ('muon', group, index in its group)."""
        if self._meta is None:
            meta = {}
            for group in self.param_groups:
                for i, p in enumerate(group["params"]):
                    meta[p] = (group["kind"], group, i)
            self._meta = meta
        return self._meta

    def issue_reduce(self, params):
        """Start the reductions of ``params`` now (their gradients are final for this update)."""
        rank, world = self._dist()
        if world == 1:
            return
        meta = self._param_meta()
        for p in params:
            if p in self._early or p in self.p2p_params or p not in meta:
                continue
            kind, group, i = meta[p]
            if kind == "adamw":
                self._early[p] = self._adamw_issue(p, rank, world)
            else:
                chunk = math.ceil(len(group["params"]) / world)
                self._early[p] = self._muon_issue(p, min(i // chunk, world - 1))

    def wait_gathers(self, group):
        """Make the current stream wait for the gathers of forward-use group ``group`` and refresh
        those parameters' bf16 shadows."""
        items = self._pending.pop(group, None)
        if not items:
            return
        for kind, p, item in items:
            if kind != "shadow":
                item.wait()
        for kind, p, item in items:
            if kind == "shadow":
                item.copy_(p.data)

    def flush(self):
        """Wait for every outstanding parameter gather (all groups, in use order)."""
        for group in sorted(self._pending):
            self.wait_gathers(group)

    def state_dict(self):
        self.flush()
        return super().state_dict()

    def use_peer_gather(self, gather, covered):
        """Parameters in ``covered`` (fp32 masters in a symmetric arena) are all-gathered, shadows
        included, by ``gather()`` at the end of every step instead of NCCL broadcasts / gathers."""
        self.gather, self.gather_params = gather, frozenset(covered)

    # -------------------------------------------------------------- helpers
    @staticmethod
    def _dist():
        if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
            return dist.get_rank(), dist.get_world_size()
        return 0, 1

    def _adamw_state(self, p, rows):
        st = self.state[p]
        if not st:
            st["step"] = 0
            st["rows"] = rows
            shape = (rows.stop - rows.start, *p.shape[1:]) if rows is not None else p.shape
            st["exp_avg"] = torch.zeros(shape, device=p.device, dtype=torch.float32)
            st["exp_avg_sq"] = torch.zeros(shape, device=p.device, dtype=torch.float32)
        return st

    # -------------------------------------------------------------- AdamW
    def _adamw_issue(self, p, rank, world):
        """(param, row slice or None, reduce work handle, reduced grad slice) of one parameter."""
        g = grad_of(p)
        if g is None:
            raise RuntimeError("missing gradient in the fixed training graph")
        if world == 1:
            return (p, None, None, g)
        if p in self.p2p_params:
            n = p.shape[0] // world   # this rank's rows were averaged in place by the peer kernel
            return (p, slice(rank * n, (rank + 1) * n), None, g[slice(rank * n, (rank + 1) * n)])
        if p.numel() < 1024 or p.shape[0] % world:
            return (p, None, dist.all_reduce(g, op=dist.ReduceOp.AVG, async_op=True), g)
        n = p.shape[0] // world
        out = torch.empty((n, *g.shape[1:]), device=g.device, dtype=g.dtype)
        work = dist.reduce_scatter_tensor(out, g.contiguous(), op=dist.ReduceOp.AVG, async_op=True)
        return (p, slice(rank * n, (rank + 1) * n), work, out)

    def _adamw_plan(self, group, rank, world):
        """Plans of a group's parameters; on several ranks the small tensors (updated whole on every
        rank) share ONE averaging all-reduce of their concatenated gradients."""
        plans, small = [], []
        for p in group["params"]:
            early = self._early.pop(p, None)
            if early is not None:
                plans.append(early)
                continue
            g = grad_of(p)
            if (world > 1 and g is not None and p not in self.p2p_params and g.is_cuda
                    and (p.numel() < 1024 or p.shape[0] % world)):
                small.append(len(plans))
                plans.append((p, None, None, g))
                continue
            plans.append(self._adamw_issue(p, rank, world))
        if small:
            grads = [plans[i][3] for i in small]
            flat = torch.cat([g.reshape(-1).float() for g in grads])
            work = dist.all_reduce(flat, op=dist.ReduceOp.AVG, async_op=True)
            off = 0
            for i, g in zip(small, grads):
                n = g.numel()
                plans[i] = (plans[i][0], None, work, flat[off:off + n].view(g.shape))
                off += n
        return plans

    def _adamw_apply(self, group, plans, world, gathers):
        b1, b2 = group["betas"]
        for p, rows, work, g in plans:
            if work is not None:
                work.wait()
            st = self._adamw_state(p, rows)
            st["step"] += 1
            pv = p.data if rows is None else p.data[rows]
            gv = g if g.dtype == torch.float32 else g.float()
            shadow = self.shadows.get(p)
            if pv.is_cuda:
                from nexttransformer_b200.ops._ext import ext
                sh = None
                if shadow is not None and rows is None and shadow.is_contiguous():
                    sh = shadow
                ext().adamw(pv, gv.contiguous(), st["exp_avg"], st["exp_avg_sq"], sh, group["lr"], b1, b2,
                            group["eps"], group["weight_decay"], st["step"])
                if shadow is not None and sh is None and p not in self.gather_params:
                    gathers.append(("shadow", p, shadow))
            else:
                adamw_reference(pv, gv, st["exp_avg"], st["exp_avg_sq"], st["step"], group["lr"], b1, b2,
                                group["eps"], group["weight_decay"])
            if rows is not None and p not in self.gather_params:
                gathers.append(("adamw", p, lambda p=p, rows=rows: dist.all_gather_into_tensor(
                    p.data, p.data[rows].contiguous(), async_op=True)))

    # -------------------------------------------------------------- Muon
    def _muon_owned(self, group, rank, world):
        params = group["params"]
        chunk = math.ceil(len(params) / world)
        lo = rank * chunk
        return params, chunk, list(range(lo, min(lo + chunk, len(params))))

    @staticmethod
    def _muon_issue(p, owner):
        return dist.reduce(grad_of(p), dst=owner, op=dist.ReduceOp.SUM, async_op=True)

    def _stacked(self, group, world):
        return (world > 1 and self.stack_muon and not self.defer_gathers
                and (group["params"][0].is_cuda or self.stack_muon == "always")
                and not any(p in self.p2p_params or p in self.gather_params or p in self._early
                            for p in group["params"]))

    def _stack(self, group, name, shape, like):
        key = (id(group), name)
        buf = self._stacks.get(key)
        if buf is None or tuple(buf.shape) != tuple(shape):
            buf = torch.zeros(shape, device=like.device, dtype=torch.float32)
            self._stacks[key] = buf
        return buf

    def _muon_reduce(self, group, rank, world):
        params, chunk, _ = self._muon_owned(group, rank, world)
        if world == 1:
            return []
        if self._stacked(group, world):
            m, n = params[0].shape[-2:]
            grads = [grad_of(p) for p in params]
            full = self._stack(group, "grads", (chunk * world, m, n), params[0])
            mine = self._stack(group, "mine", (chunk, m, n), params[0])
            torch._foreach_copy_(list(full[:len(params)].unbind(0)), [g.float() for g in grads])
            return ("stacked", dist.reduce_scatter_tensor(mine, full, op=dist.ReduceOp.SUM, async_op=True), mine)
        works = []
        for i, p in enumerate(params):
            if p in self.p2p_params:
                continue
            work = self._early.pop(p, None)
            works.append(work if work is not None else self._muon_issue(p, min(i // chunk, world - 1)))
        return works

    def _muon_apply(self, group, rank, world, works, gathers):
        stacked = isinstance(works, tuple) and works and works[0] == "stacked"
        if stacked:
            works[1].wait()
            reduced = works[2]
        else:
            for w in works:
                w.wait()
        params, chunk, owned = self._muon_owned(group, rank, world)
        shape = params[0].shape
        m, n = shape[-2], shape[-1]
        lr = group["lr"] * max(1.0, m / n) ** 0.5
        if owned:
            mine = [params[i] for i in owned]
            for p in mine:
                st = self.state[p]
                if "momentum_buffer" not in st:
                    st["momentum_buffer"] = torch.zeros_like(p, dtype=torch.float32)
                    st["second_momentum_buffer"] = torch.zeros((m, 1) if m >= n else (1, n), device=p.device,
                                                               dtype=torch.float32)
            own_grads = None
            if stacked:
                own_grads = list(reduced[:len(mine)].unbind(0))
                reduced.div_(world)
            elif world > 1:
                for p in mine:
                    if p not in self.p2p_params:
                        grad_of(p).div_(world)
            if mine[0].is_cuda and self.gemm_shape_ok(m, n):
                self._muon_cuda(group, mine, m, n, lr, own_grads)
            else:
                grads = torch.stack(own_grads if own_grads is not None else [grad_of(p).float() for p in mine])
                stack = torch.stack([p.data for p in mine])
                mom = torch.stack([self.state[p]["momentum_buffer"] for p in mine])
                smb = torch.stack([self.state[p]["second_momentum_buffer"] for p in mine])
                muon_reference(grads, stack, mom, smb, group["momentum"], lr, group["weight_decay"], group["beta2"],
                               group["ns_steps"], torch.bfloat16)
                for j, p in enumerate(mine):
                    p.data.copy_(stack[j])
                    self.state[p]["momentum_buffer"].copy_(mom[j])
                    self.state[p]["second_momentum_buffer"].copy_(smb[j])
                    if p in self.shadows:
                        self.shadows[p].copy_(p.data)
        if stacked:
            # the owner's updated matrices go out in one all-gather of the group's stack
            m, n = params[0].shape[-2:]
            if owned:
                torch._foreach_copy_(list(reduced[:len(owned)].unbind(0)), [params[i].data for i in owned])
            full = self._stack(group, "params", (chunk * world, m, n), params[0])
            work = dist.all_gather_into_tensor(full, reduced, async_op=True)
            self._stack_finish.append((work, full, params))
            return
        if world > 1:
            for i, p in enumerate(params):
                if p in self.gather_params:
                    continue
                src = min(i // chunk, world - 1)
                gathers.append(("muon", p, lambda p=p, src=src: dist.broadcast(p.data, src=src, async_op=True)))
                if p in self.shadows:
                    gathers.append(("shadow", p, self.shadows[p]))

    @staticmethod
    def gemm_shape_ok(m, n):
        """TMA needs 16-byte row strides; tiny matrices (e.g. value-embedding gates) use the plain path."""
        return m % 8 == 0 and n % 8 == 0 and min(m, n) >= 64

    def _ptrs(self, tensors):
        return torch.tensor([t.data_ptr() for t in tensors], dtype=torch.int64).to(tensors[0].device,
                                                                                   non_blocking=True)

    def _muon_cuda(self, group, mine, m, n, lr, grads=None):
        from nexttransformer_b200.ops._ext import ext
        from nexttransformer_b200.ops import gemm as G
        lib = ext()
        K = len(mine)
        dev = mine[0].device
        key = (m, n, K)
        if key not in self._work:
            s = min(m, n)
            L = m if m >= n else n
            self._work[key] = dict(
                X=torch.empty(K, m, n, device=dev, dtype=torch.bfloat16),
                X2=torch.empty(K, m, n, device=dev, dtype=torch.bfloat16),
                A=torch.empty(K, s, s, device=dev, dtype=torch.bfloat16),
                Bm=torch.empty(K, s, s, device=dev, dtype=torch.bfloat16),
                rowss=torch.empty(K, m, device=dev, dtype=torch.float32),
                tot=torch.empty(K, device=dev, dtype=torch.float32),
                red=torch.empty(K, L, device=dev, dtype=torch.float32),
                fscale=torch.empty(K, L, device=dev, dtype=torch.float32))
        w = self._work[key]
        if grads is None:
            grads = [grad_of(p) for p in mine]
        if any(g.dtype != torch.float32 or not g.is_contiguous() for g in grads):
            grads = [g.float().contiguous() for g in grads]
        g_ptr = self._ptrs(grads)
        m_ptr = self._ptrs([self.state[p]["momentum_buffer"] for p in mine])
        s_ptr = self._ptrs([self.state[p]["second_momentum_buffer"] for p in mine])
        p_ptr = self._ptrs([p.data for p in mine])
        shadows = [self.shadows.get(p) for p in mine]
        sh_ptr = self._ptrs(shadows) if all(s is not None and s.is_contiguous() for s in shadows) else None
        X, X2, A, Bm = w["X"], w["X2"], w["A"], w["Bm"]
        lib.muon_prep(g_ptr, m_ptr, X, w["rowss"], group["momentum"])
        lib.muon_normalize(X, w["rowss"], w["tot"])
        tall = m > n
        for a, b, c in POLAR_EXPRESS[:group["ns_steps"]]:
            if tall:
                G.gemm(X, X, A, a_mn=True, b_mn=True)
                G.gemm(A, A, Bm, b_mn=True, epi=G.EPI_BF16_AXPBY, r=A, s_acc=c, s_res=b)
                G.gemm(X, Bm, X2, b_mn=True, epi=G.EPI_BF16_AXPBY, r=X, s_acc=1.0, s_res=a)
            else:
                G.gemm(X, X, A)
                G.gemm(A, A, Bm, b_mn=True, epi=G.EPI_BF16_AXPBY, r=A, s_acc=c, s_res=b)
                G.gemm(Bm, X, X2, b_mn=True, epi=G.EPI_BF16_AXPBY, r=X, s_acc=1.0, s_res=a)
            X, X2 = X2, X
        lib.muon_finish(X, w["red"], w["tot"], s_ptr, w["fscale"], p_ptr, sh_ptr, group["beta2"], lr,
                        group["weight_decay"])
        if sh_ptr is None:
            for p, s in zip(mine, shadows):
                if s is not None:
                    s.copy_(p.data)

    # -------------------------------------------------------------- step
    @torch.no_grad()
    def step(self):
        self.flush()
        rank, world = self._dist()
        if self.p2p is not None and world > 1:
            self.p2p()
        plans = []
        for group in self.param_groups:
            if group["kind"] == "adamw":
                plans.append(self._adamw_plan(group, rank, world))
            elif group["kind"] == "muon":
                plans.append(self._muon_reduce(group, rank, world))
            else:
                raise ValueError(f"unknown optimizer kind {group['kind']!r}")
        gathers = []
        for group, plan in zip(self.param_groups, plans):
            if group["kind"] == "adamw":
                self._adamw_apply(group, plan, world, gathers)
            else:
                self._muon_apply(group, rank, world, plan, gathers)
        if self._early:
            raise RuntimeError("a reduction was started for a parameter outside the optimizer's groups")
        # gathers start after every update, in the order the next forward uses the parameters
        order = sorted(range(len(gathers)), key=lambda j: (self.use_group.get(gathers[j][1], -1), j))
        pending = {}
        for j in order:
            kind, p, item = gathers[j]
            pending.setdefault(self.use_group.get(p, -1), []).append((kind, p, item if kind == "shadow" else item()))
        self._pending = pending
        if not self.defer_gathers:
            self.flush()
        for work, full, params in self._stack_finish:
            work.wait()
            torch._foreach_copy_([p.data for p in params], list(full[:len(params)].unbind(0)))
            for p in params:
                if p in self.shadows:
                    self.shadows[p].copy_(p.data)
        self._stack_finish = []
        if self.gather is not None and world > 1:
            self.gather()
