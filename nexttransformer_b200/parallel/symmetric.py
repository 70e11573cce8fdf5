"""Gradients in symmetric memory and the peer-memory reduce-scatter that averages them.

``GradArena`` lays every fp32 gradient buffer out in one flat allocation (each buffer 256-byte
aligned).  With a process group the allocation is symmetric memory (``torch.distributed.
_symmetric_memory``): the same buffer is mapped into every rank's address space over NVLink, so a
kernel can read every peer's gradients directly.

``ParamArena`` / ``PeerParamGather`` do the reverse for the parameters: the fp32 masters of the
covered parameters move into a symmetric allocation laid out like the gradient arena, every
owner updates its segments in place, and one kernel per update (after an entry barrier) reads
every other owner's segments with plain peer loads and writes the bf16 shadows the forward reads
- the parameter all-gather and the shadow cast in one pass.

``PeerReduceScatter`` turns the optimizer's ownership (whole Muon matrices per owner rank, row
shards of the large AdamW tables) into per-rank segment tables and runs ``csrc/comm.cu``: one
kernel per update reads the owned segments from every peer, averages them in a fixed order and
writes them in place; the bounded flag barriers inside the kernel order it against the peers'
backward passes.  Parameters it cannot handle (small tensors, unaligned shards) stay on NCCL.
"""
import torch
import torch.distributed as dist

ALIGN = 64  # elements (256 bytes)


def peer_pointers(tensor, handle, rank):
    """Device addresses of `tensor` on every rank: the handle's buffer pointers are the bases of the
    symmetric allocations, and a tensor can start at an offset inside its allocation (the allocator
    pools symmetric memory), the same offset on every rank."""
    offset = tensor.data_ptr() - int(handle.buffer_ptrs[rank])
    return [int(p) + offset for p in handle.buffer_ptrs]


def _blocks(blocks, handle, world, device):
    """Grid size of the reduce-scatter / gather kernels: the signal pad holds four slot regions
    (entry and exit of each kernel) of one 32-bit slot per (block, peer)."""
    pad_slots = handle.signal_pad_size // 4
    return max(1, min(blocks or 2 * torch.cuda.get_device_properties(device).multi_processor_count,
                      pad_slots // (4 * world)))


class GradArena:
    def __init__(self, shapes, device, group=None):
        self.offsets, total = [], 0
        for shape in shapes:
            n = 1
            for s in shape:
                n *= int(s)
            self.offsets.append((total, tuple(shape), n))
            total += (n + ALIGN - 1) // ALIGN * ALIGN
        self.total = max(total, ALIGN)
        self.handle = None
        if group is not None:
            import torch.distributed._symmetric_memory as symm
            self.buf = symm.empty(self.total, dtype=torch.float32, device=device)
            self.buf.zero_()
            self.handle = symm.rendezvous(self.buf, group)
        else:
            self.buf = torch.zeros(self.total, dtype=torch.float32, device=device)
        self._next = 0

    def alloc(self, shape):
        """The next buffer, in the order of ``shapes`` (each call must ask for the planned shape)."""
        off, planned, n = self.offsets[self._next]
        if tuple(shape) != planned:
            raise RuntimeError(f"arena request {tuple(shape)} differs from the plan {planned}")
        self._next += 1
        return self.buf[off:off + n].view(planned)

    def offset_of(self, view):
        """Element offset of a view into the arena."""
        return (view.data_ptr() - self.buf.data_ptr()) // 4


def fused_state_with_arena(model, group=None):
    """Build the model's fused-path state with every gradient buffer inside one ``GradArena``."""
    from nexttransformer_b200.models.fused_dense import FusedState
    shapes = []
    FusedState(model, grad_alloc=lambda shape: shapes.append(tuple(shape)) or torch.empty(0), plan_only=True)
    arena = GradArena(shapes, model.get_device(), group)
    model._fused = FusedState(model, grad_alloc=arena.alloc)
    model._fused.arena = arena
    return model._fused


class PeerReduceScatter:
    """Average every owned gradient segment over the data-parallel ranks through peer memory."""

    def __init__(self, arena, ownership, rank, world, blocks=None, timeout_s=60.0):
        if arena.handle is None:
            raise ValueError("the gradient arena is not in symmetric memory")
        self.arena = arena   # keeps the symmetric-memory handle (peer mappings) alive
        h = arena.handle
        dev = arena.buf.device
        self.rank, self.world, self.timeout_s = rank, world, timeout_s
        self.peers = torch.tensor(peer_pointers(arena.buf, h, rank), dtype=torch.int64, device=dev)
        self.pads = torch.tensor(list(h.signal_pad_ptrs), dtype=torch.int64, device=dev)
        self.blocks = _blocks(blocks, h, world, dev)
        mine = [(o, n) for (o, n, owner) in ownership if owner == rank]
        if any(o % 4 or n % 4 for o, n in mine):
            raise ValueError("segments must start and end on 16-byte boundaries")
        self.seg_off = torch.tensor([o for o, _ in mine] or [0], dtype=torch.int64, device=dev)
        self.seg_len = torch.tensor([n for _, n in mine] or [0], dtype=torch.int64, device=dev)
        self.epoch = 0

    def __call__(self):
        from nexttransformer_b200.ops._ext import ext
        self.epoch += 1
        ext().p2p_reduce_scatter(self.peers, self.pads, self.seg_off, self.seg_len, self.rank, self.world,
                                 1.0 / self.world, self.epoch, self.blocks, self.timeout_s)

    @staticmethod
    def check_errors():
        from nexttransformer_b200.ops._ext import ext
        code, where = ext().read_comm_errors()
        if code:
            raise RuntimeError(f"peer reduce-scatter: a barrier wait expired (code {code} at {where:#x})")


def ownership_segments(optimizer, arena, world):
    """[(element offset, length, owner rank)] of every gradient the peer reduce-scatter averages,
    plus the set of parameters it covers (the rest stays on NCCL).  Ownership is the optimizer's:
    Muon matrices by index chunks of their shape group, AdamW tables by equal row shards."""
    import math
    from nexttransformer_b200.optim.muon_adamw import grad_of
    segs, covered = [], set()
    for group in optimizer.param_groups:
        params = group["params"]
        if group["kind"] == "muon":
            chunk = math.ceil(len(params) / world)
            for i, p in enumerate(params):
                g = grad_of(p)
                if g is None or not g.is_contiguous():
                    continue
                off = arena.offset_of(g)
                if off % 4 or g.numel() % 4:
                    continue
                segs.append((off, g.numel(), min(i // chunk, world - 1)))
                covered.add(p)
        else:
            for p in params:
                g = grad_of(p)
                if g is None or not g.is_contiguous() or p.numel() < 1024 or p.shape[0] % world:
                    continue
                rows = p.shape[0] // world
                per = rows * (p.numel() // p.shape[0])
                off = arena.offset_of(g)
                if off % 4 or per % 4:
                    continue
                segs.extend((off + r * per, per, r) for r in range(world))
                covered.add(p)
    return segs, covered


def param_segments(optimizer, arena, world):
    """[(element offset, length, owner, param, param offset)] in the gradient arena's layout for
    every fp32 parameter the peer reduce-scatter covers (same ownership as ``ownership_segments``).
    Parameters kept in another dtype (the bf16 embedding tables on CUDA) stay out: the arena holds
    fp32 masters, and moving a bf16 table into it would change the dtype its kernels read."""
    import math
    from nexttransformer_b200.optim.muon_adamw import grad_of
    out = []
    for group in optimizer.param_groups:
        params = group["params"]
        if group["kind"] == "muon":
            chunk = math.ceil(len(params) / world)
            for i, p in enumerate(params):
                g = grad_of(p)
                if g is None or not g.is_contiguous() or p.dtype != torch.float32:
                    continue
                off = arena.offset_of(g)
                if off % 4 or g.numel() % 4:
                    continue
                out.append((off, g.numel(), min(i // chunk, world - 1), p, off))
        else:
            for p in params:
                g = grad_of(p)
                if (g is None or not g.is_contiguous() or p.numel() < 1024 or p.shape[0] % world
                        or p.dtype != torch.float32):
                    continue
                per = p.shape[0] // world * (p.numel() // p.shape[0])
                off = arena.offset_of(g)
                if off % 4 or per % 4:
                    continue
                out.extend((off + r * per, per, r, p, off) for r in range(world))
    return out


class ParamArena:
    """fp32 masters of the covered parameters in symmetric memory, at their gradients' offsets."""

    def __init__(self, grad_arena, segments, group):
        import torch.distributed._symmetric_memory as symm
        self.buf = symm.empty(grad_arena.total, dtype=torch.float32, device=grad_arena.buf.device)
        self.buf.zero_()
        self.handle = symm.rendezvous(self.buf, group)
        self.params = {}
        for _, _, _, p, base in segments:
            if p in self.params:
                continue
            if p.dtype != torch.float32:
                raise ValueError("the parameter arena holds fp32 masters only")
            view = self.buf[base:base + p.numel()].view(p.shape)
            view.copy_(p.data)
            p.data = view
            self.params[p] = base


class PeerParamGather:
    """All-gather of the updated parameters (and their bf16 shadows) through peer memory."""

    def __init__(self, arena, segments, shadows, rank, world, blocks=None, timeout_s=60.0):
        # the arena (its buffer and symmetric-memory handle, i.e. the peer mappings) lives as long
        # as this object: the kernel reads the peers' buffers through those mappings
        self.arena = arena
        h = arena.handle
        dev = arena.buf.device
        self.rank, self.world, self.timeout_s = rank, world, timeout_s
        self.peers = torch.tensor(peer_pointers(arena.buf, h, rank), dtype=torch.int64, device=dev)
        self.pads = torch.tensor(list(h.signal_pad_ptrs), dtype=torch.int64, device=dev)
        self.blocks = _blocks(blocks, h, world, dev)
        offs, lens, owners, shadow = [], [], [], []
        for off, n, owner, p, base in segments:
            sh = shadows.get(p)
            ok = sh is not None and sh.is_contiguous() and sh.dtype == torch.bfloat16
            offs.append(off)
            lens.append(n)
            owners.append(owner)
            shadow.append(sh.data_ptr() + (off - base) * 2 if ok else 0)
        self.covered = frozenset(p for *_, p, _ in segments)
        self.seg_off = torch.tensor(offs or [0], dtype=torch.int64, device=dev)
        self.seg_len = torch.tensor(lens or [0], dtype=torch.int64, device=dev)
        self.seg_owner = torch.tensor(owners or [0], dtype=torch.int32, device=dev)
        self.seg_shadow = torch.tensor(shadow or [0], dtype=torch.int64, device=dev)
        self.epoch = 0

    def __call__(self):
        from nexttransformer_b200.ops._ext import ext
        self.epoch += 1
        ext().p2p_gather(self.peers, self.pads, self.seg_off, self.seg_len, self.seg_owner, self.seg_shadow,
                         self.rank, self.world, self.epoch, self.blocks, self.timeout_s)
