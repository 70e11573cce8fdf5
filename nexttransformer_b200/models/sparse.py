"""Sparse-attention mixers: DSA, QSA, Seer (learned indexers), NSA (three branches) and MoBA.

Selection semantics follow ``nexttransformer/models/sparse.py`` of the reference:
  * DSA / QSA / Seer: an indexer (its own q heads, one shared key, partial RoPE, ReLU scores)
    selects tokens (DSA) or blocks (QSA complete blocks + the final incomplete tail, Seer complete
    blocks + forced current block); it is trained only by a KL self-distillation loss towards the
    head-mean of the dense causal softmax, after a burn-in of dense attention.
  * NSA: compressed branch (MLP over key/value blocks + learned position), top-n block selection
    from the compressed scores, local sliding window; per-head sigmoid branch gates.  A compression
    stride smaller than the block (overlapping blocks) is supported; importance of overlapping
    compressed blocks is pooled onto selection blocks.
  * MoBA: mean-pooled key blocks gate top-k historical blocks plus the forced current block.
The attention over selected keys runs as gathered attention with a probability-saving backward
(``IndexedAttention``); on CUDA the block-sparse kernels of ``ops.sparse_attention`` take over.
GQA is supported (key/value heads shared by groups of query heads).
"""
import torch
from torch import nn
from torch.nn import functional as F

from nexttransformer_b200.models.shell import Linear, apply_rotary_emb, norm

BACKENDS = ("reference", "kernel")


def safe_softmax(scores, valid):
    scores = scores.masked_fill(~valid, -torch.inf)
    nonempty = valid.any(-1, keepdim=True)
    scores = torch.where(nonempty, scores, torch.zeros_like(scores))
    return scores.softmax(-1) * valid.to(scores.dtype)


def gather_keys(x, idx):
    """x [B,H,T,D], idx [B,H,Q,K] -> [B,H,Q,K,D] (expanded view, no copy before gather)."""
    B, H, _, D = x.shape
    Q, K = idx.shape[-2:]
    return x[:, :, None].expand(-1, -1, Q, -1, -1).gather(3, idx[..., None].expand(B, H, Q, K, D))


class IndexedAttention(torch.autograd.Function):
    """softmax over the selected keys only; backward recomputes nothing but the gathers."""

    @staticmethod
    def forward(ctx, q, k, v, idx, valid):
        kk, vv = gather_keys(k, idx), gather_keys(v, idx)
        scale = q.shape[-1] ** -.5
        acc = torch.float64 if q.dtype == torch.float64 else torch.float32
        s = (q.to(acc).unsqueeze(-2) * kk.to(acc)).sum(-1) * scale
        p = safe_softmax(s, valid)
        y = (p[..., None] * vv.to(acc)).sum(-2)
        ctx.save_for_backward(q, k, v, idx, p)
        ctx.scale = scale
        return y.to(q.dtype)

    @staticmethod
    def backward(ctx, dy):
        q, k, v, idx, p = ctx.saved_tensors
        acc = p.dtype
        kk, vv = gather_keys(k, idx).to(acc), gather_keys(v, idx).to(acc)
        g = dy.to(acc).unsqueeze(-2)
        dp = (g * vv).sum(-1)
        ds = p * (dp - (dp * p).sum(-1, keepdim=True)) * ctx.scale
        dq = (ds[..., None] * kk).sum(-2)
        B, H, T, D = k.shape
        flat = idx.reshape(B, H, -1, 1)
        dk = torch.zeros_like(k, dtype=acc).scatter_add(2, flat.expand(-1, -1, -1, D),
                                                         (ds[..., None] * q.to(acc).unsqueeze(-2)).reshape(B, H, -1, D))
        Dv = v.shape[-1]
        dv = torch.zeros_like(v, dtype=acc).scatter_add(2, flat.expand(-1, -1, -1, Dv),
                                                         (p[..., None] * g).reshape(B, H, -1, Dv))
        return dq.to(q.dtype), dk.to(k.dtype), dv.to(v.dtype), None, None


def indexed_attention(q, k, v, idx, valid):
    return IndexedAttention.apply(q, k, v, idx, valid)


def indices_to_mask(idx, valid, T):
    m = torch.zeros(*idx.shape[:-1], T, dtype=torch.int32, device=idx.device)
    m.scatter_add_(-1, idx, valid.to(torch.int32))
    return m > 0


def select_tokens(scores, allowed, k):
    n = min(k, scores.shape[-1])
    chosen = scores.masked_fill(~allowed, -torch.inf).topk(n, dim=-1).indices
    return chosen, allowed.expand_as(scores).gather(-1, chosen)


def block_indices(scores, full_visible, pos, size, T, topk):
    """Top-k complete historical blocks plus the forced current (partial) block, as token indices."""
    B, H, Q, nb = scores.shape
    cur = pos // size
    eligible = full_visible & (torch.arange(nb, device=scores.device)[None, :] != cur[:, None])
    chosen, ok = select_tokens(scores, eligible[None, None], topk)
    off = torch.arange(size, device=scores.device)
    idx = (chosen[..., None] * size + off).flatten(-2)
    valid = ok[..., None].expand(-1, -1, -1, -1, size).flatten(-2)
    tail = (cur[:, None] * size + off)[None, None].expand(B, H, -1, -1)
    idx = torch.cat((idx, tail), -1)
    valid = torch.cat((valid, torch.ones_like(tail, dtype=torch.bool)), -1)
    valid = valid & (idx <= pos[None, None, :, None]) & (idx < T)
    return idx.clamp_max(T - 1), valid


def qsa_indices(scores, complete, pos, size, T, budget):
    """QSA: top complete blocks (within a token budget) then the final incomplete tail."""
    top = max(1, (budget + size - 1) // size)
    chosen, ok = select_tokens(scores, complete[None, None], top)
    off = torch.arange(size, device=scores.device)
    idx = (chosen[..., None] * size + off).flatten(-2)[..., :budget]
    valid = ok[..., None].expand(*ok.shape, size).flatten(-2)[..., :budget]
    tail = ((pos + 1) // size * size)[:, None] + off
    tail = tail[None, None].expand(*scores.shape[:3], size)
    tail_ok = (tail <= pos[None, None, :, None]) & (tail < T)
    return torch.cat((idx, tail), -1).clamp_max(T - 1), torch.cat((valid, tail_ok), -1)


def pool_teacher(teacher, size, blocks, kind):
    g = F.pad(teacher, (0, blocks * size - teacher.shape[-1])).reshape(*teacher.shape[:-1], blocks, size)
    return g.amax(-1) if kind == "qsa" else g.sum(-1)


def pool_blocks(x, size):
    B, H, T, D = x.shape
    n = (T + size - 1) // size
    return F.pad(x, (0, 0, 0, n * size - T)).reshape(B, H, n, size, D).mean(-2)


def partial_rope(x, pos, dim):
    if not dim:
        return x
    inv = 100000. ** (-torch.arange(0, dim, 2, device=x.device, dtype=torch.float32) / dim)
    ang = pos.float()[:, None] * inv[None]
    cos, sin = ang.cos().to(x)[None, :, None], ang.sin().to(x)[None, :, None]
    return torch.cat((apply_rotary_emb(x[..., :dim], cos, sin), x[..., dim:]), -1)


class SparseMixer(nn.Module):
    def __init__(self, config, layer_idx, kind=None):
        super().__init__()
        from nexttransformer_b200.models.shell import CausalSelfAttention, ShellConfig
        self.config = config
        self.kind = kind or config.method
        d, H, Hk, D = config.width, config.heads, config.n_kv_head, config.head_dim
        self.n_head, self.n_kv_head, self.head_dim = H, Hk, D
        self.c_q = Linear(d, H * D, bias=False)
        self.c_k = Linear(d, Hk * D, bias=False)
        self.c_v = Linear(d, Hk * D, bias=False)
        self.c_proj = Linear(H * D, d, bias=False)
        from nexttransformer_b200.models.shell import has_ve
        self.ve_gate = Linear(12, Hk, bias=False) if (config.value_embeddings and has_ve(layer_idx, config.n_layer)) \
            else None
        self.in_burnin = True
        self.backend = "reference"
        self.last_aux = None
        self.last_stats = {}
        if self.kind in ("dsa", "qsa", "seer"):
            self.index_q = Linear(d, config.index_heads * config.index_dim, bias=False)
            self.index_k = Linear(d, config.index_dim, bias=False)
            if self.kind == "dsa":
                self.index_weights = Linear(d, config.index_heads, bias=False)
                self.index_norm = nn.LayerNorm(config.index_dim)
        if self.kind == "nsa":
            size = config.compression_size
            self.compress_k = Linear(size * D, D, bias=False)
            self.compress_v = Linear(size * D, D, bias=False)
            self.compress_position = nn.Parameter(torch.zeros(size, D))
            self.branch_gate = Linear(d, 3 * H, bias=False)

    def _qkv(self, x, ve, cos_sin):
        B, T, _ = x.shape
        H, Hk, D = self.n_head, self.n_kv_head, self.head_dim
        q = self.c_q(x).view(B, T, H, D)
        k = self.c_k(x).view(B, T, Hk, D)
        v = self.c_v(x).view(B, T, Hk, D)
        if ve is not None and self.ve_gate is not None:
            v = v + (3 * torch.sigmoid(self.ve_gate(x[..., :12]))).unsqueeze(-1) * ve.view_as(v)
        q, k = (norm(apply_rotary_emb(z, *cos_sin)) * 1.2 for z in (q, k))
        rep = H // Hk
        q, k, v = (z.transpose(1, 2) for z in (q, k, v))
        if rep > 1:
            k, v = k.repeat_interleave(rep, 1), v.repeat_interleave(rep, 1)
        return q, k, v

    def _index(self, x):
        c = self.config
        x = x.detach()  # the indexer learns only from its distillation loss
        B, T, _ = x.shape
        iq = self.index_q(x).reshape(B, T, c.index_heads, c.index_dim)
        ik = self.index_k(x).reshape(B, T, 1, c.index_dim)
        size = c.compression_size if self.kind == "qsa" else c.block_size if self.kind == "seer" else 1
        if size > 1:
            ik = pool_blocks(ik.transpose(1, 2), size).transpose(1, 2)
        if self.kind == "dsa":
            ik = self.index_norm(ik.float()).to(x.dtype)
        else:
            iq, ik = norm(iq), norm(ik)
        iq = partial_rope(iq, torch.arange(T, device=x.device), c.index_rope_dim)
        ik = partial_rope(ik, torch.arange(ik.shape[1], device=x.device) * size, c.index_rope_dim)
        w = self.index_weights(x).transpose(1, 2) if self.kind == "dsa" else None
        return iq.transpose(1, 2), ik.transpose(1, 2), w, size

    def _nsa_compress(self, k, v):
        """Compressed keys/values over blocks of `size` taken every `stride` tokens."""
        c = self.config
        size = c.compression_size
        stride = c.compression_stride or size
        B, H, T, D = k.shape
        if stride == size:
            # non-overlapping blocks: a padded reshape (the audited graph of the reference)
            n = (T + size - 1) // size
            kb = F.pad(k, (0, 0, 0, n * size - T)).reshape(B, H, n, size, D)
            vb = F.pad(v, (0, 0, 0, n * size - T)).reshape_as(kb)
        else:
            n = max(1, (T - size) // stride + 1) if T >= size else 1
            need = (n - 1) * stride + size
            kp, vp = F.pad(k, (0, 0, 0, max(0, need - T))), F.pad(v, (0, 0, 0, max(0, need - T)))
            kb = kp.unfold(2, size, stride).transpose(-1, -2)   # B,H,n,size,D
            vb = vp.unfold(2, size, stride).transpose(-1, -2)
        ck = self.compress_k((kb + self.compress_position.to(kb)).flatten(-2))
        cv = self.compress_v(vb.flatten(-2))
        ends = torch.arange(kb.shape[2], device=k.device) * stride + size - 1   # last token of each block
        return ck, cv, ends

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if kv_cache is not None:
            raise NotImplementedError("sparse mixers do not use a KV cache")
        c = self.config
        B, T, d = x.shape
        H = self.n_head
        q, k, v = self._qkv(x, ve, cos_sin)
        learned = self.kind in ("dsa", "qsa", "seer")
        burnin = learned and self.training and self.in_burnin
        if self.backend not in BACKENDS:
            raise ValueError(f"unknown sparse backend {self.backend!r}")
        kernel = self.backend == "kernel" and x.is_cuda
        if self.backend == "kernel" and self._blocks_supported(x):
            return self._forward_blocks(x, q, k, v)
        aux, outputs = [], []
        edges = teacher_edges = 0
        chunk = c.reference_chunk
        # Seer on the kernel backend: selection and distillation as below, attention in one
        # block-sparse pass over the collected block membership
        collect = self.backend == "kernel" and self.kind == "seer" and self.head_dim == 128 \
            and c.block_size % 64 == 0 and (x.dtype == torch.bfloat16 or not x.is_cuda)
        mems = []
        if learned:
            iq, ik, iw, size = self._index(x)
        else:
            size = c.compression_size if self.kind == "nsa" else c.block_size
        if self.kind == "moba":
            pooled = pool_blocks(k, size)
        if self.kind == "nsa":
            ck, cv, ends = self._nsa_compress(k, v)
            gates = self.branch_gate(x).sigmoid().view(B, T, H, 3)
        for start in range(0, T, chunk):
            stop = min(start + chunk, T)
            pos = torch.arange(start, stop, device=x.device)
            qq = q[:, :, start:stop]
            causal = torch.arange(T, device=x.device)[None, :] <= pos[:, None]
            if learned:
                sc = torch.einsum("bhqd,bhkd->bhqk", iq[:, :, start:stop], ik.expand(-1, c.index_heads, -1, -1)).relu()
                if iw is not None:
                    sc = sc * iw[:, :, start:stop, None] * (c.index_heads ** -.5)
                sc = sc.sum(1)
                if self.kind != "qsa":
                    sc = sc / c.index_dim ** .5
                complete = (torch.arange(ik.shape[2], device=x.device) + 1) * size - 1 <= pos[:, None]
                if self.kind == "dsa":
                    idx, valid = select_tokens(sc[:, None], causal[None, None], c.sparse_topk)
                elif self.kind == "qsa":
                    idx, valid = qsa_indices(sc[:, None], complete, pos, size, T, c.sparse_topk)
                else:
                    idx, valid = block_indices(sc[:, None], complete, pos, size, T,
                                               max(1, (c.sparse_topk + size - 1) // size))
                idx, valid = (a.expand(-1, H, -1, -1) for a in (idx, valid))
                if self.training:
                    with torch.no_grad():
                        domain = causal[None, None].expand(B, H, -1, -1)
                        if not burnin:
                            sel = torch.zeros_like(domain, dtype=torch.int32)
                            sel.scatter_add_(-1, idx, valid.to(torch.int32))
                            domain = sel > 0
                        from nexttransformer_b200.ops.sparse_teacher import head_mean_teacher, kernel_supported
                        if kernel_supported(qq, k):
                            # two-pass kernel: no [B, H, Q, T] scores; the domain is shared by the heads
                            teacher = head_mean_teacher(qq, k, None if burnin else domain[:, 0], start,
                                                        c.head_dim ** -.5)
                        else:
                            raw = torch.matmul(qq.float(), k.float().transpose(-2, -1)) * c.head_dim ** -.5
                            teacher = safe_softmax(raw, domain).mean(1)
                        student_dom = complete[None].expand(B, -1, -1)
                        if size > 1:
                            teacher = pool_teacher(teacher, size, ik.shape[2], self.kind)
                            if not burnin:
                                bd = F.pad(domain[:, 0], (0, ik.shape[2] * size - T)).reshape(B, stop - start, -1,
                                                                                             size).any(-1)
                                student_dom = student_dom & bd
                        elif not burnin:
                            student_dom = student_dom & domain[:, 0]
                        teacher = teacher * complete.to(teacher.dtype)
                        teacher = teacher / teacher.sum(-1, keepdim=True).clamp_min(1e-12)
                    student = safe_softmax(sc.float(), student_dom)
                    kl = (teacher * (teacher.clamp_min(1e-12).log() - student.clamp_min(1e-12).log())).sum(-1)
                    aux.append(kl.sum() / (B * T))
                    teacher_edges += B * H * (stop - start) * T
                if burnin:
                    idx = torch.arange(T, device=x.device)[None, None, None].expand(B, H, stop - start, -1)
                    valid = causal[None, None].expand_as(idx)
                if collect:
                    nsel = ik.shape[2]
                    cnt = torch.zeros(B, 1, stop - start, nsel, dtype=torch.int32, device=x.device)
                    cnt.scatter_add_(-1, (idx[:, :1] // size).clamp_max(nsel - 1), valid[:, :1].to(torch.int32))
                    mems.append(cnt > 0)
                    out = None
                else:
                    out = self._attend(qq, k, v, idx, valid, T, kernel)
            elif self.kind == "moba":
                sc = torch.matmul(qq, pooled.transpose(-2, -1))
                complete = (torch.arange(pooled.shape[2], device=x.device) + 1) * size - 1 <= pos[:, None]
                idx, valid = block_indices(sc, complete, pos, size, T, max(0, c.sparse_topk // size - 1))
                out = self._attend(qq, k, v, idx, valid, T, kernel)
            else:
                complete = ends[None, :] <= pos[:, None]
                sc = torch.matmul(qq, ck.transpose(-2, -1)) * c.head_dim ** -.5
                prob = safe_softmax(sc, complete[None, None])
                compressed = torch.matmul(prob, cv)
                if c.compression_stride:
                    # overlapping compression: pool block importance onto selection blocks of block_size
                    sel_size = c.block_size
                    imp = self._selection_importance(prob, ends, sel_size, T)
                    nsel = (T + sel_size - 1) // sel_size
                    sel_complete = (torch.arange(nsel, device=x.device) + 1) * sel_size - 1 <= pos[:, None]
                else:
                    # non-overlapping compression of the selection size: identity importance map
                    sel_size, imp, sel_complete = size, prob, complete
                idx, valid = block_indices(imp, sel_complete, pos, sel_size, T, max(1, c.sparse_topk // sel_size))
                local = (pos[:, None] - torch.arange(c.local_window, device=x.device)[None, :]).flip(-1)
                lv = (local >= 0)[None, None].expand(B, H, -1, -1)
                selected = self._attend(qq, k, v, idx, valid, T, kernel)
                local_out = self._attend(qq, k, v, local.clamp_min(0)[None, None].expand_as(lv), lv, T, kernel)
                g = gates[:, start:stop].transpose(1, 2)
                out = compressed * g[..., 0:1] + selected * g[..., 1:2] + local_out * g[..., 2:3]
                edges += int(lv.sum()) + B * H * (stop - start) * ck.shape[2]
            edges += int(valid.sum())
            outputs.append(out)
        if collect:
            y = self._collected_attention(x, q, k, v, mems, size, burnin).reshape(B, T, -1)
        else:
            y = torch.cat(outputs, 2).transpose(1, 2).reshape(B, T, -1)
        self.last_aux = sum(aux, x.new_zeros(())) * c.index_loss_weight
        self.last_stats = {"selected_edges": edges, "teacher_dense_score_edges": teacher_edges, "burnin": burnin,
                           "backend": self.backend}
        return self.c_proj(y)

    # ------------------------------------------------------------ block-sparse kernel path
    def _collected_attention(self, x, q, k, v, mems, size, dense):
        """Attention of every row over its collected blocks (all causal keys when `dense`): one pass of
        the block-sparse kernels (the causal kernel during burn-in), [B, T, H, D]."""
        from nexttransformer_b200.ops.sparse_attention import block_lists, block_sparse_attention
        B, H, T, D = q.shape
        rep = H // self.n_kv_head
        k_raw, v_raw = k[:, ::rep].transpose(1, 2), v[:, ::rep].transpose(1, 2)
        if dense:
            if x.is_cuda:
                from nexttransformer_b200.ops.attention import attention_bthd
                return attention_bthd(q.transpose(1, 2), k_raw, v_raw, -1)
            return F.scaled_dot_product_attention(q, k, v, is_causal=True).transpose(1, 2)
        blocks = torch.cat(mems, 2).repeat_interleave(size // 64, -1)[..., :(T + 63) // 64]
        lists, masks = block_lists(blocks)
        return block_sparse_attention(q.transpose(1, 2), k_raw, v_raw, lists, masks, D ** -.5)

    def _blocks_supported(self, x):
        """MoBA and NSA whose selection unit is a multiple of 64 keys run the block-sparse kernels."""
        c = self.config
        if self.kind not in ("moba", "nsa") or self.head_dim != 128:
            return False
        if x.is_cuda and x.dtype != torch.bfloat16:
            return False
        sel = c.block_size if (self.kind == "moba" or c.compression_stride) else c.compression_size
        return sel % 64 == 0

    def _forward_blocks(self, x, q, k, v, rows_per_pass=1024):
        """Same selection as the chunked reference path, computed for every row, then one pass of
        the block-sparse kernels (``ops.sparse_attention``) over the selected 64-key blocks."""
        from nexttransformer_b200.ops.attention import attention_bthd
        from nexttransformer_b200.ops.sparse_attention import block_lists, block_sparse_attention
        c = self.config
        B, T, d = x.shape
        H, Hk, D = self.n_head, self.n_kv_head, self.head_dim
        rep = H // Hk
        k_raw, v_raw = k[:, ::rep].transpose(1, 2), v[:, ::rep].transpose(1, 2)   # [B, T, Hk, D]
        dev = x.device
        mems, compressed, edges = [], [], 0
        if self.kind == "moba":
            size = c.block_size
            pooled = pool_blocks(k, size)
            topk = max(0, c.sparse_topk // size - 1)
        else:
            ck, cv, ends = self._nsa_compress(k, v)
            gates = self.branch_gate(x).sigmoid().view(B, T, H, 3)
            size = c.block_size if c.compression_stride else c.compression_size
            topk = max(1, c.sparse_topk // size)
        nsel = (T + size - 1) // size
        fused = False
        if self.kind == "nsa" and x.is_cuda:
            from nexttransformer_b200.ops.nsa_compress import nsa_compressed, supported
            qt, ckk, cvk = q.transpose(1, 2), ck[:, ::rep].transpose(1, 2), cv[:, ::rep].transpose(1, 2)
            if supported(qt, ckk) and nsel <= 256:
                # compressed attention, block importance and the top-k choice in two kernels: no
                # [B, H, T, Nc] scores, probabilities or importance in memory
                comp, mem = nsa_compressed(qt, ckk, cvk, c.compression_stride or c.compression_size,
                                           c.compression_size, size, topk, c.head_dim ** -.5)
                compressed, mems, fused = [comp.transpose(1, 2)], [mem], True
                pos = torch.arange(T, device=dev)
                edges += (int(mem.sum()) - B * H * T) * size + B * H * int(((pos % size) + 1).sum())
        for start in range(0, T if not fused else 0, rows_per_pass):
            stop = min(start + rows_per_pass, T)
            pos = torch.arange(start, stop, device=dev)
            qq = q[:, :, start:stop]
            if self.kind == "moba":
                sc = torch.matmul(qq, pooled.transpose(-2, -1))
            else:
                complete = ends[None, :] <= pos[:, None]
                sc = torch.matmul(qq, ck.transpose(-2, -1)) * c.head_dim ** -.5
                prob = safe_softmax(sc, complete[None, None])
                compressed.append(torch.matmul(prob, cv))
                sc = self._selection_importance(prob, ends, size, T) if c.compression_stride else prob
            full = (torch.arange(nsel, device=dev) + 1) * size - 1 <= pos[:, None]
            cur = pos // size
            eligible = full & (torch.arange(nsel, device=dev)[None, :] != cur[:, None])
            chosen, ok = select_tokens(sc, eligible[None, None], topk)
            mem = torch.zeros(*sc.shape[:3], nsel, dtype=torch.bool, device=dev).scatter_(-1, chosen, ok)
            mem.scatter_(-1, cur[None, None, :, None].expand(B, H, -1, 1), True)
            mems.append(mem)
            edges += int(ok.sum()) * size + B * H * int(((pos % size) + 1).sum())
        mem = torch.cat(mems, 2)                                             # [B, H, T, nsel]
        blocks = mem.repeat_interleave(size // 64, -1)[..., :(T + 63) // 64]
        lists, masks = block_lists(blocks)
        selected = block_sparse_attention(q.transpose(1, 2), k_raw, v_raw, lists, masks, D ** -.5)   # [B, T, H, D]
        if self.kind == "moba":
            y = selected
        else:
            if x.is_cuda:
                local = attention_bthd(q.transpose(1, 2), k_raw, v_raw, c.local_window - 1)
            else:
                pos = torch.arange(T, device=dev)
                win = (pos[None, :] <= pos[:, None]) & (pos[:, None] - pos[None, :] < c.local_window)
                local = F.scaled_dot_product_attention(q, k, v, attn_mask=win).transpose(1, 2)
            comp = torch.cat(compressed, 2).transpose(1, 2).to(selected.dtype)
            y = comp * gates[..., 0:1] + selected * gates[..., 1:2] + local * gates[..., 2:3]
            lw = torch.arange(T, device=dev).clamp_max(c.local_window - 1) + 1
            edges += B * H * int(lw.sum()) + B * H * T * ck.shape[2]
        y = y.reshape(B, T, -1)
        self.last_aux = x.new_zeros(())
        self.last_stats = {"selected_edges": edges, "teacher_dense_score_edges": 0, "burnin": False,
                           "backend": self.backend}
        return self.c_proj(y)

    @staticmethod
    def _selection_importance(prob, ends, sel_size, T):
        """Map compressed-block importance to selection blocks: a compressed block counts towards
        every selection block it overlaps (identity when both sizes and strides coincide)."""
        nsel = (T + sel_size - 1) // sel_size
        n = prob.shape[-1]
        size_c = int((ends[0] + 1).item()) if n else sel_size
        starts = ends - size_c + 1
        sb = torch.arange(nsel, device=prob.device)
        overlap = (starts[:, None] < (sb[None, :] + 1) * sel_size) & (ends[:, None] >= sb[None, :] * sel_size)
        return prob @ overlap.to(prob.dtype)

    def _attend(self, q, k, v, idx, valid, T, kernel):
        if kernel:
            from nexttransformer_b200.ops.sparse_attention import masked_attention
            return masked_attention(q, k, v, indices_to_mask(idx, valid, T))
        return indexed_attention(q, k, v, idx, valid)
