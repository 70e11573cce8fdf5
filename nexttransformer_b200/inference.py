"""Autoregressive decoding for the dense shell: a KV-cache engine and plain prefix re-run sampling.

``KVCache`` holds per-layer keys/values [B, T_max, Hk, D] and the position; ``decode`` runs the
shell block by block on the new tokens only (RoPE offset by the cache position, sliding windows
honoured, the smear gate reading the cached previous embedding).  Methods other than the dense
shell decode by re-running the full prefix, as the reference's ``generate`` does.
"""
import torch
import torch.nn.functional as F

from nexttransformer_b200.models.shell import Block, CausalSelfAttention, apply_rotary_emb, norm


class KVCache:
    def __init__(self, batch, max_len, n_layer, n_kv_head, head_dim, device, dtype):
        self.k = torch.zeros(n_layer, batch, max_len, n_kv_head, head_dim, device=device, dtype=dtype)
        self.v = torch.zeros_like(self.k)
        self.pos = 0
        self.prev_embedding = None


def supports_cache(model):
    return all(type(b) is Block and type(b.attn) is CausalSelfAttention for b in model.transformer.h)


@torch.no_grad()
def decode(model, idx, cache):
    """Logits of the last position after appending `idx` [B, t] to the cache."""
    B, t = idx.shape
    T0 = cache.pos
    cos, sin = model.cos[:, T0:T0 + t], model.sin[:, T0:T0 + t]
    x = norm(model.transformer.wte(idx).to(model.cos.dtype))
    prev = cache.prev_embedding
    cache.prev_embedding = x[:, -1:]
    gate_in = x
    if t > 1:
        g = model.smear_lambda.to(x.dtype) * torch.sigmoid(model.smear_gate(x[:, 1:, :24]))
        x = torch.cat((x[:, :1], x[:, 1:] + g * x[:, :-1]), 1)
    if prev is not None:
        g0 = model.smear_lambda.to(x.dtype) * torch.sigmoid(model.smear_gate(gate_in[:, :1, :24]))
        x = torch.cat((x[:, :1] + g0 * prev, x[:, 1:]), 1)
    x0 = x
    n = len(model.transformer.h)
    backout = None
    for i, blk in enumerate(model.transformer.h):
        x = model.resid_lambdas[i] * x + model.x0_lambdas[i] * x0
        a = blk.attn
        h = norm(x)
        ve = model.value_embeds[str(i)](idx).to(x.dtype) if str(i) in model.value_embeds else None
        q, k, v = a.project(h, ve, (cos, sin))
        cache.k[i, :, T0:T0 + t] = k
        cache.v[i, :, T0:T0 + t] = v
        K, V = cache.k[i, :, :T0 + t], cache.v[i, :, :T0 + t]
        w = model.window_sizes[i][0]
        qi = torch.arange(T0, T0 + t, device=idx.device)[:, None]
        kj = torch.arange(T0 + t, device=idx.device)[None, :]
        mask = (kj <= qi) & ((qi - kj) <= w if w >= 0 else torch.ones_like(kj, dtype=torch.bool))
        y = F.scaled_dot_product_attention(q.transpose(1, 2), K.transpose(1, 2), V.transpose(1, 2), attn_mask=mask,
                                           enable_gqa=K.shape[2] != q.shape[2])
        x = x + a.c_proj(y.transpose(1, 2).reshape(B, t, -1))
        x = x + blk.mlp(norm(x))
        if i == n // 2:
            backout = x
    cache.pos += t
    return model.readout(x[:, -1:], backout[:, -1:] if backout is not None else None)[:, -1]


@torch.no_grad()
def generate(model, tokens, max_tokens, temperature=1.0, top_k=None, seed=42, use_cache=True):
    """Yield sampled token ids after the prompt `tokens` (list of ints), batch 1."""
    dev = model.get_device()
    g = torch.Generator(device=dev).manual_seed(seed) if temperature > 0 else None
    ids = torch.tensor([tokens], dtype=torch.long, device=dev)
    cache = None
    if use_cache and supports_cache(model):
        cfg = model.shell
        cache = KVCache(1, len(tokens) + max_tokens, cfg.n_layer, cfg.n_kv_head, cfg.head_dim, dev, model.cos.dtype)
        logits = decode(model, ids, cache)
    for _ in range(max_tokens):
        if cache is None:
            logits = model(ids)[:, -1]
        logits = logits.float()
        if top_k:
            v, _ = torch.topk(logits, min(top_k, logits.size(-1)))
            logits[logits < v[:, [-1]]] = -float("inf")
        if temperature > 0:
            nxt = torch.multinomial(F.softmax(logits / temperature, -1), 1, generator=g)
        else:
            nxt = logits.argmax(-1, keepdim=True)
        ids = torch.cat((ids, nxt), 1)
        yield int(nxt.item())
        if cache is not None:
            logits = decode(model, nxt, cache)
