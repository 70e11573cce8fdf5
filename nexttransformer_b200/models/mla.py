"""Multi-head latent attention (DeepSeek-V2 MLA; MLA-NoPE at formal scale).

Queries and keys/values go through low-rank latents normalised with the shell's RMSNorm and
are expanded per head; RoPE (when qk_rope_dim > 0) lives on separate query dimensions and one
key shared by all heads.  Keys and values are reconstructed explicitly and attended with the
shell's causal attention; softmax scale (nope + rope)^-1/2.  Parameter names follow the
reference (``nexttransformer/models/others.py``): c_q, q_up, c_k, c_v, c_proj.
"""
import torch
from torch import nn

from nexttransformer_b200.models import shell as shell_mod
from nexttransformer_b200.models.shell import Linear, apply_rotary_emb, norm


class MLAAttention(nn.Module):
    def __init__(self, config, layer_idx):
        super().__init__()
        self.layer_idx = layer_idx
        self.heads, self.nope, self.rope = config.heads, config.qk_nope_dim, config.qk_rope_dim
        self.v_dim, self.kv_rank = config.v_head_dim, config.kv_rank
        self.c_q = Linear(config.width, config.q_rank, bias=False)
        self.q_up = Linear(config.q_rank, self.heads * (self.nope + self.rope), bias=False)
        self.c_k = Linear(config.width, self.kv_rank + self.rope, bias=False)
        self.c_v = Linear(self.kv_rank, self.heads * (self.nope + self.v_dim), bias=False)
        self.c_proj = Linear(self.heads * self.v_dim, config.width, bias=False)
        self.ve_gate = None

    @torch.no_grad()
    def init_weights(self):
        for proj in (self.q_up, self.c_v):
            bound = 3 ** .5 * proj.weight.shape[1] ** -.5
            nn.init.uniform_(proj.weight, -bound, bound)

    def forward(self, x, ve, cos_sin, window_size, kv_cache=None):
        if ve is not None:
            raise ValueError("MLA has no value-embedding input")
        if kv_cache is not None:
            raise NotImplementedError("latent KV cache decoding is not part of training")
        B, T, _ = x.shape
        H = self.heads
        q = self.q_up(norm(self.c_q(x))).view(B, T, H, self.nope + self.rope)
        comp = self.c_k(x)
        latent = comp[..., :self.kv_rank]
        k_nope, v = self.c_v(norm(latent)).view(B, T, H, self.nope + self.v_dim).split((self.nope, self.v_dim), -1)
        if self.rope:
            cos, sin = cos_sin
            cos, sin = cos[..., :self.rope // 2], sin[..., :self.rope // 2]
            q = torch.cat((q[..., :self.nope], apply_rotary_emb(q[..., self.nope:], cos, sin)), -1)
            k_rope = apply_rotary_emb(comp[..., self.kv_rank:].view(B, T, 1, self.rope), cos, sin)
            k = torch.cat((k_nope, k_rope.expand(B, T, H, self.rope)), -1)
        else:
            k = k_nope
        y = shell_mod.sdpa(q, k, v, window_size[0])
        return self.c_proj(y.reshape(B, T, H * self.v_dim))
