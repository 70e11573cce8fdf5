"""Small plain-PyTorch reference blocks of the 2K scaling expert families
(``nexttransformer/scaling/reference_blocks.py`` of the reference).

``RoutedFFN`` is the oracle of the routed feed-forward: one always-on shared ReLU^2 expert plus a
top-k mixture of routed ReLU^2 experts whose weights are the softmax of the selected router
logits, computed expert by expert with ``index_add``.  ``shared_expert_rule`` is the rule the three
expert families share (layer 0 dense, every later layer routed), as a factory keyed on the layer's
position in the whole stack.  ``KdaDsaGroup`` is the Hybrid family's four-layer group: three KDA
mixers and one DSA mixer (this package's ``LinearMixer`` / ``SparseMixer``), each followed by the
FFN the rule gives.  ``python -m nexttransformer_b200.scaling.reference_blocks`` runs them once on
CPU.  The sm_100a production path of the routed layer is ``models.moe.MoEFFN``.
"""
import torch
from torch import nn

from nexttransformer_b200.models.moe import ExpertMLP
from nexttransformer_b200.models.shell import Linear, norm


class RoutedFFN(nn.Module):
    def __init__(self, config, num_experts, top_k, expert_width):
        super().__init__()
        if not 1 <= top_k <= num_experts:
            raise ValueError("top_k must be between one and num_experts")
        if expert_width <= 0:
            raise ValueError("expert_width must be positive")
        self.top_k = top_k
        self.router = Linear(config.width, num_experts, bias=False)
        self.shared = ExpertMLP(config.width, expert_width)
        self.experts = nn.ModuleList(ExpertMLP(config.width, expert_width) for _ in range(num_experts))

    def forward(self, hidden):
        rows = hidden.reshape(-1, hidden.shape[-1])
        top, chosen = self.router(rows.float()).topk(self.top_k)
        weights = top.softmax(-1)
        out = self.shared(rows)
        for e, expert in enumerate(self.experts):
            token, slot = torch.nonzero(chosen == e, as_tuple=True)
            if token.numel():
                out = out.index_add(0, token, expert(rows[token]) * weights[token, slot, None].to(rows.dtype))
        return out.reshape(hidden.shape)


def shared_expert_rule(config, num_experts, top_k, expert_width):
    """Factory of the feed-forward of whole-stack layer `layer`: dense at 0, routed after."""
    def build(layer):
        return ExpertMLP(config.width, config.mlp_width) if layer == 0 else \
            RoutedFFN(config, num_experts, top_k, expert_width)
    return build


class KdaDsaGroup(nn.Module):
    def __init__(self, config, ffn=None, first_layer=0):
        from nexttransformer_b200.models.linear import LinearMixer
        from nexttransformer_b200.models.sparse import SparseMixer
        super().__init__()
        self.mixers = nn.ModuleList([LinearMixer(config, i, kind="kda") for i in range(3)]
                                    + [SparseMixer(config, 3, kind="dsa")])
        for m in self.mixers:
            m.ve_gate = None
        build = ffn or (lambda layer: ExpertMLP(config.width, config.mlp_width))
        self.ffns = nn.ModuleList(build(first_layer + i) for i in range(len(self.mixers)))
        self.burnin_steps = config.burnin_steps

    def forward(self, hidden, cos_sin, step):
        sparse = self.mixers[-1]
        sparse.in_burnin = step < self.burnin_steps
        for mixer, ffn in zip(self.mixers, self.ffns):
            hidden = hidden + mixer(norm(hidden), None, cos_sin, (-1, 0), None)
            hidden = hidden + ffn(norm(hidden))
        return hidden, sparse.last_aux


def rotary(config):
    freq = 10000 ** (-torch.arange(0, config.head_dim, 2) / config.head_dim)
    angle = torch.arange(config.sequence_len)[:, None] * freq
    return angle.cos()[None, :, None], angle.sin()[None, :, None]


def main():
    from nexttransformer_b200.models import build_model
    from nexttransformer_b200.models.config import debug_config
    torch.manual_seed(42)
    for method in ("mha_no_ve", "fixed_recursive"):
        config = debug_config(method)
        model = build_model(config, "cpu", seed=42)
        tokens = torch.randint(config.vocab_size, (2, config.sequence_len + 1))
        loss = model(tokens[:, :-1], tokens[:, 1:])
        loss.backward()
        if not torch.isfinite(loss):
            raise RuntimeError(f"non-finite loss: {method}")
        print(f"{method}: forward and backward complete")
    config = debug_config("dsa")
    hidden = torch.randn(2, config.sequence_len, config.width)
    rule = shared_expert_rule(config, num_experts=8, top_k=2, expert_width=config.width // 4)
    RoutedFFN(config, 8, 2, config.width // 4)(hidden).square().mean().backward()
    print("MoE: shared and selected experts, forward and backward complete")
    group = KdaDsaGroup(config, rule)
    for step in (0, config.burnin_steps):
        group.zero_grad(set_to_none=True)
        out, aux = group(hidden, rotary(config), step)
        loss = out.square().mean() + aux
        loss.backward()
        if not torch.isfinite(loss):
            raise RuntimeError("non-finite reference loss")
        print(f"KDA-DSA: step {step}, forward and backward complete")


if __name__ == "__main__":
    main()
