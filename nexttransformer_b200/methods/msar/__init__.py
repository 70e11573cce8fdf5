"""Multi-Stream Attention Residuals (MSAR, arXiv 2610.13630).

Sublayers are grouped in blocks of ``block_size_layers`` layers (2 sublayers each).  Every source of
the depth stream is kept as four temporal streams (``TemporalAugmentation``).  Sublayer 0 reads the
embedding directly; every later sublayer reads, through its ``DepthRead``, a softmax mixture over the
completed block sources plus the current block's running partial sum (merged by log-sum-exp).  After
each sublayer the block's raw output sum is re-augmented by that writer's own taps to form the new
partial source; a finished block's partial becomes a completed source.  The final MLP's output is
added to its input (no further read).  The shell's residual/x0 scalars and backout are unused.
Behaviour: ``nexttransformer/methods/msar/__init__.py:26-85`` of the reference.
"""
import torch
from torch import nn

from nexttransformer_b200.methods.msar.ops import (DepthRead, TemporalAugmentation, completed_read, merge_partial,
                                                  source_key)
from nexttransformer_b200.models.lm import LanguageModel
from nexttransformer_b200.models.shell import norm

frozen = ("resid_lambdas", "x0_lambdas", "backout_lambda")


def check(config):
    size = config.option("block_size_layers")
    if type(size) is not int or size < 1:
        raise ValueError("block_size_layers must be a positive integer")
    if config.window_pattern != "L":
        raise ValueError("MSAR keeps full causal attention in every layer")


class MSARModel(LanguageModel):
    def __init__(self, config):
        super().__init__(config)
        C, L = config.width, config.n_layer
        self.block_size_layers = config.option("block_size_layers")
        self.block_sizes = tuple(min(self.block_size_layers, L - s) for s in range(0, L, self.block_size_layers))
        self.residual_maps = nn.ModuleList(DepthRead(C) for _ in range(2 * L - 1))
        self.msar_initial = TemporalAugmentation(C)
        self.msar_writes = nn.ModuleList(TemporalAugmentation(C) for _ in range(2 * L - 1))

    def _ordinary_hidden(self, idx):
        last = 2 * self.config.n_layer - 1
        emb = self._embed(idx)
        first = self.msar_initial(emb)
        done, keys = [first], [source_key(first)]
        step = 0
        for layers in self.block_sizes:
            stop = step + 2 * layers
            lo = max(step, 1)
            queries = torch.stack([self.residual_maps[j - 1].query for j in range(lo, stop)])
            reads, lses = completed_read(queries, done, keys)
            reads, lses = reads.unbind(0), lses.unbind(0)
            raw = partial = None
            for j in range(step, stop):
                if j == 0:
                    h = emb
                else:
                    streams = reads[j - lo]
                    if partial is not None:
                        streams = merge_partial(streams, lses[j - lo], partial, source_key(partial),
                                                self.residual_maps[j - 1].query)
                    h = self.residual_maps[j - 1](streams)
                    self._record("depth_read", sublayer=j, sources=len(done) + int(partial is not None), streams=4,
                                 tokens=idx.numel())
                if j % 2 == 0:
                    out = self._attention_branch(h, idx, j // 2)
                else:
                    out = self.transformer.h[j // 2].mlp(norm(h))
                if j == last:
                    return h + out, None
                raw = out if raw is None else raw + out
                partial = self.msar_writes[j](raw)
            done.append(partial)
            keys.append(source_key(partial))
            step = stop
        raise RuntimeError("MSAR ended before its final MLP")


model = MSARModel


@torch.no_grad()
def init(model):
    model.msar_initial.reset_parameters()
    for t in model.msar_writes:
        t.reset_parameters()
