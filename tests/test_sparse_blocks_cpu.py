"""The block-list path of the sparse mixers against their gathered-key reference path (CPU, fp32).

On CPU the block-sparse attention runs its fp32 oracle and the NSA sliding branch a masked
attention, so this checks the selection, the block lists / row masks and the branch assembly that
the sm_100a kernels consume."""
from dataclasses import replace

import pytest
import torch


def _cos_sin(T, D):
    f = torch.outer(torch.arange(T, dtype=torch.float32), 1.0 / (100000 ** (torch.arange(0, D, 2).float() / D)))
    return f.cos()[None, :, None, :], f.sin()[None, :, None, :]


@pytest.mark.parametrize("kind", ["moba", "nsa"])
def test_block_path_matches_reference(kind):
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.sparse import SparseMixer
    T = 320
    c = debug_config(kind, width=256, sequence_len=T)
    extra = dict(block_size=128, sparse_topk=256) if kind == "moba" else \
        dict(compression_size=64, compression_stride=0, block_size=64, sparse_topk=128, local_window=96)
    c = replace(c, heads=2, **extra)
    torch.manual_seed(0)
    mix = SparseMixer(c, 1)
    x = torch.randn(2, T, 256)
    cs = _cos_sin(T, 128)
    outs = []
    for backend in ("reference", "kernel"):
        mix.backend = backend
        outs.append(mix(x, None, cs, None))
    torch.testing.assert_close(outs[1], outs[0], atol=2e-5, rtol=1e-4)


def test_block_lists_visibility_roundtrip():
    from nexttransformer_b200.ops.sparse_attention import block_lists, visibility
    torch.manual_seed(1)
    T, NB = 300, 5
    blocks = torch.rand(2, 3, T, NB) > 0.5
    lists, masks = block_lists(blocks)
    vis = visibility(lists, masks, T)
    pos = torch.arange(T)
    want = blocks.repeat_interleave(64, -1)[..., :T] & (pos[None, :] <= pos[:, None])
    assert torch.equal(vis, want)


@pytest.mark.parametrize("burnin", [False, True])
def test_seer_block_path_matches_reference(burnin):
    """Seer (learned 64-key block selection): the collected block pass against the gathered-key path,
    aux (distillation) loss included."""
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.sparse import SparseMixer
    T = 256
    c = replace(debug_config("seer", width=256, sequence_len=T), heads=2, block_size=64, sparse_topk=128)
    torch.manual_seed(2)
    mix = SparseMixer(c, 1)
    mix.train()
    mix.in_burnin = burnin
    x = torch.randn(2, T, 256)
    cs = _cos_sin(T, 128)
    outs, auxs = [], []
    for backend in ("reference", "kernel"):
        mix.backend = backend
        outs.append(mix(x, None, cs, None))
        auxs.append(mix.last_aux)
    torch.testing.assert_close(outs[1], outs[0], atol=2e-5, rtol=1e-4)
    torch.testing.assert_close(auxs[1], auxs[0])
