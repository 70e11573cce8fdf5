"""Every built-in method against the reference implementation on CPU (fp32, same weights).

For each method: configurations serialise identically (so fingerprints and config files are
interchangeable), parameter names/shapes match, and loss + every parameter gradient agree.
"""
import pytest
import torch

from nexttransformer_b200.models.registry import METHODS

REFERENCE_METHODS = [m for m in METHODS if m != "moe"]


@pytest.fixture(scope="module")
def ref_api(reference):
    import nexttransformer.models.config as rc
    import nexttransformer.models.lm as rlm
    return rc, rlm


@pytest.mark.parametrize("method", REFERENCE_METHODS)
def test_method_matches_reference(ref_api, method):
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.lm import build_model
    rc, rlm = ref_api
    mine_cfg, ref_cfg = debug_config(method), rc.debug_config(method)
    assert mine_cfg.serialized() == ref_cfg.serialized()
    assert mine_cfg.fingerprint == ref_cfg.fingerprint
    mine = build_model(mine_cfg, "cpu", seed=5)
    ref = rlm.build_model(ref_cfg, "cpu", seed=5)
    ms, rs = mine.state_dict(), ref.state_dict()
    assert {k: tuple(v.shape) for k, v in ms.items()} == {k: tuple(v.shape) for k, v in rs.items()}
    ref.load_state_dict(ms)
    mine.train()
    ref.train()
    if method in ("dsa", "qsa", "seer") or "qsa" in method:
        mine.set_step(10_000)
        ref.set_step(10_000)
    g = torch.Generator().manual_seed(1)
    tok = torch.randint(0, mine_cfg.vocab_size, (2, mine_cfg.sequence_len + 1), generator=g)
    x, y = tok[:, :-1].contiguous(), tok[:, 1:].contiguous()
    lm, lr = mine(x, y), ref(x, y)
    assert torch.allclose(lm, lr, rtol=1e-5, atol=1e-6), (lm.item(), lr.item())
    lm.backward()
    lr.backward()
    mg = dict(mine.named_parameters())
    for name, p in ref.named_parameters():
        if p.grad is None:
            assert mg[name].grad is None or mg[name].grad.abs().max() == 0, name
            continue
        assert torch.allclose(mg[name].grad, p.grad, rtol=1e-4, atol=1e-6), name
