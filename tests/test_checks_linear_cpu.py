"""checks.linear: the fp32 chunk form against the FP64 recurrence, and mixer-input capture."""
import pytest
import torch

from nexttransformer_b200.checks import linear as CL


@pytest.mark.parametrize("kind", CL.KINDS)
def test_chunk_fp32_within_tolerance(kind, monkeypatch):
    monkeypatch.setattr(CL, "HEADS", 2)
    monkeypatch.setattr(CL, "DIM", 32)
    inp = CL.random_inputs(kind, 1, 150, 0, torch.device("cpu"))
    res = CL.check_one(inp, ["chunk_fp32"])
    errs = res["candidates"]["chunk_fp32"]["errors"]
    assert res["ok"], res
    assert set(errs) >= {"output", "dq", "dk", "dv", "dbeta"}
    assert ("dg" in errs) == (kind != "deltanet")
    assert (res["gates"] is None) == (kind == "deltanet")


def test_wrong_candidate_is_caught(monkeypatch):
    """A candidate with a deliberate error (beta dropped) must fail the tolerance."""
    monkeypatch.setattr(CL, "HEADS", 2)
    monkeypatch.setattr(CL, "DIM", 32)
    inp = CL.random_inputs("gdn", 1, 100, 1, torch.device("cpu"))
    good = CL._candidate_forward
    monkeypatch.setattr(CL, "_candidate_forward", lambda name, a: good(name, dict(a, beta=a["beta"] * 0.5)))
    assert not CL.check_one(inp, ["chunk_fp32"])["ok"]


@pytest.mark.parametrize("method", ["gdn", "kda"])
def test_capture_mixer_inputs(method):
    from dataclasses import replace
    from nexttransformer_b200.models.config import debug_config
    from nexttransformer_b200.models.lm import build_model
    cfg = replace(debug_config(method), backend="fla_chunk64")
    model = build_model(cfg, "cpu", seed=0).eval()
    idx = CL.checkpoint_row(model)
    got = CL.capture_mixer_inputs(model, idx)
    assert got and all(x["kind"] == method for x in got)
    assert got[0]["q"].dtype == torch.float64 and got[0]["q"].shape[1] == cfg.sequence_len
    res = CL.check_one(got[0], ["chunk_fp32"])
    assert res["ok"], res
