"""CORE context policy: scoring beyond the training context through a shallow model view."""
import pytest
import torch

from nexttransformer_b200.evaluation.context import (CORE_LENGTHS, LengthProbe, check_full_context, core_context,
                                                     inference_view, resume_core_limit, validate_submission)


def test_view_accepts_longer_inputs_and_keeps_prefix():
    from nexttransformer_b200.models import build_model
    from nexttransformer_b200.models.config import debug_config
    cfg = debug_config("dense")
    model = build_model(cfg, "cpu", seed=3).eval()
    T = cfg.sequence_len
    ids = torch.randint(0, cfg.vocab_size, (2, 2 * T))
    with pytest.raises(ValueError):
        model(ids)
    assert inference_view(model, T) is model
    view = inference_view(model, None)
    assert view is not model and view.config.sequence_len == model.cos.size(1)
    assert view.config.method == model.config.method
    probe = LengthProbe(view)
    with torch.no_grad():
        long = probe(ids)
        short = model(ids[:, :T])
    assert probe.longest == 2 * T
    # causal: the first T positions see the same keys through the same (training-length) windows
    torch.testing.assert_close(long[:, :T], short, rtol=1e-4, atol=1e-4)
    # the view shares the weights
    assert view.lm_head.weight.data_ptr() == model.lm_head.weight.data_ptr()


def test_policy_checks():
    from nexttransformer_b200.models.config import debug_config
    cfg = debug_config("dense")
    check_full_context(cfg, None)
    with pytest.raises(ValueError):
        check_full_context(cfg, CORE_LENGTHS["longestAnswerTokens"])
    ctx = core_context(2048, None, CORE_LENGTHS["maxPromptTokens"])
    validate_submission(ctx)
    with pytest.raises(ValueError):
        validate_submission(core_context(2048, None, 4000))
    validate_submission(core_context(2048, 4096, 4096))
    assert resume_core_limit({}, None, 2048) == 2048
    with pytest.raises(ValueError):
        resume_core_limit({"core_max_tokens": 2048}, 4096, 2048)
