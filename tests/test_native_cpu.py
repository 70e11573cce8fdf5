"""Native track (SSSL Dense, MoR, LoopFormer, Circle) against the reference on CPU.

Same weights in both implementations: the loss dictionaries, the FLOP statistics and every
parameter gradient must agree; the reference's native configuration files load unchanged and give
the same theoretical training FLOPs per token.
"""
from pathlib import Path

import pytest
import torch

from nexttransformer_b200.models.native import model as native
from nexttransformer_b200.models.native.config import NativeModelConfig, load_config

SMALL = dict(width=48, heads=2, mlp_width=192, vocab_size=96, sequence_len=16, dense_layers=4, pre_layers=1,
             core_layers=2, post_layers=1, fourier_dim=8, window_pattern="SL")


def _cfg(arch, **extra):
    kw = dict(SMALL, architecture=arch, **extra)
    if arch == "circle":
        kw.update(circle_max_steps=6, circle_target_steps=4.0, circle_random_warmup=2, circle_route_transition=4)
    return kw


@pytest.fixture(scope="module")
def ref_native(reference):
    import nexttransformer.models.native.config as rc
    import nexttransformer.models.native.model as rm
    return rc, rm


@pytest.mark.parametrize("arch,step", [("dense", 0), ("mor", 0), ("loopformer", 0), ("circle", 0), ("circle", 3),
                                       ("circle", 100)])
def test_native_matches_reference(ref_native, arch, step):
    rc, rm = ref_native
    kw = _cfg(arch)
    mine = native.build_model(NativeModelConfig(**kw), "cpu", seed=3)
    torch.manual_seed(3)
    ref = rm.build_model(rc.NativeModelConfig(**kw), "cpu")
    ms, rs = mine.state_dict(), ref.state_dict()
    assert {k: tuple(v.shape) for k, v in ms.items()} == {k: tuple(v.shape) for k, v in rs.items()}
    ref.load_state_dict(ms)
    for m in (mine, ref):
        m.train()
        if arch == "circle":
            m.set_circle_step(step)
    g = torch.Generator().manual_seed(7)
    tok = torch.randint(0, kw["vocab_size"], (3, kw["sequence_len"] + 1), generator=g)
    x, y = tok[:, :-1], tok[:, 1:]
    om, orf = mine(x, y), ref(x, y)
    for key in orf:
        assert torch.allclose(om[key], orf[key], rtol=1e-5, atol=1e-6), key
    for key in ("forward_flops", "active_tokens", "active_depth_sum"):
        if key in ref.last_stats:
            assert mine.last_stats[key] == ref.last_stats[key], key
    om["loss"].backward()
    orf["loss"].backward()
    grads = dict(mine.named_parameters())
    for name, p in ref.named_parameters():
        if p.grad is None:
            assert grads[name].grad is None or not grads[name].grad.any(), name
        else:
            assert torch.allclose(grads[name].grad, p.grad, rtol=1e-4, atol=1e-6), name


@pytest.mark.parametrize("name", ["dense", "mor", "loopformer", "circle"])
def test_native_config_files_and_flops(reference, name):
    """The shipped native configurations load in both trees with equal theoretical FLOPs per token."""
    import nexttransformer.models.native.config as rc
    import nexttransformer.models.native.model as rm
    src = Path(__file__).resolve().parents[1] / "configs" / "native" / f"{name}.json"
    mc, tc = load_config(src)
    rmc, rtc = rc.load_config(src)
    assert native.theoretical_training_flops(mc) == rm.theoretical_training_flops(rmc)
    assert tc.steps == rtc.steps and tc.validation_steps() == rtc.validation_steps()
    assert tc.core_steps() == rtc.core_steps()


def test_budget_updates_and_depth_law():
    from nexttransformer_b200.models.native.depth import depth_reference
    probs, surv = depth_reference(9, 27, 17.5)
    assert abs(sum(probs) - 1) < 1e-12
    assert abs(sum(d * p for d, p in zip(range(9, 28), probs)) - 17.5) < 1e-9
    assert abs(sum(surv) - 17.5) < 1e-9
    c = NativeModelConfig(**_cfg("mor"))
    m = native.build_model(c, "cpu", seed=0)
    m.train()
    out = m.update_route_budget([100, 70, 20], 100, 0)
    assert out["budget_updates"] == 1
    with pytest.raises(ValueError):
        m.update_route_budget([100, 70, 20], 100, 0)


@pytest.mark.parametrize("arch", ["mor", "circle"])
def test_counted_native_evaluation(tmp_path, arch):
    """Counted BPB reads exactly its token budget and reports route accounting; CORE through the
    counted model scores every example."""
    pa = pytest.importorskip("pyarrow")
    import pyarrow.parquet as pq
    from nexttransformer_b200.evaluation.native import evaluate_native_bpb, evaluate_native_core
    from nexttransformer_b200.runtime.tokenizer import BPETokenizer
    words = ["alpha", "beta", "gamma", "delta", "epsilon", "zeta"]
    docs = [" ".join(words[(i + j) % 6] for j in range(3 + i % 11)) for i in range(300)]
    for k, name in enumerate(("shard_00000.parquet", "shard_06542.parquet")):
        pq.write_table(pa.table({"text": docs[k * 150:(k + 1) * 150]}), tmp_path / name, row_group_size=25)
    tok = BPETokenizer.train_from_iterator(docs, vocab_size=300)
    c = NativeModelConfig(**_cfg(arch, vocab_size=320))
    m = native.build_model(c, "cpu", seed=1)
    res = evaluate_native_bpb(m, tok, tmp_path, tokens=4 * c.sequence_len, batch=2, rank=0, world=1,
                              device=torch.device("cpu"))
    assert res["input_tokens"] == 4 * c.sequence_len and res["val_bpb"] > 0
    assert len(res["active_ratios"]) == c.routing_steps and res["forward_flops_estimate"] > 0
    assert ("mean_ring_steps" in res) == (arch == "circle") and m.training
    with pytest.raises(ValueError):
        evaluate_native_bpb(m, tok, tmp_path, tokens=3 * c.sequence_len, batch=2, rank=0, world=1,
                            device=torch.device("cpu"))
    tasks = [{"label": "lm", "random_baseline": 0.0, "meta": {"task_type": "language_modeling", "num_fewshot": 0},
              "data": [{"context": "alpha beta", "continuation": " gamma"}] * 2}]
    core = evaluate_native_core(m, tok, tasks, torch.device("cpu"))
    assert core["full_core"] and core["entries"] == 1 and core["input_tokens"] > 0 and 0 <= core["core_metric"] <= 1
