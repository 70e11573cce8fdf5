"""The shipped scaling configurations against the published figures of the reference's scaling
stage (configuration hashes of its result records, parameter counts, plans) and the value-embedding
switch's effect on parameters and cost."""
from dataclasses import replace
import json
from pathlib import Path

import pytest
import torch

from nexttransformer_b200.models.native.model import NativeExperiment, theoretical_training_flops
from nexttransformer_b200.scaling.config import config_hash, load_config
from nexttransformer_b200.scaling.optimizer import muon_weight_decay, scaling_params

ROOT = Path(__file__).resolve().parents[1]
# configSha256 of the reference's published scaling records
PUBLISHED = {"dense_200b": "dfee038378fd506b013da20cc1a4c8ea21d5b90104c3890a1e2e7f56b24fe3bb",
             "t3_dense_l20": "0eaafb4e317e2b7ca8bc21b41232ec95d7e63afb2f8e17351b0d79874952e000",
             "t3_dense_l28": "07dff102cab40e9e74d9f1be642e4cfea186b01bdf8cc88c5d9a9a50ff88ef45"}


def test_dense_200b_plan(capsys):
    from nexttransformer_b200.scaling import train
    mc, tc = load_config(ROOT / "configs/scaling/dense_200b.json")
    assert (tc.steps, tc.accumulation(mc, 32, 2), tc.batch_scale) == (95367, 8, 2.0)
    assert tc.core_steps() == [20000, 40000, 60000, 80000, 95367] and len(tc.validation_steps()) == 97
    assert tc.is_milestone(95367) and config_hash(mc, tc) == PUBLISHED["dense_200b"]
    with torch.device("meta"):
        model = NativeExperiment(mc)
    d, layers, t = mc.width, mc.dense_layers, mc.sequence_len
    assert sum(p.numel() for p in model.transformer.h.parameters()) == 12 * d * d * layers + 20 * 12 * mc.heads
    assert scaling_params(model) == 3_229_618_880
    assert muon_weight_decay(model, tc) == pytest.approx(0.28 * 2 * 110100912 / 3_229_618_880)
    assert theoretical_training_flops(mc) == pytest.approx(72 * d * d * layers + 12 * t * d * layers
                                                           + 6 * d * mc.vocab_size, rel=1e-5)
    train.main(["--config", str(ROOT / "configs/scaling/dense_200b.json"), "--dry-run"])
    plan = json.loads(capsys.readouterr().out)
    assert (plan["steps"], plan["accumulation"], plan["muon_lr"]) == (95367, 8, .04)


@pytest.mark.parametrize("cell_id, name, parameters, expected", [
    ("dense-T3-L20", "t3_dense_l20", 477_102_146, (29433, 32, [20000, 29433])),
    ("dense-T3-L28", "t3_dense_l28", 1_196_425_298, (11833, 32, [11833])),
])
def test_t3_dense_cells_match_the_manifest(capsys, cell_id, name, parameters, expected):
    from nexttransformer_b200.scaling import train
    cell = next(c for c in json.loads((ROOT / "configs/scaling/t3.json").read_text())["cells"] if c["id"] == cell_id)
    mc, tc = load_config(ROOT / f"configs/scaling/{name}.json")
    assert (mc.dense_layers, mc.width, mc.heads, mc.mlp_width) == (cell["layers"], cell["width"], cell["heads"],
                                                                   cell["ffnWidth"])
    assert (tc.steps, tc.total_tokens) == (cell["estimatedUpdates"], cell["estimatedTokens"])
    assert not mc.value_embeddings and config_hash(mc, tc) == PUBLISHED[name]
    with torch.device("meta"):
        model = NativeExperiment(mc)
    assert sum(p.numel() for p in model.parameters()) == parameters
    assert abs(theoretical_training_flops(mc) * tc.total_tokens - 1e20) < .01e20
    train.main(["--config", str(ROOT / f"configs/scaling/{name}.json"), "--dry-run", "--world-size", "8"])
    plan = json.loads(capsys.readouterr().out)
    assert (plan["steps"], plan["accumulation"], plan["core_steps"]) == expected


def test_value_embedding_switch_removes_tables_gates_and_their_cost():
    mc, _ = load_config(ROOT / "configs/scaling/dense_200b.json")
    off = replace(mc, value_embeddings=False)
    with torch.device("meta"):
        kept, dropped = NativeExperiment(mc), NativeExperiment(off)
    assert len(kept.value_embeds) == 20 and not dropped.value_embeds
    assert all(b.attn.ve_gate is None for b in dropped.transformer.h)
    tables = 20 * kept.transformer.wte.weight.shape[0] * mc.width
    assert sum(p.numel() for p in kept.parameters()) - sum(p.numel() for p in dropped.parameters()) == \
        tables + 20 * 12 * mc.heads
    assert theoretical_training_flops(mc) - theoretical_training_flops(off) == 3 * 20 * 24 * mc.heads
