"""checks.linear on the GPU: the fused chunk kernels against the FP64 recurrence."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("kind", ["gdn", "kda", "deltanet"])
def test_fused_within_fla_tolerances(kind):
    from nexttransformer_b200.checks import linear as CL
    inp = CL.random_inputs(kind, 1, 320, 0, torch.device("cuda"))
    res = CL.check_one(inp, ["fused", "chunk_fp32"])
    assert res["ok"], res
