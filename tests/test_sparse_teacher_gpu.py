"""Head-mean teacher kernels against the torch expression on fp32 scores."""
import pytest
import torch

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("B,H,Hk,Q,T,q_start,masked", [(2, 4, 4, 32, 256, 100, True), (1, 8, 2, 70, 300, 230, False),
                                                        (2, 2, 1, 128, 128, 0, True), (1, 4, 4, 33, 1000, 967, True)])
def test_teacher_matches_reference(B, H, Hk, Q, T, q_start, masked):
    from nexttransformer_b200.ops.sparse_teacher import _reference, head_mean_teacher
    g = torch.Generator(device="cuda").manual_seed(0)
    q = (torch.randn(B, H, Q, 128, device="cuda", generator=g) * 0.5).bfloat16()
    k = (torch.randn(B, Hk, T, 128, device="cuda", generator=g) * 0.5).bfloat16()
    mask = None
    if masked:
        mask = torch.rand(B, Q, T, device="cuda", generator=g) < 0.3
        mask[0, 3] = False   # an empty domain row gives zeros
    got = head_mean_teacher(q, k, mask, q_start, 128 ** -.5)
    ref = _reference(q, k, mask, q_start, 128 ** -.5)
    assert got.shape == (B, Q, T)
    torch.testing.assert_close(got, ref, rtol=2e-4, atol=2e-6)
    if masked:
        assert got[0, 3].abs().max() == 0
    rows = got.sum(-1)
    assert ((rows - 1).abs() < 1e-4).logical_or(rows == 0).all()


def test_teacher_on_strided_views():
    """The model passes q[:, :, start:stop] views of [B, H, T, D] tensors."""
    from nexttransformer_b200.ops.sparse_teacher import _reference, head_mean_teacher
    q_full = torch.randn(2, 4, 512, 128, device="cuda").bfloat16()
    k = torch.randn(2, 4, 512, 128, device="cuda").bfloat16()
    qq = q_full[:, :, 96:128]
    torch.testing.assert_close(head_mean_teacher(qq, k, None, 96, 0.1), _reference(qq, k, None, 96, 0.1),
                               rtol=2e-4, atol=2e-6)
