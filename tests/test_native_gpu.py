"""Native track on CUDA: the compacted (MoR / Circle) blocks' full-window attention through the causal
kernel equals the explicit-mask attention of the same gathered rows."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("arch", ["mor", "circle"])
def test_compacted_attention_kernel_route(arch, monkeypatch):
    from nexttransformer_b200.models.native import model as native
    from nexttransformer_b200.models.native.config import NativeModelConfig
    kw = dict(width=256, heads=2, mlp_width=1024, vocab_size=96, sequence_len=256, dense_layers=4, pre_layers=1,
              core_layers=2, post_layers=1, fourier_dim=8, window_pattern="L", architecture=arch)
    if arch == "circle":
        kw.update(circle_max_steps=6, circle_target_steps=4.0, circle_random_warmup=2, circle_route_transition=4)
    g = torch.Generator(device="cuda").manual_seed(7)
    tok = torch.randint(0, kw["vocab_size"], (2, kw["sequence_len"] + 1), device="cuda", generator=g)
    x, y = tok[:, :-1], tok[:, 1:]
    out = []
    for route in (True, False):
        monkeypatch.setattr(native, "_causal_route", (lambda *a: a[0].is_cuda and a[1][0] >= a[2] - 1) if route
                            else (lambda *a: False))
        m = native.build_model(NativeModelConfig(**kw), "cuda", seed=3)
        m.train()
        if arch == "circle":
            m.set_circle_step(100)
        losses = m(x, y)
        losses["loss"].backward()
        out.append((losses["loss"].detach().float(), {n: p.grad.float().clone() for n, p in m.named_parameters()
                                                       if p.grad is not None}, m.last_stats.get("active_tokens")))
    (l1, g1, a1), (l2, g2, a2) = out
    assert a1 == a2  # same routing
    assert abs(l1.item() - l2.item()) <= 1e-2 * abs(l2.item()), (l1.item(), l2.item())
    for n in g2:
        if g2[n].norm() > 0:
            assert _rel(g1[n], g2[n]) < 5e-2, (n, _rel(g1[n], g2[n]))
