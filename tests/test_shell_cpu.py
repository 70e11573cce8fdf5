"""CPU oracle tests of the shell: parity with the reference backbone, init and FLOPs."""
import torch

from nexttransformer_b200.models.shell import ShellConfig, build_shell


def _pair(reference, **kw):
    from nexttransformer.models.backbone import GPT, GPTConfig
    cfg = ShellConfig(**kw)
    mine = build_shell(cfg, "cpu", seed=3)
    with torch.device("meta"):
        ref = GPT(GPTConfig(**{k: v for k, v in kw.items() if k in GPTConfig.__dataclass_fields__}))
    ref.to_empty(device="cpu")
    ref.init_weights()
    ref.load_state_dict(mine.state_dict())
    return mine, ref


def test_shell_matches_reference_backbone(reference):
    mine, ref = _pair(reference, sequence_len=64, vocab_size=200, n_layer=4, n_head=4, n_kv_head=2, n_embd=128,
                      window_pattern="SSSL")
    assert set(mine.state_dict()) == set(ref.state_dict())
    idx = torch.randint(0, 200, (2, 64))
    tgt = torch.randint(0, 200, (2, 64))
    l1, l2 = mine(idx, tgt), ref(idx, tgt)
    l1.backward()
    l2.backward()
    assert torch.equal(l1, l2)
    mg = dict(mine.named_parameters())
    for n, p in ref.named_parameters():
        assert torch.equal(p.grad, mg[n].grad), n
    assert mine.estimate_flops() == ref.estimate_flops()


def test_window_sizes_and_init():
    cfg = ShellConfig(sequence_len=2048, vocab_size=32768, n_layer=6, n_head=4, n_kv_head=4, n_embd=256)
    with torch.device("meta"):
        from nexttransformer_b200.models.shell import GPTShell
        m = GPTShell(cfg)
    # ceil(T / 4 / 128) * 128 evaluated as the reference code does: 2048 -> 512
    assert [w for w, _ in m.window_sizes] == [512, 512, 512, 2048, 512, 2048]
    model = build_shell(ShellConfig(sequence_len=32, vocab_size=100, n_layer=3, n_head=2, n_kv_head=2, n_embd=64), "cpu",
                        seed=1)
    assert model.transformer.wte.weight.shape[0] == 128  # padded to 64
    assert torch.allclose(model.resid_lambdas.detach(), torch.tensor([1.15, 1.10, 1.05]))
    assert model.transformer.h[0].attn.c_proj.weight.abs().sum() == 0
    assert sorted(model.value_embeds) == ["0", "2"]
