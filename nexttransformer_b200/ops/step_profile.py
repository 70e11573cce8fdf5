"""One training update of a benchmark configuration, bracketed for a profiler (one GPU).

    python -m nexttransformer_b200.ops.step_profile METHOD [LAYERS] [MICRO]
    ncu --profile-from-start off --metrics gpu__time_duration.sum --clock-control none --csv \\
        python -m nexttransformer_b200.ops.step_profile METHOD LAYERS MICRO

METHOD is one of ``bench.py``'s method configurations (``gdn_hybrid_swa``, ``kda_hybrid``, ``nsa``,
``moba``, ``moe``) or ``dense`` (the headline shell, d20 by default) at LAYERS layers (default 4) and
one micro-batch of MICRO rows (default 8).  The
model is built with ``models.build_model``, its kernel state and a ``training.Trainer``; two updates
warm up, then one update runs between ``torch.cuda.profiler.start()`` and ``stop()``, so a capture
with ``--profile-from-start off`` holds exactly one update's launches.
"""
import sys
from dataclasses import replace
from pathlib import Path

import torch


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    method = argv[0]
    layers = int(argv[1]) if len(argv) > 1 else 4
    micro = int(argv[2]) if len(argv) > 2 else 8
    root = Path(__file__).resolve().parents[2]
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    import bench
    from nexttransformer_b200.models.config import candidate_config
    from nexttransformer_b200.models.lm import build_model
    from nexttransformer_b200.optim.groups import protocol_groups
    from nexttransformer_b200.optim.muon_adamw import MuonAdamW
    from nexttransformer_b200.training.engine import Trainer
    if method == "dense":
        from nexttransformer_b200.models.shell import ShellConfig, build_shell
        from nexttransformer_b200.optim.groups import shell_groups
        model = build_shell(ShellConfig(**dict(bench.MODEL, n_layer=layers)), "cuda", seed=42)
        state = model.fused_state()
        trainer = Trainer(model, MuonAdamW(shell_groups(model), shadows={p: s for p, s in state.casts}))
        vocab, seq = bench.MODEL["vocab_size"], bench.MODEL["sequence_len"]
    else:
        raw, _ = bench.METHOD_CONFIGS[method]
        fields = {k: v for k, v in raw.items() if k != "method"}
        fields.update(layers=layers)
        cfg = replace(candidate_config(raw["method"]), **fields)
        model = build_model(cfg, "cuda", seed=42)
        if raw["method"] in ("nsa", "moba"):
            model.set_sparse_backend("kernel")
        state = model.fused_state()
        trainer = Trainer(model, MuonAdamW(protocol_groups(model), shadows={p: s for p, s in state.casts}))
        vocab, seq = cfg.vocab_size, cfg.sequence_len
    x = torch.randint(0, vocab, (micro, seq), device="cuda")
    y = torch.randint(0, vocab, (micro, seq), device="cuda")
    for _ in range(2):
        trainer.step_device([x], [y])
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    trainer.step_device([x], [y])
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(f"profiled one update: {method}, {layers} layers, micro-batch {micro} x {seq}")


if __name__ == "__main__":
    main()
