"""Sample from a checkpoint: ``python -m nexttransformer_b200.generate --checkpoint DIR --prompt TEXT``."""
import argparse
from pathlib import Path

import torch


def main(argv=None):
    p = argparse.ArgumentParser(description=__doc__)
    p.add_argument("--checkpoint", type=Path, required=True)
    p.add_argument("--tokenizer", type=Path, help="directory with tokenizer.pkl")
    p.add_argument("--prompt", default="")
    p.add_argument("--tokens", type=int, default=64)
    p.add_argument("--temperature", type=float, default=1.0)
    p.add_argument("--top-k", type=int, default=50)
    p.add_argument("--seed", type=int, default=42)
    p.add_argument("--no-cache", action="store_true")
    a = p.parse_args(argv)
    from nexttransformer_b200.inference import generate
    from nexttransformer_b200.models import load_model
    dev = "cuda" if torch.cuda.is_available() else "cpu"
    model, _ = load_model(a.checkpoint, dev)
    model.eval()
    if a.tokenizer:
        from nexttransformer_b200.runtime.tokenizer import BPETokenizer
        tok = BPETokenizer.from_directory(a.tokenizer)
        ids = tok.encode(a.prompt, prepend=tok.get_bos_token_id())
        out = list(generate(model, ids, a.tokens, a.temperature, a.top_k, a.seed, not a.no_cache))
        print(tok.decode(ids + out))
    else:
        ids = [int(t) for t in a.prompt.split()] or [0]
        print(" ".join(str(t) for t in generate(model, ids, a.tokens, a.temperature, a.top_k, a.seed,
                                                 not a.no_cache)))


if __name__ == "__main__":
    main()
