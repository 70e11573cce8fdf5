"""Public model API: ``build_model``, ``load_model``, ``config_from_dict`` and the method registry."""
from nexttransformer_b200.models.registry import FAMILIES, FAMILY, METHODS

__all__ = ["FAMILIES", "FAMILY", "METHODS", "build_model", "config_from_dict", "load_model"]


def config_from_dict(raw):
    from nexttransformer_b200.models.config import config_from_dict as f
    return f(raw)


def build_model(config, device="cpu", seed=42):
    from nexttransformer_b200.models.lm import build_model as build
    return build(config, device, seed=seed)


def load_model(checkpoint, device="cpu"):
    """Load ``checkpoint_<step>/`` (formal format) strictly; returns (model, saved state)."""
    from pathlib import Path
    import torch
    from nexttransformer_b200.runtime.checkpoint import load_checkpoint
    checkpoint = Path(checkpoint)
    raw = torch.load(checkpoint / "model.pt", map_location="cpu", weights_only=False)["model_config"]
    model = build_model(config_from_dict(raw), device)
    saved = load_checkpoint(checkpoint, model)
    if hasattr(model, "set_step"):
        model.set_step(saved["state"]["step"])
    return model, saved
