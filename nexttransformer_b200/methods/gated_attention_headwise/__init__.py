"""Gated attention with one sigmoid gate per head (``granularity`` "headwise"); the module is
``nexttransformer_b200.methods.gated_attention``."""
from nexttransformer_b200.methods.gated_attention import GatedAttention, check, init, mixer  # noqa: F401
