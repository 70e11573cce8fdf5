"""Native-track trainer, benchmark and preflight (``nexttransformer/native`` of the reference)."""
