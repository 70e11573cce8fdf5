"""Bounded verification tools (``python -m nexttransformer_b200.checks.<name>``): a synchronized
multi-rank update per method (``distributed``), per-method forward/backward and causality checks
(``validate``), bitwise CPU digests between two git trees (``golden``), kernel numerics and timing
against PyTorch references (``kernels``), a secret/path scanner (``public``) and a change classifier
(``changes``)."""
