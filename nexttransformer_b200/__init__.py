"""NextTransformer-B200: a Blackwell-native (sm_100a) architecture-research trainer.

Capabilities follow Interactive-Active-AI/NextTransformer (method zoo, frozen protocol,
FLOP ledger, Muon+AdamW, checkpoints, train/evaluate/generate CLIs); the compute path is
PyTorch plus hand-written sm_100a kernels in ``nexttransformer_b200/csrc``.
"""
__version__ = "0.1.0"
