"""Native track: the historical d24 comparison of SSSL Dense, MoR, LoopFormer and Circle on the
nanochat shell (``nexttransformer/models/native`` of the reference)."""
