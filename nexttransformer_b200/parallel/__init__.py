"""Parallelism: data parallel (optimizer-owned gradient reduction; fused peer-memory reduce on
CUDA), expert parallel (all-to-all token dispatch for MoE) and tensor parallel (column/row
parallel linears with all-gather / reduce-scatter)."""
