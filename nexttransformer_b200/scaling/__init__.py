"""Scaling-stage pretraining: the native dense backbone on nodes that share no filesystem."""
