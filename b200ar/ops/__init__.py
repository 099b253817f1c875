"""Fused tensor-parallel and model ops (hand-written sm_100a kernels)."""
