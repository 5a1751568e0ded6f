"""Benchmarks: kernels, optimizer step, distributed orthogonalisation (see run.py)."""
