"""Micro-benchmarks of the native kernels (run as ``python -m flare_b200.benchmarks.<name>``)."""
