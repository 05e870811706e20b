"""Benchmark harnesses: attention sweep, TP fused-collective microbench, A/B helper."""
