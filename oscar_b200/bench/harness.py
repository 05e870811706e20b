"""A/B timing helper with the reference's semantics (``delivery/benchmark_utils.py:9-45``):
the first call of each variant is timed separately (warm-up, JIT, allocator), the
variants then run in alternating order, each sample is device-timed with CUDA events
on the launching stream, the median of the warm samples is reported, and the outputs
must match (``rtol``) before any number is trusted.  Between samples a buffer larger
than L2 is written so that every timed call starts with a cold cache.
"""
from __future__ import annotations

import os

import statistics
from dataclasses import dataclass

import torch

L2_FLUSH_BYTES = 256 << 20  # > 126 MB L2 of a B200


@dataclass
class Timing:
    first_ms: float
    median_ms: float
    samples: list


_FLUSH: dict = {}


def flush_l2(device=None) -> None:
    dev = torch.device(device or "cuda")
    buf = _FLUSH.get(dev)
    if buf is None:
        buf = _FLUSH[dev] = torch.empty(L2_FLUSH_BYTES // 4, dtype=torch.float32, device=dev)
    buf.fill_(1.0)


def time_call(fn, flush: bool = True) -> float:
    if flush:
        flush_l2()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e)


def _rel(a: torch.Tensor, b: torch.Tensor) -> float:
    a, b = a.float(), b.float()
    return float((a - b).norm() / (b.norm() + 1e-30))


def compare_calls(variants: dict, iters: int = 10, rtol: float = 1e-2, flush: bool = True) -> dict[str, Timing]:
    """``variants = {name: fn}``; each ``fn()`` returns its output tensor."""
    names = list(variants)
    outs = {n: variants[n]() for n in names}  # numeric match first
    ref = outs[names[0]]
    for n in names[1:]:
        if ref is not None and outs[n] is not None:
            err = _rel(outs[n], ref)
            if err > rtol:
                raise AssertionError(f"{n} differs from {names[0]}: rel err {err:.3e} > {rtol}")
        if outs[n] is not None and ref is not None and outs[n].data_ptr() == ref.data_ptr():
            raise AssertionError(f"{n} and {names[0]} share one output buffer: the comparison would be vacuous")
    first = {n: time_call(variants[n], flush) for n in names}
    samples = {n: [] for n in names}
    for i in range(iters):
        order = names if i % 2 == 0 else names[::-1]
        for n in order:
            samples[n].append(time_call(variants[n], flush))
    return {n: Timing(first[n], statistics.median(samples[n]), samples[n]) for n in names}


# Roofline denominators: a STREAM-style copy and a burst cuBLAS bf16 GEMM measured on the
# B200s these benchmarks were developed on; override with OSCAR_PEAK_HBM_GBS /
# OSCAR_PEAK_BF16_TFLOPS for another machine.
def peak_hbm_gbs() -> float:
    return float(os.environ.get("OSCAR_PEAK_HBM_GBS", "6554.9"))


def peak_bf16_tflops() -> float:
    return float(os.environ.get("OSCAR_PEAK_BF16_TFLOPS", "1661.4"))
