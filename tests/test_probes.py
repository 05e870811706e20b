"""Delivery probes: the CPU probes always, the kernel probes on a B200."""
import pytest

from oscar_b200.serve import probes as P


def test_cpu_probes():
    res = P.run(gpu=False)
    assert set(res) == set(P.CPU_PROBES)
    assert all(r["ok"] for r in res.values()), res


@pytest.mark.gpu
def test_gpu_probes():
    res = P.run(gpu=True)
    assert all(r["ok"] for r in res.values()), res
