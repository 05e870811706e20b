"""Platform discovery dump and runtime guard.

``python -m oscar_b200.utils.platform`` prints one JSON document: interpreter and
library versions (torch, CUDA runtime, NCCL, driver), whether the in-tree sm_100a
extension loads and from where, every visible GPU (name, compute capability, SMs,
memory), NVLS multicast support, peer access between GPUs, and the ``OSCAR_*``
environment.  It mirrors the reference's ``tools/diag_platform.py:30-91`` (which
dumps the vLLM/Ascend plugin discovery state) for this stack.

:func:`check_runtime` is the version guard (``delivery/runtime_versions.py:8-21``):
the extension must have been built against the running torch, and every GPU must be
compute capability 10.0 (the kernels are compiled for sm_100a only).
"""
from __future__ import annotations

import json
import os
import platform as _pf
import subprocess
import sys


class RuntimeMismatch(RuntimeError):
    pass


def _driver_version() -> str | None:
    try:
        out = subprocess.run(["nvidia-smi", "--query-gpu=driver_version", "--format=csv,noheader"],
                             capture_output=True, text=True, timeout=20)
        return out.stdout.strip().splitlines()[0] if out.returncode == 0 and out.stdout.strip() else None
    except (OSError, subprocess.SubprocessError, IndexError):
        return None


def extension_info() -> dict:
    info = {"loaded": False}
    try:
        import importlib

        mod = importlib.import_module("oscar_b200._C")
        info.update(loaded=True, path=getattr(mod, "__file__", None),
                    entry_points=sorted(n for n in dir(mod) if not n.startswith("_")))
        meta = os.path.join(os.path.dirname(mod.__file__), "_C_build.json")
        if os.path.exists(meta):
            with open(meta) as f:
                info["build"] = json.load(f)
    except Exception as e:  # noqa: BLE001 - reported, not raised
        info["error"] = repr(e)
    return info


def collect() -> dict:
    import torch

    d: dict = {
        "python": sys.version.split()[0], "platform": _pf.platform(), "torch": torch.__version__,
        "cuda_runtime": torch.version.cuda, "cuda_available": torch.cuda.is_available(),
        "driver": _driver_version(), "extension": extension_info(),
        "env": {k: v for k, v in sorted(os.environ.items()) if k.startswith(("OSCAR_", "NCCL_", "CUDA_VISIBLE"))},
    }
    try:
        d["nccl"] = ".".join(map(str, torch.cuda.nccl.version()))
    except Exception:  # noqa: BLE001
        d["nccl"] = None
    gpus = []
    if torch.cuda.is_available():
        n = torch.cuda.device_count()
        try:
            import torch.distributed._symmetric_memory as symm
            mc = lambda i: bool(symm._SymmetricMemory.has_multicast_support(symm.DeviceType.CUDA, i))  # noqa: E731
        except Exception:  # noqa: BLE001
            mc = lambda i: None  # noqa: E731
        for i in range(n):
            p = torch.cuda.get_device_properties(i)
            gpus.append({"index": i, "name": p.name, "cc": f"{p.major}.{p.minor}", "sms": p.multi_processor_count,
                         "memory_gib": round(p.total_memory / 2**30, 1), "nvls_multicast": mc(i),
                         "peer_access": [j for j in range(n) if j != i and torch.cuda.can_device_access_peer(i, j)]})
    d["gpus"] = gpus
    return d


def check_runtime(info: dict | None = None) -> None:
    """Raise :class:`RuntimeMismatch` when the build and the machine disagree."""
    info = info or collect()
    ext = info["extension"]
    if not ext.get("loaded"):
        raise RuntimeMismatch(f"sm_100a extension not loadable: {ext.get('error')}")
    built = ext.get("build", {}).get("torch")
    if built and built.split("+")[0] != info["torch"].split("+")[0]:
        raise RuntimeMismatch(f"extension built against torch {built}, running {info['torch']}")
    bad = [g for g in info["gpus"] if g["cc"] != "10.0"]
    if bad:
        raise RuntimeMismatch(f"kernels are built for sm_100a only; found {[(g['index'], g['cc']) for g in bad]}")


def main() -> int:
    info = collect()
    print(json.dumps(info, indent=2))
    if info["gpus"]:
        try:
            check_runtime(info)
        except RuntimeMismatch as e:
            print(f"runtime check failed: {e}", file=sys.stderr)
            return 1
    return 0


if __name__ == "__main__":
    sys.exit(main())
