"""Build the sm_100a extension in-tree: ``python setup.py build_ext --inplace``.

Produces ``oscar_b200/_C*.so``.  Every CUDA source is compiled for
``compute_100a``/``sm_100a`` only; there is no other architecture.
"""
import json
import os
import subprocess
from pathlib import Path

import torch
from setuptools import setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

ROOT = Path(__file__).parent
CSRC = ROOT / "csrc"

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_OPERATORS__", "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]

sources = ["csrc/bindings.cpp"] + sorted(str(p.relative_to(ROOT)) for p in CSRC.glob("*.cu"))

os.environ.setdefault("MAX_JOBS", str(os.cpu_count() or 4))


def _nvcc_version() -> str:
    try:
        out = subprocess.run(["nvcc", "--version"], capture_output=True, text=True).stdout
        return out.strip().splitlines()[-1]
    except OSError:
        return "unknown"


class Build(BuildExtension.with_options(use_ninja=True)):
    """Also records what the extension was built against (read by the runtime guard)."""

    def run(self):
        super().run()
        meta = {"torch": torch.__version__, "cuda": torch.version.cuda, "nvcc": _nvcc_version(),
                "nvcc_flags": NVCC_FLAGS, "sources": sources}
        (ROOT / "oscar_b200" / "_C_build.json").write_text(json.dumps(meta, indent=1))

setup(
    name="oscar_b200",
    version="0.1.0",
    packages=["oscar_b200"],
    ext_modules=[
        CUDAExtension(
            name="oscar_b200._C",
            sources=sources,
            include_dirs=[str(CSRC)],
            extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
        )
    ],
    cmdclass={"build_ext": Build},
)
