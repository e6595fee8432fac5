"""In-tree build of the native extension for B200 (sm_100a).

The extension is compiled with ninja through ``torch.utils.cpp_extension``
into ``ops/_build/`` and the resulting shared object is copied next to this
file as ``_lmc_C.so`` so it ships with the source tree (no JIT cache, no
site-packages install).  ``python -m lmcache_ascend_b200.ops.build`` rebuilds.
"""

from __future__ import annotations

import glob
import os
import shutil
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
EXT_NAME = "_lmc_C"
SO_PATH = os.path.join(HERE, EXT_NAME + ".so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xptxas=-v" if os.environ.get("LMC_PTXAS_VERBOSE") else "-Xptxas=-O3",
]
CXX_FLAGS = ["-O3", "-std=c++17", "-fPIC"]


def sources() -> list[str]:
    return sorted(
        glob.glob(os.path.join(CSRC, "*.cu")) + glob.glob(os.path.join(CSRC, "*.cpp"))
    )


def build(verbose: bool = False) -> str:
    from torch.utils import cpp_extension

    os.makedirs(BUILD_DIR, exist_ok=True)
    os.environ.setdefault("MAX_JOBS", str(max(1, os.cpu_count() or 1)))
    cpp_extension.load(
        name=EXT_NAME,
        sources=sources(),
        extra_cflags=CXX_FLAGS,
        extra_cuda_cflags=NVCC_FLAGS,
        extra_include_paths=[CSRC],
        extra_ldflags=["-lrt"],
        build_directory=BUILD_DIR,
        with_cuda=True,
        is_python_module=True,
        verbose=verbose,
    )
    built = os.path.join(BUILD_DIR, EXT_NAME + ".so")
    tmp = SO_PATH + ".tmp"
    shutil.copyfile(built, tmp)
    os.replace(tmp, SO_PATH)
    return SO_PATH


if __name__ == "__main__":
    path = build(verbose="-v" in sys.argv)
    print(path)
