"""Native ops of lmcache_ascend_b200 (sm_100a CUDA + C++ host runtime).

The compiled module ``_lmc_C.so`` lives in this directory (built in-tree by
``lmcache_ascend_b200.ops.build``).  On a machine with a GPU the native module
is mandatory: every op that receives CUDA tensors raises if it is missing
instead of falling back to PyTorch.  CPU tensors are served by the pure
PyTorch oracles in ``ops.reference`` (used by the CPU test tier and by
CPU-only deployments).
"""

from __future__ import annotations

import importlib.machinery
import importlib.util
import os
from typing import Optional

import torch

_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_lmc_C.so")
_mod = None
_err: Optional[BaseException] = None


def _load():
    global _mod, _err
    if _mod is not None or _err is not None:
        return _mod
    if not os.path.exists(_SO):
        _err = FileNotFoundError(
            f"native extension not built: {_SO} (run python -m lmcache_ascend_b200.ops.build)"
        )
        return None
    try:
        loader = importlib.machinery.ExtensionFileLoader("_lmc_C", _SO)
        spec = importlib.util.spec_from_file_location("_lmc_C", _SO, loader=loader)
        mod = importlib.util.module_from_spec(spec)
        loader.exec_module(mod)
        _mod = mod
    except Exception as e:  # pragma: no cover - depends on the build
        _err = e
    return _mod


def native_available() -> bool:
    return _load() is not None


def native():
    """The compiled module; raises (loudly) when it cannot be loaded."""
    mod = _load()
    if mod is None:
        raise RuntimeError(f"lmcache_ascend_b200 native ops unavailable: {_err}")
    return mod


def native_so_path() -> str:
    return _SO


def require_native_for(*tensors) -> None:
    """Raise if any tensor is on CUDA and the native module is missing."""
    for t in tensors:
        if isinstance(t, torch.Tensor) and t.is_cuda:
            native()
            return


class DeviceStatus:
    """Host view of the 24-byte device status word written by kernels.

    Layout matches ``lmc::DeviceStatus`` (code, where, a, b).
    """

    CODES = {
        0: "ok",
        1: "mbarrier_timeout",
        2: "flag_timeout",
        3: "bad_slot",
        4: "bad_alignment",
        5: "bad_index",
    }

    def __init__(self, device: torch.device):
        self.buf = torch.zeros(4, dtype=torch.int64, device=device)

    def reset(self) -> None:
        self.buf.zero_()

    @property
    def tensor(self) -> torch.Tensor:
        return self.buf

    def read(self) -> dict:
        v = self.buf.cpu()
        code = int(v[0].item() & 0xFFFFFFFF)
        where = int((v[0].item() >> 32) & 0xFFFFFFFF)
        return {
            "code": code,
            "name": self.CODES.get(code, f"unknown({code})"),
            "where": where,
            "a": int(v[1].item()),
            "b": int(v[2].item()),
        }

    def check(self, what: str = "kernel") -> None:
        st = self.read()
        if st["code"] != 0:
            raise RuntimeError(f"{what} reported device status {st}")
