"""evie_b200: B200 (sm_100a) kernels for the Qwen3.5 token-mixing hot path of the evie steering engine.

The product is ``libevie_cuda.so`` (C ABI in ``include/evie_cuda.h``); this package loads it with ctypes and
offers thin Python views of its entry points:
  * ``evie_b200.ops``   isolated ops on torch CUDA tensors (GDN decode step, GDN chunked prefill, paged GQA decode);
  * ``evie_b200.gpu``   ``GpuModel``, the mirror of evie-core's GPU backend (crates/evie-core/src/gpu/mod.rs);
  * ``evie_b200.checkpoint``  synthetic Qwen3.5 checkpoints.
There is no fallback: if the shared library is missing or fails to load, ``lib()`` raises.
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libevie_cuda.so")
_lib = None


class EvieError(RuntimeError):
    """A non-zero status from the C ABI, with the library's message."""

    def __init__(self, status: int, msg: str):
        super().__init__(f"evie status {status}: {msg}")
        self.status = status


def build(jobs: int = 8) -> str:
    """Compiles libevie_cuda.so for sm_100a (make in evie_b200/csrc). Returns the library path."""
    subprocess.run(["make", "-s", f"-j{jobs}", "-C", os.path.join(_HERE, "csrc")], check=True)
    return LIB_PATH


def lib() -> C.CDLL:
    """The loaded libevie_cuda.so. Raises if it is missing: there is no CPU or Python fallback."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"{LIB_PATH} is missing; build it with evie_b200.build()")
        _lib = C.CDLL(LIB_PATH)
        from . import capi

        capi.declare(_lib)
    return _lib


def check(status: int, ctx=None) -> None:
    if status != 0:
        L = lib()
        msg = (L.evie_last_error(ctx) if ctx else L.evie_last_global_error()) or b""
        raise EvieError(status, msg.decode(errors="replace"))
