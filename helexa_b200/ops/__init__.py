"""Bindings to the sm_100a kernels in csrc/ (built in-tree as helexa_b200/_C*.so).

There is no fallback: on a CUDA device every op runs the native kernel, and
`ops.C` raises with the build command when the extension is missing.
"""
from __future__ import annotations

import importlib

_C = None


def _load():
    global _C
    if _C is None:
        import torch  # noqa: F401 - loads libc10/libtorch that the extension links against

        try:
            _C = importlib.import_module("helexa_b200._C")
        except ImportError as e:  # pragma: no cover - only without a build
            raise ImportError("helexa_b200._C is not built; run `python setup.py build_ext --inplace` "
                              f"(or __graft_entry__.build()): {e}") from e
    return _C


def __getattr__(name):
    if name == "C":
        return _load()
    raise AttributeError(name)


# GEMV epilogue modes (csrc/gemv.cu)
STORE_BF16, RESID_ADD, SILU_PAIR, STORE_F32 = 0, 1, 2, 3
