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

# Streaming GEMV modes (csrc/sgemv.cu)
SG_STORE, SG_RESID, SG_SILU, SG_F32, SG_EXPERT, SG_MOEDOWN, SG_ROUTER, SG_ARGMAX = range(8)


def sgemv(mode, W, x, y=None, *, err, resid=None, norm=None, eps=0.0, ids=None, wts=None, J=0, scratch=None,
          counter=None, out_ids=None, out_wts=None, E=0, topk=0, shared=False, norm_topk=False, tok=None,
          slots=None, pos=None, out_tokens=None, step=None, pdl=True):
    """Streaming decode GEMV (see csrc/sgemv.cu for the modes)."""
    _load().sgemv(mode, W, x, y, resid, norm, eps, ids, wts, J, scratch, counter, out_ids, out_wts, E, topk,
                  shared, norm_topk, tok, slots, pos, out_tokens, step, err, pdl)


def sgemv_fits(mode: int, K: int, B: int, J: int = 1) -> bool:
    """Whether sgemv's shared-memory ring (200 KB) holds the activations plus two stages."""
    segs = J if mode == SG_MOEDOWN else 1
    rb_min = 2 if mode in (SG_SILU, SG_EXPERT) else 1
    x_bytes = (B * J if mode == SG_MOEDOWN else B) * K * 2
    return x_bytes + 2 * rb_min * segs * K * 2 <= 200 * 1024
