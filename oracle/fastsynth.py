"""Synthetic-checkpoint tensors for the oracle, through the C generator when it
is built (oracle/_build/libcsynth.so), else through the numpy one.

TEST INFRASTRUCTURE ONLY.
"""

from __future__ import annotations

import ctypes
import os

import numpy as np

from verdict_b200 import synth as _synth

_LIB = None


def _lib():
    global _LIB
    if _LIB is None:
        path = os.path.join(os.path.dirname(os.path.abspath(__file__)), "_build", "libcsynth.so")
        if not os.path.exists(path):
            try:
                from . import build
                build.build()
            except Exception:
                _LIB = False
                return None
        lib = ctypes.CDLL(path)
        lib.vd_oracle_gen_rows.argtypes = [ctypes.c_void_p, ctypes.c_uint64, ctypes.c_int64, ctypes.c_void_p,
                                           ctypes.c_int64, ctypes.c_float, ctypes.c_float]
        lib.vd_oracle_gen_rows.restype = None
        _LIB = lib
    return _LIB or None


def gen_tensor(seed: int, name: str, shape, scale: float, offset: float = 0.0, rows=None) -> np.ndarray:
    lib = _lib()
    shape = tuple(int(s) for s in shape)
    if lib is None:
        return _synth.gen_tensor(seed, name, shape, scale, offset, rows=rows)
    base = _synth.tensor_base(seed, name)
    cols = shape[-1] if len(shape) > 1 else 1
    if rows is None:
        n_rows = int(np.prod(shape)) // cols
        out = np.empty(n_rows * cols, dtype=np.float32)
        lib.vd_oracle_gen_rows(out.ctypes.data, base, n_rows, None, cols, scale, offset)
        return out.reshape(shape)
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    out = np.empty((len(rows), cols), dtype=np.float32)
    lib.vd_oracle_gen_rows(out.ctypes.data, base, len(rows), rows.ctypes.data, cols, scale, offset)
    return out


class FastCheckpoint(_synth.SyntheticCheckpoint):
    """`SyntheticCheckpoint` whose tensors come from the C generator."""

    def get(self, name: str, rows=None) -> np.ndarray:
        shape, scale, off = self.table[name]
        return gen_tensor(self.spec["seed"], name, shape, scale, off, rows=rows)
