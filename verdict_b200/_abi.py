"""ctypes binding of `include/vdexec.h` (libvdexec.so, built in-tree).

This is the same binding a Rust `Engine` would declare with `extern "C"`; the
struct layouts below mirror the header field for field.  Loading fails loudly
when the library is missing: there is no fallback path.
"""

from __future__ import annotations

import ctypes
import os

from . import build as _build

VD_OK, VD_EINVAL, VD_ECUDA, VD_EDEAD, VD_ENOMEM, VD_ESPEC, VD_EDEVICE = 0, -1, -2, -3, -4, -5, -6
VD_MEM_HOST, VD_MEM_DEVICE = 0, 1
VDK_FP16, VDK_BF16 = 0, 1

_P = ctypes.c_void_p
_I64P = ctypes.POINTER(ctypes.c_int64)


class VdBatch(ctypes.Structure):
    _fields_ = [
        ("b", ctypes.c_int64), ("l", ctypes.c_int64), ("k", ctypes.c_int64),
        ("memory", ctypes.c_int32),
        ("input_ids", _P), ("attention_mask", _P), ("marker_pos", _P), ("marker_mask", _P),
        ("qtype", _P), ("nopts", _P), ("real_len", _P), ("real_k", _P), ("prefix_len", _P),
    ]


class VdStats(ctypes.Structure):
    _fields_ = [
        ("rows", ctypes.c_int64), ("tokens", ctypes.c_int64), ("chunks", ctypes.c_int64),
        ("launches", ctypes.c_int64), ("forward_ms", ctypes.c_double),
        ("gemm_flops", ctypes.c_double), ("attn_flops", ctypes.c_double),
        ("kernel_ms", ctypes.c_double * 8), ("kernel_launches", ctypes.c_int64 * 8),
        ("kernel_flops", ctypes.c_double * 8),
        ("host_ms", ctypes.c_double), ("enqueue_ms", ctypes.c_double),
        ("fork_groups", ctypes.c_int64), ("fork_rows", ctypes.c_int64), ("shared_tokens", ctypes.c_int64),
        ("prep_ms", ctypes.c_double), ("finish_ms", ctypes.c_double), ("upload_ms", ctypes.c_double),
        ("download_ms", ctypes.c_double),
    ]


KERNEL_CLASSES = ["qkv", "o", "gateup", "down", "attention", "norm", "other", "gdn"]


# Every entry point of include/vdexec.h: name -> (restype, argtypes)
SIGNATURES = {
    "vd_abi_version": (ctypes.c_int, []),
    "vd_resolve_spec": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_size_t, ctypes.c_char_p,
                                       ctypes.c_size_t]),
    "vd_open": (ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.c_char_p, ctypes.POINTER(_P),
                               ctypes.c_char_p, ctypes.c_size_t]),
    "vd_infer": (ctypes.c_int, [_P, ctypes.POINTER(VdBatch), _P, ctypes.c_int64, ctypes.c_char_p, ctypes.c_size_t]),
    "vd_infer_async": (ctypes.c_int, [_P, ctypes.POINTER(VdBatch), _P, ctypes.c_int64, _P, ctypes.c_char_p,
                                      ctypes.c_size_t]),
    "vd_sync": (ctypes.c_int, [_P, ctypes.c_char_p, ctypes.c_size_t]),
    "vd_stream": (_P, [_P]),
    "vd_shape_buckets": (ctypes.c_int, [_P, _I64P, ctypes.c_int64]),
    "vd_media_capable": (ctypes.c_int, [_P]),
    "vd_health": (ctypes.c_int, [_P]),
    "vd_label_width": (ctypes.c_int64, [_P]),
    "vd_last_stats": (ctypes.c_int, [_P, ctypes.POINTER(VdStats)]),
    "vd_set_profiling": (ctypes.c_int, [_P, ctypes.c_int]),
    "vd_close": (None, [_P]),
    # include/vdexec_kernels.h
    "vdk_gemm": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_int,
                                ctypes.c_int, _P, _P, ctypes.c_int64, _P, ctypes.c_char_p, ctypes.c_size_t]),
    "vdk_gemm_qkrope": (ctypes.c_int, [_P, _P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _P, _P, _P,
                                       ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_float, _P,
                                       ctypes.c_double, ctypes.c_int, _P, ctypes.c_int64, _P, ctypes.c_char_p,
                                       ctypes.c_size_t]),
    "vdk_attention": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int,
                                     ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P, ctypes.c_int64, _P,
                                     ctypes.c_int64, _P, ctypes.c_char_p, ctypes.c_size_t]),
    "vdk_attention_tc": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                        ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                        ctypes.c_int64, _P, ctypes.c_int64, _P, ctypes.c_char_p, ctypes.c_size_t]),
    "vdk_attention_noalloc": (ctypes.c_int, [_P, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64, ctypes.c_int64,
                                             ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _P,
                                             ctypes.c_int64, _P, ctypes.c_int64, _P, ctypes.c_char_p,
                                             ctypes.c_size_t]),
}

_lib = None


def lib_path() -> str:
    return _build.LIB


def load(build_if_missing: bool = True) -> ctypes.CDLL:
    """Load libvdexec.so (building it with nvcc first if it is absent or stale)."""
    global _lib
    if _lib is not None:
        return _lib
    path = _build.LIB
    if build_if_missing and not _build.up_to_date():
        try:
            _build.build()
        except Exception:
            if not os.path.exists(path):
                raise
    if not os.path.exists(path):
        raise RuntimeError(f"libvdexec.so is not built ({path}); run `python -m verdict_b200.build`")
    lib = ctypes.CDLL(path)
    for name, (res, args) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = res
        fn.argtypes = args
    _lib = lib
    return lib


class VdError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code
        self.msg = msg


def check(rc: int, err: ctypes.Array) -> None:
    if rc != VD_OK:
        raise VdError(rc, err.value.decode("utf-8", "replace"))
