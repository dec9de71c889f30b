"""Host-side `Engine` backed by the B200 executor (libvdexec.so).

Mirrors the reference's executor interface (`src/engine.rs:10-44`):
    class Engine: infer(CollatedBatch) -> list[EngineRow]; media_capable(); shape_buckets(); health()
`B200Engine` is the drop-in for `TorchEngine` (`src/torch_engine.rs:445-524`): it
validates a letter batch the same way (k == 1, one nopts per row, every row has a
slot marker), runs the whole forward on one GPU through the C ABI, and returns
one `EngineRow` per row.  Letter rows hold the label-row scores with columns
>= nopts set to -1e4, as `finish_rows` does (`src/torch_engine.rs:97-114`); by
default the scores are log-probabilities restricted to the options (softmax is
shift-invariant, so `calibrate`'s `softmax(logits / t)` is unchanged).  Marker
rows hold the scorer logits with -1e4 on masked slots.

`Pool` restates the replica pool (`src/pipeline.rs:310-352`): round-robin over
replicas with spill-over to the next one when a replica is overloaded.
"""

from __future__ import annotations

import ctypes
import json
import os
import threading
from dataclasses import dataclass
from typing import Optional, Sequence

import numpy as np

from . import _abi
from .batch import CollatedBatch
from .checkpoint import resolve_spec
from .synth import with_labels


class EngineError(RuntimeError):
    """`EngineError` (`src/engine.rs:10-12`): fails every request of the batch."""


class Overloaded(RuntimeError):
    """A replica refused the batch because it is busy (`ApiError::Overloaded`)."""


@dataclass
class EngineRow:
    """`EngineRow` (`src/engine.rs:14-18`)."""
    logits: list
    expanded_len: Optional[int] = None


class Engine:
    """The executor interface (`trait Engine`, `src/engine.rs:28-40`)."""

    def infer(self, batch: CollatedBatch) -> list:
        raise NotImplementedError

    def media_capable(self) -> bool:
        return False

    def shape_buckets(self) -> list:
        return []

    def health(self) -> bool:
        raise NotImplementedError


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else ctypes.c_void_p(a.ctypes.data)


class B200Engine(Engine):
    """One model replica on one GPU (`TorchEngine::with_device`, `src/torch_engine.rs:280-316`)."""

    def __init__(self, spec, device: int = 0, *, max_tokens: int = 65536, max_rows: int = 512,
                 max_seq: int = 8192, max_markers: int = 16384, output: str = "logprobs",
                 act_dtype: str = "fp16", attention: str = "tc",
                 prune_last_layer: bool = True, fork: bool = True, gemm: str = "2sm",
                 raster_group: int = 0, gdn: str = "chunk", norm: str = "fused", split_k: bool = False,
                 attention_persistent: bool = True, attention_threads_per_row: int = 1, l2_hints: bool = False,
                 pdl: bool = True, wait_limit_us: int = 0, debug_stall_gemm: int = 0):
        """`spec`: a spec dict, or a directory holding `vdexec.json` (whose
        relative "checkpoint" path is taken from that directory).
        `norm` (decoders): "fused" folds each RMSNorm into the residual GEMM that
        produces its input and the projection that reads it; "separate" runs it
        as its own kernel.
        `split_k` (off by default: measured slower at the 9B shapes, the
        partial tiles' round trip through memory outweighing the fuller
        waves): batches of up to 1024 tokens split K over CTAs (partials added
        in a fixed order: the same bits on every run, within rounding of the
        unsplit sum).
        `attention_persistent`: the tcgen05 attention's CTAs loop over work
        items (query tile x head) instead of one CTA per item.
        `attention_threads_per_row`: softmax threads per query row in that
        kernel (1: four softmax warps; 2: eight, each with half a key tile).
        `l2_hints`: the pair GEMM's TMA loads ask L2 to keep A rows (evict
        last) and let W tiles go first (evict first).
        `pdl`: the GEMM and attention kernels are launched with programmatic
        stream serialization, so each sets up under the previous kernel's tail
        and waits for its results before touching global memory.
        `wait_limit_us`: limit of the GEMM kernels' pipeline waits (0: 2 s);
        `debug_stall_gemm` (failure-path tests only): the first one-CTA GEMM of
        every call stops loading after that many k-blocks, so its wait runs out."""
        self.lib = _abi.load()
        if isinstance(spec, (str, os.PathLike)):
            model = os.fspath(spec).encode()
            self.spec = resolve_spec(spec)
        else:
            if "hidden" not in spec and "checkpoint" in spec:
                spec = resolve_spec(spec)  # shape from the checkpoint's HF config
            self.spec = with_labels(spec)
            model = json.dumps(self.spec).encode()
        self.device = device
        self.decoder = self.spec["arch"] == "decoder"
        opts = json.dumps(dict(max_tokens=max_tokens, max_rows=max_rows, max_seq=max_seq,
                               max_markers=max_markers, output=output, act_dtype=act_dtype,
                               attention=attention, prune_last_layer=prune_last_layer, fork=fork,
                               gemm=gemm, raster_group=raster_group, gdn=gdn, norm=norm, split_k=split_k,
                               attention_persistent=attention_persistent,
                               attention_threads_per_row=attention_threads_per_row, l2_hints=l2_hints,
                               pdl=pdl, wait_limit_us=wait_limit_us,
                               debug_stall_gemm=debug_stall_gemm))
        err = ctypes.create_string_buffer(1024)
        h = ctypes.c_void_p()
        rc = self.lib.vd_open(model, device, opts.encode(), ctypes.byref(h), err, len(err))
        _abi.check(rc, err)
        self.h = h
        self._lock = threading.Lock()
        self.width = int(self.lib.vd_label_width(self.h)) if self.decoder else 0

    # -- Engine --------------------------------------------------------------
    def media_capable(self) -> bool:
        return bool(self.lib.vd_media_capable(self.h))

    def shape_buckets(self) -> list:
        out = (ctypes.c_int64 * 64)()
        n = self.lib.vd_shape_buckets(self.h, out, 64)
        return [int(out[i]) for i in range(max(0, n))]

    def health(self) -> bool:
        return bool(self.lib.vd_health(self.h))

    def infer(self, batch: CollatedBatch) -> list:
        """`Engine::infer` over host memory; raises EngineError like the reference."""
        b = batch.b
        if self.decoder and (batch.k != 1 or len(batch.nopts) != b):
            raise EngineError(f"letter batches need exactly one slot per row "
                              f"(got k={batch.k}, nopts={len(batch.nopts)})")
        if self.decoder:
            for i in range(b):
                if not batch.marker_mask[i]:
                    raise EngineError(f"row {i} has no slot marker")
        width = self.width if self.decoder else max(batch.k, 1)
        out = np.empty((b, width), dtype=np.float32)
        try:
            self.infer_host_arrays(batch, out)
        except _abi.VdError as e:
            raise EngineError(e.msg) from e
        return [EngineRow(logits=out[i].astype(np.float64).tolist()) for i in range(b)]

    # -- lower level -----------------------------------------------------------
    def _batch_struct(self, batch: CollatedBatch, arrays: dict) -> _abi.VdBatch:
        st = _abi.VdBatch()
        st.b, st.l, st.k = batch.b, batch.l, batch.k
        st.memory = _abi.VD_MEM_HOST
        st.input_ids = _ptr(arrays["ids"])
        st.attention_mask = _ptr(arrays["mask"])
        st.marker_pos = _ptr(arrays["mpos"])
        st.marker_mask = _ptr(arrays["mmask"])
        st.qtype = _ptr(arrays["qtype"])
        st.nopts = _ptr(arrays["nopts"])
        st.real_len = _ptr(arrays["real_len"])
        st.real_k = _ptr(arrays["real_k"])
        st.prefix_len = _ptr(arrays["prefix_len"])
        return st

    def infer_host_arrays(self, batch: CollatedBatch, out: np.ndarray) -> None:
        """vd_infer on host arrays; `out` is float32 [b, width] (C-contiguous)."""
        arrays = dict(
            ids=np.ascontiguousarray(batch.input_ids, dtype=np.int64),
            mask=np.ascontiguousarray(batch.attention_mask, dtype=np.int64),
            mpos=np.ascontiguousarray(batch.marker_pos, dtype=np.int64),
            mmask=np.ascontiguousarray(batch.marker_mask, dtype=np.uint8),
            qtype=np.ascontiguousarray(batch.qtype, dtype=np.int64),
            nopts=np.ascontiguousarray(batch.nopts, dtype=np.int64) if len(batch.nopts) else None,
            real_len=batch.real_len(), real_k=batch.real_k(), prefix_len=batch.prefix_len(),
        )
        st = self._batch_struct(batch, arrays)
        assert out.flags.c_contiguous and out.dtype == np.float32 and out.shape[0] == batch.b
        err = ctypes.create_string_buffer(1024)
        with self._lock:
            rc = self.lib.vd_infer(self.h, ctypes.byref(st), ctypes.c_void_p(out.ctypes.data), out.shape[1],
                                   err, len(err))
        _abi.check(rc, err)

    def infer_device(self, b: int, l: int, k: int, ptrs: dict, real_len: np.ndarray, out_ptr: int, width: int,
                     stream: Optional[int] = None, sync: bool = False,
                     prefix_len: Optional[np.ndarray] = None) -> None:
        """vd_infer_async on device-resident arrays (`ptrs`: integer device
        addresses); `prefix_len` (host) lets the engine fork shared prefixes."""
        st = _abi.VdBatch()
        st.b, st.l, st.k = b, l, k
        st.memory = _abi.VD_MEM_DEVICE
        for name in ("input_ids", "attention_mask", "marker_pos", "marker_mask", "qtype", "nopts"):
            v = ptrs.get(name)
            setattr(st, name, None if v is None else ctypes.c_void_p(v))
        real_len = np.ascontiguousarray(real_len, dtype=np.int64)
        st.real_len = ctypes.c_void_p(real_len.ctypes.data)
        if prefix_len is not None:
            prefix_len = np.ascontiguousarray(prefix_len, dtype=np.int64)
            st.prefix_len = ctypes.c_void_p(prefix_len.ctypes.data)
        err = ctypes.create_string_buffer(1024)
        with self._lock:
            rc = self.lib.vd_infer_async(self.h, ctypes.byref(st), ctypes.c_void_p(out_ptr), width,
                                         ctypes.c_void_p(stream) if stream else None, err, len(err))
            _abi.check(rc, err)
            if sync:
                rc = self.lib.vd_sync(self.h, err, len(err))
                _abi.check(rc, err)

    def sync(self) -> None:
        err = ctypes.create_string_buffer(1024)
        _abi.check(self.lib.vd_sync(self.h, err, len(err)), err)

    def stream(self) -> int:
        return int(self.lib.vd_stream(self.h) or 0)

    def last_stats(self) -> dict:
        s = _abi.VdStats()
        self.lib.vd_last_stats(self.h, ctypes.byref(s))
        return {name: getattr(s, name) for name, _ in _abi.VdStats._fields_}

    def close(self) -> None:
        if getattr(self, "h", None):
            self.lib.vd_close(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Pool:
    """Round-robin replica pool with spill-over (`Pool::route`, `src/pipeline.rs:329-352`)."""

    def __init__(self, replicas: Sequence[Engine]):
        if not replicas:
            raise ValueError("a pool needs at least one replica")
        self.replicas = list(replicas)
        self._next = 0
        self._lock = threading.Lock()

    def route(self, call):
        n = len(self.replicas)
        with self._lock:
            start = self._next
            self._next += 1
        for i in range(n):
            replica = self.replicas[(start + i) % n]
            try:
                return call(replica)
            except Overloaded:
                continue
        raise Overloaded("every replica is overloaded")

    def infer(self, batch: CollatedBatch) -> list:
        return self.route(lambda r: r.infer(batch))
