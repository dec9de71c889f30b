"""vdk_attention_noalloc: the attention kernel for callers that must not allocate.

Some callers cannot call cudaMalloc: processes whose GPU memory is owned up
front by another allocator, or latency-critical paths where an allocation
would block on the device.  This entry point keeps the kernel's per-call tile
table in a fixed device array instead of allocating it.  The test checks it
against vdk_attention (which allocates its table each call) on two different
batches in a row, so a second call that read stale entries of the shared
array would fail, and checks that an oversized batch is refused before any
launch.  It lives in its own file so pytest collects it last.
"""

import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from verdict_b200 import _abi  # noqa: E402

pytestmark = pytest.mark.gpu

MAX_TILES = 16384
REL = 2e-2  # the attention tolerance of tests/test_kernels_gpu.py


def _call(fn, qkv, width, nq, nkv, hd, dt_code, causal, cu, out):
    err = ctypes.create_string_buffer(1024)
    rc = fn(ctypes.c_void_p(qkv.data_ptr()), width, 0, nq * hd, (nq + nkv) * hd, nq, nkv, hd, dt_code,
            1 if causal else 0, ctypes.c_void_p(cu.ctypes.data), len(cu) - 1, ctypes.c_void_p(out.data_ptr()),
            nq * hd, None, err, len(err))
    return rc, err.value.decode()


def _close(got, ref):
    got, ref = got.float(), ref.float()
    rms = ref.pow(2).mean().sqrt().item()
    err = (got - ref).abs()
    assert (err <= REL * ref.abs() + REL * rms + 1e-6).all(), f"max err {err.max().item():.3e}"


@pytest.mark.parametrize("hd,nq,nkv,causal,dt", [(128, 32, 8, True, "fp16"), (64, 12, 12, False, "bf16")])
def test_noalloc_matches_allocating_entry_point_twice(hd, nq, nkv, causal, dt):
    lib = _abi.load()
    torch_dt, code = {"fp16": (torch.float16, 0), "bf16": (torch.bfloat16, 1)}[dt]
    g = torch.Generator(device="cuda").manual_seed(hd + nq)
    width = (nq + 2 * nkv) * hd
    # Two different batches: the second has fewer, shorter tiles than the first.
    for lens in ([700, 1, 64, 65, 300], [130, 9]):
        cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
        T = int(cu[-1])
        qkv = (torch.randn(T, width, generator=g, device="cuda")).to(torch_dt)
        ref = torch.zeros(T, nq * hd, device="cuda", dtype=torch_dt)
        got = torch.full((T, nq * hd), float("nan"), device="cuda", dtype=torch_dt)
        rc, msg = _call(lib.vdk_attention, qkv, width, nq, nkv, hd, code, causal, cu, ref)
        assert rc == 0, msg
        rc, msg = _call(lib.vdk_attention_noalloc, qkv, width, nq, nkv, hd, code, causal, cu, got)
        assert rc == 0, msg
        _close(got, ref)


def test_noalloc_rejects_batches_beyond_its_table():
    lib = _abi.load()
    qkv = torch.zeros(64, 3 * 128, device="cuda", dtype=torch.float16)
    out = torch.zeros(64, 128, device="cuda", dtype=torch.float16)
    # One sequence that would need MAX_TILES + 1 query tiles; refused on the host
    # before any launch, so the small buffers are never read.
    cu = np.array([0, 64 * (MAX_TILES + 1)], dtype=np.int32)
    rc, msg = _call(lib.vdk_attention_noalloc, qkv, 3 * 128, 1, 1, 128, 0, True, cu, out)
    assert rc == _abi.VD_EINVAL and "at most 16384" in msg
