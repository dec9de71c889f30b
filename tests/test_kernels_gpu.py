"""Each sm_100a kernel against a plain PyTorch fp32 reference of the same op.

Kernels are called through the C ABI (include/vdexec_kernels.h) on torch-owned
device buffers, in both 16-bit element types (fp16, bf16); torch computes the
fp32 reference from the same 16-bit inputs.
Tolerances: 16-bit outputs carry one rounding (relative 2^-8 for bf16, 2^-11
for fp16), so |got - ref| <= 1e-2 * |ref| + 1e-2 * rms(ref); fp32 outputs
(residual epilogue) differ only by fp32 accumulation order: 1e-4 relative.
"""

import ctypes
import math

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from verdict_b200 import _abi  # noqa: E402

pytestmark = pytest.mark.gpu

EPI_STORE, EPI_RESIDUAL, EPI_GATED = 0, 1, 2
DTYPES = {"fp16": (torch.float16, 0), "bf16": (torch.bfloat16, 1)}
ACT = {"none": 0, "gelu_erf": 1, "gelu_tanh": 2, "relu": 3, "silu": 4}


def lib():
    return _abi.load()


def P(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def run(fn, *args):
    err = ctypes.create_string_buffer(1024)
    rc = fn(*args, None, err, len(err))
    _abi.check(rc, err)


def torch_act(x, act):
    if act == "gelu_erf":
        return torch.nn.functional.gelu(x)
    if act == "gelu_tanh":
        return torch.nn.functional.gelu(x, approximate="tanh")
    if act == "relu":
        return torch.relu(x)
    if act == "silu":
        return torch.nn.functional.silu(x)
    return x


def close16(got, ref, rel=1e-2):
    got = got.float()
    rms = ref.pow(2).mean().sqrt().item()
    err = (got - ref).abs()
    bound = rel * ref.abs() + rel * rms + 1e-6
    bad = (err > bound).sum().item()
    assert bad == 0, f"{bad} of {ref.numel()} outside tolerance; max err {err.max().item():.3e} (rms {rms:.3e})"


def rand16(dt, *shape, scale=1.0, gen=None):
    return (torch.randn(*shape, generator=gen, device="cuda") * scale).to(DTYPES[dt][0])


@pytest.mark.parametrize("M,N,K", [(1, 256, 64), (100, 384, 256), (128, 256, 4096), (300, 1024, 512),
                                   (1000, 768, 768), (4097, 4096, 4096)])
@pytest.mark.parametrize("act", ["none", "gelu_erf"])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_gemm_store(M, N, K, act, dt):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N + K)
    A = rand16(dt, M, K, gen=g)
    W = rand16(dt, N, K, scale=K ** -0.5, gen=g)
    bias = torch.randn(N, generator=g, device="cuda") * 0.1
    out = torch.empty(M, N, device="cuda", dtype=DTYPES[dt][0])
    run(lib().vdk_gemm, P(A), P(W), M, N, K, DTYPES[dt][1], EPI_STORE, ACT[act], P(bias), P(out), N)
    ref = torch_act(A.float() @ W.float().T + bias, act)
    close16(out, ref)


@pytest.mark.parametrize("M,N,K", [(5, 256, 128), (257, 512, 1024), (2048, 4096, 12288)])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_gemm_residual(M, N, K, dt):
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    A = rand16(dt, M, K, gen=g)
    W = rand16(dt, N, K, scale=K ** -0.5, gen=g)
    h0 = torch.randn(M, N, generator=g, device="cuda")
    h = h0.clone()
    run(lib().vdk_gemm, P(A), P(W), M, N, K, DTYPES[dt][1], EPI_RESIDUAL, 0, None, P(h), N)
    ref = h0 + A.float() @ W.float().T
    torch.testing.assert_close(h, ref, rtol=1e-4, atol=1e-4)


@pytest.mark.parametrize("act", ["silu", "gelu_tanh"])
@pytest.mark.parametrize("M,F,K", [(3, 128, 256), (600, 1024, 512), (1500, 12288, 4096)])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_gemm_gated(M, F, K, act, dt):
    g = torch.Generator(device="cuda").manual_seed(M + F)
    A = rand16(dt, M, K, gen=g)
    Wg = rand16(dt, F, K, scale=K ** -0.5, gen=g)
    Wu = rand16(dt, F, K, scale=K ** -0.5, gen=g)
    # Interleave 128-row blocks: [g0, u0, g1, u1, ...]
    W = torch.stack([Wg.view(F // 128, 128, K), Wu.view(F // 128, 128, K)], 1).reshape(2 * F, K).contiguous()
    out = torch.empty(M, F, device="cuda", dtype=DTYPES[dt][0])
    run(lib().vdk_gemm, P(A), P(W), M, 2 * F, K, DTYPES[dt][1], EPI_GATED, ACT[act], None, P(out), F)
    ref = torch_act(A.float() @ Wg.float().T, act) * (A.float() @ Wu.float().T)
    close16(out, ref, rel=1.5e-2)


def rope_ref(x, pos, theta):
    hd = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, hd, 2, dtype=torch.int64, device=x.device).float() / hd))
    fr = pos.float()[:, None] * inv[None, :]
    emb = torch.cat([fr, fr], -1)
    cos, sin = emb.cos()[:, None, :], emb.sin()[:, None, :]
    rot = torch.cat([-x[..., hd // 2:], x[..., :hd // 2]], -1)
    return x * cos + rot * sin


@pytest.mark.parametrize("hd,nq,nkv,qk_norm,bias,plus_one", [
    (128, 32, 8, True, False, False),   # OneJev-9B-shaped
    (128, 4, 2, False, True, False),    # Qwen2-style bias, no q/k norm
    (128, 2, 1, True, False, False),    # k block narrower than a 256-wide tile
    (256, 8, 1, False, False, True),    # Gemma-2B-shaped MQA
])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_gemm_qkrope(hd, nq, nkv, qk_norm, bias, plus_one, dt):
    g = torch.Generator(device="cuda").manual_seed(hd + nq)
    M, K = 777, 512
    N = (nq + 2 * nkv) * hd
    A = rand16(dt, M, K, gen=g)
    W = rand16(dt, N, K, scale=K ** -0.5, gen=g)
    b = torch.randn(N, generator=g, device="cuda") * 0.1 if bias else None
    qn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")) if qk_norm else None
    kn = (1 + 0.1 * torch.randn(hd, generator=g, device="cuda")) if qk_norm else None
    pos = torch.randint(0, 4000, (M,), generator=g, device="cuda", dtype=torch.int32)
    out = torch.empty(M, N, device="cuda", dtype=DTYPES[dt][0])
    theta = 1e6 if hd == 128 else 1e4
    run(lib().vdk_gemm_qkrope, P(A), P(W), M, N, K, DTYPES[dt][1], P(b), P(qn), P(kn), nq * hd, nkv * hd, hd,
        1 if plus_one else 0, ctypes.c_float(1e-6), P(pos), ctypes.c_double(theta), 4096, P(out), N)
    y = A.float() @ W.float().T
    if b is not None:
        y = y + b
    q = y[:, :nq * hd].view(M, nq, hd)
    k = y[:, nq * hd:(nq + nkv) * hd].view(M, nkv, hd)
    v = y[:, (nq + nkv) * hd:]
    if qk_norm:
        def rms(x, w):
            return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
        q, k = rms(q, qn), rms(k, kn)
    q, k = rope_ref(q, pos, theta), rope_ref(k, pos, theta)
    ref = torch.cat([q.reshape(M, -1), k.reshape(M, -1), v], 1)
    close16(out, ref)


def attention_ref(qkv, cu, nq, nkv, hd, q0, k0, v0, causal):
    outs = []
    for i in range(len(cu) - 1):
        s, e = cu[i], cu[i + 1]
        x = qkv[s:e].float()
        q = x[:, q0:q0 + nq * hd].view(-1, nq, hd).transpose(0, 1)
        k = x[:, k0:k0 + nkv * hd].view(-1, nkv, hd).transpose(0, 1).repeat_interleave(nq // nkv, 0)
        v = x[:, v0:v0 + nkv * hd].view(-1, nkv, hd).transpose(0, 1).repeat_interleave(nq // nkv, 0)
        o = torch.nn.functional.scaled_dot_product_attention(q[None], k[None], v[None], is_causal=causal)[0]
        outs.append(o.transpose(0, 1).reshape(e - s, nq * hd))
    return torch.cat(outs, 0)


@pytest.mark.parametrize("hd,nq,nkv,causal", [(128, 32, 8, True), (256, 8, 1, True), (64, 12, 12, False),
                                              (128, 4, 4, True)])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_attention_varlen(hd, nq, nkv, causal, dt):
    g = torch.Generator(device="cuda").manual_seed(hd * 3 + nq)
    lens = [1, 63, 64, 65, 200, 17, 1000, 128]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    width = (nq + 2 * nkv) * hd
    qkv = rand16(dt, T, width, gen=g)
    out = torch.zeros(T, nq * hd, device="cuda", dtype=DTYPES[dt][0])
    q0, k0, v0 = 0, nq * hd, (nq + nkv) * hd
    run(lib().vdk_attention, P(qkv), width, q0, k0, v0, nq, nkv, hd, DTYPES[dt][1], 1 if causal else 0,
        ctypes.c_void_p(cu.ctypes.data), len(lens), P(out), nq * hd)
    ref = attention_ref(qkv, cu.tolist(), nq, nkv, hd, q0, k0, v0, causal)
    close16(out, ref, rel=2e-2)


def test_gemm_rejects_bad_shapes():
    A = torch.zeros(4, 64, device="cuda", dtype=torch.bfloat16)
    W = torch.zeros(100, 64, device="cuda", dtype=torch.bfloat16)
    out = torch.zeros(4, 100, device="cuda", dtype=torch.bfloat16)
    err = ctypes.create_string_buffer(256)
    rc = lib().vdk_gemm(P(A), P(W), 4, 100, 64, 1, 0, 0, None, P(out), 100, None, err, 256)
    assert rc == _abi.VD_EINVAL and b"N % 128" in err.value


@pytest.mark.parametrize("hd,nq,nkv", [(128, 32, 8), (128, 4, 4), (128, 40, 8), (256, 8, 1), (256, 16, 4),
                                       (256, 3, 3), (64, 12, 12), (64, 16, 4)])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_attention_tc_varlen(hd, nq, nkv, dt):
    """The tcgen05 / TMEM attention kernel (head_dim 128 and 256 causal, 64
    bidirectional) vs torch fp32 SDPA."""
    causal = hd != 64
    g = torch.Generator(device="cuda").manual_seed(hd + nq * 7 + nkv)
    lens = [1, 127, 128, 129, 300, 17, 1000, 256, 2100]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    width = (nq + 2 * nkv) * hd
    qkv = rand16(dt, T, width, gen=g)
    out = torch.zeros(T, nq * hd, device="cuda", dtype=DTYPES[dt][0])
    q0, k0, v0 = 0, nq * hd, (nq + nkv) * hd
    run(lib().vdk_attention_tc, P(qkv), width, q0, k0, v0, nq, nkv, hd, DTYPES[dt][1], int(causal),
        ctypes.c_void_p(cu.ctypes.data), len(lens), P(out), nq * hd)
    ref = attention_ref(qkv, cu.tolist(), nq, nkv, hd, q0, k0, v0, causal)
    # P enters the P.V product in the 16-bit type; with bf16 (8-bit mantissa)
    # and up to 2100 keys a few outputs drift just past 2e-2, hence 3e-2.
    close16(out, ref, rel=2e-2 if dt == "fp16" else 3e-2)


@pytest.mark.parametrize("hd,nq,nkv", [(128, 40, 8), (256, 8, 1)])
@pytest.mark.parametrize("dt", ["fp16", "bf16"])
def test_attention_tc_long_keys(hd, nq, nkv, dt):
    """Rows of 8,192 keys (the 27B shape's longest prompts) on the tcgen05
    kernel vs torch fp32 SDPA: the running max / rescale path over 128 key
    tiles and the 16-bit P at that depth."""
    g = torch.Generator(device="cuda").manual_seed(8192 + hd)
    lens = [8192, 4100, 3]
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    T = int(cu[-1])
    width = (nq + 2 * nkv) * hd
    qkv = rand16(dt, T, width, gen=g)
    out = torch.zeros(T, nq * hd, device="cuda", dtype=DTYPES[dt][0])
    q0, k0, v0 = 0, nq * hd, (nq + nkv) * hd
    run(lib().vdk_attention_tc, P(qkv), width, q0, k0, v0, nq, nkv, hd, DTYPES[dt][1], 1,
        ctypes.c_void_p(cu.ctypes.data), len(lens), P(out), nq * hd)
    ref = attention_ref(qkv, cu.tolist(), nq, nkv, hd, q0, k0, v0, True)
    # P enters P.V rounded to the 16-bit type (2^-9 relative for bf16, 2^-12
    # for fp16), so an output's error scales with sum_j p_j |v_j|, not with
    # |output|: where the terms cancel (short rows, |o| ~ 0) the relative bound
    # alone is too tight.  sum_j p_j |v_j| is the attention of |v|.
    qkv_abs = qkv.clone()
    qkv_abs[:, v0:v0 + nkv * hd] = qkv_abs[:, v0:v0 + nkv * hd].abs()
    mass = attention_ref(qkv_abs, cu.tolist(), nq, nkv, hd, q0, k0, v0, True)
    eps = 2.0 ** -9 if dt == "bf16" else 2.0 ** -12
    got = out.float()
    rms = ref.pow(2).mean().sqrt().item()
    bound = 2e-2 * ref.abs() + 2e-2 * rms + 4 * eps * mass + 1e-6
    bad = ((got - ref).abs() > bound).sum().item()
    assert bad == 0, f"{bad} of {ref.numel()} outside tolerance; max err {(got - ref).abs().max().item():.3e}"
