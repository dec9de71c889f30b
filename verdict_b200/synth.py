"""Deterministic synthetic checkpoints and seeded synthetic decision workloads.

No weights ship with this package, so every model is random-initialised from a seed.
The generator is counter-based: element `i` of tensor `name` is a pure function of
(seed, name, i).  The C library evaluates the same function on the GPU
(`csrc/synth.cuh`), the numpy code below evaluates it on the host, and both
produce bit-identical bf16 values, so the CUDA forward and the CPU oracle read
the same checkpoint without ever shipping one.

Element value: u = top 24 bits of splitmix64(base + i) / 2^24;
    w = bf16_rne(fp32((2u - 1) * scale) + offset)
with base = fnv1a64(name) XOR (seed * 0x9E3779B97F4A7C15).  A uniform with
scale = std * sqrt(3) has the standard deviation `std` that HF's normal
initialiser uses (`initializer_range`, 0.02).
"""

from __future__ import annotations

import math

import numpy as np

from .spec import label_width

MASK64 = (1 << 64) - 1
GOLDEN = 0x9E3779B97F4A7C15
SQRT3 = math.sqrt(3.0)


def fnv1a64(text: str) -> int:
    h = 0xCBF29CE484222325
    for byte in text.encode("utf-8"):
        h ^= byte
        h = (h * 0x100000001B3) & MASK64
    return h


def tensor_base(seed: int, name: str) -> int:
    return (fnv1a64(name) ^ ((seed * GOLDEN) & MASK64)) & MASK64


def _splitmix(z: np.ndarray) -> np.ndarray:
    with np.errstate(over="ignore"):
        z = z + np.uint64(GOLDEN)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even); returned as fp32 values."""
    bits = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    bias = ((bits >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        out = (bits + bias) & np.uint32(0xFFFF0000)
    return out.view(np.float32)


def gen_elements(base: int, index: np.ndarray, scale: float, offset: float) -> np.ndarray:
    """Values of the elements at flat positions `index` (uint64) of a tensor."""
    with np.errstate(over="ignore"):
        z = np.uint64(base) + index.astype(np.uint64)
    u = (_splitmix(z) >> np.uint64(40)).astype(np.float32) * np.float32(2.0 ** -24)
    v = (u * np.float32(2.0) - np.float32(1.0)) * np.float32(scale)
    v = (v + np.float32(offset)).astype(np.float32)
    return bf16_round(v)


def gen_tensor(seed: int, name: str, shape, scale: float, offset: float = 0.0,
               rows=None) -> np.ndarray:
    """A whole tensor, or only the listed rows of a 2-D tensor (row-major)."""
    base = tensor_base(seed, name)
    shape = tuple(int(s) for s in shape)
    if rows is None:
        n = int(np.prod(shape))
        out = np.empty(n, dtype=np.float32)
        chunk = 1 << 24
        for s in range(0, n, chunk):
            e = min(n, s + chunk)
            out[s:e] = gen_elements(base, np.arange(s, e, dtype=np.uint64), scale, offset)
        return out.reshape(shape)
    rows = np.asarray(rows, dtype=np.int64)
    cols = shape[1]
    idx = rows.astype(np.uint64)[:, None] * np.uint64(cols) + np.arange(cols, dtype=np.uint64)[None, :]
    return gen_elements(base, idx.reshape(-1), scale, offset).reshape(len(rows), cols)


# ---------------------------------------------------------------------------
# Tensor inventory: names, shapes and init of each synthetic checkpoint tensor.
# ---------------------------------------------------------------------------

def _lin(spec):
    return spec["init_std"] * SQRT3


def hybrid_tensors(spec: dict):
    """(name, shape, scale, offset) of a Qwen3.5 text stack (HF `Qwen3_5ForCausalLM` names).

    Every `Qwen3_5RMSNorm` applies (1 + w) and is zero-initialised in HF, so its
    synthetic w is U(-0.1, 0.1); the gated-delta-net output norm applies w
    (ones-initialised).  `A_log` = log(A) with A in [1, e^2], `dt_bias` ~ 1,
    the depthwise conv kernel U(-0.5, 0.5) (PyTorch's Conv1d bound 1/sqrt(4))."""
    d, hd = spec["hidden"], spec["head_dim"]
    nq, nkv, f = spec["heads"], spec["kv_heads"], spec["ffn"]
    kd = spec["lin_k_heads"] * spec["lin_k_dim"]
    vd = spec["lin_v_heads"] * spec["lin_v_dim"]
    lv, ck = spec["lin_v_heads"], spec["conv_kernel"]
    lin = _lin(spec)
    n_scale = 0.1
    out = [("model.embed_tokens.weight", (spec["vocab"], d), lin, 0.0)]
    for i, kind in enumerate(spec["layer_types"]):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (d,), n_scale, 0.0),
                (p + "post_attention_layernorm.weight", (d,), n_scale, 0.0)]
        if kind == "full_attention":
            out += [
                (p + "self_attn.q_proj.weight", (2 * nq * hd, d), lin, 0.0),
                (p + "self_attn.k_proj.weight", (nkv * hd, d), lin, 0.0),
                (p + "self_attn.v_proj.weight", (nkv * hd, d), lin, 0.0),
                (p + "self_attn.o_proj.weight", (d, nq * hd), lin, 0.0),
                (p + "self_attn.q_norm.weight", (hd,), n_scale, 0.0),
                (p + "self_attn.k_norm.weight", (hd,), n_scale, 0.0),
            ]
        else:
            a = p + "linear_attn."
            out += [
                (a + "in_proj_qkv.weight", (2 * kd + vd, d), lin, 0.0),
                (a + "in_proj_z.weight", (vd, d), lin, 0.0),
                (a + "in_proj_b.weight", (lv, d), lin, 0.0),
                (a + "in_proj_a.weight", (lv, d), lin, 0.0),
                (a + "conv1d.weight", (2 * kd + vd, 1, ck), 0.5, 0.0),
                (a + "dt_bias", (lv,), 0.1, 1.0),
                (a + "A_log", (lv,), 1.0, 1.0),
                (a + "norm.weight", (spec["lin_v_dim"],), 0.1, 1.0),
                (a + "out_proj.weight", (d, vd), lin, 0.0),
            ]
        out += [(p + "mlp.gate_proj.weight", (f, d), lin, 0.0),
                (p + "mlp.up_proj.weight", (f, d), lin, 0.0),
                (p + "mlp.down_proj.weight", (d, f), lin, 0.0)]
    out.append(("model.norm.weight", (d,), n_scale, 0.0))
    if not spec["tied"]:
        out.append(("lm_head.weight", (spec["vocab"], d), lin, 0.0))
    return out


def decoder_tensors(spec: dict):
    """(name, shape, scale, offset) of every decoder tensor, HF Qwen3/Gemma names."""
    if spec.get("style") == "qwen3_5":
        return hybrid_tensors(spec)
    d, hd = spec["hidden"], spec["head_dim"]
    nq, nkv, f = spec["heads"], spec["kv_heads"], spec["ffn"]
    lin = _lin(spec)
    # Norm gains: 1 + U(-0.1, 0.1).  Gemma stores w and applies (1 + w).
    n_scale, n_off = 0.1, (0.0 if spec["norm_plus_one"] else 1.0)
    out = [("model.embed_tokens.weight", (spec["vocab"], d), lin, 0.0)]
    for i in range(spec["layers"]):
        p = f"model.layers.{i}."
        out += [
            (p + "input_layernorm.weight", (d,), n_scale, n_off),
            (p + "self_attn.q_proj.weight", (nq * hd, d), lin, 0.0),
            (p + "self_attn.k_proj.weight", (nkv * hd, d), lin, 0.0),
            (p + "self_attn.v_proj.weight", (nkv * hd, d), lin, 0.0),
            (p + "self_attn.o_proj.weight", (d, nq * hd), lin, 0.0),
            (p + "post_attention_layernorm.weight", (d,), n_scale, n_off),
            (p + "mlp.gate_proj.weight", (f, d), lin, 0.0),
            (p + "mlp.up_proj.weight", (f, d), lin, 0.0),
            (p + "mlp.down_proj.weight", (d, f), lin, 0.0),
        ]
        if spec["qk_norm"]:
            out += [(p + "self_attn.q_norm.weight", (hd,), n_scale, n_off),
                    (p + "self_attn.k_norm.weight", (hd,), n_scale, n_off)]
        if spec["qkv_bias"]:
            out += [(p + "self_attn.q_proj.bias", (nq * hd,), lin, 0.0),
                    (p + "self_attn.k_proj.bias", (nkv * hd,), lin, 0.0),
                    (p + "self_attn.v_proj.bias", (nkv * hd,), lin, 0.0)]
    out.append(("model.norm.weight", (d,), n_scale, n_off))
    if not spec["tied"]:
        out.append(("lm_head.weight", (spec["vocab"], d), lin, 0.0))
    return out


def encoder_tensors(spec: dict):
    """(name, shape, scale, offset) of every marker-head encoder tensor.

    Encoder names follow HF BertModel / XLMRobertaModel; the decision head follows
    `DecisionModel` (`convert/marker_head/marker_head_converter.py:19-39`), whose
    head layers are `nn.TransformerEncoderLayer(d, d//64, 4d, norm_first=True)`."""
    d, f = spec["hidden"], spec["ffn"]
    lin = _lin(spec)
    g_scale, g_off = 0.1, 1.0
    b_scale = lin
    e = "encoder."
    out = [
        (e + "embeddings.word_embeddings.weight", (spec["vocab"], d), lin, 0.0),
        (e + "embeddings.position_embeddings.weight", (spec["max_pos"], d), lin, 0.0),
        (e + "embeddings.token_type_embeddings.weight", (spec["type_vocab"], d), lin, 0.0),
        (e + "embeddings.LayerNorm.weight", (d,), g_scale, g_off),
        (e + "embeddings.LayerNorm.bias", (d,), b_scale, 0.0),
    ]
    for i in range(spec["layers"]):
        p = f"{e}encoder.layer.{i}."
        out += [
            (p + "attention.self.query.weight", (d, d), lin, 0.0),
            (p + "attention.self.query.bias", (d,), b_scale, 0.0),
            (p + "attention.self.key.weight", (d, d), lin, 0.0),
            (p + "attention.self.key.bias", (d,), b_scale, 0.0),
            (p + "attention.self.value.weight", (d, d), lin, 0.0),
            (p + "attention.self.value.bias", (d,), b_scale, 0.0),
            (p + "attention.output.dense.weight", (d, d), lin, 0.0),
            (p + "attention.output.dense.bias", (d,), b_scale, 0.0),
            (p + "attention.output.LayerNorm.weight", (d,), g_scale, g_off),
            (p + "attention.output.LayerNorm.bias", (d,), b_scale, 0.0),
            (p + "intermediate.dense.weight", (f, d), lin, 0.0),
            (p + "intermediate.dense.bias", (f,), b_scale, 0.0),
            (p + "output.dense.weight", (d, f), lin, 0.0),
            (p + "output.dense.bias", (d,), b_scale, 0.0),
            (p + "output.LayerNorm.weight", (d,), g_scale, g_off),
            (p + "output.LayerNorm.bias", (d,), b_scale, 0.0),
        ]
    out.append(("type_emb.weight", (3, d), lin, 0.0))
    for i in range(spec["head_layers"]):
        p = f"head.layers.{i}."
        out += [
            (p + "self_attn.in_proj_weight", (3 * d, d), lin, 0.0),
            (p + "self_attn.in_proj_bias", (3 * d,), b_scale, 0.0),
            (p + "self_attn.out_proj.weight", (d, d), lin, 0.0),
            (p + "self_attn.out_proj.bias", (d,), b_scale, 0.0),
            (p + "linear1.weight", (4 * d, d), lin, 0.0),
            (p + "linear1.bias", (4 * d,), b_scale, 0.0),
            (p + "linear2.weight", (d, 4 * d), lin, 0.0),
            (p + "linear2.bias", (d,), b_scale, 0.0),
            (p + "norm1.weight", (d,), g_scale, g_off),
            (p + "norm1.bias", (d,), b_scale, 0.0),
            (p + "norm2.weight", (d,), g_scale, g_off),
            (p + "norm2.bias", (d,), b_scale, 0.0),
        ]
    out += [
        ("scorer.0.weight", (d,), g_scale, g_off),
        ("scorer.0.bias", (d,), b_scale, 0.0),
        ("scorer.1.weight", (d, d), lin, 0.0),
        ("scorer.1.bias", (d,), b_scale, 0.0),
        ("scorer.3.weight", (1, d), lin, 0.0),
        ("scorer.3.bias", (1,), b_scale, 0.0),
    ]
    return out


def von_tensors(spec: dict):
    """(name, shape, scale, offset) of an independent-options model: HF
    `ModernBertModel` under "encoder." (its LayerNorms have no bias) and a
    per-marker scorer under "scorer." laid out like the marker head's
    LayerNorm -> Linear -> GELU -> Linear(d, 1)."""
    d, f = spec["hidden"], spec["ffn"]
    lin = _lin(spec)
    g_scale, g_off = 0.1, 1.0
    e = "encoder."
    out = [(e + "embeddings.tok_embeddings.weight", (spec["vocab"], d), lin, 0.0),
           (e + "embeddings.norm.weight", (d,), g_scale, g_off)]
    for i in range(spec["layers"]):
        p = f"{e}layers.{i}."
        if i > 0:
            out.append((p + "attn_norm.weight", (d,), g_scale, g_off))
        out += [(p + "attn.Wqkv.weight", (3 * d, d), lin, 0.0),
                (p + "attn.Wo.weight", (d, d), lin, 0.0),
                (p + "mlp_norm.weight", (d,), g_scale, g_off),
                (p + "mlp.Wi.weight", (2 * f, d), lin, 0.0),
                (p + "mlp.Wo.weight", (d, f), lin, 0.0)]
    # scorer Linears at PyTorch's default scale (U(+-1/sqrt(fan_in))), so the
    # option logits are O(1) and their differences carry signal
    unit = 1.0 / np.sqrt(d)
    out += [(e + "final_norm.weight", (d,), g_scale, g_off),
            ("scorer.0.weight", (d,), g_scale, g_off),
            ("scorer.0.bias", (d,), lin, 0.0),
            ("scorer.1.weight", (d, d), unit * SQRT3, 0.0),
            ("scorer.1.bias", (d,), unit, 0.0),
            ("scorer.3.weight", (1, d), unit * SQRT3 * 4, 0.0),
            ("scorer.3.bias", (1,), unit, 0.0)]
    return out


def tensor_table(spec: dict):
    if spec["arch"] == "decoder":
        return decoder_tensors(spec)
    return von_tensors(spec) if spec.get("style") == "modernbert" else encoder_tensors(spec)


class SyntheticCheckpoint:
    """Lazy host view of a synthetic checkpoint: tensors are generated on request."""

    def __init__(self, spec: dict):
        self.spec = spec
        self.table = {name: (shape, scale, off) for name, shape, scale, off in tensor_table(spec)}

    def names(self):
        return list(self.table)

    def get(self, name: str, rows=None) -> np.ndarray:
        shape, scale, off = self.table[name]
        return gen_tensor(self.spec["seed"], name, shape, scale, off, rows=rows)

    def head_name(self) -> str:
        return "model.embed_tokens.weight" if self.spec["tied"] else "lm_head.weight"


# ---------------------------------------------------------------------------
# Label tables
# ---------------------------------------------------------------------------

def synthetic_label_ids(spec: dict) -> list:
    """Distinct seeded option-label token ids in [3, vocab), one per label row.

    Real checkpoints derive these from the tokenizer (`derive_branch_ids` /
    `derive_letter_ids`, `executor/torch_exec.py:2254-2323`); a synthetic
    checkpoint has no tokenizer, so it draws them."""
    if spec.get("label_ids"):
        return [int(x) for x in spec["label_ids"]]
    rng = np.random.default_rng(spec["seed"] ^ 0x1AB31)
    width = label_width(spec)
    ids = rng.choice(np.arange(3, spec["vocab"]), size=width, replace=False)
    return [int(x) for x in ids]


def with_labels(spec: dict) -> dict:
    """The spec with its label table filled in where it has none (decoders only)."""
    out = dict(spec)
    if out["arch"] == "decoder" and out.get("label_ids") is None:
        out["label_ids"] = synthetic_label_ids(out)
    return out
