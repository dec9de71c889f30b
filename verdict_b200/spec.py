"""Model specifications for the decision-model forward.

A spec is a plain dict (it is also the JSON the C library reads at `vd_open`):

decoder keys (letter families, `executor/torch_exec.py:2341-2386` loads these
as HF CausalLMs):
    arch="decoder", style in {"qwen3", "gemma"}, hidden, layers, heads,
    kv_heads, head_dim, ffn, vocab, rms_eps, rope_theta, qk_norm, qkv_bias,
    act in {"silu", "gelu_tanh"}, tied, embed_scale, norm_plus_one,
    family in {"letter_branches", "letter_readout"}, label_ids, seed, init_std

encoder keys (marker-head family, `convert/marker_head/marker_head_converter.py:19-57`):
    arch="encoder", style in {"bert", "xlmr"}, hidden, layers, heads, ffn,
    vocab, max_pos, type_vocab, ln_eps, pad_id, head_layers, family="marker_head",
    seed, init_std

Presets follow the five benchmark shapes: a BERT-base and an XLM-R-base marker-head
encoder, a Gemma-2B-shaped decider, and OneJev-9B / OneJev-27B-shaped decoders.
"""

from __future__ import annotations

import copy

# Option-label widths of the two letter families: letter_readout fills 255
# single-token labels (`executor/torch_exec.py:26`, MAX_LETTERS), letter_branches
# 26 letters + pairs = 256 slots (`src/family/letter_branches.rs:24`, MAX_SLOTS).
FAMILY_WIDTH = {"letter_readout": 255, "letter_branches": 256}

_DECODER_BASE = dict(
    arch="decoder", style="qwen3", rms_eps=1e-6, rope_theta=1e6, qk_norm=True,
    qkv_bias=False, act="silu", tied=False, embed_scale=False, norm_plus_one=False,
    family="letter_branches", seed=20261201, init_std=0.02, label_ids=None,
)

_ENCODER_BASE = dict(
    arch="encoder", style="bert", max_pos=512, type_vocab=2, ln_eps=1e-12,
    pad_id=0, head_layers=2, family="marker_head", seed=20261201, init_std=0.02,
)

PRESETS = {
    # OneJev-9B-shaped text decision model
    "onejev-9b": dict(_DECODER_BASE, hidden=4096, layers=40, heads=32, kv_heads=8,
                      head_dim=128, ffn=12288, vocab=152064),
    # OneJev-27B-shaped text decision model
    "onejev-27b": dict(_DECODER_BASE, hidden=5120, layers=64, heads=40, kv_heads=8,
                       head_dim=128, ffn=21504, vocab=152064),
    # Gemma-2B-shaped decider (letter readout, tied head, MQA hd=256, GeGLU)
    "decider-2b": dict(_DECODER_BASE, style="gemma", hidden=2048, layers=18, heads=8,
                       kv_heads=1, head_dim=256, ffn=16384, vocab=256000,
                       rope_theta=1e4, qk_norm=False, act="gelu_tanh", tied=True,
                       embed_scale=True, norm_plus_one=True, family="letter_readout"),
    # BERT-base-shaped marker-head encoder (laya)
    "laya-bert": dict(_ENCODER_BASE, style="bert", hidden=768, layers=12, heads=12,
                      ffn=3072, vocab=30522, pad_id=0),
    # XLM-R-base-shaped marker-head encoder (laya-multilingual)
    "laya-xlmr": dict(_ENCODER_BASE, style="xlmr", hidden=768, layers=12, heads=12,
                      ffn=3072, vocab=250002, max_pos=514, type_vocab=1, ln_eps=1e-5,
                      pad_id=1),
}


def preset(name: str, **overrides) -> dict:
    """A copy of a preset with keyword overrides (e.g. layers=2 for a parity case)."""
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    spec = copy.deepcopy(PRESETS[name])
    spec.update(overrides)
    spec["preset"] = name
    return spec


def label_width(spec: dict) -> int:
    return FAMILY_WIDTH[spec["family"]]


def qkv_width(spec: dict) -> int:
    return (spec["heads"] + 2 * spec["kv_heads"]) * spec["head_dim"]


def linear_flops_per_token(spec: dict) -> float:
    """Multiply-add FLOPs (2 per MAC) of every projection GEMM for one token."""
    d, f = spec["hidden"], spec["ffn"]
    if spec["arch"] == "decoder":
        per_layer = d * qkv_width(spec) + spec["heads"] * spec["head_dim"] * d + 3 * d * f
    else:
        per_layer = 4 * d * d + 2 * d * f
    return 2.0 * per_layer * spec["layers"]


def attention_flops(spec: dict, n: int) -> float:
    """QK^T + PV FLOPs of one sequence of n tokens (causal counts n(n+1)/2 pairs)."""
    hd, h = spec["head_dim"] if spec["arch"] == "decoder" else spec["hidden"] // spec["heads"], spec["heads"]
    pairs = n * (n + 1) / 2 if spec["arch"] == "decoder" else float(n * n)
    return 4.0 * hd * h * pairs * spec["layers"]


def weight_bytes(spec: dict) -> float:
    """Bytes of bf16 projection weights read by one forward (embedding rows excluded)."""
    return linear_flops_per_token(spec) / 2.0 * 2.0
