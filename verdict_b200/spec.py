"""Model specifications for the decision-model forward.

A spec is a plain dict (it is also the JSON the C library reads at `vd_open`):

decoder keys (letter families, `executor/torch_exec.py:2341-2386` loads these
as HF CausalLMs):
    arch="decoder", style in {"qwen3", "gemma"}, hidden, layers, heads,
    kv_heads, head_dim, ffn, vocab, rms_eps, rope_theta, qk_norm, qkv_bias,
    act in {"silu", "gelu_tanh"}, tied, embed_scale, norm_plus_one,
    family in {"letter_branches", "letter_readout"}, label_ids, seed, init_std

hybrid decoder keys (style "qwen3_5": HF Qwen3.5 text stacks, gated-delta-net
linear-attention layers with a full-attention layer every few; loaded by the
same executor path as any CausalLM):
    the decoder keys above (heads / kv_heads / head_dim describe the full-
    attention layers, whose q_proj also yields a sigmoid output gate), plus
    layer_types (list of "linear_attention" / "full_attention"),
    partial_rotary (rotary fraction of head_dim), lin_k_heads, lin_v_heads,
    lin_k_dim, lin_v_dim, conv_kernel

independent-options encoder keys (style "modernbert", family
"independent_options": a ModernBERT encoder with option-masked attention and a
per-marker scorer, the ORT graph of `convert/independent_options/`):
    arch="encoder", hidden, layers, heads, ffn, vocab, max_pos, ln_eps, pad_id,
    layer_types ("full_attention" / "sliding_attention"), global_theta,
    local_theta, sliding_window (half-window in option-invariant positions)

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

def hybrid_layer_types(layers: int, full_attention_interval: int = 4) -> list:
    """Qwen3.5's default layer pattern: every `interval`-th layer full attention."""
    return ["linear_attention" if (i + 1) % full_attention_interval else "full_attention" for i in range(layers)]


_HYBRID_BASE = dict(
    _DECODER_BASE, style="qwen3_5", qk_norm=True, norm_plus_one=True, rope_theta=1e7,
    partial_rotary=0.25, conv_kernel=4, lin_k_heads=16, lin_v_heads=32, lin_k_dim=128, lin_v_dim=128,
)

_VON_BASE = dict(
    arch="encoder", style="modernbert", family="independent_options", max_pos=8192, ln_eps=1e-5,
    pad_id=50283, head_layers=0, type_vocab=0, global_theta=160000.0, local_theta=10000.0,
    sliding_window=64, seed=20261201, init_std=0.02,
)


def modernbert_layer_types(layers: int, global_every: int = 3) -> list:
    """ModernBERT's default pattern: every `global_every`-th layer (from 0) full attention."""
    return ["sliding_attention" if i % global_every else "full_attention" for i in range(layers)]


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
    # OneJev1.6-9B-shaped hybrid (Qwen3.5 text stack: 24 gated-delta-net + 8 gated
    # full-attention layers; the shape of transformers' Qwen3_5TextConfig defaults)
    "onejev16-9b": dict(_HYBRID_BASE, hidden=4096, layers=32, heads=16, kv_heads=4, head_dim=256,
                        ffn=12288, vocab=248320, layer_types=hybrid_layer_types(32)),
    # ModernBERT-base-shaped independent-options encoder (von): 22 layers, every
    # third global, the rest sliding-window; option-masked attention
    "von-base": dict(_VON_BASE, hidden=768, layers=22, heads=12, ffn=1152, vocab=50368,
                     layer_types=modernbert_layer_types(22)),
    # BERT-base-shaped marker-head encoder (laya)
    "laya-bert": dict(_ENCODER_BASE, style="bert", hidden=768, layers=12, heads=12,
                      ffn=3072, vocab=30522, pad_id=0),
    # XLM-R-base-shaped marker-head encoder (laya-multilingual)
    "laya-xlmr": dict(_ENCODER_BASE, style="xlmr", hidden=768, layers=12, heads=12,
                      ffn=3072, vocab=250002, max_pos=514, type_vocab=1, ln_eps=1e-5,
                      pad_id=1),
}


def preset(name: str, **overrides) -> dict:
    """A copy of a preset with keyword overrides (e.g. layers=2 for a parity case).
    For hybrid presets a `layers` override without `layer_types` keeps the
    preset's pattern (every 4th layer full attention, the last one included
    when `layers` is a multiple of 4)."""
    if name not in PRESETS:
        raise KeyError(f"unknown model preset {name!r}; known: {sorted(PRESETS)}")
    spec = copy.deepcopy(PRESETS[name])
    spec.update(overrides)
    if spec.get("style") == "qwen3_5" and "layers" in overrides and "layer_types" not in overrides:
        spec["layer_types"] = hybrid_layer_types(spec["layers"])
    if spec.get("style") == "modernbert" and "layers" in overrides and "layer_types" not in overrides:
        spec["layer_types"] = modernbert_layer_types(spec["layers"])
    spec["preset"] = name
    return spec


def is_hybrid(spec: dict) -> bool:
    return spec.get("style") == "qwen3_5"


def full_attention_layers(spec: dict) -> list:
    if not is_hybrid(spec):
        return list(range(spec["layers"]))
    return [i for i, t in enumerate(spec["layer_types"]) if t == "full_attention"]


def rotary_dim(spec: dict) -> int:
    return int(spec["head_dim"] * spec.get("partial_rotary", 1.0))


def label_width(spec: dict) -> int:
    return FAMILY_WIDTH[spec["family"]]


def qkv_width(spec: dict) -> int:
    """Columns of the fused full-attention projection (q, k, v; plus the output
    gate of a hybrid's gated attention)."""
    gate = spec["heads"] if is_hybrid(spec) else 0
    return (spec["heads"] + 2 * spec["kv_heads"] + gate) * spec["head_dim"]


def gdn_dims(spec: dict) -> dict:
    """Gated-delta-net sizes: key/value widths, conv channels, in_proj columns."""
    kd = spec["lin_k_heads"] * spec["lin_k_dim"]
    vd = spec["lin_v_heads"] * spec["lin_v_dim"]
    conv = 2 * kd + vd
    return dict(kd=kd, vd=vd, conv=conv, proj=conv + vd + 2 * spec["lin_v_heads"])


def linear_flops_per_token(spec: dict) -> float:
    """Multiply-add FLOPs (2 per MAC) of every projection GEMM for one token."""
    d, f = spec["hidden"], spec["ffn"]
    if spec.get("style") == "modernbert":
        return 2.0 * (4 * d * d + 3 * d * f) * spec["layers"]
    if spec["arch"] == "decoder":
        full = d * qkv_width(spec) + spec["heads"] * spec["head_dim"] * d + 3 * d * f
        if not is_hybrid(spec):
            return 2.0 * full * spec["layers"]
        g = gdn_dims(spec)
        lin = d * g["proj"] + g["vd"] * d + 3 * d * f
        n_full = len(full_attention_layers(spec))
        return 2.0 * (full * n_full + lin * (spec["layers"] - n_full))
    per_layer = 4 * d * d + 2 * d * f
    return 2.0 * per_layer * spec["layers"]


def attention_flops(spec: dict, n: int) -> float:
    """QK^T + PV FLOPs of one sequence of n tokens (causal counts n(n+1)/2 pairs)."""
    hd, h = spec["head_dim"] if spec["arch"] == "decoder" else spec["hidden"] // spec["heads"], spec["heads"]
    pairs = n * (n + 1) / 2 if spec["arch"] == "decoder" else float(n * n)
    layers = len(full_attention_layers(spec)) if spec["arch"] == "decoder" else spec["layers"]
    return 4.0 * hd * h * pairs * layers


def weight_bytes(spec: dict) -> float:
    """Bytes of bf16 projection weights read by one forward (embedding rows excluded)."""
    return linear_flops_per_token(spec) / 2.0 * 2.0
