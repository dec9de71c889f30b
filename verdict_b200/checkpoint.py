"""Specs for real checkpoints, and synthetic checkpoints written as safetensors.

`spec_from_checkpoint(path)` reads what the reference's executors load and
returns a model spec whose "checkpoint" key points at it; `vd_open` then reads
the weights from the safetensors files by state-dict name:
- a decoder (letter families): an HF CausalLM directory, `config.json` plus
  `model.safetensors` or shards with `model.safetensors.index.json`
  (`executor/torch_exec.py:2341-2386`, checked by `src/torch_engine.rs:297-310`);
  the option-label table comes from its tokenizer by the family's rule
  (`derive_branch_ids` / `derive_letter_ids`, `executor/torch_exec.py:2379-2383`);
- a marker-head encoder: a `DecisionModel` state dict in `model.safetensors`
  with the encoder's HF config in `encoder/config.json` (or beside it)
  (`convert/marker_head/marker_head_converter.py:113-126`).

`save_synthetic(spec, out_dir)` writes the seeded synthetic weights of a spec
in that same layout (HF config, safetensors, optional shards), so that the
reader can be checked bit for bit against the on-device generator and that HF
itself can load the files.
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np

from . import labels, synth

_DTYPES = ("BF16", "F16", "F32")


# ---------------------------------------------------------------------------
# Reading configs
# ---------------------------------------------------------------------------

def _rope_theta(cfg: dict) -> float:
    rp = cfg.get("rope_parameters") or {}
    theta = cfg.get("rope_theta") or rp.get("rope_theta")
    scaling = cfg.get("rope_scaling") or None
    rtype = (rp.get("rope_type") or "default") if rp else "default"
    if scaling or rtype != "default":
        raise ValueError("rope scaling is not supported (the checkpoint uses "
                         f"{scaling or rtype!r})")
    return float(theta if theta is not None else 10000.0)


def hybrid_spec_from_config(cfg: dict) -> dict:
    """The spec keys of an HF Qwen3.5 text stack (`qwen3_5_text`, or the
    `text_config` of a `qwen3_5` vision-language checkpoint).  Multimodal RoPE
    sections are accepted: with text-only positions every section sees the same
    position, which is plain RoPE over the rotary width."""
    c = cfg.get("text_config") or cfg if cfg.get("model_type") == "qwen3_5" else cfg
    rp = c.get("rope_parameters") or {}
    if (rp.get("rope_type") or "default") != "default" or c.get("rope_scaling"):
        raise ValueError("rope scaling is not supported")
    theta = rp.get("rope_theta") or c.get("rope_theta") or 10000.0
    partial = rp.get("partial_rotary_factor", c.get("partial_rotary_factor", 0.25))
    if c.get("attention_bias"):
        raise ValueError("qwen3_5 checkpoints with attention bias are not supported")
    layers = int(c["num_hidden_layers"])
    types = c.get("layer_types")
    if not types:
        from .spec import hybrid_layer_types
        types = hybrid_layer_types(layers, int(c.get("full_attention_interval", 4)))
    act = c.get("hidden_act", "silu")
    if act not in ("silu", "swish"):
        raise ValueError(f"unsupported qwen3_5 activation {act!r}")
    heads = int(c["num_attention_heads"])
    return dict(
        arch="decoder", style="qwen3_5", hidden=int(c["hidden_size"]), layers=layers, heads=heads,
        kv_heads=int(c.get("num_key_value_heads") or heads), head_dim=int(c.get("head_dim") or 256),
        ffn=int(c["intermediate_size"]), vocab=int(c["vocab_size"]), rms_eps=float(c.get("rms_norm_eps", 1e-6)),
        rope_theta=float(theta), partial_rotary=float(partial),
        tied=bool(c.get("tie_word_embeddings", cfg.get("tie_word_embeddings", False))),
        qk_norm=True, qkv_bias=False, act="silu", embed_scale=False, norm_plus_one=True,
        layer_types=list(types), lin_k_heads=int(c["linear_num_key_heads"]),
        lin_v_heads=int(c["linear_num_value_heads"]), lin_k_dim=int(c.get("linear_key_head_dim", 128)),
        lin_v_dim=int(c.get("linear_value_head_dim", 128)), conv_kernel=int(c.get("linear_conv_kernel_dim", 4)),
    )


def decoder_spec_from_config(cfg: dict) -> dict:
    """The decoder spec keys of an HF Qwen3 / Qwen2 / Gemma / Qwen3.5 config dict."""
    mt = cfg.get("model_type")
    if mt in ("qwen3_5", "qwen3_5_text"):
        return hybrid_spec_from_config(cfg)
    if mt not in ("qwen3", "qwen2", "gemma"):
        raise ValueError(f"unsupported decoder model_type {mt!r} (qwen3, qwen2 and gemma are supported)")
    heads = int(cfg["num_attention_heads"])
    hidden = int(cfg["hidden_size"])
    spec = dict(
        arch="decoder", style=mt, hidden=hidden, layers=int(cfg["num_hidden_layers"]), heads=heads,
        kv_heads=int(cfg.get("num_key_value_heads") or heads),
        head_dim=int(cfg.get("head_dim") or hidden // heads),
        ffn=int(cfg["intermediate_size"]), vocab=int(cfg["vocab_size"]),
        rms_eps=float(cfg.get("rms_norm_eps", 1e-6)), rope_theta=_rope_theta(cfg),
        tied=bool(cfg.get("tie_word_embeddings", mt == "gemma")),
    )
    if mt == "qwen3":
        if cfg.get("attention_bias"):
            raise ValueError("qwen3 checkpoints with attention_bias (o_proj bias) are not supported")
        spec.update(qk_norm=True, qkv_bias=False, act="silu", embed_scale=False, norm_plus_one=False)
    elif mt == "qwen2":
        spec.update(qk_norm=False, qkv_bias=True, act="silu", embed_scale=False, norm_plus_one=False)
    else:
        spec.update(qk_norm=False, qkv_bias=False, act="gelu_tanh", embed_scale=True, norm_plus_one=True)
    act = cfg.get("hidden_activation") or cfg.get("hidden_act")
    want = {"silu": ("silu", "swish"), "gelu_tanh": ("gelu_pytorch_tanh", "gelu_tanh")}[spec["act"]]
    if act not in want:
        raise ValueError(f"unsupported {mt} activation {act!r}")
    if cfg.get("use_sliding_window"):
        raise ValueError("sliding-window attention is not supported")
    return spec


def encoder_spec_from_config(cfg: dict, head_layers: int = 2) -> dict:
    """The encoder spec keys of an HF BERT / XLM-R config dict."""
    mt = cfg.get("model_type")
    styles = {"bert": "bert", "xlm-roberta": "xlmr"}
    if mt not in styles:
        raise ValueError(f"unsupported encoder model_type {mt!r} (bert and xlm-roberta are supported)")
    if cfg.get("position_embedding_type", "absolute") not in (None, "absolute"):
        raise ValueError("only absolute position embeddings are supported")
    if cfg.get("hidden_act", "gelu") != "gelu":
        raise ValueError(f"unsupported encoder activation {cfg.get('hidden_act')!r}")
    return dict(
        arch="encoder", style=styles[mt], hidden=int(cfg["hidden_size"]), layers=int(cfg["num_hidden_layers"]),
        heads=int(cfg["num_attention_heads"]), ffn=int(cfg["intermediate_size"]), vocab=int(cfg["vocab_size"]),
        max_pos=int(cfg["max_position_embeddings"]), type_vocab=int(cfg.get("type_vocab_size", 2)),
        ln_eps=float(cfg.get("layer_norm_eps", 1e-12)), pad_id=int(cfg.get("pad_token_id", 0) or 0),
        head_layers=int(head_layers), family="marker_head",
    )


def von_spec_from_config(cfg: dict) -> dict:
    """The spec keys of an independent-options model's ModernBERT encoder config."""
    if cfg.get("norm_bias") or cfg.get("attention_bias") or cfg.get("mlp_bias"):
        raise ValueError("modernbert checkpoints with norm / attention / MLP biases are not supported")
    if cfg.get("hidden_activation", "gelu") != "gelu":
        raise ValueError(f"unsupported modernbert activation {cfg.get('hidden_activation')!r}")
    rp = cfg.get("rope_parameters") or {}
    g = (rp.get("full_attention") or {}).get("rope_theta", cfg.get("global_rope_theta", 160000.0))
    l = (rp.get("sliding_attention") or {}).get("rope_theta", cfg.get("local_rope_theta", 10000.0))
    layers = int(cfg["num_hidden_layers"])
    types = cfg.get("layer_types")
    if not types:
        from .spec import modernbert_layer_types
        types = modernbert_layer_types(layers, int(cfg.get("global_attn_every_n_layers", 3)))
    return dict(
        arch="encoder", style="modernbert", family="independent_options", hidden=int(cfg["hidden_size"]),
        layers=layers, heads=int(cfg["num_attention_heads"]), ffn=int(cfg["intermediate_size"]),
        vocab=int(cfg["vocab_size"]), max_pos=int(cfg.get("max_position_embeddings", 8192)),
        ln_eps=float(cfg.get("norm_eps", 1e-5)), pad_id=int(cfg.get("pad_token_id") or 0), head_layers=0,
        type_vocab=0, global_theta=float(g), local_theta=float(l),
        sliding_window=int(cfg.get("local_attention", 128)) // 2, layer_types=list(types))


def _load_tokenizer(path: str):
    from transformers import AutoTokenizer
    tok_dir = os.path.join(path, "tokenizer")
    return AutoTokenizer.from_pretrained(
        tok_dir if os.path.isfile(os.path.join(tok_dir, "tokenizer.json")) else path)


def has_weights(path: str) -> bool:
    return os.path.isfile(os.path.join(path, "model.safetensors")) or os.path.isfile(
        os.path.join(path, "model.safetensors.index.json"))


def spec_from_checkpoint(path: str, *, family: str | None = None, label_ids=None, tokenizer=None,
                         manifest: dict | None = None, head_layers: int | None = None) -> dict:
    """A spec for the checkpoint at `path`, with "checkpoint" set to its absolute path.

    Decoders: the family is `family`, else `manifest["family"]`, else
    "letter_readout" (the torch executor's default); the label table is
    `label_ids`, else derived from `tokenizer` (default: the checkpoint's own,
    loaded with transformers).  Encoders: `head_layers` (the converter
    config's key) defaults to 2."""
    path = os.path.abspath(path)
    if not has_weights(path):
        raise FileNotFoundError(f"no model.safetensors or model.safetensors.index.json in {path}")
    enc_cfg = os.path.join(path, "encoder", "config.json")
    cfg_path = enc_cfg if os.path.isfile(enc_cfg) else os.path.join(path, "config.json")
    with open(cfg_path) as f:
        cfg = json.load(f)
    if cfg.get("model_type") == "modernbert":
        spec = von_spec_from_config(cfg)
    elif cfg.get("model_type") in ("bert", "xlm-roberta"):
        spec = encoder_spec_from_config(cfg, 2 if head_layers is None else head_layers)
    else:
        spec = decoder_spec_from_config(cfg)
        fam = family or (manifest or {}).get("family") or "letter_readout"
        fam = fam.replace("-", "_")
        if fam not in ("letter_readout", "letter_branches"):
            raise ValueError(f"decoder family must be letter_readout or letter_branches, not {fam!r}")
        spec["family"] = fam
        if label_ids is None:
            label_ids = labels.derive_label_ids(fam, tokenizer if tokenizer is not None else _load_tokenizer(path))
        spec["label_ids"] = [int(i) for i in label_ids]
    spec.update(checkpoint=path, seed=0, init_std=0.02)
    return spec


def resolve_spec(model) -> dict:
    """The spec the C library would load for `model` (a spec dict, a JSON
    string, or a directory holding vdexec.json), as it resolves it."""
    import ctypes
    from . import _abi
    if isinstance(model, dict):
        model = json.dumps(model)
    lib = _abi.load()
    err = ctypes.create_string_buffer(1024)
    out = ctypes.create_string_buffer(1 << 20)
    rc = lib.vd_resolve_spec(os.fspath(model).encode(), out, len(out), err, len(err))
    _abi.check(rc, err)
    return json.loads(out.value.decode())


# ---------------------------------------------------------------------------
# Writing safetensors
# ---------------------------------------------------------------------------

def _encode(arr: np.ndarray, dtype: str) -> bytes:
    a = np.ascontiguousarray(arr, dtype=np.float32)
    if dtype == "F32":
        return a.astype("<f4").tobytes()
    if dtype == "F16":
        return a.astype("<f2").tobytes()
    if dtype == "BF16":
        # The synthetic values are bf16 already: the upper half of the fp32 bits is exact.
        return (a.view(np.uint32) >> np.uint32(16)).astype("<u2").tobytes()
    raise ValueError(f"dtype must be one of {_DTYPES}")


def write_safetensors(path: str, tensors) -> int:
    """Write [(name, fp32 array, dtype)] as one safetensors file; returns its data bytes."""
    blobs, header, off = [], {}, 0
    for name, arr, dtype in tensors:
        b = _encode(arr, dtype)
        header[name] = {"dtype": dtype, "shape": [int(s) for s in np.shape(arr)], "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * (-len(h) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)))
        f.write(h)
        for b in blobs:
            f.write(b)
    return off


def _hf_config(spec: dict) -> dict:
    if spec["arch"] == "decoder" and spec["style"] == "qwen3_5":
        return dict(
            model_type="qwen3_5_text", architectures=["Qwen3_5ForCausalLM"], hidden_size=spec["hidden"],
            num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
            num_key_value_heads=spec["kv_heads"], head_dim=spec["head_dim"], intermediate_size=spec["ffn"],
            vocab_size=spec["vocab"], rms_norm_eps=spec["rms_eps"], tie_word_embeddings=spec["tied"],
            hidden_act="silu", attention_bias=False, layer_types=list(spec["layer_types"]),
            linear_num_key_heads=spec["lin_k_heads"], linear_num_value_heads=spec["lin_v_heads"],
            linear_key_head_dim=spec["lin_k_dim"], linear_value_head_dim=spec["lin_v_dim"],
            linear_conv_kernel_dim=spec["conv_kernel"], max_position_embeddings=32768,
            rope_parameters={"rope_type": "default", "rope_theta": spec["rope_theta"],
                             "partial_rotary_factor": spec["partial_rotary"]},
            torch_dtype="bfloat16")
    if spec["arch"] == "decoder":
        cfg = dict(
            model_type=spec["style"], hidden_size=spec["hidden"], num_hidden_layers=spec["layers"],
            num_attention_heads=spec["heads"], num_key_value_heads=spec["kv_heads"], head_dim=spec["head_dim"],
            intermediate_size=spec["ffn"], vocab_size=spec["vocab"], rms_norm_eps=spec["rms_eps"],
            rope_theta=spec["rope_theta"], tie_word_embeddings=spec["tied"], max_position_embeddings=32768,
            torch_dtype="bfloat16",
        )
        cfg["architectures"] = [{"qwen3": "Qwen3ForCausalLM", "qwen2": "Qwen2ForCausalLM",
                                 "gemma": "GemmaForCausalLM"}[spec["style"]]]
        if spec["style"] == "gemma":
            cfg["hidden_act"] = cfg["hidden_activation"] = "gelu_pytorch_tanh"
        else:
            cfg["hidden_act"] = "silu"
            cfg["attention_bias"] = bool(spec["qkv_bias"]) if spec["style"] == "qwen3" else None
            if cfg["attention_bias"] is None:
                del cfg["attention_bias"]
        return cfg
    if spec["style"] == "modernbert":
        return dict(
            model_type="modernbert", architectures=["ModernBertModel"], hidden_size=spec["hidden"],
            num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"], intermediate_size=spec["ffn"],
            vocab_size=spec["vocab"], max_position_embeddings=spec["max_pos"], norm_eps=spec["ln_eps"],
            norm_bias=False, attention_bias=False, mlp_bias=False, hidden_activation="gelu",
            pad_token_id=spec["pad_id"], layer_types=list(spec["layer_types"]),
            local_attention=2 * spec["sliding_window"],
            rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": spec["global_theta"]},
                             "sliding_attention": {"rope_type": "default", "rope_theta": spec["local_theta"]}})
    return dict(
        model_type="bert" if spec["style"] == "bert" else "xlm-roberta", hidden_size=spec["hidden"],
        num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"], intermediate_size=spec["ffn"],
        vocab_size=spec["vocab"], max_position_embeddings=spec["max_pos"], type_vocab_size=spec["type_vocab"],
        layer_norm_eps=spec["ln_eps"], pad_token_id=spec["pad_id"], hidden_act="gelu",
        position_embedding_type="absolute",
        architectures=["BertModel" if spec["style"] == "bert" else "XLMRobertaModel"],
    )


def save_synthetic(spec: dict, out_dir: str, *, dtype: str = "BF16", dtypes: dict | None = None,
                   shard_bytes: int | None = None, write_spec: bool = False, gen=None) -> str:
    """Write the synthetic weights of `spec` as an HF-layout safetensors checkpoint.

    `dtypes` overrides the dtype per tensor name; `shard_bytes` splits the
    tensors into `model-0000i-of-0000n.safetensors` files with an index;
    `write_spec` also writes `vdexec.json` (the spec with "checkpoint": ".") so
    that `vd_open(out_dir)` opens it; `gen(seed, name, shape, scale, offset)`
    replaces the numpy generator.  Returns `out_dir`."""
    gen = gen or synth.gen_tensor
    os.makedirs(out_dir, exist_ok=True)
    table = [(name, shape, (dtypes or {}).get(name, dtype), scale, off)
             for name, shape, scale, off in synth.tensor_table(spec)]
    for _, _, dt, _, _ in table:
        if dt not in _DTYPES:
            raise ValueError(f"dtype must be one of {_DTYPES}, not {dt!r}")
    groups, cur, cur_bytes = [], [], 0
    for row in table:
        nbytes = int(np.prod(row[1])) * (4 if row[2] == "F32" else 2)
        if shard_bytes and cur and cur_bytes + nbytes > shard_bytes:
            groups.append(cur)
            cur, cur_bytes = [], 0
        cur.append(row)
        cur_bytes += nbytes
    groups.append(cur)
    weight_map, total = {}, 0
    for gi, group in enumerate(groups):
        fname = "model.safetensors" if len(groups) == 1 else f"model-{gi + 1:05d}-of-{len(groups):05d}.safetensors"
        tensors = [(name, gen(spec["seed"], name, shape, scale, off), dt) for name, shape, dt, scale, off in group]
        total += write_safetensors(os.path.join(out_dir, fname), tensors)
        weight_map.update({name: fname for name, *_ in group})
    if len(groups) > 1:
        with open(os.path.join(out_dir, "model.safetensors.index.json"), "w") as f:
            json.dump({"metadata": {"total_size": total}, "weight_map": weight_map}, f, indent=1)
    cfg_dir = out_dir if spec["arch"] == "decoder" else os.path.join(out_dir, "encoder")
    os.makedirs(cfg_dir, exist_ok=True)
    with open(os.path.join(cfg_dir, "config.json"), "w") as f:
        json.dump(_hf_config(spec), f, indent=1)
    if write_spec:
        s = {k: v for k, v in spec.items() if k != "preset"}
        s["checkpoint"] = "."
        with open(os.path.join(out_dir, "vdexec.json"), "w") as f:
            json.dump(s, f)
    return out_dir
