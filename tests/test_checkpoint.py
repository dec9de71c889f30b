"""Safetensors checkpoints on the host: the synthetic writer against the
safetensors library and HF's own loaders, config -> spec mapping, and the C
reader's header checks (which run before any device work, so on CPU too)."""

import ctypes
import json
import os
import struct

import numpy as np
import pytest

torch = pytest.importorskip("torch")
safetensors_torch = pytest.importorskip("safetensors.torch")

from verdict_b200 import _abi  # noqa: E402
from verdict_b200 import checkpoint as ck  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.synth import gen_tensor, tensor_table, with_labels  # noqa: E402

# Small shapes the GPU path also accepts (head_dim 128 / 256, multiples of 128).
TINY = {
    "qwen3": dict(hidden=256, layers=2, heads=2, kv_heads=1, head_dim=128, ffn=512, vocab=1024),
    "qwen2": dict(style="qwen2", qk_norm=False, qkv_bias=True, hidden=256, layers=2, heads=2, kv_heads=1,
                  head_dim=128, ffn=512, vocab=1024),
}


def tiny_decoder(kind="qwen3", **over):
    return with_labels(specs.preset("onejev-9b", **dict(TINY[kind], **over)))


def tiny_gemma(**over):
    return with_labels(specs.preset("decider-2b", **dict(dict(hidden=256, layers=2, heads=2, kv_heads=1,
                                                                   head_dim=256, ffn=512, vocab=1024), **over)))


def tiny_hybrid(**over):
    return with_labels(specs.preset("onejev16-9b", **dict(dict(hidden=256, layers=4, heads=2, kv_heads=1, head_dim=256,
                                                                ffn=512, vocab=1024, lin_k_heads=2, lin_v_heads=4),
                                                           **over)))


def tiny_encoder(preset="laya-bert", **over):
    return specs.preset(preset, **dict(dict(hidden=256, layers=2, heads=4, ffn=512, vocab=2048), **over))


def load_all(d):
    out = {}
    for f in sorted(os.listdir(d)):
        if f.endswith(".safetensors"):
            out.update(safetensors_torch.load_file(os.path.join(d, f)))
    return out


def test_writer_matches_the_generator_through_the_safetensors_library(tmp_path):
    spec = tiny_decoder()
    ck.save_synthetic(spec, str(tmp_path), dtypes={"model.layers.0.self_attn.q_proj.weight": "F32",
                                                   "model.norm.weight": "F16"})
    got = load_all(str(tmp_path))
    names = [n for n, *_ in tensor_table(spec)]
    assert sorted(got) == sorted(names)
    assert got["model.layers.0.self_attn.q_proj.weight"].dtype == torch.float32
    assert got["model.norm.weight"].dtype == torch.float16
    assert got["model.embed_tokens.weight"].dtype == torch.bfloat16
    for name, shape, scale, off in tensor_table(spec):
        want = gen_tensor(spec["seed"], name, shape, scale, off)
        np.testing.assert_array_equal(got[name].float().numpy(), want.astype(np.float16).astype(np.float32)
                                      if name == "model.norm.weight" else want)


def test_sharded_writer_and_index(tmp_path):
    spec = tiny_decoder()
    ck.save_synthetic(spec, str(tmp_path), shard_bytes=600_000)
    with open(tmp_path / "model.safetensors.index.json") as f:
        index = json.load(f)
    files = sorted(set(index["weight_map"].values()))
    assert len(files) >= 3 and not (tmp_path / "model.safetensors").exists()
    assert sorted(index["weight_map"]) == sorted(n for n, *_ in tensor_table(spec))
    assert sorted(load_all(str(tmp_path))) == sorted(index["weight_map"])
    assert ck.has_weights(str(tmp_path))


@pytest.mark.parametrize("make", [tiny_decoder, lambda: tiny_decoder("qwen2"), tiny_gemma, tiny_hybrid])
def test_hf_loads_the_written_decoder_with_no_missing_or_extra_tensors(tmp_path, make):
    from transformers import AutoModelForCausalLM
    spec = make()
    ck.save_synthetic(spec, str(tmp_path))
    model, info = AutoModelForCausalLM.from_pretrained(str(tmp_path), output_loading_info=True,
                                                       dtype=torch.float32)
    assert not info["missing_keys"] and not info["unexpected_keys"], info
    sd = model.state_dict()
    name = "model.layers.1.mlp.up_proj.weight"  # (every layer type has an MLP)
    shape = tuple(sd[name].shape)
    want = gen_tensor(spec["seed"], name, shape, spec["init_std"] * 3 ** 0.5, 0.0)
    np.testing.assert_array_equal(sd[name].numpy(), want)


@pytest.mark.parametrize("make", [tiny_decoder, lambda: tiny_decoder("qwen2"), tiny_gemma, tiny_hybrid])
def test_spec_from_checkpoint_round_trips_the_config(tmp_path, make):
    spec = make()
    ck.save_synthetic(spec, str(tmp_path))
    got = ck.spec_from_checkpoint(str(tmp_path), family=spec["family"], label_ids=spec["label_ids"])
    for k in ("arch", "style", "hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab", "rms_eps",
              "rope_theta", "qk_norm", "qkv_bias", "act", "tied", "embed_scale", "norm_plus_one", "family",
              "label_ids"):
        assert got[k] == spec[k], k
    assert got["checkpoint"] == str(tmp_path)


def test_spec_from_checkpoint_derives_labels_from_a_tokenizer(tmp_path):
    spec = tiny_decoder()
    ck.save_synthetic(spec, str(tmp_path))

    class Tok:  # every label is its own single token
        vocab = {}

        def encode(self, text, add_special_tokens=False):
            return [self.vocab.setdefault(text, 10 + len(self.vocab))]

        def decode(self, ids):
            inv = {v: k for k, v in self.vocab.items()}
            return "".join(inv[i] for i in ids)

    got = ck.spec_from_checkpoint(str(tmp_path), manifest={"family": "letter-branches"}, tokenizer=Tok())
    assert got["family"] == "letter_branches" and len(got["label_ids"]) == 256
    got = ck.spec_from_checkpoint(str(tmp_path), tokenizer=Tok())
    assert got["family"] == "letter_readout" and len(got["label_ids"]) == 255


@pytest.mark.parametrize("preset,model_cls", [("laya-bert", "BertModel"), ("laya-xlmr", "XLMRobertaModel")])
def test_encoder_checkpoint_names_and_config(tmp_path, preset, model_cls):
    import transformers
    spec = tiny_encoder(preset)
    ck.save_synthetic(spec, str(tmp_path))
    got = ck.spec_from_checkpoint(str(tmp_path), head_layers=spec["head_layers"])
    for k in ("arch", "style", "hidden", "layers", "heads", "ffn", "vocab", "max_pos", "type_vocab", "ln_eps",
              "pad_id", "head_layers"):
        assert got[k] == spec[k], k
    cfg = transformers.AutoConfig.from_pretrained(str(tmp_path / "encoder"))
    enc = getattr(transformers, model_cls)(cfg, add_pooling_layer=False)
    want = {"encoder." + k for k in enc.state_dict() if not k.endswith("position_ids")}
    have = set(load_all(str(tmp_path)))
    assert want <= have, sorted(want - have)[:5]


def test_unsupported_configs_are_refused():
    base = ck._hf_config(tiny_decoder())
    with pytest.raises(ValueError, match="rope scaling"):
        ck.decoder_spec_from_config(dict(base, rope_scaling={"rope_type": "yarn", "factor": 4.0}))
    with pytest.raises(ValueError, match="attention_bias"):
        ck.decoder_spec_from_config(dict(base, attention_bias=True))
    with pytest.raises(ValueError, match="model_type"):
        ck.decoder_spec_from_config(dict(base, model_type="llama"))
    assert ck.decoder_spec_from_config(dict(base, rope_theta=None, rope_parameters={
        "rope_theta": 5e5, "rope_type": "default"}))["rope_theta"] == 5e5


# --- the C reader: header parsing happens in vd_open before the device -----

def open_rc(spec):
    lib = _abi.load()
    err = ctypes.create_string_buffer(1024)
    h = ctypes.c_void_p()
    rc = lib.vd_open(json.dumps(spec).encode(), 0, None, ctypes.byref(h), err, len(err))
    if h.value:
        lib.vd_close(h)
    return rc, err.value.decode()


def write_raw(path, header: dict, data: bytes):
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + data)


def test_c_reader_rejects_missing_and_malformed_checkpoints(tmp_path):
    spec = tiny_decoder()
    rc, msg = open_rc(dict(spec, checkpoint=str(tmp_path / "nowhere")))
    assert rc == _abi.VD_ESPEC and "cannot open checkpoint directory" in msg
    rc, msg = open_rc(dict(spec, checkpoint=str(tmp_path)))
    assert rc == _abi.VD_ESPEC and "no .safetensors files" in msg

    bad = tmp_path / "bad"
    bad.mkdir()
    with open(bad / "model.safetensors", "wb") as f:
        f.write(struct.pack("<Q", 1 << 40) + b"{}")
    rc, msg = open_rc(dict(spec, checkpoint=str(bad)))
    assert rc == _abi.VD_ESPEC and "bad safetensors header" in msg

    write_raw(bad / "model.safetensors", {"x": {"dtype": "I64", "shape": [2], "data_offsets": [0, 16]}}, bytes(16))
    rc, msg = open_rc(dict(spec, checkpoint=str(bad)))
    assert rc == _abi.VD_ESPEC and "unsupported dtype I64" in msg

    write_raw(bad / "model.safetensors", {"x": {"dtype": "BF16", "shape": [4], "data_offsets": [0, 6]}}, bytes(8))
    rc, msg = open_rc(dict(spec, checkpoint=str(bad)))
    assert rc == _abi.VD_ESPEC and "inconsistent offsets" in msg

    write_raw(bad / "model.safetensors", {"x": {"dtype": "F32", "shape": [4], "data_offsets": [0, 16]}}, bytes(8))
    rc, msg = open_rc(dict(spec, checkpoint=str(bad)))
    assert rc == _abi.VD_ESPEC and "inconsistent offsets" in msg


# --- the C library's HF-config mapping agrees with spec_from_checkpoint ------

SHAPE_KEYS = ("arch", "style", "hidden", "layers", "heads", "kv_heads", "head_dim", "ffn", "vocab", "rms_eps",
              "rope_theta", "qk_norm", "qkv_bias", "act", "tied", "embed_scale", "norm_plus_one", "family")
HYBRID_KEYS = ("layer_types", "partial_rotary", "lin_k_heads", "lin_v_heads", "lin_k_dim", "lin_v_dim", "conv_kernel")


@pytest.mark.parametrize("make", [tiny_decoder, lambda: tiny_decoder("qwen2"), tiny_gemma, tiny_hybrid])
def test_c_library_fills_a_decoder_spec_from_the_hf_config(tmp_path, make):
    spec = make()
    ck.save_synthetic(spec, str(tmp_path))
    py = ck.spec_from_checkpoint(str(tmp_path), family=spec["family"], label_ids=spec["label_ids"])
    c = ck.resolve_spec({"checkpoint": str(tmp_path), "family": spec["family"], "label_ids": spec["label_ids"]})
    for k in SHAPE_KEYS + (HYBRID_KEYS if spec["style"] == "qwen3_5" else ()):
        assert c[k] == py[k] == spec[k], k
    assert c["label_ids"] == spec["label_ids"] and c["checkpoint"] == str(tmp_path)
    # the torch executor's default family when the spec names none
    assert ck.resolve_spec({"checkpoint": str(tmp_path), "label_ids": [1, 2]})["family"] == "letter_readout"


@pytest.mark.parametrize("preset", ["laya-bert", "laya-xlmr"])
def test_c_library_fills_an_encoder_spec_from_the_hf_config(tmp_path, preset):
    spec = tiny_encoder(preset)
    ck.save_synthetic(spec, str(tmp_path))
    py = ck.spec_from_checkpoint(str(tmp_path))
    c = ck.resolve_spec({"checkpoint": str(tmp_path)})
    for k in ("arch", "style", "hidden", "layers", "heads", "ffn", "vocab", "max_pos", "type_vocab", "ln_eps",
              "pad_id", "family"):
        assert c[k] == py[k], k


def test_c_library_resolves_spec_files_and_refuses_unsupported_configs(tmp_path):
    spec = tiny_decoder()
    ck.save_synthetic(spec, str(tmp_path), write_spec=True)
    got = ck.resolve_spec(str(tmp_path))
    assert got["checkpoint"] == str(tmp_path) + "/." and got["hidden"] == spec["hidden"]
    cfg_path = tmp_path / "config.json"
    base = json.loads(cfg_path.read_text())
    for over, msg in [(dict(model_type="llama"), "unsupported model_type"),
                      (dict(rope_scaling={"rope_type": "yarn", "factor": 4.0}), "rope scaling"),
                      (dict(attention_bias=True), "attention_bias"),
                      (dict(hidden_act="relu"), "activation")]:
        cfg_path.write_text(json.dumps(dict(base, **over)))
        with pytest.raises(_abi.VdError, match=msg) as e:
            ck.resolve_spec({"checkpoint": str(tmp_path), "label_ids": [1]})
        assert e.value.code == _abi.VD_ESPEC
    cfg_path.write_text(json.dumps(dict(base, head_dim=96)))
    with pytest.raises(_abi.VdError, match="head_dim"):
        ck.resolve_spec({"checkpoint": str(tmp_path), "label_ids": [1]})
