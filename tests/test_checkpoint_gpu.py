"""Weights read from safetensors checkpoints give the same bits as the same
weights generated on the device: the checkpoint path changes where the
values come from, never what the forward computes."""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.fastsynth import gen_tensor as fast_gen  # noqa: E402
from verdict_b200 import checkpoint as ck  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import Layout, collate, decoder_rows, encoder_rows  # noqa: E402
from verdict_b200.engine import B200Engine  # noqa: E402
from verdict_b200.synth import with_labels  # noqa: E402

pytestmark = pytest.mark.gpu

DEC = dict(hidden=1024, layers=2, heads=8, kv_heads=2, head_dim=128, ffn=2816, vocab=4096, seed=5)


def decoder_batch(spec, seed=3, n=5):
    rng = np.random.default_rng(seed)
    rows = decoder_rows(rng, n, spec["vocab"], lengths="lognormal-9b")
    for r in rows:
        m = min(len(r.ids), 600)
        r.ids, r.markers = r.ids[:m], [m - 1]
    return collate(rows, Layout(pad_id=0))


def outputs(spec, batch, **kw):
    eng = B200Engine(spec, max_tokens=8192, max_rows=64, max_seq=2048, **kw)
    try:
        return np.array([r.logits for r in eng.infer(batch)], dtype=np.float64)
    finally:
        eng.close()


CASES = {
    "qwen3-bf16": (dict(DEC), {}),
    "qwen3-sharded-mixed": (dict(DEC), dict(shard_bytes=8 << 20, dtypes={
        "model.layers.0.self_attn.q_proj.weight": "F32", "model.layers.1.mlp.gate_proj.weight": "F32",
        "model.layers.0.input_layernorm.weight": "F32", "lm_head.weight": "F32",
        "model.embed_tokens.weight": "F32"})),
    "qwen2-bias": (dict(DEC, style="qwen2", qk_norm=False, qkv_bias=True), {}),
}


@pytest.mark.parametrize("case", sorted(CASES))
@pytest.mark.parametrize("act_dtype", ["fp16", "bf16"])
def test_decoder_checkpoint_is_bit_identical_to_generated_weights(tmp_path, case, act_dtype):
    over, save_kw = CASES[case]
    spec = with_labels(specs.preset("onejev-9b", **over))
    ck.save_synthetic(spec, str(tmp_path), gen=fast_gen, **save_kw)
    batch = decoder_batch(spec)
    want = outputs(spec, batch, act_dtype=act_dtype)
    got = outputs(dict(spec, checkpoint=str(tmp_path), seed=999), batch, act_dtype=act_dtype)
    np.testing.assert_array_equal(got, want)


def test_gemma_tied_checkpoint_opened_from_its_spec_file(tmp_path):
    spec = with_labels(specs.preset("decider-2b", hidden=1024, layers=2, heads=4, kv_heads=1, head_dim=256,
                                    ffn=2048, vocab=4096, seed=6))
    ck.save_synthetic(spec, str(tmp_path), gen=fast_gen, write_spec=True)
    batch = decoder_batch(spec, seed=4)
    np.testing.assert_array_equal(outputs(str(tmp_path), batch), outputs(spec, batch))


@pytest.mark.parametrize("preset", ["laya-bert", "laya-xlmr"])
def test_encoder_checkpoint_is_bit_identical_to_generated_weights(tmp_path, preset):
    spec = specs.preset(preset, layers=2, vocab=8192, seed=8)
    ck.save_synthetic(spec, str(tmp_path), gen=fast_gen)
    rng = np.random.default_rng(9)
    cls_id, sep_id = (101, 102) if preset == "laya-bert" else (0, 2)
    rows = encoder_rows(rng, 6, spec["vocab"], lengths="uniform-bert", cls_id=cls_id, sep_id=sep_id, id_low=5,
                        max_len=spec["max_pos"] - 2)
    batch = collate(rows, Layout(pad_id=spec["pad_id"]))
    batch.qtype[:] = rng.integers(0, 3, size=batch.b)
    from_ckpt = ck.spec_from_checkpoint(str(tmp_path), head_layers=spec["head_layers"])
    np.testing.assert_array_equal(outputs(from_ckpt, batch), outputs(spec, batch))


def test_missing_tensor_and_wrong_shape_fail_the_open(tmp_path):
    from verdict_b200._abi import VD_ESPEC, VdError
    spec = with_labels(specs.preset("onejev-9b", **DEC))
    ck.save_synthetic(dict(spec, tied=True), str(tmp_path), gen=fast_gen)  # no lm_head.weight
    small = dict(max_tokens=1024, max_rows=4, max_seq=1024)
    cases = [(dict(tied=True, ffn=2944), "shape"),
             (dict(tied=True, layers=3), "has no tensor model.layers.2."),
             (dict(tied=False), "has no tensor lm_head.weight")]
    for over, msg in cases:
        with pytest.raises(VdError, match=msg) as e:
            B200Engine(dict(spec, checkpoint=str(tmp_path), **over), **small)
        assert e.value.code == VD_ESPEC
    B200Engine(dict(spec, checkpoint=str(tmp_path), tied=True), **small).close()


def test_minimal_spec_takes_its_shape_from_the_hf_config(tmp_path):
    """{"checkpoint", "label_ids", "family"} is enough: the library reads the
    rest from config.json and computes the same bits."""
    spec = with_labels(specs.preset("onejev-9b", **DEC))
    ck.save_synthetic(spec, str(tmp_path), gen=fast_gen)
    batch = decoder_batch(spec, seed=12)
    minimal = {"checkpoint": str(tmp_path), "label_ids": spec["label_ids"], "family": spec["family"]}
    np.testing.assert_array_equal(outputs(minimal, batch), outputs(spec, batch))
