"""16-bit activation overflow: reported, never returned as scores.

fp16 activations (the default element type) stop at 65504.  A checkpoint
whose MLP intermediate exceeds that turns the stored activation into inf, the
next GEMM turns it into inf / NaN in the residual stream, and every later
token of the row inherits it through attention.  The readout (decoders) and
the marker scorer (encoders) check the slot / marker hidden state and the
logits for inf / NaN and fail the batch with VD_EDEVICE, naming the bf16
activation mode; the handle stays healthy.  bf16 activations have fp32's
exponent range and give the oracle's answer on the same checkpoint.

The overflow is planted in the weights: the checkpoint is the synthetic one
with the first layer's MLP input projections scaled by a power of two (exact
in bf16 and fp16), written as safetensors and opened from disk; the oracle
reads the same scaled tensors.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.decoder import DecoderOracle, option_logprobs  # noqa: E402
from oracle.encoder import EncoderOracle  # noqa: E402
from oracle.fastsynth import gen_tensor  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import Layout, collate, decoder_rows, encoder_rows  # noqa: E402
from verdict_b200.checkpoint import save_synthetic  # noqa: E402
from verdict_b200.engine import B200Engine, EngineError  # noqa: E402
from verdict_b200.synth import with_labels  # noqa: E402

pytestmark = pytest.mark.gpu

LOGPROB_TOL = 2e-2
BF16_ENC_TOL = 5e-2  # bf16 encoder logits vs the fp32 oracle, relative to max(1, |ref|)


class GainCheckpoint:
    """The oracle's synthetic checkpoint with some tensors multiplied by a gain."""

    def __init__(self, inner, gains):
        self.inner, self.gains = inner, gains

    def get(self, name, rows=None):
        t = self.inner.get(name, rows=rows)
        return t * np.float32(self.gains.get(name, 1.0))

    def head_name(self):
        return self.inner.head_name()


def write_gained(spec, out_dir, gains):
    def gen(seed, name, shape, scale, off):
        return gen_tensor(seed, name, shape, scale, off) * np.float32(gains.get(name, 1.0))
    return save_synthetic(spec, str(out_dir), gen=gen, write_spec=True)


def decoder_setup(tmp_path):
    spec = with_labels(specs.preset("onejev-9b", hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128,
                                    ffn=512, vocab=8448, seed=101))
    # silu(g) * u of layer 0 reaches ~2.3e5 (g, u ~ 164 rms): far past fp16's 65504.
    gains = {"model.layers.0.mlp.gate_proj.weight": 2.0 ** 9, "model.layers.0.mlp.up_proj.weight": 2.0 ** 9}
    path = write_gained(spec, tmp_path / "ckpt", gains)
    rng = np.random.default_rng(3)
    rows = decoder_rows(rng, 4, spec["vocab"], lengths="fixed:8")
    for r, n in zip(rows, (17, 60, 200, 333)):
        r.ids = rng.integers(3, spec["vocab"], size=n).tolist()
        r.markers = [n - 1]
    batch = collate(rows, Layout(pad_id=0))
    orc = DecoderOracle(spec)
    orc.ckpt = GainCheckpoint(orc.ckpt, gains)
    with np.errstate(over="ignore"):
        ref = orc.infer(batch)
    return spec, path, batch, ref


def test_fp16_overflow_fails_the_batch_and_bf16_matches_the_oracle(tmp_path):
    spec, path, batch, ref = decoder_setup(tmp_path)
    assert np.isfinite(ref).all()
    eng = B200Engine(path, max_tokens=2048, max_rows=16, max_seq=1024)
    try:
        with pytest.raises(EngineError, match="non-finite.*bf16"):
            eng.infer(batch)
        assert eng.health(), "an overflow is a property of the batch and weights, not a broken handle"
        with pytest.raises(EngineError, match="non-finite"):
            eng.infer(batch)  # the error word was cleared and set again
    finally:
        eng.close()
    eng = B200Engine(path, max_tokens=2048, max_rows=16, max_seq=1024, act_dtype="bf16")
    try:
        got = np.array([r.logits for r in eng.infer(batch)], dtype=np.float64)
    finally:
        eng.close()
    ref_lp = option_logprobs(ref, batch.nopts)
    for i, k in enumerate(batch.nopts):
        k = int(k)
        d = np.abs(got[i, :k] - ref_lp[i, :k]).max()
        assert d <= LOGPROB_TOL, f"row {i}: bf16 vs oracle {d:.3e}"
        assert np.all(got[i, k:] == -1e4)


def test_fp16_without_overflow_still_answers(tmp_path):
    """The same engine and rows without the planted gains: no error."""
    spec = with_labels(specs.preset("onejev-9b", hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128,
                                    ffn=512, vocab=8448, seed=101))
    path = write_gained(spec, tmp_path / "plain", {})
    _, _, batch, _ = decoder_setup(tmp_path)
    ref = DecoderOracle(spec).infer(batch)
    eng = B200Engine(path, max_tokens=2048, max_rows=16, max_seq=1024)
    try:
        got = np.array([r.logits for r in eng.infer(batch)], dtype=np.float64)
    finally:
        eng.close()
    ref_lp = option_logprobs(ref, batch.nopts)
    for i, k in enumerate(batch.nopts):
        assert np.abs(got[i, :int(k)] - ref_lp[i, :int(k)]).max() <= LOGPROB_TOL


def test_encoder_fp16_overflow_fails_the_batch(tmp_path):
    spec = specs.preset("laya-bert", hidden=128, layers=2, heads=2, ffn=512, vocab=4096, seed=44)
    # GELU(x W1^T) of layer 0 reaches ~1e5 (x W1^T ~ 3e4 rms) in fp16.
    gains = {"encoder.encoder.layer.0.intermediate.dense.weight": 2.0 ** 17}
    path = write_gained(spec, tmp_path / "enc", gains)
    rng = np.random.default_rng(44)
    rows = encoder_rows(rng, 6, spec["vocab"], lengths="uniform-bert", cls_id=101, sep_id=102, id_low=1000,
                        max_len=120)
    batch = collate(rows, Layout(pad_id=spec["pad_id"]))
    batch.qtype[:] = rng.integers(0, 3, size=batch.b)
    orc = EncoderOracle(spec)
    orc.ckpt = GainCheckpoint(orc.ckpt, gains)
    ref = orc.infer(batch)
    live = ref > -1e4
    assert np.isfinite(ref).all()
    eng = B200Engine(path, max_tokens=4096, max_rows=16, max_seq=512)
    try:
        with pytest.raises(EngineError, match="non-finite.*bf16"):
            eng.infer(batch)
        assert eng.health()
    finally:
        eng.close()
    eng = B200Engine(path, max_tokens=4096, max_rows=16, max_seq=512, act_dtype="bf16")
    try:
        got = np.array([r.logits for r in eng.infer(batch)], dtype=np.float64)
    finally:
        eng.close()
    assert np.all(got[~live] == -1e4)
    scale = max(1.0, float(np.abs(ref[live]).max()))
    assert np.abs(got[live] - ref[live]).max() / scale <= BF16_ENC_TOL
