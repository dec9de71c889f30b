"""Pin the CPU oracle to outputs of the reference's own code (tests/golden/*.npz,
made by tests/golden/make_golden.py from executor/torch_exec.py and the
marker-head DecisionModel run in fp32 on CPU)."""

import glob
import json
import os

import numpy as np
import pytest

from oracle.decoder import DecoderOracle, option_logprobs
from oracle.encoder import EncoderOracle
from verdict_b200.batch import CollatedBatch, RowMeta

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def load(path):
    z = np.load(path)
    spec = json.loads(str(z["spec"]))
    rows = [RowMeta(int(n), 0, 0) for n in z["real_len"]]
    nopts = z["nopts"] if "nopts" in z.files else np.zeros(0, np.int64)
    batch = CollatedBatch(z["input_ids"], z["attention_mask"], z["marker_pos"], z["marker_mask"], z["qtype"],
                          nopts, int(z["b"]), int(z["l"]), int(z["k"]), rows)
    return z, spec, batch


DEC = sorted(p for p in glob.glob(os.path.join(GOLDEN, "*.npz"))
             if "_marker_" not in p and "fork_" not in p and "von_" not in p)
VON = sorted(glob.glob(os.path.join(GOLDEN, "von_*.npz")))
ENC = sorted(glob.glob(os.path.join(GOLDEN, "*_marker_*.npz")))


def test_fixtures_present():
    assert len(DEC) >= 4 and len(ENC) >= 8


@pytest.mark.parametrize("path", DEC, ids=os.path.basename)
def test_decoder_oracle_matches_reference(path):
    z, spec, batch = load(path)
    got = DecoderOracle(spec).infer(batch)
    ref = z["logits"]
    assert got.shape == ref.shape
    np.testing.assert_allclose(got, ref, atol=1e-4, rtol=0)
    # and the restricted log-softmax the C ABI returns
    np.testing.assert_allclose(option_logprobs(got, batch.nopts), option_logprobs(ref, batch.nopts), atol=1e-4)


@pytest.mark.parametrize("path", ENC, ids=os.path.basename)
def test_encoder_oracle_matches_reference(path):
    z, spec, batch = load(path)
    got = EncoderOracle(spec).infer(batch)
    np.testing.assert_allclose(got, z["logits"], atol=1e-5, rtol=0)


@pytest.mark.parametrize("path", DEC, ids=os.path.basename)
def test_label_table_port_matches_reference(path):
    """verdict_b200.labels reproduces the reference's derive_branch_ids /
    derive_letter_ids on the same synthetic tokenizer (token ids bit-exact)."""
    pytest.importorskip("tokenizers")
    from tests.golden.make_golden import synthetic_tokenizer
    from verdict_b200.labels import derive_label_ids

    z, spec, _ = load(path)
    tok = synthetic_tokenizer(int(z["tok_vocab"]), int(z["tok_seed"]))
    assert derive_label_ids(spec["family"], tok) == [int(x) for x in z["label_table"]]
    assert spec["label_ids"] == [int(x) for x in z["label_table"]]


def test_oracle_is_sensitive():
    """A planted mistake in the oracle (a wrong RoPE base) breaks the match."""
    z, spec, batch = load(DEC[0])
    bad = dict(spec, rope_theta=spec["rope_theta"] * 0.5)
    got = DecoderOracle(bad).infer(batch)
    assert np.abs(got - z["logits"]).max() > 1e-3


@pytest.mark.parametrize("path", VON, ids=os.path.basename)
def test_von_oracle_matches_hf_modernbert(path):
    """Independent-options fixtures: HF ModernBertModel with the reference's
    option masks and positions (tests/golden/make_von_golden.py)."""
    from oracle.von import VonOracle
    z, spec, batch = load(path)
    got = VonOracle(spec).infer(batch)
    np.testing.assert_allclose(got, z["logits"], atol=2e-5, rtol=0)
