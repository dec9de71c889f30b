"""Independent-options (ModernBERT + option masks) on the GPU against the fp32
oracle, which tests/golden/von_*.npz pin to transformers' ModernBertModel.

Tolerance as the marker-head encoder: scorer logits within ENC_TOL of
max(1, |ref|) (the reference's own export check allows 1e-3 relative,
convert/compare.py:9-25)."""

import glob
import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.fastsynth import gen_tensor as fast_gen  # noqa: E402
from oracle.von import VonOracle  # noqa: E402
from verdict_b200 import checkpoint as ck  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import CollatedBatch, Layout, RowMeta, collate, von_rows  # noqa: E402
from verdict_b200.engine import B200Engine, EngineError  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")
ENC_TOL = 2e-3


def load_fixture(path):
    z = np.load(path)
    spec = json.loads(str(z["spec"]))
    rows = [RowMeta(int(n), int(k), 0) for n, k in zip(z["real_len"], z["real_k"])]
    batch = CollatedBatch(z["input_ids"], z["attention_mask"], z["marker_pos"], z["marker_mask"], z["qtype"],
                          np.zeros(0, np.int64), int(z["b"]), int(z["l"]), int(z["k"]), rows)
    return spec, batch, z["logits"]


def run(spec, batch, **kw):
    eng = B200Engine(spec, **dict(dict(max_tokens=16384, max_rows=64, max_seq=2048), **kw))
    try:
        return np.array([r.logits for r in eng.infer(batch)], dtype=np.float64)
    finally:
        eng.close()


def check(got, ref, tol=ENC_TOL):
    live = ref > -1e4
    assert np.all(got[~live] == -1e4)
    scale = max(1.0, float(np.abs(ref[live]).max()))
    d = np.abs(got[live] - ref[live]).max() / scale
    assert d <= tol, f"max relative deviation {d:.3e}"


@pytest.mark.parametrize("path", sorted(glob.glob(os.path.join(GOLDEN, "von_*.npz"))), ids=os.path.basename)
@pytest.mark.parametrize("act_dtype", ["fp16", "bf16"])
def test_von_golden(path, act_dtype):
    """fp16 (the default) at ENC_TOL; bf16 activations keep 8 mantissa bits, so
    their logits are held to 3e-2."""
    spec, batch, ref = load_fixture(path)
    check(run(spec, batch, act_dtype=act_dtype)[:, :batch.k], ref, ENC_TOL if act_dtype == "fp16" else 3e-2)


def von_batch(spec, seed, n):
    rng = np.random.default_rng(seed)
    rows = von_rows(rng, n, spec["vocab"])
    return collate(rows, Layout(pad_id=spec["pad_id"]))


def test_von_base_full_depth_vs_oracle():
    """All 22 layers of the ModernBERT-base shape (7 global, 15 local).  At this
    depth fp16 activation storage alone moves the logits by ~ENC_TOL (the
    oracle with every 16-bit store of the GPU path emulated, `store16`), so the
    bound is ENC_TOL beyond that storage deviation."""
    spec = specs.preset("von-base", seed=71)
    batch = von_batch(spec, 71, 6)
    ref = VonOracle(spec).infer(batch)
    ref16 = VonOracle(spec, store16=True).infer(batch)
    live = ref > -1e4
    storage = np.abs(ref16 - ref)[live].max() / max(1.0, float(np.abs(ref[live]).max()))
    check(run(spec, batch), ref, ENC_TOL + storage)


def test_von_chunking_is_bit_exact_and_windows_matter():
    spec = specs.preset("von-base", layers=6, seed=72)
    batch = von_batch(spec, 72, 9)
    # split_k off: small chunks would otherwise sum K in split order (exact to
    # rounding, not to the bit).
    a = run(spec, batch, split_k=False)
    b = run(spec, batch, max_tokens=512, max_rows=2, split_k=False)
    np.testing.assert_array_equal(a, b)
    wide = run(dict(spec, sliding_window=4096), batch)  # a window covering every row: all layers global
    assert np.abs(wide - a)[a > -1e4].max() > 1e-4


def test_von_checkpoint_is_bit_identical(tmp_path):
    spec = specs.preset("von-base", layers=4, seed=73)
    ck.save_synthetic(spec, str(tmp_path), gen=fast_gen)
    batch = von_batch(spec, 73, 5)
    np.testing.assert_array_equal(run({"checkpoint": str(tmp_path)}, batch), run(spec, batch))


def test_rows_without_markers_fail_the_batch():
    spec = specs.preset("von-base", layers=2, seed=74)
    batch = von_batch(spec, 74, 3)
    batch.marker_mask[batch.k:2 * batch.k] = False  # row 1 loses every marker
    eng = B200Engine(spec, max_tokens=4096, max_rows=8, max_seq=1024)
    try:
        with pytest.raises(EngineError, match="row 1: no marker positions inside the real ids"):
            eng.infer(batch)
        assert eng.health()
    finally:
        eng.close()
