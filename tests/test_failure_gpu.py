"""Failure detection on the GPU without a GPU fault: a bounded wait runs out.

Every barrier wait in the tcgen05 pipelines is bounded; a wait that runs out
records an error code in the handle's device error word, raises the CTA's
abort flag, and the CTA leaves its loops, lets the tensor-core ops it issued
finish (bounded), frees its tensor memory and exits.  The call then fails with
VD_ECUDA, the handle reports unhealthy and refuses work, and the GPU context
stays usable: a fresh handle answers correctly.

The stall is made on purpose and stays in bounds: with `debug_stall_gemm` the
first one-CTA GEMM of the call issues only its first two k-blocks of TMA loads
(valid tiles) and then stops, so its MMA warp waits for a stage nothing will
fill; `wait_limit_us` shortens that wait to 1 ms.
"""

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle.decoder import DecoderOracle, option_logprobs  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import Layout, collate, decoder_rows  # noqa: E402
from verdict_b200.engine import B200Engine, EngineError  # noqa: E402
from verdict_b200.synth import with_labels  # noqa: E402

pytestmark = pytest.mark.gpu


def small_case():
    spec = with_labels(specs.preset("onejev-9b", hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128,
                                    ffn=512, vocab=8448, seed=61))
    rng = np.random.default_rng(61)
    rows = decoder_rows(rng, 3, spec["vocab"], lengths="fixed:8")
    for r, n in zip(rows, (40, 130, 257)):
        r.ids = rng.integers(3, spec["vocab"], size=n).tolist()
        r.markers = [n - 1]
    return spec, collate(rows, Layout(pad_id=0))


def test_stalled_gemm_times_out_and_the_handle_reports_it():
    spec, batch = small_case()
    eng = B200Engine(spec, max_tokens=1024, max_rows=8, max_seq=512, gemm="1sm", wait_limit_us=1000,
                     debug_stall_gemm=2)
    try:
        assert eng.health()
        with pytest.raises(EngineError, match="timed out"):
            eng.infer(batch)
        assert not eng.health()
        with pytest.raises(EngineError, match="dead"):
            eng.infer(batch)
    finally:
        eng.close()
    # The context survived: a fresh handle on the same GPU gives the oracle's answer.
    fresh = B200Engine(spec, max_tokens=1024, max_rows=8, max_seq=512, gemm="1sm")
    try:
        got = np.array([r.logits for r in fresh.infer(batch)], dtype=np.float64)
        assert fresh.health()
    finally:
        fresh.close()
    ref = option_logprobs(DecoderOracle(spec).infer(batch), batch.nopts)
    for i, k in enumerate(batch.nopts):
        assert np.abs(got[i, :int(k)] - ref[i, :int(k)]).max() <= 2e-2


def test_short_wait_limit_alone_changes_nothing():
    """A 1 ms wait limit without the stall: every wait of these small GEMMs
    ends well inside it, and the result is bit-identical to the default."""
    spec, batch = small_case()
    a = B200Engine(spec, max_tokens=1024, max_rows=8, max_seq=512, gemm="1sm", wait_limit_us=1000)
    b = B200Engine(spec, max_tokens=1024, max_rows=8, max_seq=512, gemm="1sm")
    try:
        la = np.array([r.logits for r in a.infer(batch)])
        lb = np.array([r.logits for r in b.infer(batch)])
        assert a.health() and b.health()
        np.testing.assert_array_equal(la, lb)
    finally:
        a.close()
        b.close()
