"""Shared-prefix fork on the GPU: rows that share a prefix compute it once.

The engine must (a) fork exactly the groups the reference's grouping rules
form (oracle/fork.py, pinned to the reference's own `_text_fork_forward` by
tests/golden/fork_groups.npz), and (b) return what the whole-row forward
returns: within the log-prob tolerance of the fp32 oracle, and within
FORK_TOL of the same engine with the fork off (the two differ only in where
attention splits its key tiles; the reference gates its fork at 5e-2 of the
whole-row softmax, executor/torch_exec.py:2024-2066)."""

import json
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from oracle import fork  # noqa: E402
from oracle.decoder import DecoderOracle, option_logprobs  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import BuiltSequence, Layout, collate  # noqa: E402
from verdict_b200.engine import B200Engine  # noqa: E402
from verdict_b200.synth import with_labels  # noqa: E402

pytestmark = pytest.mark.gpu

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fork_groups.npz")
LOGPROB_TOL = 2e-2
FORK_TOL = 5e-3


def batch_of(rows, prefix_len, slots=None, seed=0):
    rng = np.random.default_rng(seed)
    seqs = []
    for i, r in enumerate(rows):
        slot = len(r) - 1 if slots is None else int(slots[i])
        seqs.append(BuiltSequence(ids=list(map(int, r)), markers=[slot], nopts=[int(rng.integers(2, 9))],
                                  prefix_len=int(prefix_len[i])))
    return collate(seqs, Layout(pad_id=0))


def expected_stats(batch):
    ids = batch.input_ids.reshape(batch.b, batch.l)
    groups = fork.plan(ids, batch.real_len(), batch.marker_pos.reshape(batch.b, batch.k)[:, 0],
                       batch.prefix_len(), single=False)
    return dict(fork_groups=len(groups), fork_rows=sum(len(m) for m, _ in groups),
                shared_tokens=sum(n * (len(m) - 1) for m, n in groups))


def run(eng, batch):
    rows = eng.infer(batch)
    return np.array([r.logits for r in rows], dtype=np.float64), eng.last_stats()


def check(spec, batch, ref=None, fork_tol=FORK_TOL, **kw):
    on = B200Engine(spec, max_tokens=16384, max_rows=64, max_seq=4096, **kw)
    off = B200Engine(spec, max_tokens=16384, max_rows=64, max_seq=4096, fork=False, **kw)
    try:
        got, st = run(on, batch)
        whole, st_off = run(off, batch)
    finally:
        on.close()
        off.close()
    want = expected_stats(batch)
    assert {k: st[k] for k in want} == want
    assert st_off["fork_groups"] == 0 and st["tokens"] == st_off["tokens"] - want["shared_tokens"]
    live = whole > -1e4
    assert np.all(got[~live] == -1e4)
    d = np.abs(got - whole)[live].max()
    assert d <= fork_tol, f"fork vs whole rows: {d:.3e}"
    if ref is not None:
        ref_lp = option_logprobs(ref, batch.nopts)
        for i, k in enumerate(batch.nopts):
            assert np.abs(got[i, :k] - ref_lp[i, :k]).max() <= LOGPROB_TOL, f"row {i}"
    return st


def spec9b(layers=2, **over):
    return with_labels(specs.preset("onejev-9b", layers=layers, vocab=8192, seed=21, **over))


def golden_cases():
    z = np.load(GOLDEN)
    for m in json.loads(str(z["meta"])):
        n = m["name"]
        yield n, z[f"{n}_ids"], z[f"{n}_real_len"], z[f"{n}_slot"], z[f"{n}_prefix_len"]


@pytest.mark.parametrize("case", list(golden_cases()), ids=lambda c: c[0])
def test_golden_groupings_fork_and_match_whole_rows(case):
    name, ids, real_len, slot, prefix_len = case
    rows = [ids[i, :real_len[i]] for i in range(len(real_len))]
    batch = batch_of(rows, prefix_len, slot, seed=3)
    spec = spec9b()
    check(spec, batch, DecoderOracle(spec).infer(batch))


def long_prefix_batch(vocab, seed, prefix_lens=(1500, 700), members=4, declared=True):
    rng = np.random.default_rng(seed)
    rows, pl = [], []
    for plen in prefix_lens:
        pre = rng.integers(3, vocab, size=plen).tolist()
        for _ in range(members):
            rows.append(pre + rng.integers(3, vocab, size=int(rng.integers(20, 260))).tolist())
            pl.append(plen if declared else 0)
    rows.append(rng.integers(3, vocab, size=900).tolist())
    pl.append(0)
    order = rng.permutation(len(rows))
    return batch_of([rows[i] for i in order], [pl[i] for i in order], seed=seed)


@pytest.mark.parametrize("attention", ["tc", "tc2", "mma"])
@pytest.mark.parametrize("declared", [True, False])
def test_long_shared_prefixes_hd128(attention, declared):
    spec = spec9b()
    batch = long_prefix_batch(spec["vocab"], 5, declared=declared)
    st = check(spec, batch, DecoderOracle(spec).infer(batch), attention=attention)
    assert st["fork_groups"] == 2 and st["shared_tokens"] == 3 * 1500 + 3 * 700


def test_long_shared_prefixes_gemma_hd256():
    spec = with_labels(specs.preset("decider-2b", layers=2, vocab=8192, seed=22))
    batch = long_prefix_batch(spec["vocab"], 6, prefix_lens=(1100, 300), members=3)
    check(spec, batch, DecoderOracle(spec).infer(batch))


def test_fork_with_bf16_activations():
    """bf16 activations: fork against whole rows of the same engine (bf16's
    own deviation from the fp32 oracle on long rows can exceed 2e-2, which is
    why fp16 is the default element type)."""
    spec = spec9b()
    batch = long_prefix_batch(spec["vocab"], 9, prefix_lens=(800,), members=4)
    check(spec, batch, act_dtype="bf16", fork_tol=LOGPROB_TOL)


def test_fork_at_full_depth_and_in_chunks():
    """All 40 layers (rounding differences of the two key-tile splits
    accumulate with depth: held to the log-prob tolerance), and a workspace
    that splits a group over chunks (each chunk forks its own part)."""
    spec = spec9b(layers=40)
    batch = long_prefix_batch(spec["vocab"], 7, prefix_lens=(1000,), members=6)
    check(spec, batch, fork_tol=LOGPROB_TOL)
    small_on = B200Engine(spec, max_tokens=4096, max_rows=3, max_seq=2048)
    small_off = B200Engine(spec, max_tokens=4096, max_rows=3, max_seq=2048, fork=False)
    try:
        a, st = run(small_on, batch)
        b, _ = run(small_off, batch)
        assert st["chunks"] >= 3 and st["fork_groups"] >= 2
        live = b > -1e4
        assert np.abs(a - b)[live].max() <= LOGPROB_TOL
    finally:
        small_on.close()
        small_off.close()


def test_device_resident_batches_fork_when_they_declare_prefixes():
    """A device-memory batch is planned from a copy of its ids when it passes
    prefix_len; without prefix_len it runs whole rows (no copy back)."""
    spec = spec9b()
    batch = long_prefix_batch(spec["vocab"], 8, prefix_lens=(600,), members=3)
    eng = B200Engine(spec, max_tokens=8192, max_rows=16, max_seq=2048)
    try:
        host, st = run(eng, batch)
        assert st["fork_groups"] == 1
        dev = {k: torch.from_numpy(np.ascontiguousarray(v)).cuda() for k, v in dict(
            input_ids=batch.input_ids, marker_pos=batch.marker_pos,
            marker_mask=batch.marker_mask.astype(np.uint8), nopts=batch.nopts).items()}
        ptrs = {k: v.data_ptr() for k, v in dev.items()}
        live = host > -1e4
        for prefix_len, groups in ((None, 0), (batch.prefix_len(), 1)):
            out = torch.empty((batch.b, eng.width), dtype=torch.float32, device="cuda")
            eng.infer_device(batch.b, batch.l, batch.k, ptrs, batch.real_len(), out.data_ptr(), eng.width,
                             sync=True, prefix_len=prefix_len)
            assert eng.last_stats()["fork_groups"] == groups
            got = out.cpu().numpy().astype(np.float64)
            if groups:
                np.testing.assert_array_equal(got, host)
            else:
                assert np.abs(got - host)[live].max() <= FORK_TOL
    finally:
        eng.close()


def letter_branches_batch(vocab, seed, chat=72, states=(700, 350, 1200), questions=3):
    """Rows as letter_branches renders them (`build_row`,
    src/family/letter_branches.rs:89-121): one chat/system prompt shared by
    every row, then the state, then the question; the declared prefix_len is
    chat + state.  Without it the 32-token common-prefix key would put every
    row in one group that forks only the chat prompt."""
    rng = np.random.default_rng(seed)
    head = rng.integers(3, vocab, size=chat).tolist()
    rows, pl = [], []
    for n in states:
        pre = head + rng.integers(3, vocab, size=n).tolist()
        for _ in range(questions):
            rows.append(pre + rng.integers(3, vocab, size=int(rng.integers(30, 120))).tolist())
            pl.append(len(pre))
    order = rng.permutation(len(rows))
    return batch_of([rows[i] for i in order], [pl[i] for i in order], seed=seed)


def vd_infer_raw(eng, batch, with_prefix_len):
    """vd_infer through ctypes exactly as the Rust binding calls it: host
    buffers, RowMeta's real_len / real_k / prefix_len passed as arrays."""
    import ctypes
    from verdict_b200 import _abi
    ids = np.ascontiguousarray(batch.input_ids, dtype=np.int64)
    amask = np.ascontiguousarray(batch.attention_mask, dtype=np.int64)
    mpos = np.ascontiguousarray(batch.marker_pos, dtype=np.int64)
    mmask = np.ascontiguousarray(batch.marker_mask, dtype=np.uint8)
    qtype = np.ascontiguousarray(batch.qtype, dtype=np.int64)
    nopts = np.ascontiguousarray(batch.nopts, dtype=np.int64)
    real_len = np.array([r.real_len for r in batch.rows], dtype=np.int64)
    real_k = np.array([r.real_k for r in batch.rows], dtype=np.int64)
    prefix_len = np.array([r.prefix_len for r in batch.rows], dtype=np.int64)
    st = _abi.VdBatch()
    st.b, st.l, st.k, st.memory = batch.b, batch.l, batch.k, _abi.VD_MEM_HOST
    for name, a in (("input_ids", ids), ("attention_mask", amask), ("marker_pos", mpos), ("marker_mask", mmask),
                    ("qtype", qtype), ("nopts", nopts), ("real_len", real_len), ("real_k", real_k)):
        setattr(st, name, ctypes.c_void_p(a.ctypes.data))
    st.prefix_len = ctypes.c_void_p(prefix_len.ctypes.data) if with_prefix_len else None
    out = np.empty((batch.b, eng.width), dtype=np.float32)
    err = ctypes.create_string_buffer(1024)
    rc = eng.lib.vd_infer(eng.h, ctypes.byref(st), ctypes.c_void_p(out.ctypes.data), eng.width, err, len(err))
    _abi.check(rc, err)
    return out.astype(np.float64), eng.last_stats()


def test_rust_binding_passes_declared_prefixes():
    """The C ABI called as the Rust `Engine` binding calls it forms the
    reference's declared-prefix groups (one per state) when prefix_len is
    passed, and the common-prefix groups when it is not; both give the
    whole-row answer."""
    spec = spec9b()
    batch = letter_branches_batch(spec["vocab"], 12)
    ids = batch.input_ids.reshape(batch.b, batch.l)
    slot = batch.marker_pos.reshape(batch.b, batch.k)[:, 0]
    declared = fork.plan(ids, batch.real_len(), slot, batch.prefix_len(), single=False)
    undeclared = fork.plan(ids, batch.real_len(), slot, None, single=False)
    assert len(declared) == 3 and len(undeclared) == 1 and undeclared[0][1] == 72
    on = B200Engine(spec, max_tokens=16384, max_rows=64, max_seq=4096)
    off = B200Engine(spec, max_tokens=16384, max_rows=64, max_seq=4096, fork=False)
    try:
        whole, _ = vd_infer_raw(off, batch, True)
        for with_pl, groups in ((True, declared), (False, undeclared)):
            got, st = vd_infer_raw(on, batch, with_pl)
            assert st["fork_groups"] == len(groups)
            assert st["fork_rows"] == sum(len(m) for m, _ in groups)
            assert st["shared_tokens"] == sum(n * (len(m) - 1) for m, n in groups)
            live = whole > -1e4
            assert np.all(got[~live] == -1e4)
            assert np.abs(got - whole)[live].max() <= FORK_TOL
    finally:
        on.close()
        off.close()
