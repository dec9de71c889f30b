"""Scheduler-side batch types: `BuiltSequence`, `RowMeta`, `CollatedBatch`, `collate`.

These restate the Rust types that cross the `Engine` boundary, field for field:
- `BuiltSequence` and `real_k`: `src/tokenize.rs:62-104`
- `CollatedBatch`, `RowMeta`: `src/scheduler.rs:79-103`
- `collate`: `src/scheduler.rs:108-172`
The executor receives a right-padded `[b, l]` batch exactly as `collate` lays it
out; the C library packs it into a ragged varlen batch on the device.

Seeded synthetic workloads (`decoder_rows`, `encoder_rows`) stand in for the
reference's private benchmark corpus: they draw prompt lengths, option counts
and token ids from the distributions of the five benchmark configurations.
"""

from __future__ import annotations

from dataclasses import dataclass, field

import numpy as np


@dataclass
class BuiltSequence:
    """One tokenised row (`src/tokenize.rs:62-78`)."""
    ids: list
    markers: list
    nopts: list = field(default_factory=list)
    prefix_len: int = 0
    full_len: int = 0
    task: str = "choice"

    def real_k(self) -> int:
        """`BuiltSequence::real_k` (`src/tokenize.rs:98-104`)."""
        return len(self.markers) if not self.nopts else int(sum(self.nopts))


@dataclass
class RowMeta:
    real_len: int
    real_k: int
    prefix_len: int


@dataclass
class Layout:
    """The collate-relevant part of `tokenize::Layout` (`src/tokenize.rs:27-45`)."""
    pad_id: int
    seq_align: int = 1
    fixed_classes: tuple = ()


@dataclass
class CollatedBatch:
    """`CollatedBatch` (`src/scheduler.rs:79-97`), arrays flattened row-major."""
    input_ids: np.ndarray        # int64 [b*l]
    attention_mask: np.ndarray   # int64 [b*l]
    marker_pos: np.ndarray       # int64 [b*k]
    marker_mask: np.ndarray      # bool  [b*k]
    qtype: np.ndarray            # int64 [b]
    nopts: np.ndarray            # int64 [b] (empty for marker families)
    b: int
    l: int
    k: int
    rows: list                   # [RowMeta]

    def real_len(self) -> np.ndarray:
        return np.array([r.real_len for r in self.rows], dtype=np.int64)

    def real_k(self) -> np.ndarray:
        return np.array([r.real_k for r in self.rows], dtype=np.int64)

    def prefix_len(self) -> np.ndarray:
        return np.array([r.prefix_len for r in self.rows], dtype=np.int64)


QTYPE = {"choice": 0, "score": 1, "noul": 2}  # `calibration::qtype_of`, src/calibration.rs


def collate(items: list, layout: Layout) -> CollatedBatch:
    """Right-pad rows into one batch; same arithmetic as `src/scheduler.rs:108-172`."""
    b = len(items)
    l = max((len(r.ids) for r in items), default=0)
    if layout.fixed_classes:
        for c in layout.fixed_classes:
            if c >= l:
                l = c
                break
    elif layout.seq_align > 1:
        l = -(-l // layout.seq_align) * layout.seq_align
    k = max((len(r.markers) for r in items), default=0)
    input_ids = np.full(b * l, layout.pad_id, dtype=np.int64)
    attention_mask = np.zeros(b * l, dtype=np.int64)
    marker_pos = np.zeros(b * k, dtype=np.int64)
    marker_mask = np.zeros(b * k, dtype=bool)
    qtype = np.zeros(b, dtype=np.int64)
    nopts = []
    rows = []
    for i, req in enumerate(items):
        n = len(req.ids)
        input_ids[i * l:i * l + n] = req.ids
        attention_mask[i * l:i * l + n] = 1
        for j, m in enumerate(req.markers):
            marker_pos[i * k + j] = m
            marker_mask[i * k + j] = True
        qtype[i] = QTYPE.get(req.task, 0)
        if req.nopts:
            nopts.append(req.real_k())
        rows.append(RowMeta(real_len=n, real_k=req.real_k(), prefix_len=req.prefix_len))
    return CollatedBatch(input_ids, attention_mask, marker_pos, marker_mask, qtype,
                         np.array(nopts, dtype=np.int64), b, l, k, rows)


# ---------------------------------------------------------------------------
# Seeded synthetic workloads
# ---------------------------------------------------------------------------

def decoder_rows(rng: np.random.Generator, n: int, vocab: int, *, lengths: str,
                 min_opts: int = 2, max_opts: int = 8, fixed_opts: int | None = None,
                 id_low: int = 3) -> list:
    """Letter-family rows: slot = last prompt token (`src/family/letter_branches.rs:102`).

    lengths: "lognormal-9b" = clip(lognormal(6, 0.7), 32, 4096) (OneJev-9B),
             "uniform-2b"   = U[64, 1024] (Gemma-2B decider),
             "uniform-27b"  = U[512, 8192] (OneJev-27B),
             "fixed:<n>"    = every prompt n tokens long.
    Option texts only lengthen the prompt; the score is always read at one slot."""
    if lengths == "lognormal-9b":
        lens = np.clip(np.rint(rng.lognormal(6.0, 0.7, size=n)), 32, 4096).astype(int)
    elif lengths == "uniform-2b":
        lens = rng.integers(64, 1025, size=n)
    elif lengths == "uniform-27b":
        lens = rng.integers(512, 8193, size=n)
    elif lengths.startswith("fixed:"):
        lens = np.full(n, int(lengths.split(":")[1]))
    else:
        raise ValueError(lengths)
    rows = []
    for i in range(n):
        m = int(lens[i])
        ids = rng.integers(id_low, vocab, size=m).tolist()
        k = fixed_opts if fixed_opts else int(rng.integers(min_opts, max_opts + 1))
        rows.append(BuiltSequence(ids=ids, markers=[m - 1], nopts=[k], prefix_len=0,
                                  full_len=m))
    return rows


def shared_prefix_rows(rng: np.random.Generator, n: int, vocab: int, *, per_state: int = 8,
                       min_opts: int = 2, max_opts: int = 8, id_low: int = 3) -> list:
    """Letter-branches rows that ask `per_state` questions about each state:
    the rendered prompt is chat prefix + state, then question + options + answer
    line (`build_row`, `src/family/letter_branches.rs:89-121`), so the rows of
    one state share the prompt up to `prefix_len`.  State (prefix) lengths
    clip(lognormal(6.5, 0.5), 128, 3072) (mean ~750), question suffixes
    U[40, 160] tokens; slot = last token."""
    rows = []
    while len(rows) < n:
        plen = int(np.clip(np.rint(rng.lognormal(6.5, 0.5)), 128, 3072))
        prefix = rng.integers(id_low, vocab, size=plen).tolist()
        for _ in range(min(per_state, n - len(rows))):
            ids = prefix + rng.integers(id_low, vocab, size=int(rng.integers(40, 161))).tolist()
            k = int(rng.integers(min_opts, max_opts + 1))
            rows.append(BuiltSequence(ids=ids, markers=[len(ids) - 1], nopts=[k], prefix_len=plen,
                                      full_len=len(ids)))
    order = rng.permutation(len(rows))
    return [rows[i] for i in order]


def von_rows(rng: np.random.Generator, n: int, vocab: int, *, cls_id: int = 50281, sep_id: int = 50282,
             mask_id: int = 50284, id_low: int = 5, k_low: int = 2, k_high: int = 6,
             prefix_low: int = 16, prefix_high: int = 200, desc_high: int = 12) -> list:
    """Independent-options rows laid out like `independent_options::build_sequence`
    (`src/family/independent_options.rs:86-130`): [CLS] question+state [SEP]
    ([MASK] option text)* [SEP], one marker per [MASK].  Prefix U[16, 200]
    tokens, 2-6 options of U[1, 12] tokens each."""
    rows = []
    special = min(cls_id, sep_id, mask_id)
    top = min(vocab, special) if special > id_low else vocab  # text ids avoid the special ids
    for _ in range(n):
        prefix = int(rng.integers(prefix_low, prefix_high + 1))
        k = int(rng.integers(k_low, k_high + 1))
        ids = [cls_id] + rng.integers(id_low, top, size=prefix).tolist() + [sep_id]
        markers = []
        for _ in range(k):
            markers.append(len(ids))
            ids.append(mask_id)
            ids += rng.integers(id_low, top, size=int(rng.integers(1, desc_high + 1))).tolist()
        ids.append(sep_id)
        rows.append(BuiltSequence(ids=ids, markers=markers, nopts=[], full_len=len(ids)))
    return rows


def encoder_rows(rng: np.random.Generator, n: int, vocab: int, *, lengths: str,
                 cls_id: int, sep_id: int, id_low: int, k_low: int = 2, k_high: int = 6,
                 max_len: int = 512) -> list:
    """Marker-head rows laid out like `marker_head::build_sequence`
    (`src/family/marker_head.rs:35-103`): [CLS] head [SEP] (marker opt)* [SEP] state [SEP].

    lengths: "uniform-bert" = U[16, 128] with K=3 (laya BERT-base),
             "lognormal-xlmr" = clip(lognormal(4.5, 0.6), 8, 512) with K~U{2..6}."""
    rows = []
    for _ in range(n):
        if lengths == "uniform-bert":
            total, k = int(rng.integers(16, 129)), 3
        elif lengths == "lognormal-xlmr":
            total = int(np.clip(np.rint(rng.lognormal(4.5, 0.6)), 8, max_len))
            k = int(rng.integers(k_low, k_high + 1))
        else:
            raise ValueError(lengths)
        total = max(total, 2 * k + 4)
        # Split the budget: head text, k options of >=1 token (marker first), state.
        body = total - 4
        opt_tokens = max(k, body // 3)
        head = max(1, (body - opt_tokens) // 2)
        state = body - opt_tokens - head
        per = [1] * k
        for j in range(opt_tokens - k):
            per[j % k] += 1
        ids = [cls_id] + rng.integers(id_low, vocab, size=head).tolist() + [sep_id]
        markers = []
        for c in per:
            markers.append(len(ids))
            ids += rng.integers(id_low, vocab, size=c).tolist()
        ids.append(sep_id)
        ids += rng.integers(id_low, vocab, size=max(0, state)).tolist()
        ids.append(sep_id)
        ids = ids[:max_len]
        markers = [m for m in markers if m < max_len]
        rows.append(BuiltSequence(ids=ids, markers=markers, nopts=[], full_len=len(ids)))
    return rows
