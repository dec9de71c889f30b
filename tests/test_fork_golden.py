"""The shared-prefix grouping restated in oracle/fork.py against the groups
the reference's own `_text_fork_forward` formed on the same batches
(tests/golden/fork_groups.npz, made by tests/golden/make_fork_golden.py)."""

import json
import os

import numpy as np
import pytest

from oracle import fork

GOLDEN = os.path.join(os.path.dirname(__file__), "golden", "fork_groups.npz")


def cases():
    z = np.load(GOLDEN)
    for m in json.loads(str(z["meta"])):
        n = m["name"]
        yield n, z[f"{n}_ids"], z[f"{n}_real_len"], z[f"{n}_slot"], z[f"{n}_prefix_len"], m["groups"]


@pytest.mark.parametrize("case", list(cases()), ids=lambda c: c[0])
def test_grouping_matches_the_reference(case):
    name, ids, real_len, slot, prefix_len, want = case
    got = fork.plan(ids, real_len, slot, prefix_len)
    assert [(list(m), n) for m, n in got] == [(list(m), n) for m, n in want]


def test_golden_covers_every_rule():
    names = {c[0] for c in cases()}
    assert {"declared", "lcp", "refusals", "empty_suffix", "lcp_floor", "declared_below_floor", "mixed"} <= names
    lone = [g for c in cases() for g in c[5] if len(g[0]) == 1]
    assert lone, "the golden must hold a one-row declared group (the engine runs it whole)"
    assert all(len(m) >= 2 for c in cases() for m, _ in fork.plan(*c[1:5], single=False))
