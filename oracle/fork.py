"""Shared-prefix fork grouping — TEST INFRASTRUCTURE ONLY.

Restates the row grouping of `_text_fork_forward`
(`executor/torch_exec.py:1935-1977`), so that the tests can say which rows the
engine must fork and at which prefix length:
- a row whose slot is not its last token runs whole;
- a row with a declared prefix_len >= 32 and < real_len is grouped with the
  rows that declare the same length and the same prefix tokens;
- any other row longer than 32 tokens is grouped by its first 32 tokens; such
  a group of two or more rows forks at its members' longest common prefix;
- a group whose prefix is shorter than 32 tokens, or that leaves a member no
  suffix, runs its rows whole.
The engine runs groups of one row whole too (the reference forks a lone row
with a declared prefix, computing the same function in two steps);
`plan(..., single=False)` drops those groups, as the engine does.

The fork is exact arithmetic of the whole-row forward (the reference gates it
at 5e-2 of the whole-row softmax, `executor/torch_exec.py:2024-2066`), so the
parity check of forked rows is the oracle's whole-row forward.
"""

from __future__ import annotations

import numpy as np

FLOOR = 32  # TEXT_FORK_MIN_PREFIX = GRAPH_PREFIX_STEP (executor/torch_exec.py:41,363)


def plan(ids: np.ndarray, real_len, slot, prefix_len=None, single: bool = True):
    """[(sorted member rows, prefix length)] in first-appearance order."""
    b = ids.shape[0]
    groups, order = {}, []
    splits = []
    for i in range(b):
        n = int(real_len[i])
        declared = int(prefix_len[i]) if prefix_len is not None else 0
        if int(slot[i]) != n - 1:
            continue
        if FLOOR <= declared < n:
            key = ("declared", ids[i, :declared].tobytes(), declared)
            if key not in groups:
                groups[key] = []
                order.append(key)
            groups[key].append(i)
            continue
        splits.append(i)
    for i in splits:
        if int(real_len[i]) <= FLOOR:
            continue
        key = ("lcp", ids[i, :FLOOR].tobytes(), 0)
        if key not in groups:
            groups[key] = []
            order.append(key)
        groups[key].append(i)
    out = []
    for key in order:
        members = groups[key]
        n = key[2]
        if key[0] == "lcp":
            if len(members) < 2:
                continue
            mlen = min(int(real_len[i]) for i in members)
            eq = (ids[members, :mlen] == ids[members[0], :mlen]).all(0)
            nz = np.flatnonzero(~eq)
            n = int(nz[0]) if nz.size else int(mlen)
        if n < FLOOR or any(int(real_len[i]) - n == 0 for i in members):
            continue
        if not single and len(members) < 2:
            continue
        out.append((sorted(members), n))
    return out
