"""Golden shared-prefix groupings from the reference's own `_text_fork_forward`.

Run in a container that has the reference checkout (read-only) and torch:
    python tests/golden/make_fork_golden.py [/path/to/reference]

`executor/torch_exec.py` is imported unchanged.  `_text_fork_forward`
(`:1935-2022`) is called on CPU with `fork_graphs=None`, a stub model whose
whole-row forward returns zeros, and `_fork_one_group` replaced by a recorder
that answers each group's rows with (group number, prefix length, member
index) as their logits, so the returned rows tell which rows the reference
forked together and at which prefix length.  The batches are seeded and cover
declared prefixes, the 32-token common-prefix key, and every refusal rule.

Output: `fork_groups.npz` next to this script.  Nothing at test time reads the
reference.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys
from types import SimpleNamespace

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def load_executor(ref_root):
    spec = importlib.util.spec_from_file_location("torch_exec", os.path.join(ref_root, "executor", "torch_exec.py"))
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    mod.DEV = "cpu"
    return mod


def reference_groups(ex, ids, real_len, slot, prefix_len):
    b, L = ids.shape
    width = 8
    calls = []

    def recorder(model, head_w, pad_id, ids1, n, suffixes, fork_graphs, prefix_bytes=b""):
        calls.append(n)
        g = len(calls)
        out = torch.zeros(len(suffixes), width)
        for r in range(len(suffixes)):
            out[r, 0], out[r, 1], out[r, 2] = g, n, r
        return out, False

    class Stub:
        def model(self, input_ids=None, use_cache=False, **kw):
            return SimpleNamespace(last_hidden_state=torch.zeros(input_ids.shape[0], input_ids.shape[1], 4))

    ex._fork_one_group = recorder
    mask = np.zeros((b, L), np.int64)
    for i, n in enumerate(real_len):
        mask[i, :n] = 1
    head_w = torch.zeros(width, 4)
    out = ex._text_fork_forward(Stub(), None, head_w, 0, torch.from_numpy(ids), torch.from_numpy(mask),
                                torch.from_numpy(np.asarray(slot, np.int64)), None,
                                list(prefix_len) if prefix_len is not None else None)
    if out is None:
        return []
    groups = {}
    for i in range(b):
        g = int(out[i, 0])
        if g > 0:
            groups.setdefault(g, (int(out[i, 1]), []))[1].append(i)
    return [(sorted(rows), n) for g, (n, rows) in sorted(groups.items())]


def make_cases():
    rng = np.random.default_rng(20261201)
    V = 5000

    def toks(n):
        return rng.integers(3, V, size=n).tolist()

    cases = []
    # 1. declared prefixes: three groups of three rows, two unrelated rows
    rows, pl = [], []
    for plen in (40, 100, 300):
        pre = toks(plen)
        for _ in range(3):
            rows.append(pre + toks(int(rng.integers(5, 120))))
            pl.append(plen)
    for _ in range(2):
        rows.append(toks(int(rng.integers(40, 200))))
        pl.append(0)
    cases.append(("declared", rows, pl, None))
    # 2. no declared prefix: a 50-token common prefix (common-prefix key)
    pre = toks(50)
    rows = [pre + toks(int(rng.integers(3, 90))) for _ in range(4)] + [toks(70)]
    cases.append(("lcp", rows, [0] * len(rows), None))
    # 3. refusals: declared >= real_len, short rows, slot not last, a lone declared row
    pre = toks(64)
    rows = [pre + toks(10), pre + toks(12), pre + toks(20), toks(20), toks(31), pre[:40] + toks(30)]
    pl = [len(rows[0]), 64, 64, 0, 0, 40]
    slot = [len(r) - 1 for r in rows]
    slot[2] = len(rows[2]) - 2
    cases.append(("refusals", rows, pl, slot))
    # 4. a member with no suffix past the common prefix refuses the whole group
    pre = toks(60)
    rows = [pre + toks(30), pre + toks(25), list(pre)]
    cases.append(("empty_suffix", rows, [0, 0, 0], None))
    # 5. same first 32 tokens, then diverging at different points
    head = toks(32)
    rows = [head + toks(40), head + toks(5) + toks(30), head + toks(60)]
    cases.append(("lcp_floor", rows, [0, 0, 0], None))
    # 6. a declared prefix below the floor falls back to the common-prefix key
    pre = toks(45)
    rows = [pre + toks(20), pre + toks(33)]
    cases.append(("declared_below_floor", rows, [20, 20], None))
    # 7. two declared groups with equal lengths but different tokens, mixed with lcp rows
    a, b2, c = toks(48), toks(48), toks(80)
    rows = [a + toks(9), b2 + toks(7), a + toks(14), b2 + toks(3), c + toks(11), c + toks(19)]
    cases.append(("mixed", rows, [48, 48, 48, 48, 0, 0], None))
    return cases


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.basename(__file__)} <path of the reference checkout>")
    ref_root = sys.argv[1]
    ex = load_executor(ref_root)
    out = {}
    meta = []
    for name, rows, pl, slot in make_cases():
        L = max(len(r) for r in rows)
        ids = np.zeros((len(rows), L), np.int64)
        for i, r in enumerate(rows):
            ids[i, :len(r)] = r
        real_len = np.array([len(r) for r in rows], np.int64)
        slot = np.array(slot if slot is not None else real_len - 1, np.int64)
        prefix_len = np.array(pl, np.int64)
        groups = reference_groups(ex, ids, real_len, slot, prefix_len)
        out[f"{name}_ids"] = ids
        out[f"{name}_real_len"] = real_len
        out[f"{name}_slot"] = slot
        out[f"{name}_prefix_len"] = prefix_len
        meta.append({"name": name, "groups": groups})
        print(name, groups)
    out["meta"] = np.array(json.dumps(meta))
    np.savez_compressed(os.path.join(HERE, "fork_groups.npz"), **out)


if __name__ == "__main__":
    main()
