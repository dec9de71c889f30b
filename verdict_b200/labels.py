"""Option-label tables: which LM-head rows the letter families read.

Restates the two rules the reference implements twice (Rust and Python):
- letter_readout: `derive_letter_table` (`src/tokenize.rs:96-134`) /
  `derive_letter_ids` (`executor/torch_exec.py:2254-2290`): the single-token ids
  of "A".."Z", then of "AA".."ZZ" in order, until 255 labels.
- letter_branches: `derive_branch_table` (`src/tokenize.rs:136-171`) /
  `derive_branch_ids` (`executor/torch_exec.py:2292-2323`): the 26 letters (each
  must round-trip as one token), then the pair labels of `slot_labels()`
  (`src/family/letter_branches.rs:30-44`), i.e. "AA".."ZZ" minus the 25 pairs
  in NOT_ONE_TOKEN, up to 256 slots; pairs are appended only if all of them
  are single round-trip tokens.
Both reject tables with duplicate ids.  The tokenizer is any object with
`encode(text, add_special_tokens=False) -> list[int]` and `decode(ids) -> str`.
"""

from __future__ import annotations

MAX_LETTERS = 255
BRANCH_MAX_SLOTS = 256
LETTERS = [chr(c) for c in range(ord("A"), ord("Z") + 1)]
NOT_ONE_TOKEN = frozenset({
    "BQ", "BZ", "CJ", "CQ", "CZ", "DQ", "DZ", "EJ", "EY", "FJ", "FQ", "FV",
    "FZ", "GJ", "GK", "GQ", "GZ", "HJ", "IY", "JF", "JG", "JH", "JL", "JN", "JQ",
})


class LabelTableError(RuntimeError):
    pass


def slot_labels() -> list:
    out = list(LETTERS)
    for a in LETTERS:
        for b in LETTERS:
            if len(out) >= BRANCH_MAX_SLOTS:
                return out
            pair = a + b
            if pair not in NOT_ONE_TOKEN:
                out.append(pair)
    return out


def _encode(tok, text):
    return list(tok.encode(text, add_special_tokens=False))


def derive_letter_ids(tok) -> list:
    def single(name):
        ids = _encode(tok, name)
        return ids[0] if len(ids) == 1 else None

    table = [i for i in (single(c) for c in LETTERS) if i is not None]
    for a in LETTERS:
        if len(table) >= MAX_LETTERS:
            break
        for b in LETTERS:
            if len(table) >= MAX_LETTERS:
                break
            i = single(a + b)
            if i is not None:
                table.append(i)
    if len(table) < MAX_LETTERS:
        raise LabelTableError(
            f"this tokenizer has only {len(table)} single-token upper-case letter names; "
            f"the letter-readout family needs {MAX_LETTERS}")
    if len(set(table)) != len(table):
        raise LabelTableError("two option labels tokenize to the same id")
    return table


def derive_branch_ids(tok) -> list:
    def one(label):
        enc = _encode(tok, label)
        if len(enc) == 1 and tok.decode(enc) == label:
            return enc[0]
        return None

    table = []
    for label in LETTERS:
        i = one(label)
        if i is None:
            raise LabelTableError(
                f"answer slot {label!r} is not a single round-trip token; the "
                f"letter-branches family requires all 26 letters")
        table.append(i)
    extra = [one(p) for p in slot_labels()[len(LETTERS):]]
    if all(i is not None for i in extra):
        table += extra
    if len(set(table)) != len(table):
        raise LabelTableError("two option labels tokenize to the same id")
    return table


def derive_label_ids(family: str, tok) -> list:
    if family == "letter_branches":
        return derive_branch_ids(tok)
    if family == "letter_readout":
        return derive_letter_ids(tok)
    raise LabelTableError(f"family {family!r} has no option-label table")
