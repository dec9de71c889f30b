"""Host-side logic that needs no GPU: collate, synthetic checkpoints, label
rules, the replica pool, and the C-ABI library's exported symbols."""

import ctypes
import os
import re

import numpy as np
import pytest

from verdict_b200 import spec as specs
from verdict_b200.batch import BuiltSequence, Layout, collate, decoder_rows, encoder_rows
from verdict_b200.engine import Engine, EngineRow, Overloaded, Pool
from verdict_b200.labels import LabelTableError, derive_branch_ids, derive_letter_ids, slot_labels
from verdict_b200.synth import SyntheticCheckpoint, bf16_round, gen_tensor, tensor_base, with_labels

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


# --- collate (src/scheduler.rs:108-172) --------------------------------------

def test_collate_pads_right_and_packs_markers():
    rows = [BuiltSequence(ids=[5, 6, 7], markers=[2], nopts=[3], prefix_len=1),
            BuiltSequence(ids=[9], markers=[0], nopts=[2])]
    cb = collate(rows, Layout(pad_id=0))
    assert (cb.b, cb.l, cb.k) == (2, 3, 1)
    assert cb.input_ids.tolist() == [5, 6, 7, 9, 0, 0]
    assert cb.attention_mask.tolist() == [1, 1, 1, 1, 0, 0]
    assert cb.marker_pos.tolist() == [2, 0] and cb.marker_mask.tolist() == [True, True]
    assert cb.nopts.tolist() == [3, 2]
    assert [(r.real_len, r.real_k, r.prefix_len) for r in cb.rows] == [(3, 3, 1), (1, 2, 0)]


def test_collate_alignment_and_classes():
    rows = [BuiltSequence(ids=list(range(10)), markers=[1, 4, 6])]
    assert collate(rows, Layout(pad_id=1, seq_align=8)).l == 16
    assert collate(rows, Layout(pad_id=1, fixed_classes=(8, 32, 64))).l == 32
    cb = collate(rows + [BuiltSequence(ids=[3], markers=[0])], Layout(pad_id=1))
    assert cb.k == 3 and cb.marker_mask.tolist() == [True, True, True, True, False, False]
    assert cb.nopts.size == 0  # marker rows carry no nopts


def test_workload_generators_follow_the_benchmark_shapes():
    rng = np.random.default_rng(0)
    rows = decoder_rows(rng, 2000, 152064, lengths="lognormal-9b")
    lens = np.array([len(r.ids) for r in rows])
    assert lens.min() >= 32 and lens.max() <= 4096 and 450 < lens.mean() < 600
    assert all(r.markers == [len(r.ids) - 1] and 2 <= r.nopts[0] <= 8 for r in rows)
    enc = encoder_rows(rng, 200, 250002, lengths="lognormal-xlmr", cls_id=0, sep_id=2, id_low=5)
    for r in enc:
        assert r.ids[0] == 0 and r.ids[-1] == 2 and all(0 < m < len(r.ids) for m in r.markers)
        assert 2 <= len(r.markers) <= 6


def test_bench_marker_head_workloads():
    """bench.py's marker-head encoder batches: BERT rows U[16,128] with 3
    markers and text ids >= 1000, XLM-R rows <= 512 with 2-6 markers; every
    row gets a question type in [0, 3); models route to their row builders."""
    import sys
    sys.path.insert(0, REPO)
    import bench
    bert = bench.make_batches(0, 2, 32, 30522, 7, "marker", 0, "uniform-bert")
    for b in bert:
        assert b.b == 32 and b.k == 3 and 0 <= b.qtype.min() and b.qtype.max() < 3
        for i, r in enumerate(b.rows):
            ids = b.input_ids[i * b.l:i * b.l + r.real_len]
            assert 16 <= r.real_len <= 128 and ids[0] == 101 and ids[-1] == 102
            text = ids[(ids != 101) & (ids != 102)]
            assert text.min() >= 1000
    xlmr = bench.make_batches(0, 1, 64, 250002, 7, "marker", 1, "lognormal-xlmr")[0]
    assert xlmr.l <= 512 and 2 <= xlmr.k <= 6
    assert bench.workload_of(specs.preset("laya-xlmr"), "choice") == "marker"
    assert bench.workload_of(specs.preset("von-base"), "choice") == "von"
    assert bench.workload_of(specs.preset("onejev-9b"), "shared-prefix") == "shared-prefix"


# --- synthetic checkpoints ------------------------------------------------------

def test_bf16_round_ties_to_even():
    x = np.array([1.0, 1.00390625, 1.01171875, -2.5, 3.0e-3], dtype=np.float32)
    y = bf16_round(x)
    assert y[0] == 1.0 and y[1] == 1.0 and y[2] == 1.015625 and y[3] == -2.5
    assert (y.view(np.uint32) & 0xFFFF).max() == 0


def test_generator_rows_match_whole_tensor_and_are_pinned():
    t = gen_tensor(7, "w", (64, 96), 0.5, 0.0)
    rows = gen_tensor(7, "w", (64, 96), 0.5, 0.0, rows=[3, 0, 63])
    np.testing.assert_array_equal(rows, t[[3, 0, 63]])
    assert abs(t.std() - 0.5 / np.sqrt(3)) < 0.02 and np.abs(t).max() <= 0.5
    # known values: the CUDA generator (csrc/synth.cuh) must produce these bits
    assert tensor_base(7, "w") == 0xFCE7BE5EFD0B60C5
    assert [hex(x) for x in t.view(np.uint32)[0, :4]] == ["0xbe350000", "0x3e180000", "0x3ea70000", "0xbe430000"]


def test_checkpoint_inventory_matches_hf_names():
    ck = SyntheticCheckpoint(specs.preset("onejev-9b", layers=1))
    names = ck.names()
    assert "model.layers.0.self_attn.q_norm.weight" in names and "lm_head.weight" in names
    assert ck.table["model.layers.0.mlp.gate_proj.weight"][0] == (12288, 4096)
    g = SyntheticCheckpoint(specs.preset("decider-2b", layers=1))
    assert "lm_head.weight" not in g.names() and g.head_name() == "model.embed_tokens.weight"
    e = SyntheticCheckpoint(specs.preset("laya-xlmr", layers=1))
    assert "head.layers.1.self_attn.in_proj_weight" in e.names() and "scorer.3.bias" in e.names()


def test_preset_flop_accounting():
    s = specs.preset("onejev-9b")
    assert abs(specs.linear_flops_per_token(s) / 1e9 - 15.435) < 0.01
    assert specs.attention_flops(s, 100) == 327680 * 100 * 101


def test_synthetic_labels_distinct_and_in_range():
    s = with_labels(specs.preset("onejev-9b"))
    ids = s["label_ids"]
    assert len(ids) == 256 and len(set(ids)) == 256 and min(ids) >= 3 and max(ids) < s["vocab"]
    assert len(with_labels(specs.preset("decider-2b"))["label_ids"]) == 255


# --- label rules (src/tokenize.rs:96-171) ---------------------------------------

class _Tok:
    def __init__(self, vocab):
        self.v = vocab
        self.inv = {i: s for s, i in vocab.items()}

    def encode(self, text, add_special_tokens=False):
        return [self.v[text]] if text in self.v else [0, 0]

    def decode(self, ids):
        return "".join(self.inv[i] for i in ids)


def test_label_rules():
    labels = slot_labels()
    assert len(labels) == 256 and labels[:3] == ["A", "B", "C"] and "BQ" not in labels
    vocab = {lab: 100 + i for i, lab in enumerate(labels)}
    assert derive_branch_ids(_Tok(vocab)) == [100 + i for i in range(256)]
    letters = {chr(65 + i): i + 1 for i in range(26)}
    with pytest.raises(LabelTableError):
        derive_letter_ids(_Tok(letters))  # too few single-token labels
    pairs = dict(letters)
    for a in range(26):
        for b in range(26):
            pairs[chr(65 + a) + chr(65 + b)] = 1000 + a * 26 + b
    t = derive_letter_ids(_Tok(pairs))
    assert len(t) == 255 and t[26] == 1000


# --- replica pool (src/pipeline.rs:329-352) ---------------------------------------

class _Fake(Engine):
    def __init__(self, name, busy=False):
        self.name, self.busy, self.calls = name, busy, 0

    def infer(self, batch):
        self.calls += 1
        if self.busy:
            raise Overloaded(self.name)
        return [EngineRow([float(len(self.name))])]

    def health(self):
        return True


def test_pool_round_robin_and_spill_over():
    a, b, c = _Fake("a"), _Fake("bb", busy=True), _Fake("ccc")
    pool = Pool([a, b, c])
    outs = [pool.infer(None)[0].logits[0] for _ in range(3)]
    assert outs == [1.0, 3.0, 3.0]  # b spills to c
    assert a.calls == 1 and b.calls == 1 and c.calls == 2
    with pytest.raises(Overloaded):
        Pool([_Fake("x", busy=True)]).infer(None)


# --- the C-ABI library ---------------------------------------------------------------

def declared_symbols():
    out = []
    for name in ("vdexec.h", "vdexec_kernels.h"):
        text = open(os.path.join(REPO, "include", name)).read()
        out += re.findall(r"VD_API\s+[\w\s\*]+?\b(vdk?_\w+)\s*\(", text)
    return out


def test_library_exports_every_declared_symbol():
    from verdict_b200 import _abi
    lib = _abi.load()
    syms = declared_symbols()
    assert len(syms) >= 15
    for s in syms:
        assert hasattr(lib, s), f"{s} declared in include/ but not exported"
        assert s in _abi.SIGNATURES, f"{s} has no ctypes signature"
    assert lib.vd_abi_version() == 2


def test_headers_compile_as_c_and_match_the_python_mirror(tmp_path):
    """include/*.h are plain C, and vd_batch / vd_stats have the layout the
    ctypes mirror (verdict_b200/_abi.py) assumes: size and every field offset."""
    import shutil
    import subprocess
    from verdict_b200 import _abi
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "vdexec.h"', '#include "vdexec_kernels.h"',
             'int main(void) {']
    for cname, mirror in (("vd_batch", _abi.VdBatch), ("vd_stats", _abi.VdStats)):
        lines.append(f'  printf("{cname} size %zu\\n", sizeof({cname}));')
        for field, _ in mirror._fields_:
            lines.append(f'  printf("{cname} {field} %zu\\n", offsetof({cname}, {field}));')
    lines += ['  printf("VD_K_COUNT %d\\n", (int)VD_K_COUNT);', '  return 0;', '}']
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines) + "\n")
    exe = tmp_path / "layout"
    subprocess.run([cc, "-std=c99", "-Wall", "-Werror", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = {}
    for line in subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout.splitlines():
        *key, value = line.split()
        got[" ".join(key)] = int(value)
    for cname, mirror in (("vd_batch", _abi.VdBatch), ("vd_stats", _abi.VdStats)):
        assert got[f"{cname} size"] == ctypes.sizeof(mirror), cname
        for field, _ in mirror._fields_:
            assert got[f"{cname} {field}"] == getattr(mirror, field).offset, (cname, field)
    assert got["VD_K_COUNT"] == len(_abi.KERNEL_CLASSES)


def test_open_without_gpu_fails_cleanly():
    import torch
    if torch.cuda.is_available():
        pytest.skip("a GPU is present")
    from verdict_b200 import _abi
    lib = _abi.load()
    err = ctypes.create_string_buffer(512)
    h = ctypes.c_void_p()
    spec = b'{"arch":"decoder","hidden":256,"layers":1,"heads":2,"kv_heads":1,"head_dim":128,"ffn":256,' \
           b'"vocab":512,"label_ids":[1,2,3]}'
    rc = lib.vd_open(spec, 0, None, ctypes.byref(h), err, len(err))
    assert rc != 0 and err.value and not h.value


def test_open_rejects_bad_specs_before_touching_the_device():
    from verdict_b200 import _abi
    lib = _abi.load()
    err = ctypes.create_string_buffer(512)
    h = ctypes.c_void_p()
    rc = lib.vd_open(b'{"arch":"decoder","hidden":100,"layers":1,"heads":2,"kv_heads":1,"head_dim":128,'
                     b'"ffn":256,"vocab":512,"label_ids":[1]}', 0, None, ctypes.byref(h), err, len(err))
    assert rc == _abi.VD_ESPEC and b"hidden" in err.value
    rc = lib.vd_open(b'{"arch":"decoder","hidden":256,"layers":1,"heads":2,"kv_heads":1,"head_dim":128,'
                     b'"ffn":256,"vocab":512}', 0, None, ctypes.byref(h), err, len(err))
    assert rc == _abi.VD_ESPEC and b"label_ids" in err.value
    rc = lib.vd_open(b'{not json', 0, None, ctypes.byref(h), err, len(err))
    assert rc == _abi.VD_EINVAL
