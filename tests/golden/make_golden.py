"""Generate the golden fixtures by running the reference's OWN code on CPU in fp32.

Run in a container that has the reference checkout (read-only) and transformers:
    python tests/golden/make_golden.py [/path/to/reference]

Decoder cases import `executor/torch_exec.py` unchanged and call
`GraphRunner._eager_readout` (`executor/torch_exec.py:255-261`) on an HF model
built from config in fp32 (the executor's CPU dtype, `:2352`), whose weights are
replaced by this repo's synthetic checkpoint (`verdict_b200/synth.py`), with
`head_w = model.get_output_embeddings().weight[letter_ids].float()` (`:2385`).
The label table comes from the reference's own `derive_branch_ids` /
`derive_letter_ids` (`:2254-2323`) run on a synthetic word-level tokenizer.

Encoder cases build the reference's `DecisionModel` / `Wrapper`
(`convert/marker_head/marker_head_converter.py:19-66`) over an HF BERT /
XLM-R encoder, load the synthetic weights, and run the reference's own probe
batches `marker_head_probe.cases` (`convert/marker_head/marker_head_probe.py:35-56`)
plus one seeded ragged batch.

Output: one small .npz per case next to this script.  Nothing at test time
reads the reference; the tests read these files.
"""

from __future__ import annotations

import importlib.util
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import collate, Layout, decoder_rows, encoder_rows  # noqa: E402
from verdict_b200.synth import SyntheticCheckpoint  # noqa: E402

torch.set_grad_enabled(False)


def load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def synthetic_tokenizer(vocab_size: int, seed: int):
    """Word-level tokenizer whose option labels sit at seeded, scattered ids."""
    from tokenizers import Tokenizer, models, pre_tokenizers
    from transformers import PreTrainedTokenizerFast

    letters = [chr(c) for c in range(65, 91)]
    labels = letters + [a + b for a in letters for b in letters]
    rng = np.random.default_rng(seed)
    ids = rng.choice(np.arange(3, vocab_size), size=len(labels), replace=False)
    vocab = {"<unk>": 0, "<pad>": 1, "<eos>": 2}
    used = set(int(i) for i in ids)
    for lab, i in zip(labels, ids):
        vocab[lab] = int(i)
    for i in range(3, vocab_size):
        if i not in used:
            vocab[f"t{i}"] = i
    tk = Tokenizer(models.WordLevel(vocab=vocab, unk_token="<unk>"))
    tk.pre_tokenizer = pre_tokenizers.Whitespace()
    return PreTrainedTokenizerFast(tokenizer_object=tk, unk_token="<unk>", pad_token="<pad>")


def load_synthetic(model, ckpt: SyntheticCheckpoint, prefix: str = "", extra_ok=()):
    """Overwrite every parameter the synthetic checkpoint defines; report the rest."""
    sd = model.state_dict()
    missing = []
    for name, t in sd.items():
        key = prefix + name
        if key in ckpt.table:
            t.copy_(torch.from_numpy(ckpt.get(key)).reshape(t.shape))
        elif not any(name.startswith(x) or x in name for x in extra_ok):
            missing.append(name)
    return missing


def hf_decoder(spec):
    from transformers import AutoModelForCausalLM, GemmaConfig, Qwen2Config, Qwen3Config

    common = dict(hidden_size=spec["hidden"], intermediate_size=spec["ffn"],
                  num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"],
                  num_key_value_heads=spec["kv_heads"], head_dim=spec["head_dim"],
                  vocab_size=spec["vocab"], rms_norm_eps=spec["rms_eps"],
                  max_position_embeddings=8192, tie_word_embeddings=spec["tied"],
                  pad_token_id=1, bos_token_id=2, eos_token_id=2)
    if spec["style"] == "qwen3_5":
        from transformers import Qwen3_5TextConfig
        cfg = Qwen3_5TextConfig(
            rope_parameters={"rope_type": "default", "rope_theta": spec["rope_theta"],
                             "partial_rotary_factor": spec["partial_rotary"]},
            layer_types=list(spec["layer_types"]), linear_conv_kernel_dim=spec["conv_kernel"],
            linear_key_head_dim=spec["lin_k_dim"], linear_value_head_dim=spec["lin_v_dim"],
            linear_num_key_heads=spec["lin_k_heads"], linear_num_value_heads=spec["lin_v_heads"],
            hidden_act="silu", **common)
    elif spec["style"] == "qwen3":
        cfg = Qwen3Config(rope_theta=spec["rope_theta"], attention_bias=spec["qkv_bias"], **common)
    elif spec["style"] == "qwen2":
        # Qwen2: bias on q/k/v only, no q/k norm
        cfg = Qwen2Config(rope_theta=spec["rope_theta"], **common)
    else:
        cfg = GemmaConfig(rope_theta=spec["rope_theta"], hidden_act="gelu_pytorch_tanh",
                          hidden_activation="gelu_pytorch_tanh", **common)
    model = AutoModelForCausalLM.from_config(cfg, attn_implementation="sdpa", dtype=torch.float32)
    model.eval()
    missing = load_synthetic(model, SyntheticCheckpoint(spec), extra_ok=("rotary_emb",))
    if spec["tied"]:
        missing = [m for m in missing if m != "lm_head.weight"]
    assert not missing, f"parameters without synthetic values: {missing}"
    return model


def decoder_case(ex, name, spec, batch, note):
    tok = synthetic_tokenizer(spec["vocab"], seed=spec["seed"] + 7)
    if spec["family"] == "letter_branches":
        table = ex.derive_branch_ids(tok)
    else:
        table = ex.derive_letter_ids(tok)
    spec = dict(spec, label_ids=[int(i) for i in table])
    model = hf_decoder(spec)
    letter_ids = torch.tensor(table, dtype=torch.long)
    head_w = model.get_output_embeddings().weight[letter_ids].float()
    runner = ex.GraphRunner.__new__(ex.GraphRunner)
    runner.model, runner.head_w, runner.pad_id = model, head_w, 1
    ids = torch.from_numpy(batch.input_ids).view(batch.b, batch.l)
    mask = torch.from_numpy(batch.attention_mask).view(batch.b, batch.l)
    slot_idx = torch.from_numpy(batch.marker_pos.reshape(batch.b, batch.k)[:, 0].copy())
    slot_batch = torch.arange(batch.b)
    logits = runner._eager_readout(ids, mask, slot_batch, slot_idx).numpy()
    save(name, spec, batch, logits, note, label_table=np.array(table, dtype=np.int64),
         tok_vocab=spec["vocab"], tok_seed=spec["seed"] + 7)


def save(name, spec, batch, logits, note, **extra):
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(
        path, spec=json.dumps(spec), note=note,
        input_ids=batch.input_ids, attention_mask=batch.attention_mask,
        marker_pos=batch.marker_pos, marker_mask=batch.marker_mask, qtype=batch.qtype,
        nopts=batch.nopts, real_len=batch.real_len(), real_k=batch.real_k(),
        prefix_len=batch.prefix_len(), b=batch.b, l=batch.l, k=batch.k,
        logits=logits.astype(np.float32), **extra)
    print(f"wrote {path}: logits {logits.shape}")


def padded_batch(ids, lens, pad_id, markers=None, nopts=None):
    """A CollatedBatch from explicit [b, l] ids and lengths (slot = last token)."""
    from verdict_b200.batch import BuiltSequence
    rows = []
    for i, n in enumerate(lens):
        m = [n - 1] if markers is None else markers[i]
        k = None if nopts is None else nopts[i]
        rows.append(BuiltSequence(ids=[int(x) for x in ids[i][:n]], markers=m,
                                  nopts=[] if k is None else [k]))
    return collate(rows, Layout(pad_id=pad_id))


def encoder_spec(style):
    base = specs.preset("laya-bert" if style == "bert" else "laya-xlmr",
                        hidden=128, layers=2, heads=2, ffn=256, vocab=1000)
    return base


def hf_decision_model(ref_root, spec):
    from transformers import AutoModel, BertConfig, XLMRobertaConfig

    sys.path.insert(0, os.path.join(ref_root, "convert"))
    sys.path.insert(0, os.path.join(ref_root, "convert", "marker_head"))
    conv = load_module("marker_head_converter",
                       os.path.join(ref_root, "convert", "marker_head", "marker_head_converter.py"))
    probe = load_module("marker_head_probe",
                        os.path.join(ref_root, "convert", "marker_head", "marker_head_probe.py"))
    common = dict(hidden_size=spec["hidden"], num_hidden_layers=spec["layers"],
                  num_attention_heads=spec["heads"], intermediate_size=spec["ffn"],
                  vocab_size=spec["vocab"], max_position_embeddings=spec["max_pos"],
                  type_vocab_size=spec["type_vocab"], layer_norm_eps=spec["ln_eps"],
                  pad_token_id=spec["pad_id"], hidden_act="gelu",
                  hidden_dropout_prob=0.0, attention_probs_dropout_prob=0.0)
    cfg = BertConfig(**common) if spec["style"] == "bert" else XLMRobertaConfig(**common)
    enc = AutoModel.from_config(cfg, attn_implementation="sdpa")
    model = conv.DecisionModel(enc, spec["head_layers"], 2)
    model.eval()
    missing = load_synthetic(model, SyntheticCheckpoint(spec),
                             extra_ok=("act_head", "temperature", "pooler", "position_ids",
                                       "token_type_ids"))
    assert not missing, f"parameters without synthetic values: {missing}"
    return conv, probe, conv.Wrapper(model).eval()


def encoder_case(ref_root, name, spec, seed):
    conv, probe, wrapper = hf_decision_model(ref_root, spec)
    batches = []
    for ids, amask, pos, pmask, qtype in probe.cases(2, spec["vocab"], spec["pad_id"]):
        batches.append((ids, amask, pos, pmask, qtype))
    rng = np.random.default_rng(seed)
    cls_id, sep_id = (101, 102) if spec["style"] == "bert" else (0, 2)
    rows = encoder_rows(rng, 6, spec["vocab"], lengths="lognormal-xlmr", cls_id=cls_id,
                        sep_id=sep_id, id_low=5, max_len=spec["max_pos"] - 2)
    cb = collate(rows, Layout(pad_id=spec["pad_id"]))
    qt = rng.integers(0, 3, size=cb.b)
    batches.append((cb.input_ids.reshape(cb.b, cb.l), cb.attention_mask.reshape(cb.b, cb.l),
                    cb.marker_pos.reshape(cb.b, cb.k), cb.marker_mask.reshape(cb.b, cb.k), qt))
    for j, (ids, amask, pos, pmask, qtype) in enumerate(batches):
        with torch.no_grad():
            logits, _ = wrapper(torch.from_numpy(ids), torch.from_numpy(amask),
                                torch.from_numpy(pos), torch.from_numpy(pmask),
                                torch.from_numpy(np.asarray(qtype, dtype=np.int64)))
        b, l = ids.shape
        k = pos.shape[1]
        path = os.path.join(HERE, f"{name}_{j}.npz")
        np.savez_compressed(
            path, spec=json.dumps(spec),
            note=("marker_head_probe.cases" if j < len(batches) - 1 else "seeded ragged batch"),
            input_ids=ids.reshape(-1).astype(np.int64), attention_mask=amask.reshape(-1).astype(np.int64),
            marker_pos=pos.reshape(-1).astype(np.int64), marker_mask=pmask.reshape(-1).astype(bool),
            qtype=np.asarray(qtype, dtype=np.int64), real_len=amask.sum(1).astype(np.int64),
            b=b, l=l, k=k, logits=logits.numpy().astype(np.float32))
        print(f"wrote {path}: logits {tuple(logits.shape)}")


def main():
    if len(sys.argv) != 2:
        sys.exit(f"usage: python {os.path.basename(__file__)} <path of the reference checkout>")
    ref_root = sys.argv[1]
    ex = load_module("torch_exec", os.path.join(ref_root, "executor", "torch_exec.py"))

    qwen = specs.preset("onejev-9b", hidden=256, layers=2, heads=4, kv_heads=2, head_dim=128,
                        ffn=512, vocab=8448, seed=101)
    rng = np.random.default_rng(11)
    rows = decoder_rows(rng, 5, qwen["vocab"], lengths="fixed:8")
    lens = [1, 17, 64, 40, 130]
    for r, n in zip(rows, lens):
        r.ids = rng.integers(3, qwen["vocab"], size=n).tolist()
        r.markers = [n - 1]
    decoder_case(ex, "qwen3_tiny_ragged", qwen, collate(rows, Layout(pad_id=1)),
                 "ragged letter_branches batch, lengths 1/17/64/40/130, rng seed 11")

    # The executor's packed-vs-padded self-check batch (`executor/torch_exec.py:2500-2506`):
    # torch CPU generator seeded 20261028, ids in [1, 8192), lengths 96/40/71.
    gen = torch.Generator(device="cpu").manual_seed(20261028)
    ids = torch.randint(1, 8192, (3, 96), generator=gen).numpy()
    decoder_case(ex, "qwen3_tiny_selfcheck", qwen,
                 padded_batch(ids, (96, 40, 71), pad_id=1, nopts=(4, 2, 8)),
                 "executor packed self-check ids (seed 20261028), lengths 96/40/71")

    qbias = dict(qwen, style="qwen2", qkv_bias=True, qk_norm=False, seed=202)
    rng = np.random.default_rng(12)
    rows = decoder_rows(rng, 4, qbias["vocab"], lengths="lognormal-9b")
    for r in rows:
        n = min(len(r.ids), 200)
        r.ids, r.markers = r.ids[:n], [n - 1]
    decoder_case(ex, "qwen2style_tiny_bias", qbias, collate(rows, Layout(pad_id=1)),
                 "attention bias on, q/k norm off, rng seed 12")

    gemma = specs.preset("decider-2b", hidden=256, layers=2, heads=2, kv_heads=1, head_dim=256,
                         ffn=512, vocab=8448, seed=303)
    rng = np.random.default_rng(13)
    rows = decoder_rows(rng, 4, gemma["vocab"], lengths="uniform-2b")
    for r in rows:
        n = min(len(r.ids), 150)
        r.ids, r.markers = r.ids[:n], [n - 1]
    decoder_case(ex, "gemma_tiny_readout", gemma, collate(rows, Layout(pad_id=1)),
                 "Gemma-style letter_readout (255 labels), rng seed 13")

    # Qwen3.5 text stacks (gated delta net + gated full attention), the executor's
    # fp32 CPU path through HF's torch fallbacks (chunked gated delta rule, Conv1d).
    hybrid = specs.preset("onejev16-9b", hidden=256, layers=4, heads=2, kv_heads=1, head_dim=256,
                          ffn=512, vocab=8448, lin_k_heads=2, lin_v_heads=4, seed=404)
    rng = np.random.default_rng(16)
    rows = decoder_rows(rng, 4, hybrid["vocab"], lengths="fixed:8")
    for r, n in zip(rows, [1, 9, 70, 150]):
        r.ids = rng.integers(3, hybrid["vocab"], size=n).tolist()
        r.markers = [n - 1]
    decoder_case(ex, "qwen35_tiny_hybrid", hybrid, collate(rows, Layout(pad_id=1)),
                 "Qwen3.5 text stack, layers linear/linear/linear/full, lengths 1/9/70/150, rng seed 16")
    hybrid2 = dict(hybrid, layers=3, layer_types=["linear_attention", "full_attention", "linear_attention"],
                   family="letter_readout", seed=405)
    rng = np.random.default_rng(17)
    rows = decoder_rows(rng, 3, hybrid2["vocab"], lengths="uniform-2b")
    for r in rows:
        n = min(len(r.ids), 200)
        r.ids, r.markers = r.ids[:n], [n - 1]
    decoder_case(ex, "qwen35_tiny_lastlinear", hybrid2, collate(rows, Layout(pad_id=1)),
                 "Qwen3.5 text stack ending in a gated-delta-net layer, letter_readout, rng seed 17")

    encoder_case(ref_root, "bert_tiny_marker", encoder_spec("bert"), seed=14)
    encoder_case(ref_root, "xlmr_tiny_marker", encoder_spec("xlmr"), seed=15)


if __name__ == "__main__":
    main()
