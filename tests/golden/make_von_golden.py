"""Golden independent-options (von) outputs from HF transformers' ModernBertModel.

    python tests/golden/make_von_golden.py

The reference serves this family through an ONNX export of
`VonExportWrapper` (`convert/independent_options/independent_options_converter.py:22-36`):
HF `ModernBertModel` called with an explicit {"full_attention", "sliding_attention"}
additive mask pair and option-invariant position ids, then a scorer on the
marker rows.  Here the encoder is HF's own ModernBertModel (eager attention,
fp32, CPU) with this repo's synthetic weights; the masks and positions follow
the reference's Rust builder (`independent_options_tensors`,
`src/engine.rs:531-590`, restated in `oracle/von.py` and checked against
hand-worked cases in `tests/test_von.py`); the scorer (in the absent `von`
package) is taken to have the marker head's layout.  Output:
`von_tiny_*.npz` next to this script.
"""

from __future__ import annotations

import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)

from oracle.von import von_allowed, von_layout  # noqa: E402
from verdict_b200 import spec as specs  # noqa: E402
from verdict_b200.batch import Layout, collate, von_rows  # noqa: E402
from verdict_b200.synth import SyntheticCheckpoint  # noqa: E402

torch.set_grad_enabled(False)


def hf_model(spec):
    from transformers import ModernBertConfig, ModernBertModel
    cfg = ModernBertConfig(
        vocab_size=spec["vocab"], hidden_size=spec["hidden"], intermediate_size=spec["ffn"],
        num_hidden_layers=spec["layers"], num_attention_heads=spec["heads"], hidden_activation="gelu",
        max_position_embeddings=spec["max_pos"], norm_eps=spec["ln_eps"], norm_bias=False,
        pad_token_id=spec["pad_id"], layer_types=list(spec["layer_types"]),
        local_attention=2 * spec["sliding_window"],
        rope_parameters={"full_attention": {"rope_type": "default", "rope_theta": spec["global_theta"]},
                         "sliding_attention": {"rope_type": "default", "rope_theta": spec["local_theta"]}})
    model = ModernBertModel(cfg)
    model.config._attn_implementation = "eager"
    model.eval()
    ckpt = SyntheticCheckpoint(spec)
    missing = []
    for name, t in model.state_dict().items():
        key = "encoder." + name
        if key in ckpt.table:
            t.copy_(torch.from_numpy(ckpt.get(key)).reshape(t.shape))
        else:
            missing.append(name)
    assert not missing, f"parameters without synthetic values: {missing}"
    return model, ckpt


def scorer(ckpt, rep):
    g = {n: torch.from_numpy(ckpt.get(n)) for n in ("scorer.0.weight", "scorer.0.bias", "scorer.1.weight",
                                                    "scorer.1.bias", "scorer.3.weight", "scorer.3.bias")}
    y = torch.nn.functional.layer_norm(rep, (rep.shape[-1],), g["scorer.0.weight"], g["scorer.0.bias"], 1e-5)
    y = torch.nn.functional.gelu(y @ g["scorer.1.weight"].T + g["scorer.1.bias"])
    return (y @ g["scorer.3.weight"].T + g["scorer.3.bias"])[..., 0]


def case(name, spec, batch, note):
    model, ckpt = hf_model(spec)
    b, l, k = batch.b, batch.l, batch.k
    full = np.zeros((b, 1, l, l), np.float32)
    sliding = np.zeros((b, 1, l, l), np.float32)
    position = np.zeros((b, l), np.int64)
    neg = np.finfo(np.float32).min
    for i, row in enumerate(batch.rows):
        markers = [int(m) for m, live in zip(batch.marker_pos[i * k:(i + 1) * k],
                                             batch.marker_mask[i * k:(i + 1) * k]) if live]
        pos, opt = von_layout(row.real_len, markers, l)
        position[i] = pos
        full[i, 0] = np.where(von_allowed(row.real_len, pos, opt, None), 0.0, neg)
        sliding[i, 0] = np.where(von_allowed(row.real_len, pos, opt, spec["sliding_window"]), 0.0, neg)
    ids = torch.from_numpy(batch.input_ids.reshape(b, l))
    out = model(input_ids=ids, attention_mask={"full_attention": torch.from_numpy(full),
                                               "sliding_attention": torch.from_numpy(sliding)},
                position_ids=torch.from_numpy(position)).last_hidden_state
    mpos = torch.from_numpy(batch.marker_pos.reshape(b, k))
    reps = torch.gather(out, 1, mpos.clamp(min=0)[:, :, None].expand(b, k, out.shape[-1]))
    logits = scorer(ckpt, reps)
    logits = torch.where(torch.from_numpy(batch.marker_mask.reshape(b, k)), logits, torch.full_like(logits, -1e4))
    path = os.path.join(HERE, f"{name}.npz")
    np.savez_compressed(
        path, spec=json.dumps(spec), note=note, input_ids=batch.input_ids, attention_mask=batch.attention_mask,
        marker_pos=batch.marker_pos, marker_mask=batch.marker_mask, qtype=batch.qtype,
        real_len=batch.real_len(), real_k=batch.real_k(), b=b, l=l, k=k, logits=logits.numpy().astype(np.float32))
    print(f"wrote {path}: logits {tuple(logits.shape)}")


def main():
    spec = specs.preset("von-base", hidden=256, layers=4, heads=4, ffn=384, vocab=1024, pad_id=0, seed=505)
    rng = np.random.default_rng(18)
    rows = von_rows(rng, 5, spec["vocab"], cls_id=1, sep_id=2, mask_id=3, prefix_low=4, prefix_high=150)
    case("von_tiny_ragged", spec, collate(rows, Layout(pad_id=0)),
         "ModernBERT (full / sliding / sliding / full), 5 rows, 2-6 options, rng seed 18")
    spec2 = dict(spec, sliding_window=8, seed=506)
    rng = np.random.default_rng(19)
    rows = von_rows(rng, 3, spec2["vocab"], cls_id=1, sep_id=2, mask_id=3, prefix_low=30, prefix_high=90,
                    desc_high=20)
    case("von_tiny_window8", spec2, collate(rows, Layout(pad_id=0)),
         "sliding window of 8 positions (local layers cut inside prefixes and options), rng seed 19")


if __name__ == "__main__":
    main()
