"""fp32 numpy restatement of the marker-head `DecisionModel` forward.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Reference: `DecisionModel.forward` (`convert/marker_head/marker_head_converter.py:40-57`):
    h = encoder(input_ids, attention_mask).last_hidden_state     # HF BERT / XLM-R, post-LN
    h = h + type_emb(qtype)[:, None, :]
    for layer in head.layers:                                     # nn.TransformerEncoderLayer,
        h = layer(h, src_key_padding_mask=~attention_mask)        # norm_first, ReLU, d//64 heads
    m = gather(h, marker_pos.clamp(min=0))
    logits = scorer(m).squeeze(-1)                                # LN -> Linear -> GELU -> Linear(d, 1)
    logits = logits.masked_fill(~marker_mask, -1e4)
Encoder math is HF BertModel / XLMRobertaModel (word + position + token-type
embeddings -> LayerNorm; per layer: self-attention with key padding,
dense + residual -> LayerNorm, GELU(erf) FFN + residual -> LayerNorm).  XLM-R
positions start at padding_idx + 1.  Padded keys are never attended, so each
row is computed over its real tokens only.
"""

from __future__ import annotations

import numpy as np
from scipy.special import erf

from .decoder import attention
from .fastsynth import FastCheckpoint

SENTINEL = -1e4


def layernorm(x, w, b, eps):
    mu = x.mean(-1, keepdims=True, dtype=np.float32)
    xc = x - mu
    var = np.mean(xc * xc, axis=-1, keepdims=True, dtype=np.float32)
    return (xc / np.sqrt(var + np.float32(eps)) * w + b).astype(np.float32)


def gelu_erf(x):
    return (np.float32(0.5) * x * (np.float32(1.0) + erf(x / np.float32(np.sqrt(2.0))))).astype(np.float32)


class EncoderOracle:
    def __init__(self, spec: dict):
        self.spec = spec
        self.ckpt = FastCheckpoint(spec)
        self.w = {}

    def g(self, name):
        if name not in self.w:
            self.w[name] = self.ckpt.get(name)
        return self.w[name]

    def encode(self, ids: np.ndarray) -> np.ndarray:
        s = self.spec
        n = ids.shape[0]
        d, nh = s["hidden"], s["heads"]
        e = "encoder.embeddings."
        word = self.ckpt.get(e + "word_embeddings.weight", rows=ids)
        if s["style"] == "xlmr":
            pos = np.arange(n) + s["pad_id"] + 1
        else:
            pos = np.arange(n)
        h = word + self.g(e + "position_embeddings.weight")[pos] + self.g(e + "token_type_embeddings.weight")[0]
        h = layernorm(h.astype(np.float32), self.g(e + "LayerNorm.weight"), self.g(e + "LayerNorm.bias"), s["ln_eps"])
        for i in range(s["layers"]):
            p = f"encoder.encoder.layer.{i}."
            q = h @ self.g(p + "attention.self.query.weight").T + self.g(p + "attention.self.query.bias")
            k = h @ self.g(p + "attention.self.key.weight").T + self.g(p + "attention.self.key.bias")
            v = h @ self.g(p + "attention.self.value.weight").T + self.g(p + "attention.self.value.bias")
            hd = d // nh
            a = attention(q.reshape(n, nh, hd), k.reshape(n, nh, hd), v.reshape(n, nh, hd), causal=False)
            a = a.reshape(n, d) @ self.g(p + "attention.output.dense.weight").T + self.g(p + "attention.output.dense.bias")
            h = layernorm(a + h, self.g(p + "attention.output.LayerNorm.weight"),
                          self.g(p + "attention.output.LayerNorm.bias"), s["ln_eps"])
            f = gelu_erf(h @ self.g(p + "intermediate.dense.weight").T + self.g(p + "intermediate.dense.bias"))
            o = f @ self.g(p + "output.dense.weight").T + self.g(p + "output.dense.bias")
            h = layernorm(o + h, self.g(p + "output.LayerNorm.weight"), self.g(p + "output.LayerNorm.bias"), s["ln_eps"])
        return h

    def head(self, h: np.ndarray, qtype: int) -> np.ndarray:
        s = self.spec
        d = s["hidden"]
        nh = max(1, d // 64)
        n = h.shape[0]
        h = h + self.g("type_emb.weight")[qtype]
        for i in range(s["head_layers"]):
            p = f"head.layers.{i}."
            y = layernorm(h, self.g(p + "norm1.weight"), self.g(p + "norm1.bias"), 1e-5)
            qkv = y @ self.g(p + "self_attn.in_proj_weight").T + self.g(p + "self_attn.in_proj_bias")
            q, k, v = qkv[:, :d], qkv[:, d:2 * d], qkv[:, 2 * d:]
            hd = d // nh
            a = attention(q.reshape(n, nh, hd), k.reshape(n, nh, hd), v.reshape(n, nh, hd), causal=False)
            h = h + a.reshape(n, d) @ self.g(p + "self_attn.out_proj.weight").T + self.g(p + "self_attn.out_proj.bias")
            y = layernorm(h, self.g(p + "norm2.weight"), self.g(p + "norm2.bias"), 1e-5)
            f = np.maximum(y @ self.g(p + "linear1.weight").T + self.g(p + "linear1.bias"), np.float32(0))
            h = h + f @ self.g(p + "linear2.weight").T + self.g(p + "linear2.bias")
        return h.astype(np.float32)

    def score(self, m: np.ndarray) -> np.ndarray:
        y = layernorm(m, self.g("scorer.0.weight"), self.g("scorer.0.bias"), 1e-5)
        y = gelu_erf(y @ self.g("scorer.1.weight").T + self.g("scorer.1.bias"))
        return (y @ self.g("scorer.3.weight").T + self.g("scorer.3.bias"))[:, 0].astype(np.float32)

    def infer(self, batch) -> np.ndarray:
        """logits [b, k] for a `CollatedBatch`; masked slots = -1e4."""
        out = np.full((batch.b, batch.k), SENTINEL, dtype=np.float32)
        for i, row in enumerate(batch.rows):
            ids = np.asarray(batch.input_ids[i * batch.l:i * batch.l + row.real_len], dtype=np.int64)
            h = self.head(self.encode(ids), int(batch.qtype[i]))
            pos = np.clip(batch.marker_pos[i * batch.k:(i + 1) * batch.k], 0, None)
            mask = np.asarray(batch.marker_mask[i * batch.k:(i + 1) * batch.k], dtype=bool)
            sc = self.score(h[pos])
            out[i] = np.where(mask, sc, np.float32(SENTINEL))
        return out
