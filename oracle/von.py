"""fp32 numpy restatement of the independent-options (von) forward.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

The graph the reference serves for this family is exported by
`VonExportWrapper.forward` (`convert/independent_options/independent_options_converter.py:22-36`):
    h = encoder(input_ids, attention_mask={"full_attention": full,
                "sliding_attention": sliding}, position_ids=position).last_hidden_state
    logits = scorer(gather(h, marker_pos)).reshape(b, k), masked slots -1e4
with the inputs built on the Rust side by `independent_options_tensors`
(`src/engine.rs:531-590`), restated in `von_layout` / `von_allowed` below:
- option j spans tokens [marker_j, marker_{j+1}) (the last one up to, not
  including, the final token); inside a span the position restarts at the
  first marker ("option-invariant" positions), everywhere else it is the
  column index;
- a token outside the options attends to every token outside the options, an
  option token to those and to its own option; only keys < real_len; every
  token attends to itself;
- sliding layers keep only keys within `sliding_window` positions.
The encoder is HF `ModernBertModel` (transformers): bias-free LayerNorms,
fused Wqkv, RoPE with a global / local theta per layer type, GeGLU MLP with
the exact GELU, pre-norm layers (no attention norm in layer 0), a final norm.
The scorer lives in the absent third-party `von` package; it is taken here to
have the marker head's layout (LayerNorm -> Linear -> GELU -> Linear(d, 1),
`convert/marker_head/marker_head_converter.py:35-37`).
"""

from __future__ import annotations

import numpy as np

from .decoder import apply_rope, rope_tables
from .encoder import SENTINEL, gelu_erf, layernorm
from .fastsynth import FastCheckpoint


def von_layout(real_len: int, markers, length: int):
    """(position [length], option_id [length]) of one row (src/engine.rs:544-568)."""
    markers = [int(m) for m in markers]
    if not markers or markers[0] >= real_len:
        raise ValueError("no marker positions inside the real ids")
    position = np.arange(length, dtype=np.int64)
    option = np.full(length, -1, dtype=np.int64)
    prefix = markers[0]
    for j, start in enumerate(markers):
        end = min(markers[j + 1] if j + 1 < len(markers) else real_len - 1, real_len)
        for pos in range(start, end):
            option[pos] = j
            position[pos] = prefix + (pos - start)
    return position, option


def von_allowed(real_len: int, position, option, window: int | None):
    """Boolean [length, length] attention masks (query, key): the full one, or
    the sliding one when `window` is given (src/engine.rs:569-588)."""
    length = len(option)
    oq, ok = option[:, None], option[None, :]
    base = np.where(oq == -1, ok == -1, (ok == -1) | (ok == oq)) & (np.arange(length)[None, :] < real_len)
    eye = np.eye(length, dtype=bool)
    if window is None:
        return base | eye
    local = np.abs(position[:, None] - position[None, :]) <= window
    return eye | (base & local)


def masked_attention(q, k, v, allowed):
    """softmax(q k^T / sqrt(hd), disallowed keys excluded) v; q/k/v [n, h, hd]."""
    n, heads, hd = q.shape
    out = np.empty_like(q)
    scale = np.float32(hd ** -0.5)
    for h in range(heads):
        s = (q[:, h, :] @ k[:, h, :].T) * scale
        s = np.where(allowed, s, np.float32(-np.inf))
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s, dtype=np.float32)
        p /= p.sum(axis=-1, keepdims=True)
        out[:, h, :] = p @ v[:, h, :]
    return out


class VonOracle:
    def __init__(self, spec: dict, store16: bool = False):
        """store16: round every activation the GPU path keeps in 16 bits (norm
        outputs, q/k after RoPE, v, the attention output, the GeGLU product) to
        fp16 where it is stored; the residual stream stays fp32.  It measures
        what fp16 storage alone does to the logits."""
        self.spec = spec
        self.store16 = store16
        self.ckpt = FastCheckpoint(spec)
        self.w = {name: self.ckpt.get(name) for name in self.ckpt.names()
                  if not name.endswith("tok_embeddings.weight")}

    def hidden(self, ids: np.ndarray, markers) -> np.ndarray:
        """Final-norm hidden states of one row's real tokens, [n, d]."""
        s, w = self.spec, self.w
        n, d, heads = len(ids), s["hidden"], s["heads"]
        hd = d // heads
        zero = np.zeros(d, np.float32)
        eps = s["ln_eps"]
        position, option = von_layout(n, markers, n)
        full = von_allowed(n, position, option, None)
        sliding = von_allowed(n, position, option, s["sliding_window"])
        tabs = {t: rope_tables(position, hd, s["global_theta"] if t == "full_attention" else s["local_theta"])
                for t in set(s["layer_types"])}
        uniq, inv = np.unique(ids, return_inverse=True)
        emb = self.ckpt.get("encoder.embeddings.tok_embeddings.weight", rows=uniq)[inv]
        h = layernorm(emb, w["encoder.embeddings.norm.weight"], zero, eps)
        st = (lambda t: t.astype(np.float16).astype(np.float32)) if self.store16 else (lambda t: t)
        for i, kind in enumerate(s["layer_types"]):
            p = f"encoder.layers.{i}."
            x = st(h if i == 0 else layernorm(h, w[p + "attn_norm.weight"], zero, eps))
            qkv = (x @ w[p + "attn.Wqkv.weight"].T).reshape(n, 3, heads, hd)
            cos, sin = tabs[kind]
            q, k = st(apply_rope(qkv[:, 0], cos, sin)), st(apply_rope(qkv[:, 1], cos, sin))
            a = st(masked_attention(q, k, st(qkv[:, 2]), full if kind == "full_attention" else sliding))
            h = h + a.reshape(n, d) @ w[p + "attn.Wo.weight"].T
            x = st(layernorm(h, w[p + "mlp_norm.weight"], zero, eps))
            inp, gate = np.split(x @ w[p + "mlp.Wi.weight"].T, 2, axis=-1)
            h = (h + st(gelu_erf(inp) * gate) @ w[p + "mlp.Wo.weight"].T).astype(np.float32)
        return layernorm(h, w["encoder.final_norm.weight"], zero, eps)

    def score(self, rep: np.ndarray) -> np.ndarray:
        w = self.w
        y = layernorm(rep, w["scorer.0.weight"], w["scorer.0.bias"], 1e-5)
        y = gelu_erf(y @ w["scorer.1.weight"].T + w["scorer.1.bias"])
        return (y @ w["scorer.3.weight"].T + w["scorer.3.bias"])[..., 0].astype(np.float32)

    def infer(self, batch) -> np.ndarray:
        """Scorer logits [b, k] (masked slots -1e4) for a `CollatedBatch`."""
        out = np.full((batch.b, batch.k), SENTINEL, dtype=np.float32)
        for i, row in enumerate(batch.rows):
            ids = np.asarray(batch.input_ids[i * batch.l:i * batch.l + row.real_len], dtype=np.int64)
            mpos = batch.marker_pos[i * batch.k:(i + 1) * batch.k]
            mmask = batch.marker_mask[i * batch.k:(i + 1) * batch.k]
            markers = [int(m) for m, live in zip(mpos, mmask) if live]
            h = self.hidden(ids, markers)
            logits = self.score(h[np.asarray(markers)])
            for j, lg in enumerate(logits):
                out[i, j] = lg
        return out
