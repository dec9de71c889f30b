"""fp32 numpy restatement of the letter-family decoder forward + option readout.

TEST INFRASTRUCTURE ONLY (see `oracle/__init__.py`).

Reference path: `GraphRunner._eager_readout` (`executor/torch_exec.py:255-261`):
    hs = model.model(input_ids=ids, use_cache=False[, attention_mask]).last_hidden_state
    logits = hs[slot_batch, slot_idx].float() @ head_w.T
with `head_w = model.get_output_embeddings().weight[letter_ids].float()`
(`executor/torch_exec.py:2383-2386`), the model in fp32 on CPU
(`executor/torch_exec.py:2352`).  The per-layer math is HF transformers'
Qwen3 (`Qwen3RMSNorm`, q/k RMSNorm, `rotate_half` RoPE, SDPA causal GQA,
SiLU-gated MLP) and Gemma (`(1 + w)` RMSNorm, sqrt(d) embedding scale,
tanh-GELU gated MLP, tied head).  Right padding is never attended by a causal
model, so each row is computed over its `real_len` tokens only.
"""

from __future__ import annotations

import numpy as np

from verdict_b200.synth import synthetic_label_ids

from .fastsynth import FastCheckpoint


def rmsnorm(x: np.ndarray, w: np.ndarray, eps: float, plus_one: bool) -> np.ndarray:
    """Qwen3RMSNorm: w * (x * rsqrt(mean(x^2) + eps)); GemmaRMSNorm: (1 + w) * (...)."""
    var = np.mean(np.square(x, dtype=np.float32), axis=-1, keepdims=True, dtype=np.float32)
    y = x * (np.float32(1.0) / np.sqrt(var + np.float32(eps))).astype(np.float32)
    g = (np.float32(1.0) + w) if plus_one else w
    return (y * g).astype(np.float32)


def rope_tables(positions: np.ndarray, head_dim: int, theta: float):
    """cos/sin of the default RoPE: inv_freq = 1 / theta^(2i/hd), emb = cat(freqs, freqs)."""
    exps = np.arange(0, head_dim, 2, dtype=np.int64).astype(np.float32) / np.float32(head_dim)
    inv_freq = (np.float32(1.0) / np.power(np.float32(theta), exps)).astype(np.float32)
    freqs = positions.astype(np.float32)[:, None] * inv_freq[None, :]
    emb = np.concatenate([freqs, freqs], axis=-1)
    return np.cos(emb).astype(np.float32), np.sin(emb).astype(np.float32)


def apply_rope(x: np.ndarray, cos: np.ndarray, sin: np.ndarray) -> np.ndarray:
    """x * cos + rotate_half(x) * sin with rotate_half(x) = cat(-x2, x1); x is [n, h, hd]."""
    half = x.shape[-1] // 2
    rot = np.concatenate([-x[..., half:], x[..., :half]], axis=-1)
    return (x * cos[:, None, :] + rot * sin[:, None, :]).astype(np.float32)


def attention(q: np.ndarray, k: np.ndarray, v: np.ndarray, causal: bool) -> np.ndarray:
    """softmax(q k^T / sqrt(hd) [+ causal mask]) v with GQA head sharing; q [n,hq,hd], k/v [n,hkv,hd]."""
    n, hq, hd = q.shape
    hkv = k.shape[1]
    group = hq // hkv
    scale = np.float32(hd ** -0.5)
    out = np.empty_like(q)
    mask = np.triu(np.ones((n, n), dtype=bool), 1) if causal else None
    for h in range(hq):
        s = (q[:, h, :] @ k[:, h // group, :].T) * scale
        if mask is not None:
            s = np.where(mask, np.float32(-np.inf), s)
        s = s - s.max(axis=-1, keepdims=True)
        p = np.exp(s, dtype=np.float32)
        p /= p.sum(axis=-1, keepdims=True)
        out[:, h, :] = p @ v[:, h // group, :]
    return out


def gelu_tanh(x: np.ndarray) -> np.ndarray:
    c = np.float32(np.sqrt(2.0 / np.pi))
    return (np.float32(0.5) * x * (np.float32(1.0) + np.tanh(c * (x + np.float32(0.044715) * x * x * x)))).astype(np.float32)


def silu(x: np.ndarray) -> np.ndarray:
    return (x / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def sigmoid(x: np.ndarray) -> np.ndarray:
    return (np.float32(1.0) / (np.float32(1.0) + np.exp(-x))).astype(np.float32)


def softplus(x: np.ndarray) -> np.ndarray:
    """torch.nn.functional.softplus (beta 1, threshold 20)."""
    return np.where(x > 20, x, np.log1p(np.exp(np.minimum(x, np.float32(20))))).astype(np.float32)


def l2norm(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    """x * rsqrt(sum(x^2) + eps) over the last axis (the FLA-aligned l2norm of HF Qwen3.5)."""
    return (x / np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=np.float32) + np.float32(eps))).astype(np.float32)


def causal_conv_silu(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Depthwise causal conv1d (kernel K, zero history) then SiLU; x [n, C], w [C, K]:
    y[t, c] = silu(sum_j w[c, j] * x[t - (K - 1) + j, c])."""
    n, _ = x.shape
    k = w.shape[1]
    xp = np.concatenate([np.zeros((k - 1, x.shape[1]), np.float32), x], axis=0)
    y = np.zeros_like(x)
    for j in range(k):
        y += xp[j:j + n] * w[:, j][None, :]
    return silu(y)


def gated_delta_rule(q: np.ndarray, k: np.ndarray, v: np.ndarray, g: np.ndarray, beta: np.ndarray) -> np.ndarray:
    """The gated delta rule in its recurrent form (HF `torch_recurrent_gated_delta_rule`;
    the chunked form computes the same function): per head, state S [dk, dv] = 0,
    for each token: S *= exp(g); delta = (v - k^T S) * beta; S += k delta^T; o = q^T S.
    q, k [n, H, dk] (normalised, q scaled), v [n, H, dv], g, beta [n, H]."""
    n, heads, dk = k.shape
    dv = v.shape[-1]
    S = np.zeros((heads, dk, dv), np.float32)
    out = np.empty((n, heads, dv), np.float32)
    decay = np.exp(g).astype(np.float32)
    for t in range(n):
        S *= decay[t][:, None, None]
        kv = np.einsum("hk,hkv->hv", k[t], S)
        delta = (v[t] - kv) * beta[t][:, None]
        S += k[t][:, :, None] * delta[:, None, :]
        out[t] = np.einsum("hk,hkv->hv", q[t], S)
    return out


class DecoderOracle:
    """Holds the synthetic checkpoint (host, fp32 copies of the bf16 weights).

    cache_layers=False regenerates each layer's weights when it is used and
    drops them afterwards, so a 40-layer 9B model runs in ~2 GB of host memory."""

    def __init__(self, spec: dict, layers: int | None = None, cache_layers: bool = True, store16: bool = False):
        """store16: round every activation the GPU path keeps in 16 bits to fp16
        where it is stored (norm outputs, projection outputs, q/k/v after their
        norms and rotary embedding, mixer outputs, the MLP activation); the
        residual stream stays fp32.  It measures what fp16 storage alone does to
        the outputs, as a yardstick for the GPU's deviation from fp32."""
        self.spec = spec
        self.store16 = store16
        self.ckpt = FastCheckpoint(spec)
        self.cache_layers = cache_layers
        self.n_layers = spec["layers"] if layers is None else layers
        self.label_ids = synthetic_label_ids(spec)
        self._layers = {}
        self.final_norm = self.ckpt.get("model.norm.weight")
        self.head_w = self.ckpt.get(self.ckpt.head_name(), rows=self.label_ids)

    def _layer_names(self, i: int) -> list:
        s = self.spec
        if s.get("style") == "qwen3_5":
            common = ["input_layernorm.weight", "post_attention_layernorm.weight", "mlp.gate_proj.weight",
                      "mlp.up_proj.weight", "mlp.down_proj.weight"]
            if s["layer_types"][i] == "full_attention":
                return common + ["self_attn." + n for n in ("q_proj.weight", "k_proj.weight", "v_proj.weight",
                                                            "o_proj.weight", "q_norm.weight", "k_norm.weight")]
            return common + ["linear_attn." + n for n in (
                "in_proj_qkv.weight", "in_proj_z.weight", "in_proj_b.weight", "in_proj_a.weight",
                "conv1d.weight", "dt_bias", "A_log", "norm.weight", "out_proj.weight")]
        return None

    def layer(self, i: int) -> dict:
        if i not in self._layers:
            p = f"model.layers.{i}."
            hybrid = self._layer_names(i)
            if hybrid is not None:
                w = {n: self.ckpt.get(p + n) for n in hybrid}
                if not self.cache_layers:
                    return w
                self._layers[i] = w
                return w
            names = ["input_layernorm.weight", "self_attn.q_proj.weight", "self_attn.k_proj.weight",
                     "self_attn.v_proj.weight", "self_attn.o_proj.weight",
                     "post_attention_layernorm.weight", "mlp.gate_proj.weight",
                     "mlp.up_proj.weight", "mlp.down_proj.weight"]
            if self.spec["qk_norm"]:
                names += ["self_attn.q_norm.weight", "self_attn.k_norm.weight"]
            if self.spec["qkv_bias"]:
                names += ["self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias"]
            w = {n: self.ckpt.get(p + n) for n in names}
            if not self.cache_layers:
                return w
            self._layers[i] = w
        return self._layers[i]

    def embed(self, ids: np.ndarray) -> np.ndarray:
        uniq, inv = np.unique(ids, return_inverse=True)
        rows = self.ckpt.get("model.embed_tokens.weight", rows=uniq)
        h = rows[inv].astype(np.float32)
        if self.spec["embed_scale"]:
            h = h * np.float32(self.spec["hidden"] ** 0.5)
        return h

    def hybrid_layer_forward(self, i: int, h: np.ndarray, cos, sin) -> np.ndarray:
        """One Qwen3.5 decoder layer (HF `Qwen3_5DecoderLayer`): (1 + w) RMSNorms;
        full attention with q/k norm, partial RoPE and a sigmoid output gate
        (`Qwen3_5Attention`), or a gated delta net (`Qwen3_5GatedDeltaNet`:
        in_proj_qkv -> causal depthwise conv + SiLU -> l2-normalised q, k ->
        gated delta rule with g = -exp(A_log) softplus(a + dt_bias), beta =
        sigmoid(b) -> RMSNorm(o) * w * silu(z) -> out_proj); then the SiLU MLP."""
        s = self.spec
        w = self.layer(i)
        n = h.shape[0]
        eps = s["rms_eps"]
        st = (lambda t: t.astype(np.float16).astype(np.float32)) if self.store16 else (lambda t: t)
        x = st(rmsnorm(h, w["input_layernorm.weight"], eps, True))
        if s["layer_types"][i] == "full_attention":
            hd, nq, nkv = s["head_dim"], s["heads"], s["kv_heads"]
            qg = (x @ w["self_attn.q_proj.weight"].T).reshape(n, nq, 2 * hd)
            q, gate = qg[..., :hd], st(qg[..., hd:].reshape(n, nq * hd))
            k = (x @ w["self_attn.k_proj.weight"].T).reshape(n, nkv, hd)
            v = st((x @ w["self_attn.v_proj.weight"].T).reshape(n, nkv, hd))
            q = rmsnorm(q, w["self_attn.q_norm.weight"], eps, True)
            k = rmsnorm(k, w["self_attn.k_norm.weight"], eps, True)
            rd = cos.shape[-1]
            q = st(np.concatenate([apply_rope(q[..., :rd], cos, sin), q[..., rd:]], axis=-1))
            k = st(np.concatenate([apply_rope(k[..., :rd], cos, sin), k[..., rd:]], axis=-1))
            a = st(attention(q, k, v, causal=True).reshape(n, nq * hd) * sigmoid(gate))
            h = h + a @ w["self_attn.o_proj.weight"].T
        else:
            lk, lv, dk, dv = s["lin_k_heads"], s["lin_v_heads"], s["lin_k_dim"], s["lin_v_dim"]
            kd, vd = lk * dk, lv * dv
            p = "linear_attn."
            mixed = st(x @ w[p + "in_proj_qkv.weight"].T)
            z = st((x @ w[p + "in_proj_z.weight"].T).reshape(n, lv, dv))
            b = st(x @ w[p + "in_proj_b.weight"].T)
            a = st(x @ w[p + "in_proj_a.weight"].T)
            conv = causal_conv_silu(mixed, w[p + "conv1d.weight"][:, 0, :])
            q = conv[:, :kd].reshape(n, lk, dk)
            k = conv[:, kd:2 * kd].reshape(n, lk, dk)
            v = st(conv[:, 2 * kd:].reshape(n, lv, dv))
            beta = sigmoid(b)
            g = (-np.exp(w[p + "A_log"]) * softplus(a + w[p + "dt_bias"])).astype(np.float32)
            rep = lv // lk
            q = st(l2norm(np.repeat(q, rep, axis=1)) * np.float32(dk ** -0.5))
            k = st(l2norm(np.repeat(k, rep, axis=1)))
            o = gated_delta_rule(q, k, v, g, beta)
            o = st(rmsnorm(o, w[p + "norm.weight"], eps, False) * silu(z))
            h = h + o.reshape(n, vd) @ w[p + "out_proj.weight"].T
        x = st(rmsnorm(h, w["post_attention_layernorm.weight"], eps, True))
        act = st(silu(x @ w["mlp.gate_proj.weight"].T) * (x @ w["mlp.up_proj.weight"].T))
        h = h + act @ w["mlp.down_proj.weight"].T
        return h.astype(np.float32)

    def rope(self, n: int):
        s = self.spec
        rd = int(s["head_dim"] * s.get("partial_rotary", 1.0)) if s.get("style") == "qwen3_5" else s["head_dim"]
        return rope_tables(np.arange(n), rd, s["rope_theta"])

    def layer_forward(self, i: int, h: np.ndarray, cos, sin) -> np.ndarray:
        s = self.spec
        if s.get("style") == "qwen3_5":
            return self.hybrid_layer_forward(i, h, cos, sin)
        w = self.layer(i)
        hd, nq, nkv = s["head_dim"], s["heads"], s["kv_heads"]
        n = h.shape[0]
        st = (lambda t: t.astype(np.float16).astype(np.float32)) if self.store16 else (lambda t: t)
        x = st(rmsnorm(h, w["input_layernorm.weight"], s["rms_eps"], s["norm_plus_one"]))
        q = x @ w["self_attn.q_proj.weight"].T
        k = x @ w["self_attn.k_proj.weight"].T
        v = x @ w["self_attn.v_proj.weight"].T
        if s["qkv_bias"]:
            q = q + w["self_attn.q_proj.bias"]
            k = k + w["self_attn.k_proj.bias"]
            v = v + w["self_attn.v_proj.bias"]
        q = q.reshape(n, nq, hd)
        k = k.reshape(n, nkv, hd)
        v = v.reshape(n, nkv, hd)
        if s["qk_norm"]:
            q = rmsnorm(q, w["self_attn.q_norm.weight"], s["rms_eps"], s["norm_plus_one"])
            k = rmsnorm(k, w["self_attn.k_norm.weight"], s["rms_eps"], s["norm_plus_one"])
        q = st(apply_rope(q, cos, sin))
        k = st(apply_rope(k, cos, sin))
        a = st(attention(q, k, st(v), causal=True).reshape(n, nq * hd))
        h = h + a @ w["self_attn.o_proj.weight"].T
        x = st(rmsnorm(h, w["post_attention_layernorm.weight"], s["rms_eps"], s["norm_plus_one"]))
        g = x @ w["mlp.gate_proj.weight"].T
        u = x @ w["mlp.up_proj.weight"].T
        act = silu(g) if s["act"] == "silu" else gelu_tanh(g)
        h = h + st(act * u) @ w["mlp.down_proj.weight"].T
        return h.astype(np.float32)

    def hidden(self, ids: np.ndarray) -> np.ndarray:
        """Final-norm hidden states of one sequence, [n, d] fp32."""
        ids = np.asarray(ids, dtype=np.int64)
        n = ids.shape[0]
        cos, sin = self.rope(n)
        h = self.embed(ids)
        for i in range(self.n_layers):
            h = self.layer_forward(i, h, cos, sin)
        return rmsnorm(h, self.final_norm, self.spec["rms_eps"], self.spec["norm_plus_one"])

    def readout(self, ids: np.ndarray, slot: int) -> np.ndarray:
        """Label-row logits at one slot: hs[slot] @ head_w.T, width = #labels."""
        hs = self.hidden(ids)
        return (hs[slot] @ self.head_w.T).astype(np.float32)

    def infer(self, batch) -> np.ndarray:
        """Raw label logits [b, width] for a `CollatedBatch` (slot = marker_pos[i*k])."""
        if not self.cache_layers:
            return self._infer_streaming(batch)
        out = np.empty((batch.b, len(self.label_ids)), dtype=np.float32)
        for i, row in enumerate(batch.rows):
            ids = batch.input_ids[i * batch.l:i * batch.l + row.real_len]
            out[i] = self.readout(ids, int(batch.marker_pos[i * batch.k]))
        return out

    def _infer_streaming(self, batch) -> np.ndarray:
        """Layer-major order: each layer's weights are generated once for all rows."""
        s = self.spec
        hs, tabs = [], []
        for i, row in enumerate(batch.rows):
            ids = np.asarray(batch.input_ids[i * batch.l:i * batch.l + row.real_len], dtype=np.int64)
            hs.append(self.embed(ids))
            tabs.append(self.rope(len(ids)))
        for layer in range(self.n_layers):
            w = self.layer(layer)
            self._layers[layer] = w
            for i in range(len(hs)):
                hs[i] = self.layer_forward(layer, hs[i], *tabs[i])
            del self._layers[layer]
        out = np.empty((batch.b, len(self.label_ids)), dtype=np.float32)
        for i in range(len(hs)):
            slot = int(batch.marker_pos[i * batch.k])
            hn = rmsnorm(hs[i][slot:slot + 1], self.final_norm, s["rms_eps"], s["norm_plus_one"])
            out[i] = (hn[0] @ self.head_w.T).astype(np.float32)
        return out


def option_logprobs(logits: np.ndarray, nopts) -> np.ndarray:
    """log_softmax over the first nopts[i] columns, -1e4 elsewhere (what `vd_infer` returns).

    Softmax is shift-invariant, so this carries the same information the
    reference's Rust side computes with `finish_rows` (columns >= nopts set to
    -1e4, `src/torch_engine.rs:97-114`) and `softmax(logits / t)`
    (`src/calibration.rs:248-253`)."""
    logits = np.asarray(logits, dtype=np.float64)
    out = np.full(logits.shape, -1e4, dtype=np.float64)
    for i, k in enumerate(nopts):
        z = logits[i, :int(k)]
        m = z.max()
        out[i, :int(k)] = z - m - np.log(np.exp(z - m).sum())
    return out
