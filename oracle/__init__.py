"""CPU oracle for the decision-model forward — TEST INFRASTRUCTURE ONLY.

Only `tests/`, `__graft_entry__.smoke()` and the CPU-baseline leg of `bench.py`
may import this package, and only as the reference answer the tests compare
with or as the timed CPU baseline.
Nothing on the product path (the `verdict_b200` package and its CUDA library)
imports, links or calls it.

What it restates (fp32, numpy):
- `decoder.py`: the reference executor's letter readout, i.e. the HF decoder
  forward run by `GraphRunner._eager_readout` (`executor/torch_exec.py:255-261`)
  followed by `hs[slot].float() @ head_w.T` with
  `head_w = lm_head.weight[label_ids].float()` (`executor/torch_exec.py:2383-2386`).
  The decoder arithmetic itself lives in HF `transformers` (the reference pins
  5.19.0; its Qwen3 / Gemma modelling files define RMSNorm, RoPE, GQA SDPA and
  the gated MLPs restated here).
- `encoder.py`: the marker-head `DecisionModel.forward`
  (`convert/marker_head/marker_head_converter.py:40-57`) over an HF BERT /
  XLM-RoBERTa encoder.
- `labels.py`: the option-label table rules (`src/tokenize.rs:96-171`,
  `executor/torch_exec.py:2254-2323`).

Pinning: `tests/golden/make_golden.py` runs the reference's own code
(`executor/torch_exec.py` imported unchanged, and `DecisionModel`) on CPU in
fp32 with the same synthetic weights and inputs and commits the outputs as
fixtures; `tests/test_oracle_golden.py` checks this oracle against them.
"""
