"""Decision-forward throughput on B200: decisions/s for OneJev-9B-shaped text decisions.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
    (N > 1: torchrun --nproc-per-node N ... bench.py --gpus N ...)

A step is one forward + option readout of one batch of `--batch` (64) seeded
synthetic decisions of the OneJev-9B-shaped workload (prompt lengths
clip(lognormal(6, 0.7), 32, 4096), 2-8 options, slot = last token, ids
U[3, 152064)); every step uses a different batch.  One full-weight replica per
GPU, each rank runs its own shard of decisions: no collective on the data path
("scaling": "weak"); ranks meet only at the barriers and the max-over-ranks
timing reduction.

Printed JSON (rank 0, one line):
  value  decisions/s over all ranks, inputs already resident in HBM, device time
         (CUDA events on the executor's stream), max over ranks
  e2e    the same through the public C ABI `vd_infer` with pinned host buffers:
         each step copies the padded batch to the device and the logits back
  roofline  the gate/up projection GEMM (tcgen05, the largest kernel): its
         algorithmic FLOPs per launch / its mean launch time from events around
         each launch, against the measured sustained dense 16-bit tensor peak
  dtype  fp16 (default): activations and projection weights in fp16 (the bf16
         checkpoint values are exact in fp16), fp32 accumulation and fp32
         residual stream; --act-dtype bf16 keeps them in bf16
  sweep  the same workload at 1, 8 and 256 decisions per step per GPU:
         whole-job decisions/s (slowest rank), mean and p99 step time, SM clock
  models the other presets' workloads, each rank its own shard (decider-2b
         batch 64, onejev-27b batch 8 (~35k tokens), laya-xlmr batch 128,
         laya-bert batch 32 per GPU): whole-job decisions/s, step time, p99
  cpu_baseline  the CPU oracle (fp32 numpy restatement of the reference's CPU
         executor path) on a bounded sample of the workload's decisions, every
         layer timed, on all of this host's cores
--impl reference runs that CPU implementation as the reference arm: one
decision of the workload per step through every layer (nothing extrapolated).
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import time

if "reference" in sys.argv[1:]:
    # The reference arm runs on the host cores: torchrun sets OMP_NUM_THREADS=1,
    # and BLAS / OpenMP read these variables when they load (before numpy).
    _cores = str(len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count())
    for _var in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[_var] = _cores

import numpy as np

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REPO)

METRIC = "decisions/sec (9B text, 1/2/4/8 B200); p99 latency; GEMM tensor-pipe % of peak"
UNIT = "decisions/s"
WORKLOAD = ("OneJev-9B-shaped text decisions: 40 layers, d=4096, 32/8 heads hd=128, SwiGLU 12288, "
            "vocab 152064, causal varlen prefill + option log-softmax; lengths clip(lognormal(6,0.7),32,4096), "
            "2-8 options")
SHARED_WORKLOAD = ("OneJev-9B-shaped letter-branches decisions, 8 questions per state: rows of a state share "
                   "its prefix (declared prefix_len), state prefix clip(lognormal(6.5,0.5),128,3072) tokens, "
                   "question suffix U[40,160] tokens, 2-8 options")
HYBRID_WORKLOAD = ("OneJev1.6-9B-shaped hybrid text decisions (Qwen3.5 text stack: 24 gated-delta-net + 8 gated "
                   "full-attention layers, d=4096, attention 16/4 heads hd=256, linear 16/32 heads of 128, SwiGLU "
                   "12288, vocab 248320); lengths clip(lognormal(6,0.7),32,4096), 2-8 options")
VON_WORKLOAD = ("ModernBERT-base-shaped independent-options decisions (22 layers, d=768, 12 heads, GeGLU 1152, "
                "vocab 50368, every 3rd layer global, the rest a 64-position window), option-masked attention; "
                "[CLS] prefix U[16,200] [SEP] then 2-6 [MASK]-led options of U[1,12] tokens")
OTHER_WORKLOAD = "{} text decisions (all layers, synthetic weights), lengths {}, 2-8 options"
BERT_WORKLOAD = ("BERT-base-shaped marker-head encoder decisions (laya: 12 layers, d=768, 12 heads, GELU 3072, "
                 "post-LN, vocab 30522, 2 head layers), lengths U[16,128], K=3 markers, ids U[1000,30522)")
XLMR_WORKLOAD = ("XLM-R-base-shaped marker-head encoder decisions (laya-multilingual: 12 layers, d=768, 12 heads, "
                 "GELU 3072, vocab 250002), lengths clip(lognormal(4.5,0.6),8,512), K~U{2..6}, ids U[5,250002)")
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
# DRAM traffic of one gate/up GEMM launch (dram__bytes_read.sum + dram__bytes_write.sum) from an ncu
# capture of a small case (`--layers 2 --batch 32`, layer 0 of the second warm-up batch) and the
# tokens that launch had, per (model, GEMM kernel); the bench scales it to its own launch by tokens.
# Weight re-streaming grows a little faster than the tokens, so the scaled figure is a lower estimate.
GATEUP_TRAFFIC = {("onejev-9b", "2sm"): (1.2605e9 + 0.3454e9, 14316)}


def peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            return json.load(f), "measured"
    return FALLBACK_PEAKS, "fallback"


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", str(rank)))
    return world, rank, local


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.proc = None
        self.path = f"/tmp/vd_clocks_{os.getpid()}.csv"
        try:
            self.out = open(self.path, "w")
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "200",
                 "-i", str(gpu_index)], stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.out.close()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax.append(float(parts[2]))
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        os.unlink(self.path)
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(smax), "reasons": sorted(reasons),
                "samples": len(sm)}


def max_over_ranks(x: float, world: int, device: str = "cpu") -> float:
    """The slowest rank's value (all ranks take part; no-op on one rank)."""
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def whole_job_rate(decisions_per_rank: int, world: int, max_ms: float) -> float:
    """decisions/s of the whole job: every rank's decisions over the slowest rank's time."""
    return decisions_per_rank * world / (max_ms / 1e3)


# Concurrency sweep: (decisions per step, timed steps), each after 3 warm-up steps.
SWEEP = ((1, 16), (8, 8), (256, 3))

LENGTHS = {"onejev-9b": "lognormal-9b", "onejev16-9b": "lognormal-9b", "decider-2b": "uniform-2b",
           "onejev-27b": "uniform-27b", "laya-bert": "uniform-bert", "laya-xlmr": "lognormal-xlmr"}
# Marker-head encoder rows: ([CLS], [SEP]) ids, lowest text id, longest row.
MARKER_ROWS = {"uniform-bert": (101, 102, 1000, 510), "lognormal-xlmr": (0, 2, 5, 512)}


def workload_of(spec, workload):
    """Row generator of a model: independent options (von), marker head, or the decoder workloads."""
    if spec["arch"] != "encoder":
        return workload
    return "von" if spec.get("family") == "independent_options" else "marker"


def workload_text(model, shared=False):
    return {"onejev-9b": SHARED_WORKLOAD if shared else WORKLOAD, "onejev16-9b": HYBRID_WORKLOAD,
            "von-base": VON_WORKLOAD, "laya-bert": BERT_WORKLOAD, "laya-xlmr": XLMR_WORKLOAD,
            "decider-2b": OTHER_WORKLOAD.format("Gemma-2B-shaped decider", "U[64,1024]"),
            "onejev-27b": OTHER_WORKLOAD.format("OneJev-27B-shaped", "U[512,8192]")}[model]


def make_batches(rank, n_batches, per_batch, vocab, seed, workload="choice", pad_id=0, lengths="lognormal-9b"):
    """Each rank's own shard of the workload: batch j of rank r is seeded by
    (seed, r, j), so ranks never share a decision."""
    from verdict_b200.batch import Layout, collate, decoder_rows, encoder_rows, shared_prefix_rows, von_rows
    out = []
    for j in range(n_batches):
        rng = np.random.default_rng([seed, rank, j])
        if workload == "shared-prefix":
            rows = shared_prefix_rows(rng, per_batch, vocab)
        elif workload == "von":
            rows = von_rows(rng, per_batch, vocab)
        elif workload == "marker":
            cls_id, sep_id, id_low, max_len = MARKER_ROWS[lengths]
            rows = encoder_rows(rng, per_batch, vocab, lengths=lengths, cls_id=cls_id, sep_id=sep_id,
                                id_low=id_low, max_len=max_len)
        else:
            rows = decoder_rows(rng, per_batch, vocab, lengths=lengths)
        batch = collate(rows, Layout(pad_id=pad_id))
        if workload == "marker":
            batch.qtype[:] = rng.integers(0, 3, size=batch.b)
        out.append(batch)
    return out


def host_threads():
    """Set up the CPU legs: BLAS / OpenMP threads on every core this process may
    run on, whatever OMP_NUM_THREADS the launcher set (torchrun sets 1), and
    glibc malloc keeping freed blocks (the forward's large temporaries are then
    reused instead of faulted in afresh each time, as torch's CPU allocator
    does).  Returns the thread count the BLAS library reports afterwards."""
    n = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else os.cpu_count()
    try:
        import ctypes
        libc = ctypes.CDLL("libc.so.6")
        libc.mallopt(-3, 1 << 30)      # M_MMAP_THRESHOLD: heap, not mmap, up to 1 GiB
        libc.mallopt(-1, 2 ** 31 - 1)  # M_TRIM_THRESHOLD: keep freed memory
    except Exception:
        pass
    try:
        from threadpoolctl import threadpool_info, threadpool_limits
        threadpool_limits(limits=n)
        blas = [i["num_threads"] for i in threadpool_info() if i.get("user_api") == "blas"]
        return int(blas[0]) if blas else n
    except Exception:
        return n


def decoder_cpu_times(spec, seqs):
    """Seconds of the oracle's full-depth fp32 forward + readout per decision
    (every layer, nothing scaled).  Layer-major, as a batch runs through a
    model: each layer's weights are generated once (untimed; the reference
    holds them in memory) and each decision's pass through that layer is timed
    on its own.  `seqs`: [(token ids, nopts)], slot = last token."""
    from oracle.decoder import DecoderOracle, rmsnorm
    orc = DecoderOracle(spec, cache_layers=False)
    times = np.zeros(len(seqs))
    hs, tabs = [], []
    for j, (ids, _) in enumerate(seqs):
        h = orc.embed(np.asarray(ids, dtype=np.int64))  # embedding rows (generated untimed)
        t0 = time.perf_counter()
        tabs.append(orc.rope(len(ids)))
        hs.append(h.copy())
        times[j] += time.perf_counter() - t0
    for layer in range(spec["layers"]):
        orc._layers[layer] = orc.layer(layer)
        for j in range(len(seqs)):
            t0 = time.perf_counter()
            hs[j] = orc.layer_forward(layer, hs[j], *tabs[j])
            times[j] += time.perf_counter() - t0
        del orc._layers[layer]
    for j, (_, nopts) in enumerate(seqs):
        t0 = time.perf_counter()
        hn = rmsnorm(hs[j][-1:], orc.final_norm, spec["rms_eps"], spec["norm_plus_one"])
        logits = hn[0] @ orc.head_w[:int(nopts)].T
        z = logits - logits.max()
        _ = z - np.log(np.exp(z).sum())
        times[j] += time.perf_counter() - t0
    return times


def decoder_cpu_sample(batches, n):
    """The first n decisions of the workload's batches (row order), for the CPU legs."""
    out = []
    for b in batches:
        for i in range(b.b):
            out.append((b.input_ids[i * b.l:i * b.l + int(b.rows[i].real_len)], int(b.nopts[i])))
            if len(out) == n:
                return out
    return out


def cpu_baseline_decoder(spec, batches, budget_s=20.0):
    """The CPU baseline of the repo's own bench line: the oracle on decisions of
    the same workload, all layers, on this host's cores.  Takes the first
    decisions of the timed batches until their tokens add up to about
    `budget_s` of CPU work (at least 2 decisions; the first one absorbs the
    first use of each layer's weights and is not counted)."""
    tok_per_s = 515.0 / 8.0  # rough fp32 throughput of 16 cores on the 9B shape, for sizing only
    seqs, tokens = [], 0
    for ids, nopts in decoder_cpu_sample(batches, 1 << 30):
        seqs.append((ids, nopts))
        tokens += len(ids)
        if len(seqs) >= 3 and tokens * spec["layers"] / 40.0 >= budget_s * tok_per_s:
            break
    threads = host_threads()
    t = decoder_cpu_times(spec, seqs)[1:]
    toks = [len(ids) for ids, _ in seqs[1:]]
    sample = (f"{len(t)} decisions of the workload (first rows of the timed batches, {int(np.sum(toks))} tokens, "
              f"lengths {min(toks)}-{max(toks)}), every one of the {spec['layers']} layers timed, nothing scaled; "
              "one more decision run first, untimed")
    return len(t) / float(np.sum(t)), sample, float(np.mean(t)), threads


def encoder_cpu_sample(spec, batch):
    """The oracle (fp32 numpy) on the batch's first 4 rows, all layers; decisions/s."""
    from oracle.encoder import EncoderOracle
    from oracle.von import VonOracle
    from verdict_b200.batch import CollatedBatch
    n = min(4, batch.b)
    sub = CollatedBatch(batch.input_ids[:n * batch.l], batch.attention_mask[:n * batch.l],
                        batch.marker_pos[:n * batch.k], batch.marker_mask[:n * batch.k], batch.qtype[:n],
                        batch.nopts, n, batch.l, batch.k, batch.rows[:n])
    orc = VonOracle(spec) if spec.get("family") == "independent_options" else EncoderOracle(spec)
    one = CollatedBatch(batch.input_ids[:batch.l], batch.attention_mask[:batch.l], batch.marker_pos[:batch.k],
                        batch.marker_mask[:batch.k], batch.qtype[:1], batch.nopts, 1, batch.l, batch.k,
                        batch.rows[:1])
    orc.infer(one)  # generates the weights outside the timed region
    t0 = time.perf_counter()
    orc.infer(sub)
    dt = time.perf_counter() - t0
    return n / dt, f"{n} rows, all {spec['layers']} layers", dt / n


# Other model shapes measured in the same run (one GPU): (preset, decisions per step, timed steps).
EXTRA_MODELS = (("decider-2b", 64, 5), ("onejev-27b", 8, 3), ("laya-xlmr", 128, 10), ("laya-bert", 32, 10))


def other_model(model, per_step, steps, warmup, seed, local, rank, world, barrier, reduce_max):
    """decisions/s of another preset's workload over all ranks (each its own
    shard of `per_step` decisions per step on its GPU; device-resident inputs,
    CUDA events, the slowest rank's time; encoder steps after a 256 MB L2
    flush, outside their events), with the step time, p99, tokens per step and
    this GPU's SM clock."""
    import torch
    from verdict_b200 import spec as specs
    from verdict_b200.engine import B200Engine
    from verdict_b200.synth import with_labels
    spec = with_labels(specs.preset(model))
    encoder = spec["arch"] == "encoder"
    batches = make_batches(rank, warmup + steps, per_step, spec["vocab"], seed + 7, workload_of(spec, "choice"),
                           spec.get("pad_id", 0), LENGTHS.get(model, "lognormal-9b"))
    eng = B200Engine(spec, device=local, max_tokens=max(4096, max(int(b.real_len().sum()) for b in batches)),
                     max_rows=max(per_step, 8), max_seq=max(4096, max(int(b.real_len().max()) for b in batches)))
    try:
        width = eng.width if not encoder else max(b.k for b in batches)
        dev = [{k: torch.from_numpy(np.ascontiguousarray(v)).to(f"cuda:{local}") for k, v in dict(
            input_ids=b.input_ids, marker_pos=b.marker_pos, marker_mask=b.marker_mask.astype(np.uint8),
            nopts=b.nopts, qtype=b.qtype).items()} for b in batches]
        out = torch.empty(per_step, width, device=f"cuda:{local}", dtype=torch.float32)
        stream = torch.cuda.ExternalStream(eng.stream())

        def run(j):
            b = batches[j]
            eng.infer_device(b.b, b.l, b.k, {k: v.data_ptr() for k, v in dev[j].items()}, b.real_len(),
                             out.data_ptr(), width)

        for j in range(warmup):
            run(j)
        eng.sync()
        flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}") if encoder else None
        ck = Clocks(local)
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * steps)]
        with torch.cuda.stream(stream):
            for i in range(steps):
                if flush is not None:
                    flush.fill_(i & 0xFF)
                ev[2 * i].record(stream)
                run(warmup + i)
                ev[2 * i + 1].record(stream)
        eng.sync()
        barrier()
        cl = ck.stop()
        ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(steps)]
        total = reduce_max(float(np.sum(ms)) if encoder else ev[0].elapsed_time(ev[-1]))
        return {"workload": workload_text(model), "decisions_per_step_per_gpu": per_step, "steps": steps,
                "warmup": warmup, "value": whole_job_rate(per_step * steps, world, total), "unit": UNIT,
                "ms_per_step": total / steps, "p99_ms": reduce_max(float(np.percentile(ms, 99))),
                "mean_tokens_per_step_per_gpu": float(np.mean([b.real_len().sum() for b in batches[warmup:]])),
                "sm_mhz": cl.get("sm_mhz"), "reasons": cl.get("reasons"),
                "l2": "flushed before each step" if encoder else "not flushed (steps stream GBs of weights)"}
    finally:
        eng.close()


def run_reference(args, world, rank):
    """The reference arm: the reference executor's CPU path (fp32), as the
    oracle port, on all of this host's cores; rank 0 only.  A decoder step is
    one decision of the workload through every layer (no extrapolation), an
    encoder step four decisions."""
    if rank != 0:
        return
    from verdict_b200 import spec as specs
    from verdict_b200.synth import with_labels
    spec = with_labels(specs.preset(args.model))
    encoder = spec["arch"] == "encoder"
    threads = host_threads()
    t_start = time.perf_counter()
    if encoder:
        batches = make_batches(0, args.warmup + args.steps, 4, spec["vocab"], args.seed,
                               workload_of(spec, "choice"), spec.get("pad_id", 0),
                               LENGTHS.get(args.model, "lognormal-9b"))
        per = [encoder_cpu_sample(spec, b)[2] * 4 for b in batches]
        per_step = 4
        sample = "per step 4 decisions of the workload, all layers"
    else:
        # Steps take the workload's own decisions in order (the repo arm's
        # batches, seeded identically), one per step.
        batches = make_batches(0, 1, max(args.batch, args.warmup + args.steps), spec["vocab"], args.seed,
                               workload_of(spec, "choice"), spec.get("pad_id", 0),
                               LENGTHS.get(args.model, "lognormal-9b"))
        seqs = decoder_cpu_sample(batches, args.warmup + args.steps)
        per = list(decoder_cpu_times(spec, seqs))
        per_step = 1
        toks = [len(ids) for ids, _ in seqs[args.warmup:]]
        sample = (f"per step 1 decision of the workload through all {spec['layers']} layers (nothing scaled); "
                  f"timed decisions {int(np.sum(toks))} tokens, lengths {min(toks)}-{max(toks)}")
    times = per[args.warmup:]
    mean = float(np.mean(times))
    value = per_step / mean
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": mean * 1e3,
        "p99_ms": float(np.percentile(times, 99)) * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded)",
        "config": {"workload": workload_text(args.model), "model": args.model,
                   "decisions_per_step": per_step, "parallelism": f"host cores ({threads} BLAS threads)"},
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "timed_s": float(np.sum(times)), "run_s": time.perf_counter() - t_start,
    }
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=64, help="decisions per step (concurrency)")
    ap.add_argument("--layers", type=int, default=None, help="override depth (default: full 40)")
    ap.add_argument("--seed", type=int, default=20261201)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--attention", default="tc", choices=["tc", "tc2", "mma"],
                    help="head_dim-128 causal attention kernel: tcgen05 with one query head per CTA (tc) or "
                         "two (tc2), or warp-level mma.sync")
    ap.add_argument("--workload", default="choice", choices=["choice", "shared-prefix"],
                    help="choice: the OneJev-9B decision workload (headline); shared-prefix: 8 questions "
                         "per state, rows of a state share the state prefix (prefix_len declared)")
    ap.add_argument("--fork", default="on", choices=["on", "off"],
                    help="compute shared prefixes once (on) or every row whole (off)")
    ap.add_argument("--model", default="onejev-9b",
                    choices=["onejev-9b", "onejev16-9b", "von-base", "laya-bert", "laya-xlmr", "decider-2b",
                             "onejev-27b"],
                    help="onejev-9b: the dense OneJev-9B shape (headline); onejev16-9b: the Qwen3.5-style hybrid "
                         "(gated delta nets + gated attention); von-base: the ModernBERT-base independent-options "
                         "encoder; laya-bert / laya-xlmr: the BERT-base / XLM-R-base marker-head encoders; "
                         "decider-2b (lengths U[64,1024]) and onejev-27b (lengths U[512,8192]): the "
                         "other decoder shapes")
    ap.add_argument("--gemm", default="2sm", choices=["2sm", "1sm"],
                    help="256-wide projections on CTA pairs (2sm) or one CTA per tile (1sm)")
    ap.add_argument("--gdn", default="chunk", choices=["chunk", "scan"],
                    help="gated delta nets in 64-token chunks on the tensor cores (chunk) or token by token (scan)")
    ap.add_argument("--norm", default="fused", choices=["fused", "separate"],
                    help="decoders' RMSNorm fused into the residual GEMMs and the projections (fused) or a kernel "
                         "of its own (separate)")
    ap.add_argument("--attn-persistent", default="on", choices=["on", "off"],
                    help="tcgen05 attention: CTAs loop over work items (on) or one CTA per item (off)")
    ap.add_argument("--l2-hints", default="off", choices=["on", "off"],
                    help="pair GEMM: L2 evict-last hints on A loads and evict-first on W loads")
    ap.add_argument("--pdl", default="on", choices=["on", "off"],
                    help="GEMM and attention kernels set up under the previous kernel's tail (programmatic "
                         "dependent launch)")
    ap.add_argument("--attn-spr", type=int, default=1, choices=[1, 2],
                    help="tcgen05 attention: softmax threads per query row")
    ap.add_argument("--split-k", default="off", choices=["on", "off"],
                    help="batches of <= 1024 tokens: split K over CTAs where that fills the GPU better")
    ap.add_argument("--act-dtype", default="fp16", choices=["fp16", "bf16"],
                    help="16-bit element type of activations and projection weights (fp32 accumulation and "
                         "residual stream either way)")
    ap.add_argument("--no-extra-models", dest="extra_models", action="store_false",
                    help="skip the other presets' lines (decider-2b, onejev-27b, laya-xlmr, laya-bert)")
    ap.add_argument("--no-sweep", dest="sweep", action="store_false",
                    help="skip the concurrency sweep (decoders: 1, 8 and 256 decisions per step per GPU)")
    ap.add_argument("--raster-group", type=int, default=0,
                    help="M tiles per GEMM raster group (0: the kernels' default)")
    args = ap.parse_args()
    if args.warmup < 3:
        ap.error("--warmup must be >= 3")

    world, rank, local = dist_env()
    if args.impl == "reference":
        run_reference(args, world, rank)
        return

    import torch
    import torch.distributed as dist

    torch.cuda.set_device(local)
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                device_id=torch.device(f"cuda:{local}"))

    from verdict_b200 import spec as specs
    from verdict_b200.engine import B200Engine
    from verdict_b200.synth import with_labels

    over = {} if args.layers is None else {"layers": args.layers}
    spec = with_labels(specs.preset(args.model, **over))
    n_batches = args.warmup + args.steps
    encoder = spec["arch"] == "encoder"
    batches = make_batches(rank, n_batches, args.batch, spec["vocab"], args.seed,
                           workload_of(spec, args.workload), spec.get("pad_id", 0),
                           LENGTHS.get(args.model, "lognormal-9b"))
    # Concurrency sweep (decoders, one GPU): other batch sizes of the same
    # workload, timed after the headline, each from its own seeded batches.
    sweep_sets = {}
    if args.sweep and not encoder and args.workload == "choice":
        for c, steps in SWEEP:
            sweep_sets[c] = make_batches(rank, 3 + steps, c, spec["vocab"], args.seed + 1000 + c,
                                         workload_of(spec, args.workload), spec.get("pad_id", 0),
                                         LENGTHS.get(args.model, "lognormal-9b"))
    every = batches + [b for bs in sweep_sets.values() for b in bs]
    max_len = max(int(b.real_len().max()) for b in every)
    max_tokens = max(int(b.real_len().sum()) for b in every)
    max_batch = max(b.b for b in every)
    eng = B200Engine(spec, device=local, max_tokens=max(max_tokens, 4096), max_rows=max(max_batch, 8),
                     max_seq=max(4096, max_len), attention=args.attention, fork=args.fork == "on",
                     gemm=args.gemm, raster_group=args.raster_group, gdn=args.gdn, act_dtype=args.act_dtype,
                     norm=args.norm, split_k=args.split_k == "on",
                     attention_persistent=args.attn_persistent == "on", attention_threads_per_row=args.attn_spr,
                     l2_hints=args.l2_hints == "on", pdl=args.pdl == "on")
    # Declared state-prefix lengths travel with the batch (host metadata, like real_len).
    shared = args.workload == "shared-prefix"
    width = eng.width if not encoder else max(b.k for b in batches)  # encoders: one logit per marker slot
    stream_ptr = eng.stream()
    stream = torch.cuda.ExternalStream(stream_ptr)

    # Device-resident inputs for every step.
    dev = []
    for b in batches:
        d = {k: torch.from_numpy(np.ascontiguousarray(v)).to(f"cuda:{local}") for k, v in dict(
            input_ids=b.input_ids, marker_pos=b.marker_pos, marker_mask=b.marker_mask.astype(np.uint8),
            nopts=b.nopts, qtype=b.qtype).items()}
        dev.append(d)
    out = torch.empty(args.batch, width, device=f"cuda:{local}", dtype=torch.float32)

    def step_dev(j):
        b = batches[j]
        eng.infer_device(b.b, b.l, b.k, {k: v.data_ptr() for k, v in dev[j].items()}, b.real_len(),
                         out.data_ptr(), width, prefix_len=b.prefix_len() if shared else None)

    def barrier():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    def reduce_max(x):
        return max_over_ranks(x, world, f"cuda:{local}")

    # Warm-up.
    for j in range(args.warmup):
        step_dev(j)
    eng.sync()
    barrier()

    # Timed region: device-resident inputs.  Encoder steps touch less than the
    # 126 MB L2, so a 256 MB write flushes it before each of their steps,
    # outside the step's events; decoder steps stream far more than L2.
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=f"cuda:{local}") if encoder else None
    clocks = Clocks(local)
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(2 * args.steps)]
    launches = 0
    with torch.cuda.stream(stream):
        for i in range(args.steps):
            if flush is not None:
                flush.fill_(i & 0xFF)
            evs[2 * i].record(stream)
            step_dev(args.warmup + i)
            evs[2 * i + 1].record(stream)
    eng.sync()
    launches = eng.last_stats()["launches"] * args.steps
    computed_tokens = eng.last_stats()["tokens"]  # last timed step, after any shared-prefix fork
    barrier()
    clk = clocks.stop()
    step_ms = [evs[2 * i].elapsed_time(evs[2 * i + 1]) for i in range(args.steps)]
    total_ms = reduce_max(float(np.sum(step_ms)) if encoder else evs[0].elapsed_time(evs[-1]))
    p99_ms = reduce_max(float(np.percentile(step_ms, 99)))
    decisions = args.batch * args.steps * world
    value = whole_job_rate(args.batch * args.steps, world, total_ms)
    tokens_per_step = float(np.mean([b.real_len().sum() for b in batches[args.warmup:]]))

    # Per-kernel timing pass (events around each launch), for the roofline.
    eng.lib.vd_set_profiling(eng.h, 1)
    kern = {}
    prof_steps = min(3, args.steps)
    acc_ms = np.zeros(8)
    acc_fl = np.zeros(8)
    acc_n = np.zeros(8)
    for i in range(prof_steps):
        b = batches[args.warmup + i]
        eng.infer_device(b.b, b.l, b.k, {k: v.data_ptr() for k, v in dev[args.warmup + i].items()}, b.real_len(),
                         out.data_ptr(), width, sync=True, prefix_len=b.prefix_len() if shared else None)
        st = eng.last_stats()
        acc_ms += np.array(st["kernel_ms"][:])
        acc_fl += np.array(st["kernel_flops"][:])
        acc_n += np.array(st["kernel_launches"][:])
    eng.lib.vd_set_profiling(eng.h, 0)
    from verdict_b200._abi import KERNEL_CLASSES
    for c, name in enumerate(KERNEL_CLASSES):
        if acc_n[c] > 0:
            kern[name] = {"ms_per_step": acc_ms[c] / prof_steps, "launches_per_step": acc_n[c] / prof_steps,
                          "tflops": (acc_fl[c] / (acc_ms[c] / 1e3) / 1e12) if acc_ms[c] > 0 and acc_fl[c] > 0
                          else None}
    gu = 2  # VD_K_GATEUP
    gu_launch_ms = acc_ms[gu] / acc_n[gu]
    gu_flops = acc_fl[gu] / acc_n[gu]
    pk, pk_kind = peaks()
    peak = pk["bf16_tflops_sustained"]
    achieved = gu_flops / (gu_launch_ms / 1e3) / 1e12
    gemm_ms = acc_ms[:4].sum() / prof_steps
    gemm_tf = acc_fl[:4].sum() / (acc_ms[:4].sum() / 1e3) / 1e12
    cap_bytes, cap_tokens = GATEUP_TRAFFIC.get((args.model, args.gemm), (None, None))
    traffic = cap_bytes * tokens_per_step / cap_tokens if cap_bytes and not encoder else None
    roofline = {
        "kernel": ("gemm2_tcgen05_kernel<store> (FFN up projection with GELU, CTA pairs)" if encoder else
                   "gemm2_tcgen05_kernel<gated> (gate/up projection, CTA pairs)" if args.gemm == "2sm"
                   else "gemm_tcgen05_kernel<256,gated> (gate/up projection)"),
        "bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s", "frac": achieved / peak,
        "peak_source": f"{pk_kind} bf16_tflops_sustained (dense fp16 and bf16 share the tensor-core rate)",
        "traffic": traffic,
        "traffic_source": (f"ncu dram__bytes_read.sum + dram__bytes_write.sum of a {cap_tokens}-token gate/up launch "
                           f"({cap_bytes / 1e9:.3f} GB), scaled by tokens to this launch; a lower estimate (weights "
                           "re-streamed once per 4,096-row raster group)") if traffic else None,
        # 16-bit A rows in, the ffn-wide output (act(g)*u, or act(x W) for the
        # encoders' up projection) out, and W once (2 ffn rows when gated).
        "algorithmic_bytes_per_launch": 2.0 * tokens_per_step * (spec["hidden"] + spec["ffn"])
        + 2.0 * (1 if encoder else 2) * spec["ffn"] * spec["hidden"],
        "flops_per_launch": gu_flops, "launch_ms": gu_launch_ms,
        "all_gemms": {"tflops": gemm_tf, "frac": gemm_tf / peak, "ms_per_step": gemm_ms},
    }

    # End to end through the C ABI with pinned host buffers.
    e2e = None
    if not args.no_e2e:
        host = []
        for b in batches:
            pinned = {}
            for k, v in dict(ids=b.input_ids, mpos=b.marker_pos, mmask=b.marker_mask.astype(np.uint8),
                             nopts=b.nopts, qtype=b.qtype).items():
                t = torch.from_numpy(np.ascontiguousarray(v)).pin_memory()
                pinned[k] = t
            host.append(pinned)
        out_h = torch.empty(args.batch, width, dtype=torch.float32).pin_memory()

        def step_host(j):
            b, p = batches[j], host[j]
            from verdict_b200._abi import VdBatch, VD_MEM_HOST
            import ctypes
            st = VdBatch()
            st.b, st.l, st.k, st.memory = b.b, b.l, b.k, VD_MEM_HOST
            st.input_ids = ctypes.c_void_p(p["ids"].data_ptr())
            st.marker_pos = ctypes.c_void_p(p["mpos"].data_ptr())
            st.marker_mask = ctypes.c_void_p(p["mmask"].data_ptr())
            st.nopts = ctypes.c_void_p(p["nopts"].data_ptr())
            st.qtype = ctypes.c_void_p(p["qtype"].data_ptr())
            rl = b.real_len()
            st.real_len = ctypes.c_void_p(rl.ctypes.data)
            pl = b.prefix_len()
            if shared:
                st.prefix_len = ctypes.c_void_p(pl.ctypes.data)
            err = ctypes.create_string_buffer(512)
            rc = eng.lib.vd_infer(eng.h, ctypes.byref(st), ctypes.c_void_p(out_h.data_ptr()), width, err, 512)
            if rc != 0:
                raise RuntimeError(err.value.decode())
            return int(b.input_ids.nbytes + b.marker_pos.nbytes + b.b * b.k + b.nopts.nbytes + b.qtype.nbytes), \
                int(b.b * width * 4)

        for j in range(args.warmup):
            step_host(j)
        barrier()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        e2e_clocks = Clocks(local)
        e0.record(stream)
        h2d = d2h = 0
        host_ms, fwd_ms, enq_ms, call_ms = [], [], [], []
        parts = {"prep_ms": [], "upload_ms": [], "download_ms": [], "finish_ms": []}
        for i in range(args.steps):
            t0 = time.perf_counter()
            bi, bo = step_host(args.warmup + i)
            host_ms.append((time.perf_counter() - t0) * 1e3)
            st = eng.last_stats()
            fwd_ms.append(st["forward_ms"])
            enq_ms.append(st["enqueue_ms"])
            call_ms.append(st["host_ms"])
            for key, acc in parts.items():
                acc.append(st[key])
            h2d += bi
            d2h += bo
        e1.record(stream)
        barrier()
        e2e_clk = e2e_clocks.stop()
        e2e_ms = reduce_max(e0.elapsed_time(e1))
        e2e = {"value": whole_job_rate(args.batch * args.steps, world, e2e_ms), "unit": UNIT,
               "host_ms_per_call": float(np.mean(host_ms)), "device_forward_ms_per_call": float(np.mean(fwd_ms)),
               "library_call_ms": float(np.mean(call_ms)), "enqueue_ms_per_call": float(np.mean(enq_ms)),
               "call_breakdown_ms": {key: float(np.mean(acc)) for key, acc in parts.items()},
               "clocks": e2e_clk, "h2d_bytes_per_step": h2d // args.steps,
               "d2h_bytes_per_step": d2h // args.steps}

    sweep = None
    if sweep_sets:
        sweep = {}
        for c, bs in sweep_sets.items():
            dv = [{k: torch.from_numpy(np.ascontiguousarray(v)).to(f"cuda:{local}") for k, v in dict(
                input_ids=b.input_ids, marker_pos=b.marker_pos, marker_mask=b.marker_mask.astype(np.uint8),
                nopts=b.nopts, qtype=b.qtype).items()} for b in bs]
            o = torch.empty(c, width, device=f"cuda:{local}", dtype=torch.float32)

            def run_c(j, bs=bs, dv=dv, o=o):
                b = bs[j]
                eng.infer_device(b.b, b.l, b.k, {k: v.data_ptr() for k, v in dv[j].items()}, b.real_len(),
                                 o.data_ptr(), width)

            for j in range(3):
                run_c(j)
            eng.sync()
            ck = Clocks(local)
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * (len(bs) - 3))]
            with torch.cuda.stream(stream):
                for i in range(len(bs) - 3):
                    ev[2 * i].record(stream)
                    run_c(3 + i)
                    ev[2 * i + 1].record(stream)
            eng.sync()
            barrier()
            cl = ck.stop()
            ms = [ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(len(bs) - 3)]
            span = reduce_max(ev[0].elapsed_time(ev[-1]))
            sweep[f"c{c}"] = {"decisions_per_step_per_gpu": c, "steps": len(ms), "warmup": 3,
                              "value": whole_job_rate(c * len(ms), world, span), "unit": UNIT,
                              "ms_per_step": span / len(ms), "p99_ms": reduce_max(float(np.percentile(ms, 99))),
                              "ms_per_decision": span / len(ms) / c,
                              "mean_tokens_per_step_per_gpu": float(np.mean([b.real_len().sum() for b in bs[3:]])),
                              "sm_mhz": cl.get("sm_mhz"), "reasons": cl.get("reasons")}

    eng.close()
    models = None
    if args.extra_models and args.model == "onejev-9b" and args.workload == "choice":
        models = {m: other_model(m, per_step, n, 3, args.seed, local, rank, world, barrier, reduce_max)
                  for m, per_step, n in EXTRA_MODELS}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        if encoder:
            threads = host_threads()
            v, sample, _ = encoder_cpu_sample(spec, batches[0])
        else:
            v, sample, _, threads = cpu_baseline_decoder(spec, batches[args.warmup:])
        cpu = {"value": v, "unit": UNIT, "cores": threads, "kind": "port", "sample": sample}

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "p99_ms": p99_ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": args.act_dtype,
            "data": "synthetic (seeded; random-init weights generated on device)",
            "config": {"workload": workload_text(args.model, shared),
                       "model": args.model,
                       "layers": spec["layers"], "attention": args.attention, "fork": args.fork, "gemm": args.gemm,
                       "norm": args.norm, "split_k": args.split_k, "attn_persistent": args.attn_persistent,
                       "attn_threads_per_row": args.attn_spr, "l2_hints": args.l2_hints, "pdl": args.pdl,
                       "raster_group": args.raster_group or "default",
                       **({"gdn": args.gdn} if specs.is_hybrid(spec) else {}),
                       "decisions_per_step_per_gpu": args.batch, "mean_tokens_per_step": tokens_per_step,
                       "computed_tokens_last_step": int(computed_tokens),
                       "parallelism": f"replicas x{world} (one full-weight replica per GPU, no collectives)",
                       "l2": ("flushed: 256 MB written before each timed step, outside its events (the e2e "
                              "leg does not flush)" if encoder else
                              "no flush: each step streams every layer's weights (GBs) and the activations, far "
                              "above the 126 MB L2")},
            "e2e": e2e, "gpu_launches": int(launches), "clocks": clk, "roofline": roofline, "sweep": sweep,
            "models": models,
            "kernels": kern, "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
