/*
 * vdexec — B200 (sm_100a) executor for Verdict's decision-model forward.
 *
 * C ABI that a Verdict `Engine` implementation binds instead of spawning the
 * Python torch executor.  It replaces:
 *   - trait Engine { infer, media_capable, shape_buckets, health }   src/engine.rs:28-40
 *   - TorchEngine::with_device / spawn_child_ready (model load)       src/torch_engine.rs:215-316
 *   - TorchEngine::infer / infer_json / unpack_logits / finish_rows   src/torch_engine.rs:34-114,354-494
 *   - the executor's per-batch forward + readout                      executor/torch_exec.py:2654-2972
 * The batch layout is the scheduler's CollatedBatch (src/scheduler.rs:79-103)
 * passed as plain pointers; nothing here uses torch or any C++ type.
 *
 * Threading: one handle per GPU; calls on one handle are serialised by an
 * internal mutex (the scheduler keeps one batch in flight per replica,
 * src/scheduler.rs:458-466); different handles may be used concurrently.
 * Errors: functions return 0 on success or a negative VD_E* code, and write a
 * UTF-8 message into err[0..errlen) when err is non-null.
 */
#ifndef VDEXEC_H_
#define VDEXEC_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define VDEXEC_ABI_VERSION 2

#if defined(__GNUC__)
#define VD_API __attribute__((visibility("default")))
#else
#define VD_API
#endif

/* Error codes. */
#define VD_OK 0
#define VD_EINVAL -1   /* malformed batch or arguments (maps to EngineError)      */
#define VD_ECUDA -2    /* CUDA failure; the handle is unhealthy afterwards         */
#define VD_EDEAD -3    /* the handle is dead (sticky fault earlier)                */
#define VD_ENOMEM -4   /* device allocation failed                                 */
#define VD_ESPEC -5    /* model spec / checkpoint not supported                    */
#define VD_EDEVICE -6  /* a kernel reported bad input (token id or slot range)     */

typedef struct vd_handle vd_handle;

/* Memory kinds of the bulk arrays in a vd_batch. */
#define VD_MEM_HOST 0
#define VD_MEM_DEVICE 1

/*
 * One collated batch, field for field the scheduler's CollatedBatch
 * (src/scheduler.rs:79-103): right-padded rows of length l.
 * Bulk arrays live in host or device memory as `memory` says; the per-row
 * metadata (real_len, real_k, prefix_len — RowMeta, src/scheduler.rs:98-103)
 * is always host memory.  Buffers are only read during the call.
 */
typedef struct vd_batch {
  int64_t b, l, k;
  int32_t memory;                 /* VD_MEM_HOST or VD_MEM_DEVICE                  */
  const int64_t* input_ids;       /* [b*l], padded with the pad id                 */
  const int64_t* attention_mask;  /* [b*l] or NULL (real_len is authoritative)     */
  const int64_t* marker_pos;      /* [b*k]                                         */
  const uint8_t* marker_mask;     /* [b*k] (bool)                                  */
  const int64_t* qtype;           /* [b] or NULL (marker families)                 */
  const int64_t* nopts;           /* [b] or NULL (letter families need it)         */
  const int64_t* real_len;        /* [b] host                                      */
  const int64_t* real_k;          /* [b] host or NULL                              */
  const int64_t* prefix_len;      /* [b] host or NULL                              */
} vd_batch;

/* Kernel classes of the per-kernel timing in vd_stats (profiling on). */
#define VD_K_QKV 0      /* QKV projection GEMM (+ q/k norm, RoPE epilogue) */
#define VD_K_O 1        /* attention output GEMM (+ residual)              */
#define VD_K_GATEUP 2   /* gate/up GEMM (+ gated activation)               */
#define VD_K_DOWN 3     /* down / FFN-out GEMM (+ residual)                */
#define VD_K_ATTN 4     /* varlen attention                                */
#define VD_K_NORM 5     /* RMSNorm / LayerNorm rows                        */
#define VD_K_OTHER 6    /* pack, embed, readout, marker scoring            */
#define VD_K_GDN 7      /* gated delta net: conv + gates, recurrence       */
#define VD_K_COUNT 8

/* Per-call statistics of the last completed vd_infer / vd_infer_async. */
typedef struct vd_stats {
  int64_t rows;          /* decisions in the batch                 */
  int64_t tokens;        /* real (packed) tokens                   */
  int64_t chunks;        /* forwards the batch was split into      */
  int64_t launches;      /* kernels this library launched         */
  double forward_ms;     /* device time of the forward(s)          */
  double gemm_flops;     /* algorithmic projection-GEMM FLOPs      */
  double attn_flops;     /* algorithmic attention FLOPs            */
  /* With profiling on (vd_set_profiling): device time, launches and
   * algorithmic FLOPs per kernel class VD_K_*, from CUDA events around each launch. */
  double kernel_ms[VD_K_COUNT];
  int64_t kernel_launches[VD_K_COUNT];
  double kernel_flops[VD_K_COUNT];
  /* Host wall time of the call and of its enqueue part (up to the last launch). */
  double host_ms;
  double enqueue_ms;
  /* Shared-prefix fork: groups formed, rows in them, prefix tokens computed
   * once instead of once per row. */
  int64_t fork_groups;
  int64_t fork_rows;
  int64_t shared_tokens;
  /* vd_infer on host memory: host time before the forward's first event
   * (validation, staging, uploads enqueued) and after its last launch
   * (download, synchronisation, error check); device time of the uploads
   * before the forward and of the download after it. */
  double prep_ms;
  double finish_ms;
  double upload_ms;
  double download_ms;
} vd_stats;

/*
 * Load a model onto `device` once (weights, workspaces, kernel tables).
 * model: JSON model spec (keys documented in verdict_b200/spec.py), or a path
 *   to a directory holding `vdexec.json` with the same spec.  Weights come
 *   from "checkpoint": a directory of safetensors files (`model.safetensors`,
 *   or the shards of `model.safetensors.index.json`; BF16, F16 or F32 tensors
 *   under their HF / DecisionModel state-dict names; relative to the spec
 *   file's directory), else they are generated from "seed".  A spec with a
 *   checkpoint and no "hidden" takes its shape from the checkpoint's HF
 *   config.json (decoders: Qwen3 / Qwen2 / Gemma; encoders: BERT / XLM-R
 *   under encoder/); decoders still need "label_ids" (the family's table,
 *   src/tokenize.rs:96-171) and default to "family": "letter_readout".
 * opts_json: NULL or {"max_tokens": N, "max_rows": N, "max_seq": N,
 *   "max_markers": N, "output": "logprobs"|"logits", "act_dtype":
 *   "fp16"|"bf16", "attention": "tc"|"tc2"|"mma", "prune_last_layer": bool,
 *   "fork": bool (default true: decoder rows that share a prefix — declared
 *   prefix_len, else a common prefix of >= 32 tokens — compute it once, as
 *   executor/torch_exec.py:1935-2022 does; planned on the host from the ids:
 *   host-memory batches always, device-memory batches when they pass
 *   prefix_len, at the cost of one copy back and synchronisation)}.
 * Replaces TorchEngine::with_device (src/torch_engine.rs:280-316) and the
 * executor's checkpoint load (executor/torch_exec.py:2341-2386).
 */
VD_API int vd_open(const char* model, int device, const char* opts_json, vd_handle** out, char* err, size_t errlen);

/*
 * Synchronous forward + readout of one collated batch.
 * Letter families (decoders, src/torch_engine.rs:452-494 rules): k must be 1,
 * nopts must be given, marker_mask[i] must be set; logits_out[b*out_width]
 * receives, per row, the log-softmax over the first nopts[i] option-label rows
 * (or raw label logits when opened with "output":"logits") and -1e4 in the
 * remaining columns (finish_rows, src/torch_engine.rs:97-114).
 * Marker family (encoders): logits_out[b*out_width] receives the scorer
 * logits of the k markers with -1e4 where marker_mask is false and for
 * columns >= k (DecisionModel.forward, convert/marker_head/marker_head_converter.py:40-57).
 * logits_out is host memory for VD_MEM_HOST batches and device memory for
 * VD_MEM_DEVICE batches.
 */
VD_API int vd_infer(vd_handle* h, const vd_batch* batch, float* logits_out, int64_t out_width, char* err, size_t errlen);

/*
 * Asynchronous variant for device-resident batches (memory = VD_MEM_DEVICE):
 * enqueues the forward on the handle's stream after work already submitted to
 * `stream` (a cudaStream_t, or NULL), makes `stream` wait for its completion,
 * and returns.  Input-range errors surface at the next vd_sync.
 */
VD_API int vd_infer_async(vd_handle* h, const vd_batch* batch, float* logits_out_dev, int64_t out_width, void* stream,
                   char* err, size_t errlen);

/* Wait for all work on the handle and report device-side input errors. */
VD_API int vd_sync(vd_handle* h, char* err, size_t errlen);

/* The handle's CUDA stream (cudaStream_t), for event timing by the caller. */
VD_API void* vd_stream(vd_handle* h);

/* Engine::shape_buckets (src/engine.rs:36-38): length classes; returns the count
 * (this executor packs ragged batches, so it reports none and returns 0). */
VD_API int vd_shape_buckets(vd_handle* h, int64_t* out, int64_t cap);

/* Engine::media_capable (src/engine.rs:32-34): always 0 (text-only path). */
VD_API int vd_media_capable(vd_handle* h);

/* Engine::health (src/engine.rs:40): 1 healthy, 0 after a sticky CUDA error. */
VD_API int vd_health(vd_handle* h);

/* Output width the model family produces (255/256 label rows for letter families). */
VD_API int64_t vd_label_width(vd_handle* h);

/* Turn per-kernel event timing on (1) or off (0) for later calls. */
VD_API int vd_set_profiling(vd_handle* h, int on);

/* Statistics of the last completed call. */
VD_API int vd_last_stats(vd_handle* h, vd_stats* out);

/* Free everything the handle owns. */
VD_API void vd_close(vd_handle* h);

/* The spec vd_open would load for `model`, as one JSON object (checkpoint
 * path resolved, HF config keys filled in); host only, no device needed.
 * VD_EINVAL when out[0..outlen) cannot hold it (the message gives the size). */
VD_API int vd_resolve_spec(const char* model, char* out, size_t outlen, char* err, size_t errlen);

/* ABI version (VDEXEC_ABI_VERSION). */
VD_API int vd_abi_version(void);

#ifdef __cplusplus
}
#endif

#endif /* VDEXEC_H_ */
