/*
 * vdexec kernel-level entry points: the individual sm_100a kernels of the
 * decision forward on caller-owned DEVICE buffers, for composing other
 * forwards and for testing each kernel against a reference implementation.
 *
 * These have no single counterpart in the reference (which runs cuBLAS / SDPA
 * through torch, executor/torch_exec.py:205-261); each entry names the torch op
 * it replaces.  All calls are synchronous on `stream` (a cudaStream_t, or NULL
 * for the legacy default stream) and return 0 or a negative VD_E* code from
 * vdexec.h with a message in err.
 */
#ifndef VDEXEC_KERNELS_H_
#define VDEXEC_KERNELS_H_

#include <stddef.h>
#include <stdint.h>

#include "vdexec.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Epilogues of vdk_gemm. */
#define VDK_EPI_STORE 0     /* out = act(A W^T + bias), 16-bit                                     */
#define VDK_EPI_RESIDUAL 1  /* out_f32 += A W^T + bias                                              */
#define VDK_EPI_GATED 2     /* out[:, j] = act(g_j) * u_j, 16-bit; W rows interleaved in 128-row blocks */
#define VDK_EPI_QKROPE 3    /* per-head q/k RMSNorm + rotary embedding (see vdk_gemm_qkrope)   */

/* 16-bit element types of A, W, qkv and 16-bit outputs. */
#define VDK_FP16 0
#define VDK_BF16 1

/* Activations. */
#define VDK_ACT_NONE 0
#define VDK_ACT_GELU_ERF 1
#define VDK_ACT_GELU_TANH 2
#define VDK_ACT_RELU 3
#define VDK_ACT_SILU 4

/*
 * tcgen05 GEMM: A [M, K] row-major, W [N, K] row-major (nn.Linear weight
 * layout), both of the 16-bit type `dtype`, fp32 accumulation; replaces
 * torch.nn.functional.linear.  N % 128 == 0 (N % 256 == 0 for
 * VDK_EPI_GATED), K % 64 == 0.
 * out: dtype [M, ld_out] (store, gated) or fp32 [M, ld_out] (residual).
 */
VD_API int vdk_gemm(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int dtype, int epi, int act,
                    const float* bias, void* out, int64_t ld_out, void* stream, char* err, size_t errlen);

/*
 * QKV projection with the attention-input epilogue: columns [0, q_cols) are
 * query heads and [q_cols, q_cols + k_cols) key heads of size head_dim (128 or
 * 256); each gets the optional bias, the optional per-head RMSNorm with gains
 * q_norm / k_norm (NULL: none; plus_one: gain = 1 + w) and the rotary embedding
 * at positions[m] with base theta; the remaining columns (values) are stored as
 * they are.  Replaces q_norm(q_proj(x)) / k_norm(k_proj(x)) + apply_rotary_pos_emb.
 */
VD_API int vdk_gemm_qkrope(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int dtype, const float* bias,
                           const float* q_norm, const float* k_norm, int q_cols, int k_cols, int head_dim,
                           int plus_one, float eps, const int32_t* positions, double theta, int max_pos, void* out,
                           int64_t ld_out, void* stream, char* err, size_t errlen);

/*
 * Varlen attention over packed rows.  qkv [T, ld_qkv] (16-bit dtype) holds query head h
 * at column q_col0 + h*head_dim and K/V head g at k_col0 / v_col0 + g*head_dim
 * (g = h / (heads / kv_heads)); cu_seqlens_host [nseq + 1] (host) delimits the
 * sequences; out [T, ld_out] (dtype) at column h*head_dim.  causal = 1 for
 * decoders.  Replaces F.scaled_dot_product_attention (is_causal) per sequence.
 */
VD_API int vdk_attention(const void* qkv, int64_t ld_qkv, int64_t q_col0, int64_t k_col0, int64_t v_col0, int heads,
                         int kv_heads, int head_dim, int dtype, int causal, const int32_t* cu_seqlens_host,
                         int64_t nseq, void* out, int64_t ld_out, void* stream, char* err, size_t errlen);

/*
 * The same attention on the 5th-generation tensor cores (tcgen05 MMAs with
 * TMEM accumulators, TMA-fed), causal with head_dim 128 or 256 or
 * bidirectional with head_dim 64, one query head per CTA, 128-row query tiles
 * and 64-key tiles; the kernel the engine uses for decoders with those head
 * sizes and for the marker-head encoders.  Same arguments and result as
 * vdk_attention; strides and column offsets multiples of 8.
 */
VD_API int vdk_attention_tc(const void* qkv, int64_t ld_qkv, int64_t q_col0, int64_t k_col0, int64_t v_col0,
                            int heads, int kv_heads, int head_dim, int dtype, int causal,
                            const int32_t* cu_seqlens_host, int64_t nseq, void* out, int64_t ld_out, void* stream,
                            char* err, size_t errlen);

/*
 * vdk_attention with no allocation of its own.  It has no counterpart in the
 * reference; it exists for callers that must not call cudaMalloc: a host
 * process whose GPU memory is entirely owned by another allocator (a serving
 * framework's caching pool that reserves the HBM budget up front), or a
 * latency-critical path where cudaMalloc/cudaFree would block on the device.
 *
 * Same arguments and results as vdk_attention.  The per-call work table (one
 * entry per 64-row query tile) lives in a fixed device array of 16384 entries
 * (512 KiB) that every GPU loading this library keeps until the process
 * exits; a batch needing more tiles (sum over sequences of ceil(len / 64)) is
 * rejected with VD_EINVAL before anything is launched.
 * The first call on a device looks up that array's device address (with the
 * device current) and keeps it; make that first call before any stream
 * capture.  All calls in a process share the one array per GPU and it keeps
 * the last call's contents; calls that overlapped on the GPU would race on it,
 * so each call holds a process-wide lock until its kernel has finished.  Every
 * entry a call reads is written by that same call, so nothing needs clearing.
 */
VD_API int vdk_attention_noalloc(const void* qkv, int64_t ld_qkv, int64_t q_col0, int64_t k_col0, int64_t v_col0,
                                 int heads, int kv_heads, int head_dim, int dtype, int causal,
                                 const int32_t* cu_seqlens_host, int64_t nseq, void* out, int64_t ld_out,
                                 void* stream, char* err, size_t errlen);

#ifdef __cplusplus
}
#endif

#endif /* VDEXEC_KERNELS_H_ */
