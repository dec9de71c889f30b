// Gated delta net (the linear-attention token mixer of Qwen3.5 text stacks,
// HF `Qwen3_5GatedDeltaNet`), prefill over packed ragged sequences.
//
//   proj = x @ [W_qkv; W_z; W_a; W_b]^T        (GEMM, one fused weight)
//   c    = silu(causal depthwise conv_K(proj[:, :C]))          C = 2*kd + vd
//   q, k = l2norm per 128-wide head (q also * 1/sqrt(dk)),  v = c[:, 2kd:]
//   beta = sigmoid(b),  g = -exp(A_log) * softplus(a + dt_bias)   per v head
//   per v head (k head = v head / (lv / lk)), state S [dk, dv] = 0 at each
//   sequence start, for every token:
//       S *= exp(g);  delta = (v - k^T S) * beta;  S += k delta^T;  o = q^T S
//   y    = RMSNorm(o over the head) * w * silu(z)               (gated norm)
//   out  = y @ W_out^T                          (GEMM, residual epilogue)
//
// gdn_conv_prep_kernel does the conv, the l2 norms and the gates for one token
// per CTA; gdn_scan_kernel runs the recurrence for one (sequence, v head) per
// CTA with two threads per state column (dk = dv = 128: 64 fp32 registers of
// state per thread), k and q of the next token staged in shared memory while
// the current one is consumed, and applies the gated norm of token t in step
// t + 1 (the head's sum of squares needs the CTA-wide reduction that step's
// barrier already provides).
#pragma once

#include "common.cuh"

namespace vd {

struct GdnParams {
  const void* proj;        // T [T, ld_proj]: conv input (C), z (vd), a (lv), b (lv)
  int ld_proj;
  const float* conv_w;     // [C, K]
  const float* A_log;      // [lv]
  const float* dt_bias;    // [lv]
  const float* norm_w;     // [dv]
  const int* positions;    // [T] position of the token inside its sequence
  int ntok;
  int kd, vd, lk, lv;      // key / value widths, key / value heads (head dims 128)
  int col_z, col_a, col_b; // column offsets in proj
  void* qkv;               // T [T, ld_qkv]: q (kd), k (kd), v (vd) after conv / norms
  int ld_qkv;
  float* g;                // [T, lv]
  float* beta;             // [T, lv]
  void* out;               // T [T, ld_out]: gated-norm output (vd)
  int ld_out;
  float q_scale;           // 1 / sqrt(dk)
  float eps;               // RMSNorm epsilon of the gated norm
  const int4* segs;        // packed sequences {start, len, col0, src_row}
};

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// One token per CTA (256 threads = 8 warps); warp w handles heads w, w + 8, ...
// of the 2*lk + lv conv heads (q heads, then k heads, then v heads), 4
// channels per lane.  K is the conv width.
template <class T, int K>
__global__ void __launch_bounds__(256) gdn_conv_prep_kernel(GdnParams p) {
  const int t = blockIdx.x;
  if (t >= p.ntok) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int pos = p.positions[t];
  const T* proj = static_cast<const T*>(p.proj);
  T* out = static_cast<T*>(p.qkv);
  const int heads = 2 * p.lk + p.lv;
  for (int h = warp; h < heads; h += 8) {
    const int c = h * 128 + lane * 4;
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float4* wr = reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(c) * K);
    float w[4][K];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
#pragma unroll
      for (int j = 0; j < K; j += 4) {
        const float4 v = __ldg(wr + (i * K + j) / 4);
        w[i][j] = v.x;
        if (j + 1 < K) w[i][j + 1] = v.y;
        if (j + 2 < K) w[i][j + 2] = v.z;
        if (j + 3 < K) w[i][j + 3] = v.w;
      }
    }
#pragma unroll
    for (int j = 0; j < K; ++j) {
      const int back = K - 1 - j;  // tokens before t
      if (back > pos) continue;    // before the sequence start: zero history
      const uint2 raw = *reinterpret_cast<const uint2*>(proj + static_cast<size_t>(t - back) * p.ld_proj + c);
      const float2 a = Elem<T>::unpack2(raw.x), b = Elem<T>::unpack2(raw.y);
      acc[0] += w[0][j] * a.x;
      acc[1] += w[1][j] * a.y;
      acc[2] += w[2][j] * b.x;
      acc[3] += w[3][j] * b.y;
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) acc[i] = silu_f(acc[i]);
    if (h < 2 * p.lk) {  // q or k head: l2 norm over its 128 channels
      float ss = acc[0] * acc[0] + acc[1] * acc[1] + acc[2] * acc[2] + acc[3] * acc[3];
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
      float r = rsqrtf(ss + 1e-6f);
      if (h < p.lk) r *= p.q_scale;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] *= r;
    }
    uint2 o;
    o.x = Elem<T>::pack2(acc[0], acc[1]);
    o.y = Elem<T>::pack2(acc[2], acc[3]);
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * p.ld_qkv + c) = o;
  }
  for (int h = threadIdx.x; h < p.lv; h += 256) {
    const float a = Elem<T>::to(proj[static_cast<size_t>(t) * p.ld_proj + p.col_a + h]);
    const float b = Elem<T>::to(proj[static_cast<size_t>(t) * p.ld_proj + p.col_b + h]);
    const float x = a + p.dt_bias[h];
    const float sp = x > 20.0f ? x : log1pf(__expf(x));  // softplus (threshold 20)
    p.g[static_cast<size_t>(t) * p.lv + h] = -__expf(p.A_log[h]) * sp;
    p.beta[static_cast<size_t>(t) * p.lv + h] = 1.0f / (1.0f + __expf(-b));
  }
}

// One (sequence, v head) per CTA of 256 threads; thread pair (2c, 2c+1) owns
// column c of the head's state, each thread 64 of its 128 rows (64 fp32
// registers), and the pair combines its two partial dot products with one
// shuffle.  Every global load is issued one token ahead of its use (k and q two
// tokens ahead, staged through shared memory one token ahead), so the
// per-token critical path is the state arithmetic only.
template <class T>
__global__ void __launch_bounds__(256, 1) gdn_scan_kernel(GdnParams p) {
  // [buffer][k, q][row half][64 rows + 4 pad]: the pad puts the two halves in
  // different banks, so the two threads of a pair read without conflict.
  __shared__ __align__(16) float kq[2][2][2][68];
  __shared__ float red[2][8];  // per-warp sums of o^2, by token parity
  const int4 sg = p.segs[blockIdx.x];
  const int start = sg.x, len = sg.y;
  const int head = blockIdx.y;
  const int kh = head / (p.lv / p.lk);
  const int tid = threadIdx.x, col = tid >> 1, half = tid & 1, warp = tid >> 5, lane = tid & 31;
  const T* qkv = static_cast<const T*>(p.qkv);
  const T* proj = static_cast<const T*>(p.proj);
  T* out = static_cast<T*>(p.out);
  // staging role: thread tid stages element (tid & 127) of k (tid < 128) or q
  const int st_kind = tid >> 7, st_idx = tid & 127;
  const int st_col = st_kind ? kh * 128 + st_idx : p.kd + kh * 128 + st_idx;
  const int v_col = 2 * p.kd + head * 128 + col;
  const int z_col = p.col_z + head * 128 + col;
  const float w_norm = p.norm_w[col];
  if (len <= 0) return;

  auto row = [&](int t) { return static_cast<size_t>(start + t); };
  float S[64];
#pragma unroll
  for (int i = 0; i < 64; ++i) S[i] = 0.0f;

  kq[0][st_kind][st_idx >> 6][st_idx & 63] = Elem<T>::to(qkv[row(0) * p.ld_qkv + st_col]);
  T st_next = Elem<T>::from(0.0f);
  if (len > 1) st_next = qkv[row(1) * p.ld_qkv + st_col];
  T v_cur = qkv[row(0) * p.ld_qkv + v_col];
  float g_cur = p.g[row(0) * p.lv + head], b_cur = p.beta[row(0) * p.lv + head];
  T z_cur = proj[row(0) * p.ld_proj + z_col];
  T z_prev = z_cur;
  float o_prev = 0.0f;
  __syncthreads();

  for (int t = 0; t < len; ++t) {
    const int b = t & 1;
    if (t + 1 < len) kq[b ^ 1][st_kind][st_idx >> 6][st_idx & 63] = Elem<T>::to(st_next);
    if (t + 2 < len) st_next = qkv[row(t + 2) * p.ld_qkv + st_col];
    T v_nxt = v_cur, z_nxt = z_cur;
    float g_nxt = g_cur, b_nxt = b_cur;
    if (t + 1 < len) {
      v_nxt = qkv[row(t + 1) * p.ld_qkv + v_col];
      g_nxt = p.g[row(t + 1) * p.lv + head];
      b_nxt = p.beta[row(t + 1) * p.lv + head];
      z_nxt = proj[row(t + 1) * p.ld_proj + z_col];
    }
    // The gated norm of token t-1 (its head's sum of squares is in red[b ^ 1]).
    if (t > 0 && half == 0) {
      float ss = 0.0f;
#pragma unroll
      for (int w = 0; w < 8; ++w) ss += red[b ^ 1][w];
      const float rstd = rsqrtf(ss / 128.0f + p.eps);
      out[row(t - 1) * p.ld_out + head * 128 + col] =
          Elem<T>::from(o_prev * rstd * w_norm * silu_f(Elem<T>::to(z_prev)));
    }
    // Token t.
    const float decay = __expf(g_cur);
    const float4* k4 = reinterpret_cast<const float4*>(kq[b][0][half]);
    const float4* q4 = reinterpret_cast<const float4*>(kq[b][1][half]);
    float kv0 = 0.0f, kv1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float4 ka = k4[i], kb = k4[i + 1];
#pragma unroll
      for (int e = 0; e < 8; ++e) S[4 * i + e] *= decay;
      kv0 += S[4 * i + 0] * ka.x + S[4 * i + 1] * ka.y + S[4 * i + 2] * ka.z + S[4 * i + 3] * ka.w;
      kv1 += S[4 * i + 4] * kb.x + S[4 * i + 5] * kb.y + S[4 * i + 6] * kb.z + S[4 * i + 7] * kb.w;
    }
    float kv = kv0 + kv1;
    kv += __shfl_xor_sync(0xffffffffu, kv, 1);
    const float delta = (Elem<T>::to(v_cur) - kv) * b_cur;
    float o0 = 0.0f, o1 = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; i += 2) {
      const float4 ka = k4[i], kb = k4[i + 1], qa = q4[i], qb = q4[i + 1];
      S[4 * i + 0] += ka.x * delta;
      S[4 * i + 1] += ka.y * delta;
      S[4 * i + 2] += ka.z * delta;
      S[4 * i + 3] += ka.w * delta;
      S[4 * i + 4] += kb.x * delta;
      S[4 * i + 5] += kb.y * delta;
      S[4 * i + 6] += kb.z * delta;
      S[4 * i + 7] += kb.w * delta;
      o0 += S[4 * i + 0] * qa.x + S[4 * i + 1] * qa.y + S[4 * i + 2] * qa.z + S[4 * i + 3] * qa.w;
      o1 += S[4 * i + 4] * qb.x + S[4 * i + 5] * qb.y + S[4 * i + 6] * qb.z + S[4 * i + 7] * qb.w;
    }
    float o = o0 + o1;
    o += __shfl_xor_sync(0xffffffffu, o, 1);
    float ss = half == 0 ? o * o : 0.0f;
#pragma unroll
    for (int sft = 16; sft > 0; sft >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sft);
    if (lane == 0) red[b][warp] = ss;
    o_prev = o;
    z_prev = z_cur;
    v_cur = v_nxt;
    g_cur = g_nxt;
    b_cur = b_nxt;
    z_cur = z_nxt;
    __syncthreads();  // kq[b ^ 1] staged, red[b] published; kq[b] and red[b ^ 1] free again
  }
  if (half == 0) {
    float ss = 0.0f;
#pragma unroll
    for (int w = 0; w < 8; ++w) ss += red[(len - 1) & 1][w];
    const float rstd = rsqrtf(ss / 128.0f + p.eps);
    out[row(len - 1) * p.ld_out + head * 128 + col] =
        Elem<T>::from(o_prev * rstd * w_norm * silu_f(Elem<T>::to(z_prev)));
  }
}

}  // namespace vd
