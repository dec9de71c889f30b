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
// CTA with one thread per state column (dk = dv = 128: 128 fp32 registers of
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

// One (sequence, v head) per CTA of 128 threads; thread j owns column j of the
// head's state.
template <class T>
__global__ void __launch_bounds__(128) gdn_scan_kernel(GdnParams p) {
  __shared__ __align__(16) float kq[2][2][128];  // [buffer][k, q][dk]
  __shared__ float red[2][4];                     // per-warp sums of o^2, by token parity
  const int4 sg = p.segs[blockIdx.x];
  const int start = sg.x, len = sg.y;
  const int head = blockIdx.y;
  const int kh = head / (p.lv / p.lk);
  const int j = threadIdx.x, warp = j >> 5, lane = j & 31;
  const T* qkv = static_cast<const T*>(p.qkv);
  const T* proj = static_cast<const T*>(p.proj);
  T* out = static_cast<T*>(p.out);
  const int q_col = kh * 128, k_col = p.kd + kh * 128, v_col = 2 * p.kd + head * 128;
  const float w_norm = p.norm_w[j];

  float S[128];
#pragma unroll
  for (int i = 0; i < 128; ++i) S[i] = 0.0f;

  auto stage = [&](int t, int b) {
    const size_t row = static_cast<size_t>(start + t) * p.ld_qkv;
    kq[b][0][j] = Elem<T>::to(qkv[row + k_col + j]);
    kq[b][1][j] = Elem<T>::to(qkv[row + q_col + j]);
  };
  // The gated norm of the token whose o this thread holds: its head's sum of
  // squares was published in red[parity] before the last barrier.
  auto finish = [&](int t, float o) {
    const int b = t & 1;
    const float ss = red[b][0] + red[b][1] + red[b][2] + red[b][3];
    const float rstd = rsqrtf(ss / 128.0f + p.eps);
    const size_t tok = static_cast<size_t>(start + t);
    const float z = Elem<T>::to(proj[tok * p.ld_proj + p.col_z + head * 128 + j]);
    out[tok * p.ld_out + head * 128 + j] = Elem<T>::from(o * rstd * w_norm * silu_f(z));
  };

  if (len > 0) stage(0, 0);
  __syncthreads();
  float o_prev = 0.0f;
  for (int t = 0; t < len; ++t) {
    const int b = t & 1;
    if (t + 1 < len) stage(t + 1, b ^ 1);
    if (t > 0) finish(t - 1, o_prev);
    const size_t tok = static_cast<size_t>(start + t);
    const float decay = __expf(p.g[tok * p.lv + head]);
    const float beta = p.beta[tok * p.lv + head];
    const float v = Elem<T>::to(qkv[tok * p.ld_qkv + v_col + j]);
    const float4* k4 = reinterpret_cast<const float4*>(kq[b][0]);
    const float4* q4 = reinterpret_cast<const float4*>(kq[b][1]);
    float kv = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float4 k = k4[i];
      S[4 * i + 0] *= decay;
      S[4 * i + 1] *= decay;
      S[4 * i + 2] *= decay;
      S[4 * i + 3] *= decay;
      kv += S[4 * i + 0] * k.x + S[4 * i + 1] * k.y + S[4 * i + 2] * k.z + S[4 * i + 3] * k.w;
    }
    const float delta = (v - kv) * beta;
    float o = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) {
      const float4 k = k4[i], q = q4[i];
      S[4 * i + 0] += k.x * delta;
      S[4 * i + 1] += k.y * delta;
      S[4 * i + 2] += k.z * delta;
      S[4 * i + 3] += k.w * delta;
      o += S[4 * i + 0] * q.x + S[4 * i + 1] * q.y + S[4 * i + 2] * q.z + S[4 * i + 3] * q.w;
    }
    float ss = o * o;
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, s);
    if (lane == 0) red[b][warp] = ss;
    o_prev = o;
    __syncthreads();  // kq[b ^ 1] staged, red[b] published; kq[b] and red[b ^ 1] free again
  }
  if (len > 0) finish(len - 1, o_prev);
}

}  // namespace vd
