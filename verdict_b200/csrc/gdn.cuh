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
// gdn_conv_prep_kernel does the conv, the l2 norms and the gates (32-token
// tiles, one conv head per warp).  The recurrence and the gated norm run in
// gdn_chunk_kernel (64-token chunks on the tensor cores, the default) or in
// gdn_scan_kernel (token by token: one (sequence, v head) per CTA with two
// threads per state column (dk = dv = 128: 64 fp32 registers of state per
// thread), k and q of the next token staged in shared memory while the
// current one is consumed, and the gated norm of token t applied in step t + 1
// (the head's sum of squares needs the CTA-wide reduction that step's barrier
// already provides)).
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

__device__ __forceinline__ float silu_f(float x) { return x * __fdividef(1.0f, 1.0f + __expf(-x)); }

// Tiles of GDN_CONV_TOKENS tokens; warp w of block row y owns conv head
// 8y + w (q heads, then k heads, then v heads, 128 channels each, 4 per
// lane), keeps its conv weights and the last K - 1 inputs in registers and
// walks the tile's tokens in order, so every input row is read once.  The
// history restarts at each sequence start (position 0) and, at the tile start,
// is loaded for the tokens the position says are inside the sequence.  The
// last block row computes the gates g and beta of the tile's tokens.
constexpr int GDN_CONV_TOKENS = 32;

template <class T, int K>
__global__ void __launch_bounds__(256) gdn_conv_prep_kernel(GdnParams p) {
  const int t_begin = blockIdx.x * GDN_CONV_TOKENS;
  const int t_end = min(t_begin + GDN_CONV_TOKENS, p.ntok);
  const int heads = 2 * p.lk + p.lv;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const T* proj = static_cast<const T*>(p.proj);
  if (blockIdx.y == gridDim.y - 1) {  // gates
    for (int i = threadIdx.x; i < GDN_CONV_TOKENS * p.lv; i += 256) {
      const int t = t_begin + i / p.lv, h = i % p.lv;
      if (t >= t_end) break;
      const float a = Elem<T>::to(proj[static_cast<size_t>(t) * p.ld_proj + p.col_a + h]);
      const float b = Elem<T>::to(proj[static_cast<size_t>(t) * p.ld_proj + p.col_b + h]);
      const float x = a + p.dt_bias[h];
      const float sp = x > 20.0f ? x : log1pf(__expf(x));  // softplus (threshold 20)
      p.g[static_cast<size_t>(t) * p.lv + h] = -__expf(p.A_log[h]) * sp;
      p.beta[static_cast<size_t>(t) * p.lv + h] = __fdividef(1.0f, 1.0f + __expf(-b));
    }
    return;
  }
  const int h = blockIdx.y * 8 + warp;
  if (h >= heads) return;
  const int c = h * 128 + lane * 4;
  T* out = static_cast<T*>(p.qkv);
  float w[4][K];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float4* wr = reinterpret_cast<const float4*>(p.conv_w + static_cast<size_t>(c + i) * K);
#pragma unroll
    for (int j = 0; j < K; j += 4) {
      const float4 v = __ldg(wr + j / 4);
      w[i][j] = v.x;
      if (j + 1 < K) w[i][j + 1] = v.y;
      if (j + 2 < K) w[i][j + 2] = v.z;
      if (j + 3 < K) w[i][j + 3] = v.w;
    }
  }
  const bool is_qk = h < 2 * p.lk;
  const float scale = h < p.lk ? p.q_scale : 1.0f;
  auto load4 = [&](int t, float (&x)[4]) {
    const uint2 raw = *reinterpret_cast<const uint2*>(proj + static_cast<size_t>(t) * p.ld_proj + c);
    const float2 a = Elem<T>::unpack2(raw.x), b = Elem<T>::unpack2(raw.y);
    x[0] = a.x;
    x[1] = a.y;
    x[2] = b.x;
    x[3] = b.y;
  };
  // hist[j]: input of token t - 1 - j (0 outside the sequence)
  float hist[K - 1][4];
  {
    const int pos0 = p.positions[t_begin];
#pragma unroll
    for (int j = 0; j < K - 1; ++j) {
      if (j < pos0) {
        load4(t_begin - 1 - j, hist[j]);
      } else {
#pragma unroll
        for (int i = 0; i < 4; ++i) hist[j][i] = 0.0f;
      }
    }
  }
  for (int t = t_begin; t < t_end; ++t) {
    float x[4];
    load4(t, x);
    if (p.positions[t] == 0) {
#pragma unroll
      for (int j = 0; j < K - 1; ++j)
#pragma unroll
        for (int i = 0; i < 4; ++i) hist[j][i] = 0.0f;
    }
    float acc[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float a = w[i][K - 1] * x[i];
#pragma unroll
      for (int j = 0; j < K - 1; ++j) a += w[i][K - 2 - j] * hist[j][i];
      acc[i] = silu_f(a);
    }
    if (is_qk) {  // l2 norm over the head's 128 channels
      float ss = acc[0] * acc[0] + acc[1] * acc[1] + acc[2] * acc[2] + acc[3] * acc[3];
#pragma unroll
      for (int sft = 16; sft > 0; sft >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, sft);
      const float r = rsqrtf(ss + 1e-6f) * scale;
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] *= r;
    }
    uint2 o;
    o.x = Elem<T>::pack2(acc[0], acc[1]);
    o.y = Elem<T>::pack2(acc[2], acc[3]);
    *reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * p.ld_qkv + c) = o;
#pragma unroll
    for (int j = K - 2; j > 0; --j)
#pragma unroll
      for (int i = 0; i < 4; ++i) hist[j][i] = hist[j - 1][i];
#pragma unroll
    for (int i = 0; i < 4; ++i) hist[0][i] = x[i];
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

// ---------------------------------------------------------------------------
// Chunked form of the same recurrence on the tensor cores (mma.sync m16n8k16,
// fp32 accumulate), chunks of C = 64 tokens.  For a chunk entered with state
// S0, let G_t be the inclusive sum of g from the chunk start to token t.
// Unrolling the per-token rule inside the chunk gives, for the deltas
// d_t = (v_t - k_t^T S_{t-1}) b_t of all its tokens at once,
//     (I + A) D = R,   R = diag(b) (V - diag(e^G) K S0),
//     A[t,s] = b_t e^(G_t - G_s) (k_t . k_s)   for s < t   (0 otherwise);
// then
//     O  = diag(e^G) Q S0 + P D,   P[t,s] = e^(G_t - G_s) (q_t . k_s), s <= t,
//     S1 = e^(G_C) S0 + (diag(e^(G_C - G)) K)^T D.
// Every exponent is <= 0 (g <= 0 and s <= t), so nothing overflows.  Tokens
// past the sequence end enter as k = q = v = 0, g = b = 0 and drop out.
//
// (I + A) D = R is solved by 16-row blocks: the four diagonal blocks are
// inverted in fp32 by forward substitution (one warp each), then for block
// rows i = 0..3,  D_i = (I + A_ii)^-1 (R_i - sum_{k<i} A_ik D_k),  all on the
// tensor cores.  The value columns are independent, so warp w carries its own
// 16 columns through the four block rows with no cross-warp dependency.
//
// One (sequence, value head) per CTA of 8 warps, chunks in order.  The state
// stays in fp32 registers across chunks (warp w holds key rows 16w..16w+15,
// all 128 value columns, as mma accumulators) with a 16-bit copy in shared
// memory for the K S0 / Q S0 products.  K, Q, V and the gates of chunk i + 1
// and z of chunk i load (cp.async) while chunk i computes.
// ---------------------------------------------------------------------------
struct GdnChunkConfig {
  static constexpr int C = 64;    // tokens per chunk
  static constexpr int D = 128;   // key = value head dim
  static constexpr int TILE = C * D * 2;          // one [64][128] 16-bit tile
  static constexpr int KQV = 3 * TILE;            // K, Q, V of one chunk (two buffers)
  static constexpr int OFF_Z = 2 * KQV;           // z of the current chunk
  static constexpr int OFF_S = OFF_Z + TILE;      // [128][128] 16-bit state copy
  static constexpr int OFF_R = OFF_S + 2 * TILE;
  static constexpr int OFF_D = OFF_R + TILE;
  static constexpr int OFF_P = OFF_D + TILE;      // [64][64] 16-bit
  static constexpr int OFF_A = OFF_P + C * C * 2; // [64][64] 16-bit, -A below the diagonal blocks
  static constexpr int OFF_TII = OFF_A + C * C * 2;  // 4 x [16][16] 16-bit diagonal-block inverses
  static constexpr int OFF_X = OFF_TII + 4 * 512;    // 8 warps x [16][16] 16-bit scratch
  static constexpr int OFF_F32 = OFF_X + 8 * 512;
  static constexpr int F32_ADIAG = 0;             // 4 x [16][17] fp32 diagonal blocks of A
  static constexpr int F32_G = 4 * 16 * 17;       // [2][64] gates g (then G), by buffer
  static constexpr int F32_B = F32_G + 2 * C;     // [2][64] beta
  static constexpr int F32_RED = F32_B + 2 * C;   // [64][2] row sums of o^2
  static constexpr int F32_COUNT = F32_RED + 2 * C;
  static constexpr int SMEM_BYTES = OFF_F32 + F32_COUNT * 4;
};

// Byte offset of element (r, col) in a swizzled [rows][W] 16-bit tile.
template <int W>
__device__ __forceinline__ uint32_t gdn_elem(int r, int col) {
  return static_cast<uint32_t>(r * W * 2 + ((((col >> 3) ^ (r & 7)) << 4) | ((col & 7) << 1)));
}
// Byte offset of 16-byte chunk c of row r in a swizzled [rows][W] 16-bit tile.
template <int W>
__device__ __forceinline__ uint32_t gdn_chunk16(int r, int c) {
  return static_cast<uint32_t>(r * W * 2 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

template <class T>
__global__ void __launch_bounds__(256, 1) gdn_chunk_kernel(GdnParams p) {
  using Cfg = GdnChunkConfig;
  constexpr int C = Cfg::C, D = Cfg::D;
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t base = smem_u32(smem);
  const uint32_t sS = base + Cfg::OFF_S, sD = base + Cfg::OFF_D, sZ = base + Cfg::OFF_Z;
  const uint32_t sP = base + Cfg::OFF_P, sA = base + Cfg::OFF_A, sTii = base + Cfg::OFF_TII;
  float* f32 = reinterpret_cast<float*>(smem + Cfg::OFF_F32);
  float* sAd = f32 + Cfg::F32_ADIAG;
  float* sRed = f32 + Cfg::F32_RED;

  // blockIdx.x: value head (fastest, so the heads of the longest sequences,
  // listed first, start first), blockIdx.y: sequence
  const int4 sg = p.segs[blockIdx.y];
  const int start = sg.x, len = sg.y;
  if (len <= 0) return;
  const int head = blockIdx.x;
  const int kh = head / (p.lv / p.lk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int wr = warp & 3;
  const T* qkv = static_cast<const T*>(p.qkv);
  const T* proj = static_cast<const T*>(p.proj);
  T* out = static_cast<T*>(p.out);
  const int n_chunks = (len + C - 1) / C;

  // K, Q, V rows of chunk ci (zero past the end) and its gates into buffer b.
  auto load_chunk = [&](int ci, int b) {
    const int c0 = ci * C, valid = min(C, len - c0);
    for (int i = tid; i < 3 * C * (D / 8); i += 256) {
      const int tile = i / (C * (D / 8)), r = (i >> 4) & (C - 1), c = i & 15;
      const bool ok = r < valid;
      const int col = tile == 0 ? p.kd + kh * D : (tile == 1 ? kh * D : 2 * p.kd + head * D);  // K, Q, V
      cp_async16(base + b * Cfg::KQV + tile * Cfg::TILE + gdn_chunk16<D>(r, c),
                 qkv + static_cast<size_t>(start + c0 + (ok ? r : 0)) * p.ld_qkv + col + c * 8, ok);
    }
    if (tid < 2 * C) {
      const int t = tid & (C - 1);
      const bool ok = t < valid;
      const float* src = (tid < C ? p.g : p.beta) + static_cast<size_t>(start + c0 + (ok ? t : 0)) * p.lv + head;
      cp_async4(smem_u32(f32 + (tid < C ? Cfg::F32_G : Cfg::F32_B) + b * C + t), src, ok);
    }
    cp_async_commit();
  };
  auto load_z = [&](int ci) {
    const int c0 = ci * C, valid = min(C, len - c0);
    for (int i = tid; i < C * (D / 8); i += 256) {
      const int r = i >> 4, c = i & 15;
      const bool ok = r < valid;
      cp_async16(sZ + gdn_chunk16<D>(r, c),
                 proj + static_cast<size_t>(start + c0 + (ok ? r : 0)) * p.ld_proj + p.col_z + head * D + c * 8, ok);
    }
    cp_async_commit();
  };

  // Fragment coordinates of the [64 x 128] products: rows r0.., columns c0n..
  const int r0 = 16 * wr, c0n = 64 * (warp >> 2);
  const int t0 = r0 + (lane >> 2);

  float S[16][4];  // state rows 16*warp + lane/4 (+8), columns nb*8 + 2*(lane&3) (+1)
#pragma unroll
  for (int i = 0; i < 16; ++i) S[i][0] = S[i][1] = S[i][2] = S[i][3] = 0.0f;

  load_chunk(0, 0);
  float2 wn[8];  // gated-norm weights of this thread's output columns
#pragma unroll
  for (int nb = 0; nb < 8; ++nb) wn[nb] = *reinterpret_cast<const float2*>(p.norm_w + c0n + nb * 8 + 2 * (lane & 3));
  for (int ci = 0; ci < n_chunks; ++ci) {
    const int c0 = ci * C;
    const int valid = min(C, len - c0);
    const bool first = ci == 0, last = ci + 1 == n_chunks;
    const int buf = ci & 1;
    const uint32_t sK = base + buf * Cfg::KQV, sQ = sK + Cfg::TILE;  // V at sK + 2 * TILE, read by byte offset
    uint8_t* kbytes = smem + buf * Cfg::KQV;
    float* sG = f32 + Cfg::F32_G + buf * C;
    float* sB = f32 + Cfg::F32_B + buf * C;
    __syncthreads();  // the previous chunk is done with z, the other K/Q/V buffer and the scratch
    load_z(ci);
    if (!last) {
      load_chunk(ci + 1, buf ^ 1);
      cp_async_wait<2>();
    } else {
      cp_async_wait<1>();
    }
    __syncthreads();
    if (warp == 0) {  // inclusive prefix sum of g over the chunk (two tokens per lane)
      const float a = sG[2 * lane], b = sG[2 * lane + 1];
      float x = a + b;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, x, o);
        if (lane >= o) x += y;
      }
      sG[2 * lane] = x - b;
      sG[2 * lane + 1] = x;
    }
    __syncthreads();

    // (1) warps 0-3: A = b_t e^(G_t-G_s) K K^T (s < t): diagonal blocks fp32,
    // blocks left of them negated in 16 bits;  warps 4-7: P (s <= t), 16-bit.
    // Key blocks right of the row block are zero and skipped.
    {
      const uint32_t sM = warp < 4 ? sK : sQ;
      float acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i][0] = acc[i][1] = acc[i][2] = acc[i][3] = 0.0f;
#pragma unroll
      for (int ks = 0; ks < D / 16; ++ks) {
        uint32_t a[4];
        ldmatrix_x4(sM + gdn_chunk16<D>(r0 + (lane & 15), ks * 2 + (lane >> 4)), a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nb2 = 0; nb2 < 4; ++nb2) {
          if (nb2 > wr) continue;
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4(sK + gdn_chunk16<D>(nb2 * 16 + (lane & 7) + ((lane >> 4) << 3), ks * 2 + ((lane >> 3) & 1)), b0,
                      b1, b2, b3);
          mma_16816<T>(acc[2 * nb2], a, b0, b1);
          mma_16816<T>(acc[2 * nb2 + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        if ((nb >> 1) > wr) continue;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int t = t0 + 8 * h, s = nb * 8 + 2 * (lane & 3);
          const float gt = sG[t];
          if (warp < 4) {
            const float bt = sB[t];
            const float v0 = s < t ? bt * __expf(gt - sG[s]) * acc[nb][2 * h] : 0.0f;
            const float v1 = s + 1 < t ? bt * __expf(gt - sG[s + 1]) * acc[nb][2 * h + 1] : 0.0f;
            if ((nb >> 1) == wr) {
              float* ad = sAd + wr * 272 + (t - r0) * 17 + (s - r0);
              ad[0] = v0;
              ad[1] = v1;
            } else {
              *reinterpret_cast<uint32_t*>(smem + Cfg::OFF_A + gdn_elem<C>(t, s)) = Elem<T>::pack2(-v0, -v1);
            }
          } else {
            const float v0 = s <= t ? __expf(gt - sG[s]) * acc[nb][2 * h] : 0.0f;
            const float v1 = s + 1 <= t ? __expf(gt - sG[s + 1]) * acc[nb][2 * h + 1] : 0.0f;
            *reinterpret_cast<uint32_t*>(smem + Cfg::OFF_P + gdn_elem<C>(t, s)) = Elem<T>::pack2(v0, v1);
          }
        }
      }
    }

    // (2) R = b (V - e^G K S0) -> sR;  O = e^G Q S0 kept in registers.
    float o[8][4];
    {
      float ks_acc[8][4];
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        ks_acc[i][0] = ks_acc[i][1] = ks_acc[i][2] = ks_acc[i][3] = 0.0f;
        o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
      }
      if (!first) {
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          uint32_t aK[4], aQ[4];
          const uint32_t off = gdn_chunk16<D>(r0 + (lane & 15), kk * 2 + (lane >> 4));
          ldmatrix_x4(sK + off, aK[0], aK[1], aK[2], aK[3]);
          ldmatrix_x4(sQ + off, aQ[0], aQ[1], aQ[2], aQ[3]);
#pragma unroll
          for (int nd2 = 0; nd2 < 4; ++nd2) {
            uint32_t b0, b1, b2, b3;
            ldmatrix_x4_trans(sS + gdn_chunk16<D>(kk * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                                  (c0n >> 3) + nd2 * 2 + (lane >> 4)),
                              b0, b1, b2, b3);
            mma_16816<T>(ks_acc[2 * nd2], aK, b0, b1);
            mma_16816<T>(ks_acc[2 * nd2 + 1], aK, b2, b3);
            mma_16816<T>(o[2 * nd2], aQ, b0, b1);
            mma_16816<T>(o[2 * nd2 + 1], aQ, b2, b3);
          }
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int t = t0 + 8 * h;
        const float eg = __expf(sG[t]), bt = sB[t];
#pragma unroll
        for (int nb = 0; nb < 8; ++nb) {
          const int col = c0n + nb * 8 + 2 * (lane & 3);
          const uint32_t off = gdn_elem<D>(t, col);
          const float2 v = Elem<T>::unpack2(*reinterpret_cast<const uint32_t*>(kbytes + 2 * Cfg::TILE + off));
          *reinterpret_cast<uint32_t*>(smem + Cfg::OFF_R + off) =
              Elem<T>::pack2(bt * (v.x - eg * ks_acc[nb][2 * h]), bt * (v.y - eg * ks_acc[nb][2 * h + 1]));
          o[nb][2 * h] *= eg;
          o[nb][2 * h + 1] *= eg;
        }
      }
    }
    __syncthreads();

    // (3) Warps 0-3 invert diagonal block w of I + A (lane j: column j);
    // warps 4-7 scale K rows by e^(G_C - G_t) for the state update.
    if (warp < 4) {
      if (lane < 16) {
        const float* ad = sAd + warp * 272;
        const int j = lane;
        float x[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          float a0 = i == j ? 1.0f : 0.0f, a1 = 0.0f;  // two chains: half the dependent FMA latency
#pragma unroll
          for (int m = 0; m + 1 < i; m += 2) {
            a0 -= ad[i * 17 + m] * x[m];
            a1 -= ad[i * 17 + m + 1] * x[m + 1];
          }
          if (i & 1) a0 -= ad[i * 17 + i - 1] * x[i - 1];
          x[i] = a0 + a1;
        }
        T* tii = reinterpret_cast<T*>(smem + Cfg::OFF_TII + warp * 512);
#pragma unroll
        for (int i = 0; i < 16; ++i) tii[i * 16 + j] = Elem<T>::from(x[i]);
      }
    } else if (!last) {
      const float gc = sG[C - 1];
      for (int i = tid - 128; i < C * (D / 8); i += 128) {
        const int r = i >> 4, c = i & 15;
        const float f = __expf(gc - sG[r]);
        uint4* q = reinterpret_cast<uint4*>(kbytes + gdn_chunk16<D>(r, c));
        uint4 v = *q;
        uint32_t* w = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 x = Elem<T>::unpack2(w[e]);
          w[e] = Elem<T>::pack2(x.x * f, x.y * f);
        }
        *q = v;
      }
    }
    __syncthreads();

    // (4) Block forward substitution for this warp's 16 value columns.
    {
      const int cw = 16 * warp;
      uint8_t* xs = smem + Cfg::OFF_X + warp * 512;
      const uint32_t sX = base + Cfg::OFF_X + warp * 512;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float acc[2][4];
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const float2 r = Elem<T>::unpack2(*reinterpret_cast<const uint32_t*>(
                smem + Cfg::OFF_R + gdn_elem<D>(16 * i + (lane >> 2) + 8 * h, cw + nt * 8 + 2 * (lane & 3))));
            acc[nt][2 * h] = r.x;
            acc[nt][2 * h + 1] = r.y;
          }
        }
#pragma unroll
        for (int k = 0; k < 3; ++k) {
          if (k >= i) continue;
          uint32_t a[4], b0, b1, b2, b3;
          ldmatrix_x4(sA + gdn_chunk16<C>(16 * i + (lane & 15), 2 * k + (lane >> 4)), a[0], a[1], a[2], a[3]);
          ldmatrix_x4_trans(sD + gdn_chunk16<D>(16 * k + (lane & 7) + (((lane >> 3) & 1) << 3), (cw >> 3) + (lane >> 4)),
                            b0, b1, b2, b3);
          mma_16816<T>(acc[0], a, b0, b1);
          mma_16816<T>(acc[1], a, b2, b3);
        }
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            *reinterpret_cast<uint32_t*>(xs + ((lane >> 2) + 8 * h) * 32 + (nt * 8 + 2 * (lane & 3)) * 2) =
                Elem<T>::pack2(acc[nt][2 * h], acc[nt][2 * h + 1]);
          }
        }
        __syncwarp();
        uint32_t a[4], b0, b1, b2, b3;
        ldmatrix_x4_trans(sX + ((lane & 7) + (((lane >> 3) & 1) << 3)) * 32 + (lane >> 4) * 16, b0, b1, b2, b3);
        ldmatrix_x4(sTii + i * 512 + (lane & 15) * 32 + (lane >> 4) * 16, a[0], a[1], a[2], a[3]);
        float d[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
        mma_16816<T>(d[0], a, b0, b1);
        mma_16816<T>(d[1], a, b2, b3);
#pragma unroll
        for (int nt = 0; nt < 2; ++nt) {
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            *reinterpret_cast<uint32_t*>(
                smem + Cfg::OFF_D + gdn_elem<D>(16 * i + (lane >> 2) + 8 * h, cw + nt * 8 + 2 * (lane & 3))) =
                Elem<T>::pack2(d[nt][2 * h], d[nt][2 * h + 1]);
          }
        }
        __syncwarp();
      }
    }
    __syncthreads();

    // (5a) O += P D (key blocks right of the row block are zero in P).
#pragma unroll
    for (int ks = 0; ks < C / 16; ++ks) {
      if (ks > wr) continue;
      uint32_t a[4];
      ldmatrix_x4(sP + gdn_chunk16<C>(r0 + (lane & 15), ks * 2 + (lane >> 4)), a[0], a[1], a[2], a[3]);
#pragma unroll
      for (int nd2 = 0; nd2 < 4; ++nd2) {
        uint32_t b0, b1, b2, b3;
        ldmatrix_x4_trans(sD + gdn_chunk16<D>(ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3),
                                              (c0n >> 3) + nd2 * 2 + (lane >> 4)),
                          b0, b1, b2, b3);
        mma_16816<T>(o[2 * nd2], a, b0, b1);
        mma_16816<T>(o[2 * nd2 + 1], a, b2, b3);
      }
    }

    // (5b) S = e^(G_C) S + (e^(G_C - G) K)^T D; its 16-bit copy for the next chunk.
    if (!last) {
      const float ec = __expf(sG[C - 1]);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        S[i][0] *= ec;
        S[i][1] *= ec;
        S[i][2] *= ec;
        S[i][3] *= ec;
      }
      const int m0 = 16 * warp;
#pragma unroll
      for (int ks = 0; ks < C / 16; ++ks) {
        uint32_t a[4];
        ldmatrix_x4_trans(sK + gdn_chunk16<D>(ks * 16 + (lane & 7) + ((lane >> 4) << 3), (m0 >> 3) + ((lane >> 3) & 1)),
                          a[0], a[1], a[2], a[3]);
#pragma unroll
        for (int nd2 = 0; nd2 < 8; ++nd2) {
          uint32_t b0, b1, b2, b3;
          ldmatrix_x4_trans(sD + gdn_chunk16<D>(ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3), nd2 * 2 + (lane >> 4)),
                            b0, b1, b2, b3);
          mma_16816<T>(S[2 * nd2], a, b0, b1);
          mma_16816<T>(S[2 * nd2 + 1], a, b2, b3);
        }
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int row = m0 + (lane >> 2) + 8 * h;
#pragma unroll
        for (int nb = 0; nb < 16; ++nb) {
          const int col = nb * 8 + 2 * (lane & 3);
          *reinterpret_cast<uint32_t*>(smem + Cfg::OFF_S + gdn_elem<D>(row, col)) =
              Elem<T>::pack2(S[nb][2 * h], S[nb][2 * h + 1]);
        }
      }
    }

    // (5c) Gated RMSNorm over each token's 128 outputs (two warps per row).
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      float ss = 0.0f;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) ss += o[nb][2 * h] * o[nb][2 * h] + o[nb][2 * h + 1] * o[nb][2 * h + 1];
      ss += __shfl_xor_sync(0xffffffffu, ss, 1);
      ss += __shfl_xor_sync(0xffffffffu, ss, 2);
      if ((lane & 3) == 0) sRed[(t0 + 8 * h) * 2 + (warp >> 2)] = ss;
    }
    if (!last) {
      cp_async_wait<1>();  // z of this chunk (the next chunk's K, Q, V may still be in flight)
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int t = t0 + 8 * h;
      if (t >= valid) continue;
      const float rstd = rsqrtf((sRed[2 * t] + sRed[2 * t + 1]) * (1.0f / D) + p.eps);
      T* orow = out + static_cast<size_t>(start + c0 + t) * p.ld_out + head * D;
#pragma unroll
      for (int nb = 0; nb < 8; ++nb) {
        const int col = c0n + nb * 8 + 2 * (lane & 3);
        const float2 z = Elem<T>::unpack2(*reinterpret_cast<const uint32_t*>(smem + Cfg::OFF_Z + gdn_elem<D>(t, col)));
        *reinterpret_cast<uint32_t*>(orow + col) = Elem<T>::pack2(o[nb][2 * h] * rstd * wn[nb].x * silu_f(z.x),
                                                                  o[nb][2 * h + 1] * rstd * wn[nb].y * silu_f(z.y));
      }
    }
  }
}

}  // namespace vd
