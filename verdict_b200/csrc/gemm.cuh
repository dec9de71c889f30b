// Persistent tcgen05 GEMM for sm_100a: C[M, N] = A[M, K] * W[N, K]^T, 16-bit in,
// fp32 accumulate in tensor memory, with the layer's elementwise work fused
// into the epilogue.
//
// CTA layout (320 threads, one CTA per SM):
//   warp 0      : TMA producer (one elected lane) - A and W tiles, 128-byte swizzle
//   warp 1      : TMEM allocator + MMA issuer (one lane issues tcgen05.mma)
//   warps 2..9  : epilogue - two warps per TMEM lane quarter (lanes
//                 32*(warp%4) .. +31, the quarter a warp may access), each
//                 draining half of the tile's columns, one accumulator row per
//                 thread, results leaving through shared memory and TMA
//                 (tensor stores; reduce-add into the fp32 residual).
// Tiles are BM=128 x BN (128 or 256) x BK=64; a STAGES-deep smem ring feeds the
// MMA warp, and two TMEM accumulators (2*BN columns) let the epilogue of tile i
// overlap the MMAs of tile i+1.  Tiles are visited in groups of 16 M-tiles so the
// ~148 tiles in flight share A row-blocks and W column-blocks in L2.
//
// Epilogues:
//   kEpiStore     : out_T = act(acc + bias)            (T = fp16 or bf16)
//   kEpiResidual  : out_f32 += acc + bias                (residual stream in fp32)
//   kEpiGated     : out_T[:, n/2 + j] = act(acc[:, j]) * acc[:, BN/2 + j]
//                   (W rows are interleaved at load time in blocks of BN/2: gate, up)
//   kEpiQKRope    : per attention head of the tile: optional bias, optional
//                   q/k RMSNorm over the head, rotary embedding for q and k
//                   heads; v heads are stored as they are.
//   kEpiResidualNorm : the residual add that feeds an RMSNorm (decoders' O /
//                   out_proj and down projections): res_f32 += acc + bias,
//                   then from the new residual row h a 16-bit copy of
//                   h * g * prescale (g: the following norm's gains; the next
//                   projection's A operand) and the sum of squares of each
//                   64-column block of h (its RMS statistics).
// RMSNorm fused into the consuming projection: RMSNorm(h) W^T = rstd ((h g) W^T),
// so a consumer reads A = the producer's copy and multiplies each accumulator
// row by rstd / prescale (row factor, from the producer's block sums) before its
// own epilogue.  One 16-bit rounding of h g, as the standalone norm rounds its
// output once; the weights are used as loaded.
#pragma once

#include "common.cuh"

namespace vd {

enum EpiKind : int { kEpiStore = 0, kEpiResidual = 1, kEpiGated = 2, kEpiQKRope = 3, kEpiResidualNorm = 4 };

constexpr int kNormBlock = 64;  // columns per partial sum of squares of the fused RMSNorm
enum ActKind : int { kActNone = 0, kActGeluErf = 1, kActGeluTanh = 2, kActRelu = 3, kActSilu = 4 };

struct EpiParams {
  const float* bias;      // [N] or null
  int act;                // ActKind
  // kEpiQKRope
  const float* q_norm;    // [head_dim] gains (null: no q/k norm)
  const float* k_norm;
  int q_cols, k_cols;     // heads*head_dim, kv_heads*head_dim
  int head_dim;
  int plus_one;           // gain applied as (1 + w)
  float eps;
  const int* positions;   // [M] token position inside its sequence
  const float2* rope;     // [max_pos][rot_dim/2] (cos, sin)
  int rot_dim;            // rotary width: the first rot_dim columns of a head (multiple of 64; 0 = head_dim)
  // kEpiResidualNorm: the residual (the fp32 output map, updated in place), the
  // 16-bit copy of the new rows times the gains and `prescale` (the second
  // output map) and the block sums of squares ([M, N / kNormBlock]).
  float prescale;
  float* ss_out;
  const float* norm_gain;  // [N] gains of the following RMSNorm, applied as norm_gain + norm_add
  float norm_add;
  // Fused RMSNorm of the A rows (store, gated and QK-rope epilogues): row
  // factor rsqrt(sum(ss_in[m, :]) * ss_inv_n + ss_eps) * ss_post, applied to
  // the accumulators first; ss_in == null: none.
  const float* ss_in;
  int ss_slots;
  float ss_inv_n, ss_eps, ss_post;
};

// The fused RMSNorm's factor for accumulator row `row`: the block sums are added
// in a fixed order, so the result does not depend on how rows were tiled.
__device__ __forceinline__ float row_factor(const EpiParams& p, int row, bool row_ok) {
  if (p.ss_in == nullptr || !row_ok) return 1.0f;
  const float4* b = reinterpret_cast<const float4*>(p.ss_in + static_cast<size_t>(row) * p.ss_slots);
  float ss = 0.0f;
#pragma unroll 4
  for (int i = 0; i < p.ss_slots / 4; ++i) {
    const float4 t = __ldg(b + i);
    ss += t.x;
    ss += t.y;
    ss += t.z;
    ss += t.w;
  }
  return rsqrtf(ss * p.ss_inv_n + p.ss_eps) * p.ss_post;
}

__device__ __forceinline__ void scale32(float (&v)[32], float f) {
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] *= f;
}

// group_m: M tiles per raster group (tiles walk M fastest inside a group, so a
// group's A rows stay in L2 while W streams past them once per group).
// wait_ns: limit of every barrier wait (0: VD_WAIT_TIMEOUT_NS).  stall_after
// (one-CTA kernel, failure-path tests only; 0 = off): the producer stops after
// issuing this many k-blocks, so the MMA warp's wait for the next stage runs
// out and the launch ends through its abort path with kErrTimeoutFull.
// splits > 1 (one-CTA kernel, small batches): K is split over `splits` work
// units per output tile; each unit writes its fp32 partial tile to
// part[split] (tiles * 128 * BN floats per split), and the unit that finishes
// last (per-tile arrival counters, left at zero) adds the partials in split
// order into its accumulator and runs the epilogue, so the result does not
// depend on which unit finished when.
struct GemmShape {
  int M, N, K;
  int group_m;
  uint64_t wait_ns;
  int stall_after;
  int splits;
  float* part;
  int* counters;
  int l2_hints;  // pair kernel: L2 evict-last for A, evict-first for W loads
};

// GELU in its exact form, x * Phi(x), Phi the standard normal CDF, with erf
// from Abramowitz & Stegun, Handbook of Mathematical Functions, formula
// 7.1.26 (|error| <= 1.5e-7 for z >= 0):
//   erf(z) = 1 - q(z),  q(z) = (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) e^(-z^2),
//   t = 1 / (1 + p z).
// q is the tail 1 - erf(|z|) itself, so Phi(x) = q / 2 for x < 0 and
// 1 - q / 2 otherwise come out without cancellation.  One reciprocal and one
// exp2 on the special-function unit plus a handful of FMAs per element: the
// encoders' up projections (K = 768) are bound by this epilogue.
__device__ __forceinline__ float gelu_erf(float x) {
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = __fdividef(1.0f, fmaf(0.3275911f, z, 1.0f));
  float poly = fmaf(t, 1.061405429f, -1.453152027f);
  poly = fmaf(t, poly, 1.421413741f);
  poly = fmaf(t, poly, -0.284496736f);
  poly = fmaf(t, poly, 0.254829592f);
  float e;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(e) : "f"(-z * z * 1.4426950408889634f));
  const float q = poly * t * e;
  return x * (x < 0.0f ? 0.5f * q : fmaf(-0.5f, q, 1.0f));
}

__device__ __forceinline__ float apply_act(float x, int act) {
  switch (act) {
    case kActGeluErf: return gelu_erf(x);
    case kActGeluTanh: {
      const float c = 0.7978845608028654f;  // sqrt(2/pi)
      return 0.5f * x * (1.0f + tanhf(c * (x + 0.044715f * x * x * x)));
    }
    case kActRelu: return fmaxf(x, 0.0f);
    case kActSilu: return x / (1.0f + expf(-x));
    default: return x;
  }
}

__device__ __forceinline__ void add_bias32(float (&v)[32], const float* bias, int col) {
  if (bias == nullptr) return;
  const float4* b = reinterpret_cast<const float4*>(bias + col);
#pragma unroll
  for (int q = 0; q < 8; ++q) {
    float4 t = __ldg(b + q);
    v[q * 4 + 0] += t.x;
    v[q * 4 + 1] += t.y;
    v[q * 4 + 2] += t.z;
    v[q * 4 + 3] += t.w;
  }
}

// ---------------------------------------------------------------------------
// Epilogue output through shared memory and TMA.  Each epilogue warp owns a
// 4 KB staging buffer; a chunk is this warp's 32 rows x 32 columns.  16-bit
// chunks (2 KB, 64-byte swizzle) are written with a TMA tensor store, two
// buffers in flight; fp32 residual chunks (4 KB, 128-byte swizzle) are added
// into the residual stream with a TMA reduce-add performed at L2, so the SM
// never reads the residual.  Rows past M land in rows of the output that no
// one reads (tensor maps built for the workspace extent) or are clipped by the
// map (per-call maps).
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem_gemm() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

struct EpiOut {
  uint8_t* stage;          // this warp's 4 KB staging buffer (1024-byte aligned)
  const CUtensorMap* map;  // output tensor map (16-bit box 32x32 SW64, or fp32 box 32x32 SW128)
  int y;                   // first output row of this warp's 32 rows
  int lane;
  int n16;                 // 16-bit chunks issued so far (selects the staging half)
  // kEpiResidualNorm: the 16-bit copy's map, this warp's TMA-load barrier and
  // its phase, the wait limit and the error word
  const CUtensorMap* map2;
  uint64_t* ld_bar;
  uint32_t ld_phase;
  uint64_t wait_ns;
  int* err;
};

// One 32x32 chunk of 16-bit outputs at column x.
template <class T>
__device__ __forceinline__ void out_chunk16(EpiOut& o, const float (&v)[32], int x) {
  const int b = o.n16++ & 1;
  if (o.lane == 0) bulk_wait_read<1>();  // the store that last used this half has read it
  __syncwarp();
  uint8_t* buf = o.stage + b * 2048;
  const int r = o.lane;
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = Elem<T>::pack2(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = Elem<T>::pack2(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = Elem<T>::pack2(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = Elem<T>::pack2(v[q * 8 + 6], v[q * 8 + 7]);
    *reinterpret_cast<uint4*>(buf + r * 64 + ((q ^ ((r >> 1) & 3)) << 4)) = w;
  }
  fence_proxy_async_smem_gemm();
  __syncwarp();
  if (o.lane == 0) {
    tma_store_2d(o.map, buf, x, o.y);
    bulk_commit();
  }
}

// One 32x32 chunk of fp32 values added into the output at column x.
__device__ __forceinline__ void out_chunk_add32(EpiOut& o, const float (&v)[32], int x) {
  if (o.lane == 0) bulk_wait_read<0>();
  __syncwarp();
  const int r = o.lane;
#pragma unroll
  for (int q = 0; q < 8; ++q)
    *reinterpret_cast<float4*>(o.stage + r * 128 + ((q ^ (r & 7)) << 4)) =
        make_float4(v[q * 4 + 0], v[q * 4 + 1], v[q * 4 + 2], v[q * 4 + 3]);
  fence_proxy_async_smem_gemm();
  __syncwarp();
  if (o.lane == 0) {
    tma_reduce_add_2d(o.map, o.stage, x, o.y);
    bulk_commit();
  }
}

// One head of kEpiQKRope: columns [col0, col0 + HD) of row `row`, TMEM at tbase.
// The head is split into work units: rotary pairs first (pair c rotates chunk
// c with chunk c + R/32, chunk c = columns [32c, 32c + 32), R = rot_dim / 2),
// then the chunks past rot_dim, which are only normalised.  This warp handles
// units [u_begin, u_end); with a gain it first computes the RMS over the whole
// head itself, so the two warps sharing a head need no exchange.
template <int HD, class T>
__device__ __forceinline__ void epi_head_rope(EpiOut& o, uint32_t tbase, int row, bool row_ok, int col0,
                                              const EpiParams& p, const float* gain, int u_begin, int u_end,
                                              float f) {
  const int rot = p.rot_dim ? p.rot_dim : HD;
  const int R = rot / 2;            // rotary half-width (columns)
  const int pairs = R / 32;         // rotary work units
  float rstd = 1.0f;
  if (gain != nullptr) {
    float ss = 0.0f;
#pragma unroll 1
    for (int c = 0; c < HD / 32; ++c) {
      float v[32];
      tmem_load_f32x32(tbase + c * 32, v);
      scale32(v, f);
      add_bias32(v, p.bias, col0 + c * 32);
#pragma unroll
      for (int j = 0; j < 32; ++j) ss += v[j] * v[j];
    }
    rstd = rsqrtf(ss / static_cast<float>(HD) + p.eps);
  }
  const int pos = row_ok ? __ldg(p.positions + row) : 0;
  const float4* rope = reinterpret_cast<const float4*>(p.rope + static_cast<size_t>(pos) * R);
  const float add = p.plus_one ? 1.0f : 0.0f;
  auto scale = [&](float (&x)[32], int colh) {
    if (gain == nullptr) return;
    const float4* g = reinterpret_cast<const float4*>(gain + colh);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 a = __ldg(g + q);
      x[4 * q + 0] *= rstd * (a.x + add);
      x[4 * q + 1] *= rstd * (a.y + add);
      x[4 * q + 2] *= rstd * (a.z + add);
      x[4 * q + 3] *= rstd * (a.w + add);
    }
  };
#pragma unroll 1
  for (int u = u_begin; u < u_end; ++u) {
    if (u < pairs) {
      const int c = u;
      float x1[32], x2[32];
      tmem_load_f32x32(tbase + c * 32, x1);
      tmem_load_f32x32(tbase + R + c * 32, x2);
      scale32(x1, f);
      scale32(x2, f);
      add_bias32(x1, p.bias, col0 + c * 32);
      add_bias32(x2, p.bias, col0 + R + c * 32);
      scale(x1, c * 32);
      scale(x2, R + c * 32);
#pragma unroll
      for (int q = 0; q < 16; ++q) {  // (cos, sin) pairs of columns 2q and 2q+1
        const float4 cs = __ldg(rope + c * 16 + q);
        const float a0 = x1[2 * q], b0 = x2[2 * q], a1 = x1[2 * q + 1], b1 = x2[2 * q + 1];
        x1[2 * q] = a0 * cs.x - b0 * cs.y;
        x2[2 * q] = b0 * cs.x + a0 * cs.y;
        x1[2 * q + 1] = a1 * cs.z - b1 * cs.w;
        x2[2 * q + 1] = b1 * cs.z + a1 * cs.w;
      }
      out_chunk16<T>(o, x1, col0 + c * 32);
      out_chunk16<T>(o, x2, col0 + R + c * 32);
    } else {
      const int c = rot / 32 + (u - pairs);  // a chunk past the rotary columns
      float x[32];
      tmem_load_f32x32(tbase + c * 32, x);
      scale32(x, f);
      add_bias32(x, p.bias, col0 + c * 32);
      scale(x, c * 32);
      out_chunk16<T>(o, x, col0 + c * 32);
    }
  }
}

// Work units [begin, end) of `half` (0 or 1) when two warps share one head:
// units cost 2 chunks (rotary pairs) or 1 (plain chunks); each warp gets half
// of the head's HD/32 chunks.
template <int HD>
__device__ __forceinline__ void head_units(const EpiParams& p, int half, int& begin, int& end) {
  const int rot = p.rot_dim ? p.rot_dim : HD;
  const int pairs = rot / 64, units = pairs + (HD - rot) / 32;
  int split = 0, cost = 0;
  while (split < units && cost < HD / 64) {
    cost += split < pairs ? 2 : 1;
    ++split;
  }
  begin = half ? split : 0;
  end = half ? units : split;
}

// Plain store of 32-column chunks [c_begin, c_end) starting at column col0.
template <class T>
__device__ __forceinline__ void epi_store_chunks(EpiOut& o, uint32_t tbase, int col0, const EpiParams& p,
                                                 int c_begin, int c_end, float f = 1.0f) {
#pragma unroll 1
  for (int c = c_begin; c < c_end; ++c) {
    float v[32];
    tmem_load_f32x32(tbase + c * 32, v);
    scale32(v, f);
    add_bias32(v, p.bias, col0 + c * 32);
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = apply_act(v[j], p.act);
    out_chunk16<T>(o, v, col0 + c * 32);
  }
}

// Epilogue of one accumulator row for one of the two warps that share a TMEM
// lane quarter: `half` (0 or 1) selects which half of the tile's columns (or
// heads) this warp drains.
template <int BN, int EPI, class T>
__device__ __forceinline__ void gemm_epilogue(EpiOut& o, uint32_t taddr, int row, bool row_ok, int n0, int half,
                                              const EpiParams& p) {
  constexpr int CH = BN / 32;  // 32-column chunks per tile
  if constexpr (EPI == kEpiStore) {
    epi_store_chunks<T>(o, taddr, n0, p, half * CH / 2, (half + 1) * CH / 2, row_factor(p, row, row_ok));
  } else if constexpr (EPI == kEpiResidual) {
#pragma unroll 1
    for (int c = half * CH / 2; c < (half + 1) * CH / 2; ++c) {
      float v[32];
      tmem_load_f32x32(taddr + c * 32, v);
      add_bias32(v, p.bias, n0 + c * 32);
      out_chunk_add32(o, v, n0 + c * 32);
    }
  } else if constexpr (EPI == kEpiResidualNorm) {
    // This thread owns row `row`, columns [n0 + 32 c, +32) for the chunks of
    // its half (an even number of chunks: whole 64-column blocks).  Per chunk
    // the warp's 32 x 32 block of the residual comes in by TMA into the
    // staging buffer (the 128-byte-swizzled layout the fp32 TMA store uses),
    // each thread adds its row, and the new block leaves by TMA store; the
    // 16-bit copy follows through the same buffer.
    static_assert((CH / 2) % 2 == 0, "a warp's columns must cover whole 64-column blocks");
    float ss = 0.0f;
    const int r = o.lane;
#pragma unroll 1
    for (int c = half * CH / 2; c < (half + 1) * CH / 2; ++c) {
      const int x = n0 + c * 32;
      // The stage is free once the previous chunk's stores have read it.
      if (o.lane == 0) {
        bulk_wait_read<0>();
        mbar_arrive_expect_tx(o.ld_bar, 32 * 32 * 4);
        tma_load_2d(o.stage, o.map, o.ld_bar, x, o.y);
      }
      float v[32];
      tmem_load_f32x32(taddr + c * 32, v);
      add_bias32(v, p.bias, x);
      // Our own load: wait for it even on an abort (it writes the stage).
      if (!mbar_wait_own(o.ld_bar, o.ld_phase, o.wait_ns)) record_error(o.err, kErrTimeoutFull);
      o.ld_phase ^= 1;
      // Rows past M (the padding of the last tile, which the box store covers)
      // keep their residual and get a zero copy: their accumulators come from
      // stale A rows, and without a norm they would grow layer after layer
      // into the keys that attention masks (0 * inf = NaN).
      const float keep = row_ok ? 1.0f : 0.0f;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        float4* a = reinterpret_cast<float4*>(o.stage + r * 128 + ((q ^ (r & 7)) << 4));
        const float4 h = *a;
        v[4 * q + 0] = row_ok ? v[4 * q + 0] + h.x : h.x;
        v[4 * q + 1] = row_ok ? v[4 * q + 1] + h.y : h.y;
        v[4 * q + 2] = row_ok ? v[4 * q + 2] + h.z : h.z;
        v[4 * q + 3] = row_ok ? v[4 * q + 3] + h.w : h.w;
        *a = make_float4(v[4 * q + 0], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
      }
      fence_proxy_async_smem_gemm();
      __syncwarp();
      if (o.lane == 0) {
        tma_store_2d(o.map, o.stage, x, o.y);
        bulk_commit();
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) ss = fmaf(v[j], v[j], ss);
      const float4* g4 = reinterpret_cast<const float4*>(p.norm_gain + x);
      const float pre = p.prescale * keep;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 g = __ldg(g4 + q);
        v[4 * q + 0] *= (g.x + p.norm_add) * pre;
        v[4 * q + 1] *= (g.y + p.norm_add) * pre;
        v[4 * q + 2] *= (g.z + p.norm_add) * pre;
        v[4 * q + 3] *= (g.w + p.norm_add) * pre;
      }
      // 16-bit copy: the first 2 KB of the stage once the fp32 store has read it.
      if (o.lane == 0) bulk_wait_read<0>();
      __syncwarp();
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        uint4 w;
        w.x = Elem<T>::pack2(v[q * 8 + 0], v[q * 8 + 1]);
        w.y = Elem<T>::pack2(v[q * 8 + 2], v[q * 8 + 3]);
        w.z = Elem<T>::pack2(v[q * 8 + 4], v[q * 8 + 5]);
        w.w = Elem<T>::pack2(v[q * 8 + 6], v[q * 8 + 7]);
        *reinterpret_cast<uint4*>(o.stage + r * 64 + ((q ^ ((r >> 1) & 3)) << 4)) = w;
      }
      fence_proxy_async_smem_gemm();
      __syncwarp();
      if (o.lane == 0) {
        tma_store_2d(o.map2, o.stage, x, o.y);
        bulk_commit();
      }
      if ((c & 1) && row_ok) {
        p.ss_out[static_cast<size_t>(row) * p.ss_slots + x / kNormBlock] = ss;
        ss = 0.0f;
      }
    }
  } else if constexpr (EPI == kEpiGated) {
    constexpr int HALF = BN / 2;         // output columns of the tile
    constexpr int OC = HALF / 32;        // output chunks
    const float f = row_factor(p, row, row_ok);
#pragma unroll 1
    for (int c = half * OC / 2; c < (half + 1) * OC / 2; ++c) {
      float g[32], u[32];
      tmem_load_f32x32(taddr + c * 32, g);
      tmem_load_f32x32(taddr + HALF + c * 32, u);
#pragma unroll
      for (int j = 0; j < 32; ++j) g[j] = apply_act(g[j] * f, p.act) * (u[j] * f);
      out_chunk16<T>(o, g, n0 / 2 + c * 32);
    }
  } else if constexpr (EPI == kEpiQKRope) {
    // Heads never straddle tiles.  head_dim 128: with two heads per tile each
    // warp takes one head; with one head (BN = 128) the warps split its two
    // rotary chunk pairs.  head_dim 256 (one head per 256-wide tile): the warps
    // split its four chunk pairs.
    // Columns past the q and k blocks (v, and a hybrid's output gate) are stored as they are.
    const float f = row_factor(p, row, row_ok);
    if (p.head_dim == 64) {
      // head_dim 64 (ModernBERT): BN / 64 heads per tile, each warp half of them;
      // one rotary pair per head (columns [0, 32) with [32, 64)).
      constexpr int HEADS = BN / 64;
#pragma unroll 1
      for (int hh = 0; hh < HEADS / 2; ++hh) {
        const int h = half * (HEADS / 2) + hh;
        const int col0 = n0 + h * 64;
        const uint32_t tb = taddr + h * 64;
        if (col0 < p.q_cols + p.k_cols)
          epi_head_rope<64, T>(o, tb, row, row_ok, col0, p, col0 < p.q_cols ? p.q_norm : p.k_norm, 0, 1, f);
        else
          epi_store_chunks<T>(o, tb, col0, p, 0, 2, f);
      }
    } else if (p.head_dim == 128) {
      constexpr int HEADS = BN / 128;
      const int h = HEADS == 2 ? half : 0;
      const int col0 = n0 + h * 128;
      const uint32_t tb = taddr + h * 128;
      int ub = 0, ue = 0;
      if (HEADS == 2) {
        const int rot = p.rot_dim ? p.rot_dim : 128;
        ue = rot / 64 + (128 - rot) / 32;  // the whole head
      } else {
        head_units<128>(p, half, ub, ue);
      }
      if (col0 < p.q_cols + p.k_cols)
        epi_head_rope<128, T>(o, tb, row, row_ok, col0, p, col0 < p.q_cols ? p.q_norm : p.k_norm, ub, ue, f);
      else
        epi_store_chunks<T>(o, tb, col0, p, HEADS == 2 ? 0 : 2 * half, HEADS == 2 ? 4 : 2 * half + 2, f);
    } else if constexpr (BN == 256) {
      if (n0 < p.q_cols + p.k_cols) {
        int ub = 0, ue = 0;
        head_units<256>(p, half, ub, ue);
        epi_head_rope<256, T>(o, taddr, row, row_ok, n0, p, n0 < p.q_cols ? p.q_norm : p.k_norm, ub, ue, f);
      } else {
        epi_store_chunks<T>(o, taddr, n0, p, 4 * half, 4 * half + 4, f);
      }
    }
  }
}

// Split-K fixup of one work unit, run by the 8 epilogue warps (threads 64..319,
// named barrier 1).  Each thread owns accumulator row `row_in_tile` of the
// tile and the columns of its `half`.  The unit's partial tile goes to
// part[split] in a layout private to this fixup, chosen so that every warp
// access is one contiguous 128-byte line: epilogue warp slot w (TMEM lane
// quarter w & 3, column half w >> 2) stores its 32 x 32 chunk c as
// [column][row].  The tile's arrival counter says whether all splits have
// landed; the last unit adds part[0..splits) in order into its TMEM
// accumulator and returns true (the caller then runs the epilogue on it), the
// others return false.
__device__ __forceinline__ void epi_bar_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Named barrier 1 over the epilogue warps that also ANDs a warp-uniform flag.
__device__ __forceinline__ bool epi_bar_and(bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %1, 0;\n\t"
      "bar.red.and.pred p, 1, 256, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

template <int BN>
__device__ __forceinline__ bool split_fixup(uint32_t taddr, const GemmShape& sh, int tile, int ks, int slot,
                                            int half, int lane, volatile int* last_flag) {
  constexpr int CH = BN / 32;
  constexpr int TILE_FLOATS = 128 * BN;
  const int tiles = ((sh.M + 127) / 128) * (sh.N / BN);
  const size_t plane = static_cast<size_t>(tiles) * TILE_FLOATS;
  // This warp's chunks: slot-major, then chunk, then [column][row] inside.
  const size_t base = static_cast<size_t>(tile) * TILE_FLOATS + static_cast<size_t>(slot) * (CH / 2) * 1024;
  float* mine = sh.part + ks * plane + base;
#pragma unroll 1
  for (int c = 0; c < CH / 2; ++c) {
    float v[32];
    tmem_load_f32x32(taddr + (half * CH / 2 + c) * 32, v);
#pragma unroll
    for (int j = 0; j < 32; ++j) mine[c * 1024 + j * 32 + lane] = v[j];
  }
  __threadfence();  // this thread's partial is visible before the arrival below
  epi_bar_sync();
  if (threadIdx.x == 64) {
    const int before = atomicAdd(sh.counters + tile, 1);
    const bool last = before == sh.splits - 1;
    if (last) sh.counters[tile] = 0;  // every unit of the tile has arrived: ready for the next launch
    *last_flag = last ? 1 : 0;
  }
  epi_bar_sync();
  if (!*last_flag) return false;
  __threadfence();
  const float* all = sh.part + base;
#pragma unroll 1
  for (int c = 0; c < CH / 2; ++c) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __ldcg(all + c * 1024 + j * 32 + lane);
#pragma unroll 1
    for (int k = 1; k < sh.splits; ++k) {
      const float* pk = all + k * plane + c * 1024;
#pragma unroll
      for (int j = 0; j < 32; ++j) v[j] += __ldcg(pk + j * 32 + lane);
    }
    tmem_st32f(taddr + (half * CH / 2 + c) * 32, v);
  }
  tmem_wait_st();
  // Both warps of a lane quarter read the whole tile row in some epilogues.
  tc_fence_before();
  epi_bar_sync();
  tc_fence_after();
  return true;
}

template <int BN>
struct GemmConfig {
  static constexpr int BM = 128;
  static constexpr int BK = 64;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int TMEM_COLS = 2 * BN;  // two accumulators
  static constexpr int BAR_BYTES = 1024;    // barriers, padded so the staging buffers stay 1 KB aligned
  static constexpr int EPI_WARPS = 8;       // two warps per TMEM lane quarter
  static constexpr int EPI_STAGE_BYTES = 4096;  // per epilogue warp: one fp32 or two 16-bit 32x32 chunks
  static constexpr int SMEM_BYTES =
      1024 /*alignment slack*/ + STAGES * STAGE_BYTES + BAR_BYTES + EPI_WARPS * EPI_STAGE_BYTES;
  static constexpr int THREADS = 64 + 32 * EPI_WARPS;
  static constexpr int GROUP_M = 16;
};

// Tile order: groups of `group_m` M-tiles; inside a group N is the slow index.
// Odd groups walk N backwards, so the W column-blocks a group ends on are the
// ones still in L2 when the next group starts.
__device__ __forceinline__ void tile_coords(int tile, int num_m, int num_n, int group_m, int& m, int& n) {
  const int group_size = group_m * num_n;
  const int g = tile / group_size;
  const int first_m = g * group_m;
  const int gm = min(num_m - first_m, group_m);
  const int local = tile - g * group_size;
  m = first_m + local % gm;
  n = local / gm;
  if (g & 1) n = num_n - 1 - n;
}

template <int BN, int EPI, class T>
__global__ void __launch_bounds__(GemmConfig<BN>::THREADS, 1)
    gemm_tcgen05_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        const __grid_constant__ CUtensorMap tmC, const __grid_constant__ CUtensorMap tmD,
                        GemmShape shape, EpiParams ep, int* err) {
  using Cfg = GemmConfig<BN>;
  constexpr int BM = Cfg::BM, BK = Cfg::BK, STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = umma_idesc_f16kind(BM, BN, Elem<T>::kUmmaFormat);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sA = smem;
  uint8_t* sB = smem + STAGES * Cfg::A_BYTES;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  uint64_t* mma_drained = acc_empty + 3;  // the MMA warp's own ops, on its abort path
  volatile int* split_last = reinterpret_cast<volatile int*>(acc_empty + 4);  // split-K: this unit finishes the tile
  uint64_t* epi_ld = acc_empty + 5;  // [EPI_WARPS] TMA loads of the residual (kEpiResidualNorm)
  uint8_t* epi_stage = smem + STAGES * Cfg::STAGE_BYTES + Cfg::BAR_BYTES;
  const uint64_t wait_ns = shape.wait_ns;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int j = 0; j < 2; ++j) {
      mbar_init(&acc_full[j], 1);
      mbar_init(&acc_empty[j], Cfg::EPI_WARPS);  // one arrival per epilogue warp
    }
    mbar_init(mma_drained, 1);
    for (int w = 0; w < Cfg::EPI_WARPS; ++w) mbar_init(&epi_ld[w], 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Launched with programmatic stream serialization, the set-up above ran
  // under the previous kernel's tail.  Every role waits for that kernel's
  // results before it touches global memory; the producer first loads the
  // weight tiles of its first k-blocks, which do not depend on it.
  pdl_trigger_next();

  const int num_m = (shape.M + BM - 1) / BM;
  const int num_n = shape.N / BN;
  const int tiles = num_m * num_n;
  const int kblocks = shape.K / BK;
  const int splits = shape.splits > 1 ? shape.splits : 1;
  const int units = tiles * splits;  // unit u: tile u / splits, K range u % splits
  auto k_range = [&](int u, int& kb0, int& kb1) {
    const int ks = u % splits;
    kb0 = static_cast<int>(static_cast<int64_t>(ks) * kblocks / splits);
    kb1 = static_cast<int>(static_cast<int64_t>(ks + 1) * kblocks / splits);
  };

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmA);
      tma_prefetch_desc(&tmB);
      tma_prefetch_desc(&tmC);
      if constexpr (EPI == kEpiResidualNorm) tma_prefetch_desc(&tmD);
      // The first unit's first `pre` stages (all free: nothing has used them
      // yet) get their W tiles now and their A rows after the wait; not on
      // the failure-path test's stalled launches.
      int pre = 0;
      if (static_cast<int>(blockIdx.x) < units && shape.stall_after == 0) {
        int m, n, kb0, kb1;
        tile_coords(blockIdx.x / splits, num_m, num_n, shape.group_m, m, n);
        k_range(blockIdx.x, kb0, kb1);
        pre = kb1 - kb0 < STAGES ? kb1 - kb0 : STAGES;
        for (int i = 0; i < pre; ++i) {
          mbar_arrive_expect_tx(&full[i], Cfg::STAGE_BYTES);
          tma_load_2d(sB + i * Cfg::B_BYTES, &tmB, &full[i], (kb0 + i) * BK, n * BN);
        }
      }
      pdl_wait_prior();
      int stage = 0;
      uint32_t phase = 0;
      int issued = 0;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int m, n, kb0, kb1;
        tile_coords(u / splits, num_m, num_n, shape.group_m, m, n);
        k_range(u, kb0, kb1);
        for (int kb = kb0; kb < kb1; ++kb) {
          if (shape.stall_after > 0 && issued == shape.stall_after) goto producer_drain;
          ++issued;
          if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrTimeoutEmpty, wait_ns)) goto producer_done;
          const bool w_loaded = u == static_cast<int>(blockIdx.x) && kb - kb0 < pre;
          if (!w_loaded) mbar_arrive_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          tma_load_2d(sA + stage * Cfg::A_BYTES, &tmA, &full[stage], kb * BK, m * BM);
          if (!w_loaded) tma_load_2d(sB + stage * Cfg::B_BYTES, &tmB, &full[stage], kb * BK, n * BN);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    producer_drain:
      // Drain: wait until the MMA warp released every stage we filled, so no TMA
      // write can land after the CTA exits.
      for (int i = 0; i < STAGES; ++i) {
        if (!mbar_wait(&empty[stage], phase ^ 1, abort_flag, err, kErrTimeoutEmpty, wait_ns)) break;
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1;
        }
      }
    producer_done:;
    }
  } else if (warp == 1) {
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units; u += gridDim.x) {
        int kb0, kb1;
        k_range(u, kb0, kb1);
        if (!mbar_wait(&acc_empty[acc], acc_phase ^ 1, abort_flag, err, kErrTimeoutAccEmpty, wait_ns)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + acc * BN;
        for (int kb = kb0; kb < kb1; ++kb) {
          if (!mbar_wait(&full[stage], phase, abort_flag, err, kErrTimeoutFull, wait_ns)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t a_addr = smem_u32(sA + stage * Cfg::A_BYTES);
          const uint32_t b_addr = smem_u32(sB + stage * Cfg::B_BYTES);
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            umma_f16kind(d_tmem, sw128_kmajor_desc(a_addr + k * 32), sw128_kmajor_desc(b_addr + k * 32), IDESC,
                      (kb != kb0 || k != 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&acc_full[acc]);
        if (++acc == 2) {
          acc = 0;
          acc_phase ^= 1;
        }
      }
      if (!ok) {
        // Aborted: let the MMAs this thread already issued finish (bounded)
        // before the CTA frees the tensor memory they write.
        umma_commit(mma_drained);
        mbar_wait_own(mma_drained, 0, wait_ns);
      }
    }
  } else {
    pdl_wait_prior();
    // Epilogue warps 2..9: warp w drains TMEM lanes 32*(w%4).. (the quarter it
    // may access) and column half (w-2)/4 of the tile.
    const int lane_group = warp & 3;
    const int half = (warp - 2) >> 2;
    const int row_in_tile = lane_group * 32 + lane;
    EpiOut o{epi_stage + (warp - 2) * Cfg::EPI_STAGE_BYTES, &tmC, 0, lane, 0, &tmD, &epi_ld[warp - 2], 0u,
             wait_ns, err};
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x) {
      const int tile = u / splits;
      int m, n;
      tile_coords(tile, num_m, num_n, shape.group_m, m, n);
      bool got = mbar_wait(&acc_full[acc], acc_phase, abort_flag, err, kErrTimeoutAccFull, wait_ns);
      // The split fixup synchronises the 8 epilogue warps, so they must agree
      // on going on (one giving up on an abort while another saw the
      // accumulator land would leave the other at a barrier).
      if (splits > 1) got = epi_bar_and(__all_sync(0xffffffffu, got));
      if (!got) break;
      tc_fence_after();
      const uint32_t taddr = tmem_base + acc * BN + (static_cast<uint32_t>(lane_group * 32) << 16);
      const int row = m * BM + row_in_tile;
      o.y = m * BM + lane_group * 32;
      if (splits == 1 || split_fixup<BN>(taddr, shape, tile, u % splits, warp - 2, half, lane, split_last))
        gemm_epilogue<BN, EPI, T>(o, taddr, row, row < shape.M, n * BN, half, ep);
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[acc]);
      if (++acc == 2) {
        acc = 0;
        acc_phase ^= 1;
      }
    }
    // Every TMA store / reduce of this warp has finished before the CTA exits.
    if (lane == 0) bulk_wait_all();
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

}  // namespace vd
