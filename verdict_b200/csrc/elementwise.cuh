// HBM-bound kernels around the GEMMs: batch packing, embedding gather, row
// norms, and the option / marker scoring at the end of the forward.
#pragma once

#include "common.cuh"

namespace vd {

constexpr float kSentinel = -1e4f;  // masked option / marker slots (src/torch_engine.rs:97-114)

template <int NT>
__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) red[warp] = v;
  __syncthreads();
  float t = (threadIdx.x < NT / 32) ? red[threadIdx.x] : 0.0f;
  if (warp == 0) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (lane == 0) red[NT / 32] = t;
  }
  __syncthreads();
  const float r = red[NT / 32];
  __syncthreads();
  return r;
}

// One packed sequence: `len` tokens taken from columns [col0, col0 + len) of
// batch row `src_row`, stored from packed index `start` on.  A whole row has
// col0 = 0; a shared prefix is stored once (from its first member's row) and
// each member's suffix starts at col0 = prefix length.
struct PackSeg {
  int start, len, col0, src_row;
};

// Where a decision's slot lives: packed token base + slot, slot in [lo, hi).
struct RowMap {
  int base, lo, hi, pad;
};

// Packed int32 tokens, positions and source row of every sequence (grid.y =
// sequences).  Token ids outside [0, vocab) are reported and replaced by 0 so
// no gather reads outside the table.
__global__ void pack_segments_kernel(const int64_t* __restrict__ ids, int64_t l, const PackSeg* __restrict__ segs,
                                     int n_seg, int vocab, int pos_offset, int* __restrict__ tokens,
                                     int* __restrict__ positions, int* __restrict__ seq_id, int* err) {
  const int sgi = blockIdx.y;
  if (sgi >= n_seg) return;
  const PackSeg sg = segs[sgi];
  const int64_t* row = ids + static_cast<int64_t>(sg.src_row) * l + sg.col0;
  for (int j = blockIdx.x * blockDim.x + threadIdx.x; j < sg.len; j += gridDim.x * blockDim.x) {
    int64_t id = row[j];
    if (id < 0 || id >= vocab) {
      record_error(err, kErrTokenRange);
      id = 0;
    }
    tokens[sg.start + j] = static_cast<int>(id);
    positions[sg.start + j] = sg.col0 + j + pos_offset;
    seq_id[sg.start + j] = sg.src_row;
  }
}

// h[t, :] = emb[tokens[t], :] * scale (bf16 table -> fp32 residual stream).
__global__ void embed_kernel(const int* __restrict__ tokens, int T, const __nv_bfloat16* __restrict__ emb, int d,
                             float scale, float* __restrict__ h) {
  const int t = blockIdx.x;
  if (t >= T) return;
  const uint4* src = reinterpret_cast<const uint4*>(emb + static_cast<size_t>(tokens[t]) * d);
  float4* dst = reinterpret_cast<float4*>(h + static_cast<size_t>(t) * d);
  for (int i = threadIdx.x; i < d / 8; i += blockDim.x) {
    const uint4 v = __ldg(src + i);
    const float2 a = unpack_bf16x2(v.x), b = unpack_bf16x2(v.y), c = unpack_bf16x2(v.z), e = unpack_bf16x2(v.w);
    dst[2 * i] = make_float4(a.x * scale, a.y * scale, b.x * scale, b.y * scale);
    dst[2 * i + 1] = make_float4(c.x * scale, c.y * scale, e.x * scale, e.y * scale);
  }
}

// Decoder embedding that starts the fused-RMSNorm chain (one 128-thread block
// per token): h[t, :] = emb[tokens[t], :] * scale (fp32 residual stream), the
// 16-bit copy xcopy[t, :] = T(h[t, :] * (g + add) * prescale) that the first
// QKV GEMM reads as its A operand (g: the first layer's input-norm gains), and
// ss[t, b] = the sum of squares of h[t, 64b .. 64b + 63] (the block sums the
// GEMM's row factor adds up).  d % 64 == 0.
template <class T>
__global__ void embed_norm_kernel(const int* __restrict__ tokens, int n_tok, const __nv_bfloat16* __restrict__ emb,
                                  int d, float scale, const float* __restrict__ g, float add, float prescale,
                                  float* __restrict__ h, T* __restrict__ xcopy, float* __restrict__ ss) {
  const int t = blockIdx.x;
  if (t >= n_tok) return;
  const uint4* src = reinterpret_cast<const uint4*>(emb + static_cast<size_t>(tokens[t]) * d);
  float4* dst = reinterpret_cast<float4*>(h + static_cast<size_t>(t) * d);
  uint4* cp = reinterpret_cast<uint4*>(xcopy + static_cast<size_t>(t) * d);
  const int groups = d / 8;  // 8 elements per thread and pass; 8 consecutive threads make one 64-column block
  for (int base = 0; base < groups; base += blockDim.x) {  // every thread runs every pass (shuffles below)
    const int i = base + threadIdx.x;
    const bool ok = i < groups;
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (ok) {
      const uint4 w = __ldg(src + i);
      const float2 a = unpack_bf16x2(w.x), b = unpack_bf16x2(w.y), c = unpack_bf16x2(w.z), e = unpack_bf16x2(w.w);
      v[0] = a.x * scale, v[1] = a.y * scale, v[2] = b.x * scale, v[3] = b.y * scale;
      v[4] = c.x * scale, v[5] = c.y * scale, v[6] = e.x * scale, v[7] = e.y * scale;
      dst[2 * i] = make_float4(v[0], v[1], v[2], v[3]);
      dst[2 * i + 1] = make_float4(v[4], v[5], v[6], v[7]);
      const float4 g0 = __ldg(reinterpret_cast<const float4*>(g) + 2 * i);
      const float4 g1 = __ldg(reinterpret_cast<const float4*>(g) + 2 * i + 1);
      uint4 o;
      o.x = Elem<T>::pack2(v[0] * ((g0.x + add) * prescale), v[1] * ((g0.y + add) * prescale));
      o.y = Elem<T>::pack2(v[2] * ((g0.z + add) * prescale), v[3] * ((g0.w + add) * prescale));
      o.z = Elem<T>::pack2(v[4] * ((g1.x + add) * prescale), v[5] * ((g1.y + add) * prescale));
      o.w = Elem<T>::pack2(v[6] * ((g1.z + add) * prescale), v[7] * ((g1.w + add) * prescale));
      cp[i] = o;
    }
    float q = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) q = fmaf(v[j], v[j], q);
    q += __shfl_xor_sync(0xffffffffu, q, 1);
    q += __shfl_xor_sync(0xffffffffu, q, 2);
    q += __shfl_xor_sync(0xffffffffu, q, 4);
    if (ok && (i & 7) == 0) ss[static_cast<size_t>(t) * (d / 64) + i / 8] = q;
  }
}

// RMSNorm of fp32 rows -> 16-bit T: out = T(x * rsqrt(mean(x^2) + eps) * g),
// g = w or (1 + w).
template <int NT, class T>
__global__ void __launch_bounds__(NT) rmsnorm_kernel(const float* __restrict__ x, int d, const float* __restrict__ w,
                                                     int plus_one, float eps, T* __restrict__ out, int rows) {
  __shared__ float red[NT / 32 + 1];
  const int r = blockIdx.x;
  if (r >= rows) return;
  const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(r) * d);
  float ss = 0.0f;
  for (int i = threadIdx.x; i < d / 4; i += NT) {
    const float4 v = xr[i];
    ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
  }
  ss = block_sum<NT>(ss, red);
  const float rstd = rsqrtf(ss / static_cast<float>(d) + eps);
  const float add = plus_one ? 1.0f : 0.0f;
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * d);
  const float4* wv = reinterpret_cast<const float4*>(w);
  for (int i = threadIdx.x; i < d / 4; i += NT) {
    const float4 v = xr[i];
    const float4 g = __ldg(wv + i);
    uint2 pk;
    pk.x = Elem<T>::pack2(v.x * rstd * (g.x + add), v.y * rstd * (g.y + add));
    pk.y = Elem<T>::pack2(v.z * rstd * (g.z + add), v.w * rstd * (g.w + add));
    o[i] = pk;
  }
}

// LayerNorm of fp32 rows: y = (x - mean) / sqrt(var + eps) * w + b.  Writes the
// fp32 result back in place when `inplace` and always a 16-bit copy to `out`.
template <int NT, class T>
__global__ void __launch_bounds__(NT)
    layernorm_kernel(float* __restrict__ x, int d, const float* __restrict__ w, const float* __restrict__ bvec,
                     float eps, int inplace, T* __restrict__ out, int rows) {
  __shared__ float red[NT / 32 + 1];
  const int r = blockIdx.x;
  if (r >= rows) return;
  float4* xr = reinterpret_cast<float4*>(x + static_cast<size_t>(r) * d);
  float s = 0.0f;
  for (int i = threadIdx.x; i < d / 4; i += NT) {
    const float4 v = xr[i];
    s += v.x + v.y + v.z + v.w;
  }
  const float mean = block_sum<NT>(s, red) / static_cast<float>(d);
  float ss = 0.0f;
  for (int i = threadIdx.x; i < d / 4; i += NT) {
    const float4 v = xr[i];
    const float a = v.x - mean, b = v.y - mean, c = v.z - mean, e = v.w - mean;
    ss += a * a + b * b + c * c + e * e;
  }
  const float rstd = rsqrtf(block_sum<NT>(ss, red) / static_cast<float>(d) + eps);
  const float4* wv = reinterpret_cast<const float4*>(w);
  const float4* bv = reinterpret_cast<const float4*>(bvec);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * d);
  for (int i = threadIdx.x; i < d / 4; i += NT) {
    float4 v = xr[i];
    const float4 g = __ldg(wv + i), bb = __ldg(bv + i);
    v.x = (v.x - mean) * rstd * g.x + bb.x;
    v.y = (v.y - mean) * rstd * g.y + bb.y;
    v.z = (v.z - mean) * rstd * g.z + bb.z;
    v.w = (v.w - mean) * rstd * g.w + bb.w;
    if (inplace) xr[i] = v;
    uint2 pk;
    pk.x = Elem<T>::pack2(v.x, v.y);
    pk.y = Elem<T>::pack2(v.z, v.w);
    o[i] = pk;
  }
}

// The same LayerNorm with one warp per row for d = 128 * VPT (VPT float4 per
// lane held in registers, shuffle reductions, no block barrier): 8 rows per
// CTA of 256 threads.  The encoder widths (768: VPT 6) are far too narrow to
// keep a 256-thread CTA per row busy.
template <int VPT, class T>
__global__ void __launch_bounds__(256)
    layernorm_warp_kernel(float* __restrict__ x, int d, const float* __restrict__ w, const float* __restrict__ bvec,
                          float eps, int inplace, T* __restrict__ out, int rows) {
  const int lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (r >= rows) return;
  float4* xr = reinterpret_cast<float4*>(x + static_cast<size_t>(r) * d);
  float4 v[VPT];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    v[k] = xr[lane + 32 * k];
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(d);
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const float a = v[k].x - mean, b = v[k].y - mean, c = v[k].z - mean, e = v[k].w - mean;
    ss += a * a + b * b + c * c + e * e;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / static_cast<float>(d) + eps);
  const float4* wv = reinterpret_cast<const float4*>(w);
  const float4* bv = reinterpret_cast<const float4*>(bvec);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<size_t>(r) * d);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    const float4 g = __ldg(wv + i), bb = __ldg(bv + i);
    float4 y;
    y.x = (v[k].x - mean) * rstd * g.x + bb.x;
    y.y = (v[k].y - mean) * rstd * g.y + bb.y;
    y.z = (v[k].z - mean) * rstd * g.z + bb.z;
    y.w = (v[k].w - mean) * rstd * g.w + bb.w;
    if (inplace) xr[i] = y;
    uint2 pk;
    pk.x = Elem<T>::pack2(y.x, y.y);
    pk.y = Elem<T>::pack2(y.z, y.w);
    o[i] = pk;
  }
}

// Encoder embeddings: h = LN(word[tok] + pos[p] + type[0]); fp32 h and a 16-bit copy.
template <int NT, class T>
__global__ void __launch_bounds__(NT)
    embed_ln_kernel(const int* __restrict__ tokens, const int* __restrict__ positions, int n_tokens,
                    const __nv_bfloat16* __restrict__ word, const __nv_bfloat16* __restrict__ pos_emb,
                    const __nv_bfloat16* __restrict__ type0, int d, const float* __restrict__ w,
                    const float* __restrict__ bvec, float eps, float* __restrict__ h, T* __restrict__ out) {
  const int t = blockIdx.x;
  if (t >= n_tokens) return;
  const __nv_bfloat16* a = word + static_cast<size_t>(tokens[t]) * d;
  const __nv_bfloat16* p = pos_emb + static_cast<size_t>(positions[t]) * d;
  float* hr = h + static_cast<size_t>(t) * d;
  for (int i = threadIdx.x; i < d; i += NT)
    hr[i] = __bfloat162float(a[i]) + __bfloat162float(p[i]) + __bfloat162float(type0[i]);
  __syncthreads();
  // Reuse the LayerNorm body on this single row.
  __shared__ float red[NT / 32 + 1];
  float s = 0.0f;
  for (int i = threadIdx.x; i < d; i += NT) s += hr[i];
  const float mean = block_sum<NT>(s, red) / static_cast<float>(d);
  float ss = 0.0f;
  for (int i = threadIdx.x; i < d; i += NT) {
    const float c = hr[i] - mean;
    ss += c * c;
  }
  const float rstd = rsqrtf(block_sum<NT>(ss, red) / static_cast<float>(d) + eps);
  for (int i = threadIdx.x; i < d; i += NT) {
    const float v = (hr[i] - mean) * rstd * w[i] + bvec[i];
    hr[i] = v;
    out[static_cast<size_t>(t) * d + i] = Elem<T>::from(v);
  }
}

// The same embedding LayerNorm with one warp per token for d = 128 * VPT: the
// three bf16 rows are summed in registers, reduced with shuffles and written
// once (h fp32, out 16-bit); 8 tokens per CTA of 256 threads.
template <int VPT, class T>
__global__ void __launch_bounds__(256)
    embed_ln_warp_kernel(const int* __restrict__ tokens, const int* __restrict__ positions, int n_tokens,
                         const __nv_bfloat16* __restrict__ word, const __nv_bfloat16* __restrict__ pos_emb,
                         const __nv_bfloat16* __restrict__ type0, int d, const float* __restrict__ w,
                         const float* __restrict__ bvec, float eps, float* __restrict__ h, T* __restrict__ out) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= n_tokens) return;
  const uint2* a = reinterpret_cast<const uint2*>(word + static_cast<size_t>(tokens[t]) * d);
  const uint2* p = reinterpret_cast<const uint2*>(pos_emb + static_cast<size_t>(positions[t]) * d);
  const uint2* c = reinterpret_cast<const uint2*>(type0);
  float4 v[VPT];
  float s = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    const uint2 x = __ldg(a + i), y = __ldg(p + i), z = __ldg(c + i);
    const float2 x0 = unpack_bf16x2(x.x), x1 = unpack_bf16x2(x.y);
    const float2 y0 = unpack_bf16x2(y.x), y1 = unpack_bf16x2(y.y);
    const float2 z0 = unpack_bf16x2(z.x), z1 = unpack_bf16x2(z.y);
    v[k] = make_float4(x0.x + y0.x + z0.x, x0.y + y0.y + z0.y, x1.x + y1.x + z1.x, x1.y + y1.y + z1.y);
    s += (v[k].x + v[k].y) + (v[k].z + v[k].w);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  const float mean = s / static_cast<float>(d);
  float ss = 0.0f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const float e0 = v[k].x - mean, e1 = v[k].y - mean, e2 = v[k].z - mean, e3 = v[k].w - mean;
    ss += e0 * e0 + e1 * e1 + e2 * e2 + e3 * e3;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float rstd = rsqrtf(ss / static_cast<float>(d) + eps);
  const float4* wv = reinterpret_cast<const float4*>(w);
  const float4* bv = reinterpret_cast<const float4*>(bvec);
  float4* hr = reinterpret_cast<float4*>(h + static_cast<size_t>(t) * d);
  uint2* o = reinterpret_cast<uint2*>(out + static_cast<size_t>(t) * d);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    const float4 g = __ldg(wv + i), bb = __ldg(bv + i);
    float4 y;
    y.x = (v[k].x - mean) * rstd * g.x + bb.x;
    y.y = (v[k].y - mean) * rstd * g.y + bb.y;
    y.z = (v[k].z - mean) * rstd * g.z + bb.z;
    y.w = (v[k].w - mean) * rstd * g.w + bb.w;
    hr[i] = y;
    uint2 pk;
    pk.x = Elem<T>::pack2(y.x, y.y);
    pk.y = Elem<T>::pack2(y.z, y.w);
    o[i] = pk;
  }
}

// The question-type add below with one warp per token (d = 128 * VPT), 8
// tokens per CTA: one float4 of h and four bf16 of the table per lane and step.
template <int VPT>
__global__ void __launch_bounds__(256)
    add_type_warp_kernel(float* __restrict__ h, int T, int d, const int* __restrict__ seq_id,
                         const int64_t* __restrict__ qtype, const __nv_bfloat16* __restrict__ table, int n_types,
                         int* err) {
  const int lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
  if (t >= T) return;
  int64_t q = qtype ? qtype[seq_id[t]] : 0;
  if (q < 0 || q >= n_types) {
    if (lane == 0) record_error(err, kErrTokenRange);
    q = 0;
  }
  const uint2* e = reinterpret_cast<const uint2*>(table + static_cast<size_t>(q) * d);
  float4* hr = reinterpret_cast<float4*>(h + static_cast<size_t>(t) * d);
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int i = lane + 32 * k;
    float4 v = hr[i];
    const uint2 x = __ldg(e + i);
    const float2 x0 = unpack_bf16x2(x.x), x1 = unpack_bf16x2(x.y);
    v.x += x0.x;
    v.y += x0.y;
    v.z += x1.x;
    v.w += x1.y;
    hr[i] = v;
  }
}

// h[t, :] += table[qtype[seq_id[t]], :] (the decision head's question-type embedding).
__global__ void add_type_kernel(float* __restrict__ h, int T, int d, const int* __restrict__ seq_id,
                                const int64_t* __restrict__ qtype, const __nv_bfloat16* __restrict__ table,
                                int n_types, int* err) {
  const int t = blockIdx.x;
  if (t >= T) return;
  int64_t q = qtype ? qtype[seq_id[t]] : 0;
  if (q < 0 || q >= n_types) {
    record_error(err, kErrTokenRange);
    q = 0;
  }
  const __nv_bfloat16* e = table + static_cast<size_t>(q) * d;
  float* hr = h + static_cast<size_t>(t) * d;
  for (int i = threadIdx.x; i < d; i += blockDim.x) hr[i] += __bfloat162float(e[i]);
}

// Slot rows of the packed batch -> compact per-decision buffers for the last
// layer, whose O projection and MLP only the slot rows need:
// attn_s[i] = attn[t_i], h_s[i] = h[t_i] with t_i = rows[i].base + marker_pos[i*k].
template <class T>
__global__ void gather_slot_rows_kernel(const RowMap* __restrict__ rows, const int64_t* __restrict__ marker_pos,
                                        int k, const T* __restrict__ attn, int ld_attn, const float* __restrict__ h,
                                        int d, T* __restrict__ attn_s, float* __restrict__ h_s, int* err) {
  const int i = blockIdx.x;
  const RowMap rm = rows[i];
  int64_t slot = marker_pos[static_cast<int64_t>(i) * k];
  if (slot < rm.lo || slot >= rm.hi) {
    if (threadIdx.x == 0) record_error(err, kErrSlotRange);
    slot = rm.lo;
  }
  const int64_t t = rm.base + slot;
  const uint4* a = reinterpret_cast<const uint4*>(attn + t * ld_attn);
  uint4* as = reinterpret_cast<uint4*>(attn_s + static_cast<int64_t>(i) * ld_attn);
  for (int j = threadIdx.x; j < ld_attn / 8; j += blockDim.x) as[j] = a[j];
  const float4* x = reinterpret_cast<const float4*>(h + t * d);
  float4* xs = reinterpret_cast<float4*>(h_s + static_cast<int64_t>(i) * d);
  for (int j = threadIdx.x; j < d / 4; j += blockDim.x) xs[j] = x[j];
}

// Decoder readout, one CTA per row: final RMSNorm of the slot token's hidden
// state, dot products with the first n option-label rows of the LM head (fp32,
// as `hs[slot].float() @ head_w.T`), then either the log-softmax restricted to
// the n options or the raw logits; columns >= n are -1e4.  An inf or NaN in the
// slot's hidden state or in a logit (a 16-bit activation that overflowed on the
// way, which poisons every later token of its row) is reported as
// kErrNonFinite, so the batch fails instead of returning meaningless scores.
template <int NT>
__global__ void __launch_bounds__(NT)
    readout_kernel(const float* __restrict__ h, int d, const RowMap* __restrict__ rows,
                   const int64_t* __restrict__ marker_pos, int k, const int64_t* __restrict__ nopts,
                   const float* __restrict__ norm_w, int plus_one, float eps, const float* __restrict__ head,
                   int n_labels, float* __restrict__ out, int width, int logprobs, int compact, int* err) {
  extern __shared__ float sm[];
  float* xs = sm;                 // [d]
  float* lg = sm + d;             // [n_labels]
  __shared__ float red[NT / 32 + 1];
  const int i = blockIdx.x;
  const RowMap rm = rows[i];
  const int64_t slot = marker_pos[static_cast<int64_t>(i) * k];
  int n = nopts ? static_cast<int>(nopts[i]) : n_labels;
  n = max(0, min(n, min(n_labels, width)));
  float* orow = out + static_cast<size_t>(i) * width;
  if (slot < rm.lo || slot >= rm.hi) {
    if (threadIdx.x == 0) record_error(err, kErrSlotRange);
    for (int j = threadIdx.x; j < width; j += NT) orow[j] = kSentinel;
    return;
  }
  // compact: h holds one row per decision (the slot rows, gathered before the
  // last layer's O projection); otherwise h is the packed batch.
  const float* x = compact ? h + static_cast<size_t>(i) * d : h + static_cast<size_t>(rm.base + slot) * d;
  float ss = 0.0f;
  bool finite = true;
  // Unrolled so that several loads per thread are in flight: at small batch
  // (one block per decision) the kernel is bound by DRAM latency, not bandwidth.
#pragma unroll 4
  for (int j = threadIdx.x; j < d; j += NT) {
    const float v = x[j];
    xs[j] = v;
    ss += v * v;
    finite &= isfinite(v);
  }
  if (!__syncthreads_and(finite) && threadIdx.x == 0) record_error(err, kErrNonFinite);
  const float rstd = rsqrtf(block_sum<NT>(ss, red) / static_cast<float>(d) + eps);
  const float add = plus_one ? 1.0f : 0.0f;
  for (int j = threadIdx.x; j < d; j += NT) xs[j] = xs[j] * rstd * (norm_w[j] + add);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int o = warp; o < n; o += NT / 32) {
    const float* hr = head + static_cast<size_t>(o) * d;
    float acc = 0.0f;
#pragma unroll 8
    for (int j = lane * 4; j < d; j += 128) {
      const float4 a = *reinterpret_cast<const float4*>(xs + j);
      const float4 b = __ldg(reinterpret_cast<const float4*>(hr + j));
      acc += a.x * b.x + a.y * b.y + a.z * b.z + a.w * b.w;
    }
#pragma unroll
    for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
    if (lane == 0) {
      lg[o] = acc;
      if (!isfinite(acc)) record_error(err, kErrNonFinite);
    }
  }
  __syncthreads();
  float shift = 0.0f;
  if (logprobs && n > 0) {
    if (threadIdx.x < 32) {
      float m = -INFINITY;
      for (int j = lane; j < n; j += 32) m = fmaxf(m, lg[j]);
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, s));
      float e = 0.0f;
      for (int j = lane; j < n; j += 32) e += expf(lg[j] - m);
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) e += __shfl_xor_sync(0xffffffffu, e, s);
      if (lane == 0) red[0] = m + logf(e);
    }
    __syncthreads();
    shift = red[0];
  }
  for (int j = threadIdx.x; j < width; j += NT) orow[j] = j < n ? lg[j] - shift : kSentinel;
}

// Independent-options layout of every packed token (`independent_options_tensors`,
// src/engine.rs:544-568): option j spans [marker_j, marker_{j+1}) (the last one
// up to the row's final token, exclusive); inside a span the position restarts
// at the first marker, elsewhere it is the column; tokens outside spans get
// option -1.  Markers are the row's live slots in order.  A row whose first
// marker is missing or outside the row is reported as a slot error.
__global__ void von_layout_kernel(const PackSeg* __restrict__ segs, int n_seg, const int64_t* __restrict__ mpos,
                                  const uint8_t* __restrict__ mmask, int k, int* __restrict__ opt_id,
                                  int* __restrict__ opt_pos, int* err) {
  const int si = blockIdx.y;
  if (si >= n_seg) return;
  const PackSeg sg = segs[si];
  const int64_t* mp = mpos + static_cast<int64_t>(sg.src_row) * k;
  const uint8_t* mm = mmask + static_cast<int64_t>(sg.src_row) * k;
  int first = -1;
  for (int j = 0; j < k; ++j)
    if (mm[j]) {
      first = static_cast<int>(mp[j]);
      break;
    }
  if (first < 0 || first >= sg.len) {
    if (blockIdx.x == 0 && threadIdx.x == 0) record_error(err, kErrSlotRange);
    first = sg.len;  // no spans
  }
  for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < sg.len; c += gridDim.x * blockDim.x) {
    int option = -1, pos = c, j = 0;
    for (int s = 0; s < k && first < sg.len; ++s) {
      if (!mm[s]) continue;
      const int start = static_cast<int>(mp[s]);
      int end = sg.len - 1;
      for (int t = s + 1; t < k; ++t)
        if (mm[t]) {
          end = static_cast<int>(mp[t]);
          break;
        }
      end = min(end, sg.len);
      if (c >= start && c < end) {
        option = j;
        pos = first + (c - start);
      }
      ++j;
    }
    opt_id[sg.start + c] = option;
    opt_pos[sg.start + c] = pos;
  }
}

// Encoder markers: flat token index of every (row, slot) pair, clamped like
// `marker_pos.clamp(min=0)`; a live marker outside its row is an input error.
__global__ void marker_index_kernel(const int* __restrict__ cu, const int64_t* __restrict__ marker_pos,
                                    const uint8_t* __restrict__ marker_mask, int b, int k, int* __restrict__ idx,
                                    int* err) {
  const int q = blockIdx.x * blockDim.x + threadIdx.x;
  if (q >= b * k) return;
  const int i = q / k;
  const int start = cu[i], len = cu[i + 1] - start;
  int64_t p = marker_pos[q];
  const bool live = marker_mask[q] != 0;
  if (live && (p < 0 || p >= len)) record_error(err, kErrSlotRange);
  p = p < 0 ? 0 : (p >= len ? len - 1 : p);
  idx[q] = start + static_cast<int>(p);
}

// Gather + LayerNorm of marker rows -> 16-bit scorer input.
template <int NT, class T>
__global__ void __launch_bounds__(NT)
    gather_layernorm_kernel(const float* __restrict__ h, const int* __restrict__ idx, int n, int d,
                            const float* __restrict__ w, const float* __restrict__ bvec, float eps,
                            T* __restrict__ out) {
  __shared__ float red[NT / 32 + 1];
  const int r = blockIdx.x;
  if (r >= n) return;
  const float* x = h + static_cast<size_t>(idx[r]) * d;
  float s = 0.0f;
  for (int i = threadIdx.x; i < d; i += NT) s += x[i];
  const float mean = block_sum<NT>(s, red) / static_cast<float>(d);
  float ss = 0.0f;
  for (int i = threadIdx.x; i < d; i += NT) {
    const float c = x[i] - mean;
    ss += c * c;
  }
  const float rstd = rsqrtf(block_sum<NT>(ss, red) / static_cast<float>(d) + eps);
  for (int i = threadIdx.x; i < d; i += NT)
    out[static_cast<size_t>(r) * d + i] = Elem<T>::from((x[i] - mean) * rstd * w[i] + bvec[i]);
}

// Final scorer projection Linear(d, 1) on the GELU'd rows, then the marker mask:
// out[i, j] = y[i*k + j] . w + b for live markers, -1e4 otherwise; columns
// j >= k of a wider output are -1e4.  A non-finite live logit (an activation
// that overflowed its 16-bit range upstream) is reported as kErrNonFinite.
template <class T>
__global__ void marker_score_kernel(const T* __restrict__ y, int d, const float* __restrict__ w,
                                    const float* __restrict__ bias, const uint8_t* __restrict__ marker_mask, int b,
                                    int k, float* __restrict__ out, int width, int* err) {
  const int i = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  for (int j = warp; j < width; j += nw) {
    float acc = 0.0f;
    if (j < k && marker_mask[i * k + j]) {
      const T* yr = y + static_cast<size_t>(i * k + j) * d;
      for (int c = lane; c < d; c += 32) acc += Elem<T>::to(yr[c]) * w[c];
#pragma unroll
      for (int s = 16; s > 0; s >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, s);
      acc += bias[0];
      if (lane == 0 && !isfinite(acc)) record_error(err, kErrNonFinite);
    } else {
      acc = kSentinel;
    }
    if (lane == 0) out[static_cast<size_t>(i) * width + j] = acc;
  }
}

}  // namespace vd
