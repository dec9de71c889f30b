// Varlen (packed, ragged) multi-head attention for the prefill-only decision
// forward: causal for the decoders, bidirectional for the marker-head encoders,
// with grouped K/V heads (GQA / MQA).
//
// Input is the fused projection output qkv[T, ld] (16-bit T: fp16 or bf16): head h of Q at column
// q_col0 + h*HD, its K/V head (h / group) at k_col0 / v_col0 + (h/group)*HD.
// Output attn[T, ld_out] at column h*HD.  Sequences are given by cu_seqlens; a
// CTA processes one 64-row query tile of one sequence for one query head, as
// listed in a host-built tile table (longest causal work first).
//
// This is the warp-level (ldmatrix + mma.sync m16n8k16) flash-attention
// formulation: Q tile in smem, double-buffered K/V tiles via cp.async with a
// 16-byte XOR swizzle, online softmax in registers (exp2 with the 1/sqrt(d)
// scale folded in), fp32 accumulation.
#pragma once

#include "common.cuh"

namespace vd {

// One query tile of one packed sequence.  A sequence that continues a shared
// prefix (the suffix of a forked row) also attends to that prefix's keys,
// stored once elsewhere in the packed batch: all of them, before its own keys
// (every prefix position precedes every suffix position).
struct AttnTile {
  int seq_start;  // first token of the sequence in the packed batch
  int seq_len;
  int q_start;    // first query row of this tile inside the sequence
  int pre_start;  // first token of the shared prefix in the packed batch
  int pre_len;    // prefix keys (0: none)
  int pad[3];
};

struct AttnParams {
  const void* qkv;        // T [T, ld_qkv]
  int ld_qkv;
  int q_col0, k_col0, v_col0;
  void* out;              // T [T, ld_out]
  int ld_out;
  const AttnTile* tiles;
  int group;          // query heads per K/V head
  float scale_log2;   // softmax scale * log2(e)
  int gate_col0;      // >= 0: output *= sigmoid(qkv[row, gate_col0 + head*HD + c]) (gated attention)
  // Independent-options masking (null: none): per packed token its option
  // (-1 = shared) and option-invariant position; a token attends to shared
  // tokens and to its own option, within `window` positions when window > 0.
  const int* opt_id;
  const int* opt_pos;
  int window;
};

template <int HD>
struct AttnConfig {
  static constexpr int BM = 64, BN = 64, THREADS = 128;
  static constexpr int Q_BYTES = BM * HD * 2;
  static constexpr int KV_BYTES = BN * HD * 2;
  static constexpr int SMEM_BYTES = Q_BYTES + 4 * KV_BYTES;  // Q, K[2], V[2]
};

// Byte offset of 16-byte chunk c of row r in a [rows][HD] bf16 tile.
template <int HD>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * HD * 2 + ((c ^ (r & 7)) << 4));
}

template <int HD, class T>
__device__ __forceinline__ void load_tile_async(uint32_t s_base, const T* g, int ld, int row0,
                                                int rows_valid, int tid) {
  constexpr int CH = HD / 8;  // 16-byte chunks per row
  constexpr int TOTAL = 64 * CH;
#pragma unroll
  for (int i = tid; i < TOTAL; i += 128) {
    const int r = i / CH, c = i % CH;
    const bool ok = r < rows_valid;
    const T* src = g + static_cast<size_t>(row0 + (ok ? r : 0)) * ld + c * 8;
    cp_async16(s_base + swz<HD>(r, c), src, ok);
  }
}

template <int HD, bool CAUSAL, class T>
__global__ void __launch_bounds__(128, HD == 64 ? 4 : 1) attention_varlen_kernel(AttnParams p) {
  using Cfg = AttnConfig<HD>;
  constexpr int NB = Cfg::BN / 8;   // n-blocks of S per warp (8)
  constexpr int ND = HD / 8;        // n-blocks of O per warp
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t sQ = smem_u32(smem);
  const uint32_t sK0 = sQ + Cfg::Q_BYTES;
  const uint32_t sV0 = sK0 + 2 * Cfg::KV_BYTES;

  const AttnTile tile = p.tiles[blockIdx.x];
  const int head = blockIdx.y;
  const int kvh = head / p.group;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  const T* qkv = static_cast<const T*>(p.qkv);
  const T* gq = qkv + static_cast<size_t>(tile.seq_start) * p.ld_qkv + p.q_col0 + head * HD;
  const T* gk = qkv + p.k_col0 + kvh * HD;  // rows are absolute packed-token indices
  const T* gv = qkv + p.v_col0 + kvh * HD;

  const int q_rows = min(Cfg::BM, tile.seq_len - tile.q_start);
  int kv_end = tile.seq_len;
  if (CAUSAL) kv_end = min(tile.seq_len, tile.q_start + Cfg::BM);
  // Key tiles: first the shared prefix's (n_pre), then the sequence's own.
  const int n_pre = (tile.pre_len + Cfg::BN - 1) / Cfg::BN;
  const int n_kv = n_pre + (kv_end + Cfg::BN - 1) / Cfg::BN;
  auto kv_row = [&](int j) { return j < n_pre ? tile.pre_start + j * Cfg::BN : tile.seq_start + (j - n_pre) * Cfg::BN; };
  auto kv_rows = [&](int j) {
    return j < n_pre ? min(Cfg::BN, tile.pre_len - j * Cfg::BN) : min(Cfg::BN, tile.seq_len - (j - n_pre) * Cfg::BN);
  };

  load_tile_async<HD, T>(sQ, gq, p.ld_qkv, tile.q_start, q_rows, tid);
  load_tile_async<HD, T>(sK0, gk, p.ld_qkv, kv_row(0), kv_rows(0), tid);
  load_tile_async<HD, T>(sV0, gv, p.ld_qkv, kv_row(0), kv_rows(0), tid);
  cp_async_commit();

  float o[ND][4];
#pragma unroll
  for (int i = 0; i < ND; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.0f;
  float m_run[2] = {-INFINITY, -INFINITY};
  float l_run[2] = {0.0f, 0.0f};

  const int q_row_a = tile.q_start + warp * 16 + (lane >> 2);  // rows of c0/c1; c2/c3 are +8
  // Option id and position of this thread's two query rows (option masks only).
  int q_opt[2] = {-1, -1}, q_pos[2] = {0, 0};
  if (p.opt_id != nullptr) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int qr = q_row_a + 8 * h;
      if (qr < tile.seq_len) {
        q_opt[h] = __ldg(p.opt_id + tile.seq_start + qr);
        if (p.window > 0) q_pos[h] = __ldg(p.opt_pos + tile.seq_start + qr);
      }
    }
  }

  for (int j = 0; j < n_kv; ++j) {
    const int buf = j & 1;
    if (j + 1 < n_kv) {
      const uint32_t nb = (buf ^ 1) * Cfg::KV_BYTES;
      load_tile_async<HD, T>(sK0 + nb, gk, p.ld_qkv, kv_row(j + 1), kv_rows(j + 1), tid);
      load_tile_async<HD, T>(sV0 + nb, gv, p.ld_qkv, kv_row(j + 1), kv_rows(j + 1), tid);
      cp_async_commit();
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();

    const uint32_t sK = sK0 + buf * Cfg::KV_BYTES;
    const uint32_t sV = sV0 + buf * Cfg::KV_BYTES;
    const bool in_pre = j < n_pre;
    const int kv0 = (in_pre ? j : j - n_pre) * Cfg::BN;  // key index inside its segment

    // S = Q K^T for this warp's 16 query rows x 64 keys.
    float s[NB][4];
#pragma unroll
    for (int i = 0; i < NB; ++i) s[i][0] = s[i][1] = s[i][2] = s[i][3] = 0.0f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t a[4];
      {
        const int r = warp * 16 + (lane & 15);
        const int c = ks * 2 + (lane >> 4);
        ldmatrix_x4(sQ + swz<HD>(r, c), a[0], a[1], a[2], a[3]);
      }
#pragma unroll
      for (int nb2 = 0; nb2 < NB / 2; ++nb2) {
        uint32_t b0, b1, b2, b3;
        const int r = nb2 * 16 + (lane & 7) + ((lane >> 4) << 3);
        const int c = ks * 2 + ((lane >> 3) & 1);
        ldmatrix_x4(sK + swz<HD>(r, c), b0, b1, b2, b3);
        mma_16816<T>(s[2 * nb2], a, b0, b1);
        mma_16816<T>(s[2 * nb2 + 1], a, b2, b3);
      }
    }

    // Mask keys past the segment end and (causal, own keys only) past the query row.
    const int seg_len = in_pre ? tile.pre_len : tile.seq_len;
    const bool need_mask = (kv0 + Cfg::BN > seg_len) || (CAUSAL && !in_pre && kv0 + Cfg::BN > tile.q_start) ||
                           p.opt_id != nullptr;
    if (need_mask && p.opt_id != nullptr) {
      // Option masks (bidirectional encoders only: no prefix segment here).
      // A key is visible iff it is a shared token or in the query's own option
      // (for a shared query the two coincide), and in local layers within the
      // window.  Keys past the sequence end carry an option code nothing
      // matches.  Rows past the end are never stored, so they are not masked.
      constexpr int kKeyDead = -3;
      int kopt[NB][2], kpos[NB][2];
      bool all_shared = true;
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
        for (int e2 = 0; e2 < 2; ++e2) {
          const int kv = kv0 + nb * 8 + ((lane & 3) << 1) + e2;
          const bool in = kv < seg_len;
          const int kt = tile.seq_start + (in ? kv : 0);
          kopt[nb][e2] = in ? __ldg(p.opt_id + kt) : kKeyDead;
          kpos[nb][e2] = (in && p.window > 0) ? __ldg(p.opt_pos + kt) : 0;
          all_shared = all_shared && kopt[nb][e2] == -1;
        }
      }
      // Global layers: a tile of shared keys is visible to every query row.
      if (!(p.window <= 0 && __all_sync(0xffffffffu, all_shared))) {
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
          for (int e2 = 0; e2 < 2; ++e2) {
            const int ko = kopt[nb][e2];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              bool ok = ko == -1 || ko == q_opt[h];
              if (p.window > 0) {
                const int d = q_pos[h] - kpos[nb][e2];
                ok = ok && d <= p.window && -d <= p.window;
              }
              if (!ok) s[nb][2 * h + e2] = -INFINITY;
            }
          }
        }
      }
    } else if (need_mask) {
#pragma unroll
      for (int nb = 0; nb < NB; ++nb) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int kv = kv0 + nb * 8 + ((lane & 3) << 1) + (e & 1);
          const int qr = q_row_a + ((e >> 1) << 3);
          bool dead = kv >= seg_len;
          if (CAUSAL && !in_pre) dead = dead || kv > qr;
          if (dead) s[nb][e] = -INFINITY;
        }
      }
    }

    // Online softmax (rows r and r+8 of the warp tile; a quad of lanes shares a row).
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      mx[0] = fmaxf(mx[0], fmaxf(s[nb][0], s[nb][1]));
      mx[1] = fmaxf(mx[1], fmaxf(s[nb][2], s[nb][3]));
    }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 1));
      mx[h] = fmaxf(mx[h], __shfl_xor_sync(0xffffffffu, mx[h], 2));
    }
    float alpha[2], base[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float m_new = fmaxf(m_run[h], mx[h] * p.scale_log2);
      base[h] = (m_new == -INFINITY) ? 0.0f : m_new;
      alpha[h] = exp2f(m_run[h] - base[h]);
      m_run[h] = m_new;
    }
    float rs[2] = {0.0f, 0.0f};
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
      s[nb][0] = exp2f(s[nb][0] * p.scale_log2 - base[0]);
      s[nb][1] = exp2f(s[nb][1] * p.scale_log2 - base[0]);
      s[nb][2] = exp2f(s[nb][2] * p.scale_log2 - base[1]);
      s[nb][3] = exp2f(s[nb][3] * p.scale_log2 - base[1]);
      rs[0] += s[nb][0] + s[nb][1];
      rs[1] += s[nb][2] + s[nb][3];
    }
    l_run[0] = l_run[0] * alpha[0] + rs[0];
    l_run[1] = l_run[1] * alpha[1] + rs[1];
#pragma unroll
    for (int nd = 0; nd < ND; ++nd) {
      o[nd][0] *= alpha[0];
      o[nd][1] *= alpha[0];
      o[nd][2] *= alpha[1];
      o[nd][3] *= alpha[1];
    }

    // O += P V.
#pragma unroll
    for (int ks = 0; ks < Cfg::BN / 16; ++ks) {
      uint32_t a[4];
      a[0] = Elem<T>::pack2(s[2 * ks][0], s[2 * ks][1]);
      a[1] = Elem<T>::pack2(s[2 * ks][2], s[2 * ks][3]);
      a[2] = Elem<T>::pack2(s[2 * ks + 1][0], s[2 * ks + 1][1]);
      a[3] = Elem<T>::pack2(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
      for (int nd2 = 0; nd2 < ND / 2; ++nd2) {
        uint32_t b0, b1, b2, b3;
        const int r = ks * 16 + (lane & 7) + (((lane >> 3) & 1) << 3);
        const int c = nd2 * 2 + (lane >> 4);
        ldmatrix_x4_trans(sV + swz<HD>(r, c), b0, b1, b2, b3);
        mma_16816<T>(o[2 * nd2], a, b0, b1);
        mma_16816<T>(o[2 * nd2 + 1], a, b2, b3);
      }
    }
    __syncthreads();
  }

  // Normalise and store rows inside the sequence.
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  const float inv0 = l_run[0] > 0.0f ? 1.0f / l_run[0] : 0.0f;
  const float inv1 = l_run[1] > 0.0f ? 1.0f / l_run[1] : 0.0f;
  const int r0 = warp * 16 + (lane >> 2);
  T* out0 = static_cast<T*>(p.out) + static_cast<size_t>(tile.seq_start + tile.q_start + r0) * p.ld_out + head * HD;
  T* out1 = out0 + static_cast<size_t>(8) * p.ld_out;
  const bool ok0 = r0 < q_rows, ok1 = r0 + 8 < q_rows;
  const T* gate0 = p.gate_col0 >= 0
                       ? qkv + static_cast<size_t>(tile.seq_start + tile.q_start + r0) * p.ld_qkv + p.gate_col0 +
                             head * HD
                       : nullptr;
#pragma unroll
  for (int nd = 0; nd < ND; ++nd) {
    const int col = nd * 8 + ((lane & 3) << 1);
    float g0 = 1.0f, g1 = 1.0f, g2 = 1.0f, g3 = 1.0f;
    if (gate0 != nullptr) {
      if (ok0) {
        const float2 g = Elem<T>::unpack2(*reinterpret_cast<const uint32_t*>(gate0 + col));
        g0 = 1.0f / (1.0f + __expf(-g.x));
        g1 = 1.0f / (1.0f + __expf(-g.y));
      }
      if (ok1) {
        const float2 g = Elem<T>::unpack2(*reinterpret_cast<const uint32_t*>(gate0 + 8 * static_cast<size_t>(p.ld_qkv) + col));
        g2 = 1.0f / (1.0f + __expf(-g.x));
        g3 = 1.0f / (1.0f + __expf(-g.y));
      }
    }
    if (ok0) *reinterpret_cast<uint32_t*>(out0 + col) = Elem<T>::pack2(o[nd][0] * inv0 * g0, o[nd][1] * inv0 * g1);
    if (ok1) *reinterpret_cast<uint32_t*>(out1 + col) = Elem<T>::pack2(o[nd][2] * inv1 * g2, o[nd][3] * inv1 * g3);
  }
}

}  // namespace vd
