// Causal varlen attention on the 5th-generation tensor cores (tcgen05 + TMEM),
// head_dim 128 (the OneJev-9B / 27B shapes).
//
// One CTA = one 128-row query tile of one sequence for TWO query heads that
// share a K/V head (GQA), so every K/V tile is loaded once for both, and two
// softmax warpgroups ping-pong against the tensor core:
//   warp 0      : TMA producer: both Q tiles once, then K and V tiles of 128
//                 keys through a 2-stage ring (128-byte swizzle, straight from
//                 the packed qkv buffer; V is consumed MN-major, no transpose)
//   warp 1      : TMEM allocator + MMA issuer (one lane), per K/V tile j:
//                 PV_h(j-1) and S_h(j) for h = 0, 1 in turn, so the tensor core
//                 works on one head while the other head's warps run softmax
//   warps 2..5  : softmax for head 0; warps 6..9 : softmax for head 1.
//                 One query row per thread: S_h(j) = Q_h K_j^T read from TMEM
//                 (max pass, then exp2 pass), P written back into TMEM over S
//                 as packed 16-bit pairs (the A operand of P V), O kept in TMEM.
// Online softmax with lazy rescaling: a row keeps its running max until a tile
// raises it by more than 8 (log2 units, so P <= 2^8); only then does the warp
// rescale its O rows in TMEM (load, multiply, store) before the next P V.
// TMEM: head h uses S/P at [256h, 256h+128) and O at [256h+128, 256h+256).
// Every mbarrier wait is bounded (common.cuh); on a timeout the CTA records an
// error code, raises its abort flag and all roles leave their loops.
#pragma once

#include "attention.cuh"
#include "common.cuh"

namespace vd {

// Shared-memory descriptor of an MN-major tile in the 128-byte swizzle: rows
// of 64 16-bit elements along MN (128 B), 8-row groups along K 1024 B apart
// (stride byte offset), MN atoms `lbo` bytes apart (leading byte offset).
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t smem_addr, uint32_t lbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>(1024 >> 4) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(2) << 61;
  return d;
}

// D[tmem] (+)= A[tmem] * B[smem]: the A operand (M lanes x K, two 16-bit
// elements per 32-bit column) comes from tensor memory.
__device__ __forceinline__ void umma_f16kind_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                                uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %6, %7, %8}, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(0), "r"(0), "r"(0), "r"(0)
      : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

// 32 columns of this thread's TMEM lane into r; completes at the next tmem_wait_ld().
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

// 2^x with the hardware approximation (flush-to-zero; exp2(-inf) = 0).
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

struct AttnTcParams {
  void* out;                   // T [tokens, ld_out]
  int ld_out;
  int q_col0, k_col0, v_col0;  // column offsets of the q / k / v blocks in qkv
  const AttnTile* tiles;       // 128-row query tiles
  int group;                   // query heads per K/V head
  int pairs_per_kv;            // ceil(group / 2): CTAs per K/V head and query tile
  float scale_log2;
  int* err;
};

struct AttnTcConfig {
  static constexpr int HD = 128, BM = 128, BN = 128;
  static constexpr int HALF_BYTES = 128 * 64 * 2;    // [128 rows x 64 cols] 16-bit, 16 KB
  static constexpr int TILE_BYTES = 2 * HALF_BYTES;  // 128 x 128, 32 KB
  static constexpr int Q_OFF = 0;                    // two Q tiles
  static constexpr int K_OFF = Q_OFF + 2 * TILE_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * TILE_BYTES;
  static constexpr int BAR_OFF = V_OFF + 2 * TILE_BYTES;
  static constexpr int SMEM_BYTES = 1024 + BAR_OFF + 256;
  static constexpr int THREADS = 320;
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr float RESCALE_THRESHOLD = 8.0f;  // log2 units
};

template <class T>
__global__ void __launch_bounds__(320, 1)
    attention_tc_kernel(const __grid_constant__ CUtensorMap tm_qkv, AttnTcParams p) {
  using C = AttnTcConfig;
  constexpr uint32_t FMT = Elem<T>::kUmmaFormat;
  constexpr uint32_t IDESC_S = umma_idesc_f16kind(128, 128, FMT);               // A, B K-major
  constexpr uint32_t IDESC_PV = umma_idesc_f16kind(128, 128, FMT) | (1u << 16);  // B (V) MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2] per stage
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* kv_empty = bars + 5;  // [2]
  uint64_t* s_full = bars + 7;    // [2] per head
  uint64_t* p_full = bars + 9;    // [2] per head
  uint64_t* o_final = bars + 11;  // [2] per head
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const AttnTile tile = p.tiles[blockIdx.x];
  const int kvh = blockIdx.y / p.pairs_per_kv;
  const int pair = blockIdx.y - kvh * p.pairs_per_kv;
  const int head0 = kvh * p.group + 2 * pair;
  const int nheads = (2 * pair + 1 < p.group) ? 2 : 1;
  const int kv_end = min(tile.seq_len, tile.q_start + C::BM);
  // Key tiles: first the shared prefix's (n_pre, unmasked but for its end),
  // then the sequence's own (causal).
  const int n_pre = (tile.pre_len + C::BN - 1) / C::BN;
  const int n_kv = n_pre + (kv_end + C::BN - 1) / C::BN;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&kv_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4);
      mbar_init(&o_final[i], 1);
    }
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, C::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tm_qkv);
      const int row0 = tile.seq_start;
      const int kx = p.k_col0 + kvh * C::HD, vx = p.v_col0 + kvh * C::HD;
      mbar_arrive_expect_tx(q_full, nheads * C::TILE_BYTES);
      for (int h = 0; h < nheads; ++h) {
        const int qx = p.q_col0 + (head0 + h) * C::HD;
        tma_load_2d(smem + C::Q_OFF + h * C::TILE_BYTES, &tm_qkv, q_full, qx, row0 + tile.q_start);
        tma_load_2d(smem + C::Q_OFF + h * C::TILE_BYTES + C::HALF_BYTES, &tm_qkv, q_full, qx + 64,
                    row0 + tile.q_start);
      }
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&kv_empty[s], ((j >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutEmpty)) break;
        const int y = j < n_pre ? tile.pre_start + j * C::BN : row0 + (j - n_pre) * C::BN;
        mbar_arrive_expect_tx(&k_full[s], C::TILE_BYTES);
        tma_load_2d(smem + C::K_OFF + s * C::TILE_BYTES, &tm_qkv, &k_full[s], kx, y);
        tma_load_2d(smem + C::K_OFF + s * C::TILE_BYTES + C::HALF_BYTES, &tm_qkv, &k_full[s], kx + 64, y);
        mbar_arrive_expect_tx(&v_full[s], C::TILE_BYTES);
        tma_load_2d(smem + C::V_OFF + s * C::TILE_BYTES, &tm_qkv, &v_full[s], vx, y);
        tma_load_2d(smem + C::V_OFF + s * C::TILE_BYTES + C::HALF_BYTES, &tm_qkv, &v_full[s], vx + 64, y);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // S_h(j) = Q_h K_j^T into head h's S columns.
      auto issue_s = [&](int h, int j) {
        const uint32_t q_addr = smem_u32(smem + C::Q_OFF + h * C::TILE_BYTES);
        const uint32_t k_addr = smem_u32(smem + C::K_OFF + (j & 1) * C::TILE_BYTES);
#pragma unroll
        for (int kk = 0; kk < 8; ++kk) {
          const uint32_t off = (kk >> 2) * C::HALF_BYTES + (kk & 3) * 32;
          umma_f16kind(tmem + h * 256, sw128_kmajor_desc(q_addr + off), sw128_kmajor_desc(k_addr + off), IDESC_S,
                       kk != 0 ? 1u : 0u);
        }
        umma_commit(&s_full[h]);
      };
      bool ok = mbar_wait(q_full, 0, abort_flag, p.err, kErrTimeoutFull) &&
                mbar_wait(&k_full[0], 0, abort_flag, p.err, kErrTimeoutFull);
      if (ok) {
        tc_fence_after();
        for (int h = 0; h < nheads; ++h) issue_s(h, 0);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&v_full[s], (j >> 1) & 1, abort_flag, p.err, kErrTimeoutFull)) break;
        if (j + 1 < n_kv &&
            !mbar_wait(&k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, abort_flag, p.err, kErrTimeoutFull))
          break;
        const uint32_t v_addr = smem_u32(smem + C::V_OFF + s * C::TILE_BYTES);
        for (int h = 0; h < nheads; ++h) {
          if (!mbar_wait(&p_full[h], j & 1, abort_flag, p.err, kErrTimeoutFull)) {
            ok = false;
            break;
          }
          tc_fence_after();
          // O_h += P_h(j) V_j: A = P from TMEM (8 columns per K step of 16 keys),
          // B = V MN-major (hd halves HALF_BYTES apart), K advances 16 rows = 2 KB.
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_f16kind_ts(tmem + h * 256 + 128, tmem + h * 256 + kk * 8,
                            sw128_mnmajor_desc(v_addr + kk * 2048, C::HALF_BYTES), IDESC_PV,
                            (j > 0 || kk > 0) ? 1u : 0u);
          if (j + 1 == n_kv) umma_commit(&o_final[h]);
          // The next S overwrites P_h(j) in TMEM; MMAs of one thread run in order.
          if (j + 1 < n_kv) issue_s(h, j + 1);
        }
        if (!ok) break;
        umma_commit(&kv_empty[s]);
      }
    }
  } else {
    // Softmax warps: head h = (warp - 2) / 4, thread = query row r of the tile.
    const int h = (warp - 2) >> 2;
    if (h < nheads) {
      const int quarter = warp & 3;
      const int r = quarter * 32 + lane;
      const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
      const uint32_t s_tm = tmem + lane_base + h * 256;
      const uint32_t o_tm = s_tm + 128;
      const int q_row = tile.q_start + r;  // row inside the sequence
      float m_run = -INFINITY, l_run = 0.0f;
      bool ok = true;
      for (int j = 0; j < n_kv; ++j) {
        const bool in_pre = j < n_pre;
        const int kv0 = (in_pre ? j : j - n_pre) * C::BN;  // key index inside its segment
        const int seg_len = in_pre ? tile.pre_len : tile.seq_len;
        // Prefix keys precede every query row: only the causal limit of own keys applies.
        const int causal_row = in_pre ? 0x7fffffff : q_row;
        if (!mbar_wait(&s_full[h], j & 1, abort_flag, p.err, kErrTimeoutAccFull)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const bool need_mask = kv0 + C::BN > seg_len || (!in_pre && kv0 + C::BN > tile.q_start);
        // The whole 128-column S row: four loads in flight, one wait.
        uint32_t sr[128];
        tmem_ld32_nowait(s_tm + 0, sr + 0);
        tmem_ld32_nowait(s_tm + 32, sr + 32);
        tmem_ld32_nowait(s_tm + 64, sr + 64);
        tmem_ld32_nowait(s_tm + 96, sr + 96);
        tmem_wait_ld();
        float mx = -INFINITY;
        if (need_mask) {
#pragma unroll
          for (int i = 0; i < 128; ++i) {
            const int kv = kv0 + i;
            if (kv >= seg_len || kv > causal_row) sr[i] = __float_as_uint(-INFINITY);
            mx = fmaxf(mx, __uint_as_float(sr[i]));
          }
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
        }
        const float m_tile = mx * p.scale_log2;
        const bool raise = m_tile > m_run + C::RESCALE_THRESHOLD;
        const bool warp_raise = __any_sync(0xffffffffu, raise);
        const float m_new = raise ? m_tile : m_run;
        const float alpha = raise ? fast_exp2(m_run - m_new) : 1.0f;
        // P = exp2(s * scale - m) as packed 16-bit pairs written over S
        // (masked scores are -inf and give exactly 0).
        float rs = 0.0f;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float e0 = fast_exp2(__uint_as_float(sr[c * 32 + i]) * p.scale_log2 - m_new);
            const float e1 = fast_exp2(__uint_as_float(sr[c * 32 + i + 1]) * p.scale_log2 - m_new);
            rs += e0 + e1;
            pk[i >> 1] = Elem<T>::pack2(e0, e1);
          }
          tmem_st16(s_tm + c * 16, pk);
        }
        // A raised max rescales the O rows accumulated so far (none before tile 0).
        if (warp_raise && j > 0) {
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_load_f32x32(o_tm + c * 32, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tmem_st32f(o_tm + c * 32, v);
          }
        }
        tmem_wait_st();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[h]);
        l_run = l_run * alpha + rs;
        m_run = m_new;
      }
      if (ok && mbar_wait(&o_final[h], 0, abort_flag, p.err, kErrTimeoutAccFull)) {
        tc_fence_after();
        const float inv = l_run > 0.0f ? 1.0f / l_run : 0.0f;
        T* dst = static_cast<T*>(p.out) + static_cast<size_t>(tile.seq_start + q_row) * p.ld_out +
                 (head0 + h) * C::HD;
#pragma unroll 1
        for (int c = 0; c < 4; ++c) {
          float v[32];
          tmem_load_f32x32(o_tm + c * 32, v);
          if (q_row < tile.seq_len) {
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= inv;
            store_x32<T>(dst + c * 32, v);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) {
    __syncwarp();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

}  // namespace vd
