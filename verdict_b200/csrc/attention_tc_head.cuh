// Varlen attention on the tcgen05 tensor cores, one query head per CTA:
// causal with head_dim HD = 128 or 256 (256: the Gemma-2B decider and the
// Qwen3.5 hybrids' gated attention layers, where O alone fills 256 TMEM
// columns), or bidirectional (CAUSAL = false) with HD = 64 for the marker-head
// encoders (every key of the sequence, no option masks).
//
// Work item = one 128-row query tile of one sequence for one query head; keys
// in tiles of 64.  A CTA runs items blockIdx.x, blockIdx.x + gridDim.x, ...
// (persistent when the grid is smaller than the item count): its barriers and
// tensor memory are set up once, and the next item's Q load and first two S
// MMAs run while the previous item's O is stored.  Items are
// tile-major, head-minor over a tile table sorted by work, so the query heads
// of one K/V head read the same K/V tiles at about the same time.  TMEM: two
// S/P buffers of 64 columns (S of tile j + 1 is computed while the softmax
// warps work on tile j) and O, 128 rows x HD fp32 columns.
//   warp 0      : TMA producer of Q (once) and the K tiles (2-stage ring)
//   warp 1      : TMEM allocator + MMA issuer (one lane):
//                 S(0), S(1), then per tile j: O += P(j) V(j) (A = P from
//                 TMEM, B = V MN-major), S(j + 2) into the buffer P(j) used
//   warp 2      : TMA producer of the V tiles (2-stage ring; a K stage is
//                 released once its S is computed, a V stage once its P V is)
//   warps 3..6  : softmax, one query row per thread (TMEM lane quarter = warp
//                 & 3): S from TMEM, running max with lazy rescaling (a row
//                 keeps its max until a tile raises it by more than 8 in log2
//                 units; a raise rescales O in TMEM after the previous P V has
//                 completed), P packed to 16-bit pairs over S; at an item's end
//                 O / l (times sigmoid(gate) for gated attention) to global.
// head_dim 256 (one CTA per SM, registers to spare) moves that last step to
// four drain warps: warp 3 has no role, softmax is warps 4..7, and at an
// item's end they hand the row sums to drain warps 8..11 through shared
// memory and start the next item; the drain warps wait for the item's last
// P V, store O / l, and release O to the next item's first P V.
// Shared memory: Q HD/64 swizzled 128 x 64 atoms (HD = 256: 64 KB), K and V
// two stages of HD/64 64 x 64 atoms each (HD = 256: 2 x 32 KB each).  At HD =
// 128 a CTA takes 96 KB and 256 TMEM columns (at HD = 64, 48 KB and 256
// columns), so two run per SM and one's prologue and epilogue overlap the
// other's main loop.  Every mbarrier wait
// is bounded; on a timeout the CTA records an error code, raises its abort
// flag and all roles leave their loops.
#pragma once

#include "attention_tc.cuh"

namespace vd {

struct AttnTcHeadParams {
  void* out;                   // T [tokens, ld_out]
  int ld_out;
  const void* qkv;             // T [tokens, ld_qkv] (gate columns for gated attention)
  int ld_qkv;
  int q_col0, k_col0, v_col0;  // column offsets of the q / k / v blocks in qkv
  int gate_col0;               // >= 0: output *= sigmoid(qkv[:, gate_col0 + head * HD + c])
  const AttnTile* tiles;       // 128-row query tiles
  int n_tiles, heads;          // work items: n_tiles * heads, item = tile * heads + head
  int group;                   // query heads per K/V head
  float scale_log2;
  int* err;
};

// SPR: softmax threads per query row (1: four softmax warps, a thread holds its
// row's 64 scores of a key tile; 2: eight softmax warps, two per TMEM lane
// quarter, each holding 32 of the 64 scores and half of O's columns, the row
// max exchanged through shared memory).
template <int HD_, int SPR_ = 1>
struct AttnTcHeadConfig {
  static constexpr int HD = HD_, BM = 128, BN = 64, SPR = SPR_;
  static constexpr int ATOMS = HD / 64;             // 64-column swizzle atoms per row
  static constexpr int Q_ATOM = BM * 64 * 2;        // [128 rows x 64 cols] 16-bit, 16 KB
  static constexpr int KV_ATOM = BN * 64 * 2;       // [64 rows x 64 cols], 8 KB
  static constexpr int Q_BYTES = ATOMS * Q_ATOM;
  static constexpr int KV_BYTES = ATOMS * KV_ATOM;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + Q_BYTES;
  static constexpr int V_OFF = K_OFF + 2 * KV_BYTES;
  static constexpr int BAR_OFF = V_OFF + 2 * KV_BYTES;
  // SPR = 2 exchange: [3][4 quarters][32 rows][2 parts] floats; regions 0 and 1
  // carry the row maxima of even and odd key tiles, region 2 the row sums.
  // DRAIN: the row sums of two items in flight, [2][128] floats.
  static constexpr int XCH_OFF = BAR_OFF + 256;
  // DRAIN (head_dim 256, one CTA per SM): four more warps take each item's O
  // from TMEM to global while the softmax warps start the next item.  With
  // two CTAs per SM (head_dim 64 and 128) the extra warps would take the
  // softmax warps' registers, and the softmax warps drain O themselves.
  static constexpr bool DRAIN = SPR == 1 && HD == 256;
  static constexpr int SMEM_BYTES = 1024 + XCH_OFF + (SPR == 2 ? 3 * 4 * 32 * 2 * 4 : DRAIN ? 2 * BM * 4 : 0);
  static constexpr int SOFTMAX_WARP0 = DRAIN ? 4 : 3;
  static constexpr int DRAIN_WARP0 = 8;
  static constexpr int THREADS = DRAIN ? 384 : 96 + 128 * SPR;
  static constexpr uint32_t TMEM_COLS = HD == 256 ? 512 : 256;  // S/P [0, 128), O [128, 128 + HD)
  static constexpr int MIN_CTAS = HD == 256 ? 1 : 2;
  static constexpr float RESCALE_THRESHOLD = 8.0f;
};

// Named barrier (ids 2..5, one per TMEM lane quarter) over the two softmax
// warps of a row pair, ANDing a warp-uniform flag.
__device__ __forceinline__ bool pair_bar_and(int id, bool v) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 q, %2, 0;\n\t"
      "bar.red.and.pred p, %1, 64, q;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(r)
      : "r"(id), "r"(static_cast<uint32_t>(v))
      : "memory");
  return r != 0;
}

// Row q_row of an item's O (columns [part OC, +OC) of the head) from TMEM:
// O / l_tot, times sigmoid(gate) for gated attention, to global.  Rows past
// the sequence are read (the TMEM load is warp-wide) but not stored.
template <int HD, int OC, class T>
__device__ __forceinline__ void attn_head_store_o(const AttnTcHeadParams& p, const AttnTile& tile, int head,
                                                  int q_row, int part, uint32_t o_tm, float l_tot) {
  const float inv = l_tot > 0.0f ? 1.0f / l_tot : 0.0f;
  const size_t tok = static_cast<size_t>(tile.seq_start + q_row);
  T* dst = static_cast<T*>(p.out) + tok * p.ld_out + head * HD + part * OC;
  const T* gate =
      p.gate_col0 >= 0 ? static_cast<const T*>(p.qkv) + tok * p.ld_qkv + p.gate_col0 + head * HD + part * OC : nullptr;
  const bool live = q_row < tile.seq_len;
#pragma unroll 1
  for (int c = 0; c < OC / 32; ++c) {
    float v[32];
    tmem_load_f32x32(o_tm + c * 32, v);
    if (live) {
      if (gate != nullptr) {
        const uint4* g4 = reinterpret_cast<const uint4*>(gate + c * 32);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const uint4 gw = g4[q];
          const uint32_t ws[4] = {gw.x, gw.y, gw.z, gw.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const float2 gg = Elem<T>::unpack2(ws[e]);
            v[q * 8 + 2 * e] *= inv * __fdividef(1.0f, 1.0f + __expf(-gg.x));
            v[q * 8 + 2 * e + 1] *= inv * __fdividef(1.0f, 1.0f + __expf(-gg.y));
          }
        }
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] *= inv;
      }
      store_x32<T>(dst + c * 32, v);
    }
  }
}

template <int HD, class T, bool CAUSAL = true, int SPR = 1>
__global__ void __launch_bounds__(AttnTcHeadConfig<HD, SPR>::THREADS, AttnTcHeadConfig<HD, SPR>::MIN_CTAS)
    attention_tc_head_kernel(const __grid_constant__ CUtensorMap tm_qkv64, AttnTcHeadParams p) {
  using C = AttnTcHeadConfig<HD, SPR>;
  constexpr uint32_t FMT = Elem<T>::kUmmaFormat;
  constexpr uint32_t IDESC_S = umma_idesc_f16kind(128, 64, FMT);                // A, B K-major
  constexpr uint32_t IDESC_PV = umma_idesc_f16kind(128, HD, FMT) | (1u << 16);   // B (V) MN-major

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + C::BAR_OFF);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2] per stage
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* k_empty = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2] per S/P buffer
  uint64_t* p_full = bars + 11;   // [2]
  uint64_t* pv_done = bars + 13;  // one arrival per P V
  uint64_t* o_final = bars + 14;  // an item's last P V has landed in O
  uint64_t* q_free = bars + 15;   // an item's last S has read Q: the next Q may load
  uint64_t* o_free = bars + 16;   // the softmax warps have drained O: the next P V may overwrite it
  uint64_t* mma_drained = bars + 17;  // the MMA warp's own ops, on its abort path
  uint64_t* l_full = bars + 18;   // [2] DRAIN: an item's row sums are in lsum[qi & 1]
  uint64_t* l_empty = bars + 20;  // [2] DRAIN: the drain warps have read them
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* lsum = reinterpret_cast<float*>(smem + C::XCH_OFF);  // DRAIN: [2][128]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_items = p.n_tiles * p.heads;

  // Geometry of work item `it`: key tiles first of the shared prefix
  // (n_pre, unmasked but for its end), then of the sequence itself (causal,
  // or all of them).
  struct Item {
    AttnTile tile;
    int head, kvh, n_pre, n_kv;
  };
  auto item_at = [&](int it) {
    Item w;
    w.tile = p.tiles[it / p.heads];
    w.head = it - (it / p.heads) * p.heads;
    w.kvh = w.head / p.group;
    const int kv_end = CAUSAL ? min(w.tile.seq_len, w.tile.q_start + C::BM) : w.tile.seq_len;
    w.n_pre = (w.tile.pre_len + C::BN - 1) / C::BN;
    w.n_kv = w.n_pre + (kv_end + C::BN - 1) / C::BN;
    return w;
  };
  auto key_row = [&](const Item& w, int j) {
    return j < w.n_pre ? w.tile.pre_start + j * C::BN : w.tile.seq_start + (j - w.n_pre) * C::BN;
  };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], 4 * SPR);
    }
    mbar_init(pv_done, 1);
    mbar_init(o_final, 1);
    mbar_init(q_free, 1);
    mbar_init(o_free, 4 * SPR);
    mbar_init(mma_drained, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&l_full[i], C::BM);   // every softmax thread
      mbar_init(&l_empty[i], C::BM);  // every drain thread
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
  // Launched with programmatic stream serialization: the set-up above ran
  // under the previous kernel's tail; its results are needed from here on.
  pdl_wait_prior();
  pdl_trigger_next();

  // Key tiles are counted over all of this CTA's items (g): K / V stage and
  // S / P buffer g & 1, phase (g >> 1) & 1.  Items are counted by qi.
  if (warp < C::SOFTMAX_WARP0) {
    // Producers and the MMA issuer (with the drain warps, warp 3 has no role).
    if (warp == 0) {
      if (lane == 0) {
        tma_prefetch_desc(&tm_qkv64);
        uint32_t g = 0, qi = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++qi) {
          const Item w = item_at(it);
          if (qi > 0 && !mbar_wait(q_free, (qi - 1) & 1, abort_flag, p.err, kErrTimeoutEmpty)) break;
          const int qx = p.q_col0 + w.head * C::HD, kx = p.k_col0 + w.kvh * C::HD;
          const int qy = w.tile.seq_start + w.tile.q_start;
          mbar_arrive_expect_tx(q_full, C::Q_BYTES);
  #pragma unroll
          for (int a = 0; a < C::ATOMS; ++a) {
            tma_load_2d(smem + C::Q_OFF + a * C::Q_ATOM, &tm_qkv64, q_full, qx + 64 * a, qy);
            tma_load_2d(smem + C::Q_OFF + a * C::Q_ATOM + C::Q_ATOM / 2, &tm_qkv64, q_full, qx + 64 * a, qy + 64);
          }
          bool ok = true;
          for (int j = 0; j < w.n_kv; ++j, ++g) {
            const int s = g & 1;
            if (!mbar_wait(&k_empty[s], ((g >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&k_full[s], C::KV_BYTES);
  #pragma unroll
            for (int a = 0; a < C::ATOMS; ++a)
              tma_load_2d(smem + C::K_OFF + s * C::KV_BYTES + a * C::KV_ATOM, &tm_qkv64, &k_full[s], kx + 64 * a,
                          key_row(w, j));
          }
          if (!ok) break;
        }
      }
    } else if (warp == 2) {
      if (lane == 0) {
        uint32_t g = 0;
        for (int it = blockIdx.x; it < n_items; it += gridDim.x) {
          const Item w = item_at(it);
          const int vx = p.v_col0 + w.kvh * C::HD;
          bool ok = true;
          for (int j = 0; j < w.n_kv; ++j, ++g) {
            const int s = g & 1;
            if (!mbar_wait(&v_empty[s], ((g >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutEmpty)) {
              ok = false;
              break;
            }
            mbar_arrive_expect_tx(&v_full[s], C::KV_BYTES);
  #pragma unroll
            for (int a = 0; a < C::ATOMS; ++a)
              tma_load_2d(smem + C::V_OFF + s * C::KV_BYTES + a * C::KV_ATOM, &tm_qkv64, &v_full[s], vx + 64 * a,
                          key_row(w, j));
          }
          if (!ok) break;
        }
      }
    } else if (warp == 1) {
      if (lane == 0) {
        const uint32_t q_addr = smem_u32(smem + C::Q_OFF);
        // S(g) = Q K_g^T into S/P buffer g & 1; releases K stage g & 1 when done.
        auto issue_s = [&](uint32_t g) {
          const int b = g & 1;
          const uint32_t k_addr = smem_u32(smem + C::K_OFF + b * C::KV_BYTES);
  #pragma unroll
          for (int kk = 0; kk < HD / 16; ++kk) {
            umma_f16kind(tmem + b * 64, sw128_kmajor_desc(q_addr + (kk >> 2) * C::Q_ATOM + (kk & 3) * 32),
                         sw128_kmajor_desc(k_addr + (kk >> 2) * C::KV_ATOM + (kk & 3) * 32), IDESC_S,
                         kk != 0 ? 1u : 0u);
          }
          umma_commit(&s_full[b]);
          umma_commit(&k_empty[b]);
        };
        uint32_t g = 0, qi = 0;
        bool ok = true;
        for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++qi) {
          const Item w = item_at(it);
          ok = mbar_wait(q_full, qi & 1, abort_flag, p.err, kErrTimeoutFull);
          for (int j = 0; ok && j < 2 && j < w.n_kv; ++j) {
            if (!mbar_wait(&k_full[(g + j) & 1], ((g + j) >> 1) & 1, abort_flag, p.err, kErrTimeoutFull)) {
              ok = false;
              break;
            }
            tc_fence_after();
            issue_s(g + j);
          }
          if (ok && w.n_kv <= 2) umma_commit(q_free);  // every S of the item issued: Q may be replaced
          for (int j = 0; ok && j < w.n_kv; ++j) {
            const uint32_t gj = g + j;
            const int b = gj & 1, ph = (gj >> 1) & 1;
            if (!mbar_wait(&v_full[b], ph, abort_flag, p.err, kErrTimeoutFull) ||
                !mbar_wait(&p_full[b], ph, abort_flag, p.err, kErrTimeoutFull) ||
                (j == 0 && qi > 0 && !mbar_wait(o_free, (qi - 1) & 1, abort_flag, p.err, kErrTimeoutAccEmpty))) {
              ok = false;
              break;
            }
            tc_fence_after();
            // O += P(j) V(j): A = P from TMEM (8 columns per 16 keys), B = V
            // MN-major (64-dim atoms KV_ATOM apart), K advances 16 key rows = 2 KB.
            const uint32_t v_addr = smem_u32(smem + C::V_OFF + b * C::KV_BYTES);
  #pragma unroll
            for (int kk = 0; kk < 4; ++kk)
              umma_f16kind_ts(tmem + 128, tmem + b * 64 + kk * 8, sw128_mnmajor_desc(v_addr + kk * 2048, C::KV_ATOM),
                              IDESC_PV, (j > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&v_empty[b]);
            umma_commit(pv_done);
            if (j + 1 == w.n_kv) umma_commit(o_final);
            // S(j + 2) overwrites P(j) in TMEM; MMAs of one thread run in order.
            if (j + 2 < w.n_kv) {
              if (!mbar_wait(&k_full[b], ((gj + 2) >> 1) & 1, abort_flag, p.err, kErrTimeoutFull)) {
                ok = false;
                break;
              }
              tc_fence_after();
              issue_s(gj + 2);
              if (j + 3 == w.n_kv) umma_commit(q_free);
            }
          }
          g += w.n_kv;
        }
        if (!ok) {
          // Aborted: the MMAs already issued finish (bounded) before the CTA
          // frees the tensor memory they write.
          umma_commit(mma_drained);
          mbar_wait_own(mma_drained, 0, 0);
        }
      }
    }
  } else if (warp < C::SOFTMAX_WARP0 + 4 * SPR) {
    // Softmax warps (3..6, or 4..7 with the drain warps, or 3..10 with two
    // per row): query row r of the tile (TMEM lane quarter warp & 3); with
    // SPR = 2 the warp's `part` (0 or 1) selects key columns [32 part, +32) of
    // each S tile and O columns [part HD/2, +HD/2).
    constexpr int KC = C::BN / SPR;  // scores per thread and key tile
    constexpr int OC = HD / SPR;     // O columns per thread
    const int quarter = warp & 3;
    const int part = SPR == 2 ? (warp - C::SOFTMAX_WARP0) >> 2 : 0;
    const int r = quarter * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const uint32_t o_tm = tmem + lane_base + 128 + part * OC;
    float* xch = reinterpret_cast<float*>(smem + C::XCH_OFF);  // SPR = 2 exchange
    const int bar_id = 2 + quarter;
    uint32_t g = 0, qi = 0;
    bool ok = true;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++qi) {
      const Item w = item_at(it);
      const AttnTile& tile = w.tile;
      const int q_row = tile.q_start + r;  // row inside the sequence
      float m_run = -INFINITY, l_run = 0.0f;
      for (int j = 0; j < w.n_kv; ++j) {
        const uint32_t gj = g + j;
        const int b = gj & 1;
        const uint32_t s_tm = tmem + lane_base + b * 64;
        const bool in_pre = j < w.n_pre;
        const int kv0 = (in_pre ? j : j - w.n_pre) * C::BN + part * KC;  // first key of this thread's columns
        const int seg_len = in_pre ? tile.pre_len : tile.seq_len;
        const int causal_row = (in_pre || !CAUSAL) ? 0x7fffffff : q_row;
        bool got = mbar_wait(&s_full[b], (gj >> 1) & 1, abort_flag, p.err, kErrTimeoutAccFull);
        float mx = -INFINITY;
        uint32_t sr[KC];
        if (got) {
          tc_fence_after();
          const bool need_mask = kv0 + KC > seg_len || (CAUSAL && !in_pre && kv0 + KC > tile.q_start);
#pragma unroll
          for (int c = 0; c < KC / 32; ++c) tmem_ld32_nowait(s_tm + part * KC + c * 32, sr + c * 32);
          tmem_wait_ld();
          if (need_mask) {
#pragma unroll
            for (int i = 0; i < KC; ++i) {
              const int kv = kv0 + i;
              if (kv >= seg_len || kv > causal_row) sr[i] = __float_as_uint(-INFINITY);
              mx = fmaxf(mx, __uint_as_float(sr[i]));
            }
          } else {
#pragma unroll
            for (int i = 0; i < KC; ++i) mx = fmaxf(mx, __uint_as_float(sr[i]));
          }
        }
        if constexpr (SPR == 2) {
          // The pair agrees on going on (a barrier must not wait for a warp
          // that left) and swaps its halves' maxima; the exchange slot
          // alternates with the tile so a partner still reading never sees
          // the next tile's value.
          float* slot = xch + (((gj & 1) * 4 + quarter) * 32 + lane) * 2;
          slot[part] = mx;
          got = pair_bar_and(bar_id, __all_sync(0xffffffffu, got));
          mx = fmaxf(mx, slot[part ^ 1]);
        }
        if (!got) {
          ok = false;
          break;
        }
        const float m_tile = mx * p.scale_log2;
        const bool raise = m_tile > m_run + C::RESCALE_THRESHOLD;
        const bool warp_raise = __any_sync(0xffffffffu, raise);
        const float m_new = raise ? m_tile : m_run;
        const float alpha = raise ? fast_exp2(m_run - m_new) : 1.0f;
        float rs = 0.0f;
#pragma unroll
        for (int c = 0; c < KC / 32; ++c) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const float e0 = fast_exp2(__uint_as_float(sr[c * 32 + i]) * p.scale_log2 - m_new);
            const float e1 = fast_exp2(__uint_as_float(sr[c * 32 + i + 1]) * p.scale_log2 - m_new);
            rs += e0 + e1;
            pk[i >> 1] = Elem<T>::pack2(e0, e1);
          }
          tmem_st16(s_tm + part * (KC / 2) + c * 16, pk);
        }
        // A raised max rescales the O rows accumulated so far, once P(j - 1) V
        // has landed (P(j) V cannot start before this warp's p_full arrival).
        if (warp_raise && j > 0) {
          bool done = mbar_wait(pv_done, (gj - 1) & 1, abort_flag, p.err, kErrTimeoutAccFull);
          if constexpr (SPR == 2) done = pair_bar_and(bar_id, __all_sync(0xffffffffu, done));
          if (!done) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll 1
          for (int c = 0; c < OC / 32; ++c) {
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
        if (lane == 0) mbar_arrive(&p_full[b]);
        l_run = l_run * alpha + rs;
        m_run = m_new;
      }
      if (!ok) break;
      if constexpr (C::DRAIN) {
        // The row sums go to the drain warps, which wait for the item's last
        // P V and store O themselves; these warps go on to the next item.
        if (!mbar_wait(&l_empty[qi & 1], ((qi >> 1) & 1) ^ 1, abort_flag, p.err, kErrTimeoutEmpty)) {
          ok = false;
          break;
        }
        lsum[(qi & 1) * C::BM + r] = l_run;
        mbar_arrive(&l_full[qi & 1]);
        g += w.n_kv;
        continue;
      }
      bool fin = mbar_wait(o_final, qi & 1, abort_flag, p.err, kErrTimeoutAccFull);
      float l_tot = l_run;
      if constexpr (SPR == 2) {
        // Region 2: the next use of this slot is the next item's sum, with at
        // least one max exchange (a barrier) in between.
        float* slot = xch + ((2 * 4 + quarter) * 32 + lane) * 2;
        slot[part] = l_run;
        fin = pair_bar_and(bar_id, __all_sync(0xffffffffu, fin));
        l_tot += slot[part ^ 1];
      }
      if (!fin) {
        ok = false;
        break;
      }
      tc_fence_after();
      attn_head_store_o<HD, OC, T>(p, tile, w.head, q_row, part, o_tm, l_tot);
      // O may now be overwritten by the next item's first P V.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
      g += w.n_kv;
    }
  } else if constexpr (C::DRAIN) {
    // Drain warps 8..11: row r of each item (TMEM lane quarter warp & 3).
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const uint32_t o_tm = tmem + (static_cast<uint32_t>(quarter * 32) << 16) + 128;
    uint32_t qi = 0;
    for (int it = blockIdx.x; it < n_items; it += gridDim.x, ++qi) {
      const Item w = item_at(it);
      if (!mbar_wait(&l_full[qi & 1], (qi >> 1) & 1, abort_flag, p.err, kErrTimeoutAccFull) ||
          !mbar_wait(o_final, qi & 1, abort_flag, p.err, kErrTimeoutAccFull))
        break;
      tc_fence_after();
      const float l_tot = lsum[(qi & 1) * C::BM + r];
      mbar_arrive(&l_empty[qi & 1]);
      attn_head_store_o<HD, HD, T>(p, w.tile, w.head, w.tile.q_start + r, 0, o_tm, l_tot);
      // O may now be overwritten by the next item's first P V.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(o_free);
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
