// Kernel-level C entry points (include/vdexec_kernels.h): single kernels on
// caller-owned device buffers.  Included at the end of vdexec.cu so they share
// its tensor-map and launch helpers.
#pragma once

#include "vdexec_kernels.h"

namespace vd {

// A device error word per GPU for the kernel-level calls.
static int* ops_error_word(int device) {
  static std::mutex mu;
  static int* words[64] = {};
  std::lock_guard<std::mutex> lock(mu);
  if (device < 0 || device >= 64) fail(VD_EINVAL, "device index out of range");
  if (!words[device]) {
    cuda_check(cudaMalloc(&words[device], sizeof(int)), "error word");
    cuda_check(cudaMemset(words[device], 0, sizeof(int)), "error word");
  }
  return words[device];
}

static void ops_finish(cudaStream_t s, int* word) {
  cuda_check(cudaGetLastError(), "kernel launch");
  int e = 0;
  cuda_check(cudaMemcpyAsync(&e, word, sizeof(int), cudaMemcpyDeviceToHost, s), "read error word");
  cuda_check(cudaStreamSynchronize(s), "synchronize");
  if (e != 0) {
    cuda_check(cudaMemset(word, 0, sizeof(int)), "clear error word");
    fail(VD_ECUDA, "kernel reported device error " + std::to_string(e));
  }
}

static void ops_attrs_once() {
  static std::once_flag once[64];
  int dev = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  std::call_once(once[dev & 63], [] { init_kernel_attrs(); });
}

// 256-wide tiles run on CTA pairs (two-CTA kernel, W maps with 128-row boxes)
// when the device can co-schedule them; other shapes on one CTA per tile.
template <int EPI, class T>
static void ops_gemm_launch_t(const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& w_half,
                              const CUtensorMap& c, int bn, int M, int N, int K, const EpiParams& ep, cudaStream_t s,
                              int* word, int sms) {
  const int tiles = ((M + 127) / 128) * (N / bn);
  const int grid = std::min(tiles, sms);
  GemmShape shape{M, N, K, GemmConfig<256>::GROUP_M, 0, 0, 1, nullptr, nullptr, 0};
  const int pairs = bn == 256 ? gemm2_max_pairs(sms) : 0;
  if (pairs > 0) shape.group_m = Gemm2Config::GROUP_M;
  if (pairs > 0) {
    const int grid2 = 2 * std::min(((M + 255) / 256) * (N / 256), pairs);
    gemm2_tcgen05_kernel<EPI, T><<<grid2, Gemm2Config::THREADS, Gemm2Config::SMEM_BYTES, s>>>(a, w_half, c, c, shape,
                                                                                             ep, word);
  } else if (bn == 256)
    gemm_tcgen05_kernel<256, EPI, T><<<grid, GemmConfig<256>::THREADS, GemmConfig<256>::SMEM_BYTES, s>>>(a, w, c, c, shape, ep, word);
  else if constexpr (EPI != kEpiGated)
    gemm_tcgen05_kernel<128, EPI, T><<<grid, GemmConfig<128>::THREADS, GemmConfig<128>::SMEM_BYTES, s>>>(a, w, c, c, shape, ep, word);
  else
    fail(VD_EINVAL, "gated GEMM needs N % 256 == 0");
}

template <int EPI>
static void ops_gemm_launch(bool f16, const CUtensorMap& a, const CUtensorMap& w, const CUtensorMap& w_half,
                            const CUtensorMap& c, int bn, int M, int N, int K, const EpiParams& ep, cudaStream_t s,
                            int* word, int sms) {
  if (f16) ops_gemm_launch_t<EPI, __half>(a, w, w_half, c, bn, M, N, K, ep, s, word, sms);
  else ops_gemm_launch_t<EPI, __nv_bfloat16>(a, w, w_half, c, bn, M, N, K, ep, s, word, sms);
}

static bool ops_dtype(int dtype) {
  if (dtype != VDK_FP16 && dtype != VDK_BF16) fail(VD_EINVAL, "dtype must be VDK_FP16 or VDK_BF16");
  return dtype == VDK_FP16;
}

static int device_sms() {
  int dev = 0, sms = 0;
  cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
  cuda_check(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev), "SM count");
  return sms;
}

}  // namespace vd

extern "C" VD_API int vdk_gemm(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int dtype, int epi, int act,
                               const float* bias, void* out, int64_t ld_out, void* stream, char* err, size_t errlen) {
  return guarded(nullptr, err, errlen, [&] {
    if (M < 1 || N % 128 != 0 || K % 64 != 0 || K < 64) fail(VD_EINVAL, "need M >= 1, N % 128 == 0, K % 64 == 0");
    if (epi == kEpiGated && N % 256 != 0) fail(VD_EINVAL, "gated GEMM needs N % 256 == 0");
    if (epi < 0 || epi > kEpiGated) fail(VD_EINVAL, "unknown epilogue (use vdk_gemm_qkrope for QK-RoPE)");
    if (ld_out < (epi == kEpiGated ? N / 2 : N)) fail(VD_EINVAL, "ld_out smaller than the output width");
    if (!A || !W || !out) fail(VD_EINVAL, "null buffer");
    const bool f16 = ops_dtype(dtype);
    ops_attrs_once();
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    int* word = ops_error_word(dev);
    const int bn = (N % 256 == 0) ? 256 : 128;
    const CUtensorMap a = make_map(A, M, K, 128, f16);
    const CUtensorMap w = make_map(W, N, K, bn, f16);
    const CUtensorMap w_half = make_map(W, N, K, 128, f16);
    EpiParams ep = epi_params_for(bias, act);
    const CUtensorMap c = make_out_map(out, M, ld_out, epi == kEpiResidual, f16);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int sms = device_sms();
    const int m = static_cast<int>(M), n = static_cast<int>(N), k = static_cast<int>(K);
    switch (epi) {
      case kEpiStore: ops_gemm_launch<kEpiStore>(f16, a, w, w_half, c, bn, m, n, k, ep, s, word, sms); break;
      case kEpiResidual: ops_gemm_launch<kEpiResidual>(f16, a, w, w_half, c, bn, m, n, k, ep, s, word, sms); break;
      case kEpiGated: ops_gemm_launch<kEpiGated>(f16, a, w, w_half, c, bn, m, n, k, ep, s, word, sms); break;
    }
    ops_finish(s, word);
  });
}

extern "C" VD_API int vdk_gemm_qkrope(const void* A, const void* W, int64_t M, int64_t N, int64_t K, int dtype,
                                      const float* bias,
                                      const float* q_norm, const float* k_norm, int q_cols, int k_cols, int head_dim,
                                      int plus_one, float eps, const int32_t* positions, double theta, int max_pos,
                                      void* out, int64_t ld_out, void* stream, char* err, size_t errlen) {
  return guarded(nullptr, err, errlen, [&] {
    if (M < 1 || N % 128 != 0 || K % 64 != 0) fail(VD_EINVAL, "need N % 128 == 0, K % 64 == 0");
    if (head_dim != 128 && head_dim != 256) fail(VD_EINVAL, "head_dim must be 128 or 256");
    if (ld_out < N || !A || !W || !out || !positions) fail(VD_EINVAL, "bad output stride or null buffer");
    if (max_pos < 1) fail(VD_EINVAL, "max_pos must be positive");
    const bool f16 = ops_dtype(dtype);
    int bn = 256;
    if (head_dim == 128 && (q_cols % 256 != 0 || k_cols % 256 != 0 || N % 256 != 0)) bn = 128;
    if (head_dim == 256 && (q_cols % 256 != 0 || k_cols % 256 != 0 || N % 256 != 0))
      fail(VD_EINVAL, "head_dim 256 needs 256-aligned q/k/v blocks");
    ops_attrs_once();
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    int* word = ops_error_word(dev);
    // Rotary table for this call.
    const int half = head_dim / 2;
    std::vector<float2> tab(static_cast<size_t>(max_pos) * half);
    for (int64_t p = 0; p < max_pos; ++p)
      for (int i = 0; i < half; ++i) {
        const float inv = 1.0f / std::pow(static_cast<float>(theta), static_cast<float>(2 * i) / head_dim);
        const float a = static_cast<float>(p) * inv;
        tab[p * half + i] = make_float2(static_cast<float>(std::cos(static_cast<double>(a))),
                                        static_cast<float>(std::sin(static_cast<double>(a))));
      }
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    float2* rope = nullptr;
    cuda_check(cudaMalloc(&rope, tab.size() * sizeof(float2)), "rope table");
    std::unique_ptr<float2, decltype(&cudaFree)> guard(rope, &cudaFree);
    cuda_check(cudaMemcpy(rope, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice), "rope table");
    const CUtensorMap a = make_map(A, M, K, 128, f16);
    const CUtensorMap w = make_map(W, N, K, bn, f16);
    const CUtensorMap w_half = make_map(W, N, K, 128, f16);
    EpiParams ep = epi_params_for(bias, kActNone);
    const CUtensorMap c = make_out_map(out, M, ld_out, false, f16);
    ep.q_norm = q_norm;
    ep.k_norm = k_norm;
    ep.q_cols = q_cols;
    ep.k_cols = k_cols;
    ep.head_dim = head_dim;
    ep.plus_one = plus_one;
    ep.eps = eps;
    ep.positions = positions;
    ep.rope = rope;
    ops_gemm_launch<kEpiQKRope>(f16, a, w, w_half, c, bn, static_cast<int>(M), static_cast<int>(N), static_cast<int>(K), ep, s, word,
                                device_sms());
    ops_finish(s, word);
  });
}

extern "C" VD_API int vdk_attention(const void* qkv, int64_t ld_qkv, int64_t q_col0, int64_t k_col0, int64_t v_col0,
                                    int heads, int kv_heads, int head_dim, int dtype, int causal,
                                    const int32_t* cu_seqlens_host, int64_t nseq, void* out, int64_t ld_out,
                                    void* stream, char* err, size_t errlen) {
  return guarded(nullptr, err, errlen, [&] {
    if (heads < 1 || kv_heads < 1 || heads % kv_heads != 0) fail(VD_EINVAL, "heads must be a multiple of kv_heads");
    if (nseq < 1 || !cu_seqlens_host) fail(VD_EINVAL, "need at least one sequence");
    const bool f16 = ops_dtype(dtype);
    ops_attrs_once();
    std::vector<AttnTile> tiles;
    for (int64_t i = 0; i < nseq; ++i) {
      const int start = cu_seqlens_host[i], len = cu_seqlens_host[i + 1] - start;
      if (len < 0) fail(VD_EINVAL, "cu_seqlens must be non-decreasing");
      for (int q = 0; q < len; q += 64) tiles.push_back(AttnTile{start, len, q, 0, 0, {0, 0, 0}});
    }
    if (tiles.empty()) return;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    AttnTile* d_tiles = nullptr;
    cuda_check(cudaMalloc(&d_tiles, tiles.size() * sizeof(AttnTile)), "tile table");
    std::unique_ptr<AttnTile, decltype(&cudaFree)> guard(d_tiles, &cudaFree);
    cuda_check(cudaMemcpy(d_tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice), "tiles");
    AttnParams p{};
    p.gate_col0 = -1;
    p.qkv = qkv;
    p.ld_qkv = static_cast<int>(ld_qkv);
    p.q_col0 = static_cast<int>(q_col0);
    p.k_col0 = static_cast<int>(k_col0);
    p.v_col0 = static_cast<int>(v_col0);
    p.out = out;
    p.ld_out = static_cast<int>(ld_out);
    p.tiles = d_tiles;
    p.group = heads / kv_heads;
    p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)) * 1.4426950408889634);
    dim3 grid(static_cast<unsigned>(tiles.size()), heads);
    auto run = [&](auto tag) {
      using T = decltype(tag);
      if (head_dim == 64 && !causal)
        attention_varlen_kernel<64, false, T><<<grid, 128, AttnConfig<64>::SMEM_BYTES, s>>>(p);
      else if (head_dim == 128 && causal)
        attention_varlen_kernel<128, true, T><<<grid, 128, AttnConfig<128>::SMEM_BYTES, s>>>(p);
      else if (head_dim == 256 && causal)
        attention_varlen_kernel<256, true, T><<<grid, 128, AttnConfig<256>::SMEM_BYTES, s>>>(p);
      else
        fail(VD_EINVAL, "supported: head_dim 64 bidirectional, 128 / 256 causal");
    };
    if (f16) run(__half());
    else run(__nv_bfloat16());
    cuda_check(cudaGetLastError(), "attention launch");
    cuda_check(cudaStreamSynchronize(s), "synchronize");
  });
}

extern "C" VD_API int vdk_attention_tc(const void* qkv, int64_t ld_qkv, int64_t q_col0, int64_t k_col0,
                                       int64_t v_col0, int heads, int kv_heads, int head_dim, int dtype, int causal,
                                       const int32_t* cu_seqlens_host, int64_t nseq, void* out, int64_t ld_out,
                                       void* stream, char* err, size_t errlen) {
  return guarded(nullptr, err, errlen, [&] {
    if (!((head_dim == 128 || head_dim == 256) && causal) && !(head_dim == 64 && !causal))
      fail(VD_EINVAL, "the tcgen05 attention kernels are causal with head_dim 128 or 256, or bidirectional with 64");
    if (heads < 1 || kv_heads < 1 || heads % kv_heads != 0) fail(VD_EINVAL, "heads must be a multiple of kv_heads");
    if (nseq < 1 || !cu_seqlens_host || !qkv || !out) fail(VD_EINVAL, "need at least one sequence and buffers");
    if (ld_qkv % 8 != 0 || q_col0 % 8 != 0 || k_col0 % 8 != 0 || v_col0 % 8 != 0 || ld_out % 8 != 0)
      fail(VD_EINVAL, "qkv / out strides and column offsets must be multiples of 8 elements");
    const bool f16 = ops_dtype(dtype);
    ops_attrs_once();
    int dev = 0;
    cuda_check(cudaGetDevice(&dev), "cudaGetDevice");
    int* word = ops_error_word(dev);
    std::vector<AttnTile> tiles;
    for (int64_t i = 0; i < nseq; ++i) {
      const int start = cu_seqlens_host[i], len = cu_seqlens_host[i + 1] - start;
      if (len < 0) fail(VD_EINVAL, "cu_seqlens must be non-decreasing");
      for (int q = 0; q < len; q += 128) tiles.push_back(AttnTile{start, len, q, 0, 0, {0, 0, 0}});
    }
    if (tiles.empty()) return;
    // Most work first (a causal tile's keys end at its last query row), so the
    // persistent CTAs end together.
    std::stable_sort(tiles.begin(), tiles.end(), [causal](const AttnTile& a, const AttnTile& b) {
      const int wa = causal ? std::min(a.seq_len, a.q_start + 128) : a.seq_len;
      const int wb = causal ? std::min(b.seq_len, b.q_start + 128) : b.seq_len;
      return wa > wb;
    });
    const int64_t T = cu_seqlens_host[nseq];
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    AttnTile* d_tiles = nullptr;
    cuda_check(cudaMalloc(&d_tiles, tiles.size() * sizeof(AttnTile)), "tile table");
    std::unique_ptr<AttnTile, decltype(&cudaFree)> guard(d_tiles, &cudaFree);
    cuda_check(cudaMemcpy(d_tiles, tiles.data(), tiles.size() * sizeof(AttnTile), cudaMemcpyHostToDevice), "tiles");
    const CUtensorMap map64 = make_map(qkv, T, ld_qkv, 64, f16);
    AttnTcHeadParams p;
    p.out = out;
    p.ld_out = static_cast<int>(ld_out);
    p.qkv = qkv;
    p.ld_qkv = static_cast<int>(ld_qkv);
    p.q_col0 = static_cast<int>(q_col0);
    p.k_col0 = static_cast<int>(k_col0);
    p.v_col0 = static_cast<int>(v_col0);
    p.gate_col0 = -1;
    p.tiles = d_tiles;
    p.n_tiles = static_cast<int>(tiles.size());
    p.heads = heads;
    p.group = heads / kv_heads;
    p.scale_log2 = static_cast<float>(1.0 / std::sqrt(static_cast<double>(head_dim)) * 1.4426950408889634);
    p.err = word;
    // Persistent: as many CTAs as run at once (two per SM; one at head_dim 256).
    const int items = p.n_tiles * heads;
    const dim3 grid(static_cast<unsigned>(std::min(items, (head_dim == 256 ? 1 : 2) * device_sms())));
    if (head_dim == 64 && f16)
      attention_tc_head_kernel<64, __half, false>
          <<<grid, AttnTcHeadConfig<64>::THREADS, AttnTcHeadConfig<64>::SMEM_BYTES, s>>>(map64, p);
    else if (head_dim == 64)
      attention_tc_head_kernel<64, __nv_bfloat16, false>
          <<<grid, AttnTcHeadConfig<64>::THREADS, AttnTcHeadConfig<64>::SMEM_BYTES, s>>>(map64, p);
    else if (head_dim == 256 && f16)
      attention_tc_head_kernel<256, __half>
          <<<grid, AttnTcHeadConfig<256>::THREADS, AttnTcHeadConfig<256>::SMEM_BYTES, s>>>(map64, p);
    else if (head_dim == 256)
      attention_tc_head_kernel<256, __nv_bfloat16>
          <<<grid, AttnTcHeadConfig<256>::THREADS, AttnTcHeadConfig<256>::SMEM_BYTES, s>>>(map64, p);
    else if (f16)
      attention_tc_head_kernel<128, __half>
          <<<grid, AttnTcHeadConfig<128>::THREADS, AttnTcHeadConfig<128>::SMEM_BYTES, s>>>(map64, p);
    else
      attention_tc_head_kernel<128, __nv_bfloat16>
          <<<grid, AttnTcHeadConfig<128>::THREADS, AttnTcHeadConfig<128>::SMEM_BYTES, s>>>(map64, p);
    ops_finish(s, word);
  });
}
