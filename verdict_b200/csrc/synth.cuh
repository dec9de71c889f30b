// On-GPU generation of the synthetic checkpoints (random-init weights from a
// seed).  Element i of a tensor is a pure function of (tensor base, i); the
// host generator in verdict_b200/synth.py evaluates the same function, and both
// round the same fp32 value to bf16 (ties to even), so the CUDA forward and the
// CPU oracle read bit-identical weights.
#pragma once

#include "common.cuh"

namespace vd {

__device__ __forceinline__ uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// fp32 value before bf16 rounding; every operation rounds exactly once (no FMA
// contraction) so the host generator reproduces it bit for bit.
__device__ __forceinline__ __nv_bfloat16 synth_bf16(uint64_t base, uint64_t i, float scale, float offset) {
  const uint64_t z = splitmix64(base + i);
  const float u = static_cast<float>(static_cast<uint32_t>(z >> 40)) * 5.9604644775390625e-08f;  // 2^-24
  float v = __fmul_rn(__fsub_rn(__fmul_rn(u, 2.0f), 1.0f), scale);
  v = __fadd_rn(v, offset);
  return __float2bfloat16_rn(v);
}

// Where the rows of a source tensor land in a fused weight matrix.  Source
// row r goes to (r / group) * stride + (r % group) + off: group = n_rows with
// stride 0 is a plain copy; group 128 with stride 256 interleaves gate/up
// blocks for the fused gated-MLP GEMM.  With alt_off >= 0 the groups alternate
// between two blocks: group b goes to (b / 2) * stride + (b odd ? alt_off :
// off) — the per-head [query, gate] rows of a gated attention's q_proj split
// into a query block and a gate block.  With part_rows > 0 the source is
// parts of part_rows rows, part p placed as above plus p * part_off — the
// [input; gate] halves of a GeGLU Wi interleaved into gate/up blocks.
struct RowPlace {
  int64_t group = 1, stride = 0, off = 0, alt_off = -1, part_rows = 0, part_off = 0;
};

__host__ __device__ __forceinline__ int64_t dst_row(int64_t r, const RowPlace& p) {
  int64_t extra = 0;
  if (p.part_rows > 0) {
    extra = (r / p.part_rows) * p.part_off;
    r %= p.part_rows;
  }
  if (p.alt_off < 0) return (r / p.group) * p.stride + (r % p.group) + p.off + extra;
  const int64_t b = r / p.group;
  return (b >> 1) * p.stride + ((b & 1) ? p.alt_off : p.off) + (r % p.group) + extra;
}

// Rows r of a [n_rows, cols] source tensor land at dst_row(r) of a row-major
// [*, cols] matrix of 16-bit T.  The checkpoint value is bf16; T = fp16 holds
// it exactly when its magnitude is >= 2^-14 (below that it rounds to the fp16
// subnormal grid, an absolute change of at most 2^-25).
template <class T>
__global__ void synth_rows_kernel(T* __restrict__ dst, int64_t n_rows, int64_t cols, uint64_t base, float scale,
                                  float offset, RowPlace place) {
  const int64_t total = n_rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const int64_t dr = dst_row(r, place);
    dst[dr * cols + c] = Elem<T>::from(__bfloat162float(synth_bf16(base, static_cast<uint64_t>(i), scale, offset)));
  }
}

// A 1-D tensor as fp32 (bf16-valued), e.g. norm gains and biases.
__global__ void synth_f32_kernel(float* __restrict__ dst, int64_t n, uint64_t base, float scale, float offset) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = __bfloat162float(synth_bf16(base, static_cast<uint64_t>(i), scale, offset));
}

// Selected rows of a [*, cols] tensor as fp32 (the option-label rows of the LM head).
__global__ void synth_rows_gather_f32_kernel(float* __restrict__ dst, const int* __restrict__ rows, int n_rows,
                                             int64_t cols, uint64_t base, float scale, float offset) {
  const int64_t total = static_cast<int64_t>(n_rows) * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i - r * cols;
    const uint64_t src = static_cast<uint64_t>(rows[r]) * static_cast<uint64_t>(cols) + static_cast<uint64_t>(c);
    dst[i] = __bfloat162float(synth_bf16(base, src, scale, offset));
  }
}

}  // namespace vd
