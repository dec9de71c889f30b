// Checkpoint tensors (safetensors BF16 / F16 / F32) converted on the device
// into the executor's layouts: 16-bit GEMM weights with the same row
// placement the synthetic generator uses (fused QKV blocks, gate/up
// interleave), fp32 gains / biases / label rows.
#pragma once

#include "common.cuh"
#include "synth.cuh"

namespace vd {

// Source element types, numbered like the checkpoint reader's StDtype.
__device__ __forceinline__ float load_ckpt(const void* __restrict__ src, int dtype, int64_t i) {
  if (dtype == 0) return __bfloat162float(static_cast<const __nv_bfloat16*>(src)[i]);
  if (dtype == 1) return __half2float(static_cast<const __half*>(src)[i]);
  return static_cast<const float*>(src)[i];
}

// `src` holds rows [r0, r0 + n_rows) of a [*, cols] source tensor; source row
// r lands at destination row dst_row(r, ...), as in synth_rows_kernel.  Values
// round to T to nearest-even; a bf16 source converts to fp16 exactly for
// magnitudes >= 2^-14.
template <class T>
__global__ void convert_rows_kernel(T* __restrict__ dst, const void* __restrict__ src, int src_dtype, int64_t r0,
                                    int64_t n_rows, int64_t cols, RowPlace place) {
  const int64_t total = n_rows * cols;
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = r0 + i / cols, c = i % cols;
    const int64_t dr = dst_row(r, place);
    dst[dr * cols + c] = Elem<T>::from(load_ckpt(src, src_dtype, i));
  }
}

__global__ void convert_f32_kernel(float* __restrict__ dst, const void* __restrict__ src, int src_dtype, int64_t n) {
  for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x)
    dst[i] = load_ckpt(src, src_dtype, i);
}

}  // namespace vd
