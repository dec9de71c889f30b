/*
 * Fast host evaluation of the synthetic-checkpoint generator (the same function
 * as verdict_b200/synth.py and the CUDA generator): element i of a tensor is
 * bf16_rne(fp32((2u - 1) * scale) + offset), u = top 24 bits of
 * splitmix64(base + i) / 2^24.  TEST INFRASTRUCTURE ONLY: the CPU oracle uses it
 * to build 9B-scale reference weights in seconds.  Compiled with
 * -ffp-contract=off so every float operation rounds once, as on the GPU.
 */
#include <stdint.h>
#include <string.h>

static inline uint64_t splitmix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

static inline float bf16_rne(float x) {
  uint32_t b;
  memcpy(&b, &x, 4);
  b = (b + (((b >> 16) & 1u) + 0x7FFFu)) & 0xFFFF0000u;
  memcpy(&x, &b, 4);
  return x;
}

/* out[r, c] = element rows[r] * cols + c (rows == NULL: r) of the tensor. */
void vd_oracle_gen_rows(float* out, uint64_t base, int64_t n_rows, const int64_t* rows, int64_t cols, float scale,
                        float offset) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < n_rows; ++r) {
    const uint64_t src = (uint64_t)(rows ? rows[r] : r) * (uint64_t)cols;
    float* o = out + r * cols;
    for (int64_t c = 0; c < cols; ++c) {
      const uint64_t z = splitmix64(base + src + (uint64_t)c);
      const float u = (float)(uint32_t)(z >> 40) * 5.9604644775390625e-08f;
      float v = (u * 2.0f - 1.0f) * scale;
      v = v + offset;
      o[c] = bf16_rne(v);
    }
  }
}
