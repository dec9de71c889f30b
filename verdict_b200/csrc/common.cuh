// Shared device helpers for the sm_100a decision-model kernels: bf16 packing,
// mbarrier / TMA / tcgen05 inline-PTX wrappers, and bounded waits.
//
// Every wait on an mbarrier is bounded: after VD_WAIT_TIMEOUT_NS of polling the
// waiting thread records an error code in the kernel's device error word, raises
// the CTA's abort flag and gives up, so a broken pipeline ends the launch with
// an error status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef VD_WAIT_TIMEOUT_NS
#define VD_WAIT_TIMEOUT_NS 2000000000ull  // 2 s
#endif

namespace vd {

// Error codes written to the device error word (first writer wins).
enum DeviceError : int {
  kErrNone = 0,
  kErrTimeoutFull = 1,      // MMA warp waited too long for a TMA stage
  kErrTimeoutEmpty = 2,     // producer waited too long for a free stage
  kErrTimeoutAccFull = 3,   // epilogue waited too long for an accumulator
  kErrTimeoutAccEmpty = 4,  // MMA warp waited too long for a drained accumulator
  kErrTokenRange = 10,      // a token id outside [0, vocab)
  kErrSlotRange = 11,       // a slot / marker position outside its row
  kErrNonFinite = 12,       // inf / NaN in a slot or marker hidden state or an output logit
};

__device__ __forceinline__ void record_error(int* err, int code) {
  if (err) atomicCAS(err, 0, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// The 16-bit element type of activations and projection weights: fp16 (the
// default: 10 mantissa bits, exact for every bf16 checkpoint value >= 2^-14 in
// magnitude) or bf16.  Both feed the tensor cores at the same rate.
template <class T>
struct Elem;

template <>
struct Elem<__half> {
  static constexpr uint32_t kUmmaFormat = 0;  // kind::f16 operand format F16
  __device__ __forceinline__ static uint32_t pack2(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static float2 unpack2(uint32_t v) {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
  __device__ __forceinline__ static __half from(float x) { return __float2half_rn(x); }
  __device__ __forceinline__ static float to(__half x) { return __half2float(x); }
};

template <>
struct Elem<__nv_bfloat16> {
  static constexpr uint32_t kUmmaFormat = 1;  // kind::f16 operand format BF16
  __device__ __forceinline__ static uint32_t pack2(float lo, float hi) { return pack_bf16x2(lo, hi); }
  __device__ __forceinline__ static float2 unpack2(uint32_t v) { return unpack_bf16x2(v); }
  __device__ __forceinline__ static __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
  __device__ __forceinline__ static float to(__nv_bfloat16 x) { return __bfloat162float(x); }
};

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait for the phase with the given parity.  Returns false when the
// CTA was aborted or the wait timed out after limit_ns (the error is then
// recorded); limit_ns = 0 means VD_WAIT_TIMEOUT_NS.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                          int* err, int code, uint64_t limit_ns = 0) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t limit = limit_ns ? limit_ns : VD_WAIT_TIMEOUT_NS;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > limit) {
      *abort_flag = 1;
      record_error(err, code);
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag: an aborting thread uses it to let
// its own asynchronous work (tensor-core ops, copies) finish before the CTA
// frees the resources that work writes to.  False when limit_ns passed first.
__device__ __forceinline__ bool mbar_wait_own(uint64_t* bar, uint32_t parity, uint64_t limit_ns) {
  const uint64_t limit = limit_ns ? limit_ns : VD_WAIT_TIMEOUT_NS;
  const uint64_t t0 = globaltimer();
  while (!mbar_try_wait(bar, parity))
    if (globaltimer() - t0 > limit) return false;
  return true;
}

// ---------------------------------------------------------------------------
// TMA (tiled bulk tensor copies; no cluster multicast on any load in this library)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// 2-D tile load: box origin (x = inner/contiguous coordinate, y = row).
// x must be a multiple of 8 elements for bf16 (16 bytes); callers pass k-block
// offsets that are multiples of 64.
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in tensor memory)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// Programmatic dependent launch.  A kernel launched with programmatic stream
// serialization may start while the kernel before it in the stream is still
// running.  It sets up its barriers and tensor memory, then waits here for
// that kernel's results before it touches global memory; without such a
// predecessor the wait returns at once.  Triggering lets the next kernel do
// the same as soon as SMs free up.
__device__ __forceinline__ void pdl_wait_prior() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16 or bf16 inputs per the
// instruction descriptor, fp32 accumulate).
__device__ __forceinline__ void umma_f16kind(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on an mbarrier once all tcgen05 ops issued so far by this thread completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor for a K-major tile stored with the 128-byte
// swizzle TMA writes: rows of 64 bf16 (128 B), 8-row core groups 1024 B apart.
__device__ __forceinline__ uint64_t sw128_kmajor_desc(uint32_t smem_addr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((smem_addr & 0x3FFFFu) >> 4);  // start address
  d |= static_cast<uint64_t>(1) << 16;                        // leading byte offset (unused, K fits the swizzle)
  d |= static_cast<uint64_t>(1024 >> 4) << 32;                // stride byte offset: 8 rows x 128 B
  d |= static_cast<uint64_t>(1) << 46;                        // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;                        // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor: 16-bit x 16-bit -> fp32, both operands K-major, MxN
// tile; fmt = 0 for fp16 operands, 1 for bf16 (A and B always share the type).
__host__ __device__ constexpr uint32_t umma_idesc_f16kind(int m, int n, uint32_t fmt) {
  return (1u << 4)                                  // D format: f32
         | (fmt << 7)                               // A format
         | (fmt << 10)                              // B format
         | (static_cast<uint32_t>(n >> 3) << 17)    // N / 8
         | (static_cast<uint32_t>(m >> 4) << 24);   // M / 16
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane
// (base lane + t), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
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
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 fp32 values into 32 consecutive columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_st32f(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "f"(v[0]), "f"(v[1]), "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7]), "f"(v[8]), "f"(v[9]),
      "f"(v[10]), "f"(v[11]), "f"(v[12]), "f"(v[13]), "f"(v[14]), "f"(v[15]), "f"(v[16]), "f"(v[17]), "f"(v[18]),
      "f"(v[19]), "f"(v[20]), "f"(v[21]), "f"(v[22]), "f"(v[23]), "f"(v[24]), "f"(v[25]), "f"(v[26]), "f"(v[27]),
      "f"(v[28]), "f"(v[29]), "f"(v[30]), "f"(v[31])
      : "memory");
}

__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// 32 fp32 values -> 32 consecutive 16-bit elements (64 bytes, 16-byte aligned).
template <class T>
__device__ __forceinline__ void store_x32(T* dst, const float (&v)[32]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 w;
    w.x = Elem<T>::pack2(v[q * 8 + 0], v[q * 8 + 1]);
    w.y = Elem<T>::pack2(v[q * 8 + 2], v[q * 8 + 3]);
    w.z = Elem<T>::pack2(v[q * 8 + 4], v[q * 8 + 5]);
    w.w = Elem<T>::pack2(v[q * 8 + 6], v[q * 8 + 7]);
    d[q] = w;
  }
}

// 32 fp32 accumulator columns of this thread's TMEM lane, loads completed.
__device__ __forceinline__ void tmem_load_f32x32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
#pragma unroll
  for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
}

// ---------------------------------------------------------------------------
// Legacy warp-level MMA helpers (attention v1): ldmatrix + mma.sync m16n8k16.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
template <class T>
__device__ __forceinline__ void mma_16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (Elem<T>::kUmmaFormat == 1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool pred) {
  const int n = pred ? 16 : 0;  // zero-fill when the row is outside the sequence
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(n) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace vd
