// Shared device helpers for the nnzap B200 kernels (sm_100a only).
//
// PTX wrappers for: mbarrier + non-tensor bulk copies (TMA engine, no
// multicast), programmatic dependent launch, and the legacy int8 tensor-core
// MMA (m16n8k32 u8 x s8 -> s32) that the quantized matvec kernels use to
// unpack 1-bit and 4-bit weights with a single LOP3 per four weights.
#pragma once
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "nnzap_b200 kernels are written for sm_100a only"
#endif

namespace nnz {

// Device error flags (bitwise OR into a device int, read by the host).
enum : int {
  ERR_MBAR_TIMEOUT = 1,   // an mbarrier wait gave up (bulk copy never landed)
  ERR_BAD_TOKEN = 2,      // token id >= vocab
  ERR_BAD_POS = 4,        // position >= max_context_length
  ERR_SPIN_TIMEOUT = 8,   // a global flag/counter wait gave up
};

// Iteration cap for every spin in this library.  try_wait suspends for a
// hardware-chosen interval per call, so the cap is generous but finite.
constexpr uint32_t kSpinLimit = 1u << 22;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

// 1-D bulk copy global -> shared through the TMA engine; completion is
// signalled as transaction bytes on `bar`.  dst/src 16-byte aligned, bytes a
// multiple of 16.  No multicast.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes,
                                         uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait.  On timeout sets ERR_MBAR_TIMEOUT and returns false; the
// caller then skips its remaining waits (the data is garbage, the kernel
// still terminates and the host reports the error).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  for (uint32_t i = 0; i < kSpinLimit; ++i)
    if (mbar_try_wait(bar, parity)) return true;
  if (err) atomicOr(err, ERR_MBAR_TIMEOUT);
  return false;
}

// Programmatic dependent launch.  Every kernel here issues its weight
// prefetch (constant data) before pdl_wait(), then calls pdl_launch() right
// after it, so kernel N+1's pre-wait part may only read data written by
// kernels <= N-1.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// D(16x8 s32) += A(16x32 u8, row) * B(32x8 s8, col).
__device__ __forceinline__ void mma_u8s8(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ float bf16_trunc(float v) {
  return __uint_as_float(__float_as_uint(v) & 0xFFFF0000u);
}

// 16-bit scale/bias word -> f32 (fp16 or raw BF16 bits).
template <bool kBF16>
__device__ __forceinline__ float u16_to_f32(uint16_t raw) {
  if constexpr (kBF16) return __uint_as_float(static_cast<uint32_t>(raw) << 16);
  else return __half2float(__ushort_as_half(raw));
}

__device__ __forceinline__ int warp_sum_int(int v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Order-preserving float -> u32 key (larger float => larger key).
__device__ __forceinline__ uint32_t float_key(float f) {
  uint32_t u = __float_as_uint(f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// argmax slot: (key << 32) | (0xFFFFFFFF - index): atomicMax keeps the
// largest value and, on ties, the smallest index (first maximum wins).
__device__ __forceinline__ unsigned long long argmax_pack(float v, uint32_t idx) {
  return (static_cast<unsigned long long>(float_key(v)) << 32) | (0xFFFFFFFFu - idx);
}
__host__ __device__ __forceinline__ uint32_t argmax_index(unsigned long long packed) {
  return 0xFFFFFFFFu - static_cast<uint32_t>(packed & 0xFFFFFFFFull);
}

}  // namespace nnz
