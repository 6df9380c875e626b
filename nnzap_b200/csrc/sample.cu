// Token sampling on the device (replaces the host sampler of the reference,
// nnmetal/src/transformer.zig:3712-3908: sampleToken).
//
// One CTA of 1024 threads per row.  Same steps and order as the reference:
//   temperature  logits *= 1 / T
//   top-k        keep logits >= the k-th largest (radix select on the
//                order-preserving u32 key of the f32 value, 4 x 8-bit passes)
//   top-p        probabilities p = softmax(logits); walking them in
//                descending order, keep tokens until the mass reaches top_p:
//                the cut value is found by a radix select whose histogram
//                bins hold probability mass instead of counts; tokens with
//                p >= the cut value stay
//   sample       p = softmax(kept logits); first index (in vocabulary
//                order) whose running sum exceeds the uniform draw u, or the
//                last index when rounding leaves the sum below u.
// The uniform draws come from the host (one per row per step).  The sampled
// index is written into the row's argmax slot (the decode state's next
// token) and, optionally, to a token array.
#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "misc.cuh"

namespace nnz {

namespace {

constexpr int kSThreads = 1024;
constexpr int kSWarps = kSThreads / 32;

__device__ __forceinline__ float key_to_float(uint32_t k) {
  const uint32_t u = (k & 0x80000000u) ? (k & 0x7FFFFFFFu) : ~k;
  return __uint_as_float(u);
}

// Block-wide sum / max (all threads get the result).  `red` holds kSWarps
// floats; ends synchronised.
__device__ __forceinline__ float block_sum(float v, float* red) {
  v = warp_sum(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = threadIdx.x < kSWarps ? red[threadIdx.x] : 0.f;
  if (threadIdx.x < 32) t = warp_sum(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

__device__ __forceinline__ float block_max(float v, float* red) {
  v = warp_max(v);
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = threadIdx.x < kSWarps ? red[threadIdx.x] : -INFINITY;
  if (threadIdx.x < 32) t = warp_max(t);
  if (threadIdx.x == 0) red[0] = t;
  __syncthreads();
  return red[0];
}

// Radix select over the keys of x[0..n) (elements equal to -inf ignored):
// the largest key K such that the weight of {key >= K} reaches `need`
// (weight = 1 per element when `mass` is false, else exp(x - mx) / den).
__device__ uint32_t radix_select(const float* x, uint32_t n, bool mass, float mx, float den, float need,
                                 float* hist, float* red) {
  uint32_t prefix = 0, pmask = 0;
  float above = 0.f;   // weight of keys whose known prefix already exceeds the candidate
  for (int shift = 24; shift >= 0; shift -= 8) {
    for (int i = threadIdx.x; i < 256; i += kSThreads) hist[i] = 0.f;
    __syncthreads();
    for (uint32_t i = threadIdx.x; i < n; i += kSThreads) {
      const float v = x[i];
      if (v == -INFINITY) continue;
      const uint32_t k = float_key(v);
      if ((k & pmask) != prefix) continue;
      atomicAdd(&hist[(k >> shift) & 0xFFu], mass ? expf(v - mx) / den : 1.f);
    }
    __syncthreads();
    // walk the bins from the top: the digit where the running weight reaches need
    __shared__ uint32_t s_digit;
    __shared__ float s_above;
    if (threadIdx.x == 0) {
      float run = above;
      int d = 255;
      for (; d > 0; --d) {
        if (run + hist[d] >= need) break;
        run += hist[d];
      }
      s_digit = (uint32_t)d;
      s_above = run;
    }
    __syncthreads();
    prefix |= s_digit << shift;
    pmask |= 0xFFu << shift;
    above = s_above;
    __syncthreads();
  }
  (void)red;
  return prefix;
}

__global__ void __launch_bounds__(kSThreads) sample_kernel(float* logits, uint32_t n, uint32_t stride, float temperature,
                                                           uint32_t top_k, float top_p, const float* uniforms,
                                                           unsigned long long* argmax, uint32_t* tokens) {
  __shared__ float red[kSWarps];
  __shared__ float hist[256];
  __shared__ unsigned int s_pick;
  const uint32_t row = blockIdx.x;
  float* x = logits + (size_t)row * stride;
  // temperature (in place, like the reference)
  const float inv_t = 1.0f / temperature;
  for (uint32_t i = threadIdx.x; i < n; i += kSThreads) x[i] *= inv_t;
  __syncthreads();
  // top-k: drop values below the k-th largest
  if (top_k > 0 && top_k < n) {
    const uint32_t kk = radix_select(x, n, false, 0.f, 1.f, (float)top_k, hist, red);
    const float thr = key_to_float(kk);
    for (uint32_t i = threadIdx.x; i < n; i += kSThreads)
      if (x[i] < thr) x[i] = -INFINITY;
    __syncthreads();
  }
  // top-p: keep the most probable tokens until their mass reaches top_p
  if (top_p < 1.0f) {
    float mx = -INFINITY;
    for (uint32_t i = threadIdx.x; i < n; i += kSThreads) mx = fmaxf(mx, x[i]);
    mx = block_max(mx, red);
    float s = 0.f;
    for (uint32_t i = threadIdx.x; i < n; i += kSThreads) s += expf(x[i] - mx);
    const float den = block_sum(s, red);
    const uint32_t kp = radix_select(x, n, true, mx, den, top_p, hist, red);
    for (uint32_t i = threadIdx.x; i < n; i += kSThreads)
      if (x[i] != -INFINITY && float_key(x[i]) < kp) x[i] = -INFINITY;
    __syncthreads();
  }
  // softmax of what is left, then the inverse CDF in vocabulary order
  float mx = -INFINITY;
  for (uint32_t i = threadIdx.x; i < n; i += kSThreads) mx = fmaxf(mx, x[i]);
  mx = block_max(mx, red);
  float s = 0.f;
  for (uint32_t i = threadIdx.x; i < n; i += kSThreads) s += expf(x[i] - mx);
  const float inv_den = 1.0f / block_sum(s, red);
  // contiguous chunk per thread, exclusive scan of the chunk sums
  const uint32_t per = (n + kSThreads - 1) / kSThreads;
  const uint32_t c0 = threadIdx.x * per, c1 = min(n, c0 + per);
  float cs = 0.f;
  for (uint32_t i = c0; i < c1; ++i) cs += expf(x[i] - mx) * inv_den;
  // warp inclusive scan, then across warps
  float inc = cs;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const float t = __shfl_up_sync(0xffffffffu, inc, o);
    if ((threadIdx.x & 31) >= (unsigned)o) inc += t;
  }
  __shared__ float wsum[kSWarps];
  if ((threadIdx.x & 31) == 31) wsum[threadIdx.x >> 5] = inc;
  if (threadIdx.x == 0) s_pick = n - 1;
  __syncthreads();
  float base = 0.f;
  for (int w = 0; w < (int)(threadIdx.x >> 5); ++w) base += wsum[w];
  float run = base + inc - cs;   // exclusive prefix of this chunk
  const float u = uniforms[row];
  if (run + cs > u || c1 == n) {
    for (uint32_t i = c0; i < c1; ++i) {
      run += expf(x[i] - mx) * inv_den;
      if (run > u) {
        atomicMin(&s_pick, i);
        break;
      }
    }
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t tok = s_pick;
    argmax[row] = argmax_pack(1.0f, tok);
    if (tokens) tokens[row] = tok;
  }
}

}  // namespace

cudaError_t sample_launch(float* logits, uint32_t rows, uint32_t n, uint32_t stride, float temperature,
                          uint32_t top_k, float top_p, const float* uniforms, unsigned long long* argmax,
                          uint32_t* tokens, cudaStream_t st) {
  if (rows == 0 || n == 0 || !(temperature > 0.f) || !(top_p > 0.f) || top_p > 1.f) return cudaErrorInvalidValue;
  sample_kernel<<<rows, kSThreads, 0, st>>>(logits, n, stride, temperature, top_k, top_p, uniforms, argmax, tokens);
  return cudaGetLastError();
}

}  // namespace nnz
