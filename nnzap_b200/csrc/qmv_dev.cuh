// Device building blocks of the quantized matvec, shared by the standalone
// kernel (qmv.cuh) and the persistent decode kernel (mega.cu).  All assume a
// 128-thread CTA (kQmvThreads) and the packed layout of packing.h.
#pragma once
#include "common.cuh"
#include "packing.h"

namespace nnz {

constexpr int kQmvWarps = 4;
constexpr int kQmvThreads = kQmvWarps * 32;
constexpr int kBatchChunk = 8;     // batch rows per CTA

// rms[b] = rsqrt(mean(res_b^2) + eps) for rows b < bc of an f32 residual
// (row stride `stride`, K columns).  Every thread's loads are issued before
// any is used.  Ends with __syncthreads(); rms must hold kBatchChunk floats.
__device__ __forceinline__ void block_rms(const float* res, uint32_t stride, uint32_t K, uint32_t bc,
                                          float eps, float* rms) {
  const int lane = threadIdx.x & 31;
  if (threadIdx.x < kBatchChunk) rms[threadIdx.x] = 0.f;
  __syncthreads();
  const uint32_t q4 = K / 4, n4 = bc * q4;
  float ssr[kBatchChunk];
#pragma unroll
  for (int bb = 0; bb < kBatchChunk; ++bb) ssr[bb] = 0.f;
  for (uint32_t j0 = threadIdx.x; j0 < n4; j0 += 4 * kQmvThreads) {
    float4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t j = j0 + u * kQmvThreads;
      v[u] = j < n4 ? __ldcg(reinterpret_cast<const float4*>(res + (size_t)(j / q4) * stride + 4 * (j % q4)))
                    : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t b = (j0 + u * kQmvThreads) / q4;
      const float e = v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
#pragma unroll
      for (int bb = 0; bb < kBatchChunk; ++bb) ssr[bb] += (b == (uint32_t)bb) ? e : 0.f;
    }
  }
#pragma unroll
  for (int bb = 0; bb < kBatchChunk; ++bb) {
    if ((uint32_t)bb >= bc) break;
    const float t = warp_sum(ssr[bb]);
    if (lane == 0) atomicAdd(&rms[bb], t);
  }
  __syncthreads();
  if (threadIdx.x < bc) rms[threadIdx.x] = rsqrtf(rms[threadIdx.x] / (float)K + eps);
  __syncthreads();
}

// xs[b][k - K0] = fp16(res_b[k] * rms[b] * w[k]) for k in [K0, K0 + Kr)
// (engine BF16 mode truncates to BF16 first).  No trailing sync.
__device__ __forceinline__ void stage_norm(const float* res, uint32_t stride, const float* norm_w,
                                           const float* rms, uint32_t K0, uint32_t Kr, uint32_t bc,
                                           bool bf16r, __half* xs) {
  const uint32_t r4 = Kr / 4, m4 = bc * r4;
  for (uint32_t j0 = threadIdx.x; j0 < m4; j0 += 4 * kQmvThreads) {
    float4 v[4], w[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t j = j0 + u * kQmvThreads;
      if (j < m4) {
        const uint32_t k = K0 + 4 * (j % r4);
        v[u] = __ldcg(reinterpret_cast<const float4*>(res + (size_t)(j / r4) * stride + k));
        w[u] = *reinterpret_cast<const float4*>(norm_w + k);
      }
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t j = j0 + u * kQmvThreads;
      if (j < m4) {
        const float rr = rms[j / r4];
        float o0 = v[u].x * rr * w[u].x, o1 = v[u].y * rr * w[u].y;
        float o2 = v[u].z * rr * w[u].z, o3 = v[u].w * rr * w[u].w;
        if (bf16r) { o0 = bf16_trunc(o0); o1 = bf16_trunc(o1); o2 = bf16_trunc(o2); o3 = bf16_trunc(o3); }
        __half2* dst = reinterpret_cast<__half2*>(xs + (size_t)(j / r4) * Kr + 4 * (j % r4));
        dst[0] = __floats2half2_rn(o0, o1);
        dst[1] = __floats2half2_rn(o2, o3);
      }
    }
  }
}

// Small batches (bc * K <= 2048 floats): one round trip.  Every thread
// loads its float4s of the full rows plus the matching norm weights of the
// slice [K0, K0 + Kr), reduces the sum of squares through registers and a
// shared-memory atomic per warp and row, then normalises its own slice
// elements in registers.  rms holds kBatchChunk floats.
__device__ __forceinline__ void stage_norm_fast(const float* res, uint32_t stride, uint32_t K,
                                                const float* norm_w, float eps, uint32_t K0, uint32_t Kr,
                                                uint32_t bc, bool bf16r, float* rms, __half* xs) {
  constexpr int kItems = 4;
  const int lane = threadIdx.x & 31;
  const uint32_t q4 = K / 4, n4 = bc * q4;
  if (threadIdx.x < kBatchChunk) rms[threadIdx.x] = 0.f;
  float4 v[kItems], w[kItems];
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const uint32_t j = threadIdx.x + u * kQmvThreads;
    const uint32_t k = 4 * (j % q4);
    v[u] = j < n4 ? __ldcg(reinterpret_cast<const float4*>(res + (size_t)(j / q4) * stride + k))
                  : make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < n4 && k >= K0 && k < K0 + Kr) w[u] = *reinterpret_cast<const float4*>(norm_w + k);
  }
  float ssr[kBatchChunk];
#pragma unroll
  for (int bb = 0; bb < kBatchChunk; ++bb) ssr[bb] = 0.f;
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const uint32_t b = (threadIdx.x + u * kQmvThreads) / q4;
    const float e = v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
#pragma unroll
    for (int bb = 0; bb < kBatchChunk; ++bb) ssr[bb] += (b == (uint32_t)bb) ? e : 0.f;
  }
  __syncthreads();   // rms zeroed
#pragma unroll
  for (int bb = 0; bb < kBatchChunk; ++bb) {
    if ((uint32_t)bb >= bc) break;
    const float t = warp_sum(ssr[bb]);
    if (lane == 0) atomicAdd(&rms[bb], t);
  }
  __syncthreads();
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const uint32_t j = threadIdx.x + u * kQmvThreads;
    const uint32_t b = j / q4, k = 4 * (j % q4);
    if (j < n4 && k >= K0 && k < K0 + Kr) {
      const float rr = rsqrtf(rms[b] / (float)K + eps);
      float o0 = v[u].x * rr * w[u].x, o1 = v[u].y * rr * w[u].y;
      float o2 = v[u].z * rr * w[u].z, o3 = v[u].w * rr * w[u].w;
      if (bf16r) { o0 = bf16_trunc(o0); o1 = bf16_trunc(o1); o2 = bf16_trunc(o2); o3 = bf16_trunc(o3); }
      __half2* dst = reinterpret_cast<__half2*>(xs + (size_t)b * Kr + (k - K0));
      dst[0] = __floats2half2_rn(o0, o1);
      dst[1] = __floats2half2_rn(o2, o3);
    }
  }
}

// Quantise one 128-wide scale group of row 0 held by a warp, 4 consecutive
// fp16-representable values per lane (lane l: group columns 4l..4l+3), into
// the int8 hi/lo B fragments and the group's gsx / gsum / gsq -- the same
// arithmetic as quantize_xs.  Writes only batch-column-0 words of xf.
template <int NT>
__device__ __forceinline__ void quant_group_row0(const float (&x)[4], uint32_t gl, int lane, uint8_t* xf,
                                                 float* gsx, float* gsum, int* gsq) {
  float amax = 0.f, sumx = 0.f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    amax = fmaxf(amax, fabsf(x[i]));
    sumx += x[i];
  }
  amax = warp_max(amax);
  sumx = warp_sum(sumx);
  const int E = (amax > 0.f) ? (int)((__float_as_uint(amax) >> 23) & 0xFFu) - 126 : 0;
  const float up = __uint_as_float((uint32_t)(127 + 14 - E) << 23);
  uint32_t hiw = 0, low = 0;
  int qsum = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = (amax > 0.f) ? __float2int_rn(x[i] * up) : 0;
    qsum += q;
    const int lo = ((q + 128) & 255) - 128;
    const int hi = (q - lo) >> 8;
    hiw |= ((uint32_t)hi & 0xFFu) << (8 * i);
    low |= ((uint32_t)lo & 0xFFu) << (8 * i);
  }
  qsum = warp_sum_int(qsum);
  // lane's 4 columns = bytes 0-3 of one fragment word: chunk lane / 8,
  // k-register (lane >> 2) & 1, fragment lane (lane & 3) (hi) / 4 + (lane & 3) (lo)
  const uint32_t c = gl * (128 / kChunk) + lane / 8;
  uint8_t* base = xf + ((size_t)(c * NT) * 32) * 8 + ((lane >> 2) & 1) * 4;
  *reinterpret_cast<uint32_t*>(base + (size_t)(lane & 3) * 8) = hiw;
  *reinterpret_cast<uint32_t*>(base + (size_t)(4 + (lane & 3)) * 8) = low;
  if (lane == 0) {
    gsx[gl * kBatchChunk] = (amax > 0.f) ? __uint_as_float((uint32_t)(127 + E - 14) << 23) : 0.f;
    gsum[gl * kBatchChunk] = sumx;
    gsq[gl * kBatchChunk] = qsum;
  }
}

// Fused RMSNorm + activation quantisation for one row (bc = 1), group size
// 128 and K <= 2048: thread t holds columns 4 (t + 128 u), so warp w's item
// u is the whole scale group w + 4 u.  Each warp quantises, straight from
// registers, the groups of [G0, G0 + ng) it holds -- same arithmetic as
// stage_norm_fast followed by quantize_xs (fp16 rounding of the normalised
// value, per-group exponent, 15-bit split into int8 hi/lo B fragments).
// Writes only the batch-column-0 words of xf (which must otherwise stay
// zero) and gsx/gsum/gsq of row 0.  Ends with __syncthreads().
template <int NT>
__device__ __forceinline__ void norm_quant_row128(const float* res, uint32_t K, const float* norm_w, float eps,
                                                  uint32_t G0, uint32_t ng, bool bf16r, float* rms,
                                                  uint8_t* xf, float* gsx, float* gsum, int* gsq) {
  constexpr int kItems = 4;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t q4 = K / 4;
  if (threadIdx.x == 0) rms[0] = 0.f;
  float4 v[kItems], w[kItems];
#pragma unroll
  for (int u = 0; u < kItems; ++u) {
    const uint32_t j = threadIdx.x + u * kQmvThreads;
    const uint32_t g = warp + 4 * u;                  // this item's scale group
    v[u] = j < q4 ? __ldcg(reinterpret_cast<const float4*>(res) + j) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (j < q4 && g >= G0 && g < G0 + ng) w[u] = reinterpret_cast<const float4*>(norm_w)[j];
  }
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < kItems; ++u) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
  __syncthreads();   // rms zeroed
  ss = warp_sum(ss);
  if (lane == 0) atomicAdd(&rms[0], ss);
  __syncthreads();
  const float rr = rsqrtf(rms[0] / (float)K + eps);
  // one copy of the quantiser, run for each of this warp's groups in the
  // unit (the group's registers picked by selects, not by indexing)
#pragma unroll 1
  for (int u = 0; u < kItems; ++u) {
    const uint32_t g = warp + 4 * u;
    if (g < G0 || g >= G0 + ng || threadIdx.x + u * kQmvThreads >= q4) continue;   // warp-uniform
    const float4 vu = u == 0 ? v[0] : u == 1 ? v[1] : u == 2 ? v[2] : v[3];
    const float4 wu = u == 0 ? w[0] : u == 1 ? w[1] : u == 2 ? w[2] : w[3];
    float x[4] = {vu.x * rr * wu.x, vu.y * rr * wu.y, vu.z * rr * wu.z, vu.w * rr * wu.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      if (bf16r) x[i] = bf16_trunc(x[i]);
      x[i] = __half2float(__float2half_rn(x[i]));
    }
    quant_group_row0<NT>(x, g - G0, lane, xf, gsx, gsum, gsq);
  }
  __syncthreads();
}

// xs[b][k - K0] = x_b[k] (fp16 input, 16-byte aligned rows).  No trailing sync.
__device__ __forceinline__ void stage_f16(const __half* xh, uint32_t stride, uint32_t K0, uint32_t Kr,
                                          uint32_t bc, __half* xs) {
  const uint32_t r8 = Kr / 8, m8 = bc * r8;
  for (uint32_t j0 = threadIdx.x; j0 < m8; j0 += 4 * kQmvThreads) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t j = j0 + u * kQmvThreads;
      if (j < m8) v[u] = *reinterpret_cast<const uint4*>(xh + (size_t)(j / r8) * stride + K0 + 8 * (j % r8));
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const uint32_t j = j0 + u * kQmvThreads;
      if (j < m8) *reinterpret_cast<uint4*>(xs + (size_t)(j / r8) * Kr + 8 * (j % r8)) = v[u];
    }
  }
}

// Per (row, group): 15-bit fixed-point split of the staged fp16 x into int8
// hi/lo B fragments (xf), the group scale 2^(E-14) (gsx), sum(x) (gsum) and
// sum(q) (gsq).  q = round(x * 2^(14-E)) with amax = m * 2^E: elements within
// 1/16 of the group maximum are exact (fp16 has 11 significant bits), smaller
// ones carry at most 2^(E-15) absolute error.  Zeroes xf/gsx/gsum/gsq itself.  Syncs at start and end.
// With zero = false the caller guarantees xf/gsx/gsum/gsq were zeroed once
// and only ever rewritten at the same (row < bc) positions.
template <int NT>
__device__ __forceinline__ void quantize_xs(const __half* xs, uint32_t Kr, uint32_t bc, uint32_t ng,
                                            uint32_t gs, uint8_t* xf, float* gsx, float* gsum,
                                            int* gsq, bool zero = true) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cpg = gs / kChunk;
  if (zero) {
    const uint32_t xf_words = ng * cpg * NT * 64;
    for (uint32_t i = threadIdx.x; i < xf_words; i += kQmvThreads) reinterpret_cast<uint32_t*>(xf)[i] = 0;
    for (uint32_t i = threadIdx.x; i < ng * kBatchChunk; i += kQmvThreads) {
      gsx[i] = 0.f; gsum[i] = 0.f; gsq[i] = 0;
    }
  }
  __syncthreads();
  {
    const uint32_t per_lane = gs / 32;
    for (uint32_t p = warp; p < bc * ng; p += kQmvWarps) {
      const uint32_t b = p % bc, gl = p / bc;
      float xv[8];
      float amax = 0.f, sumx = 0.f;
#pragma unroll
      for (uint32_t m = 0; m < 8; ++m) {
        if (m < per_lane) {
          const float v = __half2float(xs[(size_t)b * Kr + gl * gs + m * 32 + lane]);
          xv[m] = v;
          amax = fmaxf(amax, fabsf(v));
          sumx += v;
        }
      }
      amax = warp_max(amax);
      sumx = warp_sum(sumx);
      // amax = m * 2^E, m in [0.5, 1): E from the exponent field (amax is a
      // normal fp16 value or 0); scale 2^(14-E) built from its bits (exact).
      const int E = (amax > 0.f) ? (int)((__float_as_uint(amax) >> 23) & 0xFFu) - 126 : 0;
      const float up = __uint_as_float((uint32_t)(127 + 14 - E) << 23);
      int qsum = 0;
      const uint32_t nt = b >> 2, ncol = 2 * (b & 3);
#pragma unroll
      for (uint32_t m = 0; m < 8; ++m) {
        if (m < per_lane) {
          const int q = (amax > 0.f) ? __float2int_rn(xv[m] * up) : 0;
          qsum += q;
          const int lo = ((q + 128) & 255) - 128;
          const int hi = (q - lo) >> 8;
          const uint32_t kk = (m * 32 + lane) % 32;               // column within chunk
          const uint32_t c = gl * cpg + (m * 32 + lane) / 32;     // chunk within CTA range
          const uint32_t fl = ((kk & 15) >> 2), reg = kk >> 4, byte = kk & 3;
          uint8_t* base = xf + ((size_t)(c * NT + nt) * 32) * 8 + reg * 4 + byte;
          base[((ncol)*4 + fl) * 8] = (uint8_t)(int8_t)hi;
          base[((ncol + 1) * 4 + fl) * 8] = (uint8_t)(int8_t)lo;
        }
      }
      for (int o = 16; o > 0; o >>= 1) qsum += __shfl_xor_sync(0xffffffffu, qsum, o);
      if (lane == 0) {
        gsx[gl * kBatchChunk + b] = (amax > 0.f) ? __uint_as_float((uint32_t)(127 + E - 14) << 23) : 0.f;
        gsum[gl * kBatchChunk + b] = sumx;
        gsq[gl * kBatchChunk + b] = qsum;
      }
    }
  }
  __syncthreads();

}

// One scale group of one row tile (per sub-matrix and batch N-tile):
// int8 MMAs over the group's chunks, then the scaled int32 -> f32
// accumulation into y (see qmv.cuh for the arithmetic).
template <int FMT, int NT, int SUB, bool BF16S>
__device__ __forceinline__ void qmv_group(const uint8_t* sb, uint32_t seg, const uint8_t* xf, uint32_t gl,
                                          uint32_t cpg, const float* gsx, const float* gsum,
                                          const int* gsq, float (&y)[SUB][NT][16]) {
  const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll
    for (int s = 0; s < SUB; ++s) {
      const uint8_t* segp = sb + s * seg;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t bcol = n * 4 + t;
        const float sx = gsx[gl * kBatchChunk + bcol];
        if constexpr (FMT == FMT_Q1) {
          const uint4 s0 = *reinterpret_cast<const uint4*>(segp + cpg * 512 + g * 32);
          const uint4 s1 = *reinterpret_cast<const uint4*>(segp + cpg * 512 + g * 32 + 16);
          const int sq = gsq[gl * kBatchChunk + bcol];
          int D[8][4];
#pragma unroll
          for (int j = 0; j < 8; ++j) D[j][0] = D[j][1] = D[j][2] = D[j][3] = 0;
          const uint8_t* xb = xf + ((size_t)(gl * cpg * NT + n) * 32 + lane) * 8;
          if (cpg == 4) {
            // common case (group 128): every operand load issued up front
            uint4 A[4];
            uint2 B[4];
#pragma unroll
            for (int cc = 0; cc < 4; ++cc) {
              A[cc] = *reinterpret_cast<const uint4*>(segp + cc * 512 + lane * 16);
              B[cc] = *reinterpret_cast<const uint2*>(xb + (size_t)cc * NT * 256);
            }
#pragma unroll
            for (int cc = 0; cc < 4; ++cc)
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t msk = 0x01010101u << j;
                mma_u8s8(D[j], A[cc].x & msk, A[cc].y & msk, A[cc].z & msk, A[cc].w & msk, B[cc].x, B[cc].y);
              }
          } else {
#pragma unroll 1
            for (uint32_t cc = 0; cc < cpg; ++cc) {
              const uint4 A = *reinterpret_cast<const uint4*>(segp + cc * 512 + lane * 16);
              const uint2 B = *reinterpret_cast<const uint2*>(xb + (size_t)cc * NT * 256);
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const uint32_t msk = 0x01010101u << j;
                mma_u8s8(D[j], A.x & msk, A.y & msk, A.z & msk, A.w & msk, B.x, B.y);
              }
            }
          }
          const uint16_t* sc0 = reinterpret_cast<const uint16_t*>(&s0);
          const uint16_t* sc1 = reinterpret_cast<const uint16_t*>(&s1);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const int v = 2 * j + h;
              const uint16_t raw = v < 8 ? sc0[v] : sc1[v - 8];
              const float scl = u16_to_f32<false>(raw) * sx;
              const int acc = ((D[j][2 * h] << 8) + D[j][2 * h + 1]) >> j;
              y[s][n][v] = fmaf((float)(2 * acc - sq), scl, y[s][n][v]);
            }
          }
        } else {
          int Dr[4][4], Dl[4][4];
#pragma unroll
          for (int u = 0; u < 4; ++u)
#pragma unroll
            for (int c = 0; c < 4; ++c) Dr[u][c] = Dl[u][c] = 0;
#pragma unroll 1
          for (uint32_t cc = 0; cc < cpg; ++cc) {
            const uint2 B = *reinterpret_cast<const uint2*>(
                xf + ((size_t)((gl * cpg + cc) * NT + n) * 32 + lane) * 8);
#pragma unroll
            for (int u = 0; u < 4; ++u) {
              const uint4 A =
                  *reinterpret_cast<const uint4*>(segp + cc * 2048 + u * 512 + lane * 16);
              mma_u8s8(Dr[u], A.x, A.y, A.z, A.w, B.x, B.y);
              mma_u8s8(Dl[u], A.x & 0x0F0F0F0Fu, A.y & 0x0F0F0F0Fu, A.z & 0x0F0F0F0Fu,
                       A.w & 0x0F0F0F0Fu, B.x, B.y);
            }
          }
          const uint16_t* scp = reinterpret_cast<const uint16_t*>(segp + cpg * 2048 + g * 64);
          uint16_t scs[16], bis[16];
          {
            const uint4 v0 = *reinterpret_cast<const uint4*>(scp);
            const uint4 v1 = *reinterpret_cast<const uint4*>(scp + 8);
            const uint4 v2 = *reinterpret_cast<const uint4*>(scp + 16);
            const uint4 v3 = *reinterpret_cast<const uint4*>(scp + 24);
            *reinterpret_cast<uint4*>(&scs[0]) = v0;
            *reinterpret_cast<uint4*>(&scs[8]) = v1;
            *reinterpret_cast<uint4*>(&bis[0]) = v2;
            *reinterpret_cast<uint4*>(&bis[8]) = v3;
          }
          const float sumx = gsum[gl * kBatchChunk + bcol];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            const int a0 = (Dl[u][0] << 8) + Dl[u][1];
            const int a1 = (Dl[u][2] << 8) + Dl[u][3];
            const int r0 = (Dr[u][0] << 8) + Dr[u][1];
            const int r1 = (Dr[u][2] << 8) + Dr[u][3];
            const int vv[4] = {a0, a1, (r0 - a0) >> 4, (r1 - a1) >> 4};
#pragma unroll
            for (int w = 0; w < 4; ++w) {
              const int v = 4 * u + w;
              const float scl = u16_to_f32<BF16S>(scs[v]) * sx;
              const float bia = u16_to_f32<BF16S>(bis[v]);
              y[s][n][v] = fmaf((float)vv[w], scl, fmaf(bia, sumx, y[s][n][v]));
            }
          }
        }
      }
    }
}

// Row of the tile held by y index v of lane-group g.
template <int FMT>
__device__ __forceinline__ uint32_t y_row(int v, int g) {
  if constexpr (FMT == FMT_Q1) return 16 * (v >> 1) + g + 8 * (v & 1);
  else return 32 * (v >> 2) + g + ((v & 3) == 0 ? 0 : (v & 3) == 1 ? 8 : (v & 3) == 2 ? 16 : 24);
}

}  // namespace nnz
