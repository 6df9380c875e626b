// Quantized matrix-vector / small-batch matrix multiply for 1-bit (Q1) and
// MLX-affine 4-bit (Q4) weights in the tile-packed layout of packing.h.
//
// Replaces the reference's specialised QMV family
// (nnmetal/src/shaders/qmv_specialized.metal:55-1621,
//  nnmetal/src/shaders/q4mv_bf16_specialized.metal:93-1181): y = x W^T with
// f32 accumulation, plus the fused prologues/epilogues those kernels carry
// (RMSNorm prologue, fp16 / f32 / residual-add / SiLU*mul / logits outputs).
//
// How a B200 CTA does it:
//  * 4 warps, each owning a private ring of R segment buffers.  Lane 0 of
//    each warp streams its groups' segments (weights + scales of one row
//    tile x one scale group) with 1-D bulk copies (TMA engine) completing on
//    an mbarrier.  The first R copies are issued BEFORE griddepcontrol.wait,
//    so under programmatic dependent launch the weight stream of kernel N+1
//    overlaps the tail of kernel N.
//  * The activation x (fp16, optionally RMSNorm'ed from the f32 residual) is
//    re-expressed per scale group as an exact 15-bit fixed-point integer
//    q = x * 2^(14-E) (E = exponent bound of the group's max |x|) split into
//    two signed bytes (hi, lo) that form the B operand (two columns per batch
//    row) of an int8 tensor-core MMA.  Elements within 1/16 of the group
//    maximum are represented exactly; smaller ones with absolute error
//    <= 2^(E-15).
//  * Q1: one AND of a packed word with 0x01010101<<j yields an MMA A register
//    of four u8 weights in {0, 2^j} for row block j (8 row blocks = 128 rows),
//    so 1-bit weights cost 0.25 integer ops each.  Sum over k of sign*x is
//    recovered exactly as 2*sum(bit*q) - sum(q).
//  * Q4: a packed byte holds two nibbles of the SAME column for two rows; the
//    raw bytes and the bytes & 0x0F are both MMA A operands, and the high
//    nibble row's dot product is (raw - low) / 16, exact in int32.
//  * Per group the int32 accumulators are scaled into f32 row sums (scale *
//    2^(E-14) [+ bias * sum(x)]), then the CTA's warps are reduced through
//    shared memory; split-K CTAs of one tile meet in a workspace and the last
//    one to arrive (atomic counter) sums the partials in split order
//    (deterministic) and runs the epilogue.
#pragma once
#include "common.cuh"
#include "packing.h"

namespace nnz {

enum Prologue : int { PRO_F16 = 0, PRO_NORM = 1 };
enum Epilogue : int { EPI_F16 = 0, EPI_F32 = 1, EPI_RESADD = 2, EPI_SILU = 3, EPI_LOGITS = 4 };

constexpr int kQmvWarps = 4;
constexpr int kQmvThreads = kQmvWarps * 32;
constexpr int kQmvRing = 4;        // segment slots per warp
constexpr int kBatchChunk = 8;     // batch rows per CTA (grid.y covers more)

struct QmvArgs {
  const uint8_t* w;          // packed weights (packing.h), 256-B aligned
  uint32_t M, K, gs;         // rows (per sub-matrix), cols, group size
  uint32_t tiles, groups;    // ceil(M/128), K/gs
  uint32_t ksplit;           // CTAs along K per tile
  uint32_t P;                // persistent CTAs per K split (each loops over tiles)
  const void* x;             // fp16 [batch][x_stride] or f32 residual (PRO_NORM)
  uint32_t x_stride;
  const float* norm_w;       // RMSNorm weight [K] (PRO_NORM)
  float eps;
  uint32_t batch;
  void* out;                 // fp16 / f32 output [batch][out_stride]
  uint32_t out_stride;
  float* logits;             // EPI_LOGITS: optional f32 logits [batch][logits_stride]
  uint32_t logits_stride;
  unsigned long long* argmax;  // EPI_LOGITS: [batch] packed (value, index) slots
  float* ws;                 // split-K partials
  uint32_t* counters;        // split-K arrival counters [ychunks][tiles], zero at rest
  int* err;
  uint32_t bf16_round;       // truncate every output to BF16 first (engine Q4 mode)
};

struct QmvSmem {
  uint32_t nslot, bars, ring, red, xf, xs, gsx, gsum, gsq, rms, flag, total;
};

// Shared-memory layout.  The ring keeps streaming the next tile's segments
// while the current tile is reduced, so the reduction buffer is separate.
__host__ __device__ inline QmvSmem qmv_smem_layout(int fmt, int nt, int sub, uint32_t gs,
                                                   uint32_t ngroups_cta, uint32_t rows) {
  QmvSmem s;
  uint32_t per_warp = (ngroups_cta + kQmvWarps - 1) / kQmvWarps;
  s.nslot = per_warp < (uint32_t)kQmvRing ? (per_warp ? per_warp : 1) : kQmvRing;
  // cap the ring at 96 KB so the staging buffers always fit
  while (s.nslot > 1 && kQmvWarps * s.nslot * sub * seg_bytes(fmt, gs) > 96u * 1024u) --s.nslot;
  uint32_t o = 0;
  s.bars = o; o += kQmvWarps * kQmvRing * 8;
  o = (o + 127) & ~127u;
  s.ring = o;
  o += kQmvWarps * s.nslot * sub * seg_bytes(fmt, gs);
  s.red = o;
  o += kQmvWarps * kTileRows * sub * kBatchChunk * 4;
  o = (o + 127) & ~127u;
  s.xf = o; o += ngroups_cta * (gs / kChunk) * nt * 256;
  s.xs = o; o += ((ngroups_cta * gs * rows * 2) + 15) & ~15u;
  s.gsx = o; o += ngroups_cta * kBatchChunk * 4;
  s.gsum = o; o += ngroups_cta * kBatchChunk * 4;
  s.gsq = o; o += ngroups_cta * kBatchChunk * 4;
  s.rms = o; o += kBatchChunk * 4;
  s.flag = o; o += 16;
  s.total = o;
  return s;
}

template <int FMT, int NT, int SUB, int PRO, int EPI, bool BF16S>
__global__ void __launch_bounds__(kQmvThreads) qmv_kernel(QmvArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  const uint32_t cpg = a.gs / kChunk;
  const uint32_t seg = seg_bytes(FMT, a.gs);
  const uint32_t split = blockIdx.x % a.ksplit;
  const uint32_t pcta = blockIdx.x / a.ksplit;          // tiles pcta, pcta + P, ...
  const uint32_t ntc = pcta < a.tiles ? (a.tiles - pcta + a.P - 1) / a.P : 0;
  const uint32_t ychunk = blockIdx.y;
  const uint32_t b0 = ychunk * kBatchChunk;
  const uint32_t bc = min(a.batch - b0, (uint32_t)kBatchChunk);
  const uint32_t G0 = (uint32_t)((uint64_t)a.groups * split / a.ksplit);
  const uint32_t G1 = (uint32_t)((uint64_t)a.groups * (split + 1) / a.ksplit);
  const uint32_t ng = G1 - G0;
  const QmvSmem L = qmv_smem_layout(FMT, NT, SUB, a.gs, ng, min(a.batch, (uint32_t)kBatchChunk));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L.bars);
  uint8_t* ring = smem + L.ring;
  uint8_t* xf = smem + L.xf;
  float* gsx = reinterpret_cast<float*>(smem + L.gsx);
  float* gsum = reinterpret_cast<float*>(smem + L.gsum);
  int* gsq = reinterpret_cast<int*>(smem + L.gsq);
  float* red = reinterpret_cast<float*>(smem + L.red);
  float* rms = reinterpret_cast<float*>(smem + L.rms);
  int* flag = reinterpret_cast<int*>(smem + L.flag);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t cnt_w = (ng > (uint32_t)warp) ? (ng - warp + kQmvWarps - 1) / kQmvWarps : 0;
  const uint32_t slot_bytes = SUB * seg;
  const uint32_t nslot = L.nslot;
  // per-warp item k -> (tile pcta + (k / cnt_w) * P, group G0 + warp + (k % cnt_w) * 4)
  auto item_src = [&](uint32_t k) -> const uint8_t* {
    const uint32_t tl = pcta + (k / cnt_w) * a.P;
    const uint32_t gi = G0 + warp + (k % cnt_w) * kQmvWarps;
    return a.w + ((size_t)tl * a.groups + gi) * slot_bytes;
  };
  const uint32_t nitems = cnt_w * ntc;

  if (lane == 0) {
    for (int s = 0; s < kQmvRing; ++s) mbar_init(&bars[warp * kQmvRing + s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  // Weight prefetch: constant data, safe before the grid dependency wait.
  if (lane == 0) {
    for (uint32_t k = 0; k < nitems && k < nslot; ++k) {
      uint64_t* bar = &bars[warp * kQmvRing + k];
      mbar_arrive_expect_tx(bar, slot_bytes);
      bulk_g2s(ring + (size_t)(warp * nslot + k) * slot_bytes, item_src(k), slot_bytes, bar);
    }
  }

  pdl_wait();
  pdl_launch();

  // ---------------- prologue: x -> per-group fixed point B fragments ------
  // Stage the CTA's slice of x as fp16 in shared memory with wide, fully
  // parallel loads (every load of a thread is issued before any is used),
  // then quantize per (row, group) from shared memory.
  const uint32_t xf_words = ng * cpg * NT * 64;  // u32 words
  for (uint32_t i = threadIdx.x; i < xf_words; i += kQmvThreads) reinterpret_cast<uint32_t*>(xf)[i] = 0;
  for (uint32_t i = threadIdx.x; i < ng * kBatchChunk; i += kQmvThreads) {
    gsx[i] = 0.f; gsum[i] = 0.f; gsq[i] = 0;
  }
  if (threadIdx.x < kBatchChunk) rms[threadIdx.x] = 0.f;
  const uint32_t K0 = G0 * a.gs, Kr = ng * a.gs;
  __half* xs = reinterpret_cast<__half*>(smem + L.xs);   // [bc][Kr]
  __syncthreads();
  if constexpr (PRO == PRO_NORM) {
    const float* res = static_cast<const float*>(a.x) + (size_t)b0 * a.x_stride;
    const uint32_t q4 = a.K / 4, n4 = bc * q4;
    float ssr[kBatchChunk];
#pragma unroll
    for (int bb = 0; bb < kBatchChunk; ++bb) ssr[bb] = 0.f;
    for (uint32_t j0 = threadIdx.x; j0 < n4; j0 += 4 * kQmvThreads) {
      float4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t j = j0 + u * kQmvThreads;
        v[u] = j < n4 ? *reinterpret_cast<const float4*>(res + (size_t)(j / q4) * a.x_stride + 4 * (j % q4))
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
    if (threadIdx.x < bc) rms[threadIdx.x] = rsqrtf(rms[threadIdx.x] / (float)a.K + a.eps);
    __syncthreads();
    const uint32_t r4 = Kr / 4, m4 = bc * r4;
    for (uint32_t j0 = threadIdx.x; j0 < m4; j0 += 4 * kQmvThreads) {
      float4 v[4], w[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t j = j0 + u * kQmvThreads;
        if (j < m4) {
          const uint32_t k = K0 + 4 * (j % r4);
          v[u] = *reinterpret_cast<const float4*>(res + (size_t)(j / r4) * a.x_stride + k);
          w[u] = *reinterpret_cast<const float4*>(a.norm_w + k);
        }
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t j = j0 + u * kQmvThreads;
        if (j < m4) {
          const float rr = rms[j / r4];
          float o0 = v[u].x * rr * w[u].x, o1 = v[u].y * rr * w[u].y;
          float o2 = v[u].z * rr * w[u].z, o3 = v[u].w * rr * w[u].w;
          if (a.bf16_round) { o0 = bf16_trunc(o0); o1 = bf16_trunc(o1); o2 = bf16_trunc(o2); o3 = bf16_trunc(o3); }
          __half2* dst = reinterpret_cast<__half2*>(xs + (size_t)(j / r4) * Kr + 4 * (j % r4));
          dst[0] = __floats2half2_rn(o0, o1);
          dst[1] = __floats2half2_rn(o2, o3);
        }
      }
    }
  } else {
    const __half* xh = static_cast<const __half*>(a.x) + (size_t)b0 * a.x_stride;
    const uint32_t r8 = Kr / 8, m8 = bc * r8;
    for (uint32_t j0 = threadIdx.x; j0 < m8; j0 += 4 * kQmvThreads) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t j = j0 + u * kQmvThreads;
        if (j < m8) v[u] = *reinterpret_cast<const uint4*>(xh + (size_t)(j / r8) * a.x_stride + K0 + 8 * (j % r8));
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t j = j0 + u * kQmvThreads;
        if (j < m8) *reinterpret_cast<uint4*>(xs + (size_t)(j / r8) * Kr + 8 * (j % r8)) = v[u];
      }
    }
  }
  __syncthreads();
  {
    const uint32_t gs = a.gs, per_lane = gs / 32;
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
      int E = 0;
      if (amax > 0.f) frexpf(amax, &E);
      int qsum = 0;
      const uint32_t nt = b >> 2, ncol = 2 * (b & 3);
#pragma unroll
      for (uint32_t m = 0; m < 8; ++m) {
        if (m < per_lane) {
          const int q = (amax > 0.f) ? __float2int_rn(ldexpf(xv[m], 14 - E)) : 0;
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
        gsx[gl * kBatchChunk + b] = (amax > 0.f) ? ldexpf(1.f, E - 14) : 0.f;
        gsum[gl * kBatchChunk + b] = sumx;
        gsq[gl * kBatchChunk + b] = qsum;
      }
    }
  }
  __syncthreads();

  // ---------------- main loop --------------------------------------------
  const int g = lane >> 2, t = lane & 3;
  bool failed = false;
  for (uint32_t ti = 0; ti < ntc; ++ti) {
  const uint32_t tile = pcta + ti * a.P;
  float y[SUB][NT][16];
#pragma unroll
  for (int s = 0; s < SUB; ++s)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int v = 0; v < 16; ++v) y[s][n][v] = 0.f;

  for (uint32_t kk = 0; kk < cnt_w; ++kk) {
    const uint32_t k = ti * cnt_w + kk;
    const uint32_t slot = k % nslot;
    uint64_t* bar = &bars[warp * kQmvRing + slot];
    if (!failed) failed = !mbar_wait(bar, (k / nslot) & 1u, a.err);
    const uint32_t gl = warp + kk * kQmvWarps;  // group within CTA range
    const uint8_t* sb = ring + (size_t)(warp * nslot + slot) * slot_bytes;
#pragma unroll
    for (int s = 0; s < SUB; ++s) {
      const uint8_t* segp = sb + s * seg;
#pragma unroll
      for (int n = 0; n < NT; ++n) {
        const uint32_t bcol = n * 4 + t;
        const float sx = gsx[gl * kBatchChunk + bcol];
        if constexpr (FMT == FMT_Q1) {
          int D[8][4];
#pragma unroll
          for (int j = 0; j < 8; ++j) D[j][0] = D[j][1] = D[j][2] = D[j][3] = 0;
#pragma unroll 1
          for (uint32_t cc = 0; cc < cpg; ++cc) {
            const uint4 A = *reinterpret_cast<const uint4*>(segp + cc * 512 + lane * 16);
            const uint2 B = *reinterpret_cast<const uint2*>(
                xf + ((size_t)((gl * cpg + cc) * NT + n) * 32 + lane) * 8);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const uint32_t msk = 0x01010101u << j;
              mma_u8s8(D[j], A.x & msk, A.y & msk, A.z & msk, A.w & msk, B.x, B.y);
            }
          }
          const uint4 s0 = *reinterpret_cast<const uint4*>(segp + cpg * 512 + g * 32);
          const uint4 s1 = *reinterpret_cast<const uint4*>(segp + cpg * 512 + g * 32 + 16);
          const uint16_t* sc0 = reinterpret_cast<const uint16_t*>(&s0);
          const uint16_t* sc1 = reinterpret_cast<const uint16_t*>(&s1);
          const int sq = gsq[gl * kBatchChunk + bcol];
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
    __syncwarp();
    if (lane == 0 && k + nslot < nitems) {
      mbar_arrive_expect_tx(bar, slot_bytes);
      bulk_g2s(ring + (size_t)(warp * nslot + slot) * slot_bytes, item_src(k + nslot), slot_bytes, bar);
    }
  }

  // ---------------- CTA reduction ----------------------------------------
  {
    float* rw = red + (size_t)warp * kTileRows * SUB * kBatchChunk;
#pragma unroll
    for (int s = 0; s < SUB; ++s)
#pragma unroll
      for (int n = 0; n < NT; ++n)
#pragma unroll
        for (int v = 0; v < 16; ++v) {
          uint32_t row;
          if constexpr (FMT == FMT_Q1) row = 16 * (v >> 1) + g + 8 * (v & 1);
          else row = 32 * (v >> 2) + g + ((v & 3) == 0 ? 0 : (v & 3) == 1 ? 8 : (v & 3) == 2 ? 16 : 24);
          rw[(s * kTileRows + row) * kBatchChunk + n * 4 + t] = y[s][n][v];
        }
  }
  __syncthreads();
  const uint32_t nval = kTileRows * SUB * kBatchChunk;
  for (uint32_t i = threadIdx.x; i < nval; i += kQmvThreads) {
    float v = 0.f;
#pragma unroll
    for (int w = 0; w < kQmvWarps; ++w) v += red[(size_t)w * nval + i];
    red[i] = v;
  }
  bool last = true;
  if (a.ksplit > 1) {
    // Split-K: partials of the bc live batch columns go to the workspace;
    // the last CTA of the tile sums them in split order (8 loads in flight
    // per step) and runs the epilogue.
    __syncthreads();
    const uint32_t bcm = min(a.batch, (uint32_t)kBatchChunk);
    const uint32_t nvc = kTileRows * SUB * bcm;
    float* wsp = a.ws + ((size_t)(ychunk * a.tiles + tile) * a.ksplit) * nvc;
    for (uint32_t i = threadIdx.x; i < nvc; i += kQmvThreads)
      wsp[(size_t)split * nvc + i] = red[(i / bcm) * kBatchChunk + (i % bcm)];
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
      const uint32_t prev = atomicAdd(&a.counters[ychunk * a.tiles + tile], 1u);
      flag[0] = (prev == a.ksplit - 1);
    }
    __syncthreads();
    last = flag[0] != 0;
    if (last) {
    __threadfence();
    for (uint32_t i0 = threadIdx.x; i0 < nvc; i0 += 2 * kQmvThreads) {
      float acc[2] = {0.f, 0.f};
      for (uint32_t s0 = 0; s0 < a.ksplit; s0 += 8) {
        float t[2][8];
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const uint32_t i = i0 + u * kQmvThreads;
            t[u][j] = (i < nvc && s0 + j < a.ksplit) ? __ldcg(&wsp[(size_t)(s0 + j) * nvc + i]) : 0.f;
          }
#pragma unroll
        for (int u = 0; u < 2; ++u)
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[u] += t[u][j];
      }
#pragma unroll
      for (int u = 0; u < 2; ++u) {
        const uint32_t i = i0 + u * kQmvThreads;
        if (i < nvc) red[(i / bcm) * kBatchChunk + (i % bcm)] = acc[u];
      }
    }
    if (threadIdx.x == 0) a.counters[ychunk * a.tiles + tile] = 0;
    }
  }
  __syncthreads();
  if (last) {

  // ---------------- epilogue ---------------------------------------------
  const bool rb = a.bf16_round != 0;
  if constexpr (EPI == EPI_LOGITS) {
    unsigned long long best[kBatchChunk];
#pragma unroll
    for (int b = 0; b < kBatchChunk; ++b) best[b] = 0ull;
    for (uint32_t i = threadIdx.x; i < kTileRows * kBatchChunk; i += kQmvThreads) {
      const uint32_t r = i / kBatchChunk, b = i % kBatchChunk;
      const uint32_t row = tile * kTileRows + r;
      if (row >= a.M || b >= bc) continue;
      float v = red[i];
      if (rb) v = bf16_trunc(v);
      if (a.logits) a.logits[(size_t)(b0 + b) * a.logits_stride + row] = v;
      const unsigned long long pk = argmax_pack(v, row);
#pragma unroll
      for (int bb = 0; bb < kBatchChunk; ++bb)
        if (bb == (int)b && pk > best[bb]) best[bb] = pk;
    }
#pragma unroll
    for (int b = 0; b < kBatchChunk; ++b) {
      unsigned long long v = best[b];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long u = __shfl_xor_sync(0xffffffffu, v, o);
        v = u > v ? u : v;
      }
      if (lane == 0 && (uint32_t)b < bc && v) atomicMax(&a.argmax[b0 + b], v);
    }
  } else {
    // compact (row, live column) index; residual-add reads of up to 4 items
    // per thread are issued before their stores
    const uint32_t n = kTileRows * bc;
    for (uint32_t i0 = threadIdx.x; i0 < n; i0 += 4 * kQmvThreads) {
      float v[4], old[4];
      size_t o[4];
      bool ok[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const uint32_t i = i0 + u * kQmvThreads;
        const uint32_t r = i / bc, b = i % bc;
        const uint32_t row = tile * kTileRows + r;
        ok[u] = i < n && row < a.M;
        o[u] = (size_t)(b0 + b) * a.out_stride + row;
        v[u] = ok[u] ? red[r * kBatchChunk + b] : 0.f;
        if constexpr (EPI == EPI_SILU) {
          const float gv = v[u], uv = ok[u] ? red[kTileRows * kBatchChunk + r * kBatchChunk + b] : 0.f;
          v[u] = gv / (1.0f + expf(-gv)) * uv;
        }
        if constexpr (EPI == EPI_RESADD) old[u] = ok[u] ? static_cast<float*>(a.out)[o[u]] : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        if (!ok[u]) continue;
        float x = v[u];
        if (rb) x = bf16_trunc(x);
        if constexpr (EPI == EPI_F16 || EPI == EPI_SILU) static_cast<__half*>(a.out)[o[u]] = __float2half_rn(x);
        else if constexpr (EPI == EPI_F32) static_cast<float*>(a.out)[o[u]] = x;
        else static_cast<float*>(a.out)[o[u]] = old[u] + x;
      }
    }
  }
  }   // if (last)
  __syncthreads();   // red is rewritten by the next tile
  }   // tile loop
}

// Host launcher (qmv.cu).  Picks ksplit and the template instance.
struct QmvLaunch {
  int fmt, sub, pro, epi, bf16_scales;
  int pdl;
};
cudaError_t qmv_launch(const QmvLaunch& L, QmvArgs a, int num_sms, cudaStream_t st);
// Raise the dynamic shared-memory limit of every instance on the current
// device.  Call once per device before the first launch or capture.
cudaError_t qmv_prepare();
// Workspace bytes / counter count a launch with these shapes may touch.
size_t qmv_ws_floats(uint32_t M, uint32_t K, uint32_t gs, int fmt, int sub, uint32_t batch,
                     int num_sms);
uint32_t qmv_pick_ksplit(uint32_t M, uint32_t K, uint32_t gs, int fmt, int sub, uint32_t batch,
                         int num_sms);

}  // namespace nnz
