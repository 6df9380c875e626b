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
#include "qmv_dev.cuh"

namespace nnz {

enum Prologue : int { PRO_F16 = 0, PRO_NORM = 1 };
enum Epilogue : int { EPI_F16 = 0, EPI_F32 = 1, EPI_RESADD = 2, EPI_SILU = 3, EPI_LOGITS = 4 };

constexpr int kQmvRing = 4;        // segment slots per warp

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
  const uint32_t K0 = G0 * a.gs, Kr = ng * a.gs;
  __half* xs = reinterpret_cast<__half*>(smem + L.xs);   // [bc][Kr]
  if constexpr (PRO == PRO_NORM) {
    const float* res = static_cast<const float*>(a.x) + (size_t)b0 * a.x_stride;
    block_rms(res, a.x_stride, a.K, bc, a.eps, rms);
    stage_norm(res, a.x_stride, a.norm_w, rms, K0, Kr, bc, a.bf16_round != 0, xs);
  } else {
    stage_f16(static_cast<const __half*>(a.x) + (size_t)b0 * a.x_stride, a.x_stride, K0, Kr, bc, xs);
  }
  quantize_xs<NT>(xs, Kr, bc, ng, a.gs, xf, gsx, gsum, gsq);

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
    qmv_group<FMT, NT, SUB, BF16S>(sb, seg, xf, gl, cpg, gsx, gsum, gsq, y);
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
          const uint32_t row = y_row<FMT>(v, g);
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
