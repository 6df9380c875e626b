// Decode attention on the tensor cores (head_dim 128, GQA group 1, 2 or 4).
//
// Same result as attn_decode_kernel (q = RoPE(RMSNorm_hd(q) * qn) in f32,
// scores q.k / sqrt(hd) in f32, f32 softmax, fp16 output; reference
// nnmetal/src/shaders/transformer.metal:1467-1695), reorganised so that a
// batch of long sequences streams the KV cache at HBM speed:
//
//  1. attn_tc_prep_kernel, one CTA per (kv head, row): QK-norm + RoPE of the
//     G query heads, stored as fp16 hi/lo pairs (q = hi + lo to ~22 bits),
//     and (decode) the new K/V written into the cache at `pos`.
//  2. attn_tc_kernel, persistent: every warp owns a stream of tasks
//     (row, kv head, 256-position chunk) and a private 3-stage shared-memory
//     ring of 16-position K/V blocks, each loaded by four 2-D TMA copies
//     (K and V, head dims 0-63 and 64-127) with the 128-byte swizzle, so
//     ldmatrix reads are conflict-free.
//     S = Q.K^T and O += P.V run as mma.m16n8k16 (f16 in, f32 accumulate)
//     with A rows [q_hi(G) | q_lo(G)] and [p_hi(G) | p_lo(G)], so each f32
//     operand enters the tensor core as an exact-to-2^-22 pair; the online
//     softmax keeps its statistics in the score fragments' lanes.  The ring
//     runs ahead across task boundaries, so a warp never drains it.
//  3. attn_tc_combine_kernel, one CTA per (kv head, row): merges the
//     chunks' (m, l, o) and writes the fp16 output.
#include <cuda.h>
#include <cuda_runtime.h>
#include <math.h>

#include "attn.cuh"
#include "gemm.cuh"
#include "rope_dev.cuh"

namespace nnz {

namespace {

constexpr int kHD = 128;
constexpr int kTcWarps = 4;
constexpr int kTcBlk = 16;              // positions per streamed block
constexpr int kTcStages = 3;
constexpr int kTcRowB = kHD * 2 + 16;   // padded shared-memory row (bytes)
constexpr int kTcBoxB = kTcBlk * 128;            // one TMA box: 16 rows x 64 dims (fp16)
constexpr int kTcSlotB = 4 * kTcBoxB;             // K dims 0-63, K 64-127, V 0-63, V 64-127
constexpr int kTcWarpB = kTcStages * kTcSlotB + 1024;   // + barriers, padded to the 1 KB swizzle atom
constexpr int kTcSmem = kTcWarps * kTcWarpB + 1024;     // + alignment slack
constexpr int kTcQRows = 8;             // hi/lo query rows per (row, kv head)

__host__ __device__ inline uint32_t tc_chunks(uint32_t max_ctx) { return (max_ctx + kTcChunk - 1) / kTcChunk; }

struct TcArgs {
  CUtensorMap tmK, tmV;   // the layer's K / V cache as [slots * n_kv * max_ctx][hd] fp16 rows
  AttnArgs a;
  uint32_t nch;        // chunks per (row, kv head) at max_ctx
  uint32_t ntasks;
  float* part;         // [rows][n_kv][nch][G][hd + 2]
  __half* q16;         // [rows][n_kv][8][hd]
};

__device__ __forceinline__ int clamp_pos(const AttnArgs& a, uint32_t row, bool report) {
  int p = a.pos[row];
  if (p < 0 || p >= (int)a.max_ctx) {
    if (report) atomicOr(a.err, ERR_BAD_POS);
    p = p < 0 ? 0 : (int)a.max_ctx - 1;
  }
  return p;
}

// ---------------------------------------------------------------------------
// 1. query prep (+ KV write)
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(160) attn_tc_prep_kernel(TcArgs t) {
  constexpr int EPL = kHD / 32;
  const AttnArgs& a = t.a;
  pdl_wait();
  pdl_launch();
  const int kvh = blockIdx.x, row = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (int)(a.n_q / a.n_kv);
  const int p = clamp_pos(a, row, threadIdx.x == 0);
  const __half* qrow = a.qkv + (size_t)row * a.qkv_stride;
  __half* q16 = t.q16 + ((size_t)row * a.n_kv + kvh) * kTcQRows * kHD;
  if (warp < G) {
    float v[EPL];
    norm_rope_head<kHD>(qrow + (size_t)(kvh * G + warp) * kHD, a.q_norm, a.eps, a.theta, a.rope_style, p,
                        lane, v, a.rope_tab ? a.rope_tab + (size_t)p * (kHD / 2) : nullptr);
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const __half hi = __float2half_rn(v[e]);
      const __half lo = __float2half_rn(v[e] - __half2float(hi));
      q16[(size_t)warp * kHD + lane * EPL + e] = hi;
      q16[(size_t)(G + warp) * kHD + lane * EPL + e] = lo;
    }
  } else if (warp == 4 && a.write_kv) {
    const int slot = a.slot ? a.slot[row] : row;
    const size_t off = (((size_t)slot * a.n_kv + kvh) * a.max_ctx + p) * kHD;
    float v[EPL];
    norm_rope_head<kHD>(qrow + (size_t)a.n_q * kHD + (size_t)kvh * kHD, a.k_norm, a.eps, a.theta,
                        a.rope_style, p, lane, v,
                        a.rope_tab ? a.rope_tab + (size_t)p * (kHD / 2) : nullptr);
    const __half* vsrc = qrow + (size_t)(a.n_q + a.n_kv) * kHD + (size_t)kvh * kHD;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      a.kc[off + lane * EPL + e] = __float2half_rn(v[e]);
      a.vc[off + lane * EPL + e] = vsrc[lane * EPL + e];
    }
  }
}

// ---------------------------------------------------------------------------
// 2. streaming attention
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                        uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  const __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* tm, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(tm)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

// Shared address of 16-byte chunk `ch` (0-15: head dims 8ch..8ch+7) of row
// r of a 16-row K or V tile stored as two 128B-swizzled TMA boxes.
__device__ __forceinline__ uint32_t swz(uint32_t tile, int r, int ch) {
  return tile + (ch >> 3) * kTcBoxB + r * 128 + (((ch & 7) ^ (r & 7)) << 4);
}

// One task's cache range; false when the chunk lies past the row's position.
struct TcTask {
  uint32_t row, kvh, c;
  int npos, nblk;
  uint32_t row0;   // cache row (of the 2-D view) of the chunk's first position
};

// Tasks are numbered chunk-major (all rows' chunk 0, then chunk 1, ...), so
// the chunks that exist at the current positions are spread evenly over the
// warps' grid-stride sequences.
__device__ __forceinline__ bool tc_task(const TcArgs& t, uint32_t task, TcTask& k) {
  const AttnArgs& a = t.a;
  const uint32_t nrk = a.rows * a.n_kv;
  k.c = task / nrk;
  const uint32_t rk = task % nrk;
  k.kvh = rk % a.n_kv;
  k.row = rk / a.n_kv;
  const int seq = clamp_pos(a, k.row, false) + 1;
  const int t0 = (int)k.c * kTcChunk;
  if (t0 >= seq) return false;
  k.npos = min(kTcChunk, seq - t0);
  k.nblk = (k.npos + kTcBlk - 1) / kTcBlk;
  const int slot = a.slot ? a.slot[k.row] : (int)k.row;
  k.row0 = ((uint32_t)slot * a.n_kv + k.kvh) * a.max_ctx + (uint32_t)t0;
  return true;
}

template <int G>
__global__ void __launch_bounds__(kTcWarps * 32) attn_tc_kernel(const __grid_constant__ TcArgs t) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const AttnArgs& a = t.a;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q4 = lane & 3;
  uint8_t* ring = smem + warp * kTcWarpB;
  uint64_t* bars = reinterpret_cast<uint64_t*>(ring + kTcStages * kTcSlotB);
  if (lane == 0) {
    for (int s = 0; s < kTcStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
  }
  __syncwarp();
  pdl_wait();
  pdl_launch();
  const uint32_t stride = gridDim.x * kTcWarps;
  const uint32_t first = blockIdx.x * kTcWarps + warp;
  bool failed = false;

  // producer cursor: next block to copy
  uint32_t ptask = first;
  TcTask pk;
  bool pvalid = false;
  while (ptask < t.ntasks && !(pvalid = tc_task(t, ptask, pk))) ptask += stride;
  int pblk = 0;
  auto issue = [&](int stg) {
    uint8_t* slot = ring + stg * kTcSlotB;
    // the slot was last read (and possibly zeroed) through the generic proxy
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0) {
      mbar_arrive_expect_tx(&bars[stg], (uint32_t)kTcSlotB);
      const int y = (int)(pk.row0 + (uint32_t)(pblk * kTcBlk));
      tma_load_2d(slot, &t.tmK, 0, y, &bars[stg]);
      tma_load_2d(slot + kTcBoxB, &t.tmK, 64, y, &bars[stg]);
      tma_load_2d(slot + 2 * kTcBoxB, &t.tmV, 0, y, &bars[stg]);
      tma_load_2d(slot + 3 * kTcBoxB, &t.tmV, 64, y, &bars[stg]);
    }
    __syncwarp();
    if (++pblk == pk.nblk) {
      pblk = 0;
      pvalid = false;
      ptask += stride;
      while (ptask < t.ntasks && !(pvalid = tc_task(t, ptask, pk))) ptask += stride;
    }
  };
  int pstg = 0;
  for (int s = 0; s < kTcStages && pvalid; ++s) {
    issue(pstg);
    pstg = pstg + 1 == kTcStages ? 0 : pstg + 1;
  }

  uint32_t ctask = first;
  int cstg = 0;
  uint32_t cphase = 0;   // bit s: parity of stage s
  const float inv = rsqrtf((float)kHD);
  for (;;) {
    TcTask ck;
    bool cvalid = false;
    while (ctask < t.ntasks && !(cvalid = tc_task(t, ctask, ck))) ctask += stride;
    if (!cvalid) break;
    // query fragments: rows g < 2G (hi then lo), zero above
    uint32_t qa[8][2];
    {
      const __half* qp = t.q16 + ((size_t)ck.row * a.n_kv + ck.kvh) * kTcQRows * kHD + (size_t)g * kHD;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        qa[ks][0] = g < 2 * G ? __ldcg(reinterpret_cast<const unsigned int*>(qp + 16 * ks + 2 * q4)) : 0u;
        qa[ks][1] = g < 2 * G ? __ldcg(reinterpret_cast<const unsigned int*>(qp + 16 * ks + 8 + 2 * q4)) : 0u;
      }
    }
    float o[16][4];
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    float m = -INFINITY, l = 0.f;
    for (int blk = 0; blk < ck.nblk; ++blk) {
      if (!failed) failed = !mbar_wait(&bars[cstg], (cphase >> cstg) & 1u, a.err);
      cphase ^= 1u << cstg;
      const uint32_t kbase = smem_u32(ring + cstg * kTcSlotB);
      const uint32_t vbase = kbase + 2 * kTcBoxB;
      const int nvalid = ck.npos - blk * kTcBlk;
      if (nvalid < kTcBlk) {
        // rows past the chunk hold other positions (or zero fill): zero V so
        // that 0-probability * V stays 0 whatever they contain
        for (int i = lane; i < (kTcBlk - nvalid) * 16; i += 32) {
          const int r = nvalid + i / 16, part = i % 16;   // 16 x 16 bytes per row (two boxes)
          const uint32_t ad = vbase + (part / 8) * kTcBoxB + r * 128 + (part % 8) * 16;
          asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(ad), "r"(0u) : "memory");
        }
        __syncwarp();
      }
      // S = Q K^T for 16 positions (two n-tiles of 8)
      float s[2][4];
#pragma unroll
      for (int nt = 0; nt < 2; ++nt) {
        s[nt][0] = s[nt][1] = s[nt][2] = s[nt][3] = 0.f;
#pragma unroll
        for (int kq = 0; kq < 4; ++kq) {
          uint32_t r0, r1, r2, r3;
          ldsm_x4(swz(kbase, nt * 8 + (lane & 7), 4 * kq + (lane >> 3)), r0, r1, r2, r3);
          mma_f16(s[nt], qa[2 * kq][0], 0u, qa[2 * kq][1], 0u, r0, r1);
          mma_f16(s[nt], qa[2 * kq + 1][0], 0u, qa[2 * kq + 1][1], 0u, r2, r3);
        }
      }
      // hi + lo rows, scale, mask
      float sv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float x = s[i >> 1][i & 1];
        const float y = __shfl_xor_sync(0xffffffffu, x, 4 * G);
        const int pl = (i >> 1) * 8 + 2 * q4 + (i & 1);
        sv[i] = pl < nvalid ? (x + y) * inv : -INFINITY;
      }
      float mx = fmaxf(fmaxf(sv[0], sv[1]), fmaxf(sv[2], sv[3]));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
      mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
      const float mn = fmaxf(m, mx);
      const float al = m == -INFINITY ? 0.f : expf(m - mn);
      m = mn;
      float pv[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) pv[i] = expf(sv[i] - mn);
      l = l * al + (pv[0] + pv[1] + pv[2] + pv[3]);
#pragma unroll
      for (int j = 0; j < 16; ++j) { o[j][0] *= al; o[j][1] *= al; }
      // P fragments: rows g < G carry fp16(p), rows G..2G-1 the residual
      uint32_t pa0, pa2;
      if (g < G) {
        pa0 = pack_h2(pv[0], pv[1]);
        pa2 = pack_h2(pv[2], pv[3]);
      } else if (g < 2 * G) {
        pa0 = pack_h2(pv[0] - __half2float(__float2half_rn(pv[0])), pv[1] - __half2float(__float2half_rn(pv[1])));
        pa2 = pack_h2(pv[2] - __half2float(__float2half_rn(pv[2])), pv[3] - __half2float(__float2half_rn(pv[3])));
      } else {
        pa0 = pa2 = 0u;
      }
      // O += P V
#pragma unroll
      for (int jp = 0; jp < 8; ++jp) {
        uint32_t r0, r1, r2, r3;
        ldsm_x4_t(swz(vbase, (lane & 7) + 8 * ((lane >> 3) & 1), 2 * jp + (lane >> 4)), r0, r1, r2, r3);
        mma_f16(o[2 * jp], pa0, 0u, pa2, 0u, r0, r1);
        mma_f16(o[2 * jp + 1], pa0, 0u, pa2, 0u, r2, r3);
      }
      __syncwarp();
      if (pvalid) issue(cstg);   // refill the slot just consumed
      cstg = cstg + 1 == kTcStages ? 0 : cstg + 1;
    }
    // task epilogue: full row sums, hi + lo output rows, partial record
    l += __shfl_xor_sync(0xffffffffu, l, 1);
    l += __shfl_xor_sync(0xffffffffu, l, 2);
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      o[j][0] += __shfl_xor_sync(0xffffffffu, o[j][0], 4 * G);
      o[j][1] += __shfl_xor_sync(0xffffffffu, o[j][1], 4 * G);
    }
    if (g < G) {
      float* rec = t.part + ((((size_t)ck.row * a.n_kv + ck.kvh) * t.nch + ck.c) * G + g) * (kHD + 2);
      if (q4 == 0) { rec[0] = m; rec[1] = l; }
#pragma unroll
      for (int j = 0; j < 16; ++j)
        *reinterpret_cast<float2*>(rec + 2 + 8 * j + 2 * q4) = make_float2(o[j][0], o[j][1]);
    }
    ctask += stride;
  }
}

// ---------------------------------------------------------------------------
// 3. merge the chunks
// ---------------------------------------------------------------------------
// Thread (head h, dim d) of a (kv head, row); up to 16 chunks' loads are
// in flight before any is used.
__global__ void __launch_bounds__(4 * kHD) attn_tc_combine_kernel(TcArgs t) {
  constexpr int kB = 16;
  const AttnArgs& a = t.a;
  pdl_wait();
  pdl_launch();
  const int kvh = blockIdx.x, row = blockIdx.y, d = threadIdx.x % kHD, h = threadIdx.x / kHD;
  const uint32_t G = a.n_q / a.n_kv;
  const int seq = clamp_pos(a, row, false) + 1;
  const uint32_t nc = (uint32_t)(seq + kTcChunk - 1) / kTcChunk;
  const float* base = t.part + (((size_t)row * a.n_kv + kvh) * t.nch * G + h) * (kHD + 2);
  const size_t cs = (size_t)G * (kHD + 2);
  float M = -INFINITY, L = 0.f, o = 0.f;
  for (uint32_t c0 = 0; c0 < nc; c0 += kB) {
    float mv[kB], lv[kB], ov[kB];
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const bool ok = c0 + j < nc;
      const float* r = base + (c0 + j) * cs;
      mv[j] = ok ? __ldcg(r) : -INFINITY;
      lv[j] = ok ? __ldcg(r + 1) : 0.f;
      ov[j] = ok ? __ldcg(r + 2 + d) : 0.f;
    }
    float nm = M;
#pragma unroll
    for (int j = 0; j < kB; ++j) nm = fmaxf(nm, mv[j]);
    const float a0 = M == -INFINITY ? 0.f : expf(M - nm);
    L *= a0;
    o *= a0;
#pragma unroll
    for (int j = 0; j < kB; ++j) {
      const float w = mv[j] == -INFINITY ? 0.f : expf(mv[j] - nm);
      L = fmaf(lv[j], w, L);
      o = fmaf(ov[j], w, o);
    }
    M = nm;
  }
  a.out[(size_t)row * a.out_stride + ((size_t)kvh * G + h) * kHD + d] = __float2half_rn(o / L);
}

// ---------------------------------------------------------------------------
// 4. causal prefill attention on the tensor cores
// ---------------------------------------------------------------------------
// One CTA per (kv head, block of query rows, key split): warp w serves
// query head w % G of the group and 16 consecutive rows (block = 16 * 4 / G
// rows), so every K/V tile in shared memory feeds all G heads; the block's
// causal key range is cut into up to kPfSplits splits of whole 64-key tiles
// (balancing the long rows against the short ones), each writing partial
// (m, l, o) records that attn_prefill_combine_kernel merges.  Each warp normalises
// and rotates its rows' queries (f32) and keeps them as fp16 hi/lo A
// fragments; S = Q_hi K^T + Q_lo K^T and O += P_hi V + P_lo V accumulate in
// f32, with the causal mask and the online softmax in registers (FA2
// layout: the score accumulators are the P operand).  64-position K/V tiles
// are double-buffered with cp.async into rows padded to 272 bytes.
constexpr int kPfTcKeys = 64;
constexpr int kPfTcQB = 2 * 16 * kTcRowB;                 // per warp: hi + lo, 16 rows
constexpr int kPfTcTile = kPfTcKeys * kTcRowB;            // one K or V tile
constexpr int kPfTcSmem = 4 * kPfTcQB + 2 * 2 * kPfTcTile;
constexpr int kPfSplits = 4;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(src) : "memory");
}

template <int G>
__global__ void __launch_bounds__(128) attn_prefill_tc_kernel(AttnArgs a) {
  constexpr int RG = 4 / G;                 // 16-row groups per CTA
  constexpr int QR = 16 * RG;               // query rows per CTA
  extern __shared__ __align__(128) uint8_t smem[];
  pdl_wait();
  pdl_launch();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, g = lane >> 2, q4 = lane & 3;
  const int kvh = blockIdx.x;
  const int hl = warp % G, rg = warp / G;
  const int h = kvh * G + hl;
  const uint32_t rbase = blockIdx.y * QR;
  uint8_t* qsm = smem + warp * kPfTcQB;
  uint8_t* kv = smem + 4 * kPfTcQB;

  // CTA key range: up to the largest position of its rows; rows share a slot
  __shared__ int s_kmax, s_slot;
  if (threadIdx.x == 0) {
    int mx = 0;
    for (int r = 0; r < QR; ++r)
      if (rbase + r < a.rows) mx = max(mx, min(max(a.pos[rbase + r], 0), (int)a.max_ctx - 1));
    s_kmax = mx;
    s_slot = a.slot ? a.slot[rbase] : (int)rbase;
  }
  __syncthreads();
  const int kmax = s_kmax;
  const size_t head_off = ((size_t)s_slot * a.n_kv + kvh) * a.max_ctx * kHD;
  // this split's key tiles [kb0, kb1)
  const int ntile = kmax / kPfTcKeys + 1;
  const int per = (ntile + kPfSplits - 1) / kPfSplits;
  const int kb0 = blockIdx.z * per, kb1 = min(ntile, kb0 + per);
  const uint32_t rec = kHD + 2;
  if (kb0 >= kb1) {
    // empty split: mark its records so the merge skips them
    if (lane < 16) {
      const uint32_t r = rbase + rg * 16 + lane;
      if (r < a.rows) a.ws[(((size_t)r * a.n_q + h) * kPfSplits + blockIdx.z) * rec] = -INFINITY;
    }
    return;
  }
  auto load_tile = [&](int kb, int stg) {
    const uint32_t kt = smem_u32(kv + stg * 2 * kPfTcTile), vt = kt + kPfTcTile;
    for (int c = threadIdx.x; c < kPfTcKeys * 16; c += 128) {
      const int r = c >> 4, ch = c & 15, t = kb * kPfTcKeys + r;
      const uint32_t off = r * kTcRowB + ch * 16;
      if (t <= kmax) {
        cp_async16(kt + off, a.kc + head_off + (size_t)t * kHD + ch * 8);
        cp_async16(vt + off, a.vc + head_off + (size_t)t * kHD + ch * 8);
      } else {
        // past the last query position: zero, so 0-probability * V stays 0
        asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(kt + off), "r"(0u) : "memory");
        asm volatile("st.shared.v4.b32 [%0], {%1,%1,%1,%1};" ::"r"(vt + off), "r"(0u) : "memory");
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };
  load_tile(kb0, 0);

  // queries: RMSNorm over the head, q_norm, RoPE (f32), then fp16 hi/lo rows
  {
    const int EPL = 4;
    int prow[16];
    float v[16][4];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t r = rbase + rg * 16 + i;
      const bool ok = r < a.rows;
      prow[i] = ok ? min(max(a.pos[r], 0), (int)a.max_ctx - 1) : 0;
      const __half* src = a.qkv + (size_t)(ok ? r : 0) * a.qkv_stride + (size_t)h * kHD + lane * EPL;
      const uint2 raw = ok ? *reinterpret_cast<const uint2*>(src) : make_uint2(0, 0);
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      v[i][0] = f0.x; v[i][1] = f0.y; v[i][2] = f1.x; v[i][3] = f1.y;
    }
    float nw[4];
#pragma unroll
    for (int e = 0; e < EPL; ++e) nw[e] = a.q_norm[lane * EPL + e];
    const double l2t = a.rope_tab ? 0.0 : log2((double)a.theta);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float ss = v[i][0] * v[i][0] + v[i][1] * v[i][1] + v[i][2] * v[i][2] + v[i][3] * v[i][3];
      ss = warp_sum(ss);
      const float rr = rsqrtf(ss / (float)kHD + a.eps);
#pragma unroll
      for (int e = 0; e < EPL; ++e) v[i][e] = v[i][e] * rr * nw[e];
      const float2* tab = a.rope_tab ? a.rope_tab + (size_t)prow[i] * (kHD / 2) : nullptr;
      if (a.rope_style == ROPE_PAIRWISE) {
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
          const float2 cs = rope_cs<kHD>(tab, l2t, prow[i], (lane * EPL + e) >> 1);
          const float x0 = v[i][e], x1 = v[i][e + 1];
          v[i][e] = x0 * cs.x - x1 * cs.y;
          v[i][e + 1] = x0 * cs.y + x1 * cs.x;
        }
      } else {
#pragma unroll
        for (int e = 0; e < EPL; ++e) {
          const float partner = __shfl_xor_sync(0xffffffffu, v[i][e], 16);
          const float2 cs = rope_cs<kHD>(tab, l2t, prow[i], (lane & 15) * EPL + e);
          v[i][e] = lane < 16 ? v[i][e] * cs.x - partner * cs.y : partner * cs.y + v[i][e] * cs.x;
        }
      }
      uint32_t hi[2], lo[2];
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const __half h0 = __float2half_rn(v[i][2 * e]), h1 = __float2half_rn(v[i][2 * e + 1]);
        const __half2 hh = __halves2half2(h0, h1);
        const __half2 ll = __floats2half2_rn(v[i][2 * e] - __half2float(h0), v[i][2 * e + 1] - __half2float(h1));
        hi[e] = *reinterpret_cast<const uint32_t*>(&hh);
        lo[e] = *reinterpret_cast<const uint32_t*>(&ll);
      }
      const uint32_t qa = smem_u32(qsm) + i * kTcRowB + lane * 8;
      asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(qa), "r"(hi[0]), "r"(hi[1]) : "memory");
      asm volatile("st.shared.v2.b32 [%0], {%1,%2};" ::"r"(qa + 16 * kTcRowB), "r"(lo[0]), "r"(lo[1]) : "memory");
    }
  }
  __syncwarp();
  // A fragments (row-major 16 x 16 per k-step) of q_hi and q_lo
  uint32_t qh[8][4], ql[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const uint32_t ad = smem_u32(qsm) + (lane & 15) * kTcRowB + (2 * ks + (lane >> 4)) * 16;
    ldsm_x4(ad, qh[ks][0], qh[ks][1], qh[ks][2], qh[ks][3]);
    ldsm_x4(ad + 16 * kTcRowB, ql[ks][0], ql[ks][1], ql[ks][2], ql[ks][3]);
  }
  int posg = -1, posg8 = -1;   // positions of this lane's rows g and g + 8
  {
    const uint32_t r0 = rbase + rg * 16 + g, r1 = r0 + 8;
    if (r0 < a.rows) posg = min(max(a.pos[r0], 0), (int)a.max_ctx - 1);
    if (r1 < a.rows) posg8 = min(max(a.pos[r1], 0), (int)a.max_ctx - 1);
  }
  int wmax = max(posg, posg8);
  wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, 4));
  wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, 8));
  wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, 16));

  float o[16][4];
#pragma unroll
  for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;
  const float inv = rsqrtf((float)kHD);
  for (int kb = kb0; kb < kb1; ++kb) {
    const int stg = (kb - kb0) & 1;
    if (kb + 1 < kb1) load_tile(kb + 1, stg ^ 1);
    else asm volatile("cp.async.commit_group;" ::: "memory");
    asm volatile("cp.async.wait_group 1;" ::: "memory");
    __syncthreads();
    if (kb * kPfTcKeys <= wmax) {
      const uint32_t kt = smem_u32(kv + stg * 2 * kPfTcTile), vt = kt + kPfTcTile;
      float sc[8][4];
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        sc[nt][0] = sc[nt][1] = sc[nt][2] = sc[nt][3] = 0.f;
#pragma unroll
        for (int kq = 0; kq < 4; ++kq) {
          uint32_t r0, r1, r2, r3;
          ldsm_x4(kt + (nt * 8 + (lane & 7)) * kTcRowB + (4 * kq + (lane >> 3)) * 16, r0, r1, r2, r3);
          mma_f16(sc[nt], qh[2 * kq][0], qh[2 * kq][1], qh[2 * kq][2], qh[2 * kq][3], r0, r1);
          mma_f16(sc[nt], ql[2 * kq][0], ql[2 * kq][1], ql[2 * kq][2], ql[2 * kq][3], r0, r1);
          mma_f16(sc[nt], qh[2 * kq + 1][0], qh[2 * kq + 1][1], qh[2 * kq + 1][2], qh[2 * kq + 1][3], r2, r3);
          mma_f16(sc[nt], ql[2 * kq + 1][0], ql[2 * kq + 1][1], ql[2 * kq + 1][2], ql[2 * kq + 1][3], r2, r3);
        }
      }
      // scale + causal mask, online softmax for rows g (c0, c1) and g + 8 (c2, c3)
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int t = kb * kPfTcKeys + nt * 8 + 2 * q4;
        sc[nt][0] = t <= posg ? sc[nt][0] * inv : -INFINITY;
        sc[nt][1] = t + 1 <= posg ? sc[nt][1] * inv : -INFINITY;
        sc[nt][2] = t <= posg8 ? sc[nt][2] * inv : -INFINITY;
        sc[nt][3] = t + 1 <= posg8 ? sc[nt][3] * inv : -INFINITY;
        mx0 = fmaxf(mx0, fmaxf(sc[nt][0], sc[nt][1]));
        mx1 = fmaxf(mx1, fmaxf(sc[nt][2], sc[nt][3]));
      }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
      const float al0 = n0 == -INFINITY ? 1.f : (m0 == -INFINITY ? 0.f : expf(m0 - n0));
      const float al1 = n1 == -INFINITY ? 1.f : (m1 == -INFINITY ? 0.f : expf(m1 - n1));
      m0 = n0;
      m1 = n1;
      float ps0 = 0.f, ps1 = 0.f;
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        sc[nt][0] = n0 == -INFINITY ? 0.f : expf(sc[nt][0] - n0);
        sc[nt][1] = n0 == -INFINITY ? 0.f : expf(sc[nt][1] - n0);
        sc[nt][2] = n1 == -INFINITY ? 0.f : expf(sc[nt][2] - n1);
        sc[nt][3] = n1 == -INFINITY ? 0.f : expf(sc[nt][3] - n1);
        ps0 += sc[nt][0] + sc[nt][1];
        ps1 += sc[nt][2] + sc[nt][3];
      }
      l0 = l0 * al0 + ps0;
      l1 = l1 * al1 + ps1;
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= al0; o[j][1] *= al0;
        o[j][2] *= al1; o[j][3] *= al1;
      }
      // O += P V, P as fp16 hi + lo
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ph[4], pl[4];
        const float* p0 = sc[2 * kk];
        const float* p1 = sc[2 * kk + 1];
        const float pv[8] = {p0[0], p0[1], p0[2], p0[3], p1[0], p1[1], p1[2], p1[3]};
        // a0: row g keys 2t..; a1: row g+8; a2: row g keys 8+2t..; a3: row g+8
        const int ord[4][2] = {{0, 1}, {2, 3}, {4, 5}, {6, 7}};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x = pv[ord[e][0]], y = pv[ord[e][1]];
          const __half hx = __float2half_rn(x), hy = __float2half_rn(y);
          const __half2 hh = __halves2half2(hx, hy);
          const __half2 ll = __floats2half2_rn(x - __half2float(hx), y - __half2float(hy));
          ph[e] = *reinterpret_cast<const uint32_t*>(&hh);
          pl[e] = *reinterpret_cast<const uint32_t*>(&ll);
        }
#pragma unroll
        for (int jp = 0; jp < 8; ++jp) {
          uint32_t r0, r1, r2, r3;
          ldsm_x4_t(vt + (kk * 16 + (lane & 7) + 8 * ((lane >> 3) & 1)) * kTcRowB + (2 * jp + (lane >> 4)) * 16,
                    r0, r1, r2, r3);
          mma_f16(o[2 * jp], ph[0], ph[1], ph[2], ph[3], r0, r1);
          mma_f16(o[2 * jp], pl[0], pl[1], pl[2], pl[3], r0, r1);
          mma_f16(o[2 * jp + 1], ph[0], ph[1], ph[2], ph[3], r2, r3);
          mma_f16(o[2 * jp + 1], pl[0], pl[1], pl[2], pl[3], r2, r3);
        }
      }
    }
    __syncthreads();
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  // partial records [row][head][split]: m, l, unnormalised o
  const uint32_t r0 = rbase + rg * 16 + g, r1 = r0 + 8;
  float* w0 = a.ws + (((size_t)r0 * a.n_q + h) * kPfSplits + blockIdx.z) * rec;
  float* w1 = a.ws + (((size_t)r1 * a.n_q + h) * kPfSplits + blockIdx.z) * rec;
  if (q4 == 0) {
    if (r0 < a.rows) { w0[0] = m0; w0[1] = l0; }
    if (r1 < a.rows) { w1[0] = m1; w1[1] = l1; }
  }
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = 8 * j + 2 * q4;
    if (r0 < a.rows) *reinterpret_cast<float2*>(w0 + 2 + d) = make_float2(o[j][0], o[j][1]);
    if (r1 < a.rows) *reinterpret_cast<float2*>(w1 + 2 + d) = make_float2(o[j][2], o[j][3]);
  }
}

// Merges the kPfSplits partial records of one (row, query head) into the
// fp16 output; one CTA per (row, head), a thread per element.
__global__ void __launch_bounds__(kHD) attn_prefill_combine_kernel(AttnArgs a) {
  pdl_wait();
  pdl_launch();
  const uint32_t r = blockIdx.x, h = blockIdx.y, d = threadIdx.x, rec = kHD + 2;
  const float* base = a.ws + ((size_t)r * a.n_q + h) * kPfSplits * rec;
  float mv[kPfSplits], lv[kPfSplits], ov[kPfSplits];
#pragma unroll
  for (int q = 0; q < kPfSplits; ++q) {
    mv[q] = __ldcg(base + q * rec);
    lv[q] = __ldcg(base + q * rec + 1);
    ov[q] = __ldcg(base + q * rec + 2 + d);
  }
  float M = -INFINITY;
#pragma unroll
  for (int q = 0; q < kPfSplits; ++q) M = fmaxf(M, mv[q]);
  float L = 0.f, o = 0.f;
#pragma unroll
  for (int q = 0; q < kPfSplits; ++q) {
    const float w = mv[q] == -INFINITY ? 0.f : expf(mv[q] - M);
    L = fmaf(w, lv[q], L);
    o = fmaf(w, ov[q], o);
  }
  a.out[(size_t)r * a.out_stride + (size_t)h * kHD + d] = __float2half_rn(o / L);
}

cudaLaunchConfig_t tc_cfg(dim3 grid, dim3 block, uint32_t smem, int pdl, cudaStream_t st, cudaLaunchAttribute* at) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cfg;
}

int g_tc_sms[64];

}  // namespace

bool attn_tc_applies(uint32_t n_q, uint32_t n_kv, int head_dim) {
  if (head_dim != kHD || n_kv == 0 || n_q % n_kv) return false;
  const uint32_t G = n_q / n_kv;
  return G == 1 || G == 2 || G == 4;
}

size_t attn_tc_ws_floats(uint32_t rows, uint32_t n_q, uint32_t n_kv, uint32_t max_ctx) {
  const size_t G = n_q / n_kv;
  return (size_t)rows * n_kv * tc_chunks(max_ctx) * G * (kHD + 2) + (size_t)rows * n_kv * kTcQRows * kHD / 2;
}

cudaError_t attn_tc_prepare() {
  cudaError_t e = cudaFuncSetAttribute(&attn_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(&attn_prefill_tc_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfTcSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(&attn_prefill_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfTcSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(&attn_prefill_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kPfTcSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(&attn_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(&attn_tc_kernel<4>, cudaFuncAttributeMaxDynamicSharedMemorySize, kTcSmem);
  return e;
}

cudaError_t attn_tc_launch(const AttnArgs& a, int pdl, cudaStream_t st) {
  if (!attn_tc_applies(a.n_q, a.n_kv, kHD) || a.rows == 0 || !a.ws) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
  if (!g_tc_sms[dev]) {
    int sms = 0;
    if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
    g_tc_sms[dev] = sms;
  }
  TcArgs t{};
  t.a = a;
  {
    const uint64_t rows = (uint64_t)(a.slots ? a.slots : a.rows) * a.n_kv * a.max_ctx;
    if (!tensor_map_f16_2d(&t.tmK, a.kc, kHD, rows, kHD * 2, 64, kTcBlk) ||
        !tensor_map_f16_2d(&t.tmV, a.vc, kHD, rows, kHD * 2, 64, kTcBlk))
      return cudaErrorInvalidValue;
  }
  t.nch = tc_chunks(a.max_ctx);
  t.ntasks = a.rows * a.n_kv * t.nch;
  const uint32_t G = a.n_q / a.n_kv;
  t.part = a.ws;
  t.q16 = reinterpret_cast<__half*>(a.ws + (size_t)a.rows * a.n_kv * t.nch * G * (kHD + 2));
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t c1 = tc_cfg(dim3(a.n_kv, a.rows), dim3(160), 0, pdl, st, at);
  if ((e = cudaLaunchKernelEx(&c1, &attn_tc_prep_kernel, t)) != cudaSuccess) return e;
  // two CTAs per SM; no more warps than tasks
  const uint32_t want = (t.ntasks + kTcWarps - 1) / kTcWarps;
  const uint32_t grid = want < 2u * g_tc_sms[dev] ? want : 2u * g_tc_sms[dev];
  cudaLaunchConfig_t c2 = tc_cfg(dim3(grid), dim3(kTcWarps * 32), kTcSmem, 1, st, at);
  if (G == 1) e = cudaLaunchKernelEx(&c2, &attn_tc_kernel<1>, t);
  else if (G == 2) e = cudaLaunchKernelEx(&c2, &attn_tc_kernel<2>, t);
  else e = cudaLaunchKernelEx(&c2, &attn_tc_kernel<4>, t);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t c3 = tc_cfg(dim3(a.n_kv, a.rows), dim3(kHD * G), 0, 1, st, at);
  return cudaLaunchKernelEx(&c3, &attn_tc_combine_kernel, t);
}

size_t attn_prefill_tc_ws_floats(uint32_t rows, uint32_t n_q) {
  return (size_t)rows * n_q * kPfSplits * (kHD + 2);
}

cudaError_t attn_prefill_tc_launch(const AttnArgs& a, int pdl, cudaStream_t st) {
  if (!attn_tc_applies(a.n_q, a.n_kv, kHD) || a.rows == 0 || !a.ws) return cudaErrorInvalidValue;
  const uint32_t G = a.n_q / a.n_kv, qr = 16 * (4 / G);
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t c = tc_cfg(dim3(a.n_kv, (a.rows + qr - 1) / qr, kPfSplits), dim3(128), kPfTcSmem, pdl, st, at);
  cudaError_t e;
  if (G == 1) e = cudaLaunchKernelEx(&c, &attn_prefill_tc_kernel<1>, a);
  else if (G == 2) e = cudaLaunchKernelEx(&c, &attn_prefill_tc_kernel<2>, a);
  else e = cudaLaunchKernelEx(&c, &attn_prefill_tc_kernel<4>, a);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t c2 = tc_cfg(dim3(a.rows, a.n_q), dim3(kHD), 0, 1, st, at);
  return cudaLaunchKernelEx(&c2, &attn_prefill_combine_kernel, a);
}

}  // namespace nnz
