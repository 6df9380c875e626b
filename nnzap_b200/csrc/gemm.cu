// tcgen05 prefill GEMM (see gemm.cuh).
#include <cuda.h>
#include <cuda_runtime.h>

#include "gemm.cuh"
#include "umma.cuh"

#include <stdlib.h>

namespace nnz {
namespace {

constexpr int kBM = 128, kBN = 128, kBK = 64;
constexpr uint32_t kTileBytes = kBM * kBK * 2;          // 16 KB per operand tile per stage
// MT 128-row M tiles per CTA share each dequantized weight tile: MT TMEM
// accumulators of 128 columns; ring stages of MT activation tiles + one
// weight tile, as many as fit (4 for MT <= 2, 2 for MT = 4).  (Per-tile
// activation slots with their own barriers, committed after each tile's
// MMAs, measured slower: 44 -> 69 us on a 512 x 2048 x 12288 GEMM.)
template <int MT> struct GemmShape {
  static constexpr int kStages = MT >= 4 ? 2 : (MT == 2 ? 4 : 6);
  static constexpr uint32_t kTmemCols = 128 * MT;
  static constexpr uint32_t kSmemBytes = kStages * (MT + 1) * kTileBytes + 1024 + 256;
};
constexpr int kGroups = 2;        // dequantizing groups of 4 warps, K steps dealt round robin
// Every stage must always be filled by the same group (stage = step %
// kStages, group = step % kGroups): a group that fills stages of several
// groups can run a whole phase ahead on a stage's empty barrier, where a
// parity wait cannot tell the pending phase from the completed one.
static_assert(GemmShape<1>::kStages % kGroups == 0 && GemmShape<2>::kStages % kGroups == 0 &&
                  GemmShape<4>::kStages % kGroups == 0,
              "ring stages must be a multiple of the dequantizing groups");
constexpr int kThreads = 128 + 128 * kGroups;
constexpr int kProducerWarps = 4;   // full-barrier arrivals per stage: one per warp of the filling group
constexpr int kPf = 4;            // raw-weight prefetch depth (steps of a producer group)

// Vector f32 reduction into global memory (16-byte aligned address).
__device__ __forceinline__ void red_add_f32x4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Raw weights of one row for one 64-wide K step.
struct Raw {
  uint4 q0, q1;    // Q1: q0.x/y = 64 sign bits; Q4: 32 bytes of nibbles
  uint16_t s, b;
};

// Row base pointers of one weight row (bits / nibbles, scales, biases).
struct RowPtr {
  const uint8_t* w;
  const uint16_t* s;
  const uint16_t* b;
};

template <int FMT>
__device__ __forceinline__ RowPtr row_ptr(const GemmArgs& a, const uint8_t* w, const uint16_t* s, const uint16_t* b,
                                          uint32_t row) {
  RowPtr p;
  const size_t groups = (size_t)row * (a.K / (uint32_t)a.gs);
  p.w = w + (size_t)row * a.K / (FMT == FMT_Q1 ? 8 : 2);
  p.s = s + groups;
  p.b = b ? b + groups : nullptr;
  return p;
}

// Raw weights of K step `step` (the caller clamps it into the matrix).  The
// loads are unconditional: a zero default selected on a predicate would make
// the select wait for the load, i.e. stall the thread for the whole memory
// latency at the prefetch instead of at the (much later) use.
template <int FMT>
__device__ __forceinline__ Raw load_raw(const RowPtr& p, uint32_t gs, uint32_t step) {
  Raw r;
  const uint32_t k0 = step * kBK;
  const uint32_t g = k0 / gs;
  if constexpr (FMT == FMT_Q1) {
    const uint2 v = *reinterpret_cast<const uint2*>(p.w + k0 / 8);
    r.q0 = make_uint4(v.x, v.y, 0u, 0u);
    r.q1 = make_uint4(0u, 0u, 0u, 0u);
    r.b = 0;
  } else {
    const uint4* q = reinterpret_cast<const uint4*>(p.w + k0 / 2);
    r.q0 = q[0]; r.q1 = q[1];
    r.b = p.b[g];
  }
  r.s = p.s[g];
  return r;
}

__device__ __forceinline__ float u16f(uint16_t v, int bf16s) {
  return bf16s ? __uint_as_float((uint32_t)v << 16) : __half2float(__ushort_as_half(v));
}

// One row's 64 weights of a K step as 32 fp16 pairs: word w holds K
// elements 2w (low half) and 2w + 1 (Q1: +-scale, exact in fp16; Q4:
// scale * q + bias rounded to fp16).
template <int FMT>
__device__ __forceinline__ void dequant_words(const Raw& raw, int bf16s, uint32_t (&h)[32]) {
  if constexpr (FMT == FMT_Q1) {
    // bits 2w / 2w + 1 -> halves 0 / 1 of word w: +s for a 1 bit, -s for a 0
    // bit.  The two cleared bits of pair p, (~q) & (3 << 2p), times
    // 2^(15-2p) + 2^(30-2p) land on bits 15/16 and 30/31 without carries;
    // bits 15 and 31 are the two sign flips, applied to s | s << 16 by xor
    // (three integer operations per word; pairs 8-15 of a 32-bit half use
    // the half shifted down by 16 bits).
    const uint32_t s2 = (uint32_t)raw.s | ((uint32_t)raw.s << 16);
#pragma unroll
    for (int hw = 0; hw < 4; ++hw) {
      const uint32_t q = hw < 2 ? raw.q0.x : raw.q0.y;
      const uint32_t t = (hw & 1) ? (q >> 16) : q;
#pragma unroll
      for (int p = 0; p < 8; ++p) {
        const uint32_t m = ~t & (3u << (2 * p));
        const uint32_t f = m * (0x40008000u >> (2 * p));
        h[8 * hw + p] = (f & 0x80008000u) ^ s2;
      }
    }
  } else {
    const float sc = u16f(raw.s, bf16s), bi = u16f(raw.b, bf16s);
#pragma unroll
    for (uint32_t c = 0; c < 8; ++c) {
      const uint32_t word = c < 4 ? (&raw.q0.x)[c] : (&raw.q1.x)[c - 4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float f0 = __fadd_rn(__fmul_rn(sc, (float)((word >> (8 * j)) & 0xFu)), bi);
        const float f1 = __fadd_rn(__fmul_rn(sc, (float)((word >> (8 * j + 4)) & 0xFu)), bi);
        const __half2 v = __floats2half2_rn(f0, f1);
        h[4 * c + j] = *reinterpret_cast<const uint32_t*>(&v);
      }
    }
  }
}

// Dequantize one row's 64 weights into the 128B-swizzled K-major stage
// (.shared addresses).
template <int FMT>
__device__ __forceinline__ void write_row(uint32_t stage, uint32_t r, const Raw& raw, int bf16s) {
  const uint32_t rowp = stage + (r >> 3) * 1024 + (r & 7) * 128;
  uint32_t h[32];
  dequant_words<FMT>(raw, bf16s, h);
#pragma unroll
  for (uint32_t c = 0; c < 8; ++c)
    asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(rowp + ((c ^ (r & 7)) << 4)), "r"(h[4 * c]),
                 "r"(h[4 * c + 1]), "r"(h[4 * c + 2]), "r"(h[4 * c + 3])
                 : "memory");
}

// Warp roles (128 + 128 kGroups threads): warp 0 lane 0 streams the MT
// X tiles of each K step with TMA up to kStages ahead; warp 1 lane 0 issues the MMAs; the warps
// from 4 on dequantize the weights into the B stages in kGroups groups of
// four -- group g takes K steps g, g + kGroups, ..., one weight row per
// thread, raw weights prefetched kPf of the group's steps ahead in
// registers -- so one group's proxy fence and barrier arrival overlap the
// others' dequantization.  Groups 0 and 1 (warps 4-11) run the epilogue
// (TMEM lane quarter = warp % 4, the two groups taking alternate column
// halves).
// warp 1 issues the MT MMA chains of a K step back to back on the one
// dequantized weight tile.
// Split-K over gridDim.z (MT = 1 only) accumulates the residual-add
// epilogue's partial sums with atomicAdd, the others' in the f32 accumulator.
// Development aid: NNZ_GEMM_PROFILE=1 makes CTA (0,0,0) record clock64()
// stamps of its pipeline (read back with nnz_debug_gemm_profile).
__device__ unsigned long long g_gemm_prof[128];
__device__ __forceinline__ void gstamp(const GemmArgs& a, int i) {
  if (a.prof && blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0 && i < 128) g_gemm_prof[i] = clock64();
}

template <int FMT, int MT>
__global__ void __launch_bounds__(kThreads, 1) gemm_kernel(const __grid_constant__ CUtensorMap tmX, GemmArgs a) {
  constexpr int kStages = GemmShape<MT>::kStages;
  constexpr uint32_t kTmemCols = GemmShape<MT>::kTmemCols;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* As = sm;                                     // [stage][MT][16 KB]
  uint8_t* Bs = sm + kStages * MT * kTileBytes;         // [stage][16 KB]
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * (MT + 1) * kTileBytes);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) gstamp(a, 0);
  const uint32_t m0 = blockIdx.y * kBM * MT;
  // M tiles of this CTA inside the matrix (the TMA, MMAs and epilogue skip the rest)
  const uint32_t nv = (a.M - m0 + kBM - 1) / kBM < (uint32_t)MT ? (a.M - m0 + kBM - 1) / kBM : (uint32_t)MT;
  const bool silu = a.epi == GEPI_SILU;
  const uint32_t ncols = silu ? kBN / 2 : kBN;           // output columns per tile
  const uint32_t n0 = blockIdx.x * ncols;
  const uint32_t nk_all = a.K / kBK;
  const uint32_t ks0 = nk_all * blockIdx.z / gridDim.z, ks1 = nk_all * (blockIdx.z + 1) / gridDim.z;
  const uint32_t nk = ks1 - ks0;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], kProducerWarps + 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  // dequantizing warps: weight row of the tile, K-step residue, and the
  // first kPf raw steps, loaded before the grid-dependency wait (the
  // weights are constant, so the HBM latency overlaps the previous kernel)
  const uint32_t r = (tid - 128) & (kBN - 1);
  const uint32_t grp = (tid - 128) / kBN;
  const uint8_t* w = a.w;
  const uint16_t* sc = a.s;
  const uint16_t* bi = a.b;
  uint32_t row = n0 + r;
  if (silu && r >= kBN / 2) { w = a.w2; sc = a.s2; bi = a.b2; row = n0 + r - kBN / 2; }
  const RowPtr rp = row_ptr<FMT>(a, w, sc, bi, row < a.N ? row : a.N - 1);
  const uint32_t klast = nk_all - 1;   // prefetches past the split read its last step (unused)
  const uint32_t gs = (uint32_t)a.gs;
  Raw raw[kPf];
#pragma unroll
  for (int d = 0; d < kPf; ++d)
    raw[d] = load_raw<FMT>(rp, gs, min(ks0 + grp + kGroups * d, klast));
  pdl_wait();
  pdl_launch();
  if (tid == 0) gstamp(a, 1);
  bool failed = false;

  if (warp == 0) {
    if (lane == 0) {
      for (uint32_t i = 0; i < nk; ++i) {
        const uint32_t s = i % kStages;
        if (i >= (uint32_t)kStages && !failed) failed = !mbar_wait(&empty[s], ((i / kStages) - 1) & 1u, a.err);
        mbar_arrive_expect_tx(&full[s], nv * kTileBytes);
        for (uint32_t mt = 0; mt < nv; ++mt)
          tma_load_2d(As + (s * MT + mt) * kTileBytes, &tmX, (int)((ks0 + i) * kBK), (int)(m0 + mt * kBM), &full[s]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, kBN);
      for (uint32_t i = 0; i < nk; ++i) {
        const uint32_t s = i % kStages;
        if (!failed) failed = !mbar_wait(&full[s], (i / kStages) & 1u, a.err);
        if (i < 32) gstamp(a, 66 + (int)i);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t db = smem_desc_sw128(Bs + s * kTileBytes);
        for (uint32_t mt = 0; mt < nv; ++mt) {
          const uint64_t da = smem_desc_sw128(As + (s * MT + mt) * kTileBytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)   // +32 B per 16-element K step inside the swizzle atom
            umma_f16(tmem + mt * kBN, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc, (i | kk) != 0);
        }
        umma_commit(&empty[s]);
      }
      umma_commit(done);
    }
  } else if (warp >= 4) {
    for (uint32_t i0 = grp; i0 < nk; i0 += kGroups * kPf) {
#pragma unroll
      for (int d = 0; d < kPf; ++d) {
        const uint32_t i = i0 + kGroups * d;
        if (i < nk) {
          const uint32_t s = i % kStages;
          if (i >= (uint32_t)kStages && !failed) failed = !mbar_wait(&empty[s], ((i / kStages) - 1) & 1u, a.err);
          if (tid == 128 && i < 32) gstamp(a, 2 + (int)i);
          write_row<FMT>(smem_u32(Bs + s * kTileBytes), r, raw[d], a.bf16s);
          if (tid == 128 && i < 32) gstamp(a, 34 + (int)i);
          asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
          __syncwarp();
          if (tid == 128 && i < 28) gstamp(a, 100 + (int)i);
          if (lane == 0) mbar_arrive(&full[s]);
          raw[d] = load_raw<FMT>(rp, gs, min(ks0 + i + kGroups * kPf, klast));
        }
      }
    }
  }
  // ---- epilogue (warps 4-11), per M tile mt (TMEM columns 128 mt ..):
  // TMEM lanes 32q..32q+31 = rows m0 + 128 mt + 32q + lane; warps 4-7 take
  // column chunks 0-1, warps 8-11 chunks 2-3 ----
  if (warp >= 4 && warp < 12) {
    if (!failed) failed = !mbar_wait(done, 0, a.err);
    if (tid == 128) gstamp(a, 98);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3, part = (warp - 4) >> 2;
    const bool rb = a.bf16r != 0;
    for (uint32_t mt = 0; mt < nv; ++mt) {
      const uint32_t m = m0 + mt * kBM + 32 * q + lane;
      const uint32_t tbase = tmem + mt * kBN + ((uint32_t)(32 * q) << 16);
      if (gridDim.z > 1 && a.epi != GEPI_RESADD) {
        // split K: f32 partials into the accumulator (gate | up halves for SILU)
        for (int cc = 2 * part; cc < 2 * part + 2; ++cc) {
          uint32_t v[32];
          tmem_ld32(tbase + cc * 32, v);
          if (m >= a.M) continue;
          const uint32_t half = silu ? (uint32_t)(cc * 32) / (kBN / 2) : 0;
          const uint32_t nb = n0 + (silu ? (uint32_t)(cc * 32) % (kBN / 2) : (uint32_t)(cc * 32));
          float* o = a.acc + (size_t)m * (silu ? 2 * a.N : a.N) + half * a.N + nb;
          if (nb + 32 <= a.N && (a.N & 3) == 0 && (reinterpret_cast<uintptr_t>(a.acc) & 15) == 0) {
  #pragma unroll
            for (int j = 0; j < 32; j += 4)
              red_add_f32x4(o + j, __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                            __uint_as_float(v[j + 3]));
          } else {
  #pragma unroll
            for (int j = 0; j < 32; ++j)
              if (nb + j < a.N) atomicAdd(&o[j], __uint_as_float(v[j]));
          }
        }
      } else if (silu) {
        for (int cc = part; cc < part + 1; ++cc) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + cc * 32, g);
          tmem_ld32(tbase + 64 + cc * 32, u);
          if (m < a.M) {
            __half* o = static_cast<__half*>(a.out) + (size_t)m * a.ldo + n0 + cc * 32;
  #pragma unroll
            for (int j = 0; j < 32; ++j) {
              const uint32_t n = n0 + cc * 32 + j;
              const float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
              float h = gv / (1.0f + expf(-gv)) * uv;
              if (rb) h = bf16_trunc(h);
              if (n < a.N) o[j] = __float2half_rn(h);
            }
          }
        }
      } else {
        for (int cc = 2 * part; cc < 2 * part + 2; ++cc) {
          uint32_t v[32];
          tmem_ld32(tbase + cc * 32, v);
          if (m >= a.M) continue;
          const uint32_t nb = n0 + cc * 32;
          if (a.epi == GEPI_F16) {
            __half* o = static_cast<__half*>(a.out) + (size_t)m * a.ldo + nb;
            if (nb + 32 <= a.N && (a.ldo & 7) == 0 && (reinterpret_cast<uintptr_t>(a.out) & 15) == 0) {
              // 16-byte stores
  #pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint32_t pk[4];
  #pragma unroll
                for (int e = 0; e < 4; ++e) {
                  float x0 = __uint_as_float(v[j + 2 * e]), x1 = __uint_as_float(v[j + 2 * e + 1]);
                  if (rb) { x0 = bf16_trunc(x0); x1 = bf16_trunc(x1); }
                  const __half2 h2 = __floats2half2_rn(x0, x1);
                  pk[e] = *reinterpret_cast<const uint32_t*>(&h2);
                }
                *reinterpret_cast<uint4*>(o + j) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
              }
            } else {
  #pragma unroll
              for (int j = 0; j < 32; ++j) {
                float x = __uint_as_float(v[j]);
                if (rb) x = bf16_trunc(x);
                if (nb + j < a.N) o[j] = __float2half_rn(x);
              }
            }
          } else {
            float* o = static_cast<float*>(a.out) + (size_t)m * a.ldo + nb;
            if (a.epi == GEPI_RESADD && gridDim.z > 1 && !rb && nb + 32 <= a.N && (a.ldo & 3) == 0 &&
                (reinterpret_cast<uintptr_t>(a.out) & 15) == 0) {
  #pragma unroll
              for (int j = 0; j < 32; j += 4)
                red_add_f32x4(o + j, __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                              __uint_as_float(v[j + 3]));
              continue;
            }
  #pragma unroll
            for (int j = 0; j < 32; ++j) {
              float x = __uint_as_float(v[j]);
              if (rb) x = bf16_trunc(x);
              if (nb + j < a.N) {
                if (a.epi == GEPI_F32) o[j] = x;
                else if (gridDim.z > 1) atomicAdd(&o[j], x);
                else o[j] += x;
              }
            }
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  if (tid == 128) gstamp(a, 99);
  __syncthreads();
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

// ---------------------------------------------------------------------------
// Decode-batch variant (M <= 128 rows): the dequantized weight tile is the A
// operand and lives in TMEM, the activations are the B operand (N = NT
// token columns).  Each dequantizing thread owns one TMEM lane (one weight
// row) and writes its 64 fp16 weights of a K step with one tcgen05.st, so
// the weights never pass through shared memory; per K step shared memory
// only holds the NT x 64 activation tile the TMA brings in (the MMA reads it
// once).  TMEM: the f32 accumulator (128 weight rows x NT tokens) in columns
// [0, NT), then kTsStages A stages of 32 columns (64 fp16 of K per lane).
// SILU tiles interleave the weight rows: lane 2i is gate row n0 + i, lane
// 2i + 1 the matching up row, so the epilogue pairs them with one shuffle.
// ---------------------------------------------------------------------------
template <int NT> struct TsShape {
  static constexpr int kStages = NT <= 64 ? 6 : 4;   // NT = 256: 4 x 32 KB of activations
  // accumulators the MMAs of a K step rotate over (the epilogue adds them);
  // measured: 4 at NT = 64 were no faster than one
  static constexpr int kAcc = 1;
  static constexpr uint32_t kXBytes = NT * kBK * 2;        // activation tile per stage
  static constexpr uint32_t kTmemCols = kAcc * NT + 32 * kStages <= 256 ? 256 : 512;
  static constexpr uint32_t kSmemBytes = kStages * kXBytes + 1024 + 256;
  static_assert(kAcc * NT + 32 * kStages <= (int)kTmemCols, "TMEM budget");
  static_assert(kStages % kGroups == 0, "ring stages must be a multiple of the dequantizing groups");
};
constexpr int kTsThreads = 128 + 128 * kGroups;
constexpr int kTsPf = 4;          // raw-weight prefetch depth (steps of a producer group)

// D(tmem) (+)= A(tmem) * B(smem descriptor)^T, kind::f16.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(tmem_d),
      "r"(tmem_a), "l"(b), "r"(idesc), "r"(acc));
}

template <int FMT, int NT>
__global__ void __launch_bounds__(kTsThreads, 1) gemm_ts_kernel(const __grid_constant__ CUtensorMap tmX, GemmArgs a) {
  using S = TsShape<NT>;
  constexpr int kStages = S::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* Xs = sm;                                             // [stage][NT rows x 128 B]
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + kStages * S::kXBytes);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tslot = reinterpret_cast<uint32_t*>(done + 1);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const bool silu = a.epi == GEPI_SILU;
  const uint32_t ncols = silu ? kBN / 2 : kBN;
  const uint32_t n0 = blockIdx.x * ncols;
  const uint32_t m0 = blockIdx.y * NT;                          // first token row of the tile
  const uint32_t nk_all = a.K / kBK;
  const uint32_t ks0 = nk_all * blockIdx.z / gridDim.z, ks1 = nk_all * (blockIdx.z + 1) / gridDim.z;
  const uint32_t nk = ks1 - ks0;

  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) {
      mbar_init(&full[st], kProducerWarps + 1);
      mbar_init(&empty[st], 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
  }
  if (warp == 2) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(S::kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tslot;
  // dequantizing warps: TMEM lane r = weight row of the tile
  const uint32_t r = (tid - 128) & (kBN - 1);
  const uint32_t grp = (tid - 128) / kBN;
  const uint8_t* w = a.w;
  const uint16_t* sc = a.s;
  const uint16_t* bi = a.b;
  uint32_t row = n0 + r;
  if (silu) {
    row = n0 + (r >> 1);
    if (r & 1) { w = a.w2; sc = a.s2; bi = a.b2; }
  }
  const RowPtr rp = row_ptr<FMT>(a, w, sc, bi, row < a.N ? row : a.N - 1);
  const uint32_t klast = nk_all - 1;   // prefetches past the split read its last step (unused)
  const uint32_t gs = (uint32_t)a.gs;
  Raw raw[kTsPf];
#pragma unroll
  for (int d = 0; d < kTsPf; ++d)
    raw[d] = load_raw<FMT>(rp, gs, min(ks0 + grp + kGroups * d, klast));
  pdl_wait();
  pdl_launch();
  bool failed = false;
  const uint32_t tA = tmem + S::kAcc * NT;                      // A stages: 32 columns each

  if (warp == 0) {
    if (lane == 0) {
      for (uint32_t i = 0; i < nk; ++i) {
        const uint32_t st = i % kStages;
        if (i >= (uint32_t)kStages && !failed) failed = !mbar_wait(&empty[st], ((i / kStages) - 1) & 1u, a.err);
        mbar_arrive_expect_tx(&full[st], S::kXBytes);
        tma_load_2d(Xs + st * S::kXBytes, &tmX, (int)((ks0 + i) * kBK), (int)m0, &full[st]);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(kBM, NT);
      for (uint32_t i = 0; i < nk; ++i) {
        const uint32_t st = i % kStages;
        if (!failed) failed = !mbar_wait(&full[st], (i / kStages) & 1u, a.err);
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint64_t db = smem_desc_sw128(Xs + st * S::kXBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)   // 8 TMEM columns / +32 B per 16-element K step
          umma_f16_ts(tmem + (kk % S::kAcc) * NT, tA + st * 32 + kk * 8, db + (uint64_t)(kk * 2), idesc,
                      (i | (uint32_t)(kk / S::kAcc)) != 0);
        umma_commit(&empty[st]);
      }
      umma_commit(done);
    }
  } else if (warp >= 4) {
    const uint32_t lane_base = (uint32_t)(32 * (warp & 3)) << 16;
    // one rolled step (a short loop body stays in the instruction cache);
    // the kTsPf prefetched steps rotate through registers
#pragma unroll 1
    for (uint32_t i = grp; i < nk; i += kGroups) {
      const uint32_t st = i % kStages;
      if (i >= (uint32_t)kStages && !failed) failed = !mbar_wait(&empty[st], ((i / kStages) - 1) & 1u, a.err);
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      uint32_t h[32];
      dequant_words<FMT>(raw[0], a.bf16s, h);
      tmem_st32(tA + lane_base + st * 32, h);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&full[st]);
#pragma unroll
      for (int d = 0; d + 1 < kTsPf; ++d) raw[d] = raw[d + 1];
      raw[kTsPf - 1] = load_raw<FMT>(rp, gs, min(ks0 + i + kGroups * kTsPf, klast));
    }
  }
  // ---- epilogue: warps 4-11; TMEM lane quarter q = warp % 4 (weight rows
  // 32q + lane), part p = (warp - 4) / 4 takes token columns [p NT/2, (p+1) NT/2) ----
  if (warp >= 4 && warp < 12) {
    if (!failed) failed = !mbar_wait(done, 0, a.err);
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    const int q = warp & 3, part = (warp - 4) >> 2;
    const bool rb = a.bf16r != 0;
    const uint32_t rr = 32 * q + lane;                            // weight row of the tile
    const bool split = gridDim.z > 1;
#pragma unroll
    for (int cc = 0; cc < NT / 64; ++cc) {
      const uint32_t tc = (uint32_t)part * (NT / 2) + cc * 32;   // first TMEM column
      const uint32_t c0 = m0 + tc;                               // its token row
      uint32_t v[32];
      tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + tc, v);
#pragma unroll
      for (int ac = 1; ac < S::kAcc; ++ac) {
        uint32_t u[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q) << 16) + ac * NT + tc, u);
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = __float_as_uint(__uint_as_float(v[j]) + __uint_as_float(u[j]));
      }
      if (c0 >= a.M) continue;
      if (silu) {
        const uint32_t n = n0 + (rr >> 1);
        if (split) {
          // f32 partials: gate | up halves of acc [M][2][N]
          if (n < a.N) {
            float* o = a.acc + (size_t)(rr & 1) * a.N + n;
#pragma unroll
            for (int j = 0; j < 32; ++j)
              if (c0 + j < a.M) atomicAdd(o + (size_t)(c0 + j) * 2 * a.N, __uint_as_float(v[j]));
          }
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float mine = __uint_as_float(v[j]);
            const float other = __shfl_xor_sync(0xffffffffu, mine, 1);
            if ((lane & 1) == 0 && n < a.N && c0 + j < a.M) {
              float hv = mine / (1.0f + expf(-mine)) * other;
              if (rb) hv = bf16_trunc(hv);
              static_cast<__half*>(a.out)[(size_t)(c0 + j) * a.ldo + n] = __float2half_rn(hv);
            }
          }
        }
        continue;
      }
      const uint32_t n = n0 + rr;
      if (n >= a.N) {
      } else if (split) {
        float* o = (a.epi == GEPI_RESADD ? static_cast<float*>(a.out) : a.acc) + n;
        const size_t ld = a.epi == GEPI_RESADD ? a.ldo : a.N;
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (c0 + j < a.M) atomicAdd(o + (size_t)(c0 + j) * ld, __uint_as_float(v[j]));
      } else if (a.epi == GEPI_F16) {
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float x = __uint_as_float(v[j]);
          if (rb) x = bf16_trunc(x);
          if (c0 + j < a.M) static_cast<__half*>(a.out)[(size_t)(c0 + j) * a.ldo + n] = __float2half_rn(x);
        }
      } else {
        float* o = static_cast<float*>(a.out) + n;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          float x = __uint_as_float(v[j]);
          if (rb) x = bf16_trunc(x);
          if (c0 + j < a.M) {
            if (a.epi == GEPI_F32) o[(size_t)(c0 + j) * a.ldo] = x;
            else o[(size_t)(c0 + j) * a.ldo] += x;
          }
        }
      }
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 2)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(S::kTmemCols) : "memory");
}

// One CTA per row; K % 4 == 0.  Every thread's float4 loads of a pass are
// issued before any is used (one round trip per 4 * 1024 columns).
__global__ void __launch_bounds__(256) rmsnorm_f16_kernel(const float* res, const float* w, float eps, uint32_t K,
                                                          int bf16r, __half* out) {
  constexpr int kU = 4;
  __shared__ float red[32];
  const uint32_t row = blockIdx.x, K4 = K / 4;
  pdl_wait();
  pdl_launch();
  const float4* x = reinterpret_cast<const float4*>(res + (size_t)row * K);
  float ss = 0.f;
  for (uint32_t k0 = threadIdx.x; k0 < K4; k0 += kU * blockDim.x) {
    float4 v[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t k = k0 + u * blockDim.x;
      v[u] = k < K4 ? x[k] : make_float4(0.f, 0.f, 0.f, 0.f);
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
  }
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < blockDim.x / 32 ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) red[0] = rsqrtf(t / (float)K + eps);
  }
  __syncthreads();
  const float r = red[0];
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (uint32_t k0 = threadIdx.x; k0 < K4; k0 += kU * blockDim.x) {
    float4 v[kU], g[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t k = k0 + u * blockDim.x;
      if (k < K4) { v[u] = x[k]; g[u] = w4[k]; }
    }
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const uint32_t k = k0 + u * blockDim.x;
      if (k >= K4) continue;
      float o[4] = {v[u].x * r * g[u].x, v[u].y * r * g[u].y, v[u].z * r * g[u].z, v[u].w * r * g[u].w};
      if (bf16r)
        for (int i = 0; i < 4; ++i) o[i] = bf16_trunc(o[i]);
      __half2* dst = reinterpret_cast<__half2*>(out + (size_t)row * K + 4 * k);
      dst[0] = __floats2half2_rn(o[0], o[1]);
      dst[1] = __floats2half2_rn(o[2], o[3]);
    }
  }
}

// Split-K finalize: the accumulated f32 tile -> the epilogue's output, and
// the accumulator back to zero for its next use.
__global__ void __launch_bounds__(256) gemm_finalize_kernel(GemmArgs a) {
  pdl_wait();
  pdl_launch();
  // row m = blockIdx.y; four consecutive columns per thread (N % 4 == 0)
  const uint32_t m = blockIdx.y, n = (blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (n >= a.N) return;
  const bool rb = a.bf16r != 0;
  float o[4];
  if (a.epi == GEPI_SILU) {
    float4* g = reinterpret_cast<float4*>(a.acc + (size_t)m * 2 * a.N + n);
    float4* u = reinterpret_cast<float4*>(a.acc + (size_t)m * 2 * a.N + a.N + n);
    const float4 gv = *g, uv = *u;
    *g = make_float4(0.f, 0.f, 0.f, 0.f);
    *u = make_float4(0.f, 0.f, 0.f, 0.f);
    const float gs[4] = {gv.x, gv.y, gv.z, gv.w}, us[4] = {uv.x, uv.y, uv.z, uv.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = gs[e] / (1.0f + expf(-gs[e])) * us[e];
  } else {
    float4* p = reinterpret_cast<float4*>(a.acc + (size_t)m * a.N + n);
    const float4 v = *p;
    *p = make_float4(0.f, 0.f, 0.f, 0.f);
    o[0] = v.x; o[1] = v.y; o[2] = v.z; o[3] = v.w;
  }
  if (rb)
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = bf16_trunc(o[e]);
  if (a.epi == GEPI_F32) {
    float* d = static_cast<float*>(a.out) + (size_t)m * a.ldo + n;
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] = o[e];
  } else {
    __half* d = static_cast<__half*>(a.out) + (size_t)m * a.ldo + n;
#pragma unroll
    for (int e = 0; e < 4; ++e) d[e] = __float2half_rn(o[e]);
  }
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeFn get_encode() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}


}  // namespace

bool tensor_map_f16_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                       uint32_t box_inner, uint32_t box_outer) {
  EncodeFn enc = get_encode();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, outer};
  const cuuint64_t strides[1] = {row_bytes};
  const cuuint32_t box[2] = {box_inner, box_outer};
  const cuuint32_t estr[2] = {1, 1};
  return enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

cudaError_t gemm_debug_profile(unsigned long long* out) {
  return cudaMemcpyFromSymbol(out, g_gemm_prof, sizeof(g_gemm_prof));
}

cudaError_t gemm_launch(const GemmArgs& a_in, const __half* x, cudaStream_t st) {
  GemmArgs a = a_in;
  static const int prof = [] {
    const char* e = getenv("NNZ_GEMM_PROFILE");
    return (e && e[0] == '1') ? 1 : 0;
  }();
  a.prof = prof;
  if (a.K % kBK || a.gs < 64 || a.K % a.gs || a.M == 0 || a.N == 0 ||
      (a.fmt != FMT_Q1 && a.fmt != FMT_Q4) || (reinterpret_cast<uintptr_t>(x) & 15))
    return cudaErrorInvalidValue;
  EncodeFn enc = get_encode();
  if (!enc) return cudaErrorNotSupported;
  CUtensorMap tm;
  const cuuint64_t dims[2] = {a.K, a.M};
  const cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
  const cuuint32_t box[2] = {kBK, kBM};
  const cuuint32_t estr[2] = {1, 1};
  if (enc(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), dims, strides, box, estr,
          CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
          CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  const uint32_t ncols = a.epi == GEPI_SILU ? kBN / 2 : kBN;
  int sms = 148, dev = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  // M tiles per CTA: the most that still gives at least 60 % of the SMs a
  // CTA (each weight tile is dequantized once per CTA and its MMAs run back
  // to back, so MT = 4 does a quarter of the dequantization of MT = 1 on a
  // 512-row chunk; fewer CTAs than that lose more to idle SMs)
  const uint32_t ntn = (a.N + ncols - 1) / ncols, ntm = (a.M + kBM - 1) / kBM;
  static const int mt_max = [] {   // NNZ_GEMM_MT caps it (1, 2 or 4; for measurements)
    const char* e = getenv("NNZ_GEMM_MT");
    return e ? atoi(e) : 4;
  }();
  int mt = 1;
  if (mt_max >= 4 && ntm >= 3 && ntn * ((ntm + 3) / 4) * 5 >= (uint32_t)sms * 3) mt = 4;
  else if (mt_max >= 2 && ntm >= 2 && ntn * ((ntm + 1) / 2) * 5 >= (uint32_t)sms * 3) mt = 2;
  dim3 grid(ntn, (ntm + mt - 1) / mt);
  // GEMMs with fewer tiles than SMs split K: residual adds accumulate their
  // partials atomically in place, the other epilogues in the f32
  // accumulator (when given one that fits), finished by gemm_finalize_kernel
  const size_t acc_need = (size_t)a.M * a.N * (a.epi == GEPI_SILU ? 2 : 1);
  // (the finalize kernel takes four columns per thread: N % 4 == 0)
  const bool can_split = a.epi == GEPI_RESADD ? a.bf16r == 0
                                              : (a.acc && acc_need <= a.acc_floats && a.N % 4 == 0 &&
                                                 (reinterpret_cast<uintptr_t>(a.acc) & 15) == 0);
  if (can_split && mt == 1) {
    uint32_t ks = (uint32_t)sms / (grid.x * grid.y);
    const uint32_t nk = a.K / kBK;
    if (ks > nk / 4) ks = nk / 4;            // >= 4 K steps per CTA
    grid.z = ks < 1 ? 1 : ks;
  }
  cudaLaunchAttribute la[1];
  la[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  la[0].val.programmaticStreamSerializationAllowed = a.pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kThreads);
  cfg.stream = st;
  cfg.attrs = la;
  cfg.numAttrs = 1;
  cudaError_t e = cudaSuccess;
  // up to 128 rows: the weights-in-TMEM variant (NNZ_GEMM_TS=0 turns it off, for measurements)
  static const bool ts_on = [] {
    const char* v = getenv("NNZ_GEMM_TS");
    return !(v && v[0] == '0');
  }();
  if (ts_on) {
    // token tiles of NT rows: 64 / 128 for decode batches, 256 for prompts
    // (tensor-bound: 64 KB of shared-memory traffic per 4.2 MFLOP K step,
    // against 208 KB per 8.4 MFLOP for four 128-row tiles sharing a
    // shared-memory weight tile)
    uint32_t nt = a.M <= 64 ? 64 : (a.M <= 128 ? 128 : 256);
    // whole-K launches whose 128-row tiles still fit in one wave take them
    // (more CTAs, shorter MMAs; measured: 512 x 2048 x 4096 22.9 -> 20.5 us;
    // with more than one wave of 128-row tiles the 256-row tiles are faster)
    if (nt == 256 && !can_split && ntn * ((a.M + 127) / 128) <= (uint32_t)sms) nt = 128;
    grid = dim3(ntn, (a.M + nt - 1) / nt, 1);
    if (can_split) {
      uint32_t ks = (uint32_t)sms / (grid.x * grid.y);
      const uint32_t nk = a.K / kBK;
      if (ks > nk / 4) ks = nk / 4;
      grid.z = ks < 1 ? 1 : ks;
    }
    cfg.gridDim = grid;
    CUtensorMap tx;
    const cuuint32_t boxt[2] = {kBK, nt};
    if (enc(&tx, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x), dims, strides, boxt, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaErrorInvalidValue;
    cfg.blockDim = dim3(kTsThreads);
    static bool ats[2][3] = {};
    auto gots = [&](auto kern, uint32_t smem, bool& attr) {
      if (!attr) {
        e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return;
        attr = true;
      }
      cfg.dynamicSmemBytes = smem;
      e = cudaLaunchKernelEx(&cfg, kern, tx, a);
    };
    const int fi = a.fmt == FMT_Q1 ? 0 : 1, ni = nt == 64 ? 0 : (nt == 128 ? 1 : 2);
    if (a.fmt == FMT_Q1) {
      if (nt == 64) gots(&gemm_ts_kernel<FMT_Q1, 64>, TsShape<64>::kSmemBytes, ats[fi][ni]);
      else if (nt == 128) gots(&gemm_ts_kernel<FMT_Q1, 128>, TsShape<128>::kSmemBytes, ats[fi][ni]);
      else gots(&gemm_ts_kernel<FMT_Q1, 256>, TsShape<256>::kSmemBytes, ats[fi][ni]);
    } else {
      if (nt == 64) gots(&gemm_ts_kernel<FMT_Q4, 64>, TsShape<64>::kSmemBytes, ats[fi][ni]);
      else if (nt == 128) gots(&gemm_ts_kernel<FMT_Q4, 128>, TsShape<128>::kSmemBytes, ats[fi][ni]);
      else gots(&gemm_ts_kernel<FMT_Q4, 256>, TsShape<256>::kSmemBytes, ats[fi][ni]);
    }
  } else {
  auto go = [&](auto kern, uint32_t smem, bool& attr) {
    if (!attr) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return;
      attr = true;
    }
    cfg.dynamicSmemBytes = smem;
    e = cudaLaunchKernelEx(&cfg, kern, tm, a);
  };
  static bool at[2][3] = {};
  const int fi = a.fmt == FMT_Q1 ? 0 : 1, mi = mt == 4 ? 2 : mt - 1;
  if (a.fmt == FMT_Q1) {
    if (mt == 4) go(&gemm_kernel<FMT_Q1, 4>, GemmShape<4>::kSmemBytes, at[fi][mi]);
    else if (mt == 2) go(&gemm_kernel<FMT_Q1, 2>, GemmShape<2>::kSmemBytes, at[fi][mi]);
    else go(&gemm_kernel<FMT_Q1, 1>, GemmShape<1>::kSmemBytes, at[fi][mi]);
  } else {
    if (mt == 4) go(&gemm_kernel<FMT_Q4, 4>, GemmShape<4>::kSmemBytes, at[fi][mi]);
    else if (mt == 2) go(&gemm_kernel<FMT_Q4, 2>, GemmShape<2>::kSmemBytes, at[fi][mi]);
    else go(&gemm_kernel<FMT_Q4, 1>, GemmShape<1>::kSmemBytes, at[fi][mi]);
  }
  }
  if (e != cudaSuccess || grid.z == 1 || a.epi == GEPI_RESADD) return e;
  cudaLaunchConfig_t fc = {};
  fc.gridDim = dim3((a.N / 4 + 255) / 256, a.M);
  fc.blockDim = dim3(256);
  fc.stream = st;
  fc.attrs = la;
  fc.numAttrs = 1;
  return cudaLaunchKernelEx(&fc, &gemm_finalize_kernel, a);
}

cudaError_t rmsnorm_f16_launch(const float* res, const float* w, float eps, uint32_t rows, uint32_t K, int bf16r,
                               __half* out, cudaStream_t st, int pdl) {
  if (K % 4) return cudaErrorInvalidValue;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(rows);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, &rmsnorm_f16_kernel, res, w, eps, K, bf16r, out);
}

}  // namespace nnz
