// Causal prefill attention on tcgen05 (head_dim 128, G = n_q / n_kv in
// {1, 2, 4}): the tensor-core replacement of the reference's per-token
// decode attention when a prompt is processed in chunks
// (nnmetal/src/shaders/transformer.metal:1467-1695 gqa_attention_fused_f16io_tg,
// dispatched once per prompt token by transformer.zig:4032-4068 chunkedPrefill).
//
// One CTA of 512 threads per (kv head, block of 128 / G query positions).
// Its 128 TMEM lanes / MMA rows are (position, query head) pairs, row
// r = G * p + h, so the G heads sharing the kv head share every K/V tile.
// Four threads own row r, one 32-column slice each (the slice of TMEM its
// warp reads): they normalise and rotate the row's query (f32 RMSNorm over
// the head with q_norm, RoPE; partial sums and the half-split RoPE partner
// meet in shared memory), write it as fp16 hi + lo into shared memory, run
// the row's online softmax straight out of TMEM (one shared-memory max
// exchange per tile) and write the output row.
// Per 128-key tile j:
//   S(j) = Q_hi K^T + Q_lo K^T (16 MMAs 128x128x16, f32 in one of two TMEM
//   buffers, columns 0-127 / 128-255) -- issued together with the previous
//   tile's P V, so it is ready when the softmax comes round;
//   P = exp(S / sqrt(128) - m) per row (computed as exp2 of log2(e)-scaled
//   scores), fp16 hi + lo into shared memory; the O accumulator (TMEM
//   columns 256-383) rescaled by exp(m_old - m_new);
//   O += P_hi V + P_lo V (16 MMAs; V as stored, [key][d], an MN-major B).
// K and V tiles arrive by TMA one tile ahead (K as soon as the S that read
// the buffer has completed, V as soon as the P V has).
// q and the probabilities keep ~22 significant bits through the hi/lo
// split, products are exact and accumulate in f32: the f32 semantics of the
// reference's scores and softmax, with the fp16 K/V cache it stores.
// Keys past the block's last position are zero in shared memory and masked
// to probability 0.  Every wait is bounded; a timeout records
// ERR_MBAR_TIMEOUT and the kernel still frees its TMEM and returns.
#include <cuda_runtime.h>

#include "attn.cuh"
#include "gemm.cuh"
#include "rope_dev.cuh"
#include "umma.cuh"

namespace nnz {

namespace {

constexpr int kHd = 128;
constexpr int kKeys = 128;                     // keys per tile
constexpr uint32_t kBlk = 128 * 64 * 2;        // one 128-row x 64-column fp16 swizzled block (16 KB)
// shared memory: Q hi, Q lo, K, V^T, P hi, P lo -- two K-blocks each
constexpr uint32_t OFF_QH = 0, OFF_QL = 2 * kBlk, OFF_K = 4 * kBlk, OFF_VT = 6 * kBlk, OFF_PH = 8 * kBlk,
                   OFF_PL = 10 * kBlk, OFF_MISC = 12 * kBlk;
constexpr uint32_t OFF_RED = OFF_MISC + 64;            // [4 chunks][128 rows] f32 partial reductions
constexpr uint32_t kPfSmem = OFF_RED + 4 * 128 * 4 + 1024;   // + alignment slack
constexpr uint32_t kTmemCols = 512;                  // S: two buffers 0-127 / 128-255, O: 256-383

// 16-byte chunk c (8 fp16 along K) of row r in a two-block K-major tile.
__device__ __forceinline__ uint32_t tile_off(uint32_t r, uint32_t c) {
  return (c >> 3) * kBlk + sw128_off(r, c & 7);
}

__device__ __forceinline__ void st_smem16(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

__device__ __forceinline__ uint32_t pack_h2(float x, float y) {
  const __half2 h = __floats2half2_rn(x, y);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// hi = fp16(x), lo = fp16(x - hi) for 8 consecutive values, into two rows.
__device__ __forceinline__ void store_hilo8(uint32_t hi_addr, uint32_t lo_addr, const float* x) {
  uint32_t h[4], l[4];
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const __half a = __float2half_rn(x[2 * e]), b = __float2half_rn(x[2 * e + 1]);
    const __half2 hh = __halves2half2(a, b);
    h[e] = *reinterpret_cast<const uint32_t*>(&hh);
    l[e] = pack_h2(x[2 * e] - __half2float(a), x[2 * e + 1] - __half2float(b));
  }
  st_smem16(hi_addr, h[0], h[1], h[2], h[3]);
  st_smem16(lo_addr, l[0], l[1], l[2], l[3]);
}

// Bounded wait on a commit barrier; on timeout records the error once.
__device__ __forceinline__ bool pf_wait(uint64_t* bar, uint32_t parity, int* err, bool& failed) {
  if (failed) return false;
  if (!mbar_wait(bar, parity, err)) failed = true;
  return !failed;
}

struct PfArgs {
  AttnArgs a;
  CUtensorMap tmK, tmV;   // the layer's K / V cache as [slots * n_kv * max_ctx][128] fp16, box {64, 128}
};

#ifdef NNZ_PF_PROFILE
__device__ unsigned long long g_pf_prof[64];
#define PF_STAMP(i) do { if (threadIdx.x == 0 && blockIdx.x == 0 && blockIdx.y == gridDim.y - 1 && (i) < 64) g_pf_prof[i] = clock64(); } while (0)
#else
#define PF_STAMP(i) do { } while (0)
#endif

template <int G>
__global__ void __launch_bounds__(512, 1) attn_pf_umma_kernel(const __grid_constant__ PfArgs pa) {
  const AttnArgs& a = pa.a;
  PF_STAMP(0);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* mb = reinterpret_cast<uint64_t*>(sm + OFF_MISC);         // MMA commits
  uint64_t* mbk = mb + 1;                                             // K tile landed
  uint64_t* mbv = mb + 2;                                             // V tile landed
  uint32_t* tslot = reinterpret_cast<uint32_t*>(sm + OFF_MISC + 24);
  int* s_kmax = reinterpret_cast<int*>(sm + OFF_MISC + 28);
  float* red = reinterpret_cast<float*>(sm + OFF_RED);     // [4][128]
  constexpr uint32_t PB = 128 / G;                 // query positions per CTA
  const uint32_t tid = threadIdx.x, warp = tid >> 5;
  const uint32_t r = 32 * (warp & 3) + (tid & 31), c = warp >> 2;   // row, 32-column chunk
  const uint32_t kvh = blockIdx.x, p0 = blockIdx.y * PB;
  const uint32_t hl = r % G, qi = p0 + r / G, h = kvh * G + hl;
  const bool valid = qi < a.rows;
  if (tid == 0) {
    mbar_init(mb, 1);
    mbar_init(mbk, 1);
    mbar_init(mbv, 1);
    fence_barrier_init();
    *s_kmax = 0;
  }
  if (warp == 0) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tslot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tslot;
  pdl_wait();
  pdl_launch();
  const int pos = valid ? min(max(a.pos[qi], 0), (int)a.max_ctx - 1) : -1;
  if (c == 0) atomicMax(s_kmax, pos);
  const int slot = a.slot ? a.slot[p0] : (int)p0;
  const int yb = (slot * (int)a.n_kv + (int)kvh) * (int)a.max_ctx;   // tensor-map row of key 0
  auto issue_k = [&](int j) {
    mbar_arrive_expect_tx(mbk, 2 * kBlk);
    tma_load_2d(sm + OFF_K, &pa.tmK, 0, yb + j * kKeys, mbk);
    tma_load_2d(sm + OFF_K + kBlk, &pa.tmK, 64, yb + j * kKeys, mbk);
  };
  auto issue_v = [&](int j) {
    mbar_arrive_expect_tx(mbv, 2 * kBlk);
    tma_load_2d(sm + OFF_VT, &pa.tmV, 0, yb + j * kKeys, mbv);
    tma_load_2d(sm + OFF_VT + kBlk, &pa.tmV, 64, yb + j * kKeys, mbv);
  };
  if (tid == 0) {   // tile 0 lands while the query is prepared
    issue_k(0);
    issue_v(0);
  }

  // ---- query row r, elements [32c, 32c + 32): RMSNorm (q_norm), RoPE, fp16 hi/lo ----
  float v[32];
  {
    const uint4* src =
        reinterpret_cast<const uint4*>(a.qkv + (size_t)(valid ? qi : 0) * a.qkv_stride + (size_t)h * kHd) + 4 * c;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 u = valid ? src[i] : make_uint4(0u, 0u, 0u, 0u);
      const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[e]));
        v[8 * i + 2 * e] = f.x;
        v[8 * i + 2 * e + 1] = f.y;
        ss = fmaf(f.x, f.x, ss);
        ss = fmaf(f.y, f.y, ss);
      }
    }
    red[c * 128 + r] = ss;
  }
  __syncthreads();
  const int kmax = *s_kmax;
  {
    const float tot = (red[r] + red[128 + r]) + (red[256 + r] + red[384 + r]);
    const float rr = rsqrtf(tot / (float)kHd + a.eps);
    const float4* qn4 = reinterpret_cast<const float4*>(a.q_norm + 32 * c);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 w = __ldg(qn4 + i);
      v[4 * i] = v[4 * i] * rr * w.x;
      v[4 * i + 1] = v[4 * i + 1] * rr * w.y;
      v[4 * i + 2] = v[4 * i + 2] * rr * w.z;
      v[4 * i + 3] = v[4 * i + 3] * rr * w.w;
    }
  }
  const int pp = pos < 0 ? 0 : pos;
  const float2* tab = a.rope_tab ? a.rope_tab + (size_t)pp * (kHd / 2) : nullptr;
  const double l2t = a.rope_tab ? 0.0 : log2((double)a.theta);
  if (a.rope_style == ROPE_PAIRWISE) {
#pragma unroll
    for (int e = 0; e < 32; e += 2) {
      const float2 cs = rope_cs<kHd>(tab, l2t, pp, (32 * c + e) >> 1);
      const float x0 = v[e], x1 = v[e + 1];
      v[e] = x0 * cs.x - x1 * cs.y;
      v[e + 1] = x0 * cs.y + x1 * cs.x;
    }
  } else {
    // element d pairs with d +- 64, held by chunk c ^ 2: exchange through
    // the (still unused) P area as f32 [128 rows][128]
    float* xq = reinterpret_cast<float*>(sm + OFF_PH);
#pragma unroll
    for (int e = 0; e < 32; ++e) xq[r * 128 + ((32 * c + e + r) & 127)] = v[e];
    __syncthreads();
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const int d = 32 * c + e, i = d & 63;
      const float2 cs = rope_cs<kHd>(tab, l2t, pp, i);
      const float partner = xq[r * 128 + ((d ^ 64) + r & 127)];
      v[e] = d < 64 ? v[e] * cs.x - partner * cs.y : partner * cs.y + v[e] * cs.x;
    }
    __syncthreads();   // the P area is rewritten below
  }
  {
    const uint32_t qh = smem_u32(sm + OFF_QH), ql = smem_u32(sm + OFF_QL);
#pragma unroll
    for (int i = 0; i < 4; ++i) store_hilo8(qh + tile_off(r, 4 * c + i), ql + tile_off(r, 4 * c + i), v + 8 * i);
  }
  PF_STAMP(1);

  const uint32_t idesc = idesc_f16(128, 128);
  const uint32_t idesc_pv = idesc_f16(128, 128) | (1u << 16);  // B MN-major
  // scores scaled by 1 / sqrt(128) and log2(e): the softmax runs on exp2
  const float sl2 = rsqrtf((float)kHd) * 1.4426950408889634f;
  const uint32_t tq = tmem + ((32 * (warp & 3)) << 16);   // this warp's TMEM lane quarter
  float m = -INFINITY, l = 0.f;                             // l: this thread's 32 columns only
  bool failed = false;
  uint32_t ph = 0;   // commit phases consumed
  const int ntile = kmax / kKeys + 1;
  const uint32_t pbh = smem_u32(sm + OFF_PH), pbl = smem_u32(sm + OFF_PL);
  // S of tile j into TMEM columns 128 (j % 2) (thread 0)
  auto issue_s = [&](int j) {
    pf_wait(mbk, (uint32_t)j & 1u, a.err, failed);
    tc_fence_after();
#pragma unroll
    for (int part = 0; part < 2; ++part)            // S = Q_hi K^T + Q_lo K^T
#pragma unroll
      for (int kb = 0; kb < 2; ++kb) {
        const uint64_t da = smem_desc_sw128(sm + (part ? OFF_QL : OFF_QH) + kb * kBlk);
        const uint64_t db = smem_desc_sw128(sm + OFF_K + kb * kBlk);
#pragma unroll
        for (int kk = 0; kk < 4; ++kk)
          umma_f16(tmem + (uint32_t)(j & 1) * 128, da + (uint64_t)(kk * 2), db + (uint64_t)(kk * 2), idesc,
                   (part | kb | kk) != 0);
      }
  };
  // the query tiles were written by every thread
  fence_async_smem();
  tc_fence_before();
  __syncthreads();
  if (tid == 0) {
    issue_s(0);
    umma_commit(mb);
  }
  pf_wait(mb, ph & 1u, a.err, failed);
  ++ph;
  tc_fence_after();
  if (tid == 0 && ntile > 1) issue_k(1);
  // Per tile: softmax of S(j) -> P; then one commit covers S(j + 1) (the
  // other TMEM buffer, its K tile loaded meanwhile) and O += P V(j), so the
  // next tile's scores are ready when the softmax loop comes round.
  for (int j = 0; j < ntile; ++j) {
    PF_STAMP(2 + 6 * j);
    // online softmax: this thread's 32 scores of row r
    float sv[32];
    {
      uint32_t u[32];
      tmem_ld32(tq + (uint32_t)(j & 1) * 128 + 32 * c, u);
      float mx = -INFINITY;
#pragma unroll
      for (int e = 0; e < 32; ++e) {
        const int t = j * kKeys + 32 * (int)c + e;
        sv[e] = t <= pos ? __uint_as_float(u[e]) * sl2 : -INFINITY;   // log2 domain
        mx = fmaxf(mx, sv[e]);
      }
      red[c * 128 + r] = mx;
    }
    tc_fence_before();
    __syncthreads();
    const float mt = fmaxf(fmaxf(red[r], red[128 + r]), fmaxf(red[256 + r], red[384 + r]));
    const float mn = fmaxf(m, mt);
    const float alpha = mn == -INFINITY ? 1.f : (m == -INFINITY ? 0.f : exp2f(m - mn));
    float sum = 0.f;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      sv[e] = sv[e] == -INFINITY ? 0.f : exp2f(sv[e] - mn);
      sum += sv[e];
    }
#pragma unroll
    for (int g = 0; g < 4; ++g) store_hilo8(pbh + tile_off(r, 4 * c + g), pbl + tile_off(r, 4 * c + g), sv + 8 * g);
    l = l * alpha + sum;
    m = mn;
    PF_STAMP(5 + 6 * j);
    if (j > 0) {   // O *= alpha (the previous tile's P V has completed)
      uint32_t u[32];
      tc_fence_after();
      tmem_ld32(tq + 256 + 32 * c, u);
#pragma unroll
      for (int e = 0; e < 32; ++e) u[e] = __float_as_uint(__uint_as_float(u[e]) * alpha);
      tmem_st32(tq + 256 + 32 * c, u);
    }
    PF_STAMP(6 + 6 * j);
    if (j == ntile - 1) {
      // keys past the block's last position: rows of other positions, other
      // heads or never written; their probabilities are 0, and zero V rows
      // keep 0 * V finite
      pf_wait(mbv, (uint32_t)j & 1u, a.err, failed);
      const int first = kmax - j * kKeys + 1;   // first stale key row of the tile
      for (int k = first + (int)(tid >> 3); k < kKeys; k += 64)
#pragma unroll
        for (int hb = 0; hb < 2; ++hb)
          st_smem16(smem_u32(sm + OFF_VT + hb * kBlk) + k * 128 + (tid & 7) * 16, 0u, 0u, 0u, 0u);
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();   // also: every thread has read red[] and S(j) before they are rewritten
    if (tid == 0) {
      if (j + 1 < ntile) issue_s(j + 1);
      pf_wait(mbv, (uint32_t)j & 1u, a.err, failed);
      tc_fence_after();
      // O += P_hi V + P_lo V: V as loaded ([key][d], MN-major B: the two
      // 64-wide d halves are the two TMA boxes, 16 KB apart); K steps of 16
      // keys = 2048 bytes of V rows
#pragma unroll
      for (int part = 0; part < 2; ++part)
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {
          const uint64_t da = smem_desc_sw128(sm + (part ? OFF_PL : OFF_PH) + kb * kBlk);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            const uint64_t db = smem_desc_sw128_mn(sm + OFF_VT + (kb * 64 + kk * 16) * 128);
            umma_f16(tmem + 256, da + (uint64_t)(kk * 2), db, idesc_pv, (j | part | kb | kk) != 0);
          }
        }
      umma_commit(mb);
    }
    pf_wait(mb, ph & 1u, a.err, failed);
    ++ph;
    tc_fence_after();
    if (tid == 0) {   // K and V tiles are free again
      if (j + 2 < ntile) issue_k(j + 2);
      if (j + 1 < ntile) issue_v(j + 1);
    }
  }
  PF_STAMP(60);
  // ---- output row r, columns [32c, 32c + 32): O / l, fp16 ----
  red[c * 128 + r] = l;
  __syncthreads();
  {
    const float il = 1.0f / ((red[r] + red[128 + r]) + (red[256 + r] + red[384 + r]));
    uint32_t u[32];
    tmem_ld32(tq + 256 + 32 * c, u);
    if (valid) {
      __half* dst = a.out + (size_t)qi * a.out_stride + (size_t)h * kHd + 32 * c;
#pragma unroll
      for (int g = 0; g < 4; ++g) {
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e)
          w[e] = pack_h2(__uint_as_float(u[8 * g + 2 * e]) * il, __uint_as_float(u[8 * g + 2 * e + 1]) * il);
        *reinterpret_cast<uint4*>(dst + g * 8) = make_uint4(w[0], w[1], w[2], w[3]);
      }
    }
  }
  PF_STAMP(61);
  tc_fence_before();
  __syncthreads();
  if (warp == 0)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
}

}  // namespace

bool attn_pf_umma_applies(uint32_t n_q, uint32_t n_kv) {
  if (n_kv == 0 || n_q % n_kv) return false;
  const uint32_t G = n_q / n_kv;
  return G == 1 || G == 2 || G == 4;
}

cudaError_t attn_pf_umma_launch(const AttnArgs& a, int pdl, cudaStream_t st) {
  if (!attn_pf_umma_applies(a.n_q, a.n_kv) || a.rows == 0) return cudaErrorInvalidValue;
  PfArgs pa;
  pa.a = a;
  {
    // the map covers exactly the cache allocation (slots x heads x positions):
    // a tile that runs past it reads zeros, never memory outside it
    const uint64_t rows = (uint64_t)(a.slots ? a.slots : 1) * a.n_kv * a.max_ctx;
    if (!tensor_map_f16_2d(&pa.tmK, a.kc, kHd, rows, kHd * 2, 64, kKeys) ||
        !tensor_map_f16_2d(&pa.tmV, a.vc, kHd, rows, kHd * 2, 64, kKeys))
      return cudaErrorInvalidValue;
  }
  const uint32_t G = a.n_q / a.n_kv, pb = 128 / G;
  static bool attr[3] = {false, false, false};
  const int gi = G == 1 ? 0 : G == 2 ? 1 : 2;
  const void* fn = G == 1 ? (const void*)&attn_pf_umma_kernel<1>
                 : G == 2 ? (const void*)&attn_pf_umma_kernel<2> : (const void*)&attn_pf_umma_kernel<4>;
  if (!attr[gi]) {
    const cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPfSmem);
    if (e != cudaSuccess) return e;
    attr[gi] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_kv, (a.rows + pb - 1) / pb);
  cfg.blockDim = dim3(512);
  cfg.dynamicSmemBytes = kPfSmem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (G == 1) return cudaLaunchKernelEx(&cfg, &attn_pf_umma_kernel<1>, pa);
  if (G == 2) return cudaLaunchKernelEx(&cfg, &attn_pf_umma_kernel<2>, pa);
  return cudaLaunchKernelEx(&cfg, &attn_pf_umma_kernel<4>, pa);
}

}  // namespace nnz
