// Decode attention kernels (see attn.cuh).
#include <cuda_runtime.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>

#include "attn.cuh"
#include "rope_dev.cuh"

namespace nnz {

namespace {

struct AttnSmem {
  uint32_t bars, kring, vring, q, knew, vnew, s, stat, flag, total;
};

template <int HD>
__host__ __device__ inline AttnSmem attn_layout() {
  AttnSmem L;
  uint32_t o = 0;
  L.bars = o; o += kAttnStages * 8;
  o = (o + 127) & ~127u;
  L.kring = o; o += kAttnStages * kAttnBlk * HD * 2;
  L.vring = o; o += kAttnStages * kAttnBlk * HD * 2;
  L.q = o; o += kAttnMaxG * HD * 4;
  L.knew = o; o += HD * 4;
  L.vnew = o; o += HD * 4;
  L.s = o; o += kAttnMaxG * kAttnBlk * 4;
  L.stat = o; o += 3 * kAttnMaxG * 4;  // m, l, alpha
  L.flag = o; o += 16;
  L.total = o;
  return L;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(AttnArgs a) {
  constexpr int EPL = HD / 32;
  extern __shared__ __align__(128) uint8_t sm[];
  const AttnSmem L = attn_layout<HD>();
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L.bars);
  __half* kring = reinterpret_cast<__half*>(sm + L.kring);
  __half* vring = reinterpret_cast<__half*>(sm + L.vring);
  float* qs = reinterpret_cast<float*>(sm + L.q);
  float* knew = reinterpret_cast<float*>(sm + L.knew);
  float* vnew = reinterpret_cast<float*>(sm + L.vnew);
  float* ss = reinterpret_cast<float*>(sm + L.s);
  float* mst = reinterpret_cast<float*>(sm + L.stat);
  float* lst = mst + kAttnMaxG;
  float* alp = lst + kAttnMaxG;
  int* flag = reinterpret_cast<int*>(sm + L.flag);

  const int kvh = blockIdx.x, row = blockIdx.y, split = blockIdx.z;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int G = (int)(a.n_q / a.n_kv);
  // Positions and past K/V were written >= 2 launches earlier: safe pre-wait.
  int p = a.pos[row];
  if (p < 0 || p >= (int)a.max_ctx) {
    if (threadIdx.x == 0) atomicOr(a.err, ERR_BAD_POS);
    p = p < 0 ? 0 : (int)a.max_ctx - 1;
  }
  const int slot = a.slot ? a.slot[row] : row;
  const int seq = p + 1;
  const int per = (seq + (int)a.splits - 1) / (int)a.splits;
  const int t0 = split * per;
  const int t1 = min(seq, t0 + per);
  const bool own_new = a.write_kv && t0 <= p && p < t1;
  const int cend = a.write_kv ? min(t1, p) : t1;
  const int ncache = cend > t0 ? cend - t0 : 0;
  const int nblk = (ncache + kAttnBlk - 1) / kAttnBlk;
  const size_t head_off = ((size_t)slot * a.n_kv + kvh) * a.max_ctx * HD;
  const __half* kb = a.kc + head_off;
  const __half* vb = a.vc + head_off;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kAttnStages; ++s) mbar_init(&bars[s], 1);
    fence_barrier_init();
    for (int b = 0; b < nblk && b < kAttnStages; ++b) {
      const int n = min(kAttnBlk, ncache - b * kAttnBlk);
      const uint32_t bytes = (uint32_t)n * HD * 2;
      mbar_arrive_expect_tx(&bars[b], 2 * bytes);
      bulk_g2s(kring + (size_t)b * kAttnBlk * HD, kb + (size_t)(t0 + b * kAttnBlk) * HD, bytes, &bars[b]);
      bulk_g2s(vring + (size_t)b * kAttnBlk * HD, vb + (size_t)(t0 + b * kAttnBlk) * HD, bytes, &bars[b]);
    }
  }
  __syncthreads();
  pdl_wait();
  pdl_launch();

  // q heads (and the new k/v) -----------------------------------------
  const __half* qrow = a.qkv + (size_t)row * a.qkv_stride;
  for (int h = warp; h < G; h += kAttnThreads / 32) {
    float v[EPL];
    norm_rope_head<HD>(qrow + (size_t)(kvh * G + h) * HD, a.q_norm, a.eps, a.theta, a.rope_style,
                       p, lane, v);
#pragma unroll
    for (int e = 0; e < EPL; ++e) qs[h * HD + lane * EPL + e] = v[e];
  }
  if (own_new && warp == (kAttnThreads / 32) - 1) {
    float v[EPL];
    norm_rope_head<HD>(qrow + (size_t)a.n_q * HD + (size_t)kvh * HD, a.k_norm, a.eps, a.theta,
                       a.rope_style, p, lane, v);
    const __half* vsrc = qrow + (size_t)(a.n_q + a.n_kv) * HD + (size_t)kvh * HD;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane * EPL + e;
      const __half kh = __float2half_rn(v[e]);
      a.kc[head_off + (size_t)p * HD + d] = kh;
      a.vc[head_off + (size_t)p * HD + d] = vsrc[d];
      knew[d] = __half2float(kh);
      vnew[d] = __half2float(vsrc[d]);
    }
  }
  if (threadIdx.x < kAttnMaxG) {
    mst[threadIdx.x] = -INFINITY;
    lst[threadIdx.x] = 0.f;
  }
  __syncthreads();

  constexpr int NHS = kAttnThreads / HD;   // thread groups over heads in PV
  const int d = threadIdx.x % HD, hs = threadIdx.x / HD;
  float acc[kAttnMaxG];
#pragma unroll
  for (int h = 0; h < kAttnMaxG; ++h) acc[h] = 0.f;
  const float inv = rsqrtf((float)HD);
  bool failed = false;

  const int total_blocks = nblk + (own_new ? 1 : 0);
  for (int b = 0; b < total_blocks; ++b) {
    const bool is_new = b == nblk;
    const int n = is_new ? 1 : min(kAttnBlk, ncache - b * kAttnBlk);
    const int stg = b % kAttnStages;
    const __half* kr = kring + (size_t)stg * kAttnBlk * HD;
    const __half* vr = vring + (size_t)stg * kAttnBlk * HD;
    if (!is_new && !failed) failed = !mbar_wait(&bars[stg], (b / kAttnStages) & 1, a.err);
    // scores
    for (int t = warp; t < n; t += kAttnThreads / 32) {
      float kv[EPL];
      if (is_new) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) kv[e] = knew[lane * EPL + e];
      } else {
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
          const __half2 k2 = *reinterpret_cast<const __half2*>(kr + (size_t)t * HD + lane * EPL + e);
          const float2 f = __half22float2(k2);
          kv[e] = f.x; kv[e + 1] = f.y;
        }
      }
      for (int h = 0; h < G; ++h) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dot = fmaf(qs[h * HD + lane * EPL + e], kv[e], dot);
        dot = warp_sum(dot);
        if (lane == 0) ss[h * kAttnBlk + t] = dot * inv;
      }
    }
    __syncthreads();
    // online softmax statistics, one warp per head
    for (int h = warp; h < G; h += kAttnThreads / 32) {
      const float sv = lane < n ? ss[h * kAttnBlk + lane] : -INFINITY;
      const float mx = warp_max(sv);
      const float mo = mst[h];
      const float mn = fmaxf(mo, mx);
      const float pe = lane < n ? expf(sv - mn) : 0.f;
      if (lane < n) ss[h * kAttnBlk + lane] = pe;
      const float ls = warp_sum(pe);
      if (lane == 0) {
        const float al = (mo == -INFINITY) ? 0.f : expf(mo - mn);
        alp[h] = al;
        lst[h] = lst[h] * al + ls;
        mst[h] = mn;
      }
    }
    __syncthreads();
    // P.V
    for (int h = hs; h < G; h += NHS) {
      float o = acc[h] * alp[h];
      if (is_new) {
        o = fmaf(ss[h * kAttnBlk], vnew[d], o);
      } else {
        for (int t = 0; t < n; ++t) o = fmaf(ss[h * kAttnBlk + t], __half2float(vr[(size_t)t * HD + d]), o);
      }
      acc[h] = o;
    }
    __syncthreads();
    if (!is_new && threadIdx.x == 0 && b + kAttnStages < nblk) {
      const int nb = b + kAttnStages;
      const int nn = min(kAttnBlk, ncache - nb * kAttnBlk);
      const uint32_t bytes = (uint32_t)nn * HD * 2;
      mbar_arrive_expect_tx(&bars[stg], 2 * bytes);
      bulk_g2s(kring + (size_t)stg * kAttnBlk * HD, kb + (size_t)(t0 + nb * kAttnBlk) * HD, bytes, &bars[stg]);
      bulk_g2s(vring + (size_t)stg * kAttnBlk * HD, vb + (size_t)(t0 + nb * kAttnBlk) * HD, bytes, &bars[stg]);
    }
  }

  __half* orow = a.out + (size_t)row * a.out_stride + (size_t)kvh * G * HD;
  if (a.splits == 1) {
    for (int h = hs; h < G; h += NHS) orow[h * HD + d] = __float2half_rn(acc[h] / lst[h]);
    return;
  }
  const uint32_t rec = HD + 2;
  float* wsp = a.ws + ((size_t)(row * a.n_kv + kvh) * a.splits) * G * rec;
  for (int h = hs; h < G; h += NHS) wsp[((size_t)split * G + h) * rec + 2 + d] = acc[h];
  if (threadIdx.x < (unsigned)G) {
    wsp[((size_t)split * G + threadIdx.x) * rec + 0] = mst[threadIdx.x];
    wsp[((size_t)split * G + threadIdx.x) * rec + 1] = lst[threadIdx.x];
  }
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t prev = atomicAdd(&a.counters[row * a.n_kv + kvh], 1u);
    flag[0] = prev == a.splits - 1;
  }
  __syncthreads();
  if (!flag[0]) return;
  __threadfence();
  // merge the splits' (m, l, o) with an online rescale; 8 splits' loads
  // are issued before any is used
  for (int h = hs; h < G; h += NHS) {
    float M = -INFINITY, Lsum = 0.f, o = 0.f;
    for (uint32_t s0 = 0; s0 < a.splits; s0 += 8) {
      float mv[8], lv[8], ov[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const bool ok = s0 + j < a.splits;
        const float* r = wsp + ((size_t)(s0 + j) * G + h) * rec;
        mv[j] = ok ? __ldcg(r) : -INFINITY;
        lv[j] = ok ? __ldcg(r + 1) : 0.f;
        ov[j] = ok ? __ldcg(r + 2 + d) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        if (mv[j] == -INFINITY) continue;
        const float nm = fmaxf(M, mv[j]);
        const float a0 = (M == -INFINITY) ? 0.f : expf(M - nm), a1 = expf(mv[j] - nm);
        Lsum = Lsum * a0 + lv[j] * a1;
        o = o * a0 + ov[j] * a1;
        M = nm;
      }
    }
    orow[h * HD + d] = __float2half_rn(o / Lsum);
  }
  if (threadIdx.x == 0) a.counters[row * a.n_kv + kvh] = 0;
}

template <int HD>
__global__ void __launch_bounds__(64) rope_kv_write_kernel(AttnArgs a) {
  constexpr int EPL = HD / 32;
  pdl_wait();
  pdl_launch();
  const int kvh = blockIdx.x, row = blockIdx.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int p = a.pos[row];
  if (p < 0 || p >= (int)a.max_ctx) {
    if (threadIdx.x == 0) atomicOr(a.err, ERR_BAD_POS);
    return;
  }
  const int slot = a.slot ? a.slot[row] : row;
  const size_t off = (((size_t)slot * a.n_kv + kvh) * a.max_ctx + p) * HD;
  const __half* qrow = a.qkv + (size_t)row * a.qkv_stride;
  if (warp == 0) {
    float v[EPL];
    norm_rope_head<HD>(qrow + (size_t)a.n_q * HD + (size_t)kvh * HD, a.k_norm, a.eps, a.theta,
                       a.rope_style, p, lane, v);
#pragma unroll
    for (int e = 0; e < EPL; ++e) a.kc[off + lane * EPL + e] = __float2half_rn(v[e]);
  } else {
    const __half* vsrc = qrow + (size_t)(a.n_q + a.n_kv) * HD + (size_t)kvh * HD;
#pragma unroll
    for (int e = 0; e < EPL; ++e) a.vc[off + lane * EPL + e] = vsrc[lane * EPL + e];
  }
}

cudaLaunchConfig_t make_cfg(dim3 grid, dim3 block, uint32_t smem, int pdl, cudaStream_t st,
                            cudaLaunchAttribute* at) {
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

template <int HD>
cudaError_t attn_launch_t(const AttnArgs& a, int pdl, cudaStream_t st) {
  const AttnSmem L = attn_layout<HD>();
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(a.n_kv, a.rows, a.splits), dim3(kAttnThreads), L.total, pdl, st, at);
  return cudaLaunchKernelEx(&cfg, &attn_decode_kernel<HD>, a);
}

}  // namespace

cudaError_t attn_prepare() {
  cudaError_t e = attn_tc_prepare();
  if (e != cudaSuccess) return e;
  e = cudaFuncSetAttribute(&attn_decode_kernel<128>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       attn_layout<128>().total);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(&attn_decode_kernel<64>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              attn_layout<64>().total);
}

size_t attn_ws_floats(uint32_t rows, uint32_t n_q, uint32_t n_kv, uint32_t splits, int head_dim,
                      uint32_t max_ctx) {
  const size_t legacy = splits <= 1 ? 0 : (size_t)rows * n_kv * splits * (n_q / n_kv) * (head_dim + 2);
  const size_t tc = attn_tc_applies(n_q, n_kv, head_dim) ? attn_tc_ws_floats(rows, n_q, n_kv, max_ctx) : 0;
  return legacy > tc ? legacy : tc;
}

namespace {
bool use_legacy_attn() {
  static const int v = [] {
    const char* e = getenv("NNZ_ATTN");
    return (e && strcmp(e, "legacy") == 0) ? 1 : 0;
  }();
  return v != 0;
}
}  // namespace

cudaError_t attn_decode_launch(const AttnArgs& a, int head_dim, int pdl, cudaStream_t st) {
  if (a.n_kv == 0 || a.n_q % a.n_kv || a.n_q / a.n_kv > (uint32_t)kAttnMaxG || a.splits == 0 ||
      a.rows == 0)
    return cudaErrorInvalidValue;
  if (attn_tc_applies(a.n_q, a.n_kv, head_dim) && a.ws && !use_legacy_attn()) return attn_tc_launch(a, pdl, st);
  if (head_dim == 128) return attn_launch_t<128>(a, pdl, st);
  if (head_dim == 64) return attn_launch_t<64>(a, pdl, st);
  return cudaErrorInvalidValue;
}

cudaError_t rope_kv_write_launch(const AttnArgs& a, int head_dim, int pdl, cudaStream_t st) {
  if (a.rows == 0 || a.n_kv == 0) return cudaErrorInvalidValue;
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(a.n_kv, a.rows), dim3(64), 0, pdl, st, at);
  if (head_dim == 128) return cudaLaunchKernelEx(&cfg, &rope_kv_write_kernel<128>, a);
  if (head_dim == 64) return cudaLaunchKernelEx(&cfg, &rope_kv_write_kernel<64>, a);
  return cudaErrorInvalidValue;
}

}  // namespace nnz

// ===========================================================================
// Causal prefill attention.  One CTA per (kv head, block of query rows);
// threads own (row, query head of the group, quarter of head_dim), so a
// score needs two shuffles and the online softmax stays per thread.  K/V
// tiles of 64 positions are staged in shared memory and shared by all rows
// of the block.  Same f32 math as the decode kernel: q = RoPE(RMSNorm(q))
// kept f32, scores q.k / sqrt(hd), online softmax, fp16 output.  The chunk's
// own K/V must already be in the cache (rope_kv_write_launch).
// ===========================================================================
namespace nnz {
namespace {

constexpr int kPfThreads = 256;
constexpr int kPfKeys = 64;

template <int HD>
__global__ void __launch_bounds__(kPfThreads) attn_prefill_kernel(AttnArgs a) {
  constexpr int Q4 = HD / 4;            // dims per thread
  __shared__ __align__(16) __half ks[kPfKeys][HD];
  __shared__ __align__(16) __half vs[kPfKeys][HD];
  pdl_wait();
  pdl_launch();
  const int G = (int)(a.n_q / a.n_kv);
  const int rows_per_cta = kPfThreads / (4 * G);
  const int tid = threadIdx.x, c = tid & 3, g = (tid >> 2) % G, rl = tid / (4 * G);
  const int kvh = blockIdx.x;
  const uint32_t r = blockIdx.y * rows_per_cta + rl;
  const bool live = r < a.rows;
  const int pos = live ? a.pos[r] : -1;
  const int slot = (live && a.slot) ? a.slot[r] : 0;
  // keys to visit: up to the largest position of the block's rows
  int maxpos = pos;
  for (int o = 16; o > 0; o >>= 1) maxpos = max(maxpos, __shfl_xor_sync(0xffffffffu, maxpos, o));
  __shared__ int s_max[kPfThreads / 32];
  __shared__ int s_slot;
  if ((tid & 31) == 0) s_max[tid >> 5] = maxpos;
  if (tid == 0) s_slot = slot;
  __syncthreads();
  int kmax = -1;
  for (int w = 0; w < kPfThreads / 32; ++w) kmax = max(kmax, s_max[w]);
  const size_t head_off = ((size_t)s_slot * a.n_kv + kvh) * a.max_ctx * HD;

  // q: RMSNorm over the head (4 threads) + RoPE, f32
  float q[Q4], o[Q4];
  const int h = kvh * G + g;
  {
    const __half* src = a.qkv + (size_t)(live ? r : 0) * a.qkv_stride + (size_t)h * HD + c * Q4;
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < Q4; ++i) { q[i] = __half2float(src[i]); ss = fmaf(q[i], q[i], ss); }
    ss += __shfl_xor_sync(0xffffffffu, ss, 1);
    ss += __shfl_xor_sync(0xffffffffu, ss, 2);
    const float rr = rsqrtf(ss / (float)HD + a.eps);
#pragma unroll
    for (int i = 0; i < Q4; ++i) q[i] = q[i] * rr * a.q_norm[c * Q4 + i];
    const double l2t = log2((double)a.theta);
    if (a.rope_style == ROPE_PAIRWISE) {
#pragma unroll
      for (int i = 0; i < Q4; i += 2) {
        const int p = (c * Q4 + i) >> 1;
        double sd, cd;
        sincos((double)max(pos, 0) * exp2(-(2.0 * p / HD) * l2t), &sd, &cd);
        const float cs = (float)cd, sn = (float)sd, x0 = q[i], x1 = q[i + 1];
        q[i] = x0 * cs - x1 * sn;
        q[i + 1] = x0 * sn + x1 * cs;
      }
    } else {
#pragma unroll
      for (int i = 0; i < Q4; ++i) {
        const float partner = __shfl_xor_sync(0xffffffffu, q[i], 2);   // quarter c <-> c^2
        const int p = (c & 1) * Q4 + i;
        double sd, cd;
        sincos((double)max(pos, 0) * exp2(-(2.0 * p / HD) * l2t), &sd, &cd);
        const float cs = (float)cd, sn = (float)sd;
        q[i] = (c < 2) ? q[i] * cs - partner * sn : partner * sn + q[i] * cs;
      }
    }
#pragma unroll
    for (int i = 0; i < Q4; ++i) o[i] = 0.f;
  }
  const float inv = rsqrtf((float)HD);
  float m = -INFINITY, l = 0.f;
  for (int t0 = 0; t0 <= kmax; t0 += kPfKeys) {
    const int n = min(kPfKeys, kmax + 1 - t0);
    __syncthreads();
    for (int i = tid; i < n * HD / 8; i += kPfThreads) {
      const int t = i / (HD / 8), d8 = i % (HD / 8);
      reinterpret_cast<uint4*>(&ks[t][0])[d8] =
          *reinterpret_cast<const uint4*>(a.kc + head_off + (size_t)(t0 + t) * HD + 8 * d8);
      reinterpret_cast<uint4*>(&vs[t][0])[d8] =
          *reinterpret_cast<const uint4*>(a.vc + head_off + (size_t)(t0 + t) * HD + 8 * d8);
    }
    __syncthreads();
    for (int t = 0; t < n; t += 4) {
      float s4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tt = min(t + u, n - 1);
        float a0 = 0.f, a1 = 0.f;
#pragma unroll
        for (int i = 0; i < Q4; i += 4) {
          const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&ks[tt][c * Q4 + i]));
          const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&ks[tt][c * Q4 + i + 2]));
          a0 = fmaf(q[i], k0.x, a0); a1 = fmaf(q[i + 1], k0.y, a1);
          a0 = fmaf(q[i + 2], k1.x, a0); a1 = fmaf(q[i + 3], k1.y, a1);
        }
        s4[u] = a0 + a1;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        s4[u] += __shfl_xor_sync(0xffffffffu, s4[u], 1);
        s4[u] += __shfl_xor_sync(0xffffffffu, s4[u], 2);
      }
      float p4[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const bool ok = (t + u < n) && (t0 + t + u <= pos);
        const float sc = ok ? s4[u] * inv : -INFINITY;
        if (sc > m) {
          const float al = (m == -INFINITY) ? 0.f : expf(m - sc);
          l *= al;
#pragma unroll
          for (int i = 0; i < Q4; ++i) o[i] *= al;
#pragma unroll
          for (int v = 0; v < u; ++v) p4[v] *= al;
          m = sc;
        }
        p4[u] = ok ? expf(sc - m) : 0.f;
        l += p4[u];
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int tt = min(t + u, n - 1);
#pragma unroll
        for (int i = 0; i < Q4; i += 2) {
          const float2 v2 = __half22float2(*reinterpret_cast<const __half2*>(&vs[tt][c * Q4 + i]));
          o[i] = fmaf(p4[u], v2.x, o[i]);
          o[i + 1] = fmaf(p4[u], v2.y, o[i + 1]);
        }
      }
    }
  }
  if (live) {
    __half* dst = a.out + (size_t)r * a.out_stride + (size_t)h * HD + c * Q4;
    const float il = 1.f / l;
#pragma unroll
    for (int i = 0; i < Q4; i += 2) *reinterpret_cast<__half2*>(&dst[i]) = __floats2half2_rn(o[i] * il, o[i + 1] * il);
  }
}

}  // namespace

cudaError_t attn_prefill_launch(const AttnArgs& a, int head_dim, int pdl, cudaStream_t st) {
  if (attn_tc_applies(a.n_q, a.n_kv, head_dim) && !use_legacy_attn()) {
    static const bool mma = [] {
      const char* e = getenv("NNZ_PREFILL_ATTN");
      return e && strcmp(e, "mma") == 0;
    }();
    if (!mma && attn_pf_umma_applies(a.n_q, a.n_kv)) return attn_pf_umma_launch(a, pdl, st);
    if (a.ws) return attn_prefill_tc_launch(a, pdl, st);
  }
  const uint32_t G = a.n_q / a.n_kv;
  if (a.rows == 0 || a.n_kv == 0 || a.n_q % a.n_kv || 4 * G > (uint32_t)kPfThreads) return cudaErrorInvalidValue;
  const uint32_t rpc = kPfThreads / (4 * G);
  cudaLaunchAttribute at[1];
  cudaLaunchConfig_t cfg = make_cfg(dim3(a.n_kv, (a.rows + rpc - 1) / rpc), dim3(kPfThreads), 0, pdl, st, at);
  if (head_dim == 128) return cudaLaunchKernelEx(&cfg, &attn_prefill_kernel<128>, a);
  if (head_dim == 64) return cudaLaunchKernelEx(&cfg, &attn_prefill_kernel<64>, a);
  return cudaErrorInvalidValue;
}

}  // namespace nnz
