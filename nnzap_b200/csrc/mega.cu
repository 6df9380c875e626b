// Persistent cooperative decode kernel (see mega.cuh).
//
// Phases (grid barriers between them, except QKV -> ATT, ATT -> O and
// GU -> DN, which are per-unit dataflow counters):
//   EMBED   CTA 0 advances the device decode state (token <- previous
//           argmax, position += 1) and writes residual version 0; the other
//           CTAs clear the accumulators;
//   per layer l:
//   QKV     fused-norm QKV matvec, split-K partials -> qkv_acc (red.add);
//   ATT     flash-decoding over the fp16 KV cache per (kv head, row, split)
//           with QK-norm + RoPE + KV write, partial (m, l, o) -> att_ws;
//   O       merges the splits into the fp16 attention output, o-proj,
//           partials -> next residual version (red.add), plus the previous
//           residual added once by the split-0 units;
//   GU      fused-norm gate/up matvec, partials -> gu_acc (red.add);
//   DN      fp16(SiLU(g) * u) from gu_acc, down-proj -> next residual;
//   LM      fused final-norm LM head, f32 logits (optional) and argmax.
// The residual rotates over three buffers: the phase producing version v+1
// accumulates into a buffer cleared during the phase that produced v, and
// no phase reads the buffer it writes.  Every read of data produced in this
// launch bypasses L1 (__ldcg).
//
// Weight streaming: each warp owns a ring of `nslot` segment buffers fed by
// 1-D bulk copies.  Its lane 0 walks the warp's static sequence of weight
// segments across ALL phases, keeping nslot copies in flight, so while a CTA
// waits at a grid barrier the next phases' weights are already landing in
// shared memory.  Every wait (mbarrier, grid barrier) is bounded.
#include <cuda_runtime.h>

#include "mega.cuh"

#include <stdlib.h>
#include "rope_dev.cuh"

namespace nnz {

namespace {

enum PhaseType : int { PH_EMBED = 0, PH_QKV, PH_ATT, PH_O, PH_GU, PH_DN, PH_LM, PH_END };

constexpr int kMaxSlots = 4;
constexpr int kAttBlk = 32;
constexpr int kAttStages = 2;
constexpr int kAttMaxG = 8;
constexpr int kMaxAttSplits = 32;
constexpr int kMaxHeadsPerUnit = 32;

struct PhaseInfo {
  int type;
  uint32_t layer, M, K, tiles, ks, groups, sub, units;
  const uint8_t* w;
};

template <typename T>
__host__ __device__ __forceinline__ const T* lptr(const MegaArgs& a, const T* p0, uint32_t l) {
  return reinterpret_cast<const T*>(reinterpret_cast<const uint8_t*>(p0) + (size_t)l * a.lstride);
}

__host__ __device__ inline PhaseInfo phase_info(const MegaArgs& a, const MegaLayer* layers,
                                                uint32_t ph) {
  PhaseInfo p{};
  const uint32_t last = 1 + 5 * a.L;
  if (ph == 0) { p.type = PH_EMBED; return p; }
  if (ph > last) { p.type = PH_END; return p; }
  p.sub = 1;
  if (ph == last) {
    p.type = PH_LM; p.w = a.lm; p.M = a.vocab; p.K = a.H; p.ks = 1;
  } else {
    const uint32_t l = (ph - 1) / 5, r = (ph - 1) % 5;
    p.layer = l;
    const uint32_t qd = a.n_q * a.hd, kvd = a.n_kv * a.hd;
    switch (r) {
      case 0: p.type = PH_QKV; p.w = lptr(a, a.l0.qkv, l); p.M = qd + 2 * kvd; p.K = a.H; p.ks = a.ks_qkv; break;
      case 1: p.type = PH_ATT; p.units = a.n_kv * a.batch * a.att_splits; return p;
      case 2: p.type = PH_O; p.w = lptr(a, a.l0.o, l); p.M = a.H; p.K = qd; p.ks = a.ks_o; break;
      case 3: p.type = PH_GU; p.w = lptr(a, a.l0.gu, l); p.M = a.I; p.K = a.H; p.ks = a.ks_gu; p.sub = 2; break;
      default: p.type = PH_DN; p.w = lptr(a, a.l0.down, l); p.M = a.H; p.K = a.I; p.ks = a.ks_dn; break;
    }
  }
  p.tiles = num_tiles(p.M);
  p.groups = p.K / a.gs;
  p.units = p.tiles * p.ks;
  return p;
}

__host__ __device__ inline void unit_range(const PhaseInfo& p, uint32_t u, uint32_t* tile, uint32_t* split,
                                           uint32_t* G0, uint32_t* ng) {
  *tile = u / p.ks;
  *split = u % p.ks;
  const uint32_t g0 = p.groups * (*split) / p.ks;     // groups * ks < 2^32
  const uint32_t g1 = p.groups * (*split + 1) / p.ks;
  *G0 = g0;
  *ng = g1 - g0;
}

// Scale groups per weight-ring item.  A ring slot holds a gate/up pair's two
// segments; the LM head (a single matrix with many groups per unit) fills it
// with two adjacent groups of its tile, contiguous in the tile-packed layout.
__host__ __device__ inline uint32_t groups_per_item(int type, uint32_t ng) {
  return type == PH_LM && ng % 2 == 0 ? 2u : 1u;
}

struct MegaSmem {
  uint32_t tmpl, bars, abars, ring, slot_bytes, u, xs, xf, gsx, gsum, gsq, red, rms, flag,
      kring, vring, qs, knew, vnew, ss, stat, tok, total, kr_max, ng_max, bcm, nt;
};

__host__ __device__ inline MegaSmem mega_layout(const MegaArgs& a, int fmt) {
  MegaSmem s{};
  s.bcm = a.batch < (uint32_t)kBatchChunk ? a.batch : kBatchChunk;
  s.nt = s.bcm > 4 ? 2 : 1;
  // widest K range any CTA quantizes
  uint32_t krm = a.H;  // LM head runs unsplit
  const uint32_t gs = a.gs;
  const uint32_t ks[4] = {a.ks_qkv, a.ks_o, a.ks_gu, a.ks_dn};
  const uint32_t Ks[4] = {a.H, a.n_q * a.hd, a.H, a.I};
  for (int i = 0; i < 4; ++i) {
    const uint32_t g = Ks[i] / gs, r = ((g + ks[i] - 1) / ks[i]) * gs;
    krm = r > krm ? r : krm;
  }
  s.kr_max = krm;
  s.ng_max = krm / gs;
  s.slot_bytes = 2 * seg_bytes(fmt, gs);
  uint32_t o = 0;
  s.tmpl = o; o += 6 * sizeof(PhaseInfo);
  o = (o + 15) & ~15u;
  s.bars = o; o += kQmvWarps * kMaxSlots * 8;
  s.abars = o; o += kAttStages * 8;
  o = (o + 127) & ~127u;
  s.ring = o; o += kQmvWarps * a.nslot * s.slot_bytes;
  o = (o + 127) & ~127u;
  // quantized-x fragments persist across phases (zeroed once per launch)
  s.xf = o; o += (krm / kChunk) * s.nt * 256;
  s.gsx = o; o += s.ng_max * kBatchChunk * 4;
  s.gsum = o; o += s.ng_max * kBatchChunk * 4;
  s.gsq = o; o += s.ng_max * kBatchChunk * 4;
  o = (o + 127) & ~127u;
  s.u = o;
  // matvec view of the union
  uint32_t q = o;
  s.xs = q; q += ((krm * s.bcm * 2) + 15) & ~15u;
  s.red = q; q += kQmvWarps * 2 * kTileRows * s.bcm * 4;
  s.rms = q; q += kBatchChunk * 4;
  s.flag = q; q += 16;
  s.tok = q; q += kBatchChunk * 4;
  // full residual rows for the one-round-trip RMSNorm (small batches only)
  // attention view of the union
  uint32_t t = o;
  s.kring = t; t += kAttStages * kAttBlk * a.hd * 2;
  s.vring = t; t += kAttStages * kAttBlk * a.hd * 2;
  s.qs = t; t += kAttMaxG * a.hd * 4;
  s.knew = t; t += a.hd * 4;
  s.vnew = t; t += a.hd * 4;
  s.ss = t; t += kAttMaxG * kAttBlk * 4;
  s.stat = t; t += 3 * kAttMaxG * 4;
  s.total = q > t ? q : t;
  return s;
}

// Grid barrier over all CTAs (co-resident by cooperative launch).  Bounded:
// after kSpinLimit polls it records ERR_SPIN_TIMEOUT and lets the CTA run
// on (results are then garbage, but every CTA terminates).
constexpr uint32_t kGridSpinLimit = 1u << 20;

__device__ __forceinline__ unsigned int ld_relaxed(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ unsigned long long ld_acquire64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

// bar[2] is the sticky abort flag (once any wait of the launch times out,
// every other wait gives up immediately); bar[4..5] a 64-bit arrival counter
// that only grows: barrier i of a launch completes when it reaches
// bar_base + (i + 1) * nblocks.  One release-add per CTA and acquire polls,
// so the barrier costs a single one-way trip after the last arrival.
__device__ __forceinline__ void grid_sync(unsigned int* bar, unsigned int nblocks, unsigned long long& target,
                                          int* err) {
  __syncthreads();
  if (threadIdx.x == 0) {
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(bar + 4);
    target += nblocks;
    // release: this CTA's writes (ordered before by bar.sync) become visible
    // to every CTA that acquires a count including this arrival
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(cnt) : "memory");
    uint32_t i = 0;
    while (ld_acquire64(cnt) < target) {
      if ((++i & 63u) == 0) {
        if (ld_relaxed(&bar[2])) break;
        if (i > kGridSpinLimit) {
          atomicOr(err, ERR_SPIN_TIMEOUT);
          atomicExch(&bar[2], 1u);
          break;
        }
      }
    }
  }
  __syncthreads();
}

// Dataflow edges (QKV -> attention, attention -> O): the producer unit adds
// one to its counter after its results are written (release: the CTA's
// writes, ordered by bar.sync, become visible to whoever acquires the
// count); the consumer waits, bounded, until every counter it reads has
// reached its target.
__device__ __forceinline__ void dep_signal(unsigned int* ctr) {
  __syncthreads();
  if (threadIdx.x == 0) asm volatile("red.release.gpu.global.add.u32 [%0], 1;" ::"l"(ctr) : "memory");
}

__device__ __forceinline__ void dep_wait(const unsigned int* ctr, unsigned int target, unsigned int* bar, int* err) {
  uint32_t i = 0;
  for (;;) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(ctr) : "memory");
    if (v >= target) return;
    if ((++i & 63u) == 0) {
      if (ld_relaxed(&bar[2])) return;
      if (i > kGridSpinLimit) {
        atomicOr(err, ERR_SPIN_TIMEOUT);
        atomicExch(&bar[2], 1u);
        return;
      }
    }
  }
}

// Bounded mbarrier wait that also gives up once the launch has aborted.
__device__ __forceinline__ bool mbar_wait_abort(uint64_t* bar, uint32_t parity, int* err,
                                                const unsigned int* abort_flag) {
  for (uint32_t i = 0; i < kGridSpinLimit; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u && ld_relaxed(abort_flag)) return false;
  }
  atomicOr(err, ERR_MBAR_TIMEOUT);
  return false;
}

struct Ctx {
  const MegaArgs* a;
  const PhaseInfo* tmpl;   // smem: layer-0 templates of QKV, ATT, O, GU, DN, and LM
  const MegaLayer* layers;
  uint8_t* smem;
  const MegaSmem* S;       // smem copy of the layout
  uint32_t cta, G, seg;
  int warp, lane;
  // consumer item counter and producer cursor (lane 0 of each warp)
  uint32_t k;
  const int* spos;                // smem: each row's position this step (read once after EMBED)
  const unsigned long long* wl;   // producer: current weight-stream entry
  unsigned long long wnext;
  bool failed;
};

// Phase geometry from the shared-memory templates: no divisions by runtime
// values beyond the layer index, no global loads.
__device__ __forceinline__ PhaseInfo phase_at(const Ctx& c, uint32_t ph) {
  const uint32_t last = 1 + 5 * c.a->L;
  if (ph == 0) { PhaseInfo p{}; p.type = PH_EMBED; return p; }
  if (ph > last) { PhaseInfo p{}; p.type = PH_END; return p; }
  if (ph == last) return c.tmpl[5];
  const uint32_t l = (ph - 1) / 5;
  PhaseInfo p = c.tmpl[(ph - 1) - 5 * l];
  p.layer = l;
  if (p.w) p.w += (size_t)l * c.a->lstride;
  return p;
}

// Issue the warp's next weight segment into slot `slot` (lane 0).  The
// entry after it is loaded now and used by the next call.
__device__ __forceinline__ void prod_issue(Ctx& c, uint32_t slot) {
  const unsigned long long e = c.wnext;
  if (!e) return;
  c.wnext = __ldg(++c.wl);
  const uint32_t bytes = (e & 1ull) ? 2 * c.seg : c.seg;
  const uint8_t* src = reinterpret_cast<const uint8_t*>(e & ~1ull);
  uint64_t* bars = reinterpret_cast<uint64_t*>(c.smem + c.S->bars);
  uint64_t* bar = &bars[c.warp * kMaxSlots + slot];
  mbar_arrive_expect_tx(bar, bytes);
  bulk_g2s(c.smem + c.S->ring + (size_t)(c.warp * c.a->nslot + slot) * c.S->slot_bytes, src, bytes, bar);
}

__device__ __forceinline__ float* resv(const MegaArgs& a, uint32_t v) {
  return a.R + (size_t)(v % 3) * a.batch * a.H;
}

// Zero n floats of `p`, spread over the whole grid.
__device__ __forceinline__ void grid_zero(float* p, size_t n, const Ctx& c) {
  for (size_t i = (size_t)c.cta * blockDim.x + threadIdx.x; i < n; i += (size_t)c.G * blockDim.x) p[i] = 0.f;
}

// ---- prologues -------------------------------------------------------------

// O phase: merge the attention splits of the heads in [K0, K0+Kr) into fp16.
// Each thread owns (row, element) pairs and issues every load it needs --
// the S (m, l) pairs of the element's head and its S partial outputs --
// before using any, so the merge costs one round trip per pass.
__device__ __forceinline__ void stage_attn(const Ctx& c, uint32_t K0, uint32_t Kr, uint32_t bc, __half* xs) {
  constexpr int kB = 8;   // splits per batch of loads
  const MegaArgs& a = *c.a;
  const uint32_t G = a.n_q / a.n_kv, S = a.att_splits, rec = a.hd + 2;
  for (uint32_t j = threadIdx.x; j < bc * Kr; j += blockDim.x) {
    const uint32_t b = j / Kr, k = K0 + j % Kr;
    const uint32_t h = k / a.hd, d = k % a.hd, kvh = h / G, hg = h % G;
    const float* base = a.att_ws + (((size_t)(b * a.n_kv + kvh) * S) * G + hg) * rec;
    const size_t sstride = (size_t)G * rec;
    float M = -INFINITY, L = 0.f, o = 0.f;
    for (uint32_t q0 = 0; q0 < S; q0 += kB) {
      float mv[kB], lv[kB], ov[kB];
#pragma unroll
      for (int q = 0; q < kB; ++q) {
        const bool ok = q0 + q < S;
        const float* r = base + (q0 + q) * sstride;
        mv[q] = ok ? __ldcg(r) : -INFINITY;
        lv[q] = ok ? __ldcg(r + 1) : 0.f;
        ov[q] = ok ? __ldcg(r + 2 + d) : 0.f;
      }
      float nm = M;
#pragma unroll
      for (int q = 0; q < kB; ++q) nm = fmaxf(nm, mv[q]);
      const float al = M == -INFINITY ? 0.f : expf(M - nm);
      L *= al;
      o *= al;
#pragma unroll
      for (int q = 0; q < kB; ++q) {
        const float w = mv[q] == -INFINITY ? 0.f : expf(mv[q] - nm);
        L = fmaf(w, lv[q], L);
        o = fmaf(w, ov[q], o);
      }
      M = nm;
    }
    xs[j] = __float2half_rn(o / L);
  }
}

// DN phase: fp16(SiLU(g) * u) for k in [K0, K0+Kr).
__device__ void stage_silu(const Ctx& c, uint32_t K0, uint32_t Kr, uint32_t bc, __half* xs) {
  const MegaArgs& a = *c.a;
  for (uint32_t j0 = threadIdx.x; j0 < bc * Kr; j0 += 4 * blockDim.x) {
    float g[4], u[4];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t j = j0 + q * blockDim.x;
      if (j < bc * Kr) {
        const uint32_t b = j / Kr, k = K0 + j % Kr;
        g[q] = __ldcg(&a.gu_acc[((size_t)b * 2) * a.I + k]);
        u[q] = __ldcg(&a.gu_acc[((size_t)b * 2 + 1) * a.I + k]);
      }
    }
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const uint32_t j = j0 + q * blockDim.x;
      if (j < bc * Kr) {
        float v = g[q] / (1.0f + expf(-g[q])) * u[q];
        if (a.bf16r) v = bf16_trunc(v);
        xs[(size_t)(j / Kr) * Kr + (j % Kr)] = __float2half_rn(v);
      }
    }
  }
}

// One row, 128-wide groups: the DN / O prologues with the quantisation done
// from registers (warp gl takes group gl of the unit, lane l its columns
// 4l..4l+3), the same values stage_silu / stage_attn + quantize_xs produce.
template <int NT>
__device__ __forceinline__ void silu_quant_row128(const Ctx& c, uint32_t K0, uint32_t ng, uint8_t* xf, float* gsx,
                                                  float* gsum, int* gsq) {
  const MegaArgs& a = *c.a;
  for (uint32_t gl = c.warp; gl < ng; gl += kQmvWarps) {
    const uint32_t k = K0 + gl * 128 + c.lane * 4;
    const float4 g4 = __ldcg(reinterpret_cast<const float4*>(a.gu_acc + k));
    const float4 u4 = __ldcg(reinterpret_cast<const float4*>(a.gu_acc + a.I + k));
    const float gv[4] = {g4.x, g4.y, g4.z, g4.w}, uv[4] = {u4.x, u4.y, u4.z, u4.w};
    float x[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      float v = gv[i] / (1.0f + expf(-gv[i])) * uv[i];
      if (a.bf16r) v = bf16_trunc(v);
      x[i] = __half2float(__float2half_rn(v));
    }
    quant_group_row0<NT>(x, gl, c.lane, xf, gsx, gsum, gsq);
  }
  __syncthreads();
}

// O prologue for one row, 128-wide groups = heads (head_dim 128): group gl
// of the unit is head K0 / 128 + gl.  The four warps share each group's
// splits (warp w merges splits w, w + 4, ...; more loads in flight per CTA),
// combine their partial (max, sum, output) through shared memory, and the
// group's owner warp quantises.
template <int NT>
__device__ __forceinline__ void attn_quant_row128(const Ctx& c, uint32_t K0, uint32_t ng, uint8_t* xf, float* gsx,
                                                  float* gsum, int* gsq, float* scratch) {
  const MegaArgs& a = *c.a;
  const uint32_t G = a.n_q / a.n_kv, S = a.att_splits, rec = a.hd + 2;
  constexpr int kPer = (kMaxAttSplits + kQmvWarps - 1) / kQmvWarps;
  for (uint32_t gl = 0; gl < ng; ++gl) {
    const uint32_t h = K0 / 128 + gl, kvh = h / G, hg = h % G;
    const float* base = a.att_ws + ((size_t)kvh * S * G + hg) * rec;
    float mv[kPer], lv[kPer];
    float2 o0[kPer], o1[kPer];
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const uint32_t q = c.warp + kQmvWarps * j;
      const bool ok = q < S;
      const float* r = base + (size_t)q * G * rec;
      mv[j] = ok ? __ldcg(r) : -INFINITY;
      lv[j] = ok ? __ldcg(r + 1) : 0.f;
      o0[j] = ok ? __ldcg(reinterpret_cast<const float2*>(r + 2 + c.lane * 4)) : make_float2(0.f, 0.f);
      o1[j] = ok ? __ldcg(reinterpret_cast<const float2*>(r + 4 + c.lane * 4)) : make_float2(0.f, 0.f);
    }
    float M = -INFINITY;
#pragma unroll
    for (int j = 0; j < kPer; ++j) M = fmaxf(M, mv[j]);
    float L = 0.f, o[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int j = 0; j < kPer; ++j) {
      const float w = mv[j] == -INFINITY ? 0.f : expf(mv[j] - M);
      L = fmaf(w, lv[j], L);
      o[0] = fmaf(w, o0[j].x, o[0]); o[1] = fmaf(w, o0[j].y, o[1]);
      o[2] = fmaf(w, o1[j].x, o[2]); o[3] = fmaf(w, o1[j].y, o[3]);
    }
    // scratch: [warp][lane][4] outputs, then [warp][2] (max, sum)
    float* so = scratch + (c.warp * 32 + c.lane) * 4;
    so[0] = o[0]; so[1] = o[1]; so[2] = o[2]; so[3] = o[3];
    if (c.lane == 0) {
      scratch[kQmvWarps * 128 + 2 * c.warp] = M;
      scratch[kQmvWarps * 128 + 2 * c.warp + 1] = L;
    }
    __syncthreads();
    if ((uint32_t)c.warp == gl % kQmvWarps) {
      float Mt = -INFINITY;
#pragma unroll
      for (int w = 0; w < kQmvWarps; ++w) Mt = fmaxf(Mt, scratch[kQmvWarps * 128 + 2 * w]);
      float Lt = 0.f, ot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int w = 0; w < kQmvWarps; ++w) {
        const float mw = scratch[kQmvWarps * 128 + 2 * w];
        const float f = mw == -INFINITY ? 0.f : expf(mw - Mt);
        Lt = fmaf(f, scratch[kQmvWarps * 128 + 2 * w + 1], Lt);
        const float* sw = scratch + (w * 32 + c.lane) * 4;
#pragma unroll
        for (int i = 0; i < 4; ++i) ot[i] = fmaf(f, sw[i], ot[i]);
      }
      float x[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) x[i] = __half2float(__float2half_rn(ot[i] / Lt));
      quant_group_row0<NT>(x, gl, c.lane, xf, gsx, gsum, gsq);
    }
    __syncthreads();
  }
}

// ---- one matvec work unit ------------------------------------------------------
__device__ __forceinline__ void stamp(const Ctx& c, const PhaseInfo& p, uint32_t u, int i) {
  const MegaArgs& a = *c.a;
  if (!a.prof || c.cta != 0 || threadIdx.x != 0 || u != 0 || (p.layer != 1 && p.type != PH_LM)) return;
  const int which = p.type == PH_QKV ? 0 : p.type == PH_O ? 1 : p.type == PH_GU ? 2 : p.type == PH_DN ? 3
                  : p.type == PH_LM ? 4 : p.type == PH_ATT ? 5 : -1;
  if (which < 0) return;
  a.prof[2 * (2 + 5 * a.L) + 8 * which + i] = clock64();
}

// Prologue of the layouts the register-fused paths above do not cover
// (batch > 1, other group sizes or widths): stage the unit's slice of x in
// fp16 shared memory, then quantise it.  Out of line, so the single-row path
// carries neither its instructions nor its registers.
template <int NT>
__device__ __noinline__ void staged_prologue(const Ctx c, const PhaseInfo p, uint32_t K0, uint32_t Kr,
                                             uint32_t ng) {
  const MegaArgs& a = *c.a;
  const uint32_t bc = c.S->bcm;
  uint8_t* sm = c.smem;
  __half* xs = reinterpret_cast<__half*>(sm + c.S->xs);
  float* rms = reinterpret_cast<float*>(sm + c.S->rms);
  if (p.type == PH_QKV || p.type == PH_GU || p.type == PH_LM) {
    const uint32_t v = p.type == PH_QKV ? 2 * p.layer : p.type == PH_GU ? 2 * p.layer + 1 : 2 * a.L;
    const float* nw = p.type == PH_QKV ? lptr(a, a.l0.attn_norm, p.layer)
                    : p.type == PH_GU ? lptr(a, a.l0.ffn_norm, p.layer) : a.fnorm;
    const float* res = resv(a, v);
    if (bc * a.H <= 2048u) {
      stage_norm_fast(res, a.H, a.H, nw, a.eps, K0, Kr, bc, a.bf16r != 0, rms, xs);
    } else {
      block_rms(res, a.H, a.H, bc, a.eps, rms);
      stage_norm(res, a.H, nw, rms, K0, Kr, bc, a.bf16r != 0, xs);
    }
  } else if (p.type == PH_O) {
    stage_attn(c, K0, Kr, bc, xs);
  } else {
    stage_silu(c, K0, Kr, bc, xs);
  }
  quantize_xs<NT>(xs, Kr, bc, ng, a.gs, sm + c.S->xf, reinterpret_cast<float*>(sm + c.S->gsx),
                  reinterpret_cast<float*>(sm + c.S->gsum), reinterpret_cast<int*>(sm + c.S->gsq), false);
}

template <int FMT, int NT, int SUB, bool BF16S>
__device__ void qmv_unit(Ctx& c, const PhaseInfo& p, uint32_t u, bool prologue = true) {
  // the gate/up pair (SUB == 2) is always PH_GU: let the compiler drop the rest
  const int ptype = SUB == 2 ? (int)PH_GU : p.type;
  if constexpr (SUB == 1) __builtin_assume(ptype != PH_GU);
  const MegaArgs& a = *c.a;
  stamp(c, p, u, 0);
  uint32_t tile, split, G0, ng;
  unit_range(p, u, &tile, &split, &G0, &ng);
  const uint32_t gs = a.gs, cpg = gs / kChunk, K0 = G0 * gs, Kr = ng * gs;
  const uint32_t bc = c.S->bcm;
  uint8_t* sm = c.smem;
  __half* xs = reinterpret_cast<__half*>(sm + c.S->xs);
  uint8_t* xf = sm + c.S->xf;
  float* gsx = reinterpret_cast<float*>(sm + c.S->gsx);
  float* gsum = reinterpret_cast<float*>(sm + c.S->gsum);
  int* gsq = reinterpret_cast<int*>(sm + c.S->gsq);
  float* red = reinterpret_cast<float*>(sm + c.S->red);
  float* rms = reinterpret_cast<float*>(sm + c.S->rms);

  // prologue: this unit's slice of x (the LM head's x is the same for all
  // of a CTA's units, so the caller runs it once)
  bool fused = false;
  if (!prologue) {
  } else if (ptype == PH_QKV || ptype == PH_GU || ptype == PH_LM) {
    const uint32_t v = ptype == PH_QKV ? 2 * p.layer : ptype == PH_GU ? 2 * p.layer + 1 : 2 * a.L;
    const float* nw = ptype == PH_QKV ? lptr(a, a.l0.attn_norm, p.layer)
                    : ptype == PH_GU ? lptr(a, a.l0.ffn_norm, p.layer) : a.fnorm;
    const float* res = resv(a, v);
    if (bc == 1 && gs == 128 && a.H <= 2048u && a.H % 128 == 0) {
      // one row, 128-wide groups: normalise and quantise from registers
      norm_quant_row128<NT>(res, a.H, nw, a.eps, G0, ng, a.bf16r != 0, rms, xf, gsx, gsum, gsq);
      fused = true;
    }
  } else if (ptype == PH_O) {
    // the attention splits of the kv heads whose outputs this unit reads
    if (threadIdx.x == 0) {
      const uint32_t G = a.n_q / a.n_kv, ntile = num_tiles((a.n_q + 2 * a.n_kv) * a.hd);
      const uint32_t h0 = K0 / a.hd, h1 = (K0 + Kr - 1) / a.hd;
      for (uint32_t b = 0; b < a.batch; ++b)
        for (uint32_t kvh = h0 / G; kvh <= h1 / G; ++kvh)
          dep_wait(&a.dep[ntile + b * a.n_kv + kvh], a.att_splits * (p.layer + 1), a.bar, a.err);
    }
    __syncthreads();
    if (bc == 1 && gs == 128 && a.hd == 128) {
      attn_quant_row128<NT>(c, K0, ng, xf, gsx, gsum, gsq, red);
      fused = true;
    }
  } else {
    // the gate/up row tiles this unit's K range reads
    if (threadIdx.x == 0) {
      const uint32_t base = num_tiles((a.n_q + 2 * a.n_kv) * a.hd) + a.batch * a.n_kv;
      for (uint32_t t = K0 / kTileRows; t <= (K0 + Kr - 1) / kTileRows; ++t)
        dep_wait(&a.dep[base + t], a.ks_gu * (p.layer + 1), a.bar, a.err);
    }
    __syncthreads();
    if (bc == 1 && gs == 128) {
      silu_quant_row128<NT>(c, K0, ng, xf, gsx, gsum, gsq);
      fused = true;
    }
  }
  stamp(c, p, u, 1);
  if (prologue && !fused) staged_prologue<NT>(c, p, K0, Kr, ng);
  // the split-0 O / down unit adds the previous residual once: fetch it now
  // (into the dead staging area) so the load overlaps the MMAs
  float* rpre = reinterpret_cast<float*>(xs);
  const bool add_res = (ptype == PH_O || ptype == PH_DN) && split == 0;
  if (add_res) {
    const uint32_t vin = ptype == PH_O ? 2 * p.layer : 2 * p.layer + 1;
    for (uint32_t i = threadIdx.x; i < kTileRows * bc; i += blockDim.x) {
      const uint32_t rl = i / bc, b = i % bc, row = tile * kTileRows + rl;
      rpre[i] = row < p.M ? __ldcg(&resv(a, vin)[(size_t)b * a.H + row]) : 0.f;
    }
  }
  stamp(c, p, u, 2);

  float y[SUB][NT][16];
#pragma unroll
  for (int s = 0; s < SUB; ++s)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int v = 0; v < 16; ++v) y[s][n][v] = 0.f;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + c.S->bars);
  // ring items: one scale group (of each matrix of the pair), or two
  // adjacent groups of the LM head (one copy fills the whole slot)
  const uint32_t gpi = groups_per_item(ptype, ng), items = ng / gpi;
  for (uint32_t it = c.warp; it < items; it += kQmvWarps) {
    const uint32_t slot = c.k % a.nslot;
    if (!c.failed) c.failed = !mbar_wait_abort(&bars[c.warp * kMaxSlots + slot], (c.k / a.nslot) & 1u, a.err, &a.bar[2]);
    if (it == (uint32_t)c.warp) stamp(c, p, u, 6);
    const uint8_t* sb = sm + c.S->ring + (size_t)(c.warp * a.nslot + slot) * c.S->slot_bytes;
    for (uint32_t j = 0; j < gpi; ++j)
      qmv_group<FMT, NT, SUB, BF16S>(sb + j * c.seg, c.seg, xf, it * gpi + j, cpg, gsx, gsum, gsq, y);
    if (it == (uint32_t)c.warp) stamp(c, p, u, 7);
    __syncwarp();
    if (c.lane == 0) prod_issue(c, slot);
    ++c.k;
  }

  stamp(c, p, u, 3);
  // CTA reduction: red[warp][sub*128 + row][b]
  const int g = c.lane >> 2, t = c.lane & 3;
  const uint32_t nrow = kTileRows * SUB;
  float* rw = red + (size_t)c.warp * nrow * bc;
#pragma unroll
  for (int s = 0; s < SUB; ++s)
#pragma unroll
    for (int n = 0; n < NT; ++n)
#pragma unroll
      for (int v = 0; v < 16; ++v) {
        const uint32_t b = n * 4 + t;
        if (b < bc) rw[(s * kTileRows + y_row<FMT>(v, g)) * bc + b] = y[s][n][v];
      }
  __syncthreads();
  stamp(c, p, u, 4);
  const uint32_t nv = nrow * bc;
  const uint32_t qd = a.n_q * a.hd, qkv_rows = qd + 2 * a.n_kv * a.hd;
  if (ptype == PH_LM) {
    // unsplit: final logits of this tile, argmax per row
    float* lg = a.logits;
    for (uint32_t b = 0; b < bc; ++b) {
      unsigned long long best = 0ull;
      for (uint32_t r = threadIdx.x; r < kTileRows; r += blockDim.x) {
        const uint32_t row = tile * kTileRows + r;
        float v = 0.f;
#pragma unroll
        for (int w = 0; w < kQmvWarps; ++w) v += red[(size_t)w * nv + r * bc + b];
        if (row < p.M) {
          if (a.bf16r) v = bf16_trunc(v);
          if (lg) lg[(size_t)b * a.vocab + row] = v;
          const unsigned long long pk = argmax_pack(v, row);
          best = pk > best ? pk : best;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
        best = q > best ? q : best;
      }
      if (c.lane == 0 && best) atomicMax(&a.st->argmax[b], best);
    }
  } else {
    for (uint32_t i = threadIdx.x; i < nv; i += blockDim.x) {
      const uint32_t rl = i / bc, b = i % bc;
      const uint32_t s = rl / kTileRows, row = tile * kTileRows + (rl % kTileRows);
      if (row >= p.M) continue;
      float v = 0.f;
#pragma unroll
      for (int w = 0; w < kQmvWarps; ++w) v += red[(size_t)w * nv + i];
      switch (ptype) {
        case PH_QKV: atomicAdd(&a.qkv_acc[(size_t)b * qkv_rows + row], v); break;
        case PH_GU: atomicAdd(&a.gu_acc[((size_t)b * 2 + s) * a.I + row], v); break;
        default: {   // O / DN: residual versions
          const uint32_t vin = ptype == PH_O ? 2 * p.layer : 2 * p.layer + 1;
          if (add_res) v += rpre[i];
          atomicAdd(&resv(a, vin + 1)[(size_t)b * a.H + row], v);
        }
      }
    }
  }
  __syncthreads();
  if (ptype == PH_QKV) dep_signal(&a.dep[tile]);
  if (ptype == PH_GU) dep_signal(&a.dep[num_tiles((a.n_q + 2 * a.n_kv) * a.hd) + a.batch * a.n_kv + tile]);
  stamp(c, p, u, 5);
}

// Scores of one 32-position block: warp w takes positions 8w..8w+7.  Each
// lane owns HD/32 dims, forms the 8 * G partial dots, and a recursive-halving
// butterfly leaves each (position, head) sum on a lane pair.
template <int HD, int G>
__device__ __forceinline__ void att_scores(const __half* kr, const float* qs, float* ss, int warp, int lane,
                                           float inv) {
  constexpr int EPL = HD / 32, NV = 8 * G;
  float v[NV];
#pragma unroll
  for (int p = 0; p < 8; ++p) {
    float kv[EPL];
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(kr + (size_t)(8 * warp + p) * HD + lane * EPL + e));
      kv[e] = f.x; kv[e + 1] = f.y;
    }
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float d = 0.f;
#pragma unroll
      for (int e = 0; e < EPL; ++e) d = fmaf(qs[h * HD + lane * EPL + e], kv[e], d);
      v[p * G + h] = d;
    }
  }
  int idx = 0;
  int o = 16;
#pragma unroll
  for (int n = NV; n > 1; n >>= 1, o >>= 1) {
    const bool up = (lane & o) != 0;
#pragma unroll
    for (int i = 0; i < n / 2; ++i) {
      const float send = up ? v[i] : v[i + n / 2];
      const float keep = up ? v[i + n / 2] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, o);
    }
    if (up) idx += n / 2;
  }
  for (; o >= 1; o >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], o);
  // lanes sharing idx hold the same sum; the lowest of them writes it
  if ((lane & ((32 / NV) - 1)) == 0) {
    const int p = idx / G, h = idx % G;
    ss[h * kAttBlk + 8 * warp + p] = v[0] * inv;
  }
}

// Cache range of one attention unit (kv head, row, split).
struct AttGeom {
  int pos, t0, ncache, nblk;
  bool own_new;
  size_t head_off;
};

__device__ __forceinline__ AttGeom att_geom(const Ctx& c, const PhaseInfo& p, uint32_t u) {
  const MegaArgs& a = *c.a;
  const uint32_t S = a.att_splits;
  const uint32_t kvh = u % a.n_kv, b = (u / a.n_kv) % a.batch, split = u / (a.n_kv * a.batch);
  AttGeom g;
  const int pos = c.spos[b];   // range-checked when read
  const int seq = pos + 1;
  const int per = (seq + (int)S - 1) / (int)S;
  g.pos = pos;
  g.t0 = (int)split * per;
  const int t1 = min(seq, g.t0 + per);
  g.own_new = g.t0 <= pos && pos < t1;
  const int cend = min(t1, pos);
  g.ncache = cend > g.t0 ? cend - g.t0 : 0;
  g.nblk = (g.ncache + kAttBlk - 1) / kAttBlk;
  g.head_off = a.kv_layer * p.layer + ((size_t)b * a.n_kv + kvh) * a.max_ctx * a.hd;
  return g;
}

// Start the K and V copies of cached block `blk` of a unit (one thread).
template <int HD>
__device__ __forceinline__ void att_issue(const Ctx& c, const AttGeom& g, int blk) {
  const MegaArgs& a = *c.a;
  uint64_t* abars = reinterpret_cast<uint64_t*>(c.smem + c.S->abars);
  __half* kring = reinterpret_cast<__half*>(c.smem + c.S->kring);
  __half* vring = reinterpret_cast<__half*>(c.smem + c.S->vring);
  const int stg = blk % kAttStages;
  const int n = min(kAttBlk, g.ncache - blk * kAttBlk);
  const uint32_t bytes = (uint32_t)n * HD * 2;
  // the ring overlays shared memory last written through the generic proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  mbar_arrive_expect_tx(&abars[stg], 2 * bytes);
  bulk_g2s(kring + (size_t)stg * kAttBlk * HD, a.kc + g.head_off + (size_t)(g.t0 + blk * kAttBlk) * HD, bytes, &abars[stg]);
  bulk_g2s(vring + (size_t)stg * kAttBlk * HD, a.vc + g.head_off + (size_t)(g.t0 + blk * kAttBlk) * HD, bytes, &abars[stg]);
}

// ---- attention work unit -----------------------------------------------------
// One (kv head, row, split): QK-norm + RoPE of the G query heads (and of the
// new key when this split owns the current position, which it then writes to
// the cache), online softmax over the split's cached positions streamed in
// 32-position blocks, partial (m, l, o) to att_ws.
template <int HD>
__device__ void att_unit(Ctx& c, const PhaseInfo& p, uint32_t u, uint32_t (&ause)[kAttStages], bool prefetched) {
  constexpr int EPL = HD / 32;
  const MegaArgs& a = *c.a;
  const uint32_t S = a.att_splits, G = a.n_q / a.n_kv;
  const uint32_t kvh = u % a.n_kv, b = (u / a.n_kv) % a.batch, split = u / (a.n_kv * a.batch);
  (void)split;
  uint8_t* sm = c.smem;
  uint64_t* abars = reinterpret_cast<uint64_t*>(sm + c.S->abars);
  __half* kring = reinterpret_cast<__half*>(sm + c.S->kring);
  __half* vring = reinterpret_cast<__half*>(sm + c.S->vring);
  float* qs = reinterpret_cast<float*>(sm + c.S->qs);
  float* knew = reinterpret_cast<float*>(sm + c.S->knew);
  float* vnew = reinterpret_cast<float*>(sm + c.S->vnew);
  float* ss = reinterpret_cast<float*>(sm + c.S->ss);
  float* mst = reinterpret_cast<float*>(sm + c.S->stat);
  float* lst = mst + kAttMaxG;
  float* alp = lst + kAttMaxG;
  const int warp = c.warp, lane = c.lane;

  stamp(c, p, u, 0);
  const AttGeom ag = att_geom(c, p, u);
  const int pos = ag.pos, ncache = ag.ncache, nblk = ag.nblk;
  const bool own_new = ag.own_new;
  const size_t head_off = ag.head_off;
  auto issue = [&](int blk) { att_issue<HD>(c, ag, blk); };
  if (threadIdx.x == 0 && !prefetched)
    for (int blk = 0; blk < nblk && blk < kAttStages; ++blk) issue(blk);

  // the QKV row tiles holding this kv head's q heads, k and v
  if (threadIdx.x == 0) {
    const uint32_t qd = a.n_q * HD, kvd = a.n_kv * HD, tgt = a.ks_qkv * (p.layer + 1);
    for (uint32_t t = (kvh * G * HD) / kTileRows; t <= ((kvh + 1) * G * HD - 1) / kTileRows; ++t)
      dep_wait(&a.dep[t], tgt, a.bar, a.err);
    dep_wait(&a.dep[(qd + kvh * HD) / kTileRows], tgt, a.bar, a.err);
    dep_wait(&a.dep[(qd + kvd + kvh * HD) / kTileRows], tgt, a.bar, a.err);
  }
  __syncthreads();
  const uint32_t qkv_rows = (a.n_q + 2 * a.n_kv) * HD;
  const float* qrow = a.qkv_acc + (size_t)b * qkv_rows;
  const float* qn = lptr(a, a.l0.q_norm, p.layer);
  const float* kn = lptr(a, a.l0.k_norm, p.layer);
  for (uint32_t h = warp; h < G; h += kQmvWarps) {
    float v[EPL];
    norm_rope_head<HD>(qrow + (size_t)(kvh * G + h) * HD, qn, a.eps, a.theta, a.rope_style, pos, lane, v,
                       a.rope_tab + (size_t)pos * (HD / 2));
#pragma unroll
    for (int e = 0; e < EPL; ++e) qs[h * HD + lane * EPL + e] = v[e];
  }
  if (own_new && warp == kQmvWarps - 1) {
    float v[EPL];
    norm_rope_head<HD>(qrow + (size_t)a.n_q * HD + (size_t)kvh * HD, kn, a.eps, a.theta, a.rope_style,
                       pos, lane, v, a.rope_tab + (size_t)pos * (HD / 2));
    const float* vsrc = qrow + (size_t)(a.n_q + a.n_kv) * HD + (size_t)kvh * HD;
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const int d = lane * EPL + e;
      const __half kh = __float2half_rn(v[e]);
      const __half vh = __float2half_rn(__ldcg(vsrc + d));
      a.kc[head_off + (size_t)pos * HD + d] = kh;
      a.vc[head_off + (size_t)pos * HD + d] = vh;
      knew[d] = __half2float(kh);
      vnew[d] = __half2float(vh);
    }
  }
  if (threadIdx.x < kAttMaxG) {
    mst[threadIdx.x] = -INFINITY;
    lst[threadIdx.x] = 0.f;
  }
  __syncthreads();
  stamp(c, p, u, 1);

  constexpr int NHS = kQmvThreads / HD;
  const int d = threadIdx.x % HD, hs = threadIdx.x / HD;
  float acc[kAttMaxG];
#pragma unroll
  for (int h = 0; h < kAttMaxG; ++h) acc[h] = 0.f;
  const float inv = rsqrtf((float)HD);
  const int total = nblk + (own_new ? 1 : 0);
  for (int blk = 0; blk < total; ++blk) {
    const bool is_new = blk == nblk;
    const int n = is_new ? 1 : min(kAttBlk, ncache - blk * kAttBlk);
    const int stg = blk % kAttStages;
    const __half* kr = kring + (size_t)stg * kAttBlk * HD;
    const __half* vr = vring + (size_t)stg * kAttBlk * HD;
    if (!is_new) {
      if (!c.failed) c.failed = !mbar_wait_abort(&abars[stg], ause[stg] & 1u, a.err, &a.bar[2]);
      ause[stg] += 1;
      if (blk == 0) stamp(c, p, u, 2);
    }
    if (!is_new && (G == 1 || G == 2 || G == 4)) {
      // 8 positions per warp; every lane forms the partial dots of its dims
      // for all (position, head) pairs, then one transposed butterfly sums
      // all of them (8 G values over 32 lanes)
      if (G == 1) att_scores<HD, 1>(kr, qs, ss, warp, lane, inv);
      else if (G == 2) att_scores<HD, 2>(kr, qs, ss, warp, lane, inv);
      else att_scores<HD, 4>(kr, qs, ss, warp, lane, inv);
    } else {
    for (int t = warp; t < n; t += kQmvWarps) {
      float kv[EPL];
      if (is_new) {
#pragma unroll
        for (int e = 0; e < EPL; ++e) kv[e] = knew[lane * EPL + e];
      } else {
#pragma unroll
        for (int e = 0; e < EPL; e += 2) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(kr + (size_t)t * HD + lane * EPL + e));
          kv[e] = f.x; kv[e + 1] = f.y;
        }
      }
      for (uint32_t h = 0; h < G; ++h) {
        float dot = 0.f;
#pragma unroll
        for (int e = 0; e < EPL; ++e) dot = fmaf(qs[h * HD + lane * EPL + e], kv[e], dot);
        dot = warp_sum(dot);
        if (lane == 0) ss[h * kAttBlk + t] = dot * inv;
      }
    }
    }
    __syncthreads();
    for (uint32_t h = warp; h < G; h += kQmvWarps) {
      const float sv = lane < n ? ss[h * kAttBlk + lane] : -INFINITY;
      const float mx = warp_max(sv);
      const float mo = mst[h], mn = fmaxf(mo, mx);
      const float pe = lane < n ? expf(sv - mn) : 0.f;
      if (lane < n) ss[h * kAttBlk + lane] = pe;
      const float ls = warp_sum(pe);
      if (lane == 0) {
        const float al = (mo == -INFINITY) ? 0.f : expf(mo - mn);
        alp[h] = al;
        lst[h] = lst[h] * al + ls;
        mst[h] = mn;
      }
    }
    __syncthreads();
    for (uint32_t h = hs; h < G; h += NHS) {
      float o = acc[h] * alp[h];
      if (is_new) o = fmaf(ss[h * kAttBlk], vnew[d], o);
      else
        for (int t = 0; t < n; ++t) o = fmaf(ss[h * kAttBlk + t], __half2float(vr[(size_t)t * HD + d]), o);
      acc[h] = o;
    }
    __syncthreads();
    if (blk == 0) stamp(c, p, u, 3);
    if (!is_new && threadIdx.x == 0 && blk + kAttStages < nblk) issue(blk + kAttStages);
  }
  stamp(c, p, u, 4);
  const uint32_t rec = HD + 2;
  float* wsp = a.att_ws + (((size_t)(b * a.n_kv + kvh) * S + split) * G) * rec;
  for (uint32_t h = hs; h < G; h += NHS) wsp[(size_t)h * rec + 2 + d] = acc[h];
  if (threadIdx.x < G) {
    wsp[(size_t)threadIdx.x * rec + 0] = mst[threadIdx.x];
    wsp[(size_t)threadIdx.x * rec + 1] = lst[threadIdx.x];
  }
  dep_signal(&a.dep[num_tiles((a.n_q + 2 * a.n_kv) * HD) + b * a.n_kv + kvh]);
  stamp(c, p, u, 5);
}

// ---- embedding phase -------------------------------------------------------------
template <int FMT, bool BF16S>
__device__ void embed_phase(Ctx& c) {
  const MegaArgs& a = *c.a;
  uint32_t* tok_s = reinterpret_cast<uint32_t*>(c.smem + c.S->tok);
  if (c.cta == 0) {
    if (threadIdx.x < a.batch) {
      const uint32_t r = threadIdx.x;
      const int adv = a.st->advance;
      const unsigned long long am = a.st->argmax[r];
      const int p0 = a.st->pos[r];
      const uint32_t t0 = a.st->token[r];
      uint32_t tok = t0;
      if (adv) {
        tok = argmax_index(am);
        const int pp = p0 + 1;
        a.st->pos[r] = pp;
        a.st->token[r] = tok;
        if (a.seq && pp >= 0 && (uint32_t)pp < a.seq_len) a.seq[(size_t)r * a.seq_len + pp] = tok;
      }
      a.st->argmax[r] = 0ull;
      if (tok >= a.vocab) {
        atomicOr(a.err, ERR_BAD_TOKEN);
        tok = 0;
      }
      tok_s[r] = tok;
    }
    __syncthreads();
    float* out0 = resv(a, 0);
    for (uint32_t i = threadIdx.x; i < a.batch * (a.H / 8); i += blockDim.x) {
      const uint32_t r = i / (a.H / 8), d8 = i % (a.H / 8);
      const uint64_t f = (uint64_t)tok_s[r] * a.H + 8 * d8;
      float v[8];
      if constexpr (FMT == FMT_Q1) {
        const uint32_t bits = a.emb_w[f >> 3];
        const float s = __half2float(__ushort_as_half(a.emb_s[f / a.gs]));
#pragma unroll
        for (int q = 0; q < 8; ++q) v[q] = ((bits >> q) & 1u) ? s : -s;
      } else {
        const uint32_t word = reinterpret_cast<const uint32_t*>(a.emb_w)[f >> 3];
        const float s = u16_to_f32<BF16S>(a.emb_s[f / a.gs]);
        const float bb = u16_to_f32<BF16S>(a.emb_b[f / a.gs]);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          v[q] = __fadd_rn(__fmul_rn(s, (float)((word >> (4 * q)) & 0xFu)), bb);
          if (a.bf16r) v[q] = bf16_trunc(v[q]);
        }
      }
      float4* o4 = reinterpret_cast<float4*>(out0 + (size_t)r * a.H + 8 * d8);
      o4[0] = make_float4(v[0], v[1], v[2], v[3]);
      o4[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
  }
  grid_zero(resv(a, 1), (size_t)a.batch * a.H, c);
  grid_zero(a.qkv_acc, (size_t)a.batch * (a.n_q + 2 * a.n_kv) * a.hd, c);
  grid_zero(a.gu_acc, (size_t)a.batch * 2 * a.I, c);
  const uint32_t ndep = num_tiles((a.n_q + 2 * a.n_kv) * a.hd) + a.batch * a.n_kv + num_tiles(a.I);
  for (uint32_t i = c.cta * blockDim.x + threadIdx.x; i < ndep; i += c.G * blockDim.x) a.dep[i] = 0u;
}

template <int FMT, int NT, bool BF16S, int HD>
__global__ void __launch_bounds__(kQmvThreads) mega_kernel(const __grid_constant__ MegaArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  Ctx c;
  c.a = &a;
  c.layers = a.layers;
  c.smem = smem;
  __shared__ MegaSmem s_layout;
  if (threadIdx.x == 0) s_layout = mega_layout(a, FMT);
  __syncthreads();
  c.S = &s_layout;
  c.cta = blockIdx.x;
  c.G = gridDim.x;
  c.seg = seg_bytes(FMT, a.gs);
  c.warp = threadIdx.x >> 5;
  c.lane = threadIdx.x & 31;
  c.k = 0;
  c.failed = false;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + c.S->bars);
  uint64_t* abars = reinterpret_cast<uint64_t*>(smem + c.S->abars);
  PhaseInfo* tm = reinterpret_cast<PhaseInfo*>(smem + c.S->tmpl);
  c.tmpl = tm;
  if (threadIdx.x < 6) tm[threadIdx.x] = phase_info(a, nullptr, threadIdx.x < 5 ? 1 + threadIdx.x : 1 + 5 * a.L);
  for (uint32_t i = threadIdx.x; i < (c.S->u - c.S->xf) / 4; i += blockDim.x)
    reinterpret_cast<uint32_t*>(smem + c.S->xf)[i] = 0;
  if (c.lane == 0) {
    for (int s = 0; s < kMaxSlots; ++s) mbar_init(&bars[c.warp * kMaxSlots + s], 1);
    if (threadIdx.x == 0)
      for (int s = 0; s < kAttStages; ++s) mbar_init(&abars[s], 1);
    fence_barrier_init();
  }
  __syncthreads();
  unsigned long long gen = a.bar_base;
  // start this warp's weight stream
  if (c.lane == 0) {
    c.wl = a.wlist + a.woff[c.cta * kQmvWarps + c.warp];
    c.wnext = __ldg(c.wl);
    for (uint32_t s = 0; s < a.nslot; ++s) prod_issue(c, s);
  }
  uint32_t ause[kAttStages] = {0, 0};
  __shared__ int s_pos[kBatchChunk];
  c.spos = s_pos;
  const uint32_t last = 1 + 5 * a.L;
  for (uint32_t ph = 0; ph <= last; ++ph) {
    const PhaseInfo p = phase_at(c, ph);
    switch (p.type) {
      case PH_EMBED:
        embed_phase<FMT, BF16S>(c);
        break;
      case PH_ATT:
        for (uint32_t u = c.cta; u < p.units; u += c.G) att_unit<HD>(c, p, u, ause, u == c.cta);
        break;
      case PH_GU:
        grid_zero(a.qkv_acc, (size_t)a.batch * (a.n_q + 2 * a.n_kv) * a.hd, c);
        for (uint32_t u = c.cta; u < p.units; u += c.G) qmv_unit<FMT, NT, 2, BF16S>(c, p, u);
        break;
      default:
        // QKV, O, down and the LM head share this one call site, so the
        // LM head runs the instructions the layers already brought into the
        // instruction cache (the LM head's x is the same for all of a CTA's
        // units: only its first unit runs the prologue)
        if (p.type == PH_QKV) grid_zero(a.gu_acc, (size_t)a.batch * 2 * a.I, c);
        if (p.type == PH_O) grid_zero(resv(a, 2 * p.layer + 2), (size_t)a.batch * a.H, c);
        if (p.type == PH_DN) grid_zero(resv(a, 2 * p.layer + 3), (size_t)a.batch * a.H, c);
        for (uint32_t u = c.cta; u < p.units; u += c.G)
          qmv_unit<FMT, NT, 1, BF16S>(c, p, u, p.type != PH_LM || u == c.cta);
        if (p.type == PH_QKV) {
          // the cached K/V blocks of this CTA's first attention unit do not
          // depend on the barrier: start their copies now (the matvec's
          // shared-memory view is dead after its last unit's final sync)
          const PhaseInfo pa = phase_at(c, ph + 1);
          if (c.cta < pa.units && threadIdx.x == 0) {
            const AttGeom ag = att_geom(c, pa, c.cta);
            for (int blk = 0; blk < ag.nblk && blk < kAttStages; ++blk) att_issue<HD>(c, ag, blk);
          }
        }
        break;
    }
    if (a.prof && c.cta == 0 && threadIdx.x == 0) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      a.prof[2 * ph] = t;
      if (ph == 0 || ph == last) a.prof[2 * (2 + 5 * a.L) + 62 + (ph == 0 ? 0 : 1)] = clock64();
    }
    if (a.prof && threadIdx.x == 0 && ph >= 6 && ph < 11 && c.cta < 1024) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      a.prof[2 * (2 + 5 * a.L) + 64 + (ph - 6) * 1024 + c.cta] = t;
    }
    // the QKV -> attention, attention -> O and gate/up -> down edges are
    // per-unit counters
    if (ph < last && p.type != PH_QKV && p.type != PH_ATT && p.type != PH_GU) grid_sync(a.bar, c.G, gen, a.err);
    if (ph == 0) {
      // positions were advanced by the embedding phase; constant from here on
      if (threadIdx.x < a.batch) {
        int pos = __ldcg(&a.st->pos[threadIdx.x]);
        if (pos < 0 || pos >= (int)a.max_ctx) {
          if (c.cta == 0) atomicOr(a.err, ERR_BAD_POS);
          pos = pos < 0 ? 0 : (int)a.max_ctx - 1;
        }
        s_pos[threadIdx.x] = pos;
      }
      __syncthreads();
    }
    if (a.prof && c.cta == 0 && threadIdx.x == 0) {
      unsigned long long t;
      asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
      a.prof[2 * ph + 1] = t;
    }
  }
}

template <int FMT, int NT, bool BF16S, int HD>
cudaError_t launch_t(const MegaArgs& a, uint32_t grid, uint32_t smem, cudaStream_t st, bool prepare) {
  auto* fn = &mega_kernel<FMT, NT, BF16S, HD>;
  if (prepare) return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQmvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeCooperative;
  at[0].val.cooperative = 1;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

template <int FMT, int NT, bool BF16S, int HD>
int occupancy_t(uint32_t smem) {
  int n = 0;
  if (cudaFuncSetAttribute(&mega_kernel<FMT, NT, BF16S, HD>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                           smem) != cudaSuccess)
    return 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, &mega_kernel<FMT, NT, BF16S, HD>, kQmvThreads,
                                                    smem) != cudaSuccess)
    return 0;
  return n;
}

// Calls f.operator()<FMT, NT, BF16S, HD>() for a supported combination and
// returns true, else returns false.
template <typename F>
bool dispatch(int fmt, int nt, int bf16s, uint32_t hd, F&& f) {
#define NNZ_MEGA_CASE(FM, N, B, H) \
  if (fmt == FM && nt == N && bf16s == B && hd == H) { f.template operator()<FM, N, (bool)B, H>(); return true; }
  NNZ_MEGA_CASE(FMT_Q1, 1, 0, 128) NNZ_MEGA_CASE(FMT_Q1, 2, 0, 128)
  NNZ_MEGA_CASE(FMT_Q1, 1, 0, 64) NNZ_MEGA_CASE(FMT_Q1, 2, 0, 64)
  NNZ_MEGA_CASE(FMT_Q4, 1, 0, 128) NNZ_MEGA_CASE(FMT_Q4, 2, 0, 128)
  NNZ_MEGA_CASE(FMT_Q4, 1, 1, 128) NNZ_MEGA_CASE(FMT_Q4, 2, 1, 128)
  NNZ_MEGA_CASE(FMT_Q4, 1, 0, 64) NNZ_MEGA_CASE(FMT_Q4, 2, 0, 64)
  NNZ_MEGA_CASE(FMT_Q4, 1, 1, 64) NNZ_MEGA_CASE(FMT_Q4, 2, 1, 64)
#undef NNZ_MEGA_CASE
  return false;
}

}  // namespace

bool mega_plan(MegaArgs& a, int fmt, int bf16s, int device, uint32_t* grid, uint32_t* smem) {
  if (a.batch == 0 || a.batch > (uint32_t)kBatchChunk || a.bf16r || (a.hd != 64 && a.hd != 128) ||
      a.n_q > (uint32_t)kMaxHeadsPerUnit ||
      a.n_q / a.n_kv > (uint32_t)kAttMaxG)
    return false;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return false;
  const int nt = a.batch > 4 ? 2 : 1;
  const uint32_t qd = a.n_q * a.hd;
  for (int occ_try = 2; occ_try >= 1; --occ_try) {
    const uint32_t G = (uint32_t)(sms * occ_try);
    // as many units as CTAs, down to one scale group per unit: the phase
    // latency is the per-unit latency
    auto pick = [&](uint32_t M, uint32_t K) {
      const uint32_t tiles = num_tiles(M), groups = K / a.gs;
      const uint32_t ks = G / tiles;               // units <= CTAs
      return ks < 1 ? 1u : ks > groups ? groups : ks;
    };
    a.ks_qkv = pick(qd + 2 * a.n_kv * a.hd, a.H);
    a.ks_o = pick(a.H, qd);
    a.ks_gu = pick(a.I, a.H);
    a.ks_dn = pick(a.H, a.I);
    // attention splits
    // one split per 40 positions of the maximum context, at most 32: with
    // 512-768 cached positions of a 776-position cache that is ~1.3 streamed
    // blocks per split (13 splits of two blocks cost ~45 us per token more;
    // 20-32 splits measure alike, the merge in the O phase growing with them)
    uint32_t sp = (a.max_ctx + 39) / 40;
    if (const char* e = getenv("NNZ_ATT_SPLITS")) sp = (uint32_t)atoi(e);   // tuning override
    a.att_splits = sp < 1 ? 1 : sp > (uint32_t)kMaxAttSplits ? (uint32_t)kMaxAttSplits : sp;
    for (uint32_t ns = kMaxSlots; ns >= 2; --ns) {
      a.nslot = ns;
      const MegaSmem S = mega_layout(a, fmt);
      const uint32_t budget = occ_try == 2 ? 112u * 1024u : 220u * 1024u;
      if (S.total > budget) continue;
      int occ = 0;
      dispatch(fmt, nt, bf16s, a.hd, [&]<int F, int N, bool B, int H>() { occ = occupancy_t<F, N, B, H>(S.total); });
      if (occ >= occ_try) {
        *grid = G;
        *smem = S.total;
        return true;
      }
    }
  }
  return false;
}

cudaError_t mega_launch(const MegaArgs& a, int fmt, int bf16s, uint32_t grid, uint32_t smem, cudaStream_t st) {
  const int nt = a.batch > 4 ? 2 : 1;
  cudaError_t e = cudaErrorInvalidValue;
  dispatch(fmt, nt, bf16s, a.hd, [&]<int F, int N, bool B, int H>() { e = launch_t<F, N, B, H>(a, grid, smem, st, false); });
  return e;
}

std::vector<unsigned long long> mega_weight_stream(const MegaArgs& a, int fmt, uint32_t grid,
                                                   std::vector<uint32_t>* off) {
  std::vector<unsigned long long> list;
  off->assign((size_t)grid * kQmvWarps + 1, 0);
  const uint32_t seg = seg_bytes(fmt, a.gs), last = 1 + 5 * a.L;
  for (uint32_t cta = 0; cta < grid; ++cta)
    for (uint32_t w = 0; w < (uint32_t)kQmvWarps; ++w) {
      (*off)[cta * kQmvWarps + w] = (uint32_t)list.size();
      for (uint32_t ph = 1; ph <= last; ++ph) {
        const PhaseInfo p = phase_info(a, nullptr, ph);
        if (p.type != PH_QKV && p.type != PH_O && p.type != PH_GU && p.type != PH_DN && p.type != PH_LM) continue;
        for (uint32_t u = cta; u < p.units; u += grid) {
          uint32_t tile, split, G0, ng;
          unit_range(p, u, &tile, &split, &G0, &ng);
          const uint32_t gpi = groups_per_item(p.type, ng);
          for (uint32_t it = w; it < ng / gpi; it += kQmvWarps) {
            const uint8_t* src = p.w + ((size_t)tile * p.groups + G0 + it * gpi) * (p.sub * seg);
            list.push_back(reinterpret_cast<unsigned long long>(src) | (p.sub * gpi == 2 ? 1ull : 0ull));
          }
        }
      }
      list.push_back(0ull);
    }
  (*off)[(size_t)grid * kQmvWarps] = (uint32_t)list.size();
  return list;
}

}  // namespace nnz
