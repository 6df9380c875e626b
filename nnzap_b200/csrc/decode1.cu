// Single-row Q1 decode kernel (see decode1.cuh for the design summary).
//
// Per token, every CTA runs the same program:
//   token start  read the decode state (token <- previous argmax, position+1);
//                the layer-0 residual is the embedding row, which every CTA
//                dequantizes for itself (no barrier);
//   per layer l:
//     QKV   fused RMSNorm (attn_norm) + q/k/v rows of this CTA (whole K),
//           fp16 out; one release-add per row block on the kv head's counter;
//           the CTA also clears its slice of the next residual and of the
//           next O accumulator;
//     ATT   CTAs [0, nkv*S): one (kv head, position split) each: QK-norm +
//           RoPE of q/k (k and v of the new position go to the fp16 cache),
//           flash-decoding partial (max, sum, output) over the split's K/V
//           blocks (prefetched with bulk copies while QKV runs);
//     O     CTAs [0, nq*nrr): one (head, row range) each: merge the head's
//           splits, o_proj rows of that range over the head's 128 columns,
//           red.add into the O accumulator Z;
//     --- grid barrier ---
//     GU    fused RMSNorm (ffn_norm) of residual + Z, gate and up rows of
//           this CTA's intermediate slice, h = fp16(SiLU(g) * u) to L2;
//     --- grid barrier ---
//     DN    down_proj of this CTA's output rows over all of h; next
//           residual = residual + Z + down (plain stores);
//     --- grid barrier ---
//   LM      fused final RMSNorm + this CTA's LM-head rows, f32 logits
//           (optional) and a packed first-max argmax (atomicMax);
//   --- grid barrier ---
//
// Memory ordering: data produced inside the launch is read with ld.global.cg
// (L2) after an acquire (counter or barrier); producers publish with a
// release-add after a CTA barrier.  Every wait is bounded: on a timeout the
// kernel records ERR_SPIN_TIMEOUT / ERR_MBAR_TIMEOUT, raises the sticky abort
// flag that releases every other waiter, stops issuing copies, drains the
// bulk copies it has in flight and returns; the host then reports
// NNZ_ETIMEDOUT.  The red.add accumulations make the f32 sums' order (and so
// their last bits) vary from run to run.
#include <cuda_runtime.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include "decode1.cuh"

namespace nnz {

namespace {

constexpr uint32_t kD1Spin = 1u << 22;

// Inlining of the kernel's pieces (instruction footprint vs call overhead).
#ifndef D1_PHASE
#define D1_PHASE __forceinline__
#endif
#ifndef D1_MV
#define D1_MV __forceinline__
#endif
#ifndef D1_SMALL
#define D1_SMALL __forceinline__
#endif
constexpr unsigned kFull = 0xffffffffu;

// ---- shared-memory layout ----------------------------------------------------
constexpr uint32_t al16(uint32_t v) { return (v + 15u) & ~15u; }
constexpr uint32_t KV_BLKB = kD1KvBlk * 128 * 2;                       // one K (or V) block, bytes
constexpr uint32_t OFF_RING = 0;
constexpr uint32_t OFF_KV = OFF_RING + kD1Slots * kD1Chunk;            // [2 stages][K, V]
constexpr uint32_t OFF_XB = OFF_KV + 4 * KV_BLKB;                      // [group][4 k32 chunks][12 lanes] uint2
constexpr uint32_t OFF_GEF = OFF_XB + kD1MaxGroups * 4 * 12 * 8;       // [group] 2^(E-22)
constexpr uint32_t OFF_GSQ = OFF_GEF + kD1MaxGroups * 4;               // [group] sum of q
constexpr uint32_t OFF_PART = al16(OFF_GSQ + kD1MaxGroups * 4);        // [warp][rb][16] f32
constexpr uint32_t OFF_ROWS = OFF_PART + kD1Warps * kD1MaxRb * 16 * 4; // [rb * 16] f32
constexpr uint32_t OFF_RED = OFF_ROWS + kD1MaxRb * 16 * 4;             // [16] f32
constexpr uint32_t OFF_AMAX = OFF_RED + 16 * 4;                        // [16] u64
constexpr uint32_t OFF_QS = OFF_AMAX + 16 * 8;                         // [G][128] f32
constexpr uint32_t OFF_SC = OFF_QS + kD1MaxG * 128 * 4;                // [G][32] f32
constexpr uint32_t OFF_KNEW = OFF_SC + kD1MaxG * kD1KvBlk * 4;         // [128] fp16
constexpr uint32_t OFF_VNEW = OFF_KNEW + 256;                          // [128] fp16
constexpr uint32_t OFF_STAT = OFF_VNEW + 256;                          // m[4], l[4], alpha[4]
constexpr uint32_t OFF_COMB = al16(OFF_STAT + 3 * kD1MaxG * 4);        // [4][128] f32
constexpr uint32_t OFF_MER = OFF_COMB + 4 * 128 * 4;                   // [4][132] f32
constexpr uint32_t OFF_XO = OFF_MER + 4 * kD1AttRec * 4;               // [128] f32
constexpr uint32_t OFF_TOK = OFF_XO + 128 * 4;                         // tok, pos, adv
constexpr uint32_t kD1CbMax = 1024;                                    // chunk sizes cached in smem
constexpr uint32_t OFF_CB = al16(OFF_TOK + 16);                        // [kD1CbMax] chunk bytes
constexpr uint32_t OFF_RELC = OFF_CB + kD1CbMax * 4;                   // [S] releases of the slot's chunk
constexpr uint32_t OFF_ISS = OFF_RELC + kD1Slots * 4;                  // [S] last chunk issued into the slot
constexpr uint32_t OFF_LAY = al16(OFF_ISS + kD1Slots * 4);             // [L] D1Layer (norm pointers)
constexpr uint32_t OFF_BAR = al16(OFF_LAY + kD1MaxLayers * sizeof(D1Layer)); // full[S], kv[2]
constexpr uint32_t SMEM_TOTAL = OFF_BAR + (kD1Slots + 2) * 8;
static_assert(SMEM_TOTAL <= 227 * 1024, "decode1 shared memory");
static_assert(OFF_KV % 128 == 0 && OFF_XB % 16 == 0, "alignment");

// ---- small PTX helpers ---------------------------------------------------------
__device__ __forceinline__ void named_sync() {
  asm volatile("bar.sync 1, %0;" ::"n"(kD1Warps * 32) : "memory");
}
__device__ __forceinline__ unsigned int ld_relaxed_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned int ld_acquire_u32(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ unsigned long long ld_acquire_u64(const unsigned long long* p) {
  unsigned long long v;
  asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void red_release_u32(unsigned int* p, unsigned int v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void red_add_v4(float* p, float a, float b, float c, float d) {
  asm volatile("red.global.add.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(p), "f"(a), "f"(b), "f"(c), "f"(d)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive1(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async;" ::: "memory"); }
// Prefetch [p, p + bytes) into L2 (bulk, no shared memory involved).
__device__ __forceinline__ void l2_prefetch(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ unsigned long long gtimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// ---- per-warp state --------------------------------------------------------------
struct Ctx {
  const D1Args* a;
  uint8_t* sm;
  uint32_t c;
  int warp, lane;
  uint32_t rel;                  // next ring chunk this warp has not released
  bool failed;                   // a wait of this thread gave up
  unsigned long long bar_target; // thread 0: grid-barrier arrival target
  uint32_t kvseq;                // K/V blocks consumed by this CTA so far
  uint32_t kv_hi;                // thread 0: K/V block sequence numbers issued so far
  unsigned long long* pf;        // profiling: non-null on the one thread that records stamps
  bool probe;                    // profiling: layer 1 of the first token
  uint32_t nbar;                 // profiling: grid barriers seen while probing
  unsigned long long* pf2;       // profiling: per-warp LM stamps (CTA 0, first token)
};
// Profiling stamp (NNZ_D1_PROFILE=1): thread 0 of CTA 0, layer 1 of the first token.
#define D1_STAMP(c, i) do { if ((c).pf) (c).pf[i] = gtimer(); } while (0)

__device__ __forceinline__ uint64_t* fullb(uint8_t* sm, uint32_t s) { return reinterpret_cast<uint64_t*>(sm + OFF_BAR) + s; }
__device__ __forceinline__ uint64_t* kvbar(uint8_t* sm, uint32_t s) {
  return reinterpret_cast<uint64_t*>(sm + OFF_BAR) + kD1Slots + s;
}

// Issue chunk K (global index over the launch's tokens) of this CTA's weight
// stream into its ring slot.
__device__ __forceinline__ void ring_issue(const D1Args& a, uint8_t* sm, uint32_t K) {
  const uint32_t nck = a.g.nck, k = K % nck, s = K % kD1Slots;
  const uint32_t bytes = k < kD1CbMax ? reinterpret_cast<const uint32_t*>(sm + OFF_CB)[k]
                                      : __ldg(a.chunk_bytes + (size_t)blockIdx.x * nck + k);
  mbar_arrive_expect_tx(fullb(sm, s), bytes);
  if (bytes)
    bulk_g2s(sm + OFF_RING + s * kD1Chunk, a.stream + ((size_t)blockIdx.x * nck + k) * kD1Chunk, bytes, fullb(sm, s));
  reinterpret_cast<uint32_t*>(sm + OFF_ISS)[s] = K;
}

__device__ __noinline__ void raise_abort(const D1Args& a, int code) {
  atomicOr(a.err, code);
  atomicExch(&a.bar[2], 1u);
}

// Bounded mbarrier wait that also gives up once the launch has aborted.
__device__ __forceinline__ bool wait_mbar(uint64_t* b, uint32_t parity, const D1Args& a) {
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(b, parity)) return true;
    if ((i & 127u) == 127u) {
      if (ld_relaxed_u32(&a.bar[2])) return false;
      if (i > kD1Spin) {
        raise_abort(a, ERR_MBAR_TIMEOUT);
        return false;
      }
    }
  }
}

// Bounded wait used only while draining: no abort check, no error.
__device__ __forceinline__ void drain_mbar(uint64_t* b, uint32_t parity) {
  for (uint32_t i = 0; i < kD1Spin; ++i)
    if (mbar_try_wait(b, parity)) return;
}

// Bounded spin until *ctr >= target (acquire).
__device__ __forceinline__ void wait_count(const unsigned int* ctr, unsigned int target, const D1Args& a) {
  for (uint32_t i = 0;; ++i) {
    if ((int)(ld_acquire_u32(ctr) - target) >= 0) return;
    if ((i & 63u) == 63u) {
      if (ld_relaxed_u32(&a.bar[2])) return;
      if (i > kD1Spin) {
        raise_abort(a, ERR_SPIN_TIMEOUT);
        return;
      }
    }
  }
}

// Grid barrier over the compute warps of every CTA (co-resident by
// cooperative launch): one release-add per CTA on a 64-bit counter that only
// grows, acquire polls until it reaches this barrier's target.
__device__ D1_SMALL void grid_bar(Ctx& c) {
  named_sync();
  if (threadIdx.x == 0) {
    const D1Args& a = *c.a;
    if (c.probe && c.nbar < 4) a.prof[64 + c.c * 8 + 2 * c.nbar] = gtimer();
    unsigned long long* cnt = reinterpret_cast<unsigned long long*>(a.bar + 4);
    c.bar_target += a.g.P;
    asm volatile("red.release.gpu.global.add.u64 [%0], 1;" ::"l"(cnt) : "memory");
    for (uint32_t i = 0;; ++i) {
      if (ld_acquire_u64(cnt) >= c.bar_target) break;
      if ((i & 63u) == 63u) {
        if (ld_relaxed_u32(&a.bar[2])) break;
        if (i > kD1Spin) {
          raise_abort(a, ERR_SPIN_TIMEOUT);
          break;
        }
      }
    }
    if (c.probe && c.nbar < 4) a.prof[64 + c.c * 8 + 2 * c.nbar + 1] = gtimer();
    if (c.probe) ++c.nbar;
  }
  named_sync();
}

// ---- weight ring ---------------------------------------------------------------------
// Every warp releases every chunk, in order.  A release waits for the chunk
// to have been issued (the slot's issue record; so it can never count toward
// the slot's previous chunk); the warp whose release is the slot's 16th
// issues the copy of the chunk kD1Slots ahead into it.  A warp that reads a
// chunk waits for it to land before it reads and so before it releases, so
// the 16th release of a chunk always follows its landing.  Nothing is issued
// once the launch aborted.
__device__ D1_SMALL void ring_release_one(Ctx& c) {
  const uint32_t K = c.rel;
  if (!c.failed) {
    const volatile uint32_t* iss = reinterpret_cast<const volatile uint32_t*>(c.sm + OFF_ISS) + K % kD1Slots;
    for (uint32_t i = 0; *iss != K; ++i) {
      if ((i & 63u) == 63u) {
        if (ld_relaxed_u32(&c.a->bar[2])) { c.failed = true; break; }
        if (i > kD1Spin) {
          raise_abort(*c.a, ERR_SPIN_TIMEOUT);
          c.failed = true;
          break;
        }
      }
    }
  }
  __syncwarp();
  if (c.lane == 0) {
    uint32_t* relc = reinterpret_cast<uint32_t*>(c.sm + OFF_RELC) + K % kD1Slots;
    if (atomicAdd(relc, 1u) == (uint32_t)kD1Warps - 1) {
      atomicExch(relc, 0u);
      const uint32_t Kn = K + kD1Slots;
      if (Kn < c.a->ntok * c.a->g.nck && !c.failed) ring_issue(*c.a, c.sm, Kn);
    }
  }
  __syncwarp();
  ++c.rel;
}
__device__ __forceinline__ void ring_release_upto(Ctx& c, uint32_t K) {
  while (c.rel < K) ring_release_one(c);
}
__device__ __forceinline__ const uint8_t* ring_get(Ctx& c, uint32_t K) {
  ring_release_upto(c, K);
  if (c.probe && c.c == 0 && c.lane == 0 && !mbar_try_wait(fullb(c.sm, K % kD1Slots), (K / kD1Slots) & 1u))
    atomicAdd(reinterpret_cast<unsigned int*>(c.sm + OFF_TOK) + 3, 1u);
  if (!c.failed) c.failed = !wait_mbar(fullb(c.sm, K % kD1Slots), (K / kD1Slots) & 1u, *c.a);
  return c.sm + OFF_RING + (K % kD1Slots) * kD1Chunk;
}

// ---- activation quantisation ----------------------------------------------------------
// One warp, one 128-wide group; lane holds elements 4 lane .. 4 lane + 3.
// q = x * 2^(22-E) (2^E > max |x|), exact for every element within 2^-11 of
// the maximum; q = hi * 65536 + mid * 256 + lo with balanced signed bytes.
// B fragment of m16n8k32 (.s8): lane n*4 + t holds column n, k = 4t..4t+3
// (reg 0) and 16 + 4t.. (reg 1); columns 0, 1, 2 = hi, mid, lo.
// For a group maximum am >= 0: E with 2^E > am (0 for am == 0 or a
// subnormal), returned as the two exact powers of two 2^(22-E) (to scale
// into the fixed-point grid) and 2^(E-22) (back), built from the exponent
// bits: frexpf/ldexpf are long branchy sequences on the critical path.
__device__ __forceinline__ void group_scales(float am, float& up, float& down) {
  const int be = (int)((__float_as_uint(am) >> 23) & 0xFFu);   // biased exponent of am
  const int E = be ? be - 126 : 0;                              // am < 2^(be-126)
  up = __uint_as_float((uint32_t)(127 + 22 - E) << 23);
  down = __uint_as_float((uint32_t)(127 - 22 + E) << 23);
}

__device__ __forceinline__ void digits(int q, uint32_t& hi, uint32_t& mid, uint32_t& lo) {
  const int l = ((q + 128) & 255) - 128;
  const int r1 = (q - l) >> 8;
  const int m = ((r1 + 128) & 255) - 128;
  const int h = (r1 - m) >> 8;
  hi = (uint32_t)(h & 255);
  mid = (uint32_t)(m & 255);
  lo = (uint32_t)(l & 255);
}

__device__ D1_SMALL void quant_group(const float (&x)[4], uint32_t gg, int lane, uint8_t* sm) {
  float am = fmaxf(fmaxf(fabsf(x[0]), fabsf(x[1])), fmaxf(fabsf(x[2]), fabsf(x[3])));
  // |x| >= 0 orders like its bit pattern: one redux instead of a shuffle tree
  am = __uint_as_float(__reduce_max_sync(kFull, __float_as_uint(am)));
  float up, down;
  group_scales(am, up, down);
  uint32_t w0 = 0, w1 = 0, w2 = 0;
  int sum = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int q = __float2int_rn(x[i] * up);
    sum += q;
    uint32_t h, m, l;
    digits(q, h, m, l);
    w0 |= h << (8 * i);
    w1 |= m << (8 * i);
    w2 |= l << (8 * i);
  }
  sum = __reduce_add_sync(kFull, sum);
  uint32_t* xb = reinterpret_cast<uint32_t*>(sm + OFF_XB) + ((size_t)gg * 4 + (lane >> 3)) * 24;
  const int t = lane & 3, reg = (lane >> 2) & 1;
  xb[(0 * 4 + t) * 2 + reg] = w0;
  xb[(1 * 4 + t) * 2 + reg] = w1;
  xb[(2 * 4 + t) * 2 + reg] = w2;
  if (lane == 0) {
    reinterpret_cast<float*>(sm + OFF_GEF)[gg] = down;
    reinterpret_cast<int*>(sm + OFF_GSQ)[gg] = sum;
  }
}

// ---- matvec core ----------------------------------------------------------------------
// One 16-row x 128-k unit: 4 int8 MMAs.  Lane's 8 bytes: word w covers MMAs
// 2w, 2w+1; bit (s + 8i) of a word, s = 4 j' + r, is byte i of A register r
// of MMA 2w + j'.
// Row sums of 16 rows (lanes 4r hold rows r and r + 8) into lanes 0..3 as
// float4 of rows 4q..4q+3, then one vector red.add per lane.
__device__ __forceinline__ void red_rows16(float* dst, float y0, float y1, int lane) {
  const int q = lane & 3;
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int src = ((4 * q + i) & 7) * 4;
    const float a = __shfl_sync(kFull, y0, src), b = __shfl_sync(kFull, y1, src);
    v[i] = q < 2 ? a : b;
  }
  if (lane < 4) red_add_v4(dst + 4 * lane, v[0], v[1], v[2], v[3]);
}

// Per-lane digit weights of the accumulator columns: lane t = 0 holds the
// (hi, mid) columns, lane t = 1 the lo column, lanes 2 and 3 zero columns.
// Each lane folds its columns to 2 * (column value) in f32 (minus sum(q)
// on lane 0), so sum over the lane pair (t = 0, 1) of a unit's terms is
// 2 * sum(bit * q) - sum(q) = sum(sign * q): the group dot product.  The
// pair is added once per row block instead of two shuffles per unit.
struct DigitW {
  float w0, w1, sqs;
};
// Exact int -> f32 for |i| < 2^22 with two full-rate instructions (the
// conversion unit runs at a quarter of the ALU rate): the integer is placed
// in the mantissa of 1.5 * 2^23, whose value is then subtracted.  The MMA
// column sums of one unit are below 2^15 in magnitude.
__device__ __forceinline__ float i2f_small(int i) {
  return __int_as_float(0x4B400000 + i) - 12582912.0f;
}

__device__ __forceinline__ DigitW digit_w(int lane) {
  const int t = lane & 3;
  DigitW d;
  d.w0 = t == 0 ? 131072.f : t == 1 ? 2.f : 0.f;
  d.w1 = t == 0 ? 512.f : 0.f;
  d.sqs = t == 0 ? 1.f : 0.f;
  return d;
}

// One unit: 4 int8 MMAs, then this lane's f32 share of the two rows
// (rows lane / 4 and lane / 4 + 8) added into y0, y1.
__device__ __forceinline__ void unit_acc(const uint8_t* unit, uint2 wb, const uint2 (&bq)[4], float ef, int sq,
                                         const DigitW& dw, int r0, float& y0, float& y1) {
  int acc[4] = {0, 0, 0, 0};
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t W = (j < 2) ? wb.x : wb.y;
    const int sh = (j & 1) * 4;
    mma_u8s8(acc, (W >> sh) & 0x01010101u, (W >> (sh + 1)) & 0x01010101u, (W >> (sh + 2)) & 0x01010101u,
             (W >> (sh + 3)) & 0x01010101u, bq[j].x, bq[j].y);
  }
  // scales of rows r0 and r0 + 8 packed in one word (see put_unit)
  const float2 sf = __half22float2(*reinterpret_cast<const __half2*>(unit + 256 + r0 * 4));
  const float nsq = -(float)sq * dw.sqs;
  y0 = fmaf(sf.x * ef, fmaf(i2f_small(acc[0]), dw.w0, fmaf(i2f_small(acc[1]), dw.w1, nsq)), y0);
  y1 = fmaf(sf.y * ef, fmaf(i2f_small(acc[2]), dw.w0, fmaf(i2f_small(acc[3]), dw.w1, nsq)), y1);
}

__device__ __forceinline__ void load_b(const uint8_t* sm, uint32_t gg, int lane, uint2 (&bq)[4]) {
  const uint2* xb = reinterpret_cast<const uint2*>(sm + OFF_XB) + gg * 48;
#pragma unroll
  for (int j = 0; j < 4; ++j) bq[j] = lane < 12 ? xb[j * 12 + lane] : make_uint2(0u, 0u);
}

// Address of chunk K in the ring, after waiting for it to have landed (no
// release: the phase releases its chunks when it ends).
__device__ __forceinline__ const uint8_t* ring_peek(Ctx& c, uint32_t K) {
  if (!c.failed) c.failed = !wait_mbar(fullb(c.sm, K % kD1Slots), (K / kD1Slots) & 1u, *c.a);
  return c.sm + OFF_RING + (K % kD1Slots) * kD1Chunk;
}

// The matvec loop of every phase.  Units (row block rbl, group gg) of a
// phase start at ring chunk Kb, unit index rbl * GH + gg.
//   mode 0: group split -- warp w takes groups w, w + 16, ... of every row
//           block (all of the phase's chunks are resident: a phase uses at
//           most 3) and writes its partial row sums to part[w][rbl];
//   mode 1: row split -- warp w takes row blocks w, w + 16, ... whole and
//           red.adds the rows into dst[(rb_base + rbl) * 16 ..];
//   mode 2: row split LM head -- f32 logits (dst, optional) and the packed
//           first-max argmax of rows < V, returned.
__device__ D1_MV unsigned long long mv_units(Ctx& c, uint32_t Kb, uint32_t nrb, uint32_t GH, int mode,
                                             float* dst, uint32_t rb_base, uint32_t V) {
  const int lane = c.lane, r0 = lane >> 2;
  const float* gef = reinterpret_cast<const float*>(c.sm + OFF_GEF);
  const int* gsq = reinterpret_cast<const int*>(c.sm + OFF_GSQ);
  const DigitW dw = digit_w(lane);
  unsigned long long best = 0ull;
  if (mode == 0) {
    float* part = reinterpret_cast<float*>(c.sm + OFF_PART) + c.warp * kD1MaxRb * 16;
    const uint32_t nch = (nrb * GH + 31) / 32;
    for (uint32_t k = 0; k < nch; ++k) ring_peek(c, Kb + k);
    uint32_t curg = 0xffffffffu;
    uint2 bq[4] = {};
    float ef = 0.f;
    int sq = 0;
    for (uint32_t rbl = 0; rbl < nrb; ++rbl) {
      float y0 = 0.f, y1 = 0.f;
      for (uint32_t gg = c.warp; gg < GH; gg += kD1Warps) {
        if (gg != curg) {   // once per phase when the group count divides 16
          curg = gg;
          load_b(c.sm, gg, lane, bq);
          ef = gef[gg];
          sq = gsq[gg];
        }
        const uint32_t u = rbl * GH + gg;
        const uint8_t* unit = c.sm + OFF_RING + ((Kb + (u >> 5)) % kD1Slots) * kD1Chunk + (u & 31u) * kD1Unit;
        unit_acc(unit, *reinterpret_cast<const uint2*>(unit + lane * 8), bq, ef, sq, dw, r0, y0, y1);
      }
      y0 += __shfl_xor_sync(kFull, y0, 1);
      y1 += __shfl_xor_sync(kFull, y1, 1);
      if ((lane & 3) == 0) {
        part[rbl * 16 + r0] = y0;
        part[rbl * 16 + r0 + 8] = y1;
      }
    }
    return 0ull;
  }
  // row split: the GH units of a row block are contiguous in one ring chunk
  // (GH divides 32): one chunk lookup per row block, the next unit's weight
  // word loaded while the current unit's MMAs run
  for (uint32_t rbl = c.warp; rbl < nrb; rbl += kD1Warps) {
    const uint32_t u0 = rbl * GH;
    const uint8_t* base = ring_get(c, Kb + (u0 >> 5)) + (u0 & 31u) * kD1Unit;
    float y0 = 0.f, y1 = 0.f;
    uint2 wn = *reinterpret_cast<const uint2*>(base + lane * 8);
#pragma unroll 2
    for (uint32_t gg = 0; gg < GH; ++gg) {
      const uint8_t* unit = base + gg * kD1Unit;
      const uint2 wb = wn;
      if (gg + 1 < GH) wn = *reinterpret_cast<const uint2*>(unit + kD1Unit + lane * 8);
      uint2 bq[4];
      load_b(c.sm, gg, lane, bq);
      unit_acc(unit, wb, bq, gef[gg], gsq[gg], dw, r0, y0, y1);
    }
    y0 += __shfl_xor_sync(kFull, y0, 1);
    y1 += __shfl_xor_sync(kFull, y1, 1);
    if (mode == 1) {
      red_rows16(dst + (rb_base + rbl) * 16, y0, y1, lane);
    } else if ((lane & 3) == 0) {
      const uint32_t ra = (rb_base + rbl) * 16 + r0, rbb = ra + 8;
      if (ra < V) {
        if (dst) dst[ra] = y0;
        const unsigned long long k = argmax_pack(y0, ra);
        best = k > best ? k : best;
      }
      if (rbb < V) {
        if (dst) dst[rbb] = y1;
        const unsigned long long k = argmax_pack(y1, rbb);
        best = k > best ? k : best;
      }
    }
  }
  return best;
}

// ---- residual sources --------------------------------------------------------------
// Four consecutive elements [k, k+4) of the layer input: the embedding row of
// `tok` (layer 0, dequantized here) or residual buffer l & 1.
__device__ __forceinline__ void emb4(const D1Args& a, uint32_t tok, uint32_t k, float (&v)[4]) {
  const uint64_t f = (uint64_t)tok * a.g.H + k;
  const uint32_t bits = (__ldg(a.emb_w + (f >> 3)) >> (f & 7)) & 0xFu;
  const float s = h2f(__ldg(a.emb_s + f / 128));
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = ((bits >> i) & 1u) ? s : -s;
}
__device__ __forceinline__ void layer_in4(const D1Args& a, uint32_t l, uint32_t tok, uint32_t k, float (&v)[4]) {
  if (l == 0) {
    emb4(a, tok, k, v);
  } else {
    const float4 r = __ldcg(reinterpret_cast<const float4*>(a.R + (size_t)(l & 1) * a.g.H + k));
    v[0] = r.x; v[1] = r.y; v[2] = r.z; v[3] = r.w;
  }
}

// RMSNorm of the input vector (H elements; warp w owns groups w and w + 16,
// lane 4 elements of each), fp16 rounding, quantisation into the B
// fragments of every group.
// kind: 0 = layer input, 1 = layer input + O accumulator, 2 = final residual.
__device__ D1_SMALL void norm_prologue(Ctx& c, int kind, uint32_t l, uint32_t tok, const float* nw) {
  const D1Args& a = *c.a;
  const uint32_t GH = a.g.GH, H = a.g.H;
  float v[2][4];
  float4 w4[2];
  float ss = 0.f;
  // the norm weights first: their load overlaps the residual's
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t gg = c.warp + 16 * i;
    if (gg < GH) w4[i] = __ldg(reinterpret_cast<const float4*>(nw + gg * 128 + 4 * c.lane));
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t gg = c.warp + 16 * i;
    if (gg < GH) {
      const uint32_t k = gg * 128 + 4 * c.lane;
      if (kind == 2) {
        const float4 r = __ldcg(reinterpret_cast<const float4*>(a.R + (size_t)(l & 1) * H + k));
        v[i][0] = r.x; v[i][1] = r.y; v[i][2] = r.z; v[i][3] = r.w;
      } else {
        layer_in4(a, l, tok, k, v[i]);
        if (kind == 1) {
          const float4 z = __ldcg(reinterpret_cast<const float4*>(a.Z + (size_t)(l & 1) * H + k));
          v[i][0] += z.x; v[i][1] += z.y; v[i][2] += z.z; v[i][3] += z.w;
        }
      }
#pragma unroll
      for (int e = 0; e < 4; ++e) ss = fmaf(v[i][e], v[i][e], ss);
    }
  }
  D1_STAMP(c, 40 + 4 * kind);
  ss = warp_sum(ss);
  float* red = reinterpret_cast<float*>(c.sm + OFF_RED);
  if (c.lane == 0) red[c.warp] = ss;
  named_sync();
  D1_STAMP(c, 41 + 4 * kind);
  const float4* r4 = reinterpret_cast<const float4*>(red);
  const float4 q0 = r4[0], q1 = r4[1], q2 = r4[2], q3 = r4[3];
  const float tot = ((q0.x + q0.y) + (q0.z + q0.w)) + ((q1.x + q1.y) + (q1.z + q1.w)) +
                    (((q2.x + q2.y) + (q2.z + q2.w)) + ((q3.x + q3.y) + (q3.z + q3.w)));
  const float r = rsqrtf(tot / (float)H + a.eps);
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const uint32_t gg = c.warp + 16 * i;
    if (gg < GH) {
      const float wv[4] = {w4[i].x, w4[i].y, w4[i].z, w4[i].w};
      float x[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) x[e] = __half2float(__float2half_rn(v[i][e] * r * wv[e]));
      quant_group(x, gg, c.lane, c.sm);
    }
  }
  D1_STAMP(c, 42 + 4 * kind);
  named_sync();
}

// ---- attention ------------------------------------------------------------------------------
struct AttGeo {
  uint32_t j, s, t0, t1, nblk;
  bool own_new;
};

__device__ __forceinline__ AttGeo att_geo(const D1Args& a, uint32_t c, int pos) {
  AttGeo g{};
  const uint32_t S = a.g.S, n = (uint32_t)pos + 1;
  g.j = c / S;
  g.s = c % S;
  g.t0 = (g.s * n) / S;          // S * max_ctx fits 32 bits (d1_geom)
  g.t1 = ((g.s + 1) * n) / S;
  g.nblk = (g.t1 - g.t0 + kD1KvBlk - 1) / kD1KvBlk;
  g.own_new = g.t1 == n && g.t1 > g.t0;
  return g;
}

// Thread 0: bulk-copy block `blk` of the split's cached K/V (positions < pos)
// into stage (kvseq + blk) & 1.  Nothing is issued once the launch aborted.
__device__ void att_issue(Ctx& c, const AttGeo& g, uint32_t l, int pos, uint32_t blk) {
  const D1Args& a = *c.a;
  if (c.failed) return;
  const uint32_t seq = c.kvseq + blk, st = seq & 1u;
  const uint32_t tb = g.t0 + blk * kD1KvBlk;
  uint32_t te = tb + kD1KvBlk;
  te = te < g.t1 ? te : g.t1;
  te = te < (uint32_t)pos ? te : (uint32_t)pos;
  const uint32_t n = te > tb ? te - tb : 0;
  uint64_t* bar = kvbar(c.sm, st);
  mbar_arrive_expect_tx(bar, 2 * n * 256);
  if (n) {
    const size_t off = (size_t)l * a.kv_layer + ((size_t)g.j * a.g.max_ctx + tb) * 128;
    uint8_t* kd = c.sm + OFF_KV + st * 2 * KV_BLKB;
    bulk_g2s(kd, a.kc + off, n * 256, bar);
    bulk_g2s(kd + KV_BLKB, a.vc + off, n * 256, bar);
  }
  c.kv_hi = seq + 1;
}

// Lane's 4 tagged QKV words of a 128-wide row written in this launch: polls
// (relaxed, bounded) until all four carry `tag`, i.e. the producer's store of
// this layer step; the fp16 halves of the value words are returned.  The
// data is its own flag: no counter, no release / acquire pair.
__device__ __forceinline__ uint2 load_tagged(const uint32_t* row, uint32_t tag, int lane, const D1Args& a) {
  const uint32_t* p = row + 4 * lane;
  uint4 w;
  for (uint32_t i = 0;; ++i) {
    asm volatile("ld.relaxed.gpu.global.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(w.x), "=r"(w.y), "=r"(w.z), "=r"(w.w) : "l"(p) : "memory");
    if ((w.x >> 16) == tag && (w.y >> 16) == tag && (w.z >> 16) == tag && (w.w >> 16) == tag) break;
    if ((i & 63u) == 63u) {
      if (ld_relaxed_u32(&a.bar[2])) break;
      if (i > kD1Spin) {
        raise_abort(a, ERR_SPIN_TIMEOUT);
        break;
      }
    }
  }
  return make_uint2((w.x & 0xffffu) | (w.y << 16), (w.z & 0xffffu) | (w.w << 16));
}

// RMSNorm (f32) + RoPE of one 128-wide head held as 4 consecutive elements
// per lane (raw: the lane's 4 fp16 values).
__device__ __forceinline__ void norm_rope(uint2 raw, const float* nw, const float2* cs, float eps,
                                          int style, int lane, float (&v)[4]) {
  const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
  const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
  v[0] = f0.x; v[1] = f0.y; v[2] = f1.x; v[3] = f1.y;
  float ss = v[0] * v[0];
  ss = fmaf(v[1], v[1], ss);
  ss = fmaf(v[2], v[2], ss);
  ss = fmaf(v[3], v[3], ss);
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / 128.f + eps);
  const float4 w4 = __ldg(reinterpret_cast<const float4*>(nw) + lane);
  v[0] = v[0] * r * w4.x; v[1] = v[1] * r * w4.y; v[2] = v[2] * r * w4.z; v[3] = v[3] * r * w4.w;
  if (style == 0) {   // pairwise (2i, 2i+1)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const float2 q = __ldg(cs + (lane * 4 + e) / 2);
      const float x0 = v[e], x1 = v[e + 1];
      v[e] = x0 * q.x - x1 * q.y;
      v[e + 1] = x0 * q.y + x1 * q.x;
    }
  } else {            // half split (i, i + 64)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float partner = __shfl_xor_sync(kFull, v[e], 16);
      const float2 q = __ldg(cs + (lane & 15) * 4 + e);
      v[e] = lane < 16 ? v[e] * q.x - partner * q.y : partner * q.y + v[e] * q.x;
    }
  }
}

template <int GT>
__device__ D1_PHASE void att_phase(Ctx& c, uint32_t l, int pos, uint32_t epoch_tok) {
  const D1Args& a = *c.a;
  constexpr uint32_t G = GT;
  const uint32_t S = a.g.S;
  const AttGeo g = att_geo(a, c.c, pos);
  uint8_t* sm = c.sm;
  float* qs = reinterpret_cast<float*>(sm + OFF_QS);
  float* wst = reinterpret_cast<float*>(sm + OFF_SC);       // [warp][G] partial maxima
  float* acc = reinterpret_cast<float*>(sm + OFF_COMB);     // [G][128] merged outputs
  float* lsum = reinterpret_cast<float*>(sm + OFF_STAT);    // [G] merged sums
  __half* knew = reinterpret_cast<__half*>(sm + OFF_KNEW);
  __half* vnew = reinterpret_cast<__half*>(sm + OFF_VNEW);
  const int warp = c.warp, lane = c.lane;

  // the q / k / v rows of this kv head, polled as tagged words (QKV phase)
  const uint32_t tag = d1_tag(epoch_tok * a.g.L + l);
  D1_STAMP(c, 12);
  const D1Layer& LW = reinterpret_cast<const D1Layer*>(sm + OFF_LAY)[l];
  const float2* cs = a.rope_tab + (size_t)pos * 64;
  if ((uint32_t)warp < G) {
    float v[4];
    norm_rope(load_tagged(a.qkv + (size_t)(g.j * G + warp) * 128, tag, lane, a), LW.q_norm, cs, a.eps,
              a.rope_style, lane, v);
    *reinterpret_cast<float4*>(qs + warp * 128 + 4 * lane) = make_float4(v[0], v[1], v[2], v[3]);
  } else if ((uint32_t)warp == G && g.own_new) {
    float v[4];
    norm_rope(load_tagged(a.qkv + (size_t)(a.g.nq + g.j) * 128, tag, lane, a), LW.k_norm, cs, a.eps,
              a.rope_style, lane, v);
    const __half2 k01 = __floats2half2_rn(v[0], v[1]), k23 = __floats2half2_rn(v[2], v[3]);
    uint2 kk;
    kk.x = *reinterpret_cast<const uint32_t*>(&k01);
    kk.y = *reinterpret_cast<const uint32_t*>(&k23);
    const uint2 vv = load_tagged(a.qkv + (size_t)(a.g.nq + a.g.nkv + g.j) * 128, tag, lane, a);
    reinterpret_cast<uint2*>(knew)[lane] = kk;
    reinterpret_cast<uint2*>(vnew)[lane] = vv;
    const size_t off = (size_t)l * a.kv_layer + ((size_t)g.j * a.g.max_ctx + (uint32_t)pos) * 128;
    reinterpret_cast<uint2*>(a.kc + off)[lane] = kk;
    reinterpret_cast<uint2*>(a.vc + off)[lane] = vv;
  }
  named_sync();
  D1_STAMP(c, 13);

  // Each warp runs its own online softmax over positions t0 + warp, + 16, ...
  // (lane: head dims 4 lane .. 4 lane + 3 of every head); K/V blocks arrive
  // two at a time, so splits longer than 64 positions refill between rounds.
  float qv[GT][4], m[GT], ls[GT], o[GT][4];
#pragma unroll
  for (int h = 0; h < GT; ++h) {
    m[h] = -INFINITY;
    ls[h] = 0.f;
    o[h][0] = o[h][1] = o[h][2] = o[h][3] = 0.f;
    if ((uint32_t)h < G) {
      const float4 q4 = *reinterpret_cast<const float4*>(qs + h * 128 + 4 * lane);
      qv[h][0] = q4.x; qv[h][1] = q4.y; qv[h][2] = q4.z; qv[h][3] = q4.w;
    }
  }
  const float inv = 1.0f / sqrtf(128.f);
  for (uint32_t b0 = 0; b0 < g.nblk; b0 += 2) {
    for (uint32_t blk = b0; blk < b0 + 2 && blk < g.nblk; ++blk) {
      const uint32_t tb = g.t0 + blk * kD1KvBlk;
      const uint32_t nb = min((uint32_t)kD1KvBlk, g.t1 - tb);
      if ((uint32_t)warp >= nb) continue;
      const uint32_t st = (c.kvseq + blk) & 1u;
      if (!c.failed) c.failed = !wait_mbar(kvbar(sm, st), ((c.kvseq + blk) >> 1) & 1u, a);
      const __half* kb = reinterpret_cast<const __half*>(sm + OFF_KV + st * 2 * KV_BLKB);
      const __half* vb = kb + KV_BLKB / 2;
      for (uint32_t i = warp; i < nb; i += kD1Warps) {
        const bool nw = tb + i == (uint32_t)pos;
        const uint2 kr = *reinterpret_cast<const uint2*>((nw ? knew : kb + i * 128) + 4 * lane);
        const uint2 vr = *reinterpret_cast<const uint2*>((nw ? vnew : vb + i * 128) + 4 * lane);
        const float2 k0 = __half22float2(*reinterpret_cast<const __half2*>(&kr.x));
        const float2 k1 = __half22float2(*reinterpret_cast<const __half2*>(&kr.y));
        const float2 v0 = __half22float2(*reinterpret_cast<const __half2*>(&vr.x));
        const float2 v1 = __half22float2(*reinterpret_cast<const __half2*>(&vr.y));
#pragma unroll
        for (int h = 0; h < GT; ++h) {
          {
            float dot = qv[h][0] * k0.x;
            dot = fmaf(qv[h][1], k0.y, dot);
            dot = fmaf(qv[h][2], k1.x, dot);
            dot = fmaf(qv[h][3], k1.y, dot);
            const float s = warp_sum(dot) * inv;
            const float mn = fmaxf(m[h], s);
            const float al = expf(m[h] - mn), p = expf(s - mn);
            ls[h] = fmaf(ls[h], al, p);
            o[h][0] = fmaf(o[h][0], al, p * v0.x);
            o[h][1] = fmaf(o[h][1], al, p * v0.y);
            o[h][2] = fmaf(o[h][2], al, p * v1.x);
            o[h][3] = fmaf(o[h][3], al, p * v1.y);
            m[h] = mn;
          }
        }
      }
    }
    if (b0 + 2 < g.nblk) {
      named_sync();
      if (threadIdx.x == 0)
        for (uint32_t blk = b0 + 2; blk < b0 + 4 && blk < g.nblk; ++blk) att_issue(c, g, l, pos, blk);
    }
  }
  c.kvseq += g.nblk;
  D1_STAMP(c, 14);
  // merge the 16 warps' partials (the K/V stages are idle now): per-warp
  // (max, sum) and output rows to shared memory, the G x 16 rescale factors
  // once, then every (head, dim) sums its 16 rescaled rows
  float* po = reinterpret_cast<float*>(sm + OFF_KV);          // [warp][G][128]
  float* fw = reinterpret_cast<float*>(sm + OFF_SC) + kD1Warps * kD1MaxG;   // [G][16] factors
  named_sync();   // every warp is done reading the K/V stages
#pragma unroll
  for (int h = 0; h < GT; ++h)
    *reinterpret_cast<float4*>(po + (warp * GT + h) * 128 + 4 * lane) = make_float4(o[h][0], o[h][1], o[h][2], o[h][3]);
  if (lane == 0)
#pragma unroll
    for (int h = 0; h < GT; ++h) {
      wst[warp * kD1MaxG + h] = m[h];
      acc[warp * kD1MaxG + h] = ls[h];
    }
  named_sync();
  if (threadIdx.x < GT * kD1Warps) {
    const uint32_t h = threadIdx.x / kD1Warps, w = threadIdx.x % kD1Warps;
    float M = -INFINITY;
#pragma unroll
    for (int q = 0; q < kD1Warps; ++q) M = fmaxf(M, wst[q * kD1MaxG + h]);
    const float mw = wst[w * kD1MaxG + h];
    fw[h * kD1Warps + w] = mw == -INFINITY ? 0.f : expf(mw - M);
    if (w == 0) lsum[h] = M;
  }
  named_sync();
  if (threadIdx.x < G * 128) {
    const uint32_t h = threadIdx.x >> 7, d = threadIdx.x & 127u;
    float ov = 0.f, lv = 0.f;
#pragma unroll
    for (int w = 0; w < kD1Warps; ++w) {
      const float f = fw[h * kD1Warps + w];
      ov = fmaf(f, po[(w * GT + h) * 128 + d], ov);
      lv = fmaf(f, acc[w * kD1MaxG + h], lv);
    }
    float* rec = a.att + ((size_t)(g.j * S + g.s) * G + h) * kD1AttRec;
    rec[4 + d] = ov;
    if (d == 0) {
      rec[0] = lsum[h];
      rec[1] = lv;
    }
    __syncwarp();
    if (lane == 0) red_release_u32(a.cnt + (size_t)(a.g.L + l) * a.g.nkv + g.j, 1u);
  }
}

// Thread 0 of an attention CTA: prefetch the first two K/V blocks of layer l.
__device__ __forceinline__ void att_prefetch(Ctx& c, const AttGeo& g, uint32_t l, int pos) {
  for (uint32_t b = 0; b < 2 && b < g.nblk; ++b) att_issue(c, g, l, pos, b);
}

// ---- O projection -----------------------------------------------------------------------------
__device__ D1_PHASE void o_phase(Ctx& c, uint32_t l, uint32_t Kb, uint32_t epoch_tok) {
  const D1Args& a = *c.a;
  const D1Geom& G_ = a.g;
  const uint32_t h = c.c / G_.nrr, r = c.c % G_.nrr;
  const uint32_t rb0 = d1_lo(r, G_.nrb_h, G_.nrr), rb1 = d1_lo(r + 1, G_.nrb_h, G_.nrr);
  const uint32_t j = h / G_.G, gq = h % G_.G, S = G_.S;
  uint8_t* sm = c.sm;
  float* mer = reinterpret_cast<float*>(sm + OFF_MER);      // [4 warps][132]
  if (threadIdx.x == 0) wait_count(a.cnt + (size_t)(G_.L + l) * G_.nkv + j, (epoch_tok + 1) * S * G_.G * 4, a);
  named_sync();
  D1_STAMP(c, 15);
  // warps 0..3 fold splits s = warp, warp + 4, ... (lane: dims 4 lane .. + 3)
  if (c.warp < 4) {
    float M = -INFINITY, Ls = 0.f, O[4] = {0.f, 0.f, 0.f, 0.f};
    for (uint32_t s0 = c.warp; s0 < S; s0 += 32) {
      float mv[8], lv[8];
      float4 ov[8];
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const uint32_t s = s0 + 4 * q;
        if (s < S) {
          const float* rec = a.att + ((size_t)(j * S + s) * G_.G + gq) * kD1AttRec;
          mv[q] = __ldcg(rec);
          lv[q] = __ldcg(rec + 1);
          ov[q] = __ldcg(reinterpret_cast<const float4*>(rec + 4) + c.lane);
        } else {
          mv[q] = -INFINITY; lv[q] = 0.f; ov[q] = make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
      float nm = M;
#pragma unroll
      for (int q = 0; q < 8; ++q) nm = fmaxf(nm, mv[q]);
      if (nm != -INFINITY) {
        const float al = M == -INFINITY ? 0.f : expf(M - nm);
        Ls *= al; O[0] *= al; O[1] *= al; O[2] *= al; O[3] *= al;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float f = mv[q] == -INFINITY ? 0.f : expf(mv[q] - nm);
          Ls = fmaf(f, lv[q], Ls);
          O[0] = fmaf(f, ov[q].x, O[0]); O[1] = fmaf(f, ov[q].y, O[1]);
          O[2] = fmaf(f, ov[q].z, O[2]); O[3] = fmaf(f, ov[q].w, O[3]);
        }
        M = nm;
      }
    }
    reinterpret_cast<float4*>(mer + c.warp * kD1AttRec + 4)[c.lane] = make_float4(O[0], O[1], O[2], O[3]);
    if (c.lane == 0) {
      mer[c.warp * kD1AttRec] = M;
      mer[c.warp * kD1AttRec + 1] = Ls;
    }
  }
  named_sync();
  if (c.warp == 0) {
    float Mt = -INFINITY;
#pragma unroll
    for (int p = 0; p < 4; ++p) Mt = fmaxf(Mt, mer[p * kD1AttRec]);
    float Lt = 0.f, Ot[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int p = 0; p < 4; ++p) {
      const float mp = mer[p * kD1AttRec];
      const float f = mp == -INFINITY ? 0.f : expf(mp - Mt);
      Lt = fmaf(f, mer[p * kD1AttRec + 1], Lt);
      const float4 op = reinterpret_cast<const float4*>(mer + p * kD1AttRec + 4)[c.lane];
      Ot[0] = fmaf(f, op.x, Ot[0]); Ot[1] = fmaf(f, op.y, Ot[1]);
      Ot[2] = fmaf(f, op.z, Ot[2]); Ot[3] = fmaf(f, op.w, Ot[3]);
    }
    float x[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) x[e] = __half2float(__float2half_rn(Ot[e] / Lt));
    quant_group(x, 0, c.lane, sm);
  }
  named_sync();
  D1_STAMP(c, 16);
  mv_units(c, Kb, rb1 - rb0, 1, 1, a.Z + (size_t)(l & 1) * G_.H, rb0, 0);
}

// ---- gate/up + SiLU*up --------------------------------------------------------------------------
__device__ D1_PHASE void gu_phase(Ctx& c, uint32_t l, uint32_t Kg, uint32_t tok) {
  const D1Args& a = *c.a;
  const D1Geom& g = a.g;
  uint8_t* sm = c.sm;
  const uint32_t i0 = d1_lo(c.c, g.nrb_i, g.P), nb = d1_lo(c.c + 1, g.nrb_i, g.P) - i0;
  if (nb) {
    norm_prologue(c, 1, l, tok, reinterpret_cast<const D1Layer*>(sm + OFF_LAY)[l].ffn_norm);
    D1_STAMP(c, 17);
    mv_units(c, Kg, 2 * nb, g.GH, 0, nullptr, 0, 0);
    D1_STAMP(c, 18);
    named_sync();
    if (threadIdx.x < nb * 16) {
      const uint32_t p = threadIdx.x / 16, rr = threadIdx.x % 16;
      const float* part = reinterpret_cast<const float*>(sm + OFF_PART);
      float gv = 0.f, uv = 0.f;
#pragma unroll
      for (int w = 0; w < kD1Warps; ++w) {
        gv += part[(w * kD1MaxRb + 2 * p) * 16 + rr];
        uv += part[(w * kD1MaxRb + 2 * p + 1) * 16 + rr];
      }
      a.h[(size_t)i0 * 16 + threadIdx.x] = __float2half_rn(gv / (1.0f + expf(-gv)) * uv);
    }
  }
  ring_release_upto(c, Kg + g.cg);
}

// ---- down projection: whole output rows, K = I ------------------------------------------------------
__device__ D1_PHASE void dn_phase(Ctx& c, uint32_t l, uint32_t Kd, uint32_t tok) {
  const D1Args& a = *c.a;
  const D1Geom& g = a.g;
  uint8_t* sm = c.sm;
  const uint32_t rb0 = d1_lo(c.c, g.nrb_h, g.P), rb1 = d1_lo(c.c + 1, g.nrb_h, g.P), nrb = rb1 - rb0;
  if (nrb) {
    // h (fp16, written before the barrier) -> B fragments of every group
    for (uint32_t gg = c.warp; gg < g.GI; gg += kD1Warps) {
      const uint2 raw = __ldcg(reinterpret_cast<const uint2*>(a.h + (size_t)gg * 128) + c.lane);
      const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&raw.x));
      const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&raw.y));
      const float x[4] = {f0.x, f0.y, f1.x, f1.y};
      quant_group(x, gg, c.lane, sm);
    }
    named_sync();
    D1_STAMP(c, 19);
    mv_units(c, Kd, nrb, g.GI, 0, nullptr, 0, 0);
    named_sync();
    // next residual = layer input + O accumulator + down projection (plain stores)
    if (threadIdx.x < nrb * 16) {
      const uint32_t rbl = threadIdx.x / 16, rr = threadIdx.x % 16, row = rb0 * 16 + threadIdx.x;
      const float* pp = reinterpret_cast<const float*>(sm + OFF_PART);
      float y = 0.f;
#pragma unroll
      for (int w = 0; w < kD1Warps; ++w) y += pp[(w * kD1MaxRb + rbl) * 16 + rr];
      float x;
      if (l == 0) {
        const uint64_t f = (uint64_t)tok * g.H + row;
        x = ((__ldg(a.emb_w + (f >> 3)) >> (f & 7)) & 1u) ? h2f(__ldg(a.emb_s + f / 128))
                                                          : -h2f(__ldg(a.emb_s + f / 128));
      } else {
        x = __ldcg(a.R + (size_t)(l & 1) * g.H + row);
      }
      x += __ldcg(a.Z + (size_t)(l & 1) * g.H + row);
      a.R[(size_t)((l + 1) & 1) * g.H + row] = x + y;
    }
    D1_STAMP(c, 20);
  }
  ring_release_upto(c, Kd + g.cd);
}

// ---- QKV ----------------------------------------------------------------------------------------
__device__ D1_PHASE void qkv_phase(Ctx& c, uint32_t l, uint32_t Kq, uint32_t tok, uint32_t tag) {
  const D1Args& a = *c.a;
  const D1Geom& g = a.g;
  const uint32_t rb0 = d1_lo(c.c, g.nrb_qkv, g.P), rb1 = d1_lo(c.c + 1, g.nrb_qkv, g.P), nrb = rb1 - rb0;
  // clear this CTA's slice of the next layer's O accumulator
  {
    const uint32_t e0 = d1_lo(c.c, g.H / 4, g.P) * 4, e1 = d1_lo(c.c + 1, g.H / 4, g.P) * 4;
    if (threadIdx.x * 4 < e1 - e0)
      *reinterpret_cast<float4*>(a.Z + (size_t)((l + 1) & 1) * g.H + e0 + threadIdx.x * 4) =
          make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (nrb) {
    D1_STAMP(c, 8);
    norm_prologue(c, 0, l, tok, reinterpret_cast<const D1Layer*>(c.sm + OFF_LAY)[l].attn_norm);
    D1_STAMP(c, 9);
    mv_units(c, Kq, nrb, g.GH, 0, nullptr, 0, 0);
    D1_STAMP(c, 10);
    named_sync();
    if (threadIdx.x < ((nrb * 16 + 31) & ~31u)) {   // whole warps
      const uint32_t rbl = threadIdx.x / 16, rr = threadIdx.x % 16;
      if (rbl < nrb) {
        const float* part = reinterpret_cast<const float*>(c.sm + OFF_PART);
        float y = 0.f;
#pragma unroll
        for (int w = 0; w < kD1Warps; ++w) y += part[(w * kD1MaxRb + rbl) * 16 + rr];
        // fp16 value and this layer step's tag in one word: the attention
        // CTAs poll the words themselves (no flag, no release fence)
        const uint32_t w = (uint32_t)__half_as_ushort(__float2half_rn(y)) | (tag << 16);
        asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(a.qkv + rb0 * 16 + threadIdx.x), "r"(w) : "memory");
      }
    }
  }
  D1_STAMP(c, 11);
  ring_release_upto(c, Kq + g.cq);
}

// ---- LM head --------------------------------------------------------------------------------------
__device__ D1_PHASE void lm_phase(Ctx& c, uint32_t Kl) {
  const D1Args& a = *c.a;
  const D1Geom& g = a.g;
  uint8_t* sm = c.sm;
  const uint32_t rb0 = d1_lo(c.c, g.nrb_v, g.P), rb1 = d1_lo(c.c + 1, g.nrb_v, g.P);
  // the O accumulator of the last layer is free now: clear this CTA's slice
  {
    const uint32_t e0 = d1_lo(c.c, g.H / 4, g.P) * 4, e1 = d1_lo(c.c + 1, g.H / 4, g.P) * 4;
    if (threadIdx.x * 4 < e1 - e0)
      *reinterpret_cast<float4*>(a.Z + (size_t)((g.L - 1) & 1) * g.H + e0 + threadIdx.x * 4) =
          make_float4(0.f, 0.f, 0.f, 0.f);
  }
  unsigned long long best = 0ull;
  if (rb1 > rb0) {
    norm_prologue(c, 2, g.L, 0, a.fnorm);
    D1_STAMP(c, 21);
    if (c.pf2 && c.lane == 0) c.pf2[c.warp * 2] = gtimer();
    best = mv_units(c, Kl, rb1 - rb0, g.GH, 2, a.logits, rb0, g.V);
    if (c.pf2 && c.lane == 0) c.pf2[c.warp * 2 + 1] = gtimer();
  }
  ring_release_upto(c, Kl + g.clm);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long other = __shfl_xor_sync(kFull, best, o);
    best = other > best ? other : best;
  }
  unsigned long long* am = reinterpret_cast<unsigned long long*>(sm + OFF_AMAX);
  if (c.lane == 0) am[c.warp] = best;
  named_sync();
  if (threadIdx.x == 0) {
    unsigned long long b = 0ull;
#pragma unroll
    for (int w = 0; w < kD1Warps; ++w) b = am[w] > b ? am[w] : b;
    if (b) atomicMax(&a.st->argmax[0], b);
  }
}

__global__ void __launch_bounds__(kD1Threads, 1) d1_kernel(const __grid_constant__ D1Args a) {
  extern __shared__ __align__(1024) uint8_t sm[];
  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  {
    uint32_t* cbs = reinterpret_cast<uint32_t*>(sm + OFF_CB);
    const uint32_t n = a.g.nck < kD1CbMax ? a.g.nck : kD1CbMax;
    for (uint32_t i = threadIdx.x; i < n; i += blockDim.x) cbs[i] = __ldg(a.chunk_bytes + (size_t)blockIdx.x * a.g.nck + i);
    if (threadIdx.x < (uint32_t)kD1Slots) {
      reinterpret_cast<uint32_t*>(sm + OFF_RELC)[threadIdx.x] = 0u;
      reinterpret_cast<uint32_t*>(sm + OFF_ISS)[threadIdx.x] = 0xffffffffu;   // nothing issued yet
    }
    for (uint32_t i = threadIdx.x; i < a.g.L; i += blockDim.x)
      reinterpret_cast<D1Layer*>(sm + OFF_LAY)[i] = a.layers[i];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kD1Slots; ++s) mbar_init(fullb(sm, s), 1);
    mbar_init(kvbar(sm, 0), 1);
    mbar_init(kvbar(sm, 1), 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t total = a.ntok * a.g.nck;
    for (uint32_t K = 0; K < (uint32_t)kD1Slots && K < total; ++K) ring_issue(a, sm, K);
  } else if (threadIdx.x == 32) {
    const D1Layer* lt = reinterpret_cast<const D1Layer*>(sm + OFF_LAY);
    l2_prefetch(lt[0].attn_norm, a.g.H * 4);
    l2_prefetch(lt[0].ffn_norm, a.g.H * 4);
    l2_prefetch(lt[0].q_norm, 512);
    l2_prefetch(lt[0].k_norm, 512);
  }
  Ctx c{};
  c.a = &a;
  c.sm = sm;
  c.c = blockIdx.x;
  c.warp = warp;
  c.lane = lane;
  c.bar_target = a.bar_base;
  const D1Geom& g = a.g;
  const bool att_cta = c.c < g.nkv * g.S;
  const bool o_cta = c.c < g.nq * g.nrr;
  uint32_t* tokp = reinterpret_cast<uint32_t*>(sm + OFF_TOK);
  const bool stamps = a.prof && c.c == 0 && threadIdx.x == 0;
  if (a.tstamp && c.c == 0 && threadIdx.x == 0) a.tstamp[0] = gtimer();
  int pos = 0;
  for (uint32_t t = 0; t < a.ntok; ++t) {
    const uint32_t ep = a.epoch + t;
    if (threadIdx.x == 0) {
      int adv;
      unsigned long long am;
      uint32_t t0;
      if (t == 0) {
        adv = a.st->advance;
        am = a.st->argmax[0];
        pos = a.st->pos[0];
        t0 = a.st->token[0];
      } else {
        adv = 1;
        am = __ldcg(&a.st->argmax[0]);
        t0 = 0;
      }
      uint32_t tok = adv ? argmax_index(am) : t0;
      if (adv) ++pos;
      int bad = 0;
      if (tok >= g.V) { bad |= ERR_BAD_TOKEN; tok = 0; }
      if (pos < 0 || (uint32_t)pos >= g.max_ctx) { bad |= ERR_BAD_POS; pos = pos < 0 ? 0 : (int)g.max_ctx - 1; }
      if (bad && c.c == 0) atomicOr(a.err, bad);
      tokp[0] = tok;
      tokp[1] = (uint32_t)pos;
      tokp[2] = (uint32_t)adv;
    }
    named_sync();
    const uint32_t tok = tokp[0];
    pos = (int)tokp[1];
    const int adv = (int)tokp[2];
    const uint32_t Kt = t * g.nck;
    AttGeo ag{};
    if (att_cta) ag = att_geo(a, c.c, pos);
    for (uint32_t l = 0; l < g.L; ++l) {
      const uint32_t Kl = Kt + l * g.cpl;
      const bool st_l = stamps && t == 0 && l == 1;
      c.pf = st_l ? a.prof : nullptr;
      c.probe = a.prof && t == 0 && l == 1;
      if (c.probe && threadIdx.x == 0) tokp[3] = 0u;
      c.nbar = 0;
      if (l > 0) grid_bar(c);
      if (st_l) a.prof[0] = gtimer();
      if (threadIdx.x == 32) {
        // the next layer's (or the final) norm vectors: L2 misses on the
        // critical path otherwise (the streamed weights evict them)
        const D1Layer* lt = reinterpret_cast<const D1Layer*>(sm + OFF_LAY);
        if (l + 1 < g.L) {
          l2_prefetch(lt[l + 1].attn_norm, g.H * 4);
          l2_prefetch(lt[l + 1].ffn_norm, g.H * 4);
          l2_prefetch(lt[l + 1].q_norm, 512);
          l2_prefetch(lt[l + 1].k_norm, 512);
        } else {
          l2_prefetch(a.fnorm, g.H * 4);
          l2_prefetch(lt[0].attn_norm, g.H * 4);
          l2_prefetch(lt[0].ffn_norm, g.H * 4);
          l2_prefetch(lt[0].q_norm, 512);
          l2_prefetch(lt[0].k_norm, 512);
        }
      }
      if (l == 0 && att_cta && threadIdx.x == 0) {
        // every cache row the bulk copies of this token read was written by
        // generic stores in earlier tokens, ordered before this point by the
        // grid barriers; one proxy fence orders them before the async reads
        fence_proxy_async();
        att_prefetch(c, ag, 0, pos);
      }
      qkv_phase(c, l, Kl, tok, d1_tag(ep * g.L + l));
      if (st_l) a.prof[1] = gtimer();
      if (att_cta) {
        if (g.G == 1) att_phase<1>(c, l, pos, ep);
        else if (g.G == 2) att_phase<2>(c, l, pos, ep);
        else att_phase<4>(c, l, pos, ep);
        if (threadIdx.x == 0 && l + 1 < g.L) att_prefetch(c, ag, l + 1, pos);
      }
      if (st_l) a.prof[2] = gtimer();
      if (o_cta) o_phase(c, l, Kl + g.cq, ep);
      ring_release_upto(c, Kl + g.cq + g.co);
      if (st_l) a.prof[3] = gtimer();
      grid_bar(c);
      if (st_l) a.prof[4] = gtimer();
      if (l == 0 && c.c == 0 && threadIdx.x == 0) {
        // every CTA has read the decode state of this token by now
        a.st->pos[0] = pos;
        a.st->token[0] = tok;
        if (adv && a.seq && (uint32_t)pos < a.seq_len) a.seq[pos] = tok;
        a.st->argmax[0] = 0ull;
      }
      gu_phase(c, l, Kl + g.cq + g.co, tok);
      grid_bar(c);
      if (st_l) a.prof[22] = gtimer();
      dn_phase(c, l, Kl + g.cq + g.co + g.cg, tok);
      if (st_l) a.prof[5] = gtimer();
      if (c.probe) {
        named_sync();
        if (threadIdx.x == 0 && c.c == 0) a.prof[30] = tokp[3];
      }
    }
    c.pf = nullptr;
    grid_bar(c);
    if (stamps && t == 0) a.prof[6] = gtimer();
    c.pf = (stamps && t == 0) ? a.prof : nullptr;
    c.pf2 = (a.prof && c.c == 0 && t == 0) ? a.prof + 64 + 8 * g.P : nullptr;
    lm_phase(c, Kt + g.L * g.cpl);
    if (stamps && t == 0) a.prof[7] = gtimer();
    c.pf = nullptr;
    grid_bar(c);
    if (a.tstamp && c.c == 0 && threadIdx.x == 0) a.tstamp[t + 1] = gtimer();
  }
  // drain copies that failed waits skipped: the last one issued into every
  // ring slot and K/V stage has landed before the CTA exits
  named_sync();
  if (threadIdx.x == 0 && (c.failed || ld_relaxed_u32(&a.bar[2]))) {
    const uint32_t total = a.ntok * g.nck;
    for (uint32_t s = 0; s < (uint32_t)kD1Slots && s < total; ++s) {
      const uint32_t K = reinterpret_cast<const uint32_t*>(sm + OFF_ISS)[s];
      drain_mbar(fullb(sm, s), (K / kD1Slots) & 1u);
    }
  }
  if (threadIdx.x == 0 && c.kv_hi > c.kvseq) {
    for (uint32_t s = c.kv_hi > 2 ? c.kv_hi - 2 : 0; s < c.kv_hi; ++s) drain_mbar(kvbar(sm, s & 1u), (s >> 1) & 1u);
  }
}

// ---- host packing helpers -----------------------------------------------------------------------------
inline uint32_t bit_at(const uint8_t* bits, uint32_t M, uint32_t K, uint32_t row, uint32_t k) {
  if (row >= M) return 0;
  const uint64_t f = (uint64_t)row * K + k;
  return (bits[f >> 3] >> (f & 7)) & 1u;
}
inline uint16_t scale_at(const uint16_t* s, uint32_t M, uint32_t K, uint32_t row, uint32_t grp) {
  if (row >= M) return 0;
  return s[(uint64_t)row * (K / 128) + grp];
}

// 16 rows from row0, group gg (128 k) of an M x K matrix -> one 288-byte unit.
void put_unit(uint8_t* dst, const uint8_t* bits, const uint16_t* s, uint32_t M, uint32_t K, uint32_t row0,
              uint32_t gg) {
  uint8_t tile[16][16];
  for (uint32_t rr = 0; rr < 16; ++rr) {
    const uint32_t row = row0 + rr;
    if (row < M) memcpy(tile[rr], bits + ((uint64_t)row * K + gg * 128) / 8, 16);
    else memset(tile[rr], 0, 16);
  }
  for (uint32_t lane = 0; lane < 32; ++lane) {
    for (uint32_t w = 0; w < 2; ++w) {
      uint32_t W = 0;
      for (uint32_t b = 0; b < 32; ++b) {
        const uint32_t s8 = b % 8, i = b / 8, j = 2 * w + s8 / 4, r = s8 % 4;
        const uint32_t rr = lane / 4 + (r & 1) * 8;
        const uint32_t k = j * 32 + (r >> 1) * 16 + (lane % 4) * 4 + i;
        W |= ((uint32_t)(tile[rr][k >> 3] >> (k & 7)) & 1u) << b;
      }
      memcpy(dst + lane * 8 + w * 4, &W, 4);
    }
  }
  // scales: word r (r < 8) = (row r, row r + 8), the two rows of lane 4 r
  for (uint32_t rr = 0; rr < 16; ++rr) {
    const uint16_t v = scale_at(s, M, K, row0 + rr, gg);
    memcpy(dst + 256 + (rr % 8) * 4 + (rr / 8) * 2, &v, 2);
  }
}

}  // namespace

uint32_t d1_smem_bytes() { return SMEM_TOTAL; }

bool d1_fits(int device, uint32_t P) {
  int nsm = 0, coop = 0, per = 0;
  if (cudaDeviceGetAttribute(&nsm, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, device) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  if (!coop || (uint32_t)nsm < P) return false;
  cudaError_t e = cudaFuncSetAttribute(d1_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_TOTAL);
  if (e == cudaSuccess) e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per, d1_kernel, kD1Threads, SMEM_TOTAL);
  const char* dbg = getenv("NNZ_D1_DEBUG");
  if (dbg && dbg[0] == '1')
    fprintf(stderr, "decode1: smem %u B, blocks/SM %d, %s\n", SMEM_TOTAL, per, cudaGetErrorString(e));
  if (e != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  return per >= 1;
}

cudaError_t d1_launch(const D1Args& a, cudaStream_t st) {
  void* args[] = {const_cast<D1Args*>(&a)};
  return cudaLaunchCooperativeKernel((const void*)d1_kernel, dim3(a.g.P), dim3(kD1Threads), args, SMEM_TOTAL, st);
}

void d1_chunk_bytes(const D1Geom& g, std::vector<uint32_t>& out) {
  out.assign((size_t)g.P * g.nck, 0u);
  auto fill = [](uint32_t* dst, uint32_t nchunks, uint32_t units, uint32_t per, uint32_t ubytes) {
    for (uint32_t q = 0; q < nchunks; ++q) {
      const uint32_t n = units > q * per ? (units - q * per < per ? units - q * per : per) : 0;
      dst[q] = n * ubytes;
    }
  };
  for (uint32_t c = 0; c < g.P; ++c) {
    uint32_t* row = out.data() + (size_t)c * g.nck;
    const uint32_t nq_rb = d1_lo(c + 1, g.nrb_qkv, g.P) - d1_lo(c, g.nrb_qkv, g.P);
    const uint32_t dn_rb = d1_lo(c + 1, g.nrb_h, g.P) - d1_lo(c, g.nrb_h, g.P);
    const uint32_t nb = d1_lo(c + 1, g.nrb_i, g.P) - d1_lo(c, g.nrb_i, g.P);
    uint32_t o_rb = 0;
    if (c < g.nq * g.nrr) {
      const uint32_t r = c % g.nrr;
      o_rb = d1_lo(r + 1, g.nrb_h, g.nrr) - d1_lo(r, g.nrb_h, g.nrr);
    }
    for (uint32_t l = 0; l < g.L; ++l) {
      uint32_t* L0 = row + (size_t)l * g.cpl;
      fill(L0, g.cq, nq_rb * g.GH, 32, kD1Unit);
      fill(L0 + g.cq, g.co, o_rb, 32, kD1Unit);
      fill(L0 + g.cq + g.co, g.cg, 2 * nb * g.GH, 32, kD1Unit);
      fill(L0 + g.cq + g.co + g.cg, g.cd, dn_rb * g.GI, 32, kD1Unit);
    }
    const uint32_t lm_rb = d1_lo(c + 1, g.nrb_v, g.P) - d1_lo(c, g.nrb_v, g.P);
    fill(row + (size_t)g.L * g.cpl, g.clm, lm_rb * g.GH, 32, kD1Unit);
  }
}

void d1_pack_layer(const D1Geom& g, const uint8_t* qkv_w, const uint16_t* qkv_s, const uint8_t* o_w,
                   const uint16_t* o_s, const uint8_t* gate_w, const uint16_t* gate_s, const uint8_t* up_w,
                   const uint16_t* up_s, const uint8_t* dn_w, const uint16_t* dn_s, uint8_t* dst) {
  const size_t stride = (size_t)g.cpl * kD1Chunk;
  for (uint32_t c = 0; c < g.P; ++c) {
    uint8_t* base = dst + (size_t)c * stride;
    memset(base, 0, stride);
    // QKV: units (rb, group) rb-major
    {
      const uint32_t rb0 = d1_lo(c, g.nrb_qkv, g.P), rb1 = d1_lo(c + 1, g.nrb_qkv, g.P);
      uint32_t u = 0;
      for (uint32_t rb = rb0; rb < rb1; ++rb)
        for (uint32_t gg = 0; gg < g.GH; ++gg, ++u)
          put_unit(base + (u / 32) * kD1Chunk + (u % 32) * kD1Unit, qkv_w, qkv_s, g.qkv_rows, g.H, rb * 16, gg);
    }
    // O: (head h, row range r): rbs of the range, group h of K = nq * 128
    if (c < g.nq * g.nrr) {
      const uint32_t h = c / g.nrr, r = c % g.nrr;
      const uint32_t rb0 = d1_lo(r, g.nrb_h, g.nrr), rb1 = d1_lo(r + 1, g.nrb_h, g.nrr);
      uint8_t* ob = base + (size_t)g.cq * kD1Chunk;
      for (uint32_t rb = rb0; rb < rb1; ++rb) {
        const uint32_t u = rb - rb0;
        put_unit(ob + (u / 32) * kD1Chunk + (u % 32) * kD1Unit, o_w, o_s, g.H, g.nq * 128, rb * 16, h);
      }
    }
    const uint32_t i0 = d1_lo(c, g.nrb_i, g.P), nb = d1_lo(c + 1, g.nrb_i, g.P) - i0;
    // gate/up: pair p -> gate rb (GH units), up rb (GH units)
    {
      uint8_t* gb = base + (size_t)(g.cq + g.co) * kD1Chunk;
      uint32_t u = 0;
      for (uint32_t p = 0; p < nb; ++p)
        for (uint32_t half = 0; half < 2; ++half)
          for (uint32_t gg = 0; gg < g.GH; ++gg, ++u)
            put_unit(gb + (u / 32) * kD1Chunk + (u % 32) * kD1Unit, half ? up_w : gate_w, half ? up_s : gate_s,
                     g.I, g.H, (i0 + p) * 16, gg);
    }
    // down: units (rb, group) rb-major over this CTA's output row blocks, K = I
    {
      uint8_t* db = base + (size_t)(g.cq + g.co + g.cg) * kD1Chunk;
      const uint32_t rb0 = d1_lo(c, g.nrb_h, g.P), rb1 = d1_lo(c + 1, g.nrb_h, g.P);
      uint32_t u = 0;
      for (uint32_t rb = rb0; rb < rb1; ++rb)
        for (uint32_t gg = 0; gg < g.GI; ++gg, ++u)
          put_unit(db + (u / 32) * kD1Chunk + (u % 32) * kD1Unit, dn_w, dn_s, g.H, g.I, rb * 16, gg);
    }
  }
}

void d1_pack_lm(const D1Geom& g, const uint8_t* w, const uint16_t* s, uint8_t* dst) {
  const size_t stride = (size_t)g.clm * kD1Chunk;
  for (uint32_t c = 0; c < g.P; ++c) {
    uint8_t* base = dst + (size_t)c * stride;
    memset(base, 0, stride);
    const uint32_t rb0 = d1_lo(c, g.nrb_v, g.P), rb1 = d1_lo(c + 1, g.nrb_v, g.P);
    uint32_t u = 0;
    for (uint32_t rb = rb0; rb < rb1; ++rb)
      for (uint32_t gg = 0; gg < g.GH; ++gg, ++u)
        put_unit(base + (u / 32) * kD1Chunk + (u % 32) * kD1Unit, w, s, g.V, g.H, rb * 16, gg);
  }
}

}  // namespace nnz
