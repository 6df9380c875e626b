// Single-row decode kernel for 1-bit (Q1, group 128) models: one cooperative
// launch runs one or many whole greedy decode steps of a batch-1 sequence.
//
// Replaces, for batch 1, the reference's per-token command buffer
// (nnmetal/src/transformer.zig:2566-2930 forwardDecode, :4072-4123
// decodeOneToken, :3942-4027 generate) and its Q1 matvec shaders
// (nnmetal/src/shaders/qmv_specialized.metal:55-939, 1096-1279).
//
// Design (B200, 148 SMs, one CTA per SM):
//  * Weights are re-laid out at load time into one contiguous byte stream per
//    CTA, in the exact order that CTA consumes them (QKV, O, gate/up, down of
//    every layer, then its LM-head rows), copied into a 16-slot shared-memory
//    ring with 9 KiB bulk copies (TMA engine, no multicast).  The warp that
//    makes the last release of a slot issues the copy of the chunk 16
//    ahead into it, so the stream runs up to two layers ahead of the
//    compute, across token boundaries when a launch decodes several tokens.
//  * The matvec core is the int8 tensor-core MMA (m16n8k32 / m16n8k16):
//    1-bit weights become u8 {0,1} operands with one shift+AND per four
//    weights, and each activation group is an exact fixed-point integer
//    x * 2^(22-E) split into three signed bytes (three B columns), so
//    sum(sign * x) = 2 * sum(bit * x) - sum(x) is computed in int32 without
//    rounding for every element within 2^-11 of its group's maximum
//    (every fp16 value representable relative to that maximum); smaller
//    elements carry at most 2^(E-23) absolute error.
//  * Per layer the critical path is QKV -> attention -> O (dataflow counters
//    per kv head) -> grid barrier -> gate/up + SiLU*up -> grid barrier ->
//    down projection (each CTA owns whole output rows) -> grid barrier.
#pragma once
#include "common.cuh"
#include "misc.cuh"
#include <vector>

namespace nnz {

constexpr int kD1Warps = 16;                        // compute warps
constexpr int kD1Threads = kD1Warps * 32;
constexpr uint32_t kD1Unit = 288;                   // 16 rows x 128 k: 256 B bits + 32 B scales
constexpr uint32_t kD1Chunk = 9216;                 // one ring slot = 32 units
constexpr int kD1Slots = 16;
constexpr int kD1KvBlk = 32;                        // attention positions per K/V block
constexpr int kD1MaxG = 4;                          // query heads per kv head
constexpr uint32_t kD1MaxGroups = 64;               // scale groups of the widest input (hidden, intermediate <= 8192)
constexpr uint32_t kD1MaxRb = 8;                    // QKV row blocks / gate+up row blocks per CTA
constexpr uint32_t kD1MaxLayers = 64;
constexpr uint32_t kD1AttRec = 132;                 // m, l, 2 pad, o[128] (floats)

// Work assignment shared by the host packer and the kernel.  Everything is a
// pure function of the model dims and the grid size P.
struct D1Geom {
  uint32_t P, H, I, nq, nkv, L, V, max_ctx;
  uint32_t G;          // query heads per kv head
  uint32_t GH;         // scale groups along H (H / 128, a power of two)
  uint32_t lgh;        // log2(GH)
  uint32_t qkv_rows, nrb_qkv, nrb_h, nrb_i, nrb_v;
  uint32_t GI;         // scale groups along I (I / 128)
  uint32_t S;          // attention splits per kv head (nkv * S <= P)
  uint32_t nrr;        // O-projection row ranges per head (nq * nrr <= P)
  uint32_t cq, co, cg, cd, cpl, clm, nck;   // chunks: per phase, per layer, LM head, per token
};

// First item of part c when n items are cut into P near-equal parts.  32-bit
// arithmetic (d1_geom checks that P * n fits): the kernel calls it in every
// phase and a 64-bit division is a long software sequence on the GPU.
__host__ __device__ inline uint32_t d1_lo(uint32_t c, uint32_t n, uint32_t P) { return (c * n) / P; }

inline bool d1_geom(D1Geom& g, uint32_t P, uint32_t H, uint32_t I, uint32_t nq, uint32_t nkv,
                    uint32_t L, uint32_t V, uint32_t max_ctx) {
  g = D1Geom{};
  g.P = P; g.H = H; g.I = I; g.nq = nq; g.nkv = nkv; g.L = L; g.V = V; g.max_ctx = max_ctx;
  if (!nkv || nq % nkv || H % 128 || H > 128 * 32 || I % 128 || I > 128 * kD1MaxGroups || !L || L > kD1MaxLayers || !V)
    return false;
  g.G = nq / nkv;
  g.GH = H / 128;
  g.GI = I / 128;
  if (g.G > (uint32_t)kD1MaxG || 4 % g.G || 32 % g.GH) return false;
  while ((1u << g.lgh) < g.GH) ++g.lgh;
  g.qkv_rows = (nq + 2 * nkv) * 128;
  g.nrb_qkv = g.qkv_rows / 16;
  g.nrb_h = H / 16;
  g.nrb_i = I / 16;
  g.nrb_v = (V + 15) / 16;
  if (P < nkv || P < nq) return false;
  const uint32_t nmax = g.nrb_v > I ? (g.nrb_v > max_ctx ? g.nrb_v : max_ctx) : (I > max_ctx ? I : max_ctx);
  if ((uint64_t)(P + 1) * (nmax + 1) >= (1ull << 32)) return false;
  g.S = P / nkv;
  g.nrr = P / nq;
  const uint32_t qrb = (g.nrb_qkv + P - 1) / P, nb = (g.nrb_i + P - 1) / P, drb = (g.nrb_h + P - 1) / P;
  if (qrb > kD1MaxRb || 2 * nb > kD1MaxRb || drb > kD1MaxRb) return false;
  const uint32_t orb = (g.nrb_h + g.nrr - 1) / g.nrr;
  g.cq = (qrb * g.GH + 31) / 32;
  g.co = (orb + 31) / 32;
  g.cg = (2 * nb * g.GH + 31) / 32;
  g.cd = (drb * g.GI + 31) / 32;
  g.cpl = g.cq + g.co + g.cg + g.cd;
  const uint32_t lrb = (g.nrb_v + P - 1) / P;
  g.clm = (lrb * g.GH + 31) / 32;
  g.nck = g.L * g.cpl + g.clm;
  return true;
}

struct D1Layer {
  const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
};

struct D1Args {
  D1Geom g;
  float eps;
  int rope_style;
  const float2* rope_tab;          // [max_ctx][64] (cos, sin)
  const uint8_t* stream;           // [P][nck][kD1Chunk]
  const uint32_t* chunk_bytes;     // [P][nck]
  const D1Layer* layers;           // [L]
  const float* fnorm;
  const uint8_t* emb_w;            // embedding, reference layout (Q1 bits)
  const uint16_t* emb_s;           // fp16 scales per 128
  __half* kc;                      // K cache [L][slots][nkv][max_ctx][128], slot 0
  __half* vc;
  size_t kv_layer;                 // elements per layer per cache
  float* R;                        // [2][H] residual versions
  float* Z;                        // [2][H] O-projection accumulators
  uint32_t* qkv;                   // [qkv_rows] fp16 value | layer tag << 16 (see d1_tag)
  __half* h;                       // [I] SiLU(gate) * up
  float* att;                      // [nkv * S * G][kD1AttRec]
  unsigned int* cnt;               // [L][nkv] QKV row blocks done, then [L][nkv] attention splits done
  unsigned int* bar;               // [2] abort flag, [4..5] u64 grid-barrier arrivals
  unsigned long long bar_base;     // arrivals before this launch
  uint32_t epoch;                  // tokens decoded by earlier launches since the counters were cleared
  uint32_t ntok;                   // decode steps in this launch
  DecodeState* st;
  uint32_t* seq;
  uint32_t seq_len;
  float* logits;                   // optional [V]
  int* err;
  unsigned long long* tstamp;      // optional [ntok + 1] %globaltimer at token boundaries
  unsigned long long* prof;        // optional per-phase stamps (CTA 0)
};

// Tag of the layer step n = token * L + layer in the tagged QKV words: 15
// bits, never 0, so a word from the previous step (or the zeroed buffer)
// never matches; every step rewrites every word before the next one reads.
__host__ __device__ inline uint32_t d1_tag(uint32_t n) { return (n & 0x7fffu) | 0x8000u; }

// Grid barriers per decoded token: per layer one after the O projection, one
// after gate/up and one after the down projection; one after the LM head.
inline uint32_t d1_barriers_per_token(const D1Geom& g) { return 3 * g.L + 1; }

// Shared-memory bytes of the kernel.
uint32_t d1_smem_bytes();
// Cooperative launch (grid = g.P CTAs of kD1Threads threads).
cudaError_t d1_launch(const D1Args& a, cudaStream_t st);
// Checks that g.P CTAs fit co-resident on `device`.
bool d1_fits(int device, uint32_t P);

// Host packing: bytes of chunk k of CTA c (same for every token).
void d1_chunk_bytes(const D1Geom& g, std::vector<uint32_t>& out);
// Writes layer l's chunks of every CTA into `dst` ([P][cpl][kD1Chunk]) from
// reference-layout matrices (Q1 bits, row-major flat index; fp16 scales per
// 128 consecutive elements): QKV rows concatenated (qkv_rows x H), O (H x nq*128),
// gate / up (I x H), down (H x I).
void d1_pack_layer(const D1Geom& g, const uint8_t* qkv_w, const uint16_t* qkv_s, const uint8_t* o_w,
                   const uint16_t* o_s, const uint8_t* gate_w, const uint16_t* gate_s, const uint8_t* up_w,
                   const uint16_t* up_s, const uint8_t* dn_w, const uint16_t* dn_s, uint8_t* dst);
// LM-head chunks of every CTA into `dst` ([P][clm][kD1Chunk]); rows >= V are zero.
void d1_pack_lm(const D1Geom& g, const uint8_t* w, const uint16_t* s, uint8_t* dst);

}  // namespace nnz
