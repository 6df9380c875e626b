// GQA decode attention over the fp16 KV cache with fused per-head
// QK-RMSNorm, RoPE and KV-cache write.
//
// Replaces nnmetal/src/shaders/transformer.metal:1467-1695
// (gqa_attention_fused_f16io_tg) and its long-context fallback
// (:840, :940, :1176): q = RoPE(RMSNorm_hd(q) * qn) kept in f32,
// k = RoPE(RMSNorm_hd(k) * kn) stored fp16 at `pos`, v stored fp16,
// scores = q.k / sqrt(hd) in f32, softmax f32, out = sum p v -> fp16.
//
// B200 design: flash-decoding.  One CTA per (kv head, query row, split);
// the CTA serves all G = n_q / n_kv query heads of its kv head, so each K/V
// byte is read once.  K/V blocks of 32 positions stream into a 4-stage
// shared-memory ring with 1-D bulk copies issued before griddepcontrol.wait
// (past positions are constant), an online softmax runs per block, and the
// splits of one (kv head, row) are merged by the last CTA to arrive.  Any
// context length up to max_context_length is handled (the reference's fused
// kernel stops at 1024).  RoPE angles are computed in double precision.
//
// Cache layout: [slot][kv_head][max_ctx][hd] for both K and V (the
// reference's V is transposed [d][t]; the values stored are identical).
#pragma once
#include "common.cuh"
#include "rope_dev.cuh"

namespace nnz {

constexpr int kAttnThreads = 128;
constexpr int kAttnBlk = 32;     // positions per streamed block
constexpr int kAttnStages = 4;
constexpr int kAttnMaxG = 8;     // query heads per kv head
constexpr int kTcChunk = 256;    // positions per task of the tensor-core kernel


struct AttnArgs {
  const __half* qkv;   // [rows][qkv_stride]: q | k | v
  uint32_t qkv_stride;
  const float* q_norm;
  const float* k_norm;
  __half* kc;          // layer base of the K cache
  __half* vc;          // layer base of the V cache
  uint32_t max_ctx;
  uint32_t slots;      // cache slots behind kc / vc (0: rows)
  const int* pos;      // [rows] position of each query row
  const int* slot;     // [rows] cache slot of each row (nullptr: slot = row)
  uint32_t rows;
  uint32_t n_q, n_kv;
  float eps, theta;
  int rope_style;
  int write_kv;        // 1: this launch writes row's k/v at pos and attends to it
  uint32_t splits;     // CTAs per (kv head, row)
  __half* out;         // [rows][n_q*hd]
  uint32_t out_stride;
  float* ws;
  uint32_t* counters;  // [rows][n_kv], zero at rest
  int* err;
  const float2* rope_tab;   // optional [max_ctx][hd / 2] (cos, sin) table
};

// Raise the dynamic shared-memory limit (once per device, before launches).
cudaError_t attn_prepare();
// Picks the tensor-core kernel (attn_tc.cu) when it applies (head_dim 128,
// G in {1, 2, 4}; NNZ_ATTN=legacy forces the other), else the CUDA-core one.
cudaError_t attn_decode_launch(const AttnArgs& a, int head_dim, int pdl, cudaStream_t st);
// Workspace (floats) either kernel may need.
size_t attn_ws_floats(uint32_t rows, uint32_t n_q, uint32_t n_kv, uint32_t splits, int head_dim,
                      uint32_t max_ctx);

// Tensor-core decode attention (attn_tc.cu).
bool attn_tc_applies(uint32_t n_q, uint32_t n_kv, int head_dim);
size_t attn_tc_ws_floats(uint32_t rows, uint32_t n_q, uint32_t n_kv, uint32_t max_ctx);
cudaError_t attn_tc_prepare();
cudaError_t attn_tc_launch(const AttnArgs& a, int pdl, cudaStream_t st);
// Causal prefill attention on the tensor cores (same contract as
// attn_prefill_launch; head_dim 128, G in {1, 2, 4}).
// Uses a.ws (attn_prefill_tc_ws_floats) for the key splits' partials.
cudaError_t attn_prefill_tc_launch(const AttnArgs& a, int pdl, cudaStream_t st);
// Causal prefill attention on tcgen05 / TMEM (attn_pf.cu): one CTA per
// (kv head, 128 / G query positions), no workspace; a.slots must be the
// number of cache slots (the K/V tensor maps cover exactly those).  The default for head_dim
// 128; NNZ_PREFILL_ATTN=mma selects attn_prefill_tc_launch instead.
bool attn_pf_umma_applies(uint32_t n_q, uint32_t n_kv);
cudaError_t attn_pf_umma_launch(const AttnArgs& a, int pdl, cudaStream_t st);
size_t attn_prefill_tc_ws_floats(uint32_t rows, uint32_t n_q);

// Writes normed+roped k and v of `rows` query rows at their positions
// (used by chunked prefill, where rows of one chunk share a cache slot and
// must all be written before any row attends).
cudaError_t rope_kv_write_launch(const AttnArgs& a, int head_dim, int pdl, cudaStream_t st);
// Causal attention of a prefill chunk (rows attend to positions <= their own;
// K/V of the chunk already written).  Writes `out` like attn_decode_launch.
cudaError_t attn_prefill_launch(const AttnArgs& a, int head_dim, int pdl, cudaStream_t st);

}  // namespace nnz
