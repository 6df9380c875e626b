// Embedding lookup + decode-state advance, packed-weight dequantizer.
#pragma once
#include "common.cuh"
#include "packing.h"

namespace nnz {

constexpr int kMaxRows = 1024;   // query rows per forward (batch or prefill chunk)

// Device-resident decode state.  The embedding kernel advances it, so a
// captured decode graph can be replayed token after token with no host work:
// it consumes the previous LM-head argmax as the next token, bumps the
// position, and records the token in `seq`.
struct DecodeState {
  int pos[kMaxRows];
  uint32_t token[kMaxRows];
  unsigned long long argmax[kMaxRows];
  int advance;            // 1: take the token from argmax (graph replay)
};

struct EmbedArgs {
  const uint8_t* wbytes;      // reference layout: Q1 bits / Q4 u32 words
  const uint16_t* scales;
  const uint16_t* biases;
  uint32_t vocab, H, gs;
  int bf16_round;
  DecodeState* st;            // may be null when `tokens` is given
  const uint32_t* tokens;     // explicit token ids (prefill); null -> state
  uint32_t* seq;              // [rows][seq_len] generated-token record
  uint32_t seq_len;
  float* residual;            // [rows][H]
  uint32_t rows;
  int* err;
};

cudaError_t embed_launch(const EmbedArgs& a, int fmt, int bf16s, int pdl, cudaStream_t st);
// argmax[r] = max(argmax[r], packed first-max of logits[r][0..n)) for r < rows
// (the packed slot the decode state consumes; see argmax_pack).
// Sampling (sample.cu): rows x n logits (row stride `stride`, modified in
// place), one uniform draw per row; the token goes to the argmax slot and,
// when `tokens` is given, to tokens[row].
cudaError_t sample_launch(float* logits, uint32_t rows, uint32_t n, uint32_t stride, float temperature,
                          uint32_t top_k, float top_p, const float* uniforms, unsigned long long* argmax,
                          uint32_t* tokens, cudaStream_t st);
cudaError_t logits_argmax_launch(const float* logits, uint32_t rows, uint32_t n, uint32_t stride,
                                 unsigned long long* argmax, cudaStream_t st);
cudaError_t dequant_launch(int fmt, int bf16s, const uint8_t* w, uint32_t M, uint32_t K, uint32_t gs,
                           uint32_t sub, uint32_t si, float* out, cudaStream_t st);

}  // namespace nnz
