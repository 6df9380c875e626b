// Persistent decode kernel: one cooperative launch runs a whole decode step
// (embedding, every decoder layer, final norm + LM head + argmax) for up to
// 8 rows.  Replaces the reference's per-token command buffer of ~172
// dispatches (nnmetal/src/transformer.zig:2566-2930, 4072-4123).
#pragma once
#include "misc.cuh"
#include "qmv_dev.cuh"
#include <vector>

namespace nnz {

struct MegaLayer {
  const uint8_t *qkv, *o, *gu, *down;
  const float *attn_norm, *ffn_norm, *q_norm, *k_norm;
};

struct MegaArgs {
  uint32_t H, I, n_q, n_kv, hd, L, vocab, gs, max_ctx, batch;
  float eps, theta;
  int rope_style, bf16r;
  const float2* rope_tab;       // [max_ctx][hd / 2] (cos, sin) of every position
  const MegaLayer* layers;      // device array [L] (unused on the hot path)
  MegaLayer l0;                 // layer 0 pointers; layer l = l0 + l * lstride bytes
  size_t lstride;
  const uint8_t* lm;            // packed LM head
  const float* fnorm;
  const uint8_t* emb_w;         // embedding, reference layout
  const uint16_t* emb_s;
  const uint16_t* emb_b;
  __half* kc;                   // K cache base [L][slots][n_kv][max_ctx][hd]
  __half* vc;
  size_t kv_layer;              // elements per layer per cache
  float* R;                     // 3 rotating residual buffers [3][batch][H]
  float* qkv_acc;               // [batch][(n_q + 2 n_kv) hd]
  float* gu_acc;                // [batch][2][I]
  float* att_ws;                // attention split partials
  uint32_t att_splits;
  uint32_t ks_qkv, ks_o, ks_gu, ks_dn;   // K splits per phase
  DecodeState* st;
  uint32_t* seq;
  uint32_t seq_len;
  float* logits;                // optional [batch][vocab]
  unsigned int* bar;            // [2] abort flag, [4..5] u64 arrival counter
  unsigned long long bar_base;  // arrival count before this launch
  // dataflow counters replacing the grid barriers after the QKV, attention
  // and gate/up phases: [qkv tiles] QKV units done per row tile,
  // [batch][n_kv] attention splits done, [I tiles] gate/up units done per
  // row tile; zeroed by the embedding phase
  unsigned int* dep;
  int* err;
  uint32_t nslot;               // weight-ring slots per warp
  unsigned long long* prof;     // optional: CTA 0 records %globaltimer after each phase
  // Weight stream: warp w of CTA c copies the segments wlist[woff[4c+w]..]
  // in order (address | 1 for a two-matrix segment), up to a 0 entry.
  const unsigned long long* wlist;
  const uint32_t* woff;
};

// Launch (cooperative) with the grid / shared memory chosen by mega_plan.
cudaError_t mega_launch(const MegaArgs& a, int fmt, int bf16s, uint32_t grid, uint32_t smem,
                        cudaStream_t st);
// Host-side plan: grid size, smem size, splits.  Returns false if the
// kernel cannot be co-resident on this device.
bool mega_plan(MegaArgs& a, int fmt, int bf16s, int device, uint32_t* grid, uint32_t* smem);
// Host-side weight stream of a plan: every warp's segment sequence, in the
// order its consumer loop visits them.  `off` gets grid * 4 + 1 offsets.
std::vector<unsigned long long> mega_weight_stream(const MegaArgs& a, int fmt, uint32_t grid,
                                                   std::vector<uint32_t>* off);

}  // namespace nnz
