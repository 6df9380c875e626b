// Batch-1 quantized matvec on the tile-packed layout: one thread-block
// cluster per 128-row tile, K split across the cluster's CTAs and reduced
// through distributed shared memory (qmvf.cu).
#pragma once
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace nnz {

struct QmvfArgs {
  const uint8_t* w;       // packed weights (packing.h)
  uint32_t M, K, gs;
  uint32_t ks;            // CTAs per cluster (set by qmvf_launch)
  const __half* x;        // [K] fp16, 16-byte aligned
  void* out;              // fp16 / f32 [M]
  int epi;                // EPI_F16, EPI_F32 or EPI_RESADD (qmv.cuh)
  uint32_t bf16_round;    // truncate outputs to BF16 first (engine Q4 mode)
  int* err;
};

// Whether the fast path takes this call (one row, a supported epilogue, and
// a K slice per CTA that fits shared memory).
bool qmvf_applies(int fmt, uint32_t M, uint32_t K, uint32_t gs, uint32_t batch, int epi, int num_sms);
uint32_t qmvf_pick_ks(int fmt, uint32_t M, uint32_t K, uint32_t gs, int num_sms);
// Raise the kernels' shared-memory limit (once per device, outside capture).
cudaError_t qmvf_prepare();
cudaError_t qmvf_launch(int fmt, bool bf16s, QmvfArgs a, int num_sms, cudaStream_t st);

}  // namespace nnz
