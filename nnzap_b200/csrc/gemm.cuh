// Prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// Y[m][n] = sum_k X[m][k] * W[n][k] for a whole prompt chunk: X are the
// fp16 activations (M = prompt tokens, K-major), W a quantized weight matrix
// in the reference's flat layout (Q1 sign bits + fp16 scale, or Q4 nibbles +
// scale/bias; nnmetal/src/metal.zig:235-469).  The reference has no prefill
// GEMM (it runs the prompt token by token through the decode path,
// nnmetal/src/transformer.zig:4032-4068); this kernel replaces that loop's
// matvecs with one GEMM per projection.
//
// Per CTA: a 128 x 128 output tile, K in steps of 64 through a 4-stage
// shared-memory ring.  Thread 0 loads the X tile with a TMA tensor copy
// (128B swizzle) and issues tcgen05.mma kind::f16 into a TMEM accumulator;
// all 128 threads dequantize the weight tile straight into the same
// canonical 128B-swizzled K-major layout (Q1: +-scale is exact in fp16).
// The epilogue reads the accumulator with tcgen05.ld and fuses the fp16
// store, the residual add, or SiLU(gate) * up.
#pragma once
#include <cuda.h>
#include "common.cuh"
#include "packing.h"

namespace nnz {

enum GemmEpi : int { GEPI_F16 = 0, GEPI_RESADD = 1, GEPI_SILU = 2, GEPI_F32 = 3 };

struct GemmArgs {
  uint32_t M, K, N;              // tokens, reduction dim, weight rows (per matrix)
  int fmt, gs, bf16s, bf16r;
  const uint8_t* w;              // weight matrix (gate for SILU), reference layout
  const uint16_t* s;
  const uint16_t* b;
  const uint8_t* w2;             // SILU: up matrix
  const uint16_t* s2;
  const uint16_t* b2;
  int epi;
  // split-K accumulator for the F16 / F32 / SILU epilogues (f32, zero at
  // rest, [M][N] or [M][2][N] for SILU; the finalize kernel re-zeroes it);
  // null: those epilogues never split K
  float* acc;
  size_t acc_floats;
  void* out;                     // f16 [M][ldo], f32 residual [M][ldo] (+=), or f32 [M][ldo] (GEPI_F32)
  uint32_t ldo;
  int* err;
  int prof;                      // set by gemm_launch from NNZ_GEMM_PROFILE
  int pdl;                       // launch with programmatic dependent launch (GEMM and finalize)
};

// Builds the TMA descriptor for X [M][K] fp16 (row stride K) and launches.
cudaError_t gemm_launch(const GemmArgs& a, const __half* x, cudaStream_t st);
// 2-D fp16 tensor map with 128-byte swizzle: `outer` rows of `inner`
// elements, row pitch row_bytes, boxes of box_outer x box_inner (box_inner
// * 2 = 128 bytes).  False if the driver entry point or the encode fails.
bool tensor_map_f16_2d(CUtensorMap* tm, const void* base, uint64_t inner, uint64_t outer, uint64_t row_bytes,
                       uint32_t box_inner, uint32_t box_outer);
// Development aid: the 128 clock64() stamps of the last profiled launch.
cudaError_t gemm_debug_profile(unsigned long long* out);
// RMSNorm rows of an f32 residual into fp16 (the prefill GEMM's X operand).
cudaError_t rmsnorm_f16_launch(const float* res, const float* w, float eps, uint32_t rows, uint32_t K,
                               int bf16r, __half* out, cudaStream_t st, int pdl = 0);

}  // namespace nnz
