// Embedding gather/dequant with device-side decode-state advance, and the
// packed-weight dequantizer used for bit-exact weight checks.
#include <cuda_runtime.h>

#include "misc.cuh"

namespace nnz {

namespace {

template <int FMT, bool BF16S>
__global__ void __launch_bounds__(256) embed_kernel(EmbedArgs a) {
  __shared__ uint32_t tok_s;
  const uint32_t r = blockIdx.x;
  pdl_wait();
  pdl_launch();
  if (threadIdx.x == 0) {
    uint32_t tok;
    if (a.tokens) {
      tok = a.tokens[r];
    } else {
      // issue the three state reads together
      const int adv = a.st->advance;
      const unsigned long long am = a.st->argmax[r];
      const int p0 = a.st->pos[r];
      const uint32_t t0 = a.st->token[r];
      if (adv) {
        tok = argmax_index(am);
        const int p = p0 + 1;
        a.st->pos[r] = p;
        a.st->token[r] = tok;
        if (a.seq && p >= 0 && (uint32_t)p < a.seq_len) a.seq[(size_t)r * a.seq_len + p] = tok;
      } else {
        tok = t0;
      }
    }
    if (a.st) a.st->argmax[r] = 0ull;
    if (tok >= a.vocab) {
      atomicOr(a.err, ERR_BAD_TOKEN);
      tok = 0;
    }
    tok_s = tok;
  }
  __syncthreads();
  const uint32_t tok = tok_s;
  float* out = a.residual + (size_t)r * a.H;
  // one thread per 8 consecutive elements: one bits byte / one nibble word
  // and one scale (gs >= 32) each, all loads independent
  for (uint32_t d8 = threadIdx.x; d8 < a.H / 8; d8 += blockDim.x) {
    const uint64_t f = (uint64_t)tok * a.H + 8 * d8;
    float v[8];
    if constexpr (FMT == FMT_Q1) {
      const uint32_t bits = a.wbytes[f >> 3];
      const float s = __half2float(__ushort_as_half(a.scales[f / a.gs]));
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = ((bits >> i) & 1u) ? s : -s;
    } else {
      const uint32_t word = reinterpret_cast<const uint32_t*>(a.wbytes)[f >> 3];
      const float s = u16_to_f32<BF16S>(a.scales[f / a.gs]);
      const float b = u16_to_f32<BF16S>(a.biases[f / a.gs]);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        v[i] = __fadd_rn(__fmul_rn(s, (float)((word >> (4 * i)) & 0xFu)), b);
        if (a.bf16_round) v[i] = bf16_trunc(v[i]);
      }
    }
    float4* o4 = reinterpret_cast<float4*>(out + 8 * d8);
    o4[0] = make_float4(v[0], v[1], v[2], v[3]);
    o4[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

template <int FMT, bool BF16S>
__global__ void dequant_kernel(const uint8_t* w, uint32_t M, uint32_t K, uint32_t gs, uint32_t sub,
                               uint32_t si, float* out) {
  const uint64_t idx = (uint64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (uint64_t)M * K) return;
  const uint32_t row = (uint32_t)(idx / K), col = (uint32_t)(idx % K);
  const uint32_t T = row / kTileRows, rr = row % kTileRows;
  const uint32_t G = col / gs, cc = (col % gs) / kChunk, kk = col % kChunk;
  const uint32_t groups = K / gs, seg = seg_bytes(FMT, gs);
  const uint8_t* base = w + ((size_t)(T * groups + G) * sub + si) * seg;
  const uint32_t t = (kk & 15) >> 2, i = kk & 3, rhi = kk >> 4;
  if constexpr (FMT == FMT_Q1) {
    const uint32_t j = rr >> 4, g = rr & 7, rlo = (rr >> 3) & 1;
    const uint32_t L = g * 4 + t, r = rhi * 2 + rlo;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(base + cc * 512 + L * 16 + r * 4);
    const uint32_t bit = (word >> (j + 8 * i)) & 1u;
    const uint32_t v = 2 * j + rlo;
    const uint16_t raw = reinterpret_cast<const uint16_t*>(base + (gs / kChunk) * 512)[g * 16 + v];
    const float s = __half2float(__ushort_as_half(raw));
    out[idx] = bit ? s : -s;
  } else {
    const uint32_t u = rr >> 5, w32 = rr & 31, hiN = w32 >> 4, g = w32 & 7, rlo = (w32 >> 3) & 1;
    const uint32_t L = g * 4 + t, r = rhi * 2 + rlo;
    const uint32_t word = *reinterpret_cast<const uint32_t*>(base + cc * 2048 + u * 512 + L * 16 + r * 4);
    const uint32_t byte = (word >> (8 * i)) & 0xFFu;
    const uint32_t q = hiN ? (byte >> 4) : (byte & 0xFu);
    const uint32_t v = 4 * u + (hiN ? 2 : 0) + rlo;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(base + (gs / kChunk) * 2048) + g * 32;
    const float s = u16_to_f32<BF16S>(sc[v]), b = u16_to_f32<BF16S>(sc[16 + v]);
    out[idx] = __fadd_rn(__fmul_rn(s, (float)q), b);
  }
}

}  // namespace

cudaError_t embed_launch(const EmbedArgs& a, int fmt, int bf16s, int pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.rows);
  cfg.blockDim = dim3(256);
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  if (fmt == FMT_Q1) return cudaLaunchKernelEx(&cfg, &embed_kernel<FMT_Q1, false>, a);
  if (bf16s) return cudaLaunchKernelEx(&cfg, &embed_kernel<FMT_Q4, true>, a);
  return cudaLaunchKernelEx(&cfg, &embed_kernel<FMT_Q4, false>, a);
}

cudaError_t dequant_launch(int fmt, int bf16s, const uint8_t* w, uint32_t M, uint32_t K, uint32_t gs,
                           uint32_t sub, uint32_t si, float* out, cudaStream_t st) {
  const uint64_t n = (uint64_t)M * K;
  const uint32_t blocks = (uint32_t)((n + 255) / 256);
  if (fmt == FMT_Q1) dequant_kernel<FMT_Q1, false><<<blocks, 256, 0, st>>>(w, M, K, gs, sub, si, out);
  else if (bf16s) dequant_kernel<FMT_Q4, true><<<blocks, 256, 0, st>>>(w, M, K, gs, sub, si, out);
  else dequant_kernel<FMT_Q4, false><<<blocks, 256, 0, st>>>(w, M, K, gs, sub, si, out);
  return cudaGetLastError();
}

namespace {
constexpr uint32_t kArgThreads = 256, kArgItems = 8;
__global__ void __launch_bounds__(kArgThreads) logits_argmax_kernel(const float* logits, uint32_t n, uint32_t stride,
                                                                    unsigned long long* argmax) {
  const uint32_t r = blockIdx.y;
  const float* x = logits + (size_t)r * stride;
  const uint32_t i0 = blockIdx.x * kArgThreads * kArgItems + threadIdx.x;
  float v[kArgItems];
#pragma unroll
  for (int u = 0; u < (int)kArgItems; ++u) {
    const uint32_t i = i0 + u * kArgThreads;
    v[u] = i < n ? __ldcg(x + i) : 0.f;
  }
  unsigned long long best = 0ull;
#pragma unroll
  for (int u = 0; u < (int)kArgItems; ++u) {
    const uint32_t i = i0 + u * kArgThreads;
    if (i < n) {
      const unsigned long long pk = argmax_pack(v[u], i);
      best = pk > best ? pk : best;
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const unsigned long long q = __shfl_xor_sync(0xffffffffu, best, o);
    best = q > best ? q : best;
  }
  if ((threadIdx.x & 31) == 0 && best) atomicMax(&argmax[r], best);
}
}  // namespace

cudaError_t logits_argmax_launch(const float* logits, uint32_t rows, uint32_t n, uint32_t stride,
                                 unsigned long long* argmax, cudaStream_t st) {
  if (rows == 0 || n == 0) return cudaErrorInvalidValue;
  const dim3 grid((n + kArgThreads * kArgItems - 1) / (kArgThreads * kArgItems), rows);
  logits_argmax_kernel<<<grid, kArgThreads, 0, st>>>(logits, n, stride, argmax);
  return cudaGetLastError();
}

}  // namespace nnz
