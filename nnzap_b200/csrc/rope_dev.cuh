// Per-head RMSNorm + rotary embedding for one warp (shared by the decode
// attention kernel and the persistent decode kernel).
#pragma once
#include "common.cuh"

namespace nnz {

enum RopeStyle : int { ROPE_PAIRWISE = 0, ROPE_HALF_SPLIT = 1 };

// A q/k/v element as the engine stores it: fp16.  An f32 split-K
// accumulator is rounded to fp16 first, exactly like the QMV's fp16 output.
// (f32 sources are produced inside the same launch: read through L2.)
__device__ __forceinline__ float load_half_value(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ float load_half_value(const float* p) { return __half2float(__float2half_rn(__ldcg(p))); }

// One warp: RMSNorm over the head (f32), scale, RoPE.  Leaves the EPL
// values this lane owns in v[] (pairwise: contiguous elements; half-split:
// element i pairs with i + HD/2, which lane + 16 owns).
template <int HD, typename T>
__device__ __forceinline__ void norm_rope_head(const T* src, const float* nw, float eps,
                                               float theta, int style, int pos, int lane,
                                               float (&v)[HD / 32]) {
  constexpr int EPL = HD / 32;
  float ss = 0.f;
#pragma unroll
  for (int e = 0; e < EPL; ++e) {
    v[e] = load_half_value(src + lane * EPL + e);
    ss = fmaf(v[e], v[e], ss);
  }
  ss = warp_sum(ss);
  const float r = rsqrtf(ss / (float)HD + eps);
#pragma unroll
  for (int e = 0; e < EPL; ++e) v[e] = v[e] * r * nw[lane * EPL + e];
  const double l2t = log2((double)theta);
  if (style == ROPE_PAIRWISE) {
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      const int i = (lane * EPL + e) >> 1;
      const double ang = (double)pos * exp2(-(2.0 * i / HD) * l2t);
      double sd, cd;
      sincos(ang, &sd, &cd);
      const float c = (float)cd, s = (float)sd;
      const float x0 = v[e], x1 = v[e + 1];
      v[e] = x0 * c - x1 * s;
      v[e + 1] = x0 * s + x1 * c;
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
      const int i = (lane & 15) * EPL + e;
      const double ang = (double)pos * exp2(-(2.0 * i / HD) * l2t);
      double sd, cd;
      sincos(ang, &sd, &cd);
      const float c = (float)cd, s = (float)sd;
      if (lane < 16) v[e] = v[e] * c - partner * s;   // first half: a*c - b*s
      else v[e] = partner * s + v[e] * c;             // second half: a*s + b*c
    }
  }
}


}  // namespace nnz
