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

// cos/sin of the rotary angle pos * theta^(-2i/HD) of pair i, evaluated in
// double and rounded to f32; `tab` (optional) holds the same values
// precomputed on the host for this position.
template <int HD>
__device__ __forceinline__ float2 rope_cs(const float2* tab, double l2t, int pos, int i) {
  if (tab) return __ldg(tab + i);
  const double ang = (double)pos * exp2(-(2.0 * i / HD) * l2t);
  double sd, cd;
  sincos(ang, &sd, &cd);
  return make_float2((float)cd, (float)sd);
}

// One warp: RMSNorm over the head (f32), scale, RoPE.  Leaves the EPL
// values this lane owns in v[] (pairwise: contiguous elements; half-split:
// element i pairs with i + HD/2, which lane + 16 owns).  `tab`, when given,
// holds the HD/2 (cos, sin) pairs of position `pos`.
template <int HD, typename T>
__device__ __forceinline__ void norm_rope_head(const T* src, const float* nw, float eps,
                                               float theta, int style, int pos, int lane,
                                               float (&v)[HD / 32], const float2* tab = nullptr) {
  constexpr int EPL = HD / 32;
  float2 cs[EPL];
  const double l2t = tab ? 0.0 : log2((double)theta);
  if (tab) {   // table loads first: they overlap the head's own load
#pragma unroll
    for (int e = 0; e < EPL; ++e)
      if (style != ROPE_PAIRWISE || (e & 1) == 0)
        cs[e] = __ldg(tab + (style == ROPE_PAIRWISE ? (lane * EPL + e) >> 1 : (lane & 15) * EPL + e));
  }
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
  if (style == ROPE_PAIRWISE) {
#pragma unroll
    for (int e = 0; e < EPL; e += 2) {
      const int i = (lane * EPL + e) >> 1;
      const float2 q = tab ? cs[e] : rope_cs<HD>(nullptr, l2t, pos, i);
      const float c = q.x, s = q.y;
      const float x0 = v[e], x1 = v[e + 1];
      v[e] = x0 * c - x1 * s;
      v[e + 1] = x0 * s + x1 * c;
    }
  } else {
#pragma unroll
    for (int e = 0; e < EPL; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
      const int i = (lane & 15) * EPL + e;
      const float2 q = tab ? cs[e] : rope_cs<HD>(nullptr, l2t, pos, i);
      const float c = q.x, s = q.y;
      if (lane < 16) v[e] = v[e] * c - partner * s;   // first half: a*c - b*s
      else v[e] = partner * s + v[e] * c;             // second half: a*s + b*c
    }
  }
}


}  // namespace nnz
