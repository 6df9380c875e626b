// Batch-1 quantized matvec for the tile-packed layout (packing.h): the fast
// path of nnz_qmv for one activation row (BASELINE configuration 0 and every
// single-row call).
//
// Replaces the single-token QMV shaders of the reference
// (nnmetal/src/shaders/q4mv_bf16_specialized.metal:93-180,
//  nnmetal/src/shaders/qmv_specialized.metal:55-205).
//
// One thread-block cluster of `ks` CTAs per 128-row tile; CTA r of the
// cluster owns the scale groups [r G / ks, (r + 1) G / ks) of that tile.
//  * Thread 0 issues ONE bulk copy (TMA engine, no multicast) of the CTA's
//    contiguous run of tile segments before anything else, so the weight
//    bytes stream while the CTA stages and quantizes its slice of x.
//  * Each of the 4 warps runs the int8 tensor-core group routine of the
//    tile-packed layout (qmv_group, qmv_dev.cuh) on groups w, w + 4, ...;
//    the warps' row sums meet in shared memory.
//  * The ks partial tiles are summed through distributed shared memory
//    (cluster rank 0 reads its peers' tiles after a cluster barrier): no
//    global workspace, no atomics, no second kernel.
#include <cooperative_groups.h>
#include <cuda_runtime.h>
#include <stdlib.h>

#include "qmv.cuh"
#include "qmvf.cuh"

namespace cg = cooperative_groups;

namespace nnz {

namespace {

constexpr uint32_t kQfMaxSmem = 200 * 1024;
constexpr uint32_t kQfSpin = 1u << 22;

struct QfLayout {
  uint32_t w, xs, xf, gsx, gsum, gsq, red, yt, bar, total, ngmax;
};

__host__ __device__ inline QfLayout qf_layout(int fmt, uint32_t K, uint32_t gs, uint32_t ks) {
  QfLayout L{};
  const uint32_t groups = K / gs, ng = (groups + ks - 1) / ks, seg = seg_bytes(fmt, gs), cpg = gs / kChunk;
  L.ngmax = ng;
  uint32_t o = 0;
  L.w = o; o += ng * seg;
  o = (o + 127) & ~127u;
  L.xs = o; o += ((ng * gs * 2) + 15) & ~15u;
  L.xf = o; o += ng * cpg * 256;
  L.gsx = o; o += ng * kBatchChunk * 4;
  L.gsum = o; o += ng * kBatchChunk * 4;
  L.gsq = o; o += ng * kBatchChunk * 4;
  L.red = o; o += kQmvWarps * kTileRows * 4;
  L.yt = o; o += 16 * kTileRows * 4;     // [cluster rank][128] partial tiles (leader's copy)
  L.bar = o; o += 16;                     // weights landed, peers' partials landed
  L.total = o;
  return L;
}

template <int FMT, bool BF16S>
__global__ void __launch_bounds__(kQmvThreads) qmvf_kernel(QmvfArgs a) {
  extern __shared__ __align__(128) uint8_t sm[];
  cg::cluster_group cl = cg::this_cluster();
  const uint32_t ks = a.ks, rank = cl.block_rank();
  const uint32_t tile = blockIdx.x / ks;
  const uint32_t groups = a.K / a.gs, cpg = a.gs / kChunk, seg = seg_bytes(FMT, a.gs);
  const uint32_t g0 = groups * rank / ks, ng = groups * (rank + 1) / ks - g0;
  const QfLayout L = qf_layout(FMT, a.K, a.gs, ks);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L.bar);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    mbar_init(bar + 1, (ks - 1) * kQmvThreads);
    fence_barrier_init();
    const uint32_t bytes = ng * seg;
    mbar_arrive_expect_tx(bar, bytes);
    if (bytes) bulk_g2s(sm + L.w, a.w + ((size_t)tile * groups + g0) * seg, bytes, bar);
  }
  // the leader's "partials" barrier must be initialised before any peer
  // arrives on it: arrive on the cluster barrier now (release), wait on it
  // only before the partial tiles are exchanged, so its latency overlaps
  // the staging and the MMAs
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  // programmatic dependent launch: the weights are constant, so their copy
  // above may overlap the previous kernel; x (and the output) may not
  pdl_wait();
  pdl_launch();
  // x slice -> fp16 staging -> int8 B fragments (overlaps the weight copy)
  __half* xs = reinterpret_cast<__half*>(sm + L.xs);
  uint8_t* xf = sm + L.xf;
  float* gsx = reinterpret_cast<float*>(sm + L.gsx);
  float* gsum = reinterpret_cast<float*>(sm + L.gsum);
  int* gsq = reinterpret_cast<int*>(sm + L.gsq);
  stage_f16(a.x, a.K, g0 * a.gs, ng * a.gs, 1, xs);
  quantize_xs<1>(xs, ng * a.gs, 1, ng, a.gs, xf, gsx, gsum, gsq);
  // weights landed (bounded wait; every thread polls the barrier)
  bool ok = false;
  for (uint32_t i = 0; i < kQfSpin && !ok; ++i) ok = mbar_try_wait(bar, 0);
  if (!ok && threadIdx.x == 0) atomicOr(a.err, ERR_MBAR_TIMEOUT);
  float y[1][1][16];
#pragma unroll
  for (int v = 0; v < 16; ++v) y[0][0][v] = 0.f;
  if (ok)
    for (uint32_t gl = warp; gl < ng; gl += kQmvWarps)
      qmv_group<FMT, 1, 1, BF16S>(sm + L.w + (size_t)gl * seg, seg, xf, gl, cpg, gsx, gsum, gsq, y);
  float* red = reinterpret_cast<float*>(sm + L.red);
  if ((lane & 3) == 0) {   // batch column 0 lives in lanes 4g
#pragma unroll
    for (int v = 0; v < 16; ++v) red[warp * kTileRows + y_row<FMT>(v, lane >> 2)] = y[0][0][v];
  }
  __syncthreads();
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
  float* yt = reinterpret_cast<float*>(sm + L.yt);
  const uint32_t r = threadIdx.x;   // kQmvThreads == kTileRows
  float part = 0.f;
#pragma unroll
  for (int w = 0; w < kQmvWarps; ++w) part += red[w * kTileRows + r];
  if (rank != 0) {
    // push the partial tile into the leader's shared memory, then arrive
    // (release, cluster scope) on the leader's barrier
    float* dst = cl.map_shared_rank(yt, 0) + rank * kTileRows + r;
    *dst = part;
    uint64_t* rbar = cl.map_shared_rank(bar + 1, 0);
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];"
                 ::"r"((uint32_t)__cvta_generic_to_shared(rbar)) : "memory");
    return;
  }
  bool got = ks == 1;
  for (uint32_t i = 0; i < kQfSpin && !got; ++i) {
    uint32_t okw;
    asm volatile("{\n .reg .pred p;\n mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], 0;\n"
                 " selp.u32 %0, 1, 0, p;\n}\n" : "=r"(okw) : "r"(smem_u32(bar + 1)) : "memory");
    got = okw != 0;
  }
  if (!got && threadIdx.x == 0) atomicOr(a.err, ERR_MBAR_TIMEOUT);
  const uint32_t row = tile * kTileRows + r;
  float v = part;
  for (uint32_t q = 1; q < ks; ++q) v += yt[q * kTileRows + r];
  if (row < a.M) {
    if (a.bf16_round) v = bf16_trunc(v);
    if (a.epi == EPI_F16) static_cast<__half*>(a.out)[row] = __float2half_rn(v);
    else if (a.epi == EPI_F32) static_cast<float*>(a.out)[row] = v;
    else static_cast<float*>(a.out)[row] += v;
  }
}

template <int FMT, bool BF16S>
cudaError_t launch_t(const QmvfArgs& a, uint32_t grid, uint32_t smem, cudaStream_t st) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kQmvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = a.ks;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, qmvf_kernel<FMT, BF16S>, a);
}

}  // namespace

uint32_t qmvf_pick_ks(int fmt, uint32_t M, uint32_t K, uint32_t gs, int num_sms) {
  const uint32_t tiles = num_tiles(M), groups = K / gs;
  // about 4 CTAs per SM (measured on config 0: 1 per SM 4.95 us, 2: 4.38,
  // 3-4 (cluster size capped at 8): 3.65); NNZ_QMVF_KS_MAX (8 or 16) is a
  // measurement aid for non-portable cluster sizes
  static const uint32_t ks_max = [] {
    const char* e = getenv("NNZ_QMVF_KS_MAX");
    return e && atoi(e) == 16 ? 16u : 8u;
  }();
  uint32_t ks = tiles >= 4u * (uint32_t)num_sms ? 1 : 4u * (uint32_t)num_sms / tiles;
  ks = ks > ks_max ? ks_max : ks;
  ks = ks > groups ? groups : ks;
  while (ks < groups && ks < ks_max && qf_layout(fmt, K, gs, ks).total > kQfMaxSmem) ++ks;
  return ks ? ks : 1;
}

bool qmvf_applies(int fmt, uint32_t M, uint32_t K, uint32_t gs, uint32_t batch, int epi, int num_sms) {
  if (batch != 1 || M == 0 || gs % kChunk || gs > 256 || K % gs || K % 8 ||
      (epi != EPI_F16 && epi != EPI_F32 && epi != EPI_RESADD))
    return false;
  (void)fmt;
  return qf_layout(fmt, K, gs, qmvf_pick_ks(fmt, M, K, gs, num_sms)).total <= kQfMaxSmem;
}

cudaError_t qmvf_prepare() {
  cudaError_t e = cudaSuccess;
  auto raise = [&](const void* f) {
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kQfMaxSmem);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(f, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
  };
  raise((const void*)qmvf_kernel<FMT_Q1, false>);
  raise((const void*)qmvf_kernel<FMT_Q4, false>);
  raise((const void*)qmvf_kernel<FMT_Q4, true>);
  return e;
}

cudaError_t qmvf_launch(int fmt, bool bf16s, QmvfArgs a, int num_sms, cudaStream_t st) {
  a.ks = qmvf_pick_ks(fmt, a.M, a.K, a.gs, num_sms);
  const uint32_t smem = qf_layout(fmt, a.K, a.gs, a.ks).total;
  if (smem > kQfMaxSmem) return cudaErrorInvalidValue;
  const uint32_t grid = num_tiles(a.M) * a.ks;
  if (fmt == FMT_Q1) return launch_t<FMT_Q1, false>(a, grid, smem, st);
  return bf16s ? launch_t<FMT_Q4, true>(a, grid, smem, st) : launch_t<FMT_Q4, false>(a, grid, smem, st);
}

}  // namespace nnz
