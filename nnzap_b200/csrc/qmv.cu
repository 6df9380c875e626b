// Host launcher and template instances for the quantized matvec kernel.
#include <cuda_runtime.h>

#include "qmv.cuh"

namespace nnz {

namespace {

constexpr uint32_t kXfCapBytes = 96 * 1024;   // x staging + B-fragment smem cap per CTA

// When set, launch_t only raises the instance's dynamic shared memory limit
// (done once per device, outside any stream capture).
thread_local bool g_prepare = false;

template <int FMT, int NT, int SUB, int PRO, int EPI, bool BF16S>
cudaError_t launch_t(QmvArgs a, dim3 grid, uint32_t smem, int pdl, cudaStream_t st) {
  auto* fn = &qmv_kernel<FMT, NT, SUB, PRO, EPI, BF16S>;
  if (g_prepare) return cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(kQmvThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fn, a);
}

template <int FMT, int NT, int SUB, int PRO, int EPI>
cudaError_t pick_bf16(const QmvLaunch& L, QmvArgs a, dim3 g, uint32_t sm, cudaStream_t st) {
  if constexpr (FMT == FMT_Q4) {
    if (L.bf16_scales) return launch_t<FMT, NT, SUB, PRO, EPI, true>(a, g, sm, L.pdl, st);
  }
  return launch_t<FMT, NT, SUB, PRO, EPI, false>(a, g, sm, L.pdl, st);
}

template <int FMT, int NT>
cudaError_t pick_variant(const QmvLaunch& L, QmvArgs a, dim3 g, uint32_t sm, cudaStream_t st) {
  if (L.sub == 2) {
    if (L.epi != EPI_SILU) return cudaErrorInvalidValue;
    if (L.pro == PRO_NORM) return pick_bf16<FMT, NT, 2, PRO_NORM, EPI_SILU>(L, a, g, sm, st);
    return pick_bf16<FMT, NT, 2, PRO_F16, EPI_SILU>(L, a, g, sm, st);
  }
  if (L.sub != 1) return cudaErrorInvalidValue;
  if (L.pro == PRO_NORM) {
    switch (L.epi) {
      case EPI_F16: return pick_bf16<FMT, NT, 1, PRO_NORM, EPI_F16>(L, a, g, sm, st);
      case EPI_F32: return pick_bf16<FMT, NT, 1, PRO_NORM, EPI_F32>(L, a, g, sm, st);
      case EPI_LOGITS: return pick_bf16<FMT, NT, 1, PRO_NORM, EPI_LOGITS>(L, a, g, sm, st);
      default: return cudaErrorInvalidValue;
    }
  }
  switch (L.epi) {
    case EPI_F16: return pick_bf16<FMT, NT, 1, PRO_F16, EPI_F16>(L, a, g, sm, st);
    case EPI_F32: return pick_bf16<FMT, NT, 1, PRO_F16, EPI_F32>(L, a, g, sm, st);
    case EPI_RESADD: return pick_bf16<FMT, NT, 1, PRO_F16, EPI_RESADD>(L, a, g, sm, st);
    case EPI_LOGITS: return pick_bf16<FMT, NT, 1, PRO_F16, EPI_LOGITS>(L, a, g, sm, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace

cudaError_t qmv_prepare() {
  g_prepare = true;
  cudaError_t err = cudaSuccess;
  QmvArgs a{};
  const dim3 g(1);
  for (int fmt = 0; fmt < 2; ++fmt)
    for (int bf = 0; bf < 2; ++bf)
      for (int sub = 1; sub <= 2; ++sub)
        for (int pro = 0; pro < 2; ++pro)
          for (int epi = 0; epi < 5; ++epi) {
            QmvLaunch L{fmt, sub, pro, epi, bf, 0};
            cudaError_t e1, e2;
            if (fmt == FMT_Q1) {
              e1 = pick_variant<FMT_Q1, 1>(L, a, g, 0, nullptr);
              e2 = pick_variant<FMT_Q1, 2>(L, a, g, 0, nullptr);
            } else {
              e1 = pick_variant<FMT_Q4, 1>(L, a, g, 0, nullptr);
              e2 = pick_variant<FMT_Q4, 2>(L, a, g, 0, nullptr);
            }
            if (e1 != cudaSuccess && e1 != cudaErrorInvalidValue) err = e1;
            if (e2 != cudaSuccess && e2 != cudaErrorInvalidValue) err = e2;
          }
  g_prepare = false;
  return err;
}

uint32_t qmv_pick_ksplit(uint32_t M, uint32_t K, uint32_t gs, int fmt, int sub, uint32_t batch,
                         int num_sms) {
  const uint32_t tiles = num_tiles(M);
  const uint32_t ych = (batch + kBatchChunk - 1) / kBatchChunk;
  const uint32_t groups = K / gs;
  const uint32_t nt = batch > 4 ? 2 : 1;
  const uint32_t target = 2u * (uint32_t)num_sms;
  uint32_t ks = (target + tiles * ych - 1) / (tiles * ych);
  if (ks < 1) ks = 1;
  uint32_t max_ks = groups / kQmvWarps;       // >= one group per warp
  if (max_ks < 1) max_ks = 1;
  if (ks > max_ks) ks = max_ks;
  // the CTA's x fragments must fit the smem cap
  const uint32_t rows = batch < (uint32_t)kBatchChunk ? batch : kBatchChunk;
  while (ks < groups && ((groups + ks - 1) / ks) * gs * (8 * nt + 2 * rows) > kXfCapBytes) ++ks;
  (void)fmt; (void)sub;
  return ks;
}

size_t qmv_ws_floats(uint32_t M, uint32_t K, uint32_t gs, int fmt, int sub, uint32_t batch,
                     int num_sms) {
  const uint32_t ks = qmv_pick_ksplit(M, K, gs, fmt, sub, batch, num_sms);
  if (ks <= 1) return 0;
  const uint32_t ych = (batch + kBatchChunk - 1) / kBatchChunk;
  return (size_t)ych * num_tiles(M) * ks * kTileRows * sub * kBatchChunk;
}

cudaError_t qmv_launch(const QmvLaunch& L, QmvArgs a, int num_sms, cudaStream_t st) {
  if (a.gs % kChunk || a.gs > 256 || a.K % a.gs || a.K % 4 || a.batch == 0 || a.M == 0)
    return cudaErrorInvalidValue;
  a.tiles = num_tiles(a.M);
  a.groups = a.K / a.gs;
  if (a.ksplit == 0) a.ksplit = qmv_pick_ksplit(a.M, a.K, a.gs, L.fmt, L.sub, a.batch, num_sms);
  if (a.ksplit > a.groups) return cudaErrorInvalidValue;
  const int nt = a.batch > 4 ? 2 : 1;
  const uint32_t ng_max = (a.groups + a.ksplit - 1) / a.ksplit;
  const QmvSmem S = qmv_smem_layout(L.fmt, nt, L.sub, a.gs, ng_max, a.batch < (uint32_t)kBatchChunk ? a.batch : kBatchChunk);
  // vector loads of x: 16-byte aligned rows
  const uintptr_t xa = reinterpret_cast<uintptr_t>(a.x);
  if (xa % 16 || (L.pro == PRO_NORM ? a.x_stride % 4 : a.x_stride % 8) ||
      (L.pro == PRO_NORM && reinterpret_cast<uintptr_t>(a.norm_w) % 16))
    return cudaErrorMisalignedAddress;
  if (S.total > 227 * 1024) return cudaErrorInvalidValue;
  const uint32_t ych = (a.batch + kBatchChunk - 1) / kBatchChunk;
  // persistent CTAs: about two resident CTAs per SM over all splits/chunks
  if (a.P == 0) {
    const uint32_t want = (2u * (uint32_t)num_sms + a.ksplit * ych - 1) / (a.ksplit * ych);
    a.P = want < a.tiles ? (want ? want : 1) : a.tiles;
  }
  dim3 grid(a.P * a.ksplit, ych);
  if (L.fmt == FMT_Q1) {
    return nt == 1 ? pick_variant<FMT_Q1, 1>(L, a, grid, S.total, st)
                   : pick_variant<FMT_Q1, 2>(L, a, grid, S.total, st);
  }
  return nt == 1 ? pick_variant<FMT_Q4, 1>(L, a, grid, S.total, st)
                 : pick_variant<FMT_Q4, 2>(L, a, grid, S.total, st);
}

}  // namespace nnz
