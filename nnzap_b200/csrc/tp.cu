// NCCL loader and the small kernels of the tensor-parallel decode path.
#include <dlfcn.h>
#include <stdlib.h>

#include <mutex>

#include "tp.cuh"
#include "common.cuh"

namespace nnz {

namespace {
std::once_flag g_once;
NcclApi g_api;
bool g_ok = false;
std::string g_err;

// NNZ_NCCL_LIB, when set, is the only library tried (so a deployment can
// pin one, and a missing one is reported rather than silently replaced).
void load() {
  const char* pinned = getenv("NNZ_NCCL_LIB");
  const char* cands[] = {pinned, pinned ? nullptr : "libnccl.so.2", pinned ? nullptr : "libnccl.so"};
  void* h = nullptr;
  for (const char* c : cands) {
    if (!c) continue;
    h = dlopen(c, RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen(c, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
  }
  if (!h) {
    g_err = pinned ? std::string("NCCL not found at NNZ_NCCL_LIB=") + pinned
                   : std::string("NCCL not found (libnccl.so.2; set NNZ_NCCL_LIB)");
    return;
  }
  g_api.get_unique_id = reinterpret_cast<decltype(g_api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
  g_api.comm_init_rank = reinterpret_cast<decltype(g_api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
  g_api.all_reduce = reinterpret_cast<decltype(g_api.all_reduce)>(dlsym(h, "ncclAllReduce"));
  g_api.comm_destroy = reinterpret_cast<decltype(g_api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
  g_api.error_string = reinterpret_cast<decltype(g_api.error_string)>(dlsym(h, "ncclGetErrorString"));
  g_api.all_gather = reinterpret_cast<decltype(g_api.all_gather)>(dlsym(h, "ncclAllGather"));
  if (!g_api.get_unique_id || !g_api.comm_init_rank || !g_api.all_reduce || !g_api.comm_destroy ||
      !g_api.error_string || !g_api.all_gather) {
    g_err = "NCCL library lacks an entry point";
    return;
  }
  g_ok = true;
}

constexpr uint32_t kTpSpinLimit = 1u << 24;
constexpr int kArThreads = 256;
constexpr size_t kArSlice = kArThreads * 8;   // floats per CTA (two float4 per thread)

__global__ void __launch_bounds__(kArThreads) tp_allreduce_kernel(float* residual, float* part,
                                                                  float* const* peer_slots, uint32_t* flags,
                                                                  uint32_t* const* peer_flags, size_t n, int rank,
                                                                  int T, int* err, uint32_t spin_limit,
                                                                  const float* norm_w, float eps, __half* xn,
                                                                  int bf16r) {
  const size_t c = blockIdx.x, base = c * kArSlice;
  const size_t stride = (size_t)(T + 1);
  pdl_wait();
  pdl_launch();
  float4 v[2];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const size_t i = base + (size_t)(threadIdx.x + u * kArThreads) * 4;
    v[u] = i < n ? *reinterpret_cast<const float4*>(part + i) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
  // 1. this GPU's partial into slot `rank` of every peer
  for (int j = 0; j < T; ++j) {
    if (j == rank) continue;
    float* dst = peer_slots[j] + (size_t)rank * n;
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const size_t i = base + (size_t)(threadIdx.x + u * kArThreads) * 4;
      if (i < n) *reinterpret_cast<float4*>(dst + i) = v[u];
    }
  }
  __threadfence_system();
  __syncthreads();
  // 2. raise this slice's flag on every peer, 3. wait for theirs
  if (threadIdx.x == 0) {
    const uint32_t cnt = flags[c * stride + T] + 1;
    flags[c * stride + T] = cnt;
    for (int j = 0; j < T; ++j)
      if (j != rank)
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(peer_flags[j] + c * stride + rank), "r"(cnt)
                     : "memory");
    for (int j = 0; j < T; ++j) {
      if (j == rank) continue;
      uint32_t f, it = 0;
      for (;;) {
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flags + c * stride + j) : "memory");
        if ((int)(f - cnt) >= 0) break;
        if (++it > spin_limit) {
          atomicOr(err, ERR_SPIN_TIMEOUT);
          break;
        }
        __nanosleep(32);
      }
    }
  }
  __syncthreads();
  // 4. fold: residual += own partial + peers' partials; re-zero the partial
  float* slots = peer_slots[rank];
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const size_t i = base + (size_t)(threadIdx.x + u * kArThreads) * 4;
    if (i >= n) continue;
    float4 acc = v[u];
    for (int j = 0; j < T; ++j) {
      if (j == rank) continue;
      const float4 w = __ldcg(reinterpret_cast<const float4*>(slots + (size_t)j * n + i));
      acc.x += w.x; acc.y += w.y; acc.z += w.z; acc.w += w.w;
    }
    float4 r = *reinterpret_cast<float4*>(residual + i);
    r.x += acc.x; r.y += acc.y; r.z += acc.z; r.w += acc.w;
    *reinterpret_cast<float4*>(residual + i) = r;
    *reinterpret_cast<float4*>(part + i) = make_float4(0.f, 0.f, 0.f, 0.f);
    v[u] = r;
  }
  if (!norm_w) return;
  // 5. fused RMSNorm of the new residual row (slice c = row c, fully inside n)
  __shared__ float red[kArThreads / 32];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < 2; ++u) ss += v[u].x * v[u].x + v[u].y * v[u].y + v[u].z * v[u].z + v[u].w * v[u].w;
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  float t = 0.f;
#pragma unroll
  for (int w = 0; w < kArThreads / 32; ++w) t += red[w];
  const float rs = rsqrtf(t / (float)kArSlice + eps);
#pragma unroll
  for (int u = 0; u < 2; ++u) {
    const uint32_t k = (threadIdx.x + u * kArThreads) * 4;
    const float4 g = *reinterpret_cast<const float4*>(norm_w + k);
    float o[4] = {v[u].x * rs * g.x, v[u].y * rs * g.y, v[u].z * rs * g.z, v[u].w * rs * g.w};
    if (bf16r)
      for (int e = 0; e < 4; ++e) o[e] = bf16_trunc(o[e]);
    __half2* dst = reinterpret_cast<__half2*>(xn + base + k);
    dst[0] = __floats2half2_rn(o[0], o[1]);
    dst[1] = __floats2half2_rn(o[2], o[3]);
  }
}

__global__ void argmax_shift_kernel(unsigned long long* am, uint32_t rows, uint32_t off) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows && am[r]) am[r] -= off;
}
}  // namespace

size_t tp_allreduce_flag_words(size_t n_max, int T) {
  return ((n_max + kArSlice - 1) / kArSlice) * (size_t)(T + 1);
}

cudaError_t tp_allreduce_launch(float* residual, float* part, float* const* peer_slots, uint32_t* flags,
                                uint32_t* const* peer_flags, size_t n, int rank, int T, int* err,
                                cudaStream_t st, uint32_t spin_limit, const float* norm_w, float eps, __half* xn,
                                int bf16r, int pdl) {
  static_assert(kArSlice == kTpNormRow, "fused RMSNorm: one slice per residual row");
  if (n % 4 || (norm_w && (n % kArSlice || !xn))) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((n + kArSlice - 1) / kArSlice);
  cudaLaunchAttribute at[1];
  at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  at[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kArThreads);
  cfg.stream = st;
  cfg.attrs = at;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, &tp_allreduce_kernel, residual, part, peer_slots, flags, peer_flags, n, rank, T,
                            err, spin_limit ? spin_limit : kTpSpinLimit, norm_w, eps, xn, bf16r);
}

const NcclApi* nccl_api(std::string* err) {
  std::call_once(g_once, load);
  if (!g_ok) {
    if (err) *err = g_err;
    return nullptr;
  }
  return &g_api;
}

cudaError_t argmax_shift_launch(unsigned long long* argmax, uint32_t rows, uint32_t offset, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  argmax_shift_kernel<<<(rows + 127) / 128, 128, 0, st>>>(argmax, rows, offset);
  return cudaGetLastError();
}

}  // namespace nnz
