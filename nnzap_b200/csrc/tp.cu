// NCCL loader and the small kernels of the tensor-parallel decode path.
#include <dlfcn.h>
#include <stdlib.h>

#include <mutex>

#include "tp.cuh"

namespace nnz {

namespace {
std::once_flag g_once;
NcclApi g_api;
bool g_ok = false;
std::string g_err;

void load() {
  const char* cands[] = {getenv("NNZ_NCCL_LIB"), "libnccl.so.2", "libnccl.so"};
  void* h = nullptr;
  for (const char* c : cands) {
    if (!c) continue;
    h = dlopen(c, RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen(c, RTLD_NOW | RTLD_GLOBAL);
    if (h) break;
  }
  if (!h) {
    g_err = "NCCL not found (libnccl.so.2; set NNZ_NCCL_LIB)";
    return;
  }
  g_api.get_unique_id = reinterpret_cast<decltype(g_api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
  g_api.comm_init_rank = reinterpret_cast<decltype(g_api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
  g_api.all_reduce = reinterpret_cast<decltype(g_api.all_reduce)>(dlsym(h, "ncclAllReduce"));
  g_api.comm_destroy = reinterpret_cast<decltype(g_api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
  g_api.error_string = reinterpret_cast<decltype(g_api.error_string)>(dlsym(h, "ncclGetErrorString"));
  if (!g_api.get_unique_id || !g_api.comm_init_rank || !g_api.all_reduce || !g_api.comm_destroy ||
      !g_api.error_string) {
    g_err = "NCCL library lacks an entry point";
    return;
  }
  g_ok = true;
}

__global__ void argmax_shift_kernel(unsigned long long* am, uint32_t rows, uint32_t off) {
  const uint32_t r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r < rows && am[r]) am[r] -= off;
}
}  // namespace

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
