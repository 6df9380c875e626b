// Tensor parallelism for batched decode: NCCL, loaded at run time.
//
// The library does not link NCCL: the first use dlopen()s libnccl.so.2
// (already resident when the host process imported torch; else found on
// the loader path or through NNZ_NCCL_LIB) and resolves the five entry
// points below.  Every rank of a tensor-parallel group is one process
// driving one GPU.
#pragma once
#include <cuda_runtime.h>
#include <nccl.h>

#include <string>

namespace nnz {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  const char* (*error_string)(ncclResult_t);
};

// nullptr (and *err set) when NCCL cannot be loaded.
const NcclApi* nccl_api(std::string* err);

// argmax slots hold (key << 32) | (0xFFFFFFFF - local index); shift them to
// global vocabulary indices by subtracting `offset` (0 slots stay 0).
cudaError_t argmax_shift_launch(unsigned long long* argmax, uint32_t rows, uint32_t offset, cudaStream_t st);

}  // namespace nnz
