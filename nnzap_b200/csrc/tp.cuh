// Tensor parallelism for batched decode: NCCL, loaded at run time.
//
// The library does not link NCCL: the first use dlopen()s libnccl.so.2
// (already resident when the host process imported torch; else found on
// the loader path or through NNZ_NCCL_LIB) and resolves the five entry
// points below.  Every rank of a tensor-parallel group is one process
// driving one GPU.
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <nccl.h>

#include <string>

namespace nnz {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*);
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int);
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t, cudaStream_t);
  ncclResult_t (*comm_destroy)(ncclComm_t);
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t);
  const char* (*error_string)(ncclResult_t);
};

// nullptr (and *err set) when NCCL cannot be loaded.
const NcclApi* nccl_api(std::string* err);

// argmax slots hold (key << 32) | (0xFFFFFFFF - local index); shift them to
// global vocabulary indices by subtracting `offset` (0 slots stay 0).
cudaError_t argmax_shift_launch(unsigned long long* argmax, uint32_t rows, uint32_t offset, cudaStream_t st);

// Group barrier over peer memory (one CTA): flags[0..T) are this GPU's
// arrival slots, flags[T] its own barrier count; peer_flags[j] points at
// GPU j's flags (mapped into this process; entry `rank` is this GPU's
// own).  Each call bumps the count c, stores c into slot `rank` of every
// GPU with release semantics (system scope), then waits (bounded; on timeout
// sets ERR_SPIN_TIMEOUT in *err) until every slot of its own flags holds c.
// Sum all-reduce of one row-split projection over peer memory, fused with
// the residual update.  Each GPU holds its own partial in `part` (n floats,
// zero at rest) and a slot array slots[T][n] that peers write into; CTA c
// owns slice c of the n floats and, with no grid-wide synchronisation:
//   1. stores its slice of `part` into slot `rank` of every peer (16-byte
//      stores over NVLink), then fences at system scope;
//   2. raises its slice flag on every peer (release, system scope);
//   3. waits (bounded; on timeout sets ERR_SPIN_TIMEOUT) until every peer's
//      flag for the slice arrived;
//   4. residual += part + the peers' slots, and re-zeroes its slice of part.
// peer_slots[j] / peer_flags[j]: GPU j's slot array / flag array mapped
// into this process (entry `rank` = this GPU's own).  Flags are
// [nslice][T + 1] u32: arrival counts per source, then this GPU's own call
// count for the slice.
// spin_limit: polls of a peer flag before giving up (0 = the library default).
// Optional fused RMSNorm (norm_w non-null; needs n = rows x 2048, i.e. one
// slice per residual row): the CTA also writes xn[row] = fp16(RMSNorm(new
// residual row) * norm_w) (BF16-truncated first when bf16r), the next
// GEMM's input.  pdl: launched with programmatic dependent launch.
cudaError_t tp_allreduce_launch(float* residual, float* part, float* const* peer_slots,
                                uint32_t* flags, uint32_t* const* peer_flags, size_t n, int rank, int T,
                                int* err, cudaStream_t st, uint32_t spin_limit = 0,
                                const float* norm_w = nullptr, float eps = 0.f, __half* xn = nullptr,
                                int bf16r = 0, int pdl = 0);
// Residual row length the fused RMSNorm of tp_allreduce_launch handles.
constexpr uint32_t kTpNormRow = 2048;
// Flag words tp_allreduce_launch needs for n floats at T ranks.
size_t tp_allreduce_flag_words(size_t n_max, int T);

}  // namespace nnz
