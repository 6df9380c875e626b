// nnz_qmv_noalloc: the quantized matvec of nnz_qmv for callers that cannot
// allocate device memory.
//
// Who needs it: a host that must not call cudaMalloc once it is running --
// for example an engine that hands the whole device memory budget to its own
// pool at start-up, or code that issues work while another thread of the
// process is capturing a CUDA graph (an allocation there invalidates the
// capture).  nnz_qmv takes its split-K scratch from a per-device workspace it
// allocates on first use; this variant instead uses fixed scratch compiled
// into the library as file-scope device arrays, so it never allocates.
//
// Costs and rules:
//  * every GPU that loads the library holds the arrays (8 MiB of partial
//    sums + 64 KiB of counters) until the process exits;
//  * problems whose split-K partials do not fit are rejected with NNZ_EINVAL;
//  * all calls share the arrays, so calls that overlap on the GPU (different
//    streams, or different host threads on one device) race -- serialise
//    them on one stream;
//  * the first call on a device resolves the arrays' device addresses,
//    clears the error word and raises the kernels' shared-memory limit:
//    make that first call before any stream capture starts on the device;
//  * a bounded wait that gives up inside the kernel sets the error word;
//    nnz_stream_check() reads and clears it (the call itself returns as
//    soon as the work is queued).
#include <cuda_runtime.h>

#include <mutex>
#include <new>
#include <string>

#include "../../include/nnz_b200.h"
#include "qmv.cuh"

namespace nnz {
void set_last_error(const std::string& msg);   // nnz_last_error() text (engine.cu)

namespace {

constexpr size_t kNoAllocWsFloats = (size_t)1 << 21;      // 8 MiB of split-K partials
constexpr size_t kNoAllocCounters = (size_t)1 << 14;      // per-tile arrival counters

static __device__ __align__(256) float g_noalloc_ws[kNoAllocWsFloats];
static __device__ __align__(256) uint32_t g_noalloc_counters[kNoAllocCounters];
static __device__ __align__(256) int g_noalloc_err[4];

struct NoAllocDev {
  bool ready = false;
  float* ws = nullptr;
  uint32_t* counters = nullptr;
  int* err = nullptr;
  int num_sms = 0;
};

constexpr int kMaxDevices = 64;
std::mutex g_mu;
NoAllocDev g_dev[kMaxDevices];


// Set-up for the current device: the arrays' device addresses (the symbols
// themselves are host-side stand-ins and must never be passed to a kernel)
// and the kernels' dynamic shared-memory limit.  No allocation.
int setup(int dev, NoAllocDev** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  NoAllocDev& d = g_dev[dev];
  if (!d.ready) {
    cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.ws), g_noalloc_ws);
    if (e == cudaSuccess)
      e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.counters), g_noalloc_counters);
    if (e == cudaSuccess) e = cudaGetSymbolAddress(reinterpret_cast<void**>(&d.err), g_noalloc_err);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaMemset(d.err, 0, sizeof(int));
    if (e == cudaSuccess) e = qmv_prepare();
    if (e != cudaSuccess) {
      set_last_error(std::string("nnz_qmv_noalloc set-up: ") + cudaGetErrorString(e));
      return NNZ_ECUDA;
    }
    d.ready = true;
  }
  *out = &d;
  return NNZ_OK;
}

}  // namespace

// Device error flags raised by no-alloc launches on device `dev` since the
// last call (read with a copy from the symbol, cleared; no allocation).
int noalloc_take_error(int dev, int* flags) {
  *flags = 0;
  if (dev < 0 || dev >= kMaxDevices) return NNZ_OK;
  int* p = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_dev[dev].ready) return NNZ_OK;
    p = g_dev[dev].err;
  }
  if (cudaMemcpy(flags, p, sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess ||
      (*flags && cudaMemset(p, 0, sizeof(int)) != cudaSuccess)) {
    set_last_error(std::string("nnz_stream_check: ") + cudaGetErrorString(cudaGetLastError()));
    return NNZ_ECUDA;
  }
  return NNZ_OK;
}
}  // namespace nnz

using namespace nnz;

static int qmv_noalloc_impl(int fmt, int scale_dtype, int bf16_round, const void* packed,
                               uint32_t M, uint32_t K, uint32_t gs, const void* x,
                               uint32_t x_stride, uint32_t batch, void* out, uint32_t out_stride,
                               int out_kind, void* stream) {
  const int epi = out_kind == NNZ_OUT_F16 ? EPI_F16
                : out_kind == NNZ_OUT_F32 ? EPI_F32
                : out_kind == NNZ_OUT_F32_ADD ? EPI_RESADD : -1;
  if (!packed || !x || !out || epi < 0 || (fmt != NNZ_Q1 && fmt != NNZ_Q4) || batch == 0 || M == 0 ||
      gs == 0 || gs % 32 || gs > 256 || K % gs) {
    set_last_error("nnz_qmv_noalloc: invalid arguments");
    return NNZ_EINVAL;
  }
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    cudaGetLastError();
    set_last_error("nnz_qmv_noalloc: no usable current device");
    return NNZ_ECUDA;
  }
  NoAllocDev* d;
  int rc = setup(dev, &d);
  if (rc) return rc;
  const size_t need_ws = qmv_ws_floats(M, K, gs, fmt, 1, batch, d->num_sms);
  const size_t need_ctr = (size_t)((batch + kBatchChunk - 1) / kBatchChunk) * num_tiles(M);
  if (need_ws > kNoAllocWsFloats || need_ctr > kNoAllocCounters) {
    set_last_error("nnz_qmv_noalloc: problem needs " + std::to_string(need_ws * 4) +
                   " B of split-K scratch and " + std::to_string(need_ctr) +
                   " counters; the fixed limits are " + std::to_string(kNoAllocWsFloats * 4) + " B and " +
                   std::to_string(kNoAllocCounters));
    return NNZ_EINVAL;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // the counters must start at zero (the error word accumulates until
  // nnz_stream_check clears it); the partial sums are fully overwritten
  // before they are read
  cudaError_t e = cudaMemsetAsync(d->counters, 0, need_ctr * sizeof(uint32_t), st);
  if (e == cudaSuccess) {
    QmvLaunch L{fmt, 1, PRO_F16, epi, fmt == NNZ_Q4 && scale_dtype == NNZ_SCALE_BF16, 0};
    QmvArgs a{};
    a.w = static_cast<const uint8_t*>(packed); a.M = M; a.K = K; a.gs = gs;
    a.x = x; a.x_stride = x_stride ? x_stride : K; a.batch = batch;
    a.out = out; a.out_stride = out_stride ? out_stride : M;
    a.ws = d->ws; a.counters = d->counters; a.err = d->err;
    a.bf16_round = (fmt == NNZ_Q4 && bf16_round) ? 1u : 0u;
    e = qmv_launch(L, a, d->num_sms, st);
  }
  if (e != cudaSuccess) {
    set_last_error(std::string("nnz_qmv_noalloc: ") + cudaGetErrorString(e));
    return NNZ_ECUDA;
  }
  return NNZ_OK;
}

// No C++ exception crosses the C ABI: the error-message building above can
// throw std::bad_alloc and the set-up mutex std::system_error.
extern "C" int nnz_qmv_noalloc(int fmt, int scale_dtype, int bf16_round, const void* packed,
                               uint32_t M, uint32_t K, uint32_t gs, const void* x,
                               uint32_t x_stride, uint32_t batch, void* out, uint32_t out_stride,
                               int out_kind, void* stream) {
  try {
    return qmv_noalloc_impl(fmt, scale_dtype, bf16_round, packed, M, K, gs, x, x_stride, batch, out,
                            out_stride, out_kind, stream);
  } catch (const std::bad_alloc&) {
    return NNZ_ENOMEM;
  } catch (...) {
    return NNZ_EINVAL;
  }
}
