// Engine and C ABI (include/nnz_b200.h).
//
// Replaces the reference's Model(Config) buffers + loader (nnmetal/src/
// model.zig), the encode/dispatch layer (nnmetal/src/transformer.zig:
// 648-2388, 2452-2930) and the generate loop (:3942-4123).  One decode step
// is 1 + 5*L + 1 kernels (embed; per layer fused-norm QKV, fused attention,
// o-proj + residual, fused-norm gate/up + SiLU*mul, down + residual; fused
// final-norm LM head + argmax) captured once into a CUDA graph with
// programmatic dependent launch edges.  Token and position live in device
// memory and the embedding kernel advances them, so generate() replays the
// graph once per token with no host synchronisation in between.
#include <cuda_runtime.h>
#include <string.h>

#include <algorithm>
#include <cmath>
#include <exception>
#include <map>
#include <mutex>
#include <new>
#include <string>
#include <vector>

#include "../../include/nnz_b200.h"
#include "attn.cuh"
#include "decode1.cuh"
#include "gemm.cuh"
#include "mega.cuh"
#include "misc.cuh"
#include "packing.h"
#include "qmv.cuh"
#include "qmvf.cuh"
#include "tp.cuh"

using namespace nnz;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
  g_err = msg;
  return code;
}

#define NNZ_CK(x)                                                                       \
  do {                                                                                  \
    cudaError_t e_ = (x);                                                               \
    if (e_ != cudaSuccess) return fail(NNZ_ECUDA, std::string(#x) + ": " + cudaGetErrorString(e_)); \
  } while (0)

constexpr uint32_t kPrefillChunk = 64;        // chunked-matvec prefill
constexpr uint32_t kGemmPrefillChunk = 512;    // tcgen05 GEMM prefill
constexpr uint32_t kGemmDecodeRows = 16;       // decode batches from here on use the GEMM

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

float f16_to_f32_host(uint16_t h) {
  const uint32_t s = (h >> 15) & 1, e = (h >> 10) & 0x1F, m = h & 0x3FF;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) bits = s << 31;
    else {
      int ee = -1;
      uint32_t mm = m;
      do { ++ee; mm <<= 1; } while (!(mm & 0x400));
      bits = (s << 31) | ((uint32_t)(127 - 15 - ee) << 23) | ((mm & 0x3FF) << 13);
    }
  } else if (e == 31) bits = (s << 31) | 0x7F800000u | (m << 13);
  else bits = (s << 31) | ((e - 15 + 127) << 23) | (m << 13);
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t f32_to_f16_host(float f) {  // round to nearest even
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t exp = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
  uint32_t mant = x & 0x7FFFFFu;
  if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    const uint32_t shift = (uint32_t)(14 - exp);
    uint32_t hm = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1), half = 1u << (shift - 1);
    if (rem > half || (rem == half && (hm & 1))) ++hm;
    return (uint16_t)(sign | hm);
  }
  uint32_t hm = mant >> 13;
  const uint32_t rem = mant & 0x1FFFu;
  uint32_t he = (uint32_t)exp;
  if (rem > 0x1000u || (rem == 0x1000u && (hm & 1))) {
    ++hm;
    if (hm == 0x400u) { hm = 0; ++he; if (he >= 31) return (uint16_t)(sign | 0x7C00u); }
  }
  return (uint16_t)(sign | (he << 10) | hm);
}

struct HostTensor {
  int dtype;
  std::vector<uint8_t> data;
};

// Weights of one matrix in the reference's flat layout (prefill GEMM operand).
struct FlatW {
  const uint8_t* w = nullptr;
  const uint16_t* s = nullptr;
  const uint16_t* b = nullptr;
};

struct LayerW {
  FlatW fqkv, fo, fgate, fup, fdown;
  uint8_t *qkv, *o, *gu, *down;
  float *attn_norm, *ffn_norm, *q_norm, *k_norm;
};

// Per-device workspace for the standalone per-kernel entry points.
struct DevWs {
  float* ws = nullptr;
  size_t ws_floats = 0;
  uint32_t* counters = nullptr;
  size_t n_counters = 0;
  int* err = nullptr;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  int num_sms = 148;
};
std::mutex g_ws_mu;
std::map<int, DevWs> g_ws;
std::map<int, bool> g_prepared;

// Kernel attributes, once per device (never inside a stream capture).
int prepare_device(int dev) {
  static std::mutex mu;
  std::lock_guard<std::mutex> lk(mu);
  if (g_prepared[dev]) return NNZ_OK;
  NNZ_CK(qmv_prepare());
  NNZ_CK(qmvf_prepare());
  NNZ_CK(attn_prepare());
  g_prepared[dev] = true;
  return NNZ_OK;
}

int get_ws(DevWs** out) {
  int dev = 0;
  NNZ_CK(cudaGetDevice(&dev));
  int rc = prepare_device(dev);
  if (rc) return rc;
  std::lock_guard<std::mutex> lk(g_ws_mu);
  DevWs& w = g_ws[dev];
  if (!w.ws) {
    NNZ_CK(cudaDeviceGetAttribute(&w.num_sms, cudaDevAttrMultiProcessorCount, dev));
    w.ws_floats = (size_t)32 << 20;
    w.n_counters = (size_t)1 << 20;
    w.scratch_bytes = (size_t)64 << 20;
    NNZ_CK(cudaMalloc(&w.ws, w.ws_floats * 4));
    NNZ_CK(cudaMalloc(&w.counters, w.n_counters * 4));
    NNZ_CK(cudaMalloc(&w.err, 4));
    NNZ_CK(cudaMalloc(&w.scratch, w.scratch_bytes));
    NNZ_CK(cudaMemset(w.counters, 0, w.n_counters * 4));
    NNZ_CK(cudaMemset(w.err, 0, 4));
  }
  *out = &w;
  return NNZ_OK;
}

std::string err_text(int flags) {
  std::string s = "device error flags:";
  if (flags & ERR_MBAR_TIMEOUT) s += " bulk-copy wait timed out;";
  if (flags & ERR_BAD_TOKEN) s += " token id >= vocab;";
  if (flags & ERR_BAD_POS) s += " position >= max_context_length;";
  if (flags & ERR_SPIN_TIMEOUT) s += " spin wait timed out;";
  return s;
}

}  // namespace

namespace nnz {
int noalloc_take_error(int dev, int* flags);   // noalloc.cu
// Lets other translation units of the library set nnz_last_error()'s text.
void set_last_error(const std::string& msg) { g_err = msg; }
}  // namespace nnz

struct nnz_model {
  nnz_config c{};          // this rank's dims (heads / intermediate divided by tp)
  nnz_config full{};       // the model's dims as given
  int tp = 1, tp_rank = 0;
  ncclComm_t comm = nullptr;
  // fused GEMM + peer-memory all-reduce (decode / prefill GEMM path)
  bool tp_fused = false;
  // the last peer-memory reduction also wrote xn (the RMSNorm the next GEMM
  // needs), so the caller skips its own RMSNorm launch
  bool xn_from_tp = false;
  float* tp_racc = nullptr;            // [2][rows_max][H] f32 local partials, zero at rest
  float* tp_slots = nullptr;           // [2][tp][rows_max * H] f32 peers' partials
  int tp_parity = 0;                   // which half the next reduction uses
  uint32_t* tp_flags = nullptr;        // per-slice arrival counts (tp_allreduce_flag_words)
  float** d_peer_slots = nullptr;      // device [2][tp]: every GPU's slot arrays, mapped here
  uint32_t** d_peer_flags = nullptr;   // device [tp]: every GPU's flags, mapped here
  std::vector<void*> ipc_opened;
  uint32_t lm_rows = 0, lm_off = 0;   // this rank's LM-head vocabulary rows
  int device = 0;
  int num_sms = 148;
  cudaStream_t st = nullptr;
  std::map<std::string, HostTensor> host;
  bool finalized = false;
  int fmt = 0, bf16s = 0, bf16r = 0;
  uint32_t qd = 0, kvd = 0, qkv_rows = 0, slots = 0, rows_max = 0;
  uint8_t* arena = nullptr;
  size_t arena_bytes = 0;
  std::vector<LayerW> L;
  uint8_t* emb_w = nullptr;
  uint16_t *emb_s = nullptr, *emb_b = nullptr;
  uint8_t* lm = nullptr;
  float* fnorm = nullptr;
  __half *kc = nullptr, *vc = nullptr;
  size_t kv_layer = 0;  // elements per layer per cache
  float* residual = nullptr;
  __half* xn = nullptr;          // fp16 RMSNorm output [rows_max][max(H, ...)] (GEMM prefill)
  bool gemm_prefill = false;
  FlatW flm;                           // LM head in the reference layout (GEMM decode of large batches)
  float* gacc = nullptr;               // split-K accumulator of decode GEMMs (zero at rest)
  size_t gacc_floats = 0;
  uint8_t* flat = nullptr;       // flat weight copies for the GEMM prefill
  __half *qkv = nullptr, *attn = nullptr, *h = nullptr;
  float* logits = nullptr;
  float* ws = nullptr;
  size_t ws_floats = 0;
  uint32_t* counters = nullptr;
  size_t n_counters = 0;
  int* err = nullptr;
  DecodeState* state = nullptr;
  uint32_t* seq = nullptr;
  uint32_t* prompt = nullptr;
  float* uniforms = nullptr;           // [max_context] sampling draws of one generate call
  int* iota = nullptr;
  int* zeros = nullptr;
  size_t dev_bytes = 0;
  std::vector<void*> allocs;
  std::map<std::pair<uint32_t, int>, cudaGraphExec_t> graphs;
  // persistent decode kernel
  bool mega_ok = false;
  MegaLayer* mlayers = nullptr;
  float *mR = nullptr, *mqkv = nullptr, *mgu = nullptr, *matt = nullptr;
  unsigned int* mbar = nullptr;
  unsigned long long mbar_count = 0;
  unsigned int* mdep = nullptr;        // persistent kernel dataflow counters
  float2* rope_tab = nullptr;          // [max_ctx][head_dim / 2] (cos, sin)   // grid-barrier arrivals so far (device counter's value)
  unsigned long long* mprof = nullptr;    // NNZ_MEGA_PROFILE=1: per-phase timestamps
  struct MegaPlan { MegaArgs a; uint32_t grid, smem; bool ok; };
  std::map<uint32_t, MegaPlan> mplans;
  std::vector<cudaEvent_t> events;
  // single-row Q1 decode kernel (decode1.cu)
  bool d1_ok = false;
  D1Args d1{};
  unsigned long long d1_bar_count = 0;   // grid-barrier arrivals so far
  uint32_t d1_epoch = 0;                 // tokens decoded since the counters were cleared
  size_t d1_cnt_words = 0;
};

namespace {

int dalloc(nnz_model* m, void** p, size_t bytes) {
  if (cudaMalloc(p, bytes) != cudaSuccess) {
    cudaGetLastError();
    return fail(NNZ_ENOMEM, "cudaMalloc failed for " + std::to_string(bytes) + " bytes");
  }
  m->allocs.push_back(*p);
  m->dev_bytes += bytes;
  return NNZ_OK;
}

const HostTensor* find_t(nnz_model* m, const std::string& name) {
  auto it = m->host.find(name);
  return it == m->host.end() ? nullptr : &it->second;
}

// Fetch a quantized projection in the reference layout, converting scale
// encodings like the reference loader.  Returns weight bytes and u16 scales
// (+ biases for Q4) in this model's scale dtype.
int get_proj(nnz_model* m, const std::string& base, uint32_t M, uint32_t K,
             std::vector<uint8_t>& w, std::vector<uint16_t>& s, std::vector<uint16_t>& b) {
  const uint32_t gs = (uint32_t)m->c.group_size;
  const size_t wbytes = m->fmt == NNZ_Q1 ? (size_t)M * K / 8 : (size_t)M * K / 2;
  const size_t ng = (size_t)M * K / gs;
  const HostTensor* tw = find_t(m, base + ".weight");
  const HostTensor* ts = find_t(m, base + ".scales");
  if (!tw || !ts) return fail(NNZ_ENOTFOUND, "tensor not found: " + base + (tw ? ".scales" : ".weight"));
  if (tw->data.size() < wbytes) return fail(NNZ_EINVAL, base + ".weight too small");
  if (ts->data.size() < ng * 2) return fail(NNZ_EINVAL, base + ".scales too small");
  w.assign(tw->data.begin(), tw->data.begin() + wbytes);
  auto conv = [&](const HostTensor* t, std::vector<uint16_t>& out) -> int {
    out.resize(ng);
    const uint16_t* src = reinterpret_cast<const uint16_t*>(t->data.data());
    if (t->dtype != NNZ_DT_F16 && t->dtype != NNZ_DT_BF16)
      return fail(NNZ_EINVAL, base + ": scales/biases must be f16 or bf16");
    const bool want_bf16 = m->fmt == NNZ_Q4 && m->bf16s;
    for (size_t i = 0; i < ng; ++i) {
      const uint16_t r = src[i];
      if (t->dtype == NNZ_DT_F16 && want_bf16) {
        // raw BF16 = high half of the f32 (truncation, model.zig:1191-1205)
        const float f = f16_to_f32_host(r);
        uint32_t u;
        memcpy(&u, &f, 4);
        out[i] = (uint16_t)(u >> 16);
      } else if (t->dtype == NNZ_DT_BF16 && !want_bf16) {
        const uint32_t u = (uint32_t)r << 16;
        float f;
        memcpy(&f, &u, 4);
        out[i] = f32_to_f16_host(f);
      } else {
        out[i] = r;
      }
    }
    return NNZ_OK;
  };
  int rc = conv(ts, s);
  if (rc) return rc;
  if (m->fmt == NNZ_Q1) {
    if (m->c.q1_scales_are_mlx) {
      // symmetric scale = mlx_scale / 2 (model.zig:944-959)
      for (auto& v : s) v = f32_to_f16_host(f16_to_f32_host(v) / 2.0f);
    }
    b.clear();
  } else {
    const HostTensor* tb = find_t(m, base + ".biases");
    if (!tb) return fail(NNZ_ENOTFOUND, "tensor not found: " + base + ".biases");
    if (tb->data.size() < ng * 2) return fail(NNZ_EINVAL, base + ".biases too small");
    rc = conv(tb, b);
    if (rc) return rc;
  }
  return NNZ_OK;
}

// Replace a flat [M][K] matrix by its rows / columns [lo, hi) (axis 0 / 1).
int shard_vec(nnz_model* m, int axis, uint32_t M, uint32_t K, uint32_t lo, uint32_t hi,
              std::vector<uint8_t>& w, std::vector<uint16_t>& s, std::vector<uint16_t>& b) {
  const uint32_t gs = (uint32_t)m->c.group_size;
  const uint32_t Mo = axis == 0 ? hi - lo : M, Ko = axis == 0 ? K : hi - lo;
  std::vector<uint8_t> wo(m->fmt == NNZ_Q1 ? (size_t)Mo * Ko / 8 : (size_t)Mo * Ko / 2);
  std::vector<uint16_t> so((size_t)Mo * Ko / gs), bo(b.empty() ? 0 : so.size());
  if (shard_host(m->fmt, axis, w.data(), s.data(), b.empty() ? nullptr : b.data(), M, K, gs, lo, hi, wo.data(),
                 so.data(), bo.empty() ? nullptr : bo.data()))
    return fail(NNZ_EINVAL, "tensor-parallel shard: bad range");
  w.swap(wo);
  s.swap(so);
  b.swap(bo);
  return NNZ_OK;
}

// get_proj of this rank's shard: (Mloc x Kloc) taken at rank * Mloc rows
// (axis 0) or rank * Kloc columns (axis 1) of the full tensor.
int get_proj_tp(nnz_model* m, const std::string& base, uint32_t Mloc, uint32_t Kloc, int axis,
                std::vector<uint8_t>& w, std::vector<uint16_t>& s, std::vector<uint16_t>& b) {
  if (m->tp == 1) return get_proj(m, base, Mloc, Kloc, w, s, b);
  const uint32_t T = (uint32_t)m->tp, r = (uint32_t)m->tp_rank;
  const uint32_t M = axis == 0 ? Mloc * T : Mloc, K = axis == 1 ? Kloc * T : Kloc;
  int rc = get_proj(m, base, M, K, w, s, b);
  if (rc) return rc;
  const uint32_t n = axis == 0 ? Mloc : Kloc;
  return shard_vec(m, axis, M, K, r * n, (r + 1) * n, w, s, b);
}

int get_norm(nnz_model* m, const std::string& name, uint32_t n, std::vector<float>& out) {
  const HostTensor* t = find_t(m, name);
  if (!t) return fail(NNZ_ENOTFOUND, "tensor not found: " + name);
  out.resize(n);
  if (t->dtype == NNZ_DT_F32) {
    if (t->data.size() < (size_t)n * 4) return fail(NNZ_EINVAL, name + " too small");
    memcpy(out.data(), t->data.data(), (size_t)n * 4);
  } else if (t->dtype == NNZ_DT_F16 || t->dtype == NNZ_DT_BF16) {
    if (t->data.size() < (size_t)n * 2) return fail(NNZ_EINVAL, name + " too small");
    const uint16_t* s = reinterpret_cast<const uint16_t*>(t->data.data());
    for (uint32_t i = 0; i < n; ++i) {
      if (t->dtype == NNZ_DT_F16) out[i] = f16_to_f32_host(s[i]);
      else {
        const uint32_t u = (uint32_t)s[i] << 16;
        memcpy(&out[i], &u, 4);
      }
    }
  } else {
    return fail(NNZ_EINVAL, name + ": norm weights must be f32/f16/bf16");
  }
  return NNZ_OK;
}

// Device copy of a matrix in the reference's flat layout (prefill GEMM).
int upload_flat(nnz_model* m, const std::vector<uint8_t>& w, const std::vector<uint16_t>& s,
                const std::vector<uint16_t>& b, FlatW* out) {
  const size_t wb = align_up(w.size(), 256), sb = align_up(s.size() * 2, 256), bb = b.size() * 2;
  uint8_t* p = nullptr;
  int rc = dalloc(m, (void**)&p, wb + sb + std::max<size_t>(bb, 16));
  if (rc) return rc;
  NNZ_CK(cudaMemcpy(p, w.data(), w.size(), cudaMemcpyHostToDevice));
  NNZ_CK(cudaMemcpy(p + wb, s.data(), s.size() * 2, cudaMemcpyHostToDevice));
  if (bb) NNZ_CK(cudaMemcpy(p + wb + sb, b.data(), bb, cudaMemcpyHostToDevice));
  out->w = p;
  out->s = reinterpret_cast<const uint16_t*>(p + wb);
  out->b = bb ? reinterpret_cast<const uint16_t*>(p + wb + sb) : nullptr;
  return NNZ_OK;
}

// ---- launch helpers --------------------------------------------------------

int qmv(nnz_model* m, int sub, int pro, int epi, const uint8_t* w, uint32_t M, uint32_t K,
        const void* x, uint32_t x_stride, const float* nw, uint32_t batch, void* out,
        uint32_t out_stride, float* logits, unsigned long long* am, int pdl) {
  QmvLaunch L{m->fmt, sub, pro, epi, m->bf16s, pdl};
  QmvArgs a{};
  a.w = w; a.M = M; a.K = K; a.gs = (uint32_t)m->c.group_size;
  a.x = x; a.x_stride = x_stride; a.norm_w = nw; a.eps = m->c.eps; a.batch = batch;
  a.out = out; a.out_stride = out_stride; a.logits = logits; a.logits_stride = M;
  a.argmax = am; a.ws = m->ws; a.counters = m->counters; a.err = m->err;
  a.bf16_round = (uint32_t)m->bf16r;
  NNZ_CK(qmv_launch(L, a, m->num_sms, m->st));
  return NNZ_OK;
}

uint32_t attn_splits(nnz_model* m, uint32_t rows) {
  uint32_t s = (uint32_t)m->num_sms / std::max(1u, m->c.num_kv_heads * rows);
  return std::min(16u, std::max(1u, s));
}

int attn(nnz_model* m, uint32_t layer, uint32_t rows, const int* pos, const int* slot, int write,
         int pdl) {
  AttnArgs a{};
  a.qkv = m->qkv; a.qkv_stride = m->qkv_rows;
  a.q_norm = m->L[layer].q_norm; a.k_norm = m->L[layer].k_norm;
  a.kc = m->kc + m->kv_layer * layer; a.vc = m->vc + m->kv_layer * layer;
  a.max_ctx = m->c.max_context_length; a.pos = pos; a.slot = slot; a.rows = rows;
  a.n_q = m->c.num_query_heads; a.n_kv = m->c.num_kv_heads;
  a.eps = m->c.eps; a.theta = m->c.rope_theta; a.rope_style = m->c.rope_style;
  a.write_kv = write; a.splits = attn_splits(m, rows); a.rope_tab = m->rope_tab; a.slots = m->slots;
  a.out = m->attn; a.out_stride = m->qd; a.ws = m->ws; a.counters = m->counters; a.err = m->err;
  NNZ_CK(attn_decode_launch(a, (int)m->c.head_dim, pdl, m->st));
  return NNZ_OK;
}

int kv_write(nnz_model* m, uint32_t layer, uint32_t rows, const int* pos, const int* slot, int pdl) {
  AttnArgs a{};
  a.qkv = m->qkv; a.qkv_stride = m->qkv_rows;
  a.q_norm = m->L[layer].q_norm; a.k_norm = m->L[layer].k_norm;
  a.kc = m->kc + m->kv_layer * layer; a.vc = m->vc + m->kv_layer * layer;
  a.max_ctx = m->c.max_context_length; a.pos = pos; a.slot = slot; a.rows = rows;
  a.n_q = m->c.num_query_heads; a.n_kv = m->c.num_kv_heads;
  a.eps = m->c.eps; a.theta = m->c.rope_theta; a.rope_style = m->c.rope_style;
  a.err = m->err;
  NNZ_CK(rope_kv_write_launch(a, (int)m->c.head_dim, pdl, m->st));
  return NNZ_OK;
}

// One decoder layer for `rows` rows.  decode: pos/slot per row, fused KV
// write; prefill chunk: rows share slot 0, K/V written first.
int gemm(nnz_model* m, const FlatW& W, const FlatW* W2, uint32_t N, uint32_t K, const __half* x,
         uint32_t rows, int epi, void* out, uint32_t ldo);

// Tensor parallelism around a row-split projection (o, down): every rank
// holds the same residual R; rank 0 accumulates R + P_0, the others start
// from zero and accumulate P_r, and a sum all-reduce leaves R + sum P_r.
int tp_pre_add(nnz_model* m, uint32_t rows) {
  if (m->tp > 1 && m->tp_rank != 0)
    NNZ_CK(cudaMemsetAsync(m->residual, 0, (size_t)rows * m->c.hidden_size * 4, m->st));
  return NNZ_OK;
}

int nccl_fail(ncclResult_t r) {
  std::string e;
  const NcclApi* api = nccl_api(&e);
  return fail(NNZ_ENCCL, std::string("NCCL: ") + (api ? api->error_string(r) : e.c_str()));
}

// A row-split projection (o / down) added into the residual of the whole
// group.  With peer memory: the GEMM accumulates this GPU's partial in a
// local buffer, then tp_allreduce_kernel pushes it into every peer's slot
// array over NVLink, exchanges per-slice flags and adds all partials into
// the residual.  The buffers alternate between two halves, so a GPU that
// runs ahead writes into the half its slower peers are not reading.
// Otherwise: zero-start + NCCL all-reduce.
int tp_post_add(nnz_model* m, uint32_t rows);
// next_norm (optional): the RMSNorm weights of the norm that follows; with
// the peer-memory reduction and hidden size 2048 the reduction kernel
// applies it and writes xn itself (m->xn_from_tp).
int gemm_resadd_tp(nnz_model* m, const FlatW& W, uint32_t K, const __half* x, uint32_t rows,
                   const float* next_norm = nullptr) {
  const uint32_t H = m->c.hidden_size;
  int rc;
  m->xn_from_tp = false;
  if (m->tp_fused) {
    const int par = m->tp_parity;
    m->tp_parity ^= 1;
    float* racc = m->tp_racc + (size_t)par * m->rows_max * H;
    if ((rc = gemm(m, W, nullptr, H, K, x, rows, GEPI_RESADD, racc, H))) return rc;
    const bool fuse = next_norm && H == kTpNormRow;
    NNZ_CK(tp_allreduce_launch(m->residual, racc, m->d_peer_slots + (size_t)par * m->tp, m->tp_flags,
                               m->d_peer_flags, (size_t)rows * H, m->tp_rank, m->tp, m->err, m->st, 0,
                               fuse ? next_norm : nullptr, m->c.eps, m->xn, m->bf16r, 1));
    m->xn_from_tp = fuse;
    return NNZ_OK;
  }
  if ((rc = tp_pre_add(m, rows))) return rc;
  if ((rc = gemm(m, W, nullptr, H, K, x, rows, GEPI_RESADD, m->residual, H))) return rc;
  return tp_post_add(m, rows);
}

int tp_post_add(nnz_model* m, uint32_t rows) {
  if (m->tp == 1) return NNZ_OK;
  const NcclApi* api = nccl_api(nullptr);
  const ncclResult_t r = api->all_reduce(m->residual, m->residual, (size_t)rows * m->c.hidden_size, ncclFloat32,
                                         ncclSum, m->comm, m->st);
  return r == ncclSuccess ? NNZ_OK : nccl_fail(r);
}

// After a vocabulary-sharded LM head: local indices -> global, then the
// packed (value, index) slots reduced with max (first maximum wins).
int tp_argmax(nnz_model* m, uint32_t rows) {
  if (m->tp == 1) return NNZ_OK;
  NNZ_CK(argmax_shift_launch(m->state->argmax, rows, m->lm_off, m->st));
  const NcclApi* api = nccl_api(nullptr);
  const ncclResult_t r = api->all_reduce(m->state->argmax, m->state->argmax, rows, ncclUint64, ncclMax, m->comm, m->st);
  return r == ncclSuccess ? NNZ_OK : nccl_fail(r);
}


int enqueue_layer(nnz_model* m, uint32_t l, uint32_t rows, const int* pos, const int* slot,
                  bool prefill, int pdl) {
  const nnz_config& c = m->c;
  const LayerW& W = m->L[l];
  int rc;
  if (!prefill && m->gemm_prefill && rows >= kGemmDecodeRows) {
    // large decode batches: the projections as tcgen05 GEMMs over the rows
    const uint32_t H = c.hidden_size, I = c.intermediate_size;
    const float* next_norm = l + 1 < c.num_layers ? m->L[l + 1].attn_norm : m->fnorm;
    if (!(l > 0 && m->xn_from_tp))
      NNZ_CK(rmsnorm_f16_launch(m->residual, W.attn_norm, c.eps, rows, H, m->bf16r, m->xn, m->st, 1));
    if ((rc = gemm(m, W.fqkv, nullptr, m->qkv_rows, H, m->xn, rows, GEPI_F16, m->qkv, m->qkv_rows))) return rc;
    if ((rc = attn(m, l, rows, pos, slot, 1, 1))) return rc;
    if ((rc = gemm_resadd_tp(m, W.fo, m->qd, m->attn, rows, W.ffn_norm))) return rc;
    if (!m->xn_from_tp)
      NNZ_CK(rmsnorm_f16_launch(m->residual, W.ffn_norm, c.eps, rows, H, m->bf16r, m->xn, m->st, 1));
    if ((rc = gemm(m, W.fgate, &W.fup, I, H, m->xn, rows, GEPI_SILU, m->h, I))) return rc;
    return gemm_resadd_tp(m, W.fdown, I, m->h, rows, next_norm);
  }
  if ((rc = qmv(m, 1, PRO_NORM, EPI_F16, W.qkv, m->qkv_rows, c.hidden_size, m->residual,
                c.hidden_size, W.attn_norm, rows, m->qkv, m->qkv_rows, nullptr, nullptr, pdl)))
    return rc;
  if (prefill) {
    if ((rc = kv_write(m, l, rows, pos, slot, pdl))) return rc;
    if ((rc = attn(m, l, rows, pos, slot, 0, pdl))) return rc;
  } else {
    if ((rc = attn(m, l, rows, pos, slot, 1, pdl))) return rc;
  }
  if ((rc = tp_pre_add(m, rows))) return rc;
  if ((rc = qmv(m, 1, PRO_F16, EPI_RESADD, W.o, c.hidden_size, m->qd, m->attn, m->qd, nullptr,
                rows, m->residual, c.hidden_size, nullptr, nullptr, pdl)))
    return rc;
  if ((rc = tp_post_add(m, rows))) return rc;
  if ((rc = qmv(m, 2, PRO_NORM, EPI_SILU, W.gu, c.intermediate_size, c.hidden_size, m->residual,
                c.hidden_size, W.ffn_norm, rows, m->h, c.intermediate_size, nullptr, nullptr, pdl)))
    return rc;
  if ((rc = tp_pre_add(m, rows))) return rc;
  if ((rc = qmv(m, 1, PRO_F16, EPI_RESADD, W.down, c.hidden_size, c.intermediate_size, m->h,
                c.intermediate_size, nullptr, rows, m->residual, c.hidden_size, nullptr, nullptr,
                pdl)))
    return rc;
  return tp_post_add(m, rows);
}

int enqueue_embed(nnz_model* m, uint32_t rows, const uint32_t* tokens, int pdl) {
  EmbedArgs e{};
  e.wbytes = m->emb_w; e.scales = m->emb_s; e.biases = m->emb_b;
  e.vocab = m->c.vocab_size; e.H = m->c.hidden_size; e.gs = (uint32_t)m->c.group_size;
  e.bf16_round = m->bf16r; e.st = m->state; e.tokens = tokens;
  e.seq = m->seq; e.seq_len = m->c.max_context_length;
  e.residual = m->residual; e.rows = rows; e.err = m->err;
  NNZ_CK(embed_launch(e, m->fmt, m->bf16s, pdl, m->st));
  return NNZ_OK;
}

int enqueue_decode(nnz_model* m, uint32_t rows, bool want_logits, int pdl) {
  int rc;
  if ((rc = enqueue_embed(m, rows, nullptr, pdl))) return rc;
  for (uint32_t l = 0; l < m->c.num_layers; ++l)
    if ((rc = enqueue_layer(m, l, rows, m->state->pos, nullptr, false, pdl))) return rc;
  if (m->gemm_prefill && rows >= kGemmDecodeRows) {
    // final norm -> LM-head GEMM into the logits buffer -> argmax per row
    const nnz_config& c = m->c;
    if (!m->xn_from_tp)
      NNZ_CK(rmsnorm_f16_launch(m->residual, m->fnorm, c.eps, rows, c.hidden_size, m->bf16r, m->xn, m->st, 1));
    if ((rc = gemm(m, m->flm, nullptr, m->lm_rows, c.hidden_size, m->xn, rows, GEPI_F32, m->logits,
                   m->lm_rows)))
      return rc;
    NNZ_CK(logits_argmax_launch(m->logits, rows, m->lm_rows, m->lm_rows, m->state->argmax, m->st));
    return tp_argmax(m, rows);
  }
  if ((rc = qmv(m, 1, PRO_NORM, EPI_LOGITS, m->lm, m->lm_rows, m->c.hidden_size, m->residual,
                m->c.hidden_size, m->fnorm, rows, nullptr, 0, want_logits ? m->logits : nullptr,
                m->state->argmax, pdl)))
    return rc;
  return tp_argmax(m, rows);
}

int get_graph(nnz_model* m, uint32_t rows, bool want_logits, cudaGraphExec_t* out) {
  auto key = std::make_pair(rows, want_logits ? 1 : 0);
  auto it = m->graphs.find(key);
  if (it != m->graphs.end()) {
    *out = it->second;
    return NNZ_OK;
  }
  cudaGraph_t g;
  NNZ_CK(cudaStreamBeginCapture(m->st, cudaStreamCaptureModeThreadLocal));
  int rc = enqueue_decode(m, rows, want_logits, 1);
  cudaError_t ce = cudaStreamEndCapture(m->st, &g);
  if (rc) return rc;
  if (ce != cudaSuccess) return fail(NNZ_ECUDA, std::string("graph capture: ") + cudaGetErrorString(ce));
  cudaGraphExec_t ex;
  NNZ_CK(cudaGraphInstantiate(&ex, g, 0));
  cudaGraphDestroy(g);
  m->graphs[key] = ex;
  *out = ex;
  return NNZ_OK;
}

int sync_check(nnz_model* m) {
  NNZ_CK(cudaStreamSynchronize(m->st));
  int flags = 0;
  NNZ_CK(cudaMemcpy(&flags, m->err, 4, cudaMemcpyDeviceToHost));
  if (flags) {
    cudaMemset(m->err, 0, 4);
    if (m->mbar) cudaMemset(m->mbar, 0, 64);   // clear a persistent-kernel abort
    m->mbar_count = 0;
    if (m->d1_ok) {   // single-row kernel: clear counters, barrier and accumulators
      cudaMemset(m->d1.bar, 0, 64);
      cudaMemset(m->d1.cnt, 0, m->d1_cnt_words * 4);
      cudaMemset(m->d1.R, 0, 4 * (size_t)m->c.hidden_size * 4);
      cudaMemset(m->d1.qkv, 0, (size_t)m->d1.g.qkv_rows * 4);   // no stale layer tags
      m->d1_bar_count = 0;
      m->d1_epoch = 0;
    }
    return fail(flags & (ERR_MBAR_TIMEOUT | ERR_SPIN_TIMEOUT) ? NNZ_ETIMEDOUT : NNZ_EDEVICE,
                err_text(flags));
  }
  return NNZ_OK;
}

int set_advance(nnz_model* m, int v) {
  NNZ_CK(cudaMemsetAsync(&m->state->advance, 0, 4, m->st));
  if (v) NNZ_CK(cudaMemsetAsync(&m->state->advance, 1, 1, m->st));
  return NNZ_OK;
}

const nnz_model::MegaPlan* mega_plan_for(nnz_model* m, uint32_t rows) {
  if (!m->mega_ok || rows > (uint32_t)kBatchChunk) return nullptr;
  auto it = m->mplans.find(rows);
  if (it != m->mplans.end()) return it->second.ok ? &it->second : nullptr;
  nnz_model::MegaPlan P{};
  MegaArgs& a = P.a;
  const nnz_config& c = m->c;
  a.H = c.hidden_size; a.I = c.intermediate_size; a.n_q = c.num_query_heads; a.n_kv = c.num_kv_heads;
  a.hd = c.head_dim; a.L = c.num_layers; a.vocab = m->lm_rows; a.gs = (uint32_t)c.group_size;
  a.max_ctx = c.max_context_length; a.batch = rows; a.eps = c.eps; a.theta = c.rope_theta;
  a.rope_style = c.rope_style; a.bf16r = m->bf16r; a.layers = m->mlayers; a.rope_tab = m->rope_tab; a.lm = m->lm; a.fnorm = m->fnorm;
  a.emb_w = m->emb_w; a.emb_s = m->emb_s; a.emb_b = m->emb_b; a.kc = m->kc; a.vc = m->vc;
  a.kv_layer = m->kv_layer; a.R = m->mR; a.qkv_acc = m->mqkv; a.gu_acc = m->mgu; a.att_ws = m->matt;
  a.st = m->state; a.seq = m->seq; a.seq_len = c.max_context_length; a.logits = nullptr;
  a.bar = m->mbar; a.err = m->err; a.prof = m->mprof; a.dep = m->mdep;
  {
    const LayerW& W0 = m->L[0];
    a.l0 = MegaLayer{W0.qkv, W0.o, W0.gu, W0.down, W0.attn_norm, W0.ffn_norm, W0.q_norm, W0.k_norm};
    a.lstride = c.num_layers > 1 ? (size_t)(m->L[1].qkv - W0.qkv) : 0;
    for (uint32_t l = 0; l < c.num_layers; ++l) {   // layers must be equally spaced
      const LayerW& W = m->L[l];
      const size_t d = (size_t)l * a.lstride;
      auto same = [&](const void* x, const void* x0) {
        return reinterpret_cast<const uint8_t*>(x) == reinterpret_cast<const uint8_t*>(x0) + d;
      };
      if (!same(W.qkv, W0.qkv) || !same(W.o, W0.o) || !same(W.gu, W0.gu) || !same(W.down, W0.down) ||
          !same(W.attn_norm, W0.attn_norm) || !same(W.ffn_norm, W0.ffn_norm) ||
          !same(W.q_norm, W0.q_norm) || !same(W.k_norm, W0.k_norm)) {
        m->mplans[rows] = P;   // ok = false
        return nullptr;
      }
    }
  }
  P.ok = mega_plan(a, m->fmt, m->bf16s, m->device, &P.grid, &P.smem);
  if (P.ok) {
    std::vector<uint32_t> off;
    const std::vector<unsigned long long> wl = mega_weight_stream(a, m->fmt, P.grid, &off);
    void *dl = nullptr, *doff = nullptr;
    if (dalloc(m, &dl, wl.size() * 8) || dalloc(m, &doff, off.size() * 4) ||
        cudaMemcpy(dl, wl.data(), wl.size() * 8, cudaMemcpyHostToDevice) != cudaSuccess ||
        cudaMemcpy(doff, off.data(), off.size() * 4, cudaMemcpyHostToDevice) != cudaSuccess) {
      P.ok = false;
    } else {
      a.wlist = static_cast<const unsigned long long*>(dl);
      a.woff = static_cast<const uint32_t*>(doff);
    }
  }
  m->mplans[rows] = P;
  return P.ok ? &m->mplans[rows] : nullptr;
}

// One decode step for `rows` rows from the device decode state: the
// persistent kernel when it applies, else the captured multi-kernel graph.
// `ntok` greedy steps of the single-row kernel in one launch (token and
// position advance on the device exactly as `ntok` separate steps would).
int d1_run(nnz_model* m, uint32_t ntok, bool want_logits) {
  if (m->d1_epoch + ntok > (1u << 24)) {   // keep the per-layer counters far from wrapping
    NNZ_CK(cudaMemsetAsync(m->d1.cnt, 0, m->d1_cnt_words * 4, m->st));
    // the layer tags restart with the epoch: clear the words they mark
    NNZ_CK(cudaMemsetAsync(m->d1.qkv, 0, (size_t)m->d1.g.qkv_rows * 4, m->st));
    m->d1_epoch = 0;
  }
  D1Args a = m->d1;
  a.ntok = ntok;
  a.logits = want_logits ? m->logits : nullptr;
  a.bar_base = m->d1_bar_count;
  a.epoch = m->d1_epoch;
  NNZ_CK(d1_launch(a, m->st));
  m->d1_bar_count += (unsigned long long)a.g.P * ntok * d1_barriers_per_token(a.g);
  m->d1_epoch += ntok;
  return NNZ_OK;
}

int run_step(nnz_model* m, uint32_t rows, bool want_logits) {
  if (rows == 1 && m->d1_ok) return d1_run(m, 1, want_logits);
  if (const nnz_model::MegaPlan* P = mega_plan_for(m, rows)) {
    MegaArgs a = P->a;
    a.logits = want_logits ? m->logits : nullptr;
    a.bar_base = m->mbar_count;
    NNZ_CK(mega_launch(a, m->fmt, m->bf16s, P->grid, P->smem, m->st));
    m->mbar_count += (unsigned long long)P->grid * (1 + 2 * a.L);   // one arrival per CTA per barrier
    return NNZ_OK;
  }
  cudaGraphExec_t g;
  int rc = get_graph(m, rows, want_logits, &g);
  if (rc) return rc;
  NNZ_CK(cudaGraphLaunch(g, m->st));
  return NNZ_OK;
}

int gemm(nnz_model* m, const FlatW& W, const FlatW* W2, uint32_t N, uint32_t K, const __half* x,
         uint32_t rows, int epi, void* out, uint32_t ldo) {
  GemmArgs g{};
  g.M = rows; g.K = K; g.N = N; g.fmt = m->fmt; g.gs = m->c.group_size; g.bf16s = m->bf16s;
  g.bf16r = m->bf16r; g.w = W.w; g.s = W.s; g.b = W.b;
  if (W2) { g.w2 = W2->w; g.s2 = W2->s; g.b2 = W2->b; }
  g.epi = epi; g.out = out; g.ldo = ldo; g.err = m->err;
  g.acc = m->gacc; g.acc_floats = m->gacc_floats;
  g.pdl = 1;
  NNZ_CK(gemm_launch(g, x, m->st));
  return NNZ_OK;
}

// Prefill of prompt rows [c0, c0 + rows) on the tensor cores: per layer
// RMSNorm -> QKV GEMM -> K/V write + causal attention -> O GEMM (+residual)
// -> RMSNorm -> gate/up GEMM (SiLU*up) -> down GEMM (+residual).
int enqueue_layer_gemm(nnz_model* m, uint32_t l, uint32_t rows, const int* pos) {
  const nnz_config& c = m->c;
  const LayerW& W = m->L[l];
  const uint32_t H = c.hidden_size, I = c.intermediate_size;
  int rc;
  if (!(l > 0 && m->xn_from_tp))
    NNZ_CK(rmsnorm_f16_launch(m->residual, W.attn_norm, c.eps, rows, H, m->bf16r, m->xn, m->st, 1));
  if ((rc = gemm(m, W.fqkv, nullptr, m->qkv_rows, H, m->xn, rows, GEPI_F16, m->qkv, m->qkv_rows))) return rc;
  if ((rc = kv_write(m, l, rows, pos, m->zeros, 0))) return rc;
  {
    AttnArgs aa{};
    aa.qkv = m->qkv; aa.qkv_stride = m->qkv_rows; aa.q_norm = W.q_norm; aa.k_norm = W.k_norm;
    aa.kc = m->kc + m->kv_layer * l; aa.vc = m->vc + m->kv_layer * l; aa.max_ctx = c.max_context_length;
    aa.pos = pos; aa.slot = m->zeros; aa.slots = m->slots; aa.rows = rows; aa.n_q = c.num_query_heads; aa.n_kv = c.num_kv_heads;
    aa.eps = c.eps; aa.theta = c.rope_theta; aa.rope_style = c.rope_style; aa.out = m->attn;
    aa.out_stride = m->qd; aa.err = m->err; aa.rope_tab = m->rope_tab; aa.ws = m->ws;
    NNZ_CK(attn_prefill_launch(aa, (int)c.head_dim, 0, m->st));
  }
  if ((rc = gemm_resadd_tp(m, W.fo, m->qd, m->attn, rows, W.ffn_norm))) return rc;
  if (!m->xn_from_tp)
    NNZ_CK(rmsnorm_f16_launch(m->residual, W.ffn_norm, c.eps, rows, H, m->bf16r, m->xn, m->st, 1));
  if ((rc = gemm(m, W.fgate, &W.fup, I, H, m->xn, rows, GEPI_SILU, m->h, I))) return rc;
  // the next layer's attention norm (the final norm is not needed here: the
  // prefill's LM head normalises the last row itself)
  return gemm_resadd_tp(m, W.fdown, I, m->h, rows, l + 1 < c.num_layers ? m->L[l + 1].attn_norm : nullptr);
}

int enqueue_prefill(nnz_model* m, uint32_t n, bool want_logits) {
  int rc;
  if (m->gemm_prefill) {
    for (uint32_t c0 = 0; c0 < n; c0 += kGemmPrefillChunk) {
      const uint32_t rows = std::min(kGemmPrefillChunk, n - c0);
      if ((rc = enqueue_embed(m, rows, m->prompt + c0, 0))) return rc;
      for (uint32_t l = 0; l < m->c.num_layers; ++l)
        if ((rc = enqueue_layer_gemm(m, l, rows, m->iota + c0))) return rc;
      if (c0 + rows == n) {
        const float* last = m->residual + (size_t)(rows - 1) * m->c.hidden_size;
        if ((rc = qmv(m, 1, PRO_NORM, EPI_LOGITS, m->lm, m->lm_rows, m->c.hidden_size, last,
                      m->c.hidden_size, m->fnorm, 1, nullptr, 0, want_logits ? m->logits : nullptr,
                      m->state->argmax, 0)))
          return rc;
        if ((rc = tp_argmax(m, 1))) return rc;
      }
    }
    return NNZ_OK;
  }
  for (uint32_t c0 = 0; c0 < n; c0 += kPrefillChunk) {
    const uint32_t rows = std::min(kPrefillChunk, n - c0);
    if ((rc = enqueue_embed(m, rows, m->prompt + c0, 0))) return rc;
    for (uint32_t l = 0; l < m->c.num_layers; ++l)
      if ((rc = enqueue_layer(m, l, rows, m->iota + c0, m->zeros, true, 0))) return rc;
    if (c0 + rows == n) {
      const float* last = m->residual + (size_t)(rows - 1) * m->c.hidden_size;
      if ((rc = qmv(m, 1, PRO_NORM, EPI_LOGITS, m->lm, m->lm_rows, m->c.hidden_size, last,
                    m->c.hidden_size, m->fnorm, 1, nullptr, 0, want_logits ? m->logits : nullptr,
                    m->state->argmax, 0)))
        return rc;
      if ((rc = tp_argmax(m, 1))) return rc;
    }
  }
  return NNZ_OK;
}

// Persistent-kernel plan for `rows` decode rows (cached).

}  // namespace

// Map every group member's reduction buffers and barrier flags into this process
// (CUDA IPC handles exchanged with an NCCL all-gather) for the fused
// GEMM + peer-memory reduction.  Collective: every rank calls it at
// finalize.
int tp_setup_peers(nnz_model* m) {
  const int T = m->tp, r = m->tp_rank;
  int rc;
  const size_t nmax = (size_t)m->rows_max * m->c.hidden_size;
  const size_t nflag = tp_allreduce_flag_words(nmax, T);
  if ((rc = dalloc(m, (void**)&m->tp_racc, 2 * nmax * 4))) return rc;
  NNZ_CK(cudaMemset(m->tp_racc, 0, 2 * nmax * 4));
  if ((rc = dalloc(m, (void**)&m->tp_slots, 2 * (size_t)T * nmax * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->tp_flags, nflag * 4))) return rc;
  NNZ_CK(cudaMemset(m->tp_flags, 0, nflag * 4));
  struct Handles { cudaIpcMemHandle_t slots, flags; };
  Handles mine;
  NNZ_CK(cudaIpcGetMemHandle(&mine.slots, m->tp_slots));
  NNZ_CK(cudaIpcGetMemHandle(&mine.flags, m->tp_flags));
  void* dbuf = nullptr;
  if ((rc = dalloc(m, &dbuf, sizeof(Handles) * (T + 1)))) return rc;
  NNZ_CK(cudaMemcpy(dbuf, &mine, sizeof(Handles), cudaMemcpyHostToDevice));
  const NcclApi* api = nccl_api(nullptr);
  const ncclResult_t nr = api->all_gather(dbuf, static_cast<uint8_t*>(dbuf) + sizeof(Handles), sizeof(Handles),
                                          ncclUint8, m->comm, m->st);
  if (nr != ncclSuccess) return nccl_fail(nr);
  std::vector<Handles> all(T);
  NNZ_CK(cudaMemcpyAsync(all.data(), static_cast<uint8_t*>(dbuf) + sizeof(Handles), sizeof(Handles) * T,
                         cudaMemcpyDeviceToHost, m->st));
  NNZ_CK(cudaStreamSynchronize(m->st));
  std::vector<float*> slots(2 * T);
  std::vector<uint32_t*> flags(T);
  for (int j = 0; j < T; ++j) {
    float* sb = m->tp_slots;
    uint32_t* fb = m->tp_flags;
    if (j != r) {
      void *ps = nullptr, *pf = nullptr;
      NNZ_CK(cudaIpcOpenMemHandle(&ps, all[j].slots, cudaIpcMemLazyEnablePeerAccess));
      m->ipc_opened.push_back(ps);
      NNZ_CK(cudaIpcOpenMemHandle(&pf, all[j].flags, cudaIpcMemLazyEnablePeerAccess));
      m->ipc_opened.push_back(pf);
      sb = static_cast<float*>(ps);
      fb = static_cast<uint32_t*>(pf);
    }
    slots[j] = sb;                                // parity 0 half
    slots[T + j] = sb + (size_t)T * nmax;         // parity 1 half
    flags[j] = fb;
  }
  if ((rc = dalloc(m, (void**)&m->d_peer_slots, sizeof(float*) * 2 * T))) return rc;
  NNZ_CK(cudaMemcpy(m->d_peer_slots, slots.data(), sizeof(float*) * 2 * T, cudaMemcpyHostToDevice));
  if ((rc = dalloc(m, (void**)&m->d_peer_flags, sizeof(uint32_t*) * T))) return rc;
  NNZ_CK(cudaMemcpy(m->d_peer_flags, flags.data(), sizeof(uint32_t*) * T, cudaMemcpyHostToDevice));
  m->tp_fused = true;
  return NNZ_OK;
}

// =========================================================================
// C ABI
// =========================================================================
// No C++ exception crosses the C ABI: the entry points that allocate host
// memory (weight packing, tensor copies, finalize) turn a failed allocation
// into NNZ_ENOMEM.
template <typename F>
static int host_guard(F&& f) {
  try {
    return f();
  } catch (const std::bad_alloc&) {
    return fail(NNZ_ENOMEM, "host memory allocation failed");
  } catch (const std::exception& e) {
    return fail(NNZ_EINVAL, std::string("host error: ") + e.what());
  }
}

extern "C" {

const char* nnz_last_error(void) { return g_err.c_str(); }
int nnz_version(void) { return 1; }
int nnz_device_count(void) {
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess) {
    cudaGetLastError();
    return 0;
  }
  return n;
}

size_t nnz_packed_bytes(int fmt, uint32_t M, uint32_t K, uint32_t gs, uint32_t sub) {
  if ((fmt != NNZ_Q1 && fmt != NNZ_Q4) || gs == 0 || gs % 32 || K % gs || sub == 0) return 0;
  return packed_bytes(fmt, M, K, gs, sub);
}

static int pack_weights_impl(int fmt, const void* weight, const uint16_t* scales, const uint16_t* biases,
                     uint32_t M, uint32_t K, uint32_t gs, uint32_t sub, uint32_t sub_index,
                     void* packed_out) {
  if (pack_host(fmt, weight, scales, biases, M, K, gs, sub, sub_index, packed_out, 0))
    return fail(NNZ_EINVAL, "nnz_pack_weights: invalid arguments");
  return NNZ_OK;
}

int nnz_pack_weights(int fmt, const void* weight, const uint16_t* scales, const uint16_t* biases,
                     uint32_t M, uint32_t K, uint32_t gs, uint32_t sub, uint32_t sub_index,
                     void* packed_out) {
  return host_guard(
      [&] { return pack_weights_impl(fmt, weight, scales, biases, M, K, gs, sub, sub_index, packed_out); });
}

static int unpack_weights_impl(int fmt, const void* packed, uint32_t M, uint32_t K, uint32_t gs,
                       uint32_t sub, uint32_t sub_index, void* weight, uint16_t* scales,
                       uint16_t* biases) {
  if (unpack_host(fmt, packed, M, K, gs, sub, sub_index, weight, scales, biases))
    return fail(NNZ_EINVAL, "nnz_unpack_weights: invalid arguments");
  return NNZ_OK;
}

int nnz_unpack_weights(int fmt, const void* packed, uint32_t M, uint32_t K, uint32_t gs,
                       uint32_t sub, uint32_t sub_index, void* weight, uint16_t* scales,
                       uint16_t* biases) {
  return host_guard(
      [&] { return unpack_weights_impl(fmt, packed, M, K, gs, sub, sub_index, weight, scales, biases); });
}

static int model_create_impl(int device, const nnz_config* cfg, nnz_model** out) {
  if (!cfg || !out) return fail(NNZ_EINVAL, "null argument");
  const nnz_config& c = *cfg;
  if (c.quant_format != NNZ_Q1 && c.quant_format != NNZ_Q4) return fail(NNZ_EINVAL, "quant_format");
  if (c.head_dim != 64 && c.head_dim != 128) return fail(NNZ_EINVAL, "head_dim must be 64 or 128");
  if (!c.num_kv_heads || c.num_query_heads % c.num_kv_heads ||
      c.num_query_heads / c.num_kv_heads > (uint32_t)kAttnMaxG)
    return fail(NNZ_EINVAL, "num_query_heads must be a multiple (<= 8x) of num_kv_heads");
  const uint32_t gs = (uint32_t)c.group_size;
  const uint32_t qd = c.num_query_heads * c.head_dim;
  if (gs == 0 || gs % 32 || gs > 256 || c.hidden_size % gs || c.intermediate_size % gs || qd % gs)
    return fail(NNZ_EINVAL, "group_size must be a multiple of 32 (<= 256) dividing hidden, "
                            "intermediate and query dims");
  if (!c.vocab_size || !c.num_layers || !c.max_context_length)
    return fail(NNZ_EINVAL, "vocab_size, num_layers and max_context_length must be > 0");
  if (c.max_batch == 0 || c.max_batch > (uint32_t)kMaxRows) return fail(NNZ_EINVAL, "max_batch");
  const int tp = c.tp_size > 1 ? c.tp_size : 1;
  if (tp > 1) {
    if (tp > 64 || c.tp_rank < 0 || c.tp_rank >= tp) return fail(NNZ_EINVAL, "tp_rank / tp_size");
    if (c.num_kv_heads % tp || c.intermediate_size % ((uint32_t)tp * gs) ||
        (qd / tp) % gs)
      return fail(NNZ_EINVAL, "tensor parallelism needs num_kv_heads, intermediate_size / group_size "
                              "and query dim / group_size divisible by tp_size");
  }
  int ndev = 0;
  NNZ_CK(cudaGetDeviceCount(&ndev));
  if (device < 0 || device >= ndev) return fail(NNZ_EINVAL, "bad device index");
  auto* m = new nnz_model();
  m->c = c;
  if (m->c.eps <= 0.f) m->c.eps = 1e-6f;
  m->full = m->c;
  m->tp = tp;
  m->tp_rank = tp > 1 ? c.tp_rank : 0;
  if (tp > 1) {
    m->c.num_query_heads /= tp;
    m->c.num_kv_heads /= tp;
    m->c.intermediate_size /= tp;
  }
  {
    const uint32_t per = (c.vocab_size + tp - 1) / tp;
    m->lm_off = std::min(c.vocab_size, per * (uint32_t)m->tp_rank);
    m->lm_rows = std::min(c.vocab_size - m->lm_off, per);
    if (m->lm_rows == 0) {
      delete m;
      return fail(NNZ_EINVAL, "vocab_size smaller than tp_size");
    }
  }
  m->device = device;
  m->fmt = c.quant_format;
  m->bf16s = (c.quant_format == NNZ_Q4 && c.scale_dtype == NNZ_SCALE_BF16) ? 1 : 0;
  m->bf16r = (c.quant_format == NNZ_Q4 && c.bf16_faithful) ? 1 : 0;
  *out = m;
  return NNZ_OK;
}

int nnz_model_create(int device, const nnz_config* cfg, nnz_model** out) {
  return host_guard([&] { return model_create_impl(device, cfg, out); });
}

static int model_load_tensor_impl(nnz_model* m, const char* name, int dtype, const void* data, size_t bytes) {
  if (!m || !name || (!data && bytes)) return fail(NNZ_EINVAL, "null argument");
  if (m->finalized) return fail(NNZ_ESTATE, "model already finalized");
  if (dtype < NNZ_DT_U8 || dtype > NNZ_DT_F32) return fail(NNZ_EINVAL, "dtype");
  HostTensor& t = m->host[name];
  t.dtype = dtype;
  t.data.assign(static_cast<const uint8_t*>(data), static_cast<const uint8_t*>(data) + bytes);
  return NNZ_OK;
}

int nnz_model_load_tensor(nnz_model* m, const char* name, int dtype, const void* data, size_t bytes) {
  return host_guard([&] { return model_load_tensor_impl(m, name, dtype, data, bytes); });
}

static int model_finalize_impl(nnz_model* m) {
  if (!m) return fail(NNZ_EINVAL, "null model");
  if (m->finalized) return fail(NNZ_ESTATE, "model already finalized");
  if (m->tp > 1 && !m->comm) return fail(NNZ_ESTATE, "tensor-parallel model: call nnz_tp_init first");
  const nnz_config& c = m->c;
  NNZ_CK(cudaSetDevice(m->device));
  NNZ_CK(cudaDeviceGetAttribute(&m->num_sms, cudaDevAttrMultiProcessorCount, m->device));
  const uint32_t H = c.hidden_size, I = c.intermediate_size, gs = (uint32_t)c.group_size;
  m->qd = c.num_query_heads * c.head_dim;
  m->kvd = c.num_kv_heads * c.head_dim;
  m->qkv_rows = m->qd + 2 * m->kvd;
  m->slots = c.max_batch;
  {
    const char* pp = getenv("NNZ_PREFILL_PATH");
    m->gemm_prefill = !(pp && strcmp(pp, "qmv") == 0) && gs >= 64 && H % 64 == 0 &&
                      I % 64 == 0 && (c.num_query_heads * c.head_dim) % 64 == 0;
  }
  m->rows_max = std::max(c.max_batch, m->gemm_prefill ? kGemmPrefillChunk : kPrefillChunk);
  const int fmt = m->fmt;

  // ---- pack weights on the host ----------------------------------------
  const size_t b_qkv = packed_bytes(fmt, m->qkv_rows, H, gs, 1);
  const size_t b_o = packed_bytes(fmt, H, m->qd, gs, 1);
  const size_t b_gu = packed_bytes(fmt, I, H, gs, 2);
  const size_t b_dn = packed_bytes(fmt, H, I, gs, 1);
  const size_t b_lm = packed_bytes(fmt, m->lm_rows, H, gs, 1);
  const size_t emb_w = fmt == NNZ_Q1 ? (size_t)c.vocab_size * H / 8 : (size_t)c.vocab_size * H / 2;
  const size_t emb_g = (size_t)c.vocab_size * H / gs;
  size_t off = 0;
  auto take = [&](size_t bytes) { size_t o = off; off = align_up(off + bytes, 256); return o; };
  struct LOff { size_t qkv, o, gu, dn, an, fn, qn, kn; };
  std::vector<LOff> lo(c.num_layers);
  for (auto& x : lo) {
    x.qkv = take(b_qkv); x.o = take(b_o); x.gu = take(b_gu); x.dn = take(b_dn);
    x.an = take(H * 4); x.fn = take(H * 4); x.qn = take(c.head_dim * 4); x.kn = take(c.head_dim * 4);
  }
  const size_t o_embw = take(emb_w), o_embs = take(emb_g * 2), o_embb = take(emb_g * 2);
  const size_t o_lm = take(b_lm), o_fn = take(H * 4);
  m->arena_bytes = off;
  int rc;
  if ((rc = dalloc(m, (void**)&m->arena, m->arena_bytes))) return rc;
  // single-row decode kernel: Q1 g128, head_dim 128, one GPU, every SM
  D1Geom d1g{};
  std::vector<uint8_t> d1buf;
  uint8_t* d1_stream = nullptr;
  {
    const char* path = getenv("NNZ_DECODE_PATH");
    const bool off = path && (strcmp(path, "graph") == 0 || strcmp(path, "mega") == 0);
    m->d1_ok = !off && fmt == NNZ_Q1 && gs == 128 && c.head_dim == 128 && m->tp == 1 && !m->bf16r &&
               d1_geom(d1g, (uint32_t)m->num_sms, H, I, c.num_query_heads, c.num_kv_heads, c.num_layers,
                       m->lm_rows, c.max_context_length) &&
               d1_fits(m->device, d1g.P);
    if (m->d1_ok) {
      if ((rc = dalloc(m, (void**)&d1_stream, (size_t)d1g.P * d1g.nck * kD1Chunk))) return rc;
      d1buf.resize((size_t)d1g.P * std::max(d1g.cpl, d1g.clm) * kD1Chunk);
    }
  }
  auto d1_upload = [&](size_t chunk0, uint32_t nchunks) -> int {
    NNZ_CK(cudaMemcpy2D(d1_stream + chunk0 * kD1Chunk, (size_t)d1g.nck * kD1Chunk, d1buf.data(),
                        (size_t)nchunks * kD1Chunk, (size_t)nchunks * kD1Chunk, d1g.P, cudaMemcpyHostToDevice));
    return NNZ_OK;
  };
  std::vector<uint8_t> d1qw, d1ow, d1gw, d1uw;
  std::vector<uint16_t> d1qs, d1os, d1gs, d1us;
  std::vector<uint8_t> buf;
  std::vector<uint8_t> w;
  std::vector<uint16_t> s, b;
  m->L.resize(c.num_layers);
  for (uint32_t l = 0; l < c.num_layers; ++l) {
    const std::string pre = "model.layers." + std::to_string(l) + ".";
    // fused QKV: q, k, v rows concatenated (flat layouts concatenate exactly)
    {
      std::vector<uint8_t> wc;
      std::vector<uint16_t> sc, bc;
      const char* names[3] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj"};
      const uint32_t rows[3] = {m->qd, m->kvd, m->kvd};
      for (int i = 0; i < 3; ++i) {
        if ((rc = get_proj_tp(m, pre + names[i], rows[i], H, 0, w, s, b))) return rc;
        wc.insert(wc.end(), w.begin(), w.end());
        sc.insert(sc.end(), s.begin(), s.end());
        bc.insert(bc.end(), b.begin(), b.end());
      }
      if (m->gemm_prefill && (rc = upload_flat(m, wc, sc, bc, &m->L[l].fqkv))) return rc;
      if (m->d1_ok) { d1qw = wc; d1qs = sc; }
      buf.assign(b_qkv, 0);
      pack_host(fmt, wc.data(), sc.data(), bc.empty() ? nullptr : bc.data(), m->qkv_rows, H, gs, 1, 0,
                buf.data(), 0);
      NNZ_CK(cudaMemcpy(m->arena + lo[l].qkv, buf.data(), b_qkv, cudaMemcpyHostToDevice));
    }
    if ((rc = get_proj_tp(m, pre + "self_attn.o_proj", H, m->qd, 1, w, s, b))) return rc;
    if (m->gemm_prefill && (rc = upload_flat(m, w, s, b, &m->L[l].fo))) return rc;
    if (m->d1_ok) { d1ow = w; d1os = s; }
    buf.assign(b_o, 0);
    pack_host(fmt, w.data(), s.data(), b.empty() ? nullptr : b.data(), H, m->qd, gs, 1, 0, buf.data(), 0);
    NNZ_CK(cudaMemcpy(m->arena + lo[l].o, buf.data(), b_o, cudaMemcpyHostToDevice));
    buf.assign(b_gu, 0);
    if ((rc = get_proj_tp(m, pre + "mlp.gate_proj", I, H, 0, w, s, b))) return rc;
    if (m->gemm_prefill && (rc = upload_flat(m, w, s, b, &m->L[l].fgate))) return rc;
    if (m->d1_ok) { d1gw = w; d1gs = s; }
    pack_host(fmt, w.data(), s.data(), b.empty() ? nullptr : b.data(), I, H, gs, 2, 0, buf.data(), 0);
    if ((rc = get_proj_tp(m, pre + "mlp.up_proj", I, H, 0, w, s, b))) return rc;
    if (m->gemm_prefill && (rc = upload_flat(m, w, s, b, &m->L[l].fup))) return rc;
    if (m->d1_ok) { d1uw = w; d1us = s; }
    pack_host(fmt, w.data(), s.data(), b.empty() ? nullptr : b.data(), I, H, gs, 2, 1, buf.data(), 0);
    NNZ_CK(cudaMemcpy(m->arena + lo[l].gu, buf.data(), b_gu, cudaMemcpyHostToDevice));
    if ((rc = get_proj_tp(m, pre + "mlp.down_proj", H, I, 1, w, s, b))) return rc;
    if (m->gemm_prefill && (rc = upload_flat(m, w, s, b, &m->L[l].fdown))) return rc;
    if (m->d1_ok) {
      d1_pack_layer(d1g, d1qw.data(), d1qs.data(), d1ow.data(), d1os.data(), d1gw.data(), d1gs.data(),
                    d1uw.data(), d1us.data(), w.data(), s.data(), d1buf.data());
      if ((rc = d1_upload((size_t)l * d1g.cpl, d1g.cpl))) return rc;
    }
    buf.assign(b_dn, 0);
    pack_host(fmt, w.data(), s.data(), b.empty() ? nullptr : b.data(), H, I, gs, 1, 0, buf.data(), 0);
    NNZ_CK(cudaMemcpy(m->arena + lo[l].dn, buf.data(), b_dn, cudaMemcpyHostToDevice));
    std::vector<float> nv;
    const std::pair<const char*, std::pair<size_t, uint32_t>> norms[4] = {
        {"input_layernorm.weight", {lo[l].an, H}},
        {"post_attention_layernorm.weight", {lo[l].fn, H}},
        {"self_attn.q_norm.weight", {lo[l].qn, c.head_dim}},
        {"self_attn.k_norm.weight", {lo[l].kn, c.head_dim}}};
    for (const auto& nm : norms) {
      if ((rc = get_norm(m, pre + nm.first, nm.second.second, nv))) return rc;
      NNZ_CK(cudaMemcpy(m->arena + nm.second.first, nv.data(), nv.size() * 4, cudaMemcpyHostToDevice));
    }
    LayerW& LW = m->L[l];
    LW.qkv = m->arena + lo[l].qkv; LW.o = m->arena + lo[l].o;
    LW.gu = m->arena + lo[l].gu; LW.down = m->arena + lo[l].dn;
    LW.attn_norm = reinterpret_cast<float*>(m->arena + lo[l].an);
    LW.ffn_norm = reinterpret_cast<float*>(m->arena + lo[l].fn);
    LW.q_norm = reinterpret_cast<float*>(m->arena + lo[l].qn);
    LW.k_norm = reinterpret_cast<float*>(m->arena + lo[l].kn);
    // release host copies as we go
    for (const char* nm : {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj",
                           "self_attn.o_proj", "mlp.gate_proj", "mlp.up_proj", "mlp.down_proj"})
      for (const char* suf : {".weight", ".scales", ".biases"}) m->host.erase(pre + nm + suf);
  }
  // embedding (reference layout, gathered per token) and LM head (packed)
  if ((rc = get_proj(m, "model.embed_tokens", c.vocab_size, H, w, s, b))) return rc;
  NNZ_CK(cudaMemcpy(m->arena + o_embw, w.data(), emb_w, cudaMemcpyHostToDevice));
  NNZ_CK(cudaMemcpy(m->arena + o_embs, s.data(), emb_g * 2, cudaMemcpyHostToDevice));
  if (fmt == NNZ_Q4) NNZ_CK(cudaMemcpy(m->arena + o_embb, b.data(), emb_g * 2, cudaMemcpyHostToDevice));
  if (!c.tie_word_embeddings) {
    if ((rc = get_proj(m, "lm_head", c.vocab_size, H, w, s, b))) return rc;
  }
  if (m->tp > 1 && (rc = shard_vec(m, 0, c.vocab_size, H, m->lm_off, m->lm_off + m->lm_rows, w, s, b))) return rc;
  if (!c.tie_word_embeddings || m->tp > 1) {
    if (m->gemm_prefill && (rc = upload_flat(m, w, s, b, &m->flm))) return rc;
  } else if (m->gemm_prefill) {
    m->flm.w = m->arena + o_embw;
    m->flm.s = reinterpret_cast<const uint16_t*>(m->arena + o_embs);
    m->flm.b = fmt == NNZ_Q4 ? reinterpret_cast<const uint16_t*>(m->arena + o_embb) : nullptr;
  }
  if (m->d1_ok) {
    d1_pack_lm(d1g, w.data(), s.data(), d1buf.data());
    if ((rc = d1_upload((size_t)c.num_layers * d1g.cpl, d1g.clm))) return rc;
    std::vector<uint8_t>().swap(d1buf);
  }
  buf.assign(b_lm, 0);
  pack_host(fmt, w.data(), s.data(), b.empty() ? nullptr : b.data(), m->lm_rows, H, gs, 1, 0,
            buf.data(), 0);
  NNZ_CK(cudaMemcpy(m->arena + o_lm, buf.data(), b_lm, cudaMemcpyHostToDevice));
  {
    std::vector<float> nv;
    if ((rc = get_norm(m, "model.norm.weight", H, nv))) return rc;
    NNZ_CK(cudaMemcpy(m->arena + o_fn, nv.data(), H * 4, cudaMemcpyHostToDevice));
  }
  m->emb_w = m->arena + o_embw;
  m->emb_s = reinterpret_cast<uint16_t*>(m->arena + o_embs);
  m->emb_b = reinterpret_cast<uint16_t*>(m->arena + o_embb);
  m->lm = m->arena + o_lm;
  m->fnorm = reinterpret_cast<float*>(m->arena + o_fn);
  m->host.clear();
  std::vector<uint8_t>().swap(buf);

  // ---- KV cache, activations, workspace -----------------------------------
  m->kv_layer = (size_t)m->slots * c.num_kv_heads * c.max_context_length * c.head_dim;
  const size_t kv_bytes = m->kv_layer * c.num_layers * 2;
  if ((rc = dalloc(m, (void**)&m->kc, kv_bytes))) return rc;
  if ((rc = dalloc(m, (void**)&m->vc, kv_bytes))) return rc;
  NNZ_CK(cudaMemset(m->kc, 0, kv_bytes));
  NNZ_CK(cudaMemset(m->vc, 0, kv_bytes));
  const uint32_t R = m->rows_max;
  if ((rc = dalloc(m, (void**)&m->residual, (size_t)R * H * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->qkv, (size_t)R * m->qkv_rows * 2))) return rc;
  if ((rc = dalloc(m, (void**)&m->attn, (size_t)R * m->qd * 2))) return rc;
  if ((rc = dalloc(m, (void**)&m->h, (size_t)R * I * 2))) return rc;
  if (m->gemm_prefill && (rc = dalloc(m, (void**)&m->xn, (size_t)R * H * 2))) return rc;
  if (m->gemm_prefill && c.max_batch >= kGemmDecodeRows) {
    const size_t n = (size_t)c.max_batch * std::max<size_t>(std::max<size_t>(m->qkv_rows, 2 * I), H);
    if ((rc = dalloc(m, (void**)&m->gacc, n * 4))) return rc;
    NNZ_CK(cudaMemset(m->gacc, 0, n * 4));
    m->gacc_floats = n;
  }
  if ((rc = dalloc(m, (void**)&m->logits, (size_t)c.max_batch * m->lm_rows * 4))) return rc;
  size_t wsf = 0, nctr = 0;
  for (uint32_t rows = 1; rows <= R; ++rows) {
    const uint32_t ych = (rows + kBatchChunk - 1) / kBatchChunk;
    const uint32_t shapes[4][4] = {{m->qkv_rows, H, 1, 0}, {H, m->qd, 1, 0}, {I, H, 2, 0}, {H, I, 1, 0}};
    for (const auto& sh : shapes) {
      wsf = std::max(wsf, qmv_ws_floats(sh[0], sh[1], gs, fmt, (int)sh[2], rows, m->num_sms));
      nctr = std::max(nctr, (size_t)ych * num_tiles(sh[0]));
    }
    wsf = std::max(wsf, attn_ws_floats(rows, c.num_query_heads, c.num_kv_heads, attn_splits(m, rows),
                                       (int)c.head_dim, c.max_context_length));
    nctr = std::max(nctr, (size_t)rows * c.num_kv_heads);
  }
  wsf = std::max(wsf, qmv_ws_floats(m->lm_rows, H, gs, fmt, 1, c.max_batch, m->num_sms));
  if (attn_tc_applies(c.num_query_heads, c.num_kv_heads, (int)c.head_dim))
    wsf = std::max(wsf, attn_prefill_tc_ws_floats(R, c.num_query_heads));
  m->ws_floats = std::max<size_t>(wsf, 1024);
  m->n_counters = std::max<size_t>(nctr, 1024);
  if ((rc = dalloc(m, (void**)&m->ws, m->ws_floats * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->counters, m->n_counters * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->err, 16))) return rc;
  if ((rc = dalloc(m, (void**)&m->state, sizeof(DecodeState)))) return rc;
  if ((rc = dalloc(m, (void**)&m->seq, (size_t)m->slots * c.max_context_length * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->prompt, (size_t)c.max_context_length * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->uniforms, (size_t)c.max_context_length * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->iota, (size_t)c.max_context_length * 4))) return rc;
  if ((rc = dalloc(m, (void**)&m->zeros, (size_t)R * 4))) return rc;
  NNZ_CK(cudaMemset(m->counters, 0, m->n_counters * 4));
  NNZ_CK(cudaMemset(m->err, 0, 16));
  NNZ_CK(cudaMemset(m->state, 0, sizeof(DecodeState)));
  NNZ_CK(cudaMemset(m->seq, 0, (size_t)m->slots * c.max_context_length * 4));
  NNZ_CK(cudaMemset(m->zeros, 0, (size_t)R * 4));
  {
    std::vector<int> io(c.max_context_length);
    for (uint32_t i = 0; i < c.max_context_length; ++i) io[i] = (int)i;
    NNZ_CK(cudaMemcpy(m->iota, io.data(), io.size() * 4, cudaMemcpyHostToDevice));
  }
  {
    // rotary (cos, sin) per position and pair, in double like the
    // kernels' own evaluation, rounded to f32
    const uint32_t half = c.head_dim / 2;
    std::vector<float2> tab((size_t)c.max_context_length * half);
    const double l2t = std::log2((double)c.rope_theta);
    for (uint32_t p = 0; p < c.max_context_length; ++p)
      for (uint32_t i = 0; i < half; ++i) {
        const double ang = (double)p * std::exp2(-(2.0 * i / c.head_dim) * l2t);
        tab[(size_t)p * half + i] = make_float2((float)std::cos(ang), (float)std::sin(ang));
      }
    if ((rc = dalloc(m, (void**)&m->rope_tab, tab.size() * sizeof(float2)))) return rc;
    NNZ_CK(cudaMemcpy(m->rope_tab, tab.data(), tab.size() * sizeof(float2), cudaMemcpyHostToDevice));
  }
  {
    // persistent decode kernel buffers (NNZ_DECODE_PATH=graph disables it)
    const char* path = getenv("NNZ_DECODE_PATH");
    m->mega_ok = !(path && strcmp(path, "graph") == 0) && !m->bf16r && m->tp == 1;
    if (m->mega_ok) {
      const uint32_t bmax = std::min<uint32_t>(c.max_batch, kBatchChunk);
      const size_t G = c.num_query_heads / c.num_kv_heads;
      if ((rc = dalloc(m, (void**)&m->mR, (size_t)3 * bmax * H * 4))) return rc;
      if ((rc = dalloc(m, (void**)&m->mqkv, (size_t)bmax * m->qkv_rows * 4))) return rc;
      if ((rc = dalloc(m, (void**)&m->mgu, (size_t)bmax * 2 * I * 4))) return rc;
      if ((rc = dalloc(m, (void**)&m->matt, (size_t)bmax * c.num_kv_heads * 32 * G * (c.head_dim + 2) * 4))) return rc;
      if ((rc = dalloc(m, (void**)&m->mbar, 64))) return rc;
      const size_t ndep = num_tiles(m->qkv_rows) + bmax * c.num_kv_heads + num_tiles(I);
      if ((rc = dalloc(m, (void**)&m->mdep, ndep * 4))) return rc;
      NNZ_CK(cudaMemset(m->mdep, 0, ndep * 4));
      const char* prof = getenv("NNZ_MEGA_PROFILE");
      if (prof && prof[0] == '1') {
        if ((rc = dalloc(m, (void**)&m->mprof, 8 * (2 * (2 + 5 * c.num_layers) + 64 + 5 * 1024)))) return rc;
      }
      if ((rc = dalloc(m, (void**)&m->mlayers, sizeof(MegaLayer) * c.num_layers))) return rc;
      NNZ_CK(cudaMemset(m->mbar, 0, 64));

      std::vector<MegaLayer> ml(c.num_layers);
      for (uint32_t l = 0; l < c.num_layers; ++l) {
        const LayerW& W = m->L[l];
        ml[l] = MegaLayer{W.qkv, W.o, W.gu, W.down, W.attn_norm, W.ffn_norm, W.q_norm, W.k_norm};
      }
      NNZ_CK(cudaMemcpy(m->mlayers, ml.data(), sizeof(MegaLayer) * ml.size(), cudaMemcpyHostToDevice));
    }
  }
  if (m->d1_ok) {
    D1Args& a = m->d1;
    a.g = d1g;
    a.eps = c.eps;
    a.rope_style = c.rope_style;
    a.rope_tab = m->rope_tab;
    a.stream = d1_stream;
    std::vector<uint32_t> cb;
    d1_chunk_bytes(d1g, cb);
    uint32_t* dcb = nullptr;
    if ((rc = dalloc(m, (void**)&dcb, cb.size() * 4))) return rc;
    NNZ_CK(cudaMemcpy(dcb, cb.data(), cb.size() * 4, cudaMemcpyHostToDevice));
    a.chunk_bytes = dcb;
    std::vector<D1Layer> dl(c.num_layers);
    for (uint32_t l = 0; l < c.num_layers; ++l)
      dl[l] = D1Layer{m->L[l].attn_norm, m->L[l].ffn_norm, m->L[l].q_norm, m->L[l].k_norm};
    D1Layer* ddl = nullptr;
    if ((rc = dalloc(m, (void**)&ddl, dl.size() * sizeof(D1Layer)))) return rc;
    NNZ_CK(cudaMemcpy(ddl, dl.data(), dl.size() * sizeof(D1Layer), cudaMemcpyHostToDevice));
    a.layers = ddl;
    a.fnorm = m->fnorm;
    a.emb_w = m->emb_w;
    a.emb_s = m->emb_s;
    a.kc = m->kc;
    a.vc = m->vc;
    a.kv_layer = m->kv_layer;
    if ((rc = dalloc(m, (void**)&a.R, 4 * (size_t)H * 4))) return rc;
    a.Z = a.R + 2 * H;
    NNZ_CK(cudaMemset(a.R, 0, 4 * (size_t)H * 4));
    if ((rc = dalloc(m, (void**)&a.qkv, (size_t)d1g.qkv_rows * 4))) return rc;
    NNZ_CK(cudaMemset(a.qkv, 0, (size_t)d1g.qkv_rows * 4));
    if ((rc = dalloc(m, (void**)&a.h, (size_t)I * 2))) return rc;
    if ((rc = dalloc(m, (void**)&a.att, (size_t)c.num_kv_heads * d1g.S * d1g.G * kD1AttRec * 4))) return rc;
    m->d1_cnt_words = (size_t)2 * c.num_layers * c.num_kv_heads;
    if ((rc = dalloc(m, (void**)&a.cnt, m->d1_cnt_words * 4))) return rc;
    NNZ_CK(cudaMemset(a.cnt, 0, m->d1_cnt_words * 4));
    if ((rc = dalloc(m, (void**)&a.bar, 64))) return rc;
    NNZ_CK(cudaMemset(a.bar, 0, 64));
    a.st = m->state;
    a.seq = m->seq;
    a.seq_len = c.max_context_length;
    a.err = m->err;
    if ((rc = dalloc(m, (void**)&a.tstamp, ((size_t)c.max_context_length + 1) * 8))) return rc;
    const char* prof = getenv("NNZ_D1_PROFILE");
    if (prof && prof[0] == '1') {
      if ((rc = dalloc(m, (void**)&a.prof, (64 + 8 * (size_t)d1g.P + 64) * 8))) return rc;
      NNZ_CK(cudaMemset(a.prof, 0, (64 + 8 * (size_t)d1g.P + 64) * 8));
    }
  }
  NNZ_CK(cudaStreamCreateWithFlags(&m->st, cudaStreamNonBlocking));
  if ((rc = prepare_device(m->device))) return rc;
  if (m->tp > 1) {
    const char* col = getenv("NNZ_TP_COLLECTIVE");
    if (!(col && strcmp(col, "nccl") == 0) && (rc = tp_setup_peers(m))) return rc;
  }
  m->finalized = true;
  return NNZ_OK;
}

int nnz_model_finalize(nnz_model* m) {
  return host_guard([&] { return model_finalize_impl(m); });
}

int nnz_model_free(nnz_model* m) {
  if (!m) return NNZ_OK;
  if (m->device >= 0) cudaSetDevice(m->device);
  if (m->st) cudaStreamSynchronize(m->st);
  for (auto& kv : m->graphs) cudaGraphExecDestroy(kv.second);
  for (auto e : m->events) cudaEventDestroy(e);
  for (void* p : m->ipc_opened) cudaIpcCloseMemHandle(p);
  for (void* p : m->allocs) cudaFree(p);
  if (m->st) cudaStreamDestroy(m->st);
  if (m->comm)
    if (const NcclApi* api = nccl_api(nullptr)) api->comm_destroy(m->comm);
  delete m;
  return NNZ_OK;
}

size_t nnz_model_device_bytes(const nnz_model* m) { return m ? m->dev_bytes : 0; }
uint32_t nnz_model_vocab_shard(const nnz_model* m) { return m ? m->lm_rows : 0; }

static int shard_weights_impl(int fmt, int axis, const void* weight, const uint16_t* scales, const uint16_t* biases,
                      uint32_t M, uint32_t K, uint32_t gs, uint32_t lo, uint32_t hi, void* weight_out,
                      uint16_t* scales_out, uint16_t* biases_out) {
  if (shard_host(fmt, axis, weight, scales, biases, M, K, gs, lo, hi, weight_out, scales_out, biases_out))
    return fail(NNZ_EINVAL, "nnz_shard_weights: invalid arguments");
  return NNZ_OK;
}

int nnz_shard_weights(int fmt, int axis, const void* weight, const uint16_t* scales, const uint16_t* biases,
                      uint32_t M, uint32_t K, uint32_t gs, uint32_t lo, uint32_t hi, void* weight_out,
                      uint16_t* scales_out, uint16_t* biases_out) {
  return host_guard([&] {
    return shard_weights_impl(fmt, axis, weight, scales, biases, M, K, gs, lo, hi, weight_out, scales_out,
                              biases_out);
  });
}

int nnz_sample(float* logits, uint32_t rows, uint32_t n, uint32_t stride, float temperature, uint32_t top_k,
               float top_p, const float* uniforms, uint32_t* tokens_out, void* stream) {
  if (!logits || !uniforms || !tokens_out || rows == 0 || n == 0 || stride < n)
    return fail(NNZ_EINVAL, "nnz_sample: bad arguments");
  DevWs* w;
  int rc = get_ws(&w);
  if (rc) return rc;
  // the argmax slots the kernel also writes land in the shared scratch
  if ((size_t)rows * 2 > w->ws_floats) return fail(NNZ_EINVAL, "nnz_sample: too many rows");
  NNZ_CK(sample_launch(logits, rows, n, stride, temperature, top_k, top_p, uniforms,
                       reinterpret_cast<unsigned long long*>(w->ws), tokens_out, (cudaStream_t)stream));
  return NNZ_OK;
}

int nnz_tp_unique_id(void* out, size_t cap) {
  if (!out || cap < sizeof(ncclUniqueId)) return fail(NNZ_EINVAL, "nnz_tp_unique_id: buffer too small");
  std::string e;
  const NcclApi* api = nccl_api(&e);
  if (!api) return fail(NNZ_ENCCL, e);
  ncclUniqueId id;
  const ncclResult_t r = api->get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r);
  memcpy(out, &id, sizeof(id));
  return (int)sizeof(id);
}

int nnz_tp_init(nnz_model* m, const void* unique_id, size_t len) {
  if (!m || !unique_id || len != sizeof(ncclUniqueId)) return fail(NNZ_EINVAL, "nnz_tp_init: bad arguments");
  if (m->tp == 1) return fail(NNZ_ESTATE, "nnz_tp_init: model was not created with tp_size > 1");
  if (m->finalized || m->comm) return fail(NNZ_ESTATE, "nnz_tp_init: call once, before finalize");
  std::string e;
  const NcclApi* api = nccl_api(&e);
  if (!api) return fail(NNZ_ENCCL, e);
  NNZ_CK(cudaSetDevice(m->device));
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  const ncclResult_t r = api->comm_init_rank(&m->comm, m->tp, id, m->tp_rank);
  if (r != ncclSuccess) {
    m->comm = nullptr;
    return nccl_fail(r);
  }
  return NNZ_OK;
}

int nnz_forward_decode(nnz_model* m, const uint32_t* tokens, const uint32_t* positions,
                       uint32_t batch, float* logits, uint32_t* argmax_out) {
  if (!m || !tokens || !positions || !argmax_out) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (batch == 0 || batch > m->c.max_batch) return fail(NNZ_EINVAL, "batch out of range");
  for (uint32_t r = 0; r < batch; ++r) {
    if (tokens[r] >= m->c.vocab_size) return fail(NNZ_EINVAL, "token id >= vocab_size");
    if (positions[r] >= m->c.max_context_length) return fail(NNZ_EINVAL, "position >= max_context_length");
  }
  NNZ_CK(cudaSetDevice(m->device));
  int rc;
  NNZ_CK(cudaMemcpyAsync(m->state->token, tokens, batch * 4, cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaMemcpyAsync(m->state->pos, positions, batch * 4, cudaMemcpyHostToDevice, m->st));
  if ((rc = set_advance(m, 0))) return rc;
  if ((rc = run_step(m, batch, logits != nullptr))) return rc;
  std::vector<unsigned long long> am(batch);
  NNZ_CK(cudaMemcpyAsync(am.data(), m->state->argmax, batch * 8, cudaMemcpyDeviceToHost, m->st));
  if (logits)
    NNZ_CK(cudaMemcpyAsync(logits, m->logits, (size_t)batch * m->lm_rows * 4,
                           cudaMemcpyDeviceToHost, m->st));
  if ((rc = sync_check(m))) return rc;
  for (uint32_t r = 0; r < batch; ++r) argmax_out[r] = argmax_index(am[r]);
  return NNZ_OK;
}

int nnz_prefill(nnz_model* m, const uint32_t* tokens, uint32_t n, uint32_t* next_token,
                float* last_logits) {
  if (!m || !tokens || !next_token) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (n == 0 || n >= m->c.max_context_length) return fail(NNZ_EINVAL, "prompt length out of range");
  for (uint32_t i = 0; i < n; ++i)
    if (tokens[i] >= m->c.vocab_size) return fail(NNZ_EINVAL, "token id >= vocab_size");
  NNZ_CK(cudaSetDevice(m->device));
  int rc;
  NNZ_CK(cudaMemcpyAsync(m->prompt, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaMemcpyAsync(m->seq, tokens, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
  if ((rc = enqueue_prefill(m, n, last_logits != nullptr))) return rc;
  const int p = (int)n - 1;
  NNZ_CK(cudaMemcpyAsync(m->state->pos, &p, 4, cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaMemcpyAsync(m->state->token, tokens + n - 1, 4, cudaMemcpyHostToDevice, m->st));
  unsigned long long am = 0;
  NNZ_CK(cudaMemcpyAsync(&am, m->state->argmax, 8, cudaMemcpyDeviceToHost, m->st));
  if (last_logits)
    NNZ_CK(cudaMemcpyAsync(last_logits, m->logits, (size_t)m->lm_rows * 4,
                           cudaMemcpyDeviceToHost, m->st));
  if ((rc = sync_check(m))) return rc;
  *next_token = argmax_index(am);
  return NNZ_OK;
}

int nnz_generate(nnz_model* m, const nnz_generate_opts* o, nnz_generate_result* res) {
  if (!m || !o || !res || !o->prompt_ids || !o->output_tokens) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (o->n_prompt == 0 || o->n_prompt >= m->c.max_context_length || o->max_new == 0)
    return fail(NNZ_EINVAL, "prompt length / max_new out of range");
  for (uint32_t i = 0; i < o->n_prompt; ++i)
    if (o->prompt_ids[i] >= m->c.vocab_size) return fail(NNZ_EINVAL, "token id >= vocab_size");
  const bool sample = o->temperature > 0.f;
  if (sample && (!o->uniforms || !(o->top_p > 0.f) || o->top_p > 1.f))
    return fail(NNZ_EINVAL, "sampling needs uniforms[max_new] and 0 < top_p <= 1");
  if (sample && m->tp > 1) return fail(NNZ_EINVAL, "sampling with tensor parallelism is not supported");
  NNZ_CK(cudaSetDevice(m->device));
  const uint32_t n = o->n_prompt;
  // the reference stops when position reaches max_context_length (transformer.zig:3993)
  const uint32_t steps = std::min<uint32_t>(o->max_new, m->c.max_context_length - n);
  int rc;
  while (m->events.size() < (size_t)steps + 2) {
    cudaEvent_t e;
    NNZ_CK(cudaEventCreate(&e));
    m->events.push_back(e);
  }
  NNZ_CK(cudaMemsetAsync(m->state, 0, sizeof(DecodeState), m->st));
  NNZ_CK(cudaMemcpyAsync(m->prompt, o->prompt_ids, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaMemcpyAsync(m->seq, o->prompt_ids, (size_t)n * 4, cudaMemcpyHostToDevice, m->st));
  if (sample)
    NNZ_CK(cudaMemcpyAsync(m->uniforms, o->uniforms, (size_t)std::min<uint32_t>(o->max_new, m->c.max_context_length) * 4,
                           cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaEventRecord(m->events[0], m->st));
  if ((rc = enqueue_prefill(m, n, sample))) return rc;
  if (sample)   // the first generated token comes from the prompt's last logits
    NNZ_CK(sample_launch(m->logits, 1, m->lm_rows, m->lm_rows, o->temperature, o->top_k, o->top_p, m->uniforms,
                         m->state->argmax, nullptr, m->st));
  const int p = (int)n - 1;
  NNZ_CK(cudaMemcpyAsync(m->state->pos, &p, 4, cudaMemcpyHostToDevice, m->st));
  if ((rc = set_advance(m, 1))) return rc;
  NNZ_CK(cudaEventRecord(m->events[1], m->st));
  const bool one_launch = m->d1_ok && !sample;
  if (one_launch) {
    if ((rc = d1_run(m, steps, false))) return rc;
    NNZ_CK(cudaEventRecord(m->events[2], m->st));
  }
  for (uint32_t i = 0; i < steps && !one_launch; ++i) {
    if ((rc = run_step(m, 1, sample))) return rc;
    if (sample && i + 1 < steps)
      NNZ_CK(sample_launch(m->logits, 1, m->lm_rows, m->lm_rows, o->temperature, o->top_k, o->top_p,
                           m->uniforms + i + 1, m->state->argmax, nullptr, m->st));
    NNZ_CK(cudaEventRecord(m->events[2 + i], m->st));
  }
  std::vector<uint32_t> toks(steps);
  NNZ_CK(cudaMemcpyAsync(toks.data(), m->seq + n, (size_t)steps * 4, cudaMemcpyDeviceToHost, m->st));
  std::vector<unsigned long long> stamps(one_launch ? steps + 1 : 0);
  if (one_launch)
    NNZ_CK(cudaMemcpyAsync(stamps.data(), m->d1.tstamp, stamps.size() * 8, cudaMemcpyDeviceToHost, m->st));
  if ((rc = set_advance(m, 0))) return rc;
  if ((rc = sync_check(m))) return rc;
  float ms = 0.f;
  NNZ_CK(cudaEventElapsedTime(&ms, m->events[0], m->events[1]));
  res->prefill_ns = (uint64_t)((double)ms * 1e6);
  uint32_t count = 0;
  uint64_t decode_ns = 0;
  for (uint32_t i = 0; i < steps; ++i) {
    bool eos = false;
    for (uint32_t k = 0; k < o->n_eos; ++k) eos |= (o->eos_ids && toks[i] == o->eos_ids[k]);
    if (eos) break;
    o->output_tokens[count] = toks[i];
    uint64_t ns;
    if (one_launch) {
      // per-token device time from the kernel's %globaltimer stamps; the
      // launch latency (event time minus stamped time) goes to the first token
      ns = stamps[i + 1] - stamps[i];
      if (i == 0) {
        NNZ_CK(cudaEventElapsedTime(&ms, m->events[1], m->events[2]));
        const double total = (double)ms * 1e6, stamped = (double)(stamps[steps] - stamps[0]);
        if (total > stamped) ns += (uint64_t)(total - stamped);
      }
    } else {
      NNZ_CK(cudaEventElapsedTime(&ms, m->events[1 + i], m->events[2 + i]));
      ns = (uint64_t)((double)ms * 1e6);
    }
    if (o->per_token_ns) o->per_token_ns[count] = ns;
    decode_ns += ns;
    ++count;
  }
  res->tokens_generated = count;
  res->decode_ns = decode_ns;
  return NNZ_OK;
}

int nnz_decode_steps(nnz_model* m, const uint32_t* tokens, const uint32_t* positions,
                     uint32_t batch, uint32_t steps, uint32_t* out_tokens, uint64_t* per_step_ns) {
  if (!m || !tokens || !positions || !out_tokens) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (batch == 0 || batch > m->c.max_batch || steps == 0) return fail(NNZ_EINVAL, "batch/steps");
  for (uint32_t r = 0; r < batch; ++r) {
    if (tokens[r] >= m->c.vocab_size) return fail(NNZ_EINVAL, "token id >= vocab_size");
    if (positions[r] + steps > m->c.max_context_length)
      return fail(NNZ_EINVAL, "positions + steps exceed max_context_length");
  }
  NNZ_CK(cudaSetDevice(m->device));
  int rc;
  while (m->events.size() < (size_t)steps + 2) {
    cudaEvent_t e;
    NNZ_CK(cudaEventCreate(&e));
    m->events.push_back(e);
  }
  NNZ_CK(cudaMemcpyAsync(m->state->token, tokens, batch * 4, cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaMemcpyAsync(m->state->pos, positions, batch * 4, cudaMemcpyHostToDevice, m->st));
  if ((rc = set_advance(m, 0))) return rc;
  NNZ_CK(cudaEventRecord(m->events[0], m->st));
  for (uint32_t s = 0; s < steps; ++s) {
    if (s == 1 && (rc = set_advance(m, 1))) return rc;
    if ((rc = run_step(m, batch, false))) return rc;
    NNZ_CK(cudaEventRecord(m->events[1 + s], m->st));
  }
  // tokens consumed at steps 1..steps-1 are recorded in seq at pos+1..; the
  // last step's result is still in the argmax slots.
  const uint32_t L = m->c.max_context_length;
  std::vector<uint32_t> seqv((size_t)batch * L);
  if (steps > 1) NNZ_CK(cudaMemcpyAsync(seqv.data(), m->seq, seqv.size() * 4, cudaMemcpyDeviceToHost, m->st));
  std::vector<unsigned long long> am(batch);
  NNZ_CK(cudaMemcpyAsync(am.data(), m->state->argmax, batch * 8, cudaMemcpyDeviceToHost, m->st));
  if ((rc = set_advance(m, 0))) return rc;
  if ((rc = sync_check(m))) return rc;
  for (uint32_t s = 0; s < steps; ++s)
    for (uint32_t r = 0; r < batch; ++r)
      out_tokens[(size_t)s * batch + r] =
          (s + 1 < steps) ? seqv[(size_t)r * L + positions[r] + 1 + s] : argmax_index(am[r]);
  if (per_step_ns) {
    for (uint32_t s = 0; s < steps; ++s) {
      float ms = 0.f;
      NNZ_CK(cudaEventElapsedTime(&ms, m->events[s], m->events[1 + s]));
      per_step_ns[s] = (uint64_t)((double)ms * 1e6);
    }
  }
  return NNZ_OK;
}

int nnz_model_write_kv(nnz_model* m, uint32_t layer, uint32_t slot, const uint16_t* k,
                       const uint16_t* v, uint32_t len) {
  if (!m || !k || !v) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  const nnz_config& c = m->c;
  if (layer >= c.num_layers || slot >= m->slots || len > c.max_context_length)
    return fail(NNZ_EINVAL, "layer/slot/len out of range");
  NNZ_CK(cudaSetDevice(m->device));
  for (uint32_t h = 0; h < c.num_kv_heads; ++h) {
    const size_t off = m->kv_layer * layer + ((size_t)slot * c.num_kv_heads + h) * c.max_context_length * c.head_dim;
    const size_t n = (size_t)len * c.head_dim;
    NNZ_CK(cudaMemcpyAsync(m->kc + off, k + h * n, n * 2, cudaMemcpyHostToDevice, m->st));
    NNZ_CK(cudaMemcpyAsync(m->vc + off, v + h * n, n * 2, cudaMemcpyHostToDevice, m->st));
  }
  return sync_check(m);
}

int nnz_model_read_kv(nnz_model* m, uint32_t layer, uint32_t slot, uint16_t* k, uint16_t* v,
                      uint32_t len) {
  if (!m || !k || !v) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  const nnz_config& c = m->c;
  if (layer >= c.num_layers || slot >= m->slots || len > c.max_context_length)
    return fail(NNZ_EINVAL, "layer/slot/len out of range");
  NNZ_CK(cudaSetDevice(m->device));
  for (uint32_t h = 0; h < c.num_kv_heads; ++h) {
    const size_t off = m->kv_layer * layer + ((size_t)slot * c.num_kv_heads + h) * c.max_context_length * c.head_dim;
    const size_t n = (size_t)len * c.head_dim;
    NNZ_CK(cudaMemcpyAsync(k + h * n, m->kc + off, n * 2, cudaMemcpyDeviceToHost, m->st));
    NNZ_CK(cudaMemcpyAsync(v + h * n, m->vc + off, n * 2, cudaMemcpyDeviceToHost, m->st));
  }
  return sync_check(m);
}

int nnz_model_layer_step(nnz_model* m, uint32_t layer, float* residual, const uint32_t* positions,
                         uint32_t batch) {
  if (!m || !residual || !positions) return fail(NNZ_EINVAL, "null argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (layer >= m->c.num_layers || batch == 0 || batch > m->c.max_batch)
    return fail(NNZ_EINVAL, "layer/batch out of range");
  for (uint32_t r = 0; r < batch; ++r)
    if (positions[r] >= m->c.max_context_length) return fail(NNZ_EINVAL, "position out of range");
  NNZ_CK(cudaSetDevice(m->device));
  const size_t bytes = (size_t)batch * m->c.hidden_size * 4;
  NNZ_CK(cudaMemcpyAsync(m->residual, residual, bytes, cudaMemcpyHostToDevice, m->st));
  NNZ_CK(cudaMemcpyAsync(m->state->pos, positions, batch * 4, cudaMemcpyHostToDevice, m->st));
  int rc = enqueue_layer(m, layer, batch, m->state->pos, nullptr, false, 0);
  if (rc) return rc;
  NNZ_CK(cudaMemcpyAsync(residual, m->residual, bytes, cudaMemcpyDeviceToHost, m->st));
  return sync_check(m);
}

int nnz_bench_decode_graph(nnz_model* m, uint32_t batch, uint32_t iters, double* us_per_step) {
  if (!m || !us_per_step || iters == 0) return fail(NNZ_EINVAL, "bad argument");
  if (!m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (batch == 0 || batch > m->c.max_batch) return fail(NNZ_EINVAL, "batch");
  NNZ_CK(cudaSetDevice(m->device));
  int rc;
  cudaEvent_t a, b;
  NNZ_CK(cudaEventCreate(&a));
  NNZ_CK(cudaEventCreate(&b));
  if ((rc = set_advance(m, 0))) return rc;
  NNZ_CK(cudaEventRecord(a, m->st));
  for (uint32_t i = 0; i < iters; ++i)
    if ((rc = run_step(m, batch, false))) return rc;
  NNZ_CK(cudaEventRecord(b, m->st));
  rc = sync_check(m);
  float ms = 0.f;
  cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (rc) return rc;
  *us_per_step = (double)ms * 1000.0 / iters;
  return NNZ_OK;
}

// ---- per-kernel entry points ---------------------------------------------

int nnz_dequant(int fmt, int scale_dtype, const void* packed, uint32_t M, uint32_t K, uint32_t gs,
                uint32_t sub, uint32_t sub_index, float* out, void* stream) {
  if (!packed || !out || (fmt != NNZ_Q1 && fmt != NNZ_Q4) || gs == 0 || gs % 32 || K % gs ||
      sub == 0 || sub_index >= sub)
    return fail(NNZ_EINVAL, "nnz_dequant: invalid arguments");
  NNZ_CK(dequant_launch(fmt, fmt == NNZ_Q4 && scale_dtype == NNZ_SCALE_BF16, (const uint8_t*)packed,
                        M, K, gs, sub, sub_index, out, (cudaStream_t)stream));
  return NNZ_OK;
}

static int qmv_common(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M,
                      uint32_t K, uint32_t gs, int pro, const void* x, uint32_t x_stride,
                      const float* nw, float eps, uint32_t batch, void* out, uint32_t out_stride,
                      int epi, float* logits, unsigned long long* am, void* stream) {
  if (!packed || !x || (fmt != NNZ_Q1 && fmt != NNZ_Q4) || batch == 0 || M == 0 || gs == 0 ||
      gs % 32 || gs > 256 || K % gs)
    return fail(NNZ_EINVAL, "qmv: invalid arguments");
  DevWs* w;
  int rc = get_ws(&w);
  if (rc) return rc;
  if (qmv_ws_floats(M, K, gs, fmt, 1, batch, w->num_sms) > w->ws_floats ||
      (size_t)((batch + 7) / 8) * num_tiles(M) > w->n_counters)
    return fail(NNZ_EINVAL, "qmv: problem too large for the shared workspace");
  if (pro == PRO_F16 && !logits && !am && qmvf_applies(fmt, M, K, gs, batch, epi, w->num_sms)) {
    // one activation row: the cluster kernel (no workspace, no split-K pass)
    QmvfArgs f{};
    f.w = (const uint8_t*)packed; f.M = M; f.K = K; f.gs = gs; f.x = (const __half*)x; f.out = out;
    f.epi = epi; f.bf16_round = (fmt == NNZ_Q4 && bf16_round) ? 1u : 0u; f.err = w->err;
    NNZ_CK(qmvf_launch(fmt, fmt == NNZ_Q4 && scale_dtype == NNZ_SCALE_BF16, f, w->num_sms, (cudaStream_t)stream));
    return NNZ_OK;
  }
  QmvLaunch L{fmt, 1, pro, epi, fmt == NNZ_Q4 && scale_dtype == NNZ_SCALE_BF16, 0};
  QmvArgs a{};
  a.w = (const uint8_t*)packed; a.M = M; a.K = K; a.gs = gs;
  a.x = x; a.x_stride = x_stride ? x_stride : K; a.norm_w = nw; a.eps = eps; a.batch = batch;
  a.out = out; a.out_stride = out_stride ? out_stride : M; a.logits = logits; a.logits_stride = M;
  a.argmax = am; a.ws = w->ws; a.counters = w->counters; a.err = w->err;
  a.bf16_round = (fmt == NNZ_Q4 && bf16_round) ? 1u : 0u;
  NNZ_CK(qmv_launch(L, a, w->num_sms, (cudaStream_t)stream));
  return NNZ_OK;
}

static int out_epi(int kind) {
  return kind == NNZ_OUT_F16 ? EPI_F16 : kind == NNZ_OUT_F32 ? EPI_F32 : kind == NNZ_OUT_F32_ADD ? EPI_RESADD : -1;
}

int nnz_qmv(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M, uint32_t K,
            uint32_t gs, const void* x, uint32_t x_stride, uint32_t batch, void* out,
            uint32_t out_stride, int out_kind, void* stream) {
  const int epi = out_epi(out_kind);
  if (epi < 0 || !out) return fail(NNZ_EINVAL, "nnz_qmv: bad out_kind/out");
  return qmv_common(fmt, scale_dtype, bf16_round, packed, M, K, gs, PRO_F16, x, x_stride, nullptr,
                    0.f, batch, out, out_stride, epi, nullptr, nullptr, stream);
}

int nnz_qmv_norm(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M,
                 uint32_t K, uint32_t gs, const float* residual, const float* norm_w, float eps,
                 uint32_t batch, void* out, uint32_t out_stride, int out_kind, void* stream) {
  const int epi = out_epi(out_kind);
  if (epi < 0 || epi == EPI_RESADD || !out || !norm_w)
    return fail(NNZ_EINVAL, "nnz_qmv_norm: bad out_kind/out/norm_w");
  return qmv_common(fmt, scale_dtype, bf16_round, packed, M, K, gs, PRO_NORM, residual, K, norm_w,
                    eps > 0.f ? eps : 1e-6f, batch, out, out_stride, epi, nullptr, nullptr, stream);
}

namespace {
__global__ void argmax_unpack_kernel(const unsigned long long* am, uint32_t* out, uint32_t n) {
  const uint32_t i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) out[i] = argmax_index(am[i]);
}
}  // namespace

int nnz_lm_head_argmax(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M,
                       uint32_t K, uint32_t gs, const float* residual, const float* norm_w,
                       float eps, uint32_t batch, float* logits, uint32_t* argmax_out,
                       void* stream) {
  if (!argmax_out || !norm_w || batch == 0) return fail(NNZ_EINVAL, "nnz_lm_head_argmax: bad arguments");
  DevWs* w;
  int rc = get_ws(&w);
  if (rc) return rc;
  if ((size_t)batch * 8 > w->scratch_bytes) return fail(NNZ_EINVAL, "batch too large");
  auto* am = reinterpret_cast<unsigned long long*>(w->scratch);
  NNZ_CK(cudaMemsetAsync(am, 0, (size_t)batch * 8, (cudaStream_t)stream));
  rc = qmv_common(fmt, scale_dtype, bf16_round, packed, M, K, gs, PRO_NORM, residual, K, norm_w,
                  eps > 0.f ? eps : 1e-6f, batch, nullptr, 0, EPI_LOGITS, logits, am, stream);
  if (rc) return rc;
  argmax_unpack_kernel<<<(batch + 127) / 128, 128, 0, (cudaStream_t)stream>>>(am, argmax_out, batch);
  NNZ_CK(cudaGetLastError());
  return NNZ_OK;
}

int nnz_mlp(int fmt, int scale_dtype, int bf16_round, const void* gate_up, const void* down,
            uint32_t hidden, uint32_t inter, uint32_t gs, const void* x, uint32_t batch,
            float* out, void* stream) {
  if (!gate_up || !down || !x || !out || batch == 0 || (fmt != NNZ_Q1 && fmt != NNZ_Q4) || gs == 0 ||
      gs % 32 || gs > 256 || hidden % gs || inter % gs)
    return fail(NNZ_EINVAL, "nnz_mlp: invalid arguments");
  DevWs* w;
  int rc = get_ws(&w);
  if (rc) return rc;
  if ((size_t)batch * inter * 2 > w->scratch_bytes) return fail(NNZ_EINVAL, "nnz_mlp: batch too large");
  if (qmv_ws_floats(inter, hidden, gs, fmt, 2, batch, w->num_sms) > w->ws_floats ||
      qmv_ws_floats(hidden, inter, gs, fmt, 1, batch, w->num_sms) > w->ws_floats)
    return fail(NNZ_EINVAL, "nnz_mlp: problem too large for the shared workspace");
  const int bf16s = fmt == NNZ_Q4 && scale_dtype == NNZ_SCALE_BF16;
  const uint32_t br = (fmt == NNZ_Q4 && bf16_round) ? 1u : 0u;
  __half* hbuf = reinterpret_cast<__half*>(w->scratch);
  QmvArgs a{};
  a.w = (const uint8_t*)gate_up; a.M = inter; a.K = hidden; a.gs = gs;
  a.x = x; a.x_stride = hidden; a.batch = batch; a.out = hbuf; a.out_stride = inter;
  a.ws = w->ws; a.counters = w->counters; a.err = w->err; a.bf16_round = br;
  NNZ_CK(qmv_launch(QmvLaunch{fmt, 2, PRO_F16, EPI_SILU, bf16s, 0}, a, w->num_sms, (cudaStream_t)stream));
  QmvArgs d{};
  d.w = (const uint8_t*)down; d.M = hidden; d.K = inter; d.gs = gs;
  d.x = hbuf; d.x_stride = inter; d.batch = batch; d.out = out; d.out_stride = hidden;
  d.ws = w->ws; d.counters = w->counters; d.err = w->err; d.bf16_round = br;
  NNZ_CK(qmv_launch(QmvLaunch{fmt, 1, PRO_F16, EPI_F32, bf16s, 0}, d, w->num_sms, (cudaStream_t)stream));
  return NNZ_OK;
}

int nnz_prefill_gemm(int fmt, int scale_dtype, const void* w, const uint16_t* scales,
                     const uint16_t* biases, uint32_t M, uint32_t K, uint32_t N, uint32_t gs,
                     const void* x, void* out, int out_kind, void* stream) {
  if (!w || !scales || !x || !out || (fmt == NNZ_Q4 && !biases) ||
      (out_kind != NNZ_OUT_F16 && out_kind != NNZ_OUT_F32_ADD))
    return fail(NNZ_EINVAL, "nnz_prefill_gemm: bad arguments");
  int dev = 0;
  NNZ_CK(cudaGetDevice(&dev));
  GemmArgs g{};
  g.M = M; g.K = K; g.N = N; g.fmt = fmt; g.gs = (int)gs;
  g.bf16s = fmt == NNZ_Q4 && scale_dtype == NNZ_SCALE_BF16; g.bf16r = 0;
  g.w = (const uint8_t*)w; g.s = scales; g.b = biases;
  g.epi = out_kind == NNZ_OUT_F16 ? GEPI_F16 : GEPI_RESADD;
  g.out = out; g.ldo = N; g.err = nullptr;
  DevWs* ws;
  int rc = get_ws(&ws);
  if (rc) return rc;
  g.err = ws->err;
  NNZ_CK(gemm_launch(g, (const __half*)x, (cudaStream_t)stream));
  return NNZ_OK;
}

int nnz_attn_decode(const void* qkv, const float* q_norm, const float* k_norm, void* k_cache,
                    void* v_cache, uint32_t max_ctx, const int32_t* positions, uint32_t rows,
                    uint32_t n_q, uint32_t n_kv, uint32_t head_dim, float eps, float theta,
                    int rope_style, uint32_t splits, void* out, void* stream) {
  if (!qkv || !q_norm || !k_norm || !k_cache || !v_cache || !positions || !out || rows == 0)
    return fail(NNZ_EINVAL, "nnz_attn_decode: null argument");
  DevWs* w;
  int rc = get_ws(&w);
  if (rc) return rc;
  AttnArgs a{};
  a.qkv = (const __half*)qkv; a.qkv_stride = (n_q + 2 * n_kv) * head_dim;
  a.q_norm = q_norm; a.k_norm = k_norm; a.kc = (__half*)k_cache; a.vc = (__half*)v_cache;
  a.max_ctx = max_ctx; a.pos = positions; a.slot = nullptr; a.rows = rows; a.n_q = n_q; a.n_kv = n_kv;
  a.eps = eps > 0.f ? eps : 1e-6f; a.theta = theta; a.rope_style = rope_style; a.write_kv = 1;
  a.splits = splits ? splits : std::min(16u, std::max(1u, (uint32_t)w->num_sms / std::max(1u, n_kv * rows)));
  a.out = (__half*)out; a.out_stride = n_q * head_dim; a.ws = w->ws; a.counters = w->counters; a.err = w->err;
  if (attn_ws_floats(rows, n_q, n_kv, a.splits, (int)head_dim, max_ctx) > w->ws_floats ||
      (size_t)rows * n_kv > w->n_counters)
    return fail(NNZ_EINVAL, "nnz_attn_decode: problem too large for the shared workspace");
  NNZ_CK(attn_decode_launch(a, (int)head_dim, 0, (cudaStream_t)stream));
  return NNZ_OK;
}

// Waits for `stream`, then reports (and clears) the device error flags that
// the per-kernel entry points' launches on the current device raised: a
// bounded wait that gave up (NNZ_ETIMEDOUT) or an out-of-range position /
// token (NNZ_EDEVICE).  Allocates nothing.
int nnz_stream_check(void* stream) {
  return host_guard([&]() -> int {
    NNZ_CK(cudaStreamSynchronize(static_cast<cudaStream_t>(stream)));
    int dev = 0;
    NNZ_CK(cudaGetDevice(&dev));
    int flags = 0;
    {
      std::lock_guard<std::mutex> lk(g_ws_mu);
      auto it = g_ws.find(dev);
      if (it != g_ws.end() && it->second.err) {
        NNZ_CK(cudaMemcpy(&flags, it->second.err, sizeof(int), cudaMemcpyDeviceToHost));
        if (flags) NNZ_CK(cudaMemset(it->second.err, 0, sizeof(int)));
      }
    }
    int na = 0;
    const int rc = noalloc_take_error(dev, &na);
    if (rc) return rc;
    flags |= na;
    if (flags)
      return fail(flags & (ERR_MBAR_TIMEOUT | ERR_SPIN_TIMEOUT) ? NNZ_ETIMEDOUT : NNZ_EDEVICE, err_text(flags));
    return NNZ_OK;
  });
}

// Development aid (not part of the documented ABI): clock64() stamps of CTA
// (0,0,0) of the last GEMM launched with NNZ_GEMM_PROFILE=1.
int nnz_debug_gemm_profile(uint64_t* out) {
  if (!out) return fail(NNZ_EINVAL, "null");
  NNZ_CK(gemm_debug_profile(reinterpret_cast<unsigned long long*>(out)));
  return NNZ_OK;
}

// Development aid (not part of the documented ABI), for the failure tests:
// the peer-memory all-reduce kernel on the current device as rank 0 of a
// 2-rank group whose "peer" is a local stand-in that never arrives, with a
// wait limit of `spin_limit` polls.  The bounded wait must give up: returns
// NNZ_ETIMEDOUT with the raised device flags in *flags_out, and the CUDA
// context stays usable.  Nothing waits on another GPU.
int nnz_debug_tp_wait_timeout(uint32_t spin_limit, int* flags_out) {
  if (!flags_out) return fail(NNZ_EINVAL, "null argument");
  return host_guard([&]() -> int {
    const size_t n = 4096;
    const size_t nflag = tp_allreduce_flag_words(n, 2);
    float *res = nullptr, *part = nullptr, *slots = nullptr;
    uint32_t* flags = nullptr;
    int* err = nullptr;
    void* tabs = nullptr;
    auto cleanup = [&] {
      cudaFree(res); cudaFree(part); cudaFree(slots); cudaFree(flags); cudaFree(err); cudaFree(tabs);
    };
    if (cudaMalloc(&res, n * 4) || cudaMalloc(&part, n * 4) || cudaMalloc(&slots, 2 * 2 * n * 4) ||
        cudaMalloc(&flags, 2 * nflag * 4) || cudaMalloc(&err, 4) || cudaMalloc(&tabs, 4 * sizeof(void*))) {
      cudaGetLastError();
      cleanup();
      return fail(NNZ_ENOMEM, "nnz_debug_tp_wait_timeout: allocation failed");
    }
    cudaMemset(res, 0, n * 4);
    cudaMemset(part, 0, n * 4);
    cudaMemset(flags, 0, 2 * nflag * 4);
    cudaMemset(err, 0, 4);
    // slot arrays and flag arrays of "GPU 0" (this one) and the stand-in "GPU 1"
    float* slot_tab[2] = {slots, slots + 2 * n};
    uint32_t* flag_tab[2] = {flags, flags + nflag};
    cudaMemcpy(tabs, slot_tab, sizeof(slot_tab), cudaMemcpyHostToDevice);
    cudaMemcpy(static_cast<char*>(tabs) + sizeof(slot_tab), flag_tab, sizeof(flag_tab), cudaMemcpyHostToDevice);
    cudaError_t e = tp_allreduce_launch(res, part, static_cast<float* const*>(tabs), flags,
                                        reinterpret_cast<uint32_t* const*>(static_cast<char*>(tabs) + sizeof(slot_tab)),
                                        n, 0, 2, err, nullptr, spin_limit);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    int flags_host = 0;
    if (e == cudaSuccess) e = cudaMemcpy(&flags_host, err, 4, cudaMemcpyDeviceToHost);
    cleanup();
    if (e != cudaSuccess) return fail(NNZ_ECUDA, std::string("nnz_debug_tp_wait_timeout: ") + cudaGetErrorString(e));
    *flags_out = flags_host;
    if (flags_host & (ERR_SPIN_TIMEOUT | ERR_MBAR_TIMEOUT)) return fail(NNZ_ETIMEDOUT, err_text(flags_host));
    return NNZ_OK;
  });
}

// Development aid (not part of the documented ABI): which kernel runs a
// batch-1 decode step: 1 = single-row kernel (decode1.cu), 2 = persistent
// multi-row kernel (mega.cu), 0 = captured multi-kernel graph.
int nnz_debug_decode_path(nnz_model* m) {
  if (!m || !m->finalized) return fail(NNZ_ESTATE, "model not finalized");
  if (m->d1_ok) return 1;
  return mega_plan_for(m, 1) ? 2 : 0;
}

// Development aid (not part of the documented ABI): %globaltimer stamps of
// the single-row decode kernel's CTA 0 (layer 1 phases of the first token of
// the last launch) when the model was finalized with NNZ_D1_PROFILE=1.
int nnz_debug_decode1_profile(nnz_model* m, uint64_t* out, uint32_t n) {
  if (!m || !out || !m->d1_ok || !m->d1.prof) return fail(NNZ_ESTATE, "profiling not enabled");
  NNZ_CK(cudaStreamSynchronize(m->st));
  NNZ_CK(cudaMemcpy(out, m->d1.prof, 8 * std::min<uint32_t>(n, 64 + 8 * m->d1.g.P + 64), cudaMemcpyDeviceToHost));
  return NNZ_OK;
}

// Development aid (not part of the documented ABI): per-phase timestamps of
// the last persistent-kernel launch when the model was finalized with
// NNZ_MEGA_PROFILE=1; out receives 2 * n entries (phase end, barrier exit).
int nnz_debug_mega_profile(nnz_model* m, uint64_t* out, uint32_t n, uint32_t* grid) {
  if (!m || !out || !m->mprof) return fail(NNZ_ESTATE, "profiling not enabled");
  NNZ_CK(cudaStreamSynchronize(m->st));
  const uint32_t nph = 2 + 5 * m->c.num_layers;
  NNZ_CK(cudaMemcpy(out, m->mprof, 8 * (2 * std::min(n, nph) + (n > nph ? 64 + 5 * 1024 : 0)), cudaMemcpyDeviceToHost));
  if (grid) {
    auto it = m->mplans.find(1);
    *grid = it != m->mplans.end() ? it->second.grid : 0;
  }
  return NNZ_OK;
}

}  // extern "C"
