/*
 * nnz_b200.h -- C ABI of the B200-native quantized Qwen3 (Bonsai) hot path.
 *
 * This library replaces the Metal backend + dispatch layer of the nnzap
 * `nnmetal` engine for the decode / prefill hot path.  Every entry point is
 * plain C: integers, sizes and pointers, no C++ or torch types, no
 * exceptions.  All functions return 0 (NNZ_OK) or a negative NNZ_E* code;
 * nnz_last_error() returns a thread-local message for the last failure.
 *
 * Citations name files of the nnzap reference tree (path:line).
 */
#ifndef NNZ_B200_H_
#define NNZ_B200_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes --------------------------------------------------- */
enum {
  NNZ_OK = 0,
  NNZ_EINVAL = -1,     /* bad argument / shape (reference: std.debug.assert) */
  NNZ_ECUDA = -2,      /* CUDA runtime error (MetalNotAvailable & co.)        */
  NNZ_ENOMEM = -3,     /* device allocation failed (MetalBufferAllocFailed)   */
  NNZ_ETIMEDOUT = -4,  /* a bounded device or host wait gave up               */
  NNZ_ENOTFOUND = -5,  /* tensor missing at finalize (TensorNotFound)          */
  NNZ_ESTATE = -6,     /* call order violated (e.g. decode before finalize)   */
  NNZ_EDEVICE = -7,    /* a kernel raised a device error flag                 */
  NNZ_ENCCL = -8,      /* NCCL failure (tensor-parallel path)                 */
  NNZ_ERANGE = -9      /* caller's output buffer too small (OutputBufferTooSmall) */
};

/* ---- enums ------------------------------------------------------------ */
/* Quantization format: transformer.zig:35-53 QuantFormat {q1_0, q4_mlx}. */
enum { NNZ_Q1 = 0, NNZ_Q4 = 1 };
/* RoPE pairing: engine consecutive pairs (transformer.metal:1535-1549) or
 * MLX/HF half split (reference/mlx_q4_layer0.py:114-136). */
enum { NNZ_ROPE_PAIRWISE = 0, NNZ_ROPE_HALF_SPLIT = 1 };
/* 16-bit scale/bias encoding (Q4): fp16, or raw BF16 (model.zig:1177-1220). */
enum { NNZ_SCALE_F16 = 0, NNZ_SCALE_BF16 = 1 };
/* Tensor dtypes accepted by nnz_model_load_tensor (safetensors.zig:46). */
enum { NNZ_DT_U8 = 0, NNZ_DT_U32 = 1, NNZ_DT_F16 = 2, NNZ_DT_BF16 = 3, NNZ_DT_F32 = 4 };
/* Output kinds of nnz_qmv. */
enum { NNZ_OUT_F16 = 0, NNZ_OUT_F32 = 1, NNZ_OUT_F32_ADD = 2 };

/* Model description.  Mirrors TransformerDesc / TransformerConfig
 * (transformer.zig:62-81, :91-276); runtime instead of comptime. */
typedef struct nnz_config {
  uint32_t vocab_size;
  uint32_t hidden_size;
  uint32_t intermediate_size;
  uint32_t num_layers;
  uint32_t num_query_heads;
  uint32_t num_kv_heads;
  uint32_t head_dim;              /* 64 or 128 */
  uint32_t max_context_length;
  uint32_t max_prefill_length;
  uint32_t max_batch;             /* decode rows (1 for the reference engine) */
  float rope_theta;
  float eps;                      /* RMSNorm epsilon, 1e-6 in the reference */
  int32_t quant_format;           /* NNZ_Q1 | NNZ_Q4 */
  int32_t group_size;             /* 128 (Q1) / 64 (Q4); multiple of 32 */
  int32_t scale_dtype;            /* Q4: NNZ_SCALE_F16 (spec) | NNZ_SCALE_BF16 (engine) */
  int32_t bf16_faithful;          /* Q4: truncate outputs to BF16 like the engine */
  int32_t rope_style;             /* NNZ_ROPE_* */
  int32_t tie_word_embeddings;
  int32_t q1_scales_are_mlx;      /* Q1: halve scales at load (model.zig:944-959) */
  /* Tensor parallelism (batched decode, one process per GPU): with
   * tp_size > 1 this model holds rank tp_rank's shard -- query/kv heads,
   * gate/up rows and the LM head's vocabulary rows split tp_size ways,
   * o/down split along their input columns -- and the full-size tensors
   * passed to nnz_model_load_tensor are sliced at finalize.  The dims
   * above stay the full model's.  Call nnz_tp_init before finalize. */
  int32_t tp_rank;
  int32_t tp_size;                /* 0 or 1 = off */
} nnz_config;

typedef struct nnz_model nnz_model;

/* GenerateOpts / GenerateResult (transformer.zig:3663-3690).  Greedy only. */
typedef struct nnz_generate_opts {
  const uint32_t* prompt_ids;
  uint32_t n_prompt;
  const uint32_t* eos_ids;
  uint32_t n_eos;
  uint32_t* output_tokens;       /* capacity max_new */
  uint32_t max_new;
  uint64_t* per_token_ns;        /* optional [max_new]: GPU time per decode step */
  /* SamplingParams (transformer.zig:3655-3660): temperature 0 = greedy.
   * With temperature > 0 every generated token is drawn on the device
   * (sampleToken, transformer.zig:3833-3869: temperature, top-k, top-p,
   * inverse CDF) with uniforms[i] in [0, 1) for the i-th token, drawn by
   * the host's generator (the reference's DefaultPrng(seed)). */
  float temperature;
  uint32_t top_k;                /* 0 = off */
  float top_p;                   /* 1 = off */
  const float* uniforms;         /* [max_new], required when temperature > 0 */
} nnz_generate_opts;

typedef struct nnz_generate_result {
  uint32_t tokens_generated;
  uint64_t prefill_ns;
  uint64_t decode_ns;
} nnz_generate_result;

/* ---- library -------------------------------------------------------- */
const char* nnz_last_error(void);
int nnz_version(void);
/* Device count visible to the CUDA runtime (0 without a GPU). */
int nnz_device_count(void);

/* ---- model: replaces Model(Config) of model.zig + Device.init -------- */
/* Device.init + Model.init (metal.zig:959, model.zig:123): allocates
 * nothing yet; buffers are sized at nnz_model_finalize. */
int nnz_model_create(int device, const nnz_config* cfg, nnz_model** out);
/* loadWeights (model.zig:196-242, :571-1026): one tensor by its checkpoint
 * name ("model.layers.{i}.self_attn.q_proj.weight", ".scales", ".biases",
 * "model.embed_tokens.*", "model.norm.weight", "lm_head.*", norm weights).
 * The bytes are copied; conversions follow the reference loader. */
int nnz_model_load_tensor(nnz_model* m, const char* name, int dtype, const void* data,
                          size_t bytes);
/* Packs the loaded tensors into the device layout, allocates the KV cache
 * and activation buffers, and releases the host copies. */
int nnz_model_finalize(nnz_model* m);
int nnz_model_free(nnz_model* m);
/* Bytes of device memory held by the model (weights + KV + scratch). */
size_t nnz_model_device_bytes(const nnz_model* m);
/* Vocabulary rows of this rank's LM-head shard (vocab_size without TP). */
uint32_t nnz_model_vocab_shard(const nnz_model* m);

/* forwardDecode (transformer.zig:2566) + host argmax (:3694): one token per
 * row at the given positions, `batch` rows (row r uses KV-cache slot r).
 * logits (optional, host, [batch][vocab] f32; with tensor parallelism
 * [batch][nnz_model_vocab_shard] of this rank's rows) and argmax_out
 * ([batch], global token ids on every rank). */
int nnz_forward_decode(nnz_model* m, const uint32_t* tokens, const uint32_t* positions,
                       uint32_t batch, float* logits, uint32_t* argmax_out);
/* Prompt prefill into slot 0 at positions 0..n-1 (replaces chunkedPrefill,
 * transformer.zig:4032-4068); returns the greedy next token and optionally
 * the last position's logits. */
int nnz_prefill(nnz_model* m, const uint32_t* tokens, uint32_t n, uint32_t* next_token,
                float* last_logits);
/* generate (transformer.zig:3942-4027), greedy: prefill then one CUDA-graph
 * replay per token; stops at the first EOS id like the reference. */
int nnz_generate(nnz_model* m, const nnz_generate_opts* opts, nnz_generate_result* res);
/* Batched greedy decode of `batch` sequences for `steps` tokens, starting
 * from tokens[] at positions[] (each row's slot must hold its KV history).
 * out_tokens [steps][batch]; per_step_ns optional [steps]. */
int nnz_decode_steps(nnz_model* m, const uint32_t* tokens, const uint32_t* positions,
                     uint32_t batch, uint32_t steps, uint32_t* out_tokens,
                     uint64_t* per_step_ns);
/* Fill KV-cache slot `slot` of layer `layer`, positions [0, len), from host
 * fp16 arrays laid out [kv_head][len][head_dim]. */
int nnz_model_write_kv(nnz_model* m, uint32_t layer, uint32_t slot, const uint16_t* k,
                       const uint16_t* v, uint32_t len);
/* Read back the same region (tests). */
int nnz_model_read_kv(nnz_model* m, uint32_t layer, uint32_t slot, uint16_t* k, uint16_t* v,
                      uint32_t len);
/* One decoder layer decode step on the model's state (benchmark configuration 2):
 * residual (host f32 [batch][hidden]) is updated in place, `positions` give
 * each row's position; row r uses KV slot r. */
int nnz_model_layer_step(nnz_model* m, uint32_t layer, float* residual,
                         const uint32_t* positions, uint32_t batch);
/* Average device time of `iters` back-to-back replays of the b=1 decode
 * graph (no host work between), in microseconds; for benchmarks. */
int nnz_bench_decode_graph(nnz_model* m, uint32_t batch, uint32_t iters, double* us_per_step);

/* ---- weight packing (host, no GPU needed) --------------------------- */
/* Bytes of the tile-packed form of an M x K matrix (sub interleaved). */
size_t nnz_packed_bytes(int fmt, uint32_t M, uint32_t K, uint32_t gs, uint32_t sub);
/* Reference flat layout -> tile layout (metal.zig:235-469 formats).
 * weight: Q1 bits (M*K/8 B) or Q4 words (M*K/2 B); scales/biases u16. */
int nnz_pack_weights(int fmt, const void* weight, const uint16_t* scales, const uint16_t* biases,
                     uint32_t M, uint32_t K, uint32_t gs, uint32_t sub, uint32_t sub_index,
                     void* packed_out);
/* Exact inverse of nnz_pack_weights. */
int nnz_unpack_weights(int fmt, const void* packed, uint32_t M, uint32_t K, uint32_t gs,
                       uint32_t sub, uint32_t sub_index, void* weight, uint16_t* scales,
                       uint16_t* biases);

/* Tensor-parallel shard of a flat [M][K] weight (reference layout): rows
 * [lo, hi) (axis 0) or columns [lo, hi) (axis 1; multiples of gs).  Host
 * memory only; outputs are flat in the shard's shape.  Q1: biases NULL. */
int nnz_shard_weights(int fmt, int axis, const void* weight, const uint16_t* scales,
                      const uint16_t* biases, uint32_t M, uint32_t K, uint32_t gs, uint32_t lo,
                      uint32_t hi, void* weight_out, uint16_t* scales_out, uint16_t* biases_out);

/* sampleToken (transformer.zig:3833-3869) on device logits: rows x n f32
 * (row stride `stride`, modified in place like the reference), one uniform
 * draw per row (device pointer); tokens_out (device, [rows]).  temperature
 * > 0, 0 < top_p <= 1, top_k 0 = off. */
int nnz_sample(float* logits, uint32_t rows, uint32_t n, uint32_t stride, float temperature, uint32_t top_k,
               float top_p, const float* uniforms, uint32_t* tokens_out, void* stream);

/* ---- tensor parallelism (NCCL over NVLink; replaces nothing in the
 * reference, which is single-device) ------------------------------------ */
/* Rank 0 creates the group id (NCCL unique id, copied into out[0..cap));
 * returns its size in bytes (> 0) or a negative error. */
int nnz_tp_unique_id(void* out, size_t cap);
/* Joins the group (blocking until all tp_size ranks joined); the model
 * must have been created with tp_size > 1 and not be finalized.  Decode
 * then all-reduces the residual after o_proj and down_proj (sum) and the
 * argmax slots after the LM head (max), inside the same CUDA graph. */
int nnz_tp_init(nnz_model* m, const void* unique_id, size_t len);

/* ---- per-kernel entry points on device pointers --------------------- */
/* All asynchronous on `stream` (a cudaStream_t, NULL = default stream).
 * They share a per-device workspace allocated on first use, except
 * nnz_qmv_noalloc, which allocates nothing (see its comment).  Errors the
 * kernels detect on the device are reported by nnz_stream_check. */

/* Waits for `stream` and returns the device-side errors raised since the
 * last check by the per-kernel entry points' launches on the current
 * device: NNZ_ETIMEDOUT when a bounded wait inside a kernel gave up (its
 * output is then invalid), NNZ_EDEVICE for an out-of-range position or
 * token id; the flags are cleared.  Allocates nothing.  No counterpart in
 * the reference (its kernels have no device-side error reporting: Metal
 * command buffers, nnmetal/src/metal.zig:1325-1352). */
int nnz_stream_check(void* stream);

/* nnz_qmv without any device allocation, for callers that cannot allocate
 * device memory once running (a host that gave the whole device memory
 * budget to its own pool at start-up, or work issued while another thread
 * captures a CUDA graph).  No counterpart in the reference: it exists only
 * for such callers.  Same arguments, results and tolerance as nnz_qmv, but
 * the split-K scratch is a fixed array compiled into the library (8 MiB of
 * partial sums + 64 KiB of counters, held on every GPU that loads the
 * library until exit); problems that need more return NNZ_EINVAL.  All calls
 * share that array: calls that overlap on the GPU race, so issue them on one
 * stream.  The first call on a device does one-time set-up (device
 * addresses of the array, kernel attributes); make it before any stream
 * capture starts on that device.  A bounded wait that gives up inside the
 * kernel is reported by nnz_stream_check, not by the call itself. */
int nnz_qmv_noalloc(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M,
                    uint32_t K, uint32_t gs, const void* x, uint32_t x_stride, uint32_t batch,
                    void* out, uint32_t out_stride, int out_kind, void* stream);

/* Dequantize a packed matrix to f32 [M][K] (bit-exact weight check).
 * Reference dequant: transformer_test.zig:286-321 (Q1), model.zig:969-1026 (Q4). */
int nnz_dequant(int fmt, int scale_dtype, const void* packed, uint32_t M, uint32_t K, uint32_t gs,
                uint32_t sub, uint32_t sub_index, float* out, void* stream);
/* y[b][row] = sum_k x[b][k] W[row][k] for b < batch.  x fp16 [batch][x_stride].
 * out_kind NNZ_OUT_F16 (fp16 y), NNZ_OUT_F32, NNZ_OUT_F32_ADD (y += into f32).
 * Replaces qmv_spec_f16io / _f16in / _f16io_resadd
 * (qmv_specialized.metal:55,217,597; q4mv_bf16_specialized.metal:93,185,394). */
int nnz_qmv(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M, uint32_t K,
            uint32_t gs, const void* x, uint32_t x_stride, uint32_t batch, void* out,
            uint32_t out_stride, int out_kind, void* stream);
/* Same with the fused RMSNorm prologue over an f32 residual [batch][K]
 * (qmv_spec_fused_norm_f16io, qmv_specialized.metal:1290). */
int nnz_qmv_norm(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M,
                 uint32_t K, uint32_t gs, const float* residual, const float* norm_w, float eps,
                 uint32_t batch, void* out, uint32_t out_stride, int out_kind, void* stream);
/* LM head + greedy argmax: optional f32 logits [batch][M], argmax_out
 * device u32 [batch] (qmv_spec_f16in + transformer.zig:3694-3707). */
int nnz_lm_head_argmax(int fmt, int scale_dtype, int bf16_round, const void* packed, uint32_t M,
                       uint32_t K, uint32_t gs, const float* residual, const float* norm_w,
                       float eps, uint32_t batch, float* logits, uint32_t* argmax_out,
                       void* stream);
/* Fused MLP block (benchmark configuration 1): out_f32[b] = down(SiLU(gate x) * up x).
 * gate_up is packed with sub = 2 (gate = sub 0, up = sub 1); x fp16
 * [batch][K]; h_scratch fp16 [batch][M_inter] may be NULL (workspace).
 * Replaces qmv_spec_fused_pair_silu_f16io + qmv_spec_mg_f16io_resadd
 * (qmv_specialized.metal:955,760). */
int nnz_mlp(int fmt, int scale_dtype, int bf16_round, const void* gate_up, const void* down,
            uint32_t hidden, uint32_t inter, uint32_t gs, const void* x, uint32_t batch,
            float* out, void* stream);
/* Prefill GEMM on the tcgen05 tensor cores: out[m][n] (+)= sum_k x[m][k] *
 * W[n][k] for m < M, n < N, with W in the reference's flat layout (Q1 bits +
 * fp16 scales, or Q4 words + scales + biases; metal.zig:235-469) and x fp16
 * [M][K] (16-byte aligned, K % 64 == 0, gs >= 64).  out_kind NNZ_OUT_F16 or
 * NNZ_OUT_F32_ADD (row stride N).  No reference counterpart: the reference
 * prefills token by token (transformer.zig:4032-4068). */
int nnz_prefill_gemm(int fmt, int scale_dtype, const void* w, const uint16_t* scales,
                     const uint16_t* biases, uint32_t M, uint32_t K, uint32_t N, uint32_t gs,
                     const void* x, void* out, int out_kind, void* stream);

/* GQA decode attention with fused QK-norm + RoPE + KV write
 * (gqa_attention_fused_f16io_tg, transformer.metal:1467-1695).
 * qkv fp16 [rows][(n_q + 2 n_kv) hd]; caches fp16 [slots][n_kv][max_ctx][hd];
 * positions device int32 [rows]; row r uses slot r; out fp16 [rows][n_q hd];
 * splits = CTAs per (kv head, row), 0 = automatic. */
int nnz_attn_decode(const void* qkv, const float* q_norm, const float* k_norm, void* k_cache,
                    void* v_cache, uint32_t max_ctx, const int32_t* positions, uint32_t rows,
                    uint32_t n_q, uint32_t n_kv, uint32_t head_dim, float eps, float theta,
                    int rope_style, uint32_t splits, void* out, void* stream);

/* ---- tokenizer: replaces Tokenizer of nnmetal/src/tokenizer.zig ------ */
/* Byte-level BPE over a HuggingFace tokenizer.json (Qwen3 format).  Host
 * code only (no device calls).  A tokenizer is immutable after creation:
 * encode / decode / chat-template calls may run concurrently on one handle.
 * Errors return NNZ_EINVAL (or NNZ_ERANGE / NNZ_ENOTFOUND where stated) and
 * nnz_last_error() starts with the reference's error name (InvalidJson,
 * MissingField, InvalidVocabEntry, VocabTooLarge, InvalidMergeEntry,
 * InputTooLong, ChunkTooLong, UnknownByte, UnknownTokenId, ...).
 * Limits as in the reference (tokenizer.zig:28-46): token ids < 200000,
 * <= 200000 merges, <= 256 special tokens (later ones are ignored), encode
 * input <= 1 MiB, pre-tokenized chunks <= 512 bytes, files <= 32 MiB. */
typedef struct nnz_tokenizer nnz_tokenizer;

typedef struct nnz_tokenizer_info {
  uint32_t vocab_size;          /* one past the highest id seen */
  uint32_t special_token_count;
  uint32_t eos_token_id;        /* "<|endoftext|>", 0 if absent */
  uint32_t im_start_token_id;   /* "<|im_start|>", 0 if absent  */
  uint32_t im_end_token_id;     /* "<|im_end|>", 0 if absent    */
  uint32_t merge_count;         /* entries of model.merges      */
} nnz_tokenizer_info;

/* Tokenizer.initFromJson (tokenizer.zig:195-229): parse an in-memory
 * tokenizer.json (model.vocab, model.merges in "a b" or ["a", "b"] form,
 * added_tokens). */
int nnz_tokenizer_from_json(const char* json, size_t len, nnz_tokenizer** out);
/* Tokenizer.init (tokenizer.zig:164-193): read and parse a file
 * (NNZ_ENOTFOUND if it cannot be opened). */
int nnz_tokenizer_from_file(const char* path, nnz_tokenizer** out);
/* Tokenizer.deinit (tokenizer.zig:232-242). */
int nnz_tokenizer_free(nnz_tokenizer* tok);
/* The fields Tokenizer exposes (vocab_size, special_token_count,
 * eos/im_start/im_end ids; tokenizer.zig:124-156). */
int nnz_tokenizer_get_info(const nnz_tokenizer* tok, nnz_tokenizer_info* info);
/* Tokenizer.encode (tokenizer.zig:247-289): special tokens matched longest
 * first, other text pre-tokenized and BPE-merged per chunk.  Writes at most
 * cap ids (NNZ_ERANGE when they do not fit; len + 1 always suffices). */
int nnz_tokenizer_encode(const nnz_tokenizer* tok, const char* text, size_t len, uint32_t* ids,
                         uint32_t cap, uint32_t* n_out);
/* Tokenizer.decode (tokenizer.zig:293-324): raw bytes of the ids (NNZ_ERANGE
 * when the next token's vocabulary string is longer than the room left). */
int nnz_tokenizer_decode(const nnz_tokenizer* tok, const uint32_t* ids, uint32_t n, char* out,
                         size_t cap, size_t* n_out);
/* Tokenizer.applyChatTemplate (tokenizer.zig:330-370):
 * <|im_start|>user\n{prompt}<|im_end|>\n<|im_start|>assistant\n
 * (len + 32 ids always suffice). */
int nnz_tokenizer_chat_template(const nnz_tokenizer* tok, const char* prompt, size_t len,
                                uint32_t* ids, uint32_t cap, uint32_t* n_out);
/* Tokenizer.bpeMerge (tokenizer.zig:761-800): greedy lowest-rank merging of
 * ids[0..n) in place; *n_out = the merged length. */
int nnz_tokenizer_bpe_merge(const nnz_tokenizer* tok, uint32_t* ids, uint32_t n, uint32_t* n_out);
/* id_to_vocab[id] (the token's vocabulary string, byte-level form);
 * NNZ_ERANGE if longer than cap, UnknownTokenId if unused. */
int nnz_tokenizer_token(const nnz_tokenizer* tok, uint32_t id, char* out, size_t cap, size_t* n_out);
/* decodeTokenToBytes (tokenizer.zig:1066-1108): raw bytes of one token
 * string in byte-level form (len bytes; cap >= len always suffices). */
int nnz_token_to_bytes(const char* token, size_t len, char* out, size_t cap, size_t* n_out);
/* nextPretokenChunk (tokenizer.zig:936-994): byte length of the first
 * pre-tokenizer chunk of text[0..len) (0 when len == 0). */
uint32_t nnz_pretoken_chunk(const char* text, size_t len);

/* ---- safetensors: replaces SafetensorsFile of nnmetal/src/safetensors.zig */
/* Host code only.  A reader memory-maps one file and describes its tensors;
 * the descriptors' data pointers stay valid until nnz_safetensors_close.
 * Model.loadWeights (model.zig:196-242) is then, per file:
 *   for i < nnz_safetensors_count(f): nnz_safetensors_tensor(f, i, &d);
 *                                     nnz_model_load_tensor(m, d.name, d.dtype, d.data, d.nbytes);
 * and nnz_model_finalize(m) once all files are read (load_tensor copies).
 * Same format, limits and error names as the reference (InvalidHeader,
 * InvalidJson, TooManyTensors, InvalidTensorEntry, MissingDtype,
 * InvalidDtype, UnsupportedDtype, MissingShape, InvalidShape,
 * TooManyDimensions, MissingDataOffsets, InvalidDataOffsets,
 * DataOffsetOutOfBounds; NNZ_EINVAL) plus one check it leaves to its loader:
 * a tensor's byte range equals element count x dtype size. */
typedef struct nnz_safetensors nnz_safetensors;

typedef struct nnz_tensor_desc {
  const char* name;      /* NUL-terminated, owned by the reader */
  int dtype;             /* NNZ_DT_* */
  uint32_t rank;         /* 0..4 */
  uint32_t dims[4];      /* dims[0..rank) */
  const void* data;      /* into the mapping */
  size_t nbytes;
} nnz_tensor_desc;

/* SafetensorsFile.init (safetensors.zig:134-161): open + mmap + parse
 * (NNZ_ENOTFOUND if the file cannot be opened). */
int nnz_safetensors_open(const char* path, nnz_safetensors** out);
/* SafetensorsFile.initFromBytes (safetensors.zig:167-181): parse a buffer
 * the caller keeps alive while the reader is open. */
int nnz_safetensors_from_bytes(const void* bytes, size_t len, nnz_safetensors** out);
/* SafetensorsFile.deinit (safetensors.zig:183-193). */
int nnz_safetensors_close(nnz_safetensors* f);
/* Number of tensors (SafetensorsFile.count), in header order. */
uint32_t nnz_safetensors_count(const nnz_safetensors* f);
/* tensors[index]. */
int nnz_safetensors_tensor(const nnz_safetensors* f, uint32_t index, nnz_tensor_desc* desc);
/* SafetensorsFile.getTensor (safetensors.zig:196-209); NNZ_ENOTFOUND if absent. */
int nnz_safetensors_find(const nnz_safetensors* f, const char* name, nnz_tensor_desc* desc);

#ifdef __cplusplus
}
#endif
#endif /* NNZ_B200_H_ */
