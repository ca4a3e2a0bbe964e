/*
 * zero_tensor_cuda.h -- device-pointer extension of the ZeroTensor native bridge (libzero_tensor.so).
 *
 * The reference ABI in zero_tensor.h takes host pointers, so every call would copy its weights over
 * PCIe.  These entry points take DEVICE pointers and a CUDA stream (cudaStream_t passed as void*;
 * NULL = the legacy default stream) and only enqueue work: nothing here synchronises the host.
 * The caller owns every buffer, as in the reference (ZeroTensorNativeBridge.cs:340-348 pins caller
 * memory and never receives library memory).  Device buffers are what ZeroTensor exposes as
 * DeviceMemoryStorage<T> with DeviceType.Cuda (ZeroTensor/src/ZeroTensor.Core/Storage/
 * DeviceMemoryStorage.cs:20-110, Storage/DeviceType.cs:16): DeviceHandle is the CUdeviceptr passed here.
 * Return codes as in zero_tensor.h (0 = success).
 *
 * Device weight layout ("SoA"), produced once per weight by zcu_q8_0_repack / zcu_q4_0_repack from the
 * reference's packed GGML blocks (BlockQ8_0.cs:10-17, BlockQ4_0.cs:10-17):
 *   Q8_0: qs  int8 [n_rows][k_cols]           d fp16 bits [n_rows][k_cols/32]
 *   Q4_0: qs  uint8[n_rows][k_cols/32][16]    d fp16 bits [n_rows][k_cols/32]
 *         (byte j of a block = element j in the low nibble, element j+16 in the high nibble)
 * Device pointers must be 16-byte aligned (cudaMalloc gives 256).
 */
#ifndef ZERO_TENSOR_CUDA_H
#define ZERO_TENSOR_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifndef ZC_API
#if defined(__GNUC__)
#define ZC_API __attribute__((visibility("default")))
#else
#define ZC_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* fp32 [n] (n a multiple of 32, 16-byte aligned) -> packed GGML blocks, bit-identical to
 * LlmQuantizer.QuantizeToQ8_0 / QuantizeToQ4_0 (ZeroLlm/src/ZeroLlm.Core/Quantization/LlmQuantizer.cs:20-57,
 * BlockQ8_0.Quantize BlockQ8_0.cs:43-71, BlockQ4_0.Quantize BlockQ4_0.cs:120-150). */
ZC_API int32_t zcu_quantize_q8_0(const float* src, uint8_t* blocks, size_t n, void* stream);
ZC_API int32_t zcu_quantize_q4_0(const float* src, uint8_t* blocks, size_t n, void* stream);

/* AoS GGML blocks (device) -> SoA device layout. Replaces nothing in the reference: the managed code
 * streams the AoS blocks straight from the mmap (GgufFormat.cs:206-244); on the GPU the one-time
 * repack makes every row 16-byte aligned for 128-bit streaming loads. */
ZC_API int32_t zcu_q8_0_repack(const uint8_t* aos, int8_t* qs, uint16_t* d, size_t n_rows, size_t k_cols, void* stream);
ZC_API int32_t zcu_q4_0_repack(const uint8_t* aos, uint8_t* qs, uint16_t* d, size_t n_rows, size_t k_cols, void* stream);

/* Decode GEMV on device buffers.  accumulate == 0: y = W x -- QuantizedKernels.MatVecMulQ8_0 /
 * MatVecMulQ4_0 (ZeroLlm/src/ZeroLlm.Core/Quantization/QuantizedKernels.cs:190-267);
 * accumulate != 0: y += W x -- MatVecAddQ8_0 / MatVecAddQ4_0 (:272-349).  x[k_cols], y[n_rows] fp32. */
ZC_API int32_t zcu_gemv_q8_0(const int8_t* qs, const uint16_t* d, const float* x, float* y, size_t n_rows, size_t k_cols,
                      int32_t accumulate, void* stream);
ZC_API int32_t zcu_gemv_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, size_t n_rows, size_t k_cols,
                      int32_t accumulate, void* stream);

/* Batched / prefill quantized GEMM on the tensor cores: Y[m][n_rows] (=|+=) X[m][k_cols] . W^T for Q8_0 W in
 * SoA layout -- LlmEngine.PrefillPrompt's token-parallel MatVecMulQ8_0 / MatVecAddQ8_0
 * (ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs:208-304) as one contraction.  X, Y fp32 row-major.
 * Numerics: weights enter the MMA as fp16(q*d), activations as fp16(x) (|x| < 65504), fp32 accumulation.
 * k_cols must be a multiple of 32; the fp16 copy of X lives in the library's per-(device, stream) workspace. */
ZC_API int32_t zcu_gemm_q8_0(const int8_t* qs, const uint16_t* d, const float* x, float* y, size_t m, size_t n_rows,
                             size_t k_cols, int32_t accumulate, void* stream);
/* The same for Q4_0 weights (SoA nibbles [n_rows][k_cols/32][16] + fp16 scales, zcu_q4_0_repack): the batched
 * MatVecMulQ4_0 / MatVecAddQ4_0 (QuantizedKernels.cs:231-267,313-349) on the tensor cores; k_cols % 32 == 0. */
ZC_API int32_t zcu_gemm_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, size_t m, size_t n_rows,
                             size_t k_cols, int32_t accumulate, void* stream);

/* Synchronises the device and returns its status word: 0 = healthy, otherwise the code a kernel recorded
 * when one of its bounded waits expired (the kernel then stopped, drained and released its resources).
 * reset != 0 clears it. */
ZC_API int32_t zcu_device_status(int32_t reset);

/* Failure-detection self-test on one GPU (no counterpart in the reference): runs the tensor-parallel all-reduce's
 * reduce kernel against a local receive area of `ranks` (2 .. 8) ranks in which only rank 0 has pushed (its
 * words carry epoch 1), with the kernel's bounded wait shortened to wait_ms (1 .. 5000).  The wait runs out, the
 * kernel records code 21 in its status word and returns, and the context stays usable.  Returns that code (0 would
 * mean the wait never ran out) or a negative status when the test could not run; seen (16 words, may be NULL)
 * receives the kernel's state: [4] the epoch it waited for, [5 + r] the epoch of rank r's first word. */
ZC_API int32_t zcu_peer_wait_selftest(int32_t ranks, int32_t wait_ms, uint32_t* seen);

/* Paged decode attention on device buffers -- GqaAttention.Forward (ZeroLlm/src/ZeroLlm.Core/Layers/
 * GqaAttention.cs:29-130) and TensorOps.PagedAttention (TensorOps.Neural.cs:2372-2476) for `batch`
 * sequences with one query token each.
 *   q, out        [batch][hq][hd] fp32
 *   k_pool/v_pool element (page p, slot t, kv head h, dim e) at p*page_stride + t*slot_stride +
 *                 h*head_stride + e (elements); kv_dtype 0 = fp32, 1 = fp16
 *   page_table    [batch][max_pages] int32 physical page ids; ids outside [0, num_pages) are skipped
 *   ctx_len       [batch] int32 tokens attended per sequence (the reference's per-layer causal length
 *                 is the caller's choice of ctx_len; ctx_len 0 yields zeros, GqaAttention.cs:38-42)
 *   max_ctx       an upper bound of ctx_len (sizes the split-K grid; the kernel reads ctx_len itself)
 * Long contexts are split across CTAs; the split partials live in a library-owned workspace per
 * (device, stream), so concurrent calls on one stream are ordered and calls on different streams do
 * not share it. */
ZC_API int32_t zcu_paged_attention(const float* q, const void* k_pool, const void* v_pool, int32_t kv_dtype,
                            const int32_t* page_table, const int32_t* ctx_len, float* out, int32_t batch, int32_t hq,
                            int32_t hkv, int32_t hd, int32_t page_size, int32_t max_pages, int32_t num_pages,
                            int64_t page_stride, int64_t slot_stride, int64_t head_stride, float scale,
                            int32_t max_ctx, void* stream);

/* The same paged attention for callers that cannot allocate device memory when they run it -- a server that
 * gave all free HBM to its KV page pool, or a host runtime whose decode loop forbids device allocation after
 * start-up (cudaMalloc / cudaFree can synchronise the whole device).  No counterpart in the
 * reference (its managed fallback allocates nothing on a device).  Same arguments as zcu_paged_attention;
 * the split-K scratch is a fixed 1 MiB array inside the library (held by every GPU that loads it until the
 * process exits), so shapes needing more than 8,192 arrival counters (batch * hq) or 253,952 partial floats
 * (batch * hq * splits * (hd + 2)) return -6 with a message in zc_cuda_last_error().  It never calls
 * cudaMalloc or cudaFree.  The first call on a device looks the array's address up (cudaGetSymbolAddress) and
 * caches it.  All calls on a device share the array: calls whose kernels overlap on the GPU
 * race (calls on one stream are ordered); each call clears the counters it uses before launching. */
ZC_API int32_t zcu_paged_attention_noalloc(const float* q, const void* k_pool, const void* v_pool, int32_t kv_dtype,
                                           const int32_t* page_table, const int32_t* ctx_len, float* out,
                                           int32_t batch, int32_t hq, int32_t hkv, int32_t hd, int32_t page_size,
                                           int32_t max_pages, int32_t num_pages, int64_t page_stride,
                                           int64_t slot_stride, int64_t head_stride, float scale, int32_t max_ctx,
                                           void* stream);

/* RmsNorm.Forward (Layers/RmsNorm.cs:14-59) on `rows` rows of n elements. */
ZC_API int32_t zcu_rmsnorm(const float* x, const float* w, float* out, int32_t rows, int32_t n, float eps, void* stream);
/* SwiGLU.Forward (Layers/SwiGLU.cs:13-51). */
ZC_API int32_t zcu_swiglu(const float* gate, const float* up, float* out, size_t n, void* stream);
/* RoPE.ApplyInplace (Layers/RoPE.cs:131-163) on x [rows][heads][hd] at positions pos[row] (pos == NULL:
 * pos0 + row), with cos/sin tables [max_pos][hd/2] as RoPE.EnsureCache builds them (:83-125). */
ZC_API int32_t zcu_rope(float* x, int32_t rows, int32_t heads, int32_t hd, const int32_t* pos, int32_t pos0,
                 const float* cos_t, const float* sin_t, int32_t max_pos, void* stream);
/* LlmEngine.LookupTokenEmbedding for a Q8_0 table in SoA layout (Engine/LlmEngine.cs:317-345):
 * out[i] = dequantized row tokens[i] (ids outside [0, vocab) read row 0). */
ZC_API int32_t zcu_embed_q8_0(const int8_t* qs, const uint16_t* d, const int32_t* tokens, int32_t n_tokens, int32_t vocab,
                       int32_t dim, float* out, void* stream);

/* ---------------------------------------------------------------------------------------------------------
 * Decode engine: LlmEngine (ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs:19-568) for Q8_0 Llama-style models
 * over a device-resident paged KV cache (Memory/PagedKvCache.cs:47-286, 16-token pages, fp16 K/V).
 * The engine owns its device memory; weights are copied in once with zcu_engine_set_weight.
 * ------------------------------------------------------------------------------------------------------- */
typedef struct {
  int32_t vocab, dim, layers, heads, kv_heads, ffn, context_length;  /* LlmModelConfig (LlmModelConfig.cs:6-41) */
  float eps, rope_base;                                               /* RmsNormEps, RopeFreqBase */
  int32_t total_pages, page_size;                                     /* PagedKvCache(totalBlocks, blockSize) */
  int32_t max_batch;                                                  /* live sequences / decode batch */
  int32_t max_pages_per_seq;                                          /* page-table width */
  int32_t max_prefill_tokens;                                         /* longest prompt prefilled at once */
  int32_t reference_causal_quirk; /* 1: non-final layers attend to [0, pos) as the reference does (LlmEngine.cs:254,
                                     PagedKvCache.cs:139-142); 0: every layer attends to [0, pos] */
} zcu_engine_config;

/* Tensor kinds for zcu_engine_set_weight.  Q8_0 tensors are the reference's packed blocks [rows][cols/32]
 * (LlmModel / LlmQuantizer layout, row-major [out][in]); norms are fp32 [dim].  `layer` is ignored for the
 * whole-model tensors. */
enum {
  ZCU_W_TOK_EMB = 0,   /* Q8_0 [vocab][dim]   TokenEmbeddings_Q8 */
  ZCU_W_LM_HEAD = 1,   /* Q8_0 [vocab][dim]   LmHead_Q8 */
  ZCU_W_FINAL_NORM = 2,
  ZCU_W_ATTN_NORM = 3,
  ZCU_W_FFN_NORM = 4,
  ZCU_W_Q = 5,         /* Q8_0 [heads*hd][dim] */
  ZCU_W_K = 6,         /* Q8_0 [kv_heads*hd][dim] */
  ZCU_W_V = 7,
  ZCU_W_O = 8,         /* Q8_0 [dim][heads*hd] */
  ZCU_W_GATE = 9,      /* Q8_0 [ffn][dim] */
  ZCU_W_UP = 10,
  ZCU_W_DOWN = 11      /* Q8_0 [dim][ffn] */
};

/* stream: the CUDA stream the engine enqueues on (NULL: the engine creates its own). */
ZC_API int32_t zcu_engine_create(const zcu_engine_config* cfg, void* stream, void** engine);

/* Tensor parallelism over tp_size GPUs of one node: one engine per GPU (one process or thread each), every
 * rank making the same calls in the same order.  Rank r keeps query heads [head_begin, +heads) with their Wq
 * rows, Wo columns and K/V pages; K/V heads [kv_head_begin, +kv_heads) with their Wk/Wv rows; FFN units
 * [ffn_begin, +ffn) (whole 32-blocks) with their Wgate/Wup rows and Wdown columns; LM-head rows [vocab_begin,
 * +vocab).  Embedding and norms are replicated.  After Wo and after Wdown the residual stream is summed over
 * ranks: up to max_batch rows over NVLink peer memory (CUDA IPC mappings, a one-shot push into every rank's
 * slot and a rank-ordered sum; on the tensor-core path fused into the GEMM's split-K partials and the next
 * RmsNorm), larger ones (prefill) by NCCL all-reduce; ZCU_TP_ALLREDUCE=nccl in the environment of every rank
 * keeps all of them on NCCL.  Greedy sampling takes the arg-max of every rank's slice and merges them.
 * zcu_tp_plan is host-only (no GPU needed) and fails when heads or kv_heads do not divide by tp_size, when a
 * rank's Wo column slice is not a whole number of 32-blocks, or when there are fewer FFN blocks than ranks. */
typedef struct {
  int32_t head_begin, heads;
  int32_t kv_head_begin, kv_heads;
  int32_t ffn_begin, ffn;
  int32_t vocab_begin, vocab;
} zcu_tp_shard;
ZC_API int32_t zcu_tp_plan(const zcu_engine_config* cfg, int32_t tp_size, int32_t tp_rank, zcu_tp_shard* out);
/* 128-byte NCCL unique id, made by one rank and given to all (e.g. by a torch.distributed broadcast). */
ZC_API int32_t zcu_nccl_unique_id(uint8_t* out, size_t cap);
/* Collective: every rank calls it with its own tp_rank and the same nccl_id (ignored when tp_size == 1). */
ZC_API int32_t zcu_engine_create_tp(const zcu_engine_config* cfg, int32_t tp_size, int32_t tp_rank,
                                   const uint8_t* nccl_id, void* stream, void** engine);
ZC_API int32_t zcu_engine_destroy(void* engine);
ZC_API const char* zcu_engine_last_error(void* engine);
/* `src` is host or device memory holding the FULL tensor; a tensor-parallel rank keeps its own slice.  The
 * call first waits for all work queued on the device (a device source may be written by any stream). */
ZC_API int32_t zcu_engine_set_weight(void* engine, int32_t kind, int32_t layer, const void* src, size_t bytes);
/* LlmEngine.PrefillPrompt (LlmEngine.cs:157-315): n prompt tokens at positions start_pos.. of seq_id; writes the
 * last token's logits [vocab] to host memory when logits != NULL.  n == 1 is ForwardToken. */
ZC_API int32_t zcu_engine_prefill(void* engine, int32_t seq_id, const int32_t* tokens, int32_t n, int32_t start_pos,
                                  float* logits);
/* LlmEngine.ForwardToken (LlmEngine.cs:347-461) for `batch` sequences at once (one token each, host arrays);
 * logits [batch][vocab] and/or greedy next tokens [batch] to host memory (either may be NULL). */
ZC_API int32_t zcu_engine_decode(void* engine, const int32_t* seq_ids, const int32_t* tokens, const int32_t* positions,
                                 int32_t batch, float* logits, int32_t* next_tokens);
/* GenerateStreamAsync with greedy sampling (LlmEngine.cs:71-150, LlmSampler.cs:21-72): prefill, then n_new
 * sample -> ForwardToken steps replayed from one captured CUDA graph with the state on the device.
 * repetition_penalty <= 1 disables it; eos_token < 0 never stops.  Returns the number of tokens written to
 * out_tokens (or a negative status); timing_ms[0] = prefill ms, timing_ms[1] = decode ms (device events). */
ZC_API int32_t zcu_engine_generate(void* engine, int32_t seq_id, const int32_t* prompt, int32_t n_prompt,
                                   int32_t n_new, float repetition_penalty, int32_t eos_token, int32_t* out_tokens,
                                   float* timing_ms);
/* Which form zcu_engine_generate runs a generation step in: 1 = one cooperative kernel per token (one GPU, shapes
 * that fit it: head size 64 or 128, dim / ffn / heads*hd multiples of 256, heads x dim <= 65536), 0 = the captured
 * graph of per-operator kernels (ZCU_FUSED_DECODE=0 in the environment forces it), -1 = not decided yet (no
 * generate call so far).  `why` (may be NULL) receives the reason the one-kernel form is not used. */
ZC_API int32_t zcu_engine_step_kind(void* engine, char* why, int32_t cap);
/* SamplingConfig (ZeroLlm/src/ZeroLlm.Core/Sampling/SamplingConfig.cs:8-26): Temperature, TopP, MinP, TopK
 * (0 = no limit), RepetitionPenalty. */
typedef struct {
  float temperature, top_p, min_p;
  int32_t top_k;
  float repetition_penalty;
} zcu_sampling_config;

/* LlmSampler.Sample (Sampling/LlmSampler.cs:21-172) for `rows` rows of device logits [rows][vocab], modified in
 * place as the reference modifies its span (penalty, temperature, probabilities).  past [rows][past_cap] with
 * past_len [rows] (device, may be NULL) are the tokens the penalty applies to; uniforms [rows] (device) stand for
 * (float)random.NextDouble() and are unused on the greedy branch (temperature <= 0.001 or top_k == 1).  out [rows]
 * (device) receives the token, or -1 when more than 4096 candidates remain after Top-K (top_k 0 over a flat
 * distribution).  cand_idx / cand_p [rows][cand_cap] and n_cand [rows] (device, may be NULL) receive the kept
 * candidates by probability descending (the lower token id first among equal probabilities), their renormalised
 * probabilities and their count.  Enqueues only. */
ZC_API int32_t zcu_sample(float* logits, int32_t rows, int32_t vocab, const int32_t* past, const int32_t* past_len,
                          int32_t past_cap, const zcu_sampling_config* cfg, const float* uniforms, int32_t* out,
                          int32_t* cand_idx, float* cand_p, int32_t* n_cand, int32_t cand_cap, void* stream);
/* The draw the engine's sampled generation uses for its i-th token: SplitMix64(seed + i), top 24 bits, in [0, 1)
 * (host helper; no counterpart in the reference, whose System.Random draws cannot be reproduced). */
ZC_API float zcu_sample_uniform(uint64_t seed, uint64_t i);
/* GenerateStreamAsync with any SamplingConfig (LlmEngine.cs:71-150): prefill, then n_new steps of sample ->
 * ForwardToken with the sampler on the device (the i-th token's draw is zcu_sample_uniform(seed, i)), replayed
 * from one captured graph; a greedy config runs zcu_engine_generate.  One GPU (tp_size 1) only: -4 otherwise.
 * Returns the tokens written to out_tokens (a token equal to eos_token >= 0 ends generation unwritten) or < 0;
 * timing_ms[0] = prefill ms, timing_ms[1] = decode ms. */
ZC_API int32_t zcu_engine_generate_sampled(void* engine, int32_t seq_id, const int32_t* prompt, int32_t n_prompt,
                                           int32_t n_new, const zcu_sampling_config* cfg, uint64_t seed,
                                           int32_t eos_token, int32_t* out_tokens, float* timing_ms);
/* Batched greedy generation (GenerateStreamAsync for `batch` live sequences at once, repetition penalty 1):
 * tokens[b] is fed at position seq_len(seq_ids[b]); each of n_new steps runs ForwardToken for every sequence
 * and samples greedily, replayed from one captured CUDA graph (collectives included).  out_tokens[b * n_new + i]
 * is sequence b's i-th sampled token.  timing_ms[0] = device ms of the n_new steps.  Returns n_new or < 0. */
ZC_API int32_t zcu_engine_generate_batch(void* engine, int32_t batch, const int32_t* seq_ids, const int32_t* tokens,
                                         int32_t n_new, int32_t* out_tokens, float* timing_ms);
/* Continuous batching (no counterpart in the reference, whose LlmEngine.GenerateStreamAsync, LlmEngine.cs:71-152,
 * runs each call's prefill and decode loop on its own over the shared PagedKvCache).  Concurrent requests share
 * every decode step: zcu_engine_submit queues one GenerateStreamAsync call (prompt tokens, SamplingConfig's numeric
 * fields, MaxTokens = max_new, EosTokenId = eos_token (-1: none) plus StopTokens); zcu_engine_serve_step admits
 * queued requests first come first served while a page-table row and the pages of prompt + max_new tokens are free
 * (PrefillPrompt, then the first token is sampled), then runs one ForwardToken + Sample for every running request
 * as one batched step (one captured graph per batch size) and reports what happened as events.  A request's i-th
 * token uses the draw zcu_sample_uniform(seed, i), so its tokens do not depend on what it was batched with beyond
 * the last bits of the logits.  One GPU (tp_size 1).  Sequences of running requests must not be freed or driven
 * through the other entry points meanwhile. */
typedef struct zcu_serve_event {
  int32_t seq_id;
  int32_t token;     /* the sampled token (ZCU_SERVE_STOP_TOKEN: the stop token, which is not part of the output;
                        cancelled / refused: -1) */
  int32_t finished;  /* 1 when the request is over and its sequence freed */
  int32_t reason;    /* ZCU_SERVE_* */
} zcu_serve_event;
enum {
  ZCU_SERVE_RUNNING = 0,
  ZCU_SERVE_STOP_TOKEN = 1,  /* eos_token or a stop token was sampled (GenerateStreamAsync breaks without yielding) */
  ZCU_SERVE_MAX_TOKENS = 2,  /* max_new tokens emitted (this event carries the last one) */
  ZCU_SERVE_CANCELLED = 3,
  ZCU_SERVE_REFUSED = 4      /* more than 4096 sampling candidates after Top-K */
};
/* Queues a request.  -2 for a live or queued seq_id or bad arguments, -6 when prompt + max_new cannot fit a
 * sequence (max_pages_per_seq, context length, total pages) or the prompt exceeds max_prefill_tokens, -4 when
 * tp_size > 1.  Host only: nothing runs until the next serve step. */
ZC_API int32_t zcu_engine_submit(void* engine, int32_t seq_id, const int32_t* prompt, int32_t n_prompt,
                                 int32_t max_new, const zcu_sampling_config* cfg, uint64_t seed, int32_t eos_token,
                                 const int32_t* stop_tokens, int32_t n_stop);
/* One scheduler iteration (blocking): cancellations, admissions, one batched decode step.  Writes the events to
 * events (cap >= 2 * max_batch + cancellations of queued requests) and returns their count, or < 0. */
ZC_API int32_t zcu_engine_serve_step(void* engine, zcu_serve_event* events, int32_t cap);
/* Cancels a queued or running request; its CANCELLED event comes with the next serve step.  -2 if unknown. */
ZC_API int32_t zcu_engine_cancel(void* engine, int32_t seq_id);
/* Running and queued request counts. */
ZC_API int32_t zcu_engine_serve_counts(void* engine, int32_t* active, int32_t* queued);

/* PagedKvCache.AppendTokenAt (Memory/PagedKvCache.cs:149-183) for tokens [start_pos, start_pos + n) of one layer:
 * k, v are [n][kv_heads][hd] (host or device; kv_dtype 0 = fp32, 1 = fp16).  Appending the last layer sets the
 * sequence length, as the reference counts a token once its last layer is stored.  Like set_weight, the call
 * first waits for all work queued on the device. */
ZC_API int32_t zcu_engine_append_kv(void* engine, int32_t seq_id, int32_t layer, int32_t start_pos, int32_t n_tokens,
                                    const void* k, const void* v, int32_t kv_dtype);
/* PagedKvCache.FreeSequence / GetSequenceLength / FreeBlockCount / the page table / GetKey+GetValue
 * (a tensor-parallel rank writes only its own K/V heads into `out`). */
ZC_API int32_t zcu_engine_free_sequence(void* engine, int32_t seq_id);
ZC_API int32_t zcu_engine_seq_len(void* engine, int32_t seq_id);
ZC_API int32_t zcu_engine_free_pages(void* engine);
ZC_API int32_t zcu_engine_page_table(void* engine, int32_t seq_id, int32_t* out, int32_t cap);
ZC_API int32_t zcu_engine_get_kv(void* engine, int32_t seq_id, int32_t layer, int32_t token, int32_t want_value,
                                 float* out);

/* ---------------------------------------------------------------------------------------------------------
 * Sparse mixture-of-experts FFN layer: SparseMoeLayer.Forward (ZeroLlm/src/ZeroLlm.Core/Layers/SparseMoeLayer.cs:
 * 32-125) for T tokens at once -- router logits (given, or an fp32 router [n_experts][dim] . xnorm), top-k
 * selection (ties keep the lowest expert index), softmax over the k selected, each selected expert's SwiGLU FFN
 * with Q4_0 (qtype 4) or Q8_0 (qtype 8) weights on the tensor cores, and residual += weight * expert output in
 * selection order.  Expert parallelism: ep_size ranks (one process per GPU, same calls on every rank), expert e
 * on rank e / (n_experts / ep_size); every rank passes its own tokens, rows travel to the experts' ranks and back
 * by NCCL all-to-all.  dim and ffn must be multiples of 256.  No shared experts.
 * ------------------------------------------------------------------------------------------------------- */
typedef struct {
  int32_t n_experts, top_k, dim, ffn; /* ExpertCount, ExpertUsedCount, EmbeddingDim, FeedForwardDim */
  int32_t qtype;                      /* 4 = Q4_0 experts, 8 = Q8_0 experts */
  int32_t max_tokens;                 /* largest T of a forward call on this rank */
} zcu_moe_config;
ZC_API int32_t zcu_moe_create(const zcu_moe_config* cfg, int32_t ep_size, int32_t ep_rank, const uint8_t* nccl_id,
                              void* stream, void** moe);
/* The expert-parallel exchange plan zcu_moe_forward follows on rank ep_rank (host only, no GPU needed).
 * counts_all [ep_size][n_experts] are the all-gathered routing counts (rows rank src sends to expert e; expert e
 * lives on rank e / (n_experts / ep_size)).  Out (each may be NULL): send_rows [ep_size] rows this rank sends to
 * each peer (its rows leave in expert order, one contiguous run per peer), recv_rows [ep_size] rows it receives
 * from each, recv_cnt [ep_size][n_experts / ep_size] rows per (source, local expert), perm [total] the position of
 * each received row (arrival order: by source, then local expert) in the [local expert][source] order the expert
 * GEMMs read.  Returns the total received (>= 0), -2 for bad arguments (n_experts % ep_size, negative counts) or
 * -6 when perm_cap is below the total.  No counterpart in the reference (SparseMoeLayer runs every expert
 * locally, SparseMoeLayer.cs:32-125). */
ZC_API int32_t zcu_moe_ep_plan(int32_t n_experts, int32_t ep_size, int32_t ep_rank, const int32_t* counts_all,
                               int32_t* send_rows, int32_t* recv_rows, int32_t* recv_cnt, int32_t* perm,
                               int32_t perm_cap);
ZC_API int32_t zcu_moe_destroy(void* moe);
ZC_API const char* zcu_moe_last_error(void* moe);
/* Expert `expert`'s gate (which 0, [ffn][dim]), up (1, [ffn][dim]) or down (2, [dim][ffn]) projection as the
 * reference's packed blocks (host or device memory); ranks that do not own the expert ignore it. */
ZC_API int32_t zcu_moe_set_expert(void* moe, int32_t expert, int32_t which, const void* src, size_t bytes);
/* Optional fp32 router weights [n_experts][dim] (host or device); without them forward needs router_logits. */
ZC_API int32_t zcu_moe_set_router(void* moe, const float* w, size_t bytes);
/* xnorm [T][dim], router_logits [T][n_experts] (or NULL: router weights, else uniform) and residual [T][dim]
 * (updated in place) are device memory; sel_idx / sel_w [T][top_k] (host or device, may be NULL) receive the
 * routing.  Synchronous. */
ZC_API int32_t zcu_moe_forward(void* moe, const float* xnorm, const float* router_logits, float* residual, int32_t T,
                               int32_t* sel_idx, float* sel_w);

#ifdef __cplusplus
}
#endif
#endif
