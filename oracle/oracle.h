/*
 * oracle.h -- CPU restatement of ZeroLlm's quantized-linear + paged-KV decode path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is the parity checker for the CUDA
 * implementation in zeroplatform_b200/csrc and the timed CPU baseline of
 * bench.py. Nothing in the product path links, loads or calls it.
 *
 * The reference (kzxl/ZeroPlatform) is C# (.NET 8) and cannot be compiled in
 * this environment, so each function below restates one C# function, in the
 * same arithmetic order, and cites the file:line it follows (paths relative
 * to the reference project root).  Conventions mirrored exactly:
 *   - Math.Round == round-half-to-even on double (rint in the default mode);
 *   - (Half)f == IEEE binary16 round-to-nearest-even;
 *   - Math.Exp / Math.Sqrt / Math.Pow / Math.Cos / Math.Sin evaluated in
 *     double and cast to float;
 *   - no multiply-add contraction except where the C# calls Fma.MultiplyAdd
 *     (built with -ffp-contract=off);
 *   - Vector<float> / Vector256<float> are 8 lanes (AVX2).
 * Horizontal reductions (Vector256.Sum, Vector.Dot) follow the .NET 8 x64 JIT
 * lowering: Sum = lower128+upper128 then two pairwise horizontal adds; Dot =
 * per-128-bit-lane dpps ((p0+p1)+(p2+p3)) then lower+upper.
 *
 * Parity is pinned against the reference's own known-answer tests (see
 * tests/test_oracle_golden.py): the Q8_0/Q4_0 GEMV goldens (192 and 48),
 * the MatVecMulQ8_0 row sums, the fused-vs-dequantized dot tests, the exact
 * int8 GEMM patterns, the PagedKvCache accounting test and the
 * batched-vs-sequential prefill identity.
 */
#ifndef ZEROLLM_ORACLE_H
#define ZEROLLM_ORACLE_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- HalfHelper (ZeroLlm/src/ZeroLlm.Core/Quantization/HalfHelper.cs:13-75) ---- */
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_f32_to_f16_array(const float* src, uint16_t* dst, size_t n);

/* ---- Block formats (BlockQ8_0.cs:25-71, BlockQ4_0.cs:25-76, LlmQuantizer.cs:20-57) ----
 * n must be a multiple of 32; dst receives n/32 packed AoS blocks
 * (Q8_0: 34 bytes {fp16 d, int8 qs[32]}, Q4_0: 18 bytes {fp16 d, u8 qs[16]}). */
void orc_quantize_q8_0(const float* src, size_t n, uint8_t* dst);
void orc_quantize_q4_0(const float* src, size_t n, uint8_t* dst);
void orc_dequantize_q8_0(const uint8_t* blocks, size_t n, float* dst);
void orc_dequantize_q4_0(const uint8_t* blocks, size_t n, float* dst);

/* ---- QuantizedKernels (QuantizedKernels.cs:21-349) ----
 * path: 0 = the AVX2/FMA branch (:26-53, :106-135), 1 = the scalar branch (:56-77, :138-167). */
float orc_dot_q8_0(const float* x, const uint8_t* w, size_t nblocks, int path);
float orc_dot_q4_0(const float* x, const uint8_t* w, size_t nblocks, int path);
/* y = W x (accumulate = 0, MatVecMul*) or y += W x (accumulate = 1, MatVecAdd*).
 * Rows run in parallel on `threads` host threads when rows >= 1024 (:205). threads <= 0: all cores. */
void orc_matvec_q8_0(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols, int accumulate, int threads);
void orc_matvec_q4_0(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols, int accumulate, int threads);
/* Batched form used by LlmEngine.PrefillPrompt (LlmEngine.cs:208-304): Y[m,:] (=|+=) W X[m,:],
 * token-parallel over m. */
void orc_matmul_q8_0(const uint8_t* w, const float* x, float* y, size_t m, size_t rows, size_t cols, int accumulate, int threads);
void orc_matmul_q4_0(const uint8_t* w, const float* x, float* y, size_t m, size_t rows, size_t cols, int accumulate, int threads);

/* ---- int8 x int8 -> int32 (TensorBlas.Quantized.cs:39-154, ZeroTensorNativeBridge.cs:108) ----
 * C[m,n] = sum_p A[m,p] * B[p,n]; A row-major [m,k], B row-major [k,n]. */
void orc_gemm_i8(const int8_t* a, const int8_t* b, int32_t* c, size_t m, size_t n, size_t k);
int32_t orc_dot_i8(const int8_t* a, const int8_t* b, size_t n);
/* Per-32-block int32 partial sums of an int8 activation against Q8_0 weights:
 * P[m][r][blk] = sum_{i<32} xq[m][32 blk + i] * qw[r][blk][i]. */
void orc_block_dots_i8(const int8_t* xq, const uint8_t* w, int32_t* p, size_t m, size_t rows, size_t cols);

/* ---- Layers ---- */
/* RmsNorm.Forward (Layers/RmsNorm.cs:14-59) */
void orc_rmsnorm(const float* x, const float* w, float* out, size_t n, float eps);
/* RoPE.EnsureCache (Layers/RoPE.cs:22-65): cos/sin tables [max_pos][head_dim/2] */
void orc_rope_table(int max_pos, int head_dim, float freq_base, float* cos_t, float* sin_t);
/* RoPE.ApplyInplace (Layers/RoPE.cs:70-127), interleaved pairs (2i, 2i+1), table path */
void orc_rope_apply(float* v, int pos, int head_dim, const float* cos_t, const float* sin_t);
/* SwiGLU.Forward (Layers/SwiGLU.cs:13-51) */
void orc_swiglu(const float* gate, const float* up, float* out, size_t n);
/* LlmEngine.DotProductSimd (Engine/LlmEngine.cs:463-500) */
float orc_dot_f32(const float* a, const float* b, int len);

/* GqaAttention.Forward (Layers/GqaAttention.cs:29-130) over a KvSequenceView
 * (Memory/PagedKvCache.cs:10-42).  K/V of one layer are addressed as
 *   pool + (page_table[t / page_size] * page_stride + (t % page_size) * token_stride)
 * with token_stride = hkv*hd floats; each token row is [hkv][hd]. */
void orc_gqa_attention(const float* q, const float* kpool, const float* vpool, const int32_t* page_table,
                       int page_size, size_t page_stride, int seq_len, int hq, int hkv, int hd, float* out);

/* TensorOps.FlashAttentionCpu (ZeroTensor/src/ZeroTensor.Core/TensorOps.Neural.cs:983-1180) with its per-row
 * FlashAttentionComputeRow (:670-975): q [batch][sq][d], k [kv batch][sk][d], v [kv batch][sk][dv], out
 * [batch][sq][dv]; kv batch of b = is_gqa ? (b / hq) * hkv + (b % hq) / group : b.  Keys in blocks of 32: scores
 * dot * scale (+ mask row), a block whose maximum is -inf skipped, weights exp(s - block max) (in double), merged
 * with alpha = exp(old max - new max), beta = exp(block max - new max); out = acc / sum (zeros for sum 0).  mask
 * may be null; else mask_batches blocks of [sq][sk] and batch b reads block b % mask_batches. */
void orc_flash_attention(size_t batch, int sq, int sk, int d, int dv, float scale, int is_gqa, int hq, int hkv,
                         int group, const float* q, const float* k, const float* v, const float* mask,
                         size_t mask_batches, float* out);

/* TensorOps.PagedAttention pure-C# fallback (ZeroTensor/src/ZeroTensor.Core/TensorOps.Neural.cs:2418-2473):
 * online softmax; K/V pools [num_blocks][block_size][hkv][hd]; q/out [hq][hd]. */
void orc_paged_attention(const float* q, const float* kcache, const float* vcache, const int32_t* block_table,
                         int hq, int hkv, int hd, int block_size, int context_len, float scale, float* out);

/* SparseMoeLayer.Forward (Layers/SparseMoeLayer.cs:32-125) for one token, Q4_0 or Q8_0 experts.
 * qtype: 8 or 4. router_logits: if non-null, used as the router output instead of the router GEMV
 * (the MoE benchmark draws router logits directly); else router_w (fp32 [E][dim]) is applied.
 * experts_gate/up: [E][ffn][dim] blocks, experts_down: [E][dim][ffn] blocks. residual += sum_k w_k * expert_k(x).
 * sel_idx/sel_w (optional, length top_k) receive the selected experts and their softmax weights. */
void orc_moe_forward(const float* xnorm, const float* router_w, const float* router_logits, int n_experts, int top_k,
                     int qtype, const uint8_t* experts_gate, const uint8_t* experts_up, const uint8_t* experts_down,
                     int dim, int ffn, float* residual, int32_t* sel_idx, float* sel_w);

/* LlmSampler.Sample, greedy branch (Sampling/LlmSampler.cs:21-72). Modifies logits in place
 * (repetition penalty). Returns the argmax (first index wins ties). */
int32_t orc_sample_greedy(float* logits, size_t vocab, const int32_t* past, size_t n_past, float repetition_penalty);

/* LlmSampler.Sample, every branch (Sampling/LlmSampler.cs:21-172) with the random draw supplied: `u` stands for
 * (float)random.NextDouble().  Modifies logits in place as the reference does (penalty, temperature, then
 * probabilities).  The candidates (p > 1e-6) are sorted by probability, descending; .NET's List.Sort leaves the
 * order of exactly equal probabilities unspecified, this restatement puts the lower token id first.  When
 * cand_idx / cand_p are given (capacity cap), they receive the candidates kept after Top-K, Min-P and Top-P and
 * their renormalised probabilities (value * invTotal), *n_cand their count (0 on the greedy branch). */
int32_t orc_sample(float* logits, size_t vocab, const int32_t* past, size_t n_past, float temperature, float top_p,
                   float min_p, int32_t top_k, float repetition_penalty, float u, int32_t* cand_idx, float* cand_p,
                   int32_t* n_cand, int32_t cap);

/* ---- Model + engine (Engine/LlmEngine.cs:157-461, Memory/PagedKvCache.cs:47-286, Memory/KvBlock.cs) ----
 * All projection weights are Q8_0 AoS blocks, concatenated over layers:
 *   wq [L][hq*hd][dim], wk/wv [L][hkv*hd][dim], wo [L][dim][hq*hd],
 *   wgate/wup [L][ffn][dim], wdown [L][dim][ffn], tok_emb/lm_head [vocab][dim].
 * Norm weights are fp32: attn_norm/ffn_norm [L][dim], final_norm [dim]. */
typedef struct {
    int vocab, dim, layers, heads, kv_heads, ffn, context_length;
    float eps, rope_base;
    const uint8_t* tok_emb;
    const uint8_t* lm_head;
    const float* final_norm;
    const float* attn_norm;
    const float* ffn_norm;
    const uint8_t* wq;
    const uint8_t* wk;
    const uint8_t* wv;
    const uint8_t* wo;
    const uint8_t* wgate;
    const uint8_t* wup;
    const uint8_t* wdown;
} orc_model;

/* kv_fp16 != 0 rounds every appended K/V element to binary16 (the storage precision of the CUDA
 * cache); 0 keeps the reference's fp32 pages. threads <= 0: all cores. */
void* orc_engine_create(const orc_model* m, int total_pages, int page_size, int kv_fp16, int threads);
void orc_engine_destroy(void* e);
/* LlmEngine.PrefillPrompt (LlmEngine.cs:157-315): T == 1 runs ForwardToken; T > 1 the batched
 * path with the per-layer causal length (l == L-1 ? pos+1 : pos). Returns 0, or -1 when the page pool
 * is exhausted. logits: [vocab] of the last token. */
int orc_engine_prefill(void* e, int seq_id, const int32_t* tokens, int n, int start_pos, float* logits);
/* LlmEngine.ForwardToken (LlmEngine.cs:347-461). */
int orc_engine_forward_token(void* e, int seq_id, int token, int pos, float* logits);
int orc_engine_seq_len(void* e, int seq_id);
int orc_engine_free_blocks(void* e);
void orc_engine_free_sequence(void* e, int seq_id);
/* Reads back one cached K or V row ([hkv*hd] floats) -- PagedKvCache.GetKey/GetValue (:318-346). */
int orc_engine_get_kv(void* e, int seq_id, int layer, int token, int want_value, float* out);
/* Page table of a sequence (physical page ids in logical order). Returns the number of pages. */
int orc_engine_page_table(void* e, int seq_id, int32_t* out, int cap);
/* Standalone PagedKvCache (PagedKvCache.cs:47-286) for the accounting tests: append with the
 * AppendToken rule (the length advances when layer == layers-1). */
int orc_engine_append_token(void* e, int seq_id, int layer, const float* k, const float* v);

int orc_num_threads(void);

#ifdef __cplusplus
}
#endif
#endif
