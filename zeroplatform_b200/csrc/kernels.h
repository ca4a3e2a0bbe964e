// kernels.h -- internal launch API of the CUDA kernels (C++ linkage; the public C ABI is in
// include/zero_tensor_cuda.h and capi.cu).  All pointers are device pointers unless stated.
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace zc {

// ---- weight layout (gemv.cu) ----
int repack_q8_0(const uint8_t* aos, int8_t* qs, uint16_t* d, size_t n, size_t k, cudaStream_t s);
int repack_q4_0(const uint8_t* aos, uint8_t* qs, uint16_t* d, size_t n, size_t k, cudaStream_t s);

// ---- fp32 -> packed AoS blocks (quant.cu); n = element count, a multiple of 32 ----
int quantize_q8_0(const float* src, uint8_t* dst, size_t n, cudaStream_t s);
int quantize_q4_0(const float* src, uint8_t* dst, size_t n, cudaStream_t s);

// ---- decode GEMV (gemv.cu): y = W x (accumulate = 0) or y += W x ----
int gemv_q8_0(const int8_t* qs, const uint16_t* d, const float* x, float* y, int n, int k, int accumulate,
              cudaStream_t s);
// Error word of the GEMV's bounded waits on its own bulk copies (0 = healthy); reset clears it.
int gemv_wait_status(int reset);
int gemv_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, int n, int k, int accumulate,
              cudaStream_t s);
// Fused prologues for the decode step: x = RmsNorm(x_raw) * norm_w, or x = SwiGLU(gate_up[0:k], gate_up[k:2k]).
int gemv_q8_0_rmsnorm(const int8_t* qs, const uint16_t* d, const float* x, const float* norm_w, float eps, float* y,
                      int n, int k, int accumulate, cudaStream_t s);
int gemv_q8_0_swiglu(const int8_t* qs, const uint16_t* d, const float* gate_up, float* y, int n, int k,
                     int accumulate, cudaStream_t s);

// ---- prefill / batched GEMM on tcgen05 (gemm_tc.cu): Y[m][n] (=|+=) X[m][:] . dequant(W)[n][:] ----
size_t gemm_q8_0_workspace_bytes(int m, int n, int k);  // fp16 activations + split-K partials
size_t gemm_workspace_max(int m_max, int n, int k);       // the largest of the above over 1 <= m <= m_max
int gemm_q8_0_tc(const int8_t* qs, const uint16_t* d, const float* x, float* y, int m, int n, int k, int accumulate,
                 void* workspace, size_t workspace_bytes, int* status, cudaStream_t s);
// The same on fp16 activations given as hi / lo pairs (x = hi + lo, see gemm_tc.cu): x_hi and x_lo rows of k
// values with a row pitch of ldx elements (producers write [rows][hi k | lo k]: x_lo = x_hi + k, ldx = 2k).
int gemm_q8_0_tc_h(const int8_t* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx, float* y,
                   int m, int n, int k, int accumulate, void* workspace, size_t workspace_bytes, int* status,
                   cudaStream_t s);
// The same GEMM without its split-K reduction (m <= 128): the products are left in the workspace as *nsplit >= 1
// partials [m][n] starting at *partials, for a consumer that sums them in split order (the tensor-parallel
// all-reduce push).  Stream-ordered like the other entries; the partials live until the next call on the
// workspace.
int gemm_q8_0_tc_h_partials(const int8_t* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx,
                            int m, int n, int k, void* workspace, size_t workspace_bytes, int* status, cudaStream_t s,
                            float** partials, int* nsplit);
// Q4_0 weights (SoA nibbles [N][K/32][16] + fp16 scales), same workspace size rule.
int gemm_q4_0_tc(const uint8_t* qs, const uint16_t* d, const float* x, float* y, int m, int n, int k, int accumulate,
                 void* workspace, size_t workspace_bytes, int* status, cudaStream_t s);
int gemm_q4_0_tc_h(const uint8_t* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx, float* y,
                   int m, int n, int k, int accumulate, void* workspace, size_t workspace_bytes, int* status,
                   cudaStream_t s);

// ---- paged decode attention (attention.cu) ----
// One query token per sequence. K/V element (page p, slot t, kv head h, dim e) lives at
//   pool + p*page_stride + t*slot_stride + h*head_stride + e          (elements)
// ctx_len[b] tokens of sequence b are attended (its page list is page_table[b*max_pages ...]).
// q/out: [batch][hq][hd] fp32.  kv_half != 0: pools are fp16, else fp32.
struct PagedAttnArgs {
  const float* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* page_table;
  const int32_t* ctx_len;
  float* out;
  int batch, hq, hkv, hd, page_size, max_pages;
  int num_pages;      // pages in each pool; entries outside [0, num_pages) are skipped (0 = unchecked)
  long long page_stride, slot_stride, head_stride;
  float scale;
  int kv_half;
  int max_ctx;        // upper bound of ctx_len over the batch (sizes the split grid)
  float* workspace;   // split-K partials; may be null when splits == 1
  int* counters;      // [batch*hq] zero-initialised arrival counters (left zeroed); null when splits == 1
  int splits;         // 0 = choose automatically
  int out_half = 0;   // 1: out is __half hi / lo pairs (the input of a tensor-core GEMM): hi at the float
                      //    layout's index, lo out_lo_offset elements after it; else float
  long long out_lo_offset = 0;
  long long q_stride = 0;     // elements between consecutive queries (0: hq*hd)
  long long out_stride = 0;   // elements between consecutive outputs (0: hq*hd)
  long long pt_stride = -1;   // elements between page-table rows (-1: max_pages; 0: all queries share row 0)
  const int32_t* pt_rows = nullptr;  // optional page-table row per query (default: the query index)
};
// kOk when the arguments describe a launchable shape: non-null pointers, batch, hq, hkv, page_size and max_pages
// positive, hq a multiple of hkv, hd one of 8/16/32/64/128/256 (else kBadArgument / kUnsupported).
int paged_attention_check(const PagedAttnArgs& a);
size_t paged_attention_workspace_floats(int batch, int hq, int hd, int splits);
int paged_attention_choose_splits(int batch, int hkv, int max_ctx, int page_size);
int paged_attention(const PagedAttnArgs& a, cudaStream_t s);

// Attention for many query rows at once (attention_prefill.cu).  Query row r of sequence z, head h reads
// q[z*q_seq_stride + h*q_head_stride + r*q_row_stride + 0..hd) and attends to key tokens [0, ctx_len[z*ctx_seq_stride
// + r]) of kv head h / group; key token t lives at page page_table[z*pt_seq_stride + t / page_size], slot
// t % page_size: element z*kv_seq_stride + kvh*head_stride + page*page_stride + slot*slot_stride + dim of k / v.
// out[z*out_seq_stride + h*out_head_stride + r*out_row_stride + dim] = softmax(q.k * scale) . v (zeros for a row
// with no key).  hd 16, 32, 64 or 128; k / v fp16 (kv_half) or fp32.
struct PrefillAttnArgs {
  const float* q;
  const void* k;
  const void* v;
  const int32_t* page_table;
  const int32_t* ctx_len;
  float* out;
  int rows, seqs, hq, group, hd;
  int page_size, max_pages, num_pages;
  long long page_stride, slot_stride, head_stride, kv_seq_stride;
  long long q_row_stride, q_head_stride, q_seq_stride;
  long long pt_seq_stride, ctx_seq_stride;
  long long out_row_stride, out_head_stride, out_seq_stride;
  int out_half = 0;            // 1: out is __half hi / lo pairs, lo out_lo_offset elements after hi
  long long out_lo_offset = 0;
  float scale_log2;            // scale * log2(e)
  int kv_half;
};
int prefill_attention(const PrefillAttnArgs& a, cudaStream_t s);

// ---- small decode-step operators (ops.cu) ----
// dst = src, `bytes` a multiple of 4, both 16-byte aligned; either side may be mapped pinned host memory.
int copy_words(const void* src, void* dst, size_t bytes, cudaStream_t s);
int rmsnorm(const float* x, const float* w, float* out, int rows, int n, float eps, cudaStream_t s);
// out [rows][hi n | lo n]: the GEMM's activation pairs (hi = fp16(v), lo = fp16(v - hi)).
int rmsnorm_h(const float* x, const float* w, __half* out, int rows, int n, float eps, cudaStream_t s);
int swiglu(const float* gate, const float* up, float* out, size_t n, cudaStream_t s);
int silu(const float* x, float* out, size_t n, cudaStream_t s);
// Interleaved RoPE on [rows][heads][hd] at positions pos[row] (or pos0 + row when pos == null),
// with host-precomputed cos/sin tables [max_pos][hd/2].
int rope(float* x, int rows, int heads, int hd, const int32_t* pos, int pos0, const float* cos_t,
         const float* sin_t, int max_pos, cudaStream_t s);
int embed_q8_0(const int8_t* qs, const uint16_t* d, const int32_t* tokens, int n_tokens, int vocab, int dim,
               float* out, cudaStream_t s);

// Decode-step pieces used by the engine (engine_ops.cu).
// qkv rows [T][q_dim + 2*kv_dim]: rotates q and k of row t at position pos[t] (RoPE.ApplyInplace), then stores
// k and v as fp16 into the layer's pools [page][kv_head][slot][hd] at page_table[rows[t]][pos/P], pos % P.
int rope_append_kv(float* qkv, int T, int hq, int hkv, int hd, const int32_t* pos, const int32_t* rows,
                   const int32_t* page_table, int max_pages, int page_size, const float* cos_t, const float* sin_t,
                   int max_pos, __half* k_pool, __half* v_pool, cudaStream_t s);
// out[t][i] = SwiGLU(gu[t][i], gu[t][ffn + i])
int swiglu_rows(const float* gu, float* out, int T, int ffn, cudaStream_t s);
int swiglu_rows_h(const float* gu, __half* out, int T, int ffn, cudaStream_t s);  // out [T][hi ffn | lo ffn]
// The same two steps fed by a GEMM's split-K partials part[splits][T][row] (summed in split order, as the
// separate reduction does) instead of its reduced output: one kernel instead of two.  rope_append_kv_parts also
// leaves the reduced rows (q and k rotated) in qkv.
int rope_append_kv_parts(const float* part, int splits, float* qkv, int T, int hq, int hkv, int hd,
                         const int32_t* pos, const int32_t* rows, const int32_t* page_table, int max_pages,
                         int page_size, const float* cos_t, const float* sin_t, int max_pos, __half* k_pool,
                         __half* v_pool, cudaStream_t s);
int swiglu_rows_h_parts(const float* part, int splits, __half* out, int T, int ffn, cudaStream_t s);
// LlmSampler greedy branch per row: repetition penalty over past[row][0:past_len[row]] then argmax
// (first index wins ties).  penalty <= 1 disables the penalty.  out[row] = token.
int greedy_sample(float* logits, int rows, int vocab, const int32_t* past, const int32_t* past_len, int past_cap,
                  float penalty, int32_t* out, cudaStream_t s);
// The same over a vocabulary slice [vocab_offset, vocab_offset + vocab): pairs[row] = (best value bits, global
// index), INT_MAX index when nothing compares (all NaN); greedy_merge picks over [ranks][rows] pairs.
int greedy_partial(float* logits, int rows, int vocab, int vocab_offset, const int32_t* past, const int32_t* past_len,
                   int past_cap, float penalty, int2* pairs, cudaStream_t s);
int greedy_merge(const int2* pairs, int ranks, int rows, int32_t* out, cudaStream_t s);
// Batched generation: out[b][*step] = tokens[b] = next[b]; pos[b]++ for b < B; then (*step)++.
int batch_advance(const int32_t* next, int32_t* tokens, int32_t* pos, int32_t* out, int out_stride, int32_t* step,
                  int B, cudaStream_t s);
// K/V rows [n][kvh][hd] (fp16 when half_input, else fp32) of positions start.. into the fp16 pools
// [page][kvh][slot][hd] through one page-table row.
int append_kv(const void* k, const void* v, int half_input, int n, int start, int kvh, int hd, const int32_t* pt_row,
              int max_pages, int page_size, __half* k_pool, __half* v_pool, cudaStream_t s);
// ctx_excl[b] = pos[b], ctx_incl[b] = pos[b] + 1 (the reference's per-layer causal lengths).
int causal_lengths(const int32_t* pos, int B, int32_t* ctx_excl, int32_t* ctx_incl, cudaStream_t s);
// Generation bookkeeping after a sampled step (B = 1): out[*step] = tok[0]; past[past_len] = tok[0];
// past_len++; pos[0]++; (*step)++ -- unless a stop token was already produced.
int advance_generation(const int32_t* tok, int32_t* pos, int32_t* out, int32_t* step, int32_t* past,
                       int32_t* past_len, int past_cap, int eos, int32_t* done, cudaStream_t s);

// ---- LlmSampler.Sample on the device (sampler.cu) ----
constexpr int SAMPLE_MAX_CAND = 4096;  // candidates kept after Top-K that one row can sort
struct SampleConfig {
  float temperature, top_p, min_p;
  int top_k;
  float penalty;
};
// Samples `rows` logit rows in place (the reference mutates its logits span); uniforms[row] stands for
// (float)random.NextDouble().  out[row] = token, or -1 when more than SAMPLE_MAX_CAND candidates survive Top-K.
// cand_idx / cand_p [rows][cand_cap] and n_cand (each may be null) receive the kept candidates, their renormalised
// probabilities and their count (0 on the greedy branch).
int sample_rows(float* logits, int rows, int vocab, const int32_t* past, const int32_t* past_len, int past_cap,
                const SampleConfig& cfg, const float* uniforms, int32_t* out, int32_t* cand_idx, float* cand_p,
                int32_t* n_cand, int cand_cap, cudaStream_t s);
// The same with a configuration and a draw per row (row_cfg[r], uniforms[r]) and row r's history in row
// past_rows[r] of past / past_len (null: row r).  Candidates are not reported.
int sample_rows_each(float* logits, int rows, int vocab, const int32_t* past, const int32_t* past_len, int past_cap,
                     const int32_t* past_rows, const SampleConfig* row_cfg, const float* uniforms, int32_t* out,
                     cudaStream_t s);
// Appends tok[r] to history row past_rows[r] (past [.][past_cap], past_len [.]) while it has room.
int append_history(const int32_t* tok, const int32_t* past_rows, int rows, int32_t* past, int32_t* past_len,
                   int past_cap, cudaStream_t s);
// u[r] = splitmix_uniform(seed + *counter + r) for r < rows (<= 1024); *counter += rows.
int draw_uniforms(uint64_t seed, int32_t* counter, int rows, float* u, cudaStream_t s);

// ---- one greedy generation step of one sequence as a single cooperative kernel (decode_fused.cu) ----
struct FusedLayerW {
  const int8_t* qkv_qs;
  const uint16_t* qkv_d;
  const int8_t* o_qs;
  const uint16_t* o_d;
  const int8_t* gu_qs;
  const uint16_t* gu_d;
  const int8_t* dn_qs;
  const uint16_t* dn_d;
};
struct FusedStepArgs {
  int dim, layers, hq, hkv, hd, ffn, vocab, q_dim, kv_dim, qkv_dim;
  float eps;
  const int8_t* emb_qs;
  const uint16_t* emb_d;
  const FusedLayerW* lw;  // [layers], device memory
  const float *attn_norm, *ffn_norm, *final_norm;
  const int8_t* lm_qs;
  const uint16_t* lm_d;
  const float *cos_t, *sin_t;
  int max_pos;
  __half *kpool, *vpool;  // [layers][pages][hkv][page_size][hd]
  size_t layer_pool_elems;
  int page_size, max_pages, num_pages;
  const int32_t* page_table;
  const int32_t* rows;  // rows[0]: the sequence's page-table row
  int32_t* pos;         // pos[0]: position of the token fed this step (advanced by the step)
  int quirk;            // the reference's causal rule (non-final layers attend to [0, pos))
  float* logits;        // [vocab]: read (sampled) at the start, written at the end
  int32_t* tokens;      // tokens[0] = the sampled token
  int32_t *gen_out, *gen_step, *past, *past_len, *done;
  int past_cap, eos;
  float penalty;
  // device scratch (fused_step_scratch_floats) and control words [3 + hq] (cleared by the launcher)
  float *x, *qbuf, *hbuf, *part, *P;
  int2* pairs;
  unsigned* ctl;
  int* status;
  // filled by fused_step_plan
  int splits, score_cap, dim_pad, vec_pad, row_cap, pt_pad;
  float scale_log2;
};
// kOk when the shapes fit the fused step on `sms` SMs (fills the plan fields and the shared-memory size), else
// kUnsupported with the reason in *why.
int fused_step_plan(FusedStepArgs& a, int sms, int max_ctx, size_t* smem, const char** why);
size_t fused_step_scratch_floats(const FusedStepArgs& a, int sms);
int fused_step_launch(const FusedStepArgs& a, int sms, size_t smem, cudaStream_t s);

int rope_tensorops(float* x, int heads, int seq, int hd, int pos0, float theta, cudaStream_t s);
int sgemm(int m, int n, int k, float alpha, const float* a, const float* b, float beta, float* c, cudaStream_t s);
int dot_i8(const int8_t* a, const int8_t* b, size_t n, int32_t* out, cudaStream_t s);

}  // namespace zc
