// engine.cu -- device decode engine: LlmEngine (ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs:19-568) over a
// device-resident paged KV cache (Memory/PagedKvCache.cs:47-286), for Q8_0 Llama-style models.
//
// Host side (C++): the page allocator (a free stack popped from the top, as Stack<int> in PagedKvCache), the
// sequence -> page-table-row map, weight upload/repack, and launch orchestration.  Device side: weights in the
// SoA layout with Wq|Wk|Wv and Wgate|Wup fused row-wise (one launch each; rows are independent, so the fused
// matrix computes exactly the separate products), fp16 K/V pools per layer [page][kv head][slot][hd], fp32
// activations.
//
// Step (one token per sequence, B sequences -- ForwardToken, LlmEngine.cs:347-461):
//   embed -> per layer: [RmsNorm + Wqkv] -> RoPE + KV append -> paged attention (per-layer causal length)
//   -> x += Wo.attn -> [RmsNorm + Wgate|Wup] -> [SwiGLU + x += Wdown.s] -> final [RmsNorm + LM head] -> greedy
// B = 1 uses the GEMV kernels with the RmsNorm / SwiGLU prologues fused; 1 < B < 9 one fp32 GEMV per row;
// B >= 9 and batched prefill the tcgen05 GEMM, whose fp16 hi / lo activation operands the kernels before it
// (RmsNorm, attention, SwiGLU) write directly.  Prefill of T > 1 tokens follows PrefillPrompt (:157-315): all T tokens per layer at once,
// K/V appended for all of them, then attention with causal length (l == L-1 ? pos + 1 : pos) per token.
// The reference's causal rule (non-final layers exclude the current token) is on by default; off gives the
// standard rule (pos + 1 everywhere).
// Greedy generation (GenerateStreamAsync, :71-150) runs as replays of one captured CUDA graph per token with
// the sampled token, position and outputs kept on the device (no host round trip per token).
//
// Tensor parallelism (tp_size > 1, one engine per GPU): every rank holds the query heads, K/V heads, FFN units
// and vocabulary rows that zcu_tp_plan assigns it.  Wq|Wk|Wv and Wgate|Wup are split by output rows, Wo and
// Wdown by input columns on 32-block boundaries, so each rank's Wo / Wdown product is a partial sum of the
// residual update: rank 0 adds its partial to x, the other ranks write theirs over x, and an all-reduce of
// x [T][dim] leaves x + sum(partials) on every rank (two per layer).  Up to max_batch rows it runs over NVLink
// peer memory (allreduce_p2p.cu; on the tensor-core path fused into the GEMM's split-K partials and the next
// RmsNorm), beyond that (prefill) as an in-place NCCL all-reduce.  Attention
// needs no exchange (whole heads and their pages stay on one rank; page tables are replicated because every
// rank runs the same allocator on the same calls).  Greedy sampling: each rank's arg-max over its vocabulary
// slice, an all-gather of (value, index) pairs, and a merge that keeps the lowest index on ties.

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <limits>
#include <map>
#include <string>
#include <vector>

#include "../../include/zero_tensor_cuda.h"
#include "allreduce_p2p.h"
#include "collective.h"
#include "common.cuh"
#include "kernels.h"

namespace zc {

// Message for zc_cuda_last_error() on the calling thread (capi.cu).
void set_last_error(const std::string& msg);

// Host-only shard plan (also exported as zcu_tp_plan).
int tp_plan(const zcu_engine_config& c, int tp, int rank, zcu_tp_shard* out, std::string* err) {
  if (tp < 1 || rank < 0 || rank >= tp || c.heads <= 0 || c.kv_heads <= 0 || c.dim % c.heads) {
    if (err) *err = "bad tp_size / tp_rank or head counts";
    return kBadArgument;
  }
  const int hd = c.dim / c.heads;
  if (c.heads % tp || c.kv_heads % tp) {
    if (err) *err = "heads and kv_heads must be multiples of tp_size";
    return kUnsupported;
  }
  const int hq = c.heads / tp, hkv = c.kv_heads / tp;
  if (tp > 1 && (hq * hd) % QK) {
    if (err) *err = "a rank's Wo column slice (heads/tp * head_dim) must be a multiple of 32";
    return kUnsupported;
  }
  const int ffn_blocks = c.ffn / QK;
  if (c.ffn % QK || ffn_blocks < tp || c.vocab < tp) {
    if (err) *err = "ffn must be a multiple of 32 with at least one 32-block, and one vocabulary row, per rank";
    return kUnsupported;
  }
  zcu_tp_shard s{};
  s.head_begin = rank * hq;
  s.heads = hq;
  s.kv_head_begin = rank * hkv;
  s.kv_heads = hkv;
  const int fb0 = (int)((long long)rank * ffn_blocks / tp), fb1 = (int)((long long)(rank + 1) * ffn_blocks / tp);
  s.ffn_begin = fb0 * QK;
  s.ffn = (fb1 - fb0) * QK;
  const int v0 = (int)((long long)rank * c.vocab / tp), v1 = (int)((long long)(rank + 1) * c.vocab / tp);
  s.vocab_begin = v0;
  s.vocab = v1 - v0;
  *out = s;
  return kOk;
}

namespace {

__global__ void add_one_kernel(int32_t* p) {
  if (threadIdx.x == 0 && blockIdx.x == 0) *p += 1;
}

struct DevW {
  int8_t* qs = nullptr;
  uint16_t* d = nullptr;
  int n = 0, k = 0;
};

struct Seq {
  int row = -1;                // row of the device page table
  std::vector<int> pages;      // physical page ids in logical order
  int len = 0;                 // tokens whose K/V are complete in every layer
};

// One request of the continuous batcher: GenerateStreamAsync's per-call state (LlmEngine.cs:71-152).
struct ServeReq {
  int seq_id = 0;
  std::vector<int32_t> prompt;
  int max_new = 0;
  SampleConfig sc{};
  uint64_t seed = 0;
  int eos = -1;
  std::vector<int32_t> stop;
  int generated = 0;   // tokens emitted
  int pending = -1;    // last sampled token, emitted and not yet run through the model
  int pos = 0;         // its position
  bool cancel = false;
};

// Continuous batching state: requests wait in `queue` (FIFO) until a page-table row and the pages for prompt +
// max_new tokens are free, then are prefilled and join every following decode step until they finish.
struct Serve {
  std::deque<ServeReq> queue;
  std::vector<ServeReq> active;
  std::vector<int> cancelled_queued;  // seq ids removed from the queue, reported at the next step
  int32_t* past = nullptr;            // device [max_batch][past_cap]: each page-table row's token history
  int32_t* past_len = nullptr;        // device [max_batch]
  int past_cap = 0;
  SampleConfig* cfg_dev = nullptr;    // device [max_batch]: the step's per-row sampling configurations
  float* u_dev = nullptr;             // device [max_batch]: the step's per-row draws
  int32_t* out_dev = nullptr;         // device [max_batch]: sampled tokens
  void* host = nullptr;               // pinned: tokens, pos, rows, out [max_batch] int32; u [max_batch]; cfg [max_batch]
  std::map<int, cudaGraphExec_t> graphs;  // decode step (embed, forward, sample, history) by batch size
};

struct Engine {
  zcu_engine_config cfg{};
  // tensor-parallel shard; hq / hkv / ffn / vocab are this rank's (the whole model's when tp_size == 1)
  int tp_rank = 0, tp_size = 1;
  zcu_tp_shard shard{};
  Comm* comm = nullptr;
  P2pAllReduce* arp = nullptr;  // NVLink peer-memory all-reduce of the residual stream (tp > 1); NCCL otherwise
  float* barrier_buf = nullptr;  // one float for rank_barrier
  int timeout_ms = 120000;
  int hq = 0, hkv = 0, ffn = 0, vocab = 0, vocab_chunk = 0;
  int hd = 0, q_dim = 0, kv_dim = 0, qkv_dim = 0;
  int prefill_row = -1;  // page-table row of the prompt in flight through forward(), else -1
  int prefill_attn_min_rows = 64;
  int device = 0;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  std::vector<void*> allocs;

  DevW tok_emb, lm_head;
  std::vector<DevW> wqkv, wo, wgu, wdown;
  float* final_norm = nullptr;
  float* attn_norm = nullptr;  // [L][dim]
  float* ffn_norm = nullptr;   // [L][dim]
  float* cos_t = nullptr;
  float* sin_t = nullptr;
  int max_pos = 0;
  __half* kpool = nullptr;  // [L][pages][hkv][P][hd]
  __half* vpool = nullptr;
  size_t layer_pool_elems = 0;

  int32_t* page_table = nullptr;  // [max_batch][max_pages_per_seq]
  int max_rows = 0;               // activation rows: max(max_batch, max_prefill_tokens)
  float *x = nullptr, *xn = nullptr, *qkv = nullptr, *attn = nullptr, *gu = nullptr, *sw = nullptr;
  __half* xh = nullptr;  // fp16 activations feeding the tensor-core GEMM: [R][2 * max(dim, q_dim, ffn)] (hi | lo)
  float* logits = nullptr;      // [max_batch][vocab] (this rank's vocabulary slice)
  float* logits_all = nullptr;  // [tp][max_batch * vocab_chunk] gathered slices (tp > 1)
  int2* pairs = nullptr;        // [max_batch] arg-max of this rank's slice (tp > 1)
  int2* pairs_all = nullptr;    // [tp][max_batch]
  void* stage = nullptr;        // upload staging buffer (grown on demand)
  size_t stage_bytes = 0;
  int32_t* batch_out = nullptr;  // [max_batch][gen_cap] tokens of zcu_engine_generate_batch
  int32_t* batch_step = nullptr;
  int32_t *tokens = nullptr, *pos = nullptr, *rows = nullptr, *ctx_ex = nullptr, *ctx_in = nullptr,
          *next = nullptr;
  float* attn_ws = nullptr;
  int* attn_ctr = nullptr;
  int attn_splits = 1;
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  int* status = nullptr;
  // generation state (B = 1)
  int32_t *gen_out = nullptr, *gen_step = nullptr, *gen_past = nullptr, *gen_past_len = nullptr,
          *gen_done = nullptr;
  int32_t* rng_ctr = nullptr;  // draws taken by sampled generation (allocated at its first call)
  float* uni = nullptr;        // the step's draw
  int gen_cap = 0;

  std::vector<int> free_stack;
  std::vector<int> free_rows;
  std::map<int, Seq> seqs;
  // one-kernel generation step (decode_fused.cu) for one sequence on one GPU, set up at the first generate
  bool fused_tried = false, fused_ok = false;
  FusedStepArgs fused{};
  size_t fused_smem = 0;
  int fused_sms = 0;
  std::string fused_why;
  std::map<int, cudaGraphExec_t> step_graphs;   // decode step graphs (B = 1 generation)
  std::map<int, cudaGraphExec_t> batch_graphs;  // batched generation step graphs, by batch size
  Serve* serve = nullptr;                       // continuous batching (zcu_engine_submit / serve_step)
  std::string err;
};

#define E_CUDA(call)                                             \
  do {                                                           \
    cudaError_t e_ = (call);                                     \
    if (e_ != cudaSuccess) {                                     \
      E->err = std::string(#call ": ") + cudaGetErrorString(e_); \
      return kCudaError;                                         \
    }                                                            \
  } while (0)

#define E_RC(call)                           \
  do {                                       \
    int rc_ = (call);                        \
    if (rc_ != kOk) {                        \
      if (E->err.empty()) E->err = #call;    \
      return rc_;                            \
    }                                        \
  } while (0)

template <class T>
int dalloc(Engine* E, T** p, size_t count) {
  void* v = nullptr;
  if (cudaMalloc(&v, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) {
    cudaGetLastError();
    E->err = "device allocation failed";
    return kOutOfMemory;
  }
  E->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return kOk;
}

int alloc_weight(Engine* E, DevW& w, int n, int k) {
  w.n = n;
  w.k = k;
  E_RC(dalloc(E, &w.qs, (size_t)n * k));
  E_RC(dalloc(E, &w.d, (size_t)n * (k / QK)));
  return kOk;
}

// Below this many rows a batched linear runs as one fp32 GEMV per row -- exactly the reference's token-parallel
// MatVec loop -- and above it on the fp16 tensor cores.
constexpr int kGemmMinRows = 9;

// y (=|+=) W x for `rows` activation rows.
int linear(Engine* E, const DevW& w, const float* x, float* y, int rows, int accumulate) {
  if (rows < kGemmMinRows) {
    for (int r = 0; r < rows; ++r) {
      const int rc = gemv_q8_0(w.qs, w.d, x + (size_t)r * w.k, y + (size_t)r * w.n, w.n, w.k, accumulate, E->stream);
      if (rc != kOk) return rc;
    }
    return kOk;
  }
  return gemm_q8_0_tc(w.qs, w.d, x, y, rows, w.n, w.k, accumulate, E->gemm_ws, E->gemm_ws_bytes, E->status,
                      E->stream);
}

// The same on fp16 activations written by the previous kernel (rows >= kGemmMinRows: the tensor-core GEMM).
// xh rows are [hi k | lo k] as the fp16 producers write them.
int linear_h(Engine* E, const DevW& w, const __half* xh, float* y, int rows, int accumulate) {
  return gemm_q8_0_tc_h(w.qs, w.d, xh, xh + w.k, 2 * w.k, y, rows, w.n, w.k, accumulate, E->gemm_ws,
                        E->gemm_ws_bytes, E->status, E->stream);
}

// Rows of one sequence's prompt (E->prefill_row >= 0) at least E->prefill_attn_min_rows (64; the environment
// variable ZCU_PREFILL_ATTN_MIN_ROWS overrides it at engine creation, 0 = never): the tiled prefill kernel, which
// reads each key once per 32 query rows; otherwise the decode kernel, which splits each row's context across CTAs.
int prefill_attn_min_rows_from_env() {
  const char* env = std::getenv("ZCU_PREFILL_ATTN_MIN_ROWS");
  if (!env || !*env) return 64;
  const int v = std::atoi(env);
  return v <= 0 ? std::numeric_limits<int>::max() : v;
}

int attention(Engine* E, int layer, int T, const int32_t* ctx, bool half_out) {
  if (E->prefill_row >= 0 && T >= E->prefill_attn_min_rows) {
    PrefillAttnArgs p{};
    p.q = E->qkv;
    p.k = E->kpool + (size_t)layer * E->layer_pool_elems;
    p.v = E->vpool + (size_t)layer * E->layer_pool_elems;
    p.page_table = E->page_table + (size_t)E->prefill_row * E->cfg.max_pages_per_seq;
    p.ctx_len = ctx;
    p.out = half_out ? reinterpret_cast<float*>(E->xh) : E->attn;
    p.rows = T;
    p.seqs = 1;
    p.hq = E->hq;
    p.group = E->hq / E->hkv;
    p.hd = E->hd;
    p.page_size = E->cfg.page_size;
    p.max_pages = E->cfg.max_pages_per_seq;
    p.num_pages = E->cfg.total_pages;
    p.page_stride = (long long)E->hkv * E->cfg.page_size * E->hd;
    p.slot_stride = E->hd;
    p.head_stride = (long long)E->cfg.page_size * E->hd;
    p.q_row_stride = E->qkv_dim;
    p.q_head_stride = E->hd;
    p.out_row_stride = half_out ? 2 * E->q_dim : E->q_dim;  // fp16 rows are [hi q_dim | lo q_dim]
    p.out_head_stride = E->hd;
    p.out_half = half_out ? 1 : 0;
    p.out_lo_offset = E->q_dim;
    p.scale_log2 = (1.0f / (float)std::sqrt((double)E->hd)) * 1.4426950408889634f;  // GqaAttention.cs:45
    p.kv_half = 1;
    return prefill_attention(p, E->stream);
  }
  PagedAttnArgs a{};
  a.out_half = half_out ? 1 : 0;
  a.q = E->qkv;
  a.k_pool = E->kpool + (size_t)layer * E->layer_pool_elems;
  a.v_pool = E->vpool + (size_t)layer * E->layer_pool_elems;
  a.page_table = E->page_table;
  a.pt_rows = E->rows;
  a.ctx_len = ctx;
  a.out = half_out ? reinterpret_cast<float*>(E->xh) : E->attn;
  a.batch = T;
  a.hq = E->hq;
  a.hkv = E->hkv;
  a.hd = E->hd;
  a.page_size = E->cfg.page_size;
  a.max_pages = E->cfg.max_pages_per_seq;
  a.num_pages = E->cfg.total_pages;
  a.page_stride = (long long)E->hkv * E->cfg.page_size * E->hd;
  a.slot_stride = E->hd;
  a.head_stride = (long long)E->cfg.page_size * E->hd;
  a.scale = 1.0f / (float)std::sqrt((double)E->hd);  // GqaAttention.cs:45
  a.kv_half = 1;
  a.max_ctx = E->cfg.max_pages_per_seq * E->cfg.page_size;
  a.q_stride = E->qkv_dim;
  a.out_stride = half_out ? 2 * E->q_dim : E->q_dim;  // fp16 rows are [hi q_dim | lo q_dim]
  a.out_lo_offset = E->q_dim;
  a.workspace = E->attn_ws;
  a.counters = E->attn_ctr;
  a.splits = (T <= E->cfg.max_batch) ? E->attn_splits : 1;
  return paged_attention(a, E->stream);
}

// Residual update of a row-split projection: rank 0 adds its partial to x, the others overwrite x with theirs.
inline int residual_mode(const Engine* E) { return E->tp_rank == 0 ? 1 : 0; }

int allreduce_x(Engine* E, int T) {
  const size_t n = (size_t)T * E->cfg.dim;
  if (E->arp && n <= arp_capacity(E->arp)) return arp_allreduce_sum(E->arp, E->x, n, E->stream);
  return comm_allreduce_sum_f32(E->comm, E->x, n, E->stream, &E->err);
}

// Tensor-parallel row-split projection whose all-reduce is fused around it: the GEMM leaves its split-K
// partials, and the push kernel sums them (rank 0 adding the residual x) straight into every rank's all-reduce
// slot; the caller follows with arp_reduce_rmsnorm_h.
int linear_push(Engine* E, const DevW& w, int rows) {
  float* part = nullptr;
  int splits = 0;
  E_RC(gemm_q8_0_tc_h_partials(w.qs, w.d, E->xh, E->xh + w.k, 2 * w.k, rows, w.n, w.k, E->gemm_ws, E->gemm_ws_bytes,
                               E->status, E->stream, &part, &splits));
  return arp_push_partials(E->arp, part, splits, (size_t)rows * w.n, residual_mode(E) ? E->x : nullptr, E->stream);
}

// Wgate|Wup on the tensor cores and SwiGLU into E->xh (fp16 hi / lo), with the split-K sum folded into the
// SwiGLU kernel when `parts`.
int gate_up_swiglu(Engine* E, int l, int T, bool parts) {
  if (!parts) {
    E_RC(linear_h(E, E->wgu[l], E->xh, E->gu, T, 0));
    return swiglu_rows_h(E->gu, E->xh, T, E->ffn, E->stream);
  }
  const DevW& w = E->wgu[l];
  float* part = nullptr;
  int splits = 0;
  E_RC(gemm_q8_0_tc_h_partials(w.qs, w.d, E->xh, E->xh + w.k, 2 * w.k, T, w.n, w.k, E->gemm_ws, E->gemm_ws_bytes,
                               E->status, E->stream, &part, &splits));
  return swiglu_rows_h_parts(part, splits, E->xh, T, E->ffn, E->stream);
}

// The forward pass over T activation rows already embedded in E->x, with tokens' positions in E->pos and
// page-table rows in E->rows.  Leaves the last row's logits (or every row's when all_logits) of this rank's
// vocabulary slice in E->logits.
int forward(Engine* E, int T, bool all_logits) {
  const zcu_engine_config& c = E->cfg;
  const int L = c.layers;
  const int acc = residual_mode(E);
  E_RC(causal_lengths(E->pos, T, E->ctx_ex, E->ctx_in, E->stream));
  // T >= kGemmMinRows: every projection runs on the tensor cores and its input is written in fp16 by the
  // kernel before it (RmsNorm, attention, SwiGLU); 1 < T < kGemmMinRows: fp32 GEMVs per row; T == 1: the
  // fused GEMVs.
  const bool tc = T >= kGemmMinRows;
  // tensor parallel on the tensor cores with rows that fit the peer all-reduce: the Wo / Wdown all-reduces are
  // fused into the kernels around them (linear_push, then arp_reduce_rmsnorm_h, which also writes the next
  // RmsNorm's fp16 operand)
  const bool fused = tc && E->arp && (size_t)T * c.dim <= arp_capacity(E->arp);
  // decode batches (at most 128 rows, where the GEMM's split-K partials have room in its workspace): the
  // Wqkv and Wgate|Wup partials go straight into the RoPE / K-V append and SwiGLU kernels
  const bool parts = tc && T <= 128;
  bool normed = false;  // E->xh already holds the next RmsNorm's output (written by arp_reduce_rmsnorm_h)
  for (int l = 0; l < L; ++l) {
    const float* an = E->attn_norm + (size_t)l * c.dim;
    const float* fn = E->ffn_norm + (size_t)l * c.dim;
    if (T == 1) {
      E_RC(gemv_q8_0_rmsnorm(E->wqkv[l].qs, E->wqkv[l].d, E->x, an, c.eps, E->qkv, E->qkv_dim, c.dim, 0, E->stream));
    } else if (tc) {
      if (!normed) E_RC(rmsnorm_h(E->x, an, E->xh, T, c.dim, c.eps, E->stream));
      if (parts) {  // the split-K sum is folded into the RoPE / K-V append kernel
        float* part = nullptr;
        int splits = 0;
        const DevW& w = E->wqkv[l];
        E_RC(gemm_q8_0_tc_h_partials(w.qs, w.d, E->xh, E->xh + w.k, 2 * w.k, T, w.n, w.k, E->gemm_ws,
                                     E->gemm_ws_bytes, E->status, E->stream, &part, &splits));
        E_RC(rope_append_kv_parts(part, splits, E->qkv, T, E->hq, E->hkv, E->hd, E->pos, E->rows, E->page_table,
                                  c.max_pages_per_seq, c.page_size, E->cos_t, E->sin_t, E->max_pos,
                                  E->kpool + (size_t)l * E->layer_pool_elems,
                                  E->vpool + (size_t)l * E->layer_pool_elems, E->stream));
      } else {
        E_RC(linear_h(E, E->wqkv[l], E->xh, E->qkv, T, 0));
      }
    } else {
      E_RC(rmsnorm(E->x, an, E->xn, T, c.dim, c.eps, E->stream));
      E_RC(linear(E, E->wqkv[l], E->xn, E->qkv, T, 0));
    }
    if (!(tc && parts))
      E_RC(rope_append_kv(E->qkv, T, E->hq, E->hkv, E->hd, E->pos, E->rows, E->page_table, c.max_pages_per_seq,
                          c.page_size, E->cos_t, E->sin_t, E->max_pos, E->kpool + (size_t)l * E->layer_pool_elems,
                          E->vpool + (size_t)l * E->layer_pool_elems, E->stream));
    const int32_t* ctx = (c.reference_causal_quirk && l != L - 1) ? E->ctx_ex : E->ctx_in;
    E_RC(attention(E, l, T, ctx, tc));
    if (fused) {
      E_RC(linear_push(E, E->wo[l], T));  // x += Wo . attn, summed over ranks
      E_RC(arp_reduce_rmsnorm_h(E->arp, E->x, fn, c.eps, E->xh, T, c.dim, E->stream));
      E_RC(gate_up_swiglu(E, l, T, parts));
      E_RC(linear_push(E, E->wdown[l], T));  // x += Wdown . s, summed over ranks
      const float* next_norm = l + 1 < L ? E->attn_norm + (size_t)(l + 1) * c.dim : E->final_norm;
      E_RC(arp_reduce_rmsnorm_h(E->arp, E->x, next_norm, c.eps, E->xh, T, c.dim, E->stream));
      normed = true;
      continue;
    }
    if (tc)
      E_RC(linear_h(E, E->wo[l], E->xh, E->x, T, acc));  // x += Wo . attn (MatVecAddQ8_0)
    else
      E_RC(linear(E, E->wo[l], E->attn, E->x, T, acc));
    E_RC(allreduce_x(E, T));
    if (T == 1) {
      E_RC(gemv_q8_0_rmsnorm(E->wgu[l].qs, E->wgu[l].d, E->x, fn, c.eps, E->gu, 2 * E->ffn, c.dim, 0, E->stream));
      E_RC(gemv_q8_0_swiglu(E->wdown[l].qs, E->wdown[l].d, E->gu, E->x, c.dim, E->ffn, acc, E->stream));
    } else if (tc) {
      E_RC(rmsnorm_h(E->x, fn, E->xh, T, c.dim, c.eps, E->stream));
      E_RC(gate_up_swiglu(E, l, T, parts));
      E_RC(linear_h(E, E->wdown[l], E->xh, E->x, T, acc));
    } else {
      E_RC(rmsnorm(E->x, fn, E->xn, T, c.dim, c.eps, E->stream));
      E_RC(linear(E, E->wgu[l], E->xn, E->gu, T, 0));
      E_RC(swiglu_rows(E->gu, E->sw, T, E->ffn, E->stream));
      E_RC(linear(E, E->wdown[l], E->sw, E->x, T, acc));
    }
    E_RC(allreduce_x(E, T));
  }
  if (all_logits && T > 1) {
    if (tc) {
      if (!normed) E_RC(rmsnorm_h(E->x, E->final_norm, E->xh, T, c.dim, c.eps, E->stream));
      E_RC(linear_h(E, E->lm_head, E->xh, E->logits, T, 0));
    } else {
      E_RC(rmsnorm(E->x, E->final_norm, E->xn, T, c.dim, c.eps, E->stream));
      E_RC(linear(E, E->lm_head, E->xn, E->logits, T, 0));
    }
  } else {  // LM head only for the last row (PrefillPrompt, LlmEngine.cs:307-314)
    const float* xl = E->x + (size_t)(T - 1) * c.dim;
    E_RC(gemv_q8_0_rmsnorm(E->lm_head.qs, E->lm_head.d, xl, E->final_norm, c.eps, E->logits, E->vocab, c.dim, 0,
                           E->stream));
  }
  return kOk;
}

// Greedy next token of `rows` logit rows (this rank's slices) into out; tp > 1 merges the ranks' arg-maxes.
int sample(Engine* E, int rows, const int32_t* past, const int32_t* past_len, int past_cap, float penalty,
           int32_t* out) {
  if (E->tp_size == 1) return greedy_sample(E->logits, rows, E->vocab, past, past_len, past_cap, penalty, out, E->stream);
  E_RC(greedy_partial(E->logits, rows, E->vocab, E->shard.vocab_begin, past, past_len, past_cap, penalty, E->pairs,
                      E->stream));
  E_RC(comm_allgather_bytes(E->comm, E->pairs, E->pairs_all, (size_t)rows * sizeof(int2), E->stream, &E->err));
  return greedy_merge(E->pairs_all, E->tp_size, rows, out, E->stream);
}

// Copies `rows` rows of full-vocabulary logits to host memory (gathering the ranks' slices when tp > 1).
int logits_to_host(Engine* E, int rows, float* host) {
  const int V = E->cfg.vocab;
  if (E->tp_size == 1) {
    E_CUDA(cudaMemcpyAsync(host, E->logits, (size_t)rows * V * 4, cudaMemcpyDeviceToHost, E->stream));
    return kOk;
  }
  const size_t chunk = (size_t)rows * E->vocab_chunk;
  E_RC(comm_allgather_bytes(E->comm, E->logits, E->logits_all, chunk * 4, E->stream, &E->err));
  std::vector<float> all(chunk * E->tp_size);
  E_CUDA(cudaMemcpyAsync(all.data(), E->logits_all, all.size() * 4, cudaMemcpyDeviceToHost, E->stream));
  E_RC(comm_wait(E->comm, E->stream, E->timeout_ms, &E->err));
  for (int r = 0; r < E->tp_size; ++r) {
    zcu_tp_shard sh{};
    E_RC(tp_plan(E->cfg, E->tp_size, r, &sh, &E->err));
    for (int b = 0; b < rows; ++b)
      std::memcpy(host + (size_t)b * V + sh.vocab_begin, all.data() + r * chunk + (size_t)b * sh.vocab, sh.vocab * 4);
  }
  return kOk;
}

int wait(Engine* E) { return comm_wait(E->comm, E->stream, E->timeout_ms, &E->err); }

// Brings every rank's host thread to the same point (after per-rank host work such as graph capture, before
// kernels that wait on their peers): a one-float NCCL all-reduce, waited for.
int rank_barrier(Engine* E) {
  if (E->tp_size == 1) return kOk;
  E_RC(comm_allreduce_sum_f32(E->comm, E->barrier_buf, 1, E->stream, &E->err));
  return wait(E);
}

// Pages covering positions [0, upto) of a sequence; allocates from the free stack and updates the device row.
int ensure_pages(Engine* E, Seq& s, int upto) {
  const int P = E->cfg.page_size;
  const int need = (upto + P - 1) / P;
  if (need > E->cfg.max_pages_per_seq) {
    E->err = "sequence longer than max_pages_per_seq * page_size";
    return kTooLarge;
  }
  const int have = (int)s.pages.size();
  if (need <= have) return kOk;
  if ((int)E->free_stack.size() < need - have) {
    E->err = "Paged KV-cache exhausted";
    return kTooLarge;
  }
  for (int i = have; i < need; ++i) {
    s.pages.push_back(E->free_stack.back());
    E->free_stack.pop_back();
  }
  E_CUDA(cudaMemcpyAsync(E->page_table + (size_t)s.row * E->cfg.max_pages_per_seq + have, s.pages.data() + have,
                         (size_t)(need - have) * sizeof(int32_t), cudaMemcpyHostToDevice, E->stream));
  return kOk;
}

int get_seq(Engine* E, int seq_id, Seq** out) {
  auto it = E->seqs.find(seq_id);
  if (it == E->seqs.end()) {
    if (E->free_rows.empty()) {
      E->err = "more live sequences than max_batch";
      return kTooLarge;
    }
    Seq s;
    s.row = E->free_rows.back();
    E->free_rows.pop_back();
    it = E->seqs.emplace(seq_id, s).first;
  }
  *out = &it->second;
  return kOk;
}

int stage(Engine* E, size_t bytes, void** out) {
  if (bytes > E->stage_bytes) {
    if (E->stage) {
      cudaStreamSynchronize(E->stream);
      cudaFree(E->stage);
      E->stage = nullptr;
      E->stage_bytes = 0;
    }
    if (cudaMalloc(&E->stage, bytes) != cudaSuccess) {
      cudaGetLastError();
      E->err = "staging allocation failed";
      return kOutOfMemory;
    }
    E->stage_bytes = bytes;
  }
  *out = E->stage;
  return kOk;
}

// Rows [r0, r0 + nr) x 32-blocks [b0, b0 + nb) of a full Q8_0 tensor with `full_blocks` blocks per row (the
// reference's packed AoS blocks, in host or device memory) into rows dst_row.. of dst (dst.k == nb * 32).
int upload_q8(Engine* E, DevW& dst, size_t dst_row, const void* src, int full_blocks, int r0, int nr, int b0, int nb) {
  if (nb * QK != dst.k || dst_row + nr > (size_t)dst.n) {
    E->err = "weight slice does not match the engine's tensor";
    return kBadArgument;
  }
  void* aos = nullptr;
  E_RC(stage(E, (size_t)nr * nb * Q8_BLOCK_BYTES, &aos));
  const size_t row_bytes = (size_t)full_blocks * Q8_BLOCK_BYTES, part = (size_t)nb * Q8_BLOCK_BYTES;
  const char* base = static_cast<const char*>(src) + (size_t)r0 * row_bytes + (size_t)b0 * Q8_BLOCK_BYTES;
  if (part == row_bytes)
    E_CUDA(cudaMemcpyAsync(aos, base, part * nr, cudaMemcpyDefault, E->stream));
  else
    E_CUDA(cudaMemcpy2DAsync(aos, part, base, row_bytes, part, nr, cudaMemcpyDefault, E->stream));
  E_RC(repack_q8_0(static_cast<const uint8_t*>(aos), dst.qs + dst_row * dst.k, dst.d + dst_row * (dst.k / QK), nr,
                   dst.k, E->stream));
  E_CUDA(cudaStreamSynchronize(E->stream));
  return kOk;
}

// Sets up the one-kernel generation step when this engine's shapes fit it (tp_size 1; ZCU_FUSED_DECODE=0 in the
// environment keeps the captured multi-kernel step instead).  Leaves E->fused_ok false otherwise.
int setup_fused(Engine* E) {
  if (E->fused_tried) return kOk;
  E->fused_tried = true;
  const char* env = std::getenv("ZCU_FUSED_DECODE");
  if (env && env[0] == '0') {
    E->fused_why = "disabled by ZCU_FUSED_DECODE=0";
    return kOk;
  }
  if (E->tp_size != 1) {
    E->fused_why = "tensor parallel";
    return kOk;
  }
  const zcu_engine_config& c = E->cfg;
  FusedStepArgs& a = E->fused;
  a.dim = c.dim;
  a.layers = c.layers;
  a.hq = E->hq;
  a.hkv = E->hkv;
  a.hd = E->hd;
  a.ffn = E->ffn;
  a.vocab = E->vocab;
  a.q_dim = E->q_dim;
  a.kv_dim = E->kv_dim;
  a.qkv_dim = E->qkv_dim;
  a.eps = c.eps;
  a.page_size = c.page_size;
  a.max_pages = c.max_pages_per_seq;
  a.num_pages = c.total_pages;
  int sms = 0;
  E_CUDA(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, E->device));
  const char* why = nullptr;
  if (fused_step_plan(a, sms, c.max_pages_per_seq * c.page_size, &E->fused_smem, &why) != kOk) {
    E->fused_why = why ? why : "unsupported shape";
    return kOk;
  }
  std::vector<FusedLayerW> lw(c.layers);
  for (int l = 0; l < c.layers; ++l)
    lw[l] = FusedLayerW{E->wqkv[l].qs, E->wqkv[l].d, E->wo[l].qs, E->wo[l].d,
                        E->wgu[l].qs,  E->wgu[l].d,  E->wdown[l].qs, E->wdown[l].d};
  FusedLayerW* dlw = nullptr;
  E_RC(dalloc(E, &dlw, lw.size()));
  E_CUDA(cudaMemcpy(dlw, lw.data(), lw.size() * sizeof(FusedLayerW), cudaMemcpyHostToDevice));
  float* scratch = nullptr;
  E_RC(dalloc(E, &scratch, fused_step_scratch_floats(a, sms)));
  unsigned* ctl = nullptr;
  E_RC(dalloc(E, &ctl, (size_t)(3 + a.hq)));
  E_CUDA(cudaMemset(ctl, 0, (3 + a.hq) * sizeof(unsigned)));
  a.part = scratch;
  a.P = a.part + (size_t)a.hq * a.splits * (a.hd + 2);
  a.qbuf = a.P + (size_t)a.hq * a.dim;
  a.hbuf = a.qbuf + a.q_dim;
  a.x = a.hbuf + a.ffn;
  a.pairs = reinterpret_cast<int2*>(a.x + ((a.dim + 3) / 4 * 4));
  a.ctl = ctl;
  a.lw = dlw;
  a.emb_qs = E->tok_emb.qs;
  a.emb_d = E->tok_emb.d;
  a.attn_norm = E->attn_norm;
  a.ffn_norm = E->ffn_norm;
  a.final_norm = E->final_norm;
  a.lm_qs = E->lm_head.qs;
  a.lm_d = E->lm_head.d;
  a.cos_t = E->cos_t;
  a.sin_t = E->sin_t;
  a.max_pos = E->max_pos;
  a.kpool = E->kpool;
  a.vpool = E->vpool;
  a.layer_pool_elems = E->layer_pool_elems;
  a.page_size = c.page_size;
  a.max_pages = c.max_pages_per_seq;
  a.num_pages = c.total_pages;
  a.page_table = E->page_table;
  a.rows = E->rows;
  a.pos = E->pos;
  a.quirk = c.reference_causal_quirk ? 1 : 0;
  a.logits = E->logits;
  a.tokens = E->tokens;
  a.gen_out = E->gen_out;
  a.gen_step = E->gen_step;
  a.past = E->gen_past;
  a.past_len = E->gen_past_len;
  a.done = E->gen_done;
  a.past_cap = E->gen_cap;
  a.status = E->status;
  E->fused_sms = sms;
  E->fused_ok = true;
  return kOk;
}

int capture_gen_step(Engine* E, float penalty, int eos, cudaGraphExec_t* out) {
  cudaGraph_t g;
  E_CUDA(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  int rc = sample(E, 1, E->gen_past, E->gen_past_len, E->gen_cap, penalty, E->tokens);
  if (rc == kOk)
    rc = advance_generation(E->tokens, E->pos, E->gen_out, E->gen_step, E->gen_past, E->gen_past_len, E->gen_cap, eos,
                            E->gen_done, E->stream);
  if (rc == kOk) rc = embed_q8_0(E->tok_emb.qs, E->tok_emb.d, E->tokens, 1, E->cfg.vocab, E->cfg.dim, E->x, E->stream);
  if (rc == kOk) rc = forward(E, 1, false);
  if (rc == kOk) {
    add_one_kernel<<<1, 32, 0, E->stream>>>(E->pos);
    if (cudaPeekAtLastError() != cudaSuccess) rc = kCudaError;
  }
  cudaError_t ce = cudaStreamEndCapture(E->stream, &g);
  if (rc != kOk) return rc;
  E_CUDA(ce);
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  E_CUDA(ce);
  return kOk;
}

// One step of sampled generation (B = 1): draw -> LlmSampler.Sample on the previous logits -> advance -> embed ->
// forward -> pos++.
int capture_sampled_step(Engine* E, const SampleConfig& sc, uint64_t seed, int eos, cudaGraphExec_t* out) {
  cudaGraph_t g;
  E_CUDA(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  int rc = draw_uniforms(seed, E->rng_ctr, 1, E->uni, E->stream);
  if (rc == kOk)
    rc = sample_rows(E->logits, 1, E->vocab, E->gen_past, E->gen_past_len, E->gen_cap, sc, E->uni, E->tokens, nullptr,
                     nullptr, nullptr, 0, E->stream);
  if (rc == kOk)
    rc = advance_generation(E->tokens, E->pos, E->gen_out, E->gen_step, E->gen_past, E->gen_past_len, E->gen_cap, eos,
                            E->gen_done, E->stream);
  if (rc == kOk) rc = embed_q8_0(E->tok_emb.qs, E->tok_emb.d, E->tokens, 1, E->cfg.vocab, E->cfg.dim, E->x, E->stream);
  if (rc == kOk) rc = forward(E, 1, false);
  if (rc == kOk) {
    add_one_kernel<<<1, 32, 0, E->stream>>>(E->pos);
    if (cudaPeekAtLastError() != cudaSuccess) rc = kCudaError;
  }
  cudaError_t ce = cudaStreamEndCapture(E->stream, &g);
  if (rc != kOk) return rc;
  E_CUDA(ce);
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  E_CUDA(ce);
  return kOk;
}

// One step of batched generation for B sequences: embed E->tokens -> forward -> greedy -> advance.
int capture_batch_step(Engine* E, int B, cudaGraphExec_t* out) {
  cudaGraph_t g;
  E_CUDA(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  int rc = embed_q8_0(E->tok_emb.qs, E->tok_emb.d, E->tokens, B, E->cfg.vocab, E->cfg.dim, E->x, E->stream);
  if (rc == kOk) rc = forward(E, B, B > 1);
  if (rc == kOk) rc = sample(E, B, nullptr, nullptr, 0, 1.0f, E->next);
  if (rc == kOk) rc = batch_advance(E->next, E->tokens, E->pos, E->batch_out, E->gen_cap, E->batch_step, B, E->stream);
  cudaError_t ce = cudaStreamEndCapture(E->stream, &g);
  if (rc != kOk) return rc;
  E_CUDA(ce);
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  E_CUDA(ce);
  return kOk;
}

// Continuous batching: one decode step of B running requests, rows [0, B) of E->tokens / pos / rows (uploaded
// before each launch), each sampled with its own configuration and draw and its token appended to its history.
int capture_serve_step(Engine* E, int B, cudaGraphExec_t* out) {
  Serve* S = E->serve;
  cudaGraph_t g;
  E_CUDA(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  int rc = embed_q8_0(E->tok_emb.qs, E->tok_emb.d, E->tokens, B, E->cfg.vocab, E->cfg.dim, E->x, E->stream);
  if (rc == kOk) rc = forward(E, B, B > 1);
  if (rc == kOk)
    rc = sample_rows_each(E->logits, B, E->vocab, S->past, S->past_len, S->past_cap, E->rows, S->cfg_dev, S->u_dev,
                          S->out_dev, E->stream);
  if (rc == kOk) rc = append_history(S->out_dev, E->rows, B, S->past, S->past_len, S->past_cap, E->stream);
  cudaError_t ce = cudaStreamEndCapture(E->stream, &g);
  if (rc != kOk) return rc;
  E_CUDA(ce);
  ce = cudaGraphInstantiate(out, g, 0);
  cudaGraphDestroy(g);
  E_CUDA(ce);
  return kOk;
}

int serve_init(Engine* E) {
  if (E->serve) return kOk;
  const int B = E->cfg.max_batch;
  Serve* S = new Serve();
  S->past_cap = E->cfg.max_pages_per_seq * E->cfg.page_size;
  int rc = dalloc(E, &S->past, (size_t)B * S->past_cap);
  if (rc == kOk) rc = dalloc(E, &S->past_len, B);
  if (rc == kOk) rc = dalloc(E, &S->cfg_dev, B);
  if (rc == kOk) rc = dalloc(E, &S->u_dev, B);
  if (rc == kOk) rc = dalloc(E, &S->out_dev, B);
  if (rc == kOk && cudaMallocHost(&S->host, (size_t)B * (5 * 4 + sizeof(SampleConfig))) != cudaSuccess) {
    cudaGetLastError();
    S->host = nullptr;
    E->err = "pinned host allocation failed";
    rc = kOutOfMemory;
  }
  if (rc != kOk) {
    delete S;
    return rc;
  }
  E->serve = S;
  return kOk;
}

// The draw of a request's i-th token: the one sampled generation uses (zcu_sample_uniform).
inline float serve_uniform(uint64_t seed, uint64_t i) { return splitmix_uniform(seed + i); }

// Pinned host views: [tokens | pos | rows | out] int32 [max_batch] each, u float [max_batch], cfg [max_batch].
struct ServeHost {
  int32_t *tokens, *pos, *rows, *out;
  float* u;
  SampleConfig* cfg;
};
ServeHost serve_host(Engine* E) {
  const int B = E->cfg.max_batch;
  char* h = static_cast<char*>(E->serve->host);
  ServeHost v;
  v.tokens = reinterpret_cast<int32_t*>(h);
  v.pos = v.tokens + B;
  v.rows = v.pos + B;
  v.out = v.rows + B;
  v.u = reinterpret_cast<float*>(v.out + B);
  v.cfg = reinterpret_cast<SampleConfig*>(v.u + B);
  return v;
}

// A token sampled for request r: decides whether it ends the request (GenerateStreamAsync's loop: a stop token
// ends it unemitted; MaxTokens ends it after the token) and records the event.
void serve_take(ServeReq& r, int tok, std::vector<zcu_serve_event>* ev, bool* done) {
  zcu_serve_event e{r.seq_id, tok, 0, ZCU_SERVE_RUNNING};
  *done = false;
  if (tok < 0) {
    e.finished = 1;
    e.reason = ZCU_SERVE_REFUSED;
    *done = true;
  } else if (tok == r.eos || std::find(r.stop.begin(), r.stop.end(), tok) != r.stop.end()) {
    e.finished = 1;
    e.reason = ZCU_SERVE_STOP_TOKEN;
    *done = true;
  } else {
    ++r.generated;
    r.pending = tok;
    if (r.generated >= r.max_new) {
      e.finished = 1;
      e.reason = ZCU_SERVE_MAX_TOKENS;
      *done = true;
    }
  }
  ev->push_back(e);
}

}  // namespace

}  // namespace zc

using zc::Engine;

extern "C" {

int32_t zcu_tp_plan(const zcu_engine_config* cfg, int32_t tp_size, int32_t tp_rank, zcu_tp_shard* out) {
  if (!cfg || !out) return zc::kBadArgument;
  std::string err;
  return zc::tp_plan(*cfg, tp_size, tp_rank, out, &err);
}

int32_t zcu_engine_create(const zcu_engine_config* cfg, void* stream, void** out) {
  return zcu_engine_create_tp(cfg, 1, 0, nullptr, stream, out);
}

int32_t zcu_engine_create_tp(const zcu_engine_config* cfg, int32_t tp_size, int32_t tp_rank, const uint8_t* nccl_id,
                             void* stream, void** out) {
  using namespace zc;
  if (!cfg || !out) return kBadArgument;
  const zcu_engine_config& c = *cfg;
  if (c.vocab <= 0 || c.dim <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.ffn <= 0 ||
      c.dim % c.heads || c.heads % c.kv_heads || c.dim % QK || c.ffn % QK || c.total_pages <= 0 || c.page_size <= 0 ||
      c.max_batch <= 0 || c.max_pages_per_seq <= 0 || c.max_prefill_tokens <= 0)
    return kBadArgument;
  const int hd = c.dim / c.heads;
  if (hd % 8 || (hd & (hd - 1)) || hd > 256) return kUnsupported;  // attention kernel head sizes
  zcu_tp_shard sh{};
  {
    std::string err;
    const int prc = tp_plan(c, tp_size, tp_rank, &sh, &err);
    if (prc != kOk) {
      set_last_error("zcu_engine_create_tp: " + err);
      return prc;
    }
  }
  Engine* E = new Engine();
  E->cfg = c;
  E->prefill_attn_min_rows = prefill_attn_min_rows_from_env();
  E->tp_size = tp_size;
  E->tp_rank = tp_rank;
  E->shard = sh;
  E->hq = sh.heads;
  E->hkv = sh.kv_heads;
  E->ffn = sh.ffn;
  E->vocab = sh.vocab;
  E->vocab_chunk = (c.vocab + tp_size - 1) / tp_size;
  E->hd = hd;
  E->q_dim = E->hq * hd;
  E->kv_dim = E->hkv * hd;
  E->qkv_dim = E->q_dim + 2 * E->kv_dim;
  if (const char* t = std::getenv("ZCU_COLLECTIVE_TIMEOUT_MS")) E->timeout_ms = std::max(1, std::atoi(t));
  cudaGetDevice(&E->device);
  if (stream) {
    E->stream = reinterpret_cast<cudaStream_t>(stream);
  } else {
    if (cudaStreamCreateWithFlags(&E->stream, cudaStreamNonBlocking) != cudaSuccess) {
      delete E;
      return kCudaError;
    }
    E->own_stream = true;
  }
  int rc = kOk;
  auto step = [&](int r) {
    if (rc == kOk) rc = r;
  };
  {
    std::string err;
    step(comm_create(tp_size, tp_rank, nccl_id, &E->comm, &err));
    if (rc != kOk) set_last_error("zcu_engine_create_tp: " + err);
  }
  const int L = c.layers;
  step(alloc_weight(E, E->tok_emb, c.vocab, c.dim));
  step(alloc_weight(E, E->lm_head, E->vocab, c.dim));
  E->wqkv.resize(L);
  E->wo.resize(L);
  E->wgu.resize(L);
  E->wdown.resize(L);
  for (int l = 0; l < L && rc == kOk; ++l) {
    step(alloc_weight(E, E->wqkv[l], E->qkv_dim, c.dim));
    step(alloc_weight(E, E->wo[l], c.dim, E->q_dim));
    step(alloc_weight(E, E->wgu[l], 2 * E->ffn, c.dim));
    step(alloc_weight(E, E->wdown[l], c.dim, E->ffn));
  }
  step(dalloc(E, &E->final_norm, c.dim));
  step(dalloc(E, &E->attn_norm, (size_t)L * c.dim));
  step(dalloc(E, &E->ffn_norm, (size_t)L * c.dim));
  // RoPE tables as RoPE.EnsureCache builds them (double precision, rounded to float), max(1024, ctx) rows
  E->max_pos = std::max(std::max(1024, c.context_length), c.max_pages_per_seq * c.page_size);
  {
    const int half = hd / 2;
    std::vector<float> ct((size_t)E->max_pos * half), st((size_t)E->max_pos * half);
    std::vector<double> freqs(half);
    for (int i = 0; i < half; ++i) freqs[i] = 1.0 / std::pow((double)c.rope_base, 2.0 * i / hd);
    for (int p = 0; p < E->max_pos; ++p)
      for (int i = 0; i < half; ++i) {
        const double th = p * freqs[i];
        ct[(size_t)p * half + i] = (float)std::cos(th);
        st[(size_t)p * half + i] = (float)std::sin(th);
      }
    step(dalloc(E, &E->cos_t, ct.size()));
    step(dalloc(E, &E->sin_t, st.size()));
    if (rc == kOk) {
      cudaMemcpy(E->cos_t, ct.data(), ct.size() * 4, cudaMemcpyHostToDevice);
      cudaMemcpy(E->sin_t, st.data(), st.size() * 4, cudaMemcpyHostToDevice);
    }
  }
  E->layer_pool_elems = (size_t)c.total_pages * E->hkv * c.page_size * hd;
  step(dalloc(E, &E->kpool, E->layer_pool_elems * L));
  step(dalloc(E, &E->vpool, E->layer_pool_elems * L));
  step(dalloc(E, &E->page_table, (size_t)c.max_batch * c.max_pages_per_seq));
  E->max_rows = std::max(c.max_batch, c.max_prefill_tokens);
  const int R = E->max_rows;
  step(dalloc(E, &E->x, (size_t)R * c.dim));
  step(dalloc(E, &E->xn, (size_t)R * c.dim));
  step(dalloc(E, &E->qkv, (size_t)R * E->qkv_dim));
  step(dalloc(E, &E->attn, (size_t)R * E->q_dim));
  step(dalloc(E, &E->gu, (size_t)R * 2 * E->ffn));
  step(dalloc(E, &E->sw, (size_t)R * E->ffn));
  step(dalloc(E, &E->xh, (size_t)R * 2 * std::max(std::max(c.dim, E->q_dim), E->ffn)));
  step(dalloc(E, &E->logits, (size_t)c.max_batch * E->vocab_chunk));
  if (tp_size > 1) {
    step(dalloc(E, &E->logits_all, (size_t)tp_size * c.max_batch * E->vocab_chunk));
    step(dalloc(E, &E->pairs, (size_t)std::max(c.max_batch, 1)));
    step(dalloc(E, &E->pairs_all, (size_t)tp_size * c.max_batch));
  }
  step(dalloc(E, &E->tokens, R));
  step(dalloc(E, &E->pos, R));
  step(dalloc(E, &E->rows, R));
  step(dalloc(E, &E->ctx_ex, R));
  step(dalloc(E, &E->ctx_in, R));
  step(dalloc(E, &E->next, R));
  E->attn_splits = paged_attention_choose_splits(c.max_batch, E->hkv, c.max_pages_per_seq * c.page_size, c.page_size);
  step(dalloc(E, &E->attn_ws, std::max<size_t>(16, paged_attention_workspace_floats(c.max_batch, E->hq, hd,
                                                                                   E->attn_splits))));
  step(dalloc(E, &E->attn_ctr, (size_t)R * E->hq));
  {  // the largest workspace any batched linear of this engine can ask for
    const int shapes[5][2] = {{E->qkv_dim, c.dim}, {c.dim, E->q_dim}, {2 * E->ffn, c.dim}, {c.dim, E->ffn},
                              {E->vocab, c.dim}};
    size_t ws = 0;
    for (auto& sh2 : shapes) ws = std::max(ws, gemm_workspace_max(R, sh2[0], sh2[1]));
    E->gemm_ws_bytes = std::max<size_t>(ws, 256);
  }
  step(dalloc(E, reinterpret_cast<uint8_t**>(&E->gemm_ws), E->gemm_ws_bytes));
  step(dalloc(E, &E->status, 1));
  E->gen_cap = c.max_pages_per_seq * c.page_size + 16;
  step(dalloc(E, &E->gen_out, E->gen_cap));
  step(dalloc(E, &E->gen_past, E->gen_cap));
  step(dalloc(E, &E->gen_step, 1));
  step(dalloc(E, &E->gen_past_len, 1));
  step(dalloc(E, &E->gen_done, 1));
  step(dalloc(E, &E->batch_out, (size_t)c.max_batch * E->gen_cap));
  step(dalloc(E, &E->batch_step, 1));
  step(dalloc(E, &E->barrier_buf, 1));
  if (rc == kOk) {
    cudaMemset(E->attn_ctr, 0, (size_t)R * E->hq * sizeof(int));
    cudaMemset(E->status, 0, sizeof(int));
    cudaMemset(E->page_table, 0xff, (size_t)c.max_batch * c.max_pages_per_seq * sizeof(int32_t));  // -1: no page
    cudaMemset(E->kpool, 0, E->layer_pool_elems * L * 2);
    cudaMemset(E->vpool, 0, E->layer_pool_elems * L * 2);
    std::vector<float> ones((size_t)L * c.dim, 1.0f);
    cudaMemcpy(E->attn_norm, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(E->ffn_norm, ones.data(), ones.size() * 4, cudaMemcpyHostToDevice);
    cudaMemcpy(E->final_norm, ones.data(), (size_t)c.dim * 4, cudaMemcpyHostToDevice);
    if (cudaDeviceSynchronize() != cudaSuccess) rc = kCudaError;
  }
  if (rc == kOk && tp_size > 1) {
    // the residual all-reduce of decode steps (up to max_batch rows) goes over peer memory when the GPUs have
    // peer access; larger ones (prefill) and systems without it use NCCL.  ZCU_TP_ALLREDUCE=nccl keeps every
    // all-reduce on NCCL (set it on every rank).
    std::string err;
    const char* ar = std::getenv("ZCU_TP_ALLREDUCE");
    const bool want_p2p = !(ar && std::string(ar) == "nccl");
    if (!want_p2p || arp_create(E->comm, (size_t)c.max_batch * c.dim, E->status, &E->arp, &err) != kOk)
      E->arp = nullptr;
    // every rank must take the same path: keep the peer all-reduce only if all ranks could map their peers
    float* ok = nullptr;
    if (cudaMalloc(&ok, sizeof(float)) == cudaSuccess) {
      const float mine = E->arp ? 1.0f : 0.0f;
      float sum = 0.f;
      cudaMemcpy(ok, &mine, sizeof(float), cudaMemcpyHostToDevice);
      if (comm_allreduce_sum_f32(E->comm, ok, 1, E->stream, &err) == kOk && cudaStreamSynchronize(E->stream) == cudaSuccess)
        cudaMemcpy(&sum, ok, sizeof(float), cudaMemcpyDeviceToHost);
      cudaFree(ok);
      if (sum != (float)tp_size && E->arp) {
        arp_destroy(E->arp);
        E->arp = nullptr;
      }
    } else {
      rc = kOutOfMemory;
    }
  }
  if (rc != kOk) {
    for (void* p : E->allocs) cudaFree(p);
    comm_destroy(E->comm);
    if (E->own_stream) cudaStreamDestroy(E->stream);
    delete E;
    cudaGetLastError();
    return rc;
  }
  for (int i = 0; i < c.total_pages; ++i) E->free_stack.push_back(i);  // Stack<int>: Pop() returns the last
  for (int r = c.max_batch - 1; r >= 0; --r) E->free_rows.push_back(r);
  *out = E;
  return kOk;
}

int32_t zcu_engine_destroy(void* engine) {
  Engine* E = static_cast<Engine*>(engine);
  if (!E) return zc::kBadArgument;
  zc::wait(E);
  // graphs that hold collectives go before the communicator
  for (auto& kv : E->step_graphs) cudaGraphExecDestroy(kv.second);
  for (auto& kv : E->batch_graphs) cudaGraphExecDestroy(kv.second);
  if (E->serve) {
    for (auto& kv : E->serve->graphs) cudaGraphExecDestroy(kv.second);
    if (E->serve->host) cudaFreeHost(E->serve->host);
    delete E->serve;
  }
  zc::arp_destroy(E->arp);
  zc::comm_destroy(E->comm);
  for (void* p : E->allocs) cudaFree(p);
  if (E->stage) cudaFree(E->stage);
  if (E->own_stream) cudaStreamDestroy(E->stream);
  delete E;
  return zc::kOk;
}

const char* zcu_engine_last_error(void* engine) {
  Engine* E = static_cast<Engine*>(engine);
  return E ? E->err.c_str() : "";
}

int32_t zcu_engine_set_weight(void* engine, int32_t kind, int32_t layer, const void* src, size_t bytes) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !src) return kBadArgument;
  E->err.clear();
  // a device-memory source may still be being written by the caller's kernels on any stream
  E_CUDA(cudaDeviceSynchronize());
  const zcu_engine_config& c = E->cfg;
  if (kind >= ZCU_W_ATTN_NORM && (layer < 0 || layer >= c.layers) && kind != ZCU_W_FINAL_NORM) return kBadArgument;
  auto q8bytes = [](size_t n, size_t k) { return n * (k / QK) * Q8_BLOCK_BYTES; };
  auto need = [&](size_t want) { return bytes == want; };
  const zcu_tp_shard& sh = E->shard;
  const int hd = E->hd, dblk = c.dim / QK, qd = c.heads * hd, kvd = c.kv_heads * hd;
  switch (kind) {
    case ZCU_W_TOK_EMB:
      if (!need(q8bytes(c.vocab, c.dim))) return kBadArgument;
      return upload_q8(E, E->tok_emb, 0, src, dblk, 0, c.vocab, 0, dblk);
    case ZCU_W_LM_HEAD:
      if (!need(q8bytes(c.vocab, c.dim))) return kBadArgument;
      return upload_q8(E, E->lm_head, 0, src, dblk, sh.vocab_begin, E->vocab, 0, dblk);
    case ZCU_W_FINAL_NORM:
      if (!need((size_t)c.dim * 4)) return kBadArgument;
      E_CUDA(cudaMemcpy(E->final_norm, src, bytes, cudaMemcpyDefault));
      return kOk;
    case ZCU_W_ATTN_NORM:
    case ZCU_W_FFN_NORM:
      if (!need((size_t)c.dim * 4)) return kBadArgument;
      E_CUDA(cudaMemcpy((kind == ZCU_W_ATTN_NORM ? E->attn_norm : E->ffn_norm) + (size_t)layer * c.dim, src, bytes,
                        cudaMemcpyDefault));
      return kOk;
    case ZCU_W_Q:
      if (!need(q8bytes(qd, c.dim))) return kBadArgument;
      return upload_q8(E, E->wqkv[layer], 0, src, dblk, sh.head_begin * hd, E->q_dim, 0, dblk);
    case ZCU_W_K:
      if (!need(q8bytes(kvd, c.dim))) return kBadArgument;
      return upload_q8(E, E->wqkv[layer], E->q_dim, src, dblk, sh.kv_head_begin * hd, E->kv_dim, 0, dblk);
    case ZCU_W_V:
      if (!need(q8bytes(kvd, c.dim))) return kBadArgument;
      return upload_q8(E, E->wqkv[layer], E->q_dim + E->kv_dim, src, dblk, sh.kv_head_begin * hd, E->kv_dim, 0, dblk);
    case ZCU_W_O:
      if (!need(q8bytes(c.dim, qd))) return kBadArgument;
      return upload_q8(E, E->wo[layer], 0, src, qd / QK, 0, c.dim, sh.head_begin * hd / QK, E->q_dim / QK);
    case ZCU_W_GATE:
      if (!need(q8bytes(c.ffn, c.dim))) return kBadArgument;
      return upload_q8(E, E->wgu[layer], 0, src, dblk, sh.ffn_begin, E->ffn, 0, dblk);
    case ZCU_W_UP:
      if (!need(q8bytes(c.ffn, c.dim))) return kBadArgument;
      return upload_q8(E, E->wgu[layer], E->ffn, src, dblk, sh.ffn_begin, E->ffn, 0, dblk);
    case ZCU_W_DOWN:
      if (!need(q8bytes(c.dim, c.ffn))) return kBadArgument;
      return upload_q8(E, E->wdown[layer], 0, src, c.ffn / QK, 0, c.dim, sh.ffn_begin / QK, E->ffn / QK);
    default:
      return kBadArgument;
  }
}

int32_t zcu_engine_prefill(void* engine, int32_t seq_id, const int32_t* tokens, int32_t n, int32_t start_pos,
                           float* logits) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !tokens || n <= 0 || start_pos < 0) return kBadArgument;
  E->err.clear();
  if (n > E->max_rows) {
    E->err = "prompt longer than max_prefill_tokens";
    return kTooLarge;
  }
  Seq* s = nullptr;
  E_RC(get_seq(E, seq_id, &s));
  E_RC(ensure_pages(E, *s, start_pos + n));
  std::vector<int32_t> pos(n), rows(n, s->row);
  for (int t = 0; t < n; ++t) pos[t] = start_pos + t;
  E_CUDA(cudaMemcpyAsync(E->tokens, tokens, n * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->pos, pos.data(), n * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->rows, rows.data(), n * 4, cudaMemcpyHostToDevice, E->stream));
  E_RC(embed_q8_0(E->tok_emb.qs, E->tok_emb.d, E->tokens, n, E->cfg.vocab, E->cfg.dim, E->x, E->stream));
  E->prefill_row = s->row;
  const int frc = forward(E, n, false);
  E->prefill_row = -1;
  E_RC(frc);
  if (logits) E_RC(logits_to_host(E, 1, logits));
  E_RC(wait(E));
  s->len = std::max(s->len, start_pos + n);  // AppendTokenAt at the last layer (PagedKvCache.cs:311-314)
  return kOk;
}

int32_t zcu_engine_decode(void* engine, const int32_t* seq_ids, const int32_t* tokens, const int32_t* positions,
                          int32_t batch, float* logits, int32_t* next_tokens) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !seq_ids || !tokens || !positions || batch <= 0) return kBadArgument;
  E->err.clear();
  if (batch > E->cfg.max_batch) {
    E->err = "batch larger than max_batch";
    return kTooLarge;
  }
  std::vector<int32_t> rows(batch);
  std::vector<Seq*> ss(batch);
  for (int b = 0; b < batch; ++b) {
    E_RC(get_seq(E, seq_ids[b], &ss[b]));
    E_RC(ensure_pages(E, *ss[b], positions[b] + 1));
    rows[b] = ss[b]->row;
  }
  E_CUDA(cudaMemcpyAsync(E->tokens, tokens, batch * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->pos, positions, batch * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->rows, rows.data(), batch * 4, cudaMemcpyHostToDevice, E->stream));
  E_RC(embed_q8_0(E->tok_emb.qs, E->tok_emb.d, E->tokens, batch, E->cfg.vocab, E->cfg.dim, E->x, E->stream));
  E_RC(forward(E, batch, true));
  // logits first: sampling may apply a penalty in place (not here: penalty 1), and both read E->logits
  if (logits) E_RC(logits_to_host(E, batch, logits));
  if (next_tokens) {
    E_RC(sample(E, batch, nullptr, nullptr, 0, 1.0f, E->next));
    E_CUDA(cudaMemcpyAsync(next_tokens, E->next, batch * 4, cudaMemcpyDeviceToHost, E->stream));
  }
  E_RC(wait(E));
  for (int b = 0; b < batch; ++b) ss[b]->len = std::max(ss[b]->len, positions[b] + 1);
  return kOk;
}

int32_t zcu_engine_generate(void* engine, int32_t seq_id, const int32_t* prompt, int32_t n_prompt, int32_t n_new,
                            float repetition_penalty, int32_t eos_token, int32_t* out_tokens, float* timing_ms) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !prompt || n_prompt <= 0 || n_new < 0 || !out_tokens) return kBadArgument;
  E->err.clear();
  if (n_prompt + n_new + 1 > E->gen_cap) {
    E->err = "prompt + generated tokens exceed the sequence capacity";
    return kTooLarge;
  }
  cudaEvent_t ev[3];
  for (auto& e : ev) E_CUDA(cudaEventCreate(&e));
  E_CUDA(cudaEventRecord(ev[0], E->stream));
  E_RC(zcu_engine_prefill(engine, seq_id, prompt, n_prompt, 0, nullptr));
  Seq* s = nullptr;
  E_RC(get_seq(E, seq_id, &s));
  E_RC(ensure_pages(E, *s, n_prompt + n_new));  // every decode page up front: no host work between tokens
  const int32_t zero = 0;
  E_CUDA(cudaMemcpyAsync(E->gen_past, prompt, n_prompt * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->gen_past_len, &n_prompt, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->gen_step, &zero, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->gen_done, &zero, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->pos, &n_prompt, 4, cudaMemcpyHostToDevice, E->stream));
  const int32_t row = s->row;
  E_CUDA(cudaMemcpyAsync(E->rows, &row, 4, cudaMemcpyHostToDevice, E->stream));
  E_RC(wait(E));
  E_CUDA(cudaEventRecord(ev[1], E->stream));
  if (n_new > 0) E_RC(setup_fused(E));
  if (n_new > 0 && E->fused_ok) {
    // one cooperative kernel per generated token (decode_fused.cu)
    E->fused.penalty = repetition_penalty;
    E->fused.eos = eos_token;
    for (int i = 0; i < n_new; ++i) {
      const int rc = fused_step_launch(E->fused, E->fused_sms, E->fused_smem, E->stream);
      if (rc != kOk) {
        E->err = std::string("fused generation step launch failed: ") + cudaGetErrorString(cudaGetLastError());
        return rc;
      }
    }
  } else if (n_new > 0) {
    // one graph per (penalty, eos) setting; the captured pointers are the engine's fixed buffers
    const int key = (int)(repetition_penalty * 1000.0f) * 1000003 + eos_token;
    auto it = E->step_graphs.find(key);
    if (it == E->step_graphs.end()) {
      cudaGraphExec_t ge;
      E_RC(capture_gen_step(E, repetition_penalty, eos_token, &ge));
      it = E->step_graphs.emplace(key, ge).first;
    }
    E_RC(rank_barrier(E));
    for (int i = 0; i < n_new; ++i) E_CUDA(cudaGraphLaunch(it->second, E->stream));
  }
  E_CUDA(cudaEventRecord(ev[2], E->stream));
  int32_t produced = 0;
  E_CUDA(cudaMemcpyAsync(&produced, E->gen_step, 4, cudaMemcpyDeviceToHost, E->stream));
  E_RC(wait(E));
  E_CUDA(cudaMemcpy(out_tokens, E->gen_out, (size_t)std::max(produced, 0) * 4, cudaMemcpyDeviceToHost));
  if (timing_ms) {
    cudaEventElapsedTime(&timing_ms[0], ev[0], ev[1]);
    cudaEventElapsedTime(&timing_ms[1], ev[1], ev[2]);
  }
  for (auto& e : ev) cudaEventDestroy(e);
  s->len = n_prompt + n_new;
  int st = 0;
  cudaMemcpy(&st, E->status, 4, cudaMemcpyDeviceToHost);
  if (st) {
    E->err = "a kernel's bounded wait expired (status " + std::to_string(st) + ")";
    if (E->arp) E->err += "; " + arp_describe(E->arp);
    return kCudaError;
  }
  return produced;
}

int32_t zcu_engine_step_kind(void* engine, char* why, int32_t cap) {
  Engine* E = static_cast<Engine*>(engine);
  if (!E) return zc::kBadArgument;
  if (why && cap > 0) {
    std::snprintf(why, (size_t)cap, "%s", E->fused_why.c_str());
  }
  if (!E->fused_tried) return -1;
  return E->fused_ok ? 1 : 0;
}

int32_t zcu_engine_generate_sampled(void* engine, int32_t seq_id, const int32_t* prompt, int32_t n_prompt,
                                    int32_t n_new, const zcu_sampling_config* cfg, uint64_t seed, int32_t eos_token,
                                    int32_t* out_tokens, float* timing_ms) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !cfg || !prompt || n_prompt <= 0 || n_new < 0 || !out_tokens || cfg->top_k < 0) return kBadArgument;
  if (cfg->temperature <= 0.001f || cfg->top_k == 1)  // LlmSampler's greedy branch: the greedy generation path
    return zcu_engine_generate(engine, seq_id, prompt, n_prompt, n_new, cfg->repetition_penalty, eos_token,
                               out_tokens, timing_ms);
  E->err.clear();
  if (E->tp_size != 1) {
    E->err = "sampled generation runs on one GPU (each tensor-parallel rank holds a vocabulary slice)";
    return kUnsupported;
  }
  if (n_prompt + n_new + 1 > E->gen_cap) {
    E->err = "prompt + generated tokens exceed the sequence capacity";
    return kTooLarge;
  }
  if (!E->rng_ctr) {
    E_RC(dalloc(E, &E->rng_ctr, 1));
    E_RC(dalloc(E, &E->uni, 1));
  }
  cudaEvent_t ev[3];
  for (auto& e : ev) E_CUDA(cudaEventCreate(&e));
  E_CUDA(cudaEventRecord(ev[0], E->stream));
  E_RC(zcu_engine_prefill(engine, seq_id, prompt, n_prompt, 0, nullptr));
  Seq* s = nullptr;
  E_RC(get_seq(E, seq_id, &s));
  E_RC(ensure_pages(E, *s, n_prompt + n_new));
  const int32_t zero = 0;
  E_CUDA(cudaMemcpyAsync(E->gen_past, prompt, n_prompt * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->gen_past_len, &n_prompt, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->gen_step, &zero, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->gen_done, &zero, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->rng_ctr, &zero, 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->pos, &n_prompt, 4, cudaMemcpyHostToDevice, E->stream));
  const int32_t row = s->row;
  E_CUDA(cudaMemcpyAsync(E->rows, &row, 4, cudaMemcpyHostToDevice, E->stream));
  E_RC(wait(E));
  E_CUDA(cudaEventRecord(ev[1], E->stream));
  if (n_new > 0) {
    const SampleConfig sc{cfg->temperature, cfg->top_p, cfg->min_p, cfg->top_k, cfg->repetition_penalty};
    cudaGraphExec_t ge;
    E_RC(capture_sampled_step(E, sc, seed, eos_token, &ge));
    for (int i = 0; i < n_new; ++i) {
      const cudaError_t ce = cudaGraphLaunch(ge, E->stream);
      if (ce != cudaSuccess) {
        cudaGraphExecDestroy(ge);
        E->err = std::string("cudaGraphLaunch: ") + cudaGetErrorString(ce);
        return kCudaError;
      }
    }
    E_CUDA(cudaStreamSynchronize(E->stream));
    cudaGraphExecDestroy(ge);
  }
  E_CUDA(cudaEventRecord(ev[2], E->stream));
  int32_t produced = 0;
  E_CUDA(cudaMemcpyAsync(&produced, E->gen_step, 4, cudaMemcpyDeviceToHost, E->stream));
  E_RC(wait(E));
  E_CUDA(cudaMemcpy(out_tokens, E->gen_out, (size_t)std::max(produced, 0) * 4, cudaMemcpyDeviceToHost));
  if (timing_ms) {
    cudaEventElapsedTime(&timing_ms[0], ev[0], ev[1]);
    cudaEventElapsedTime(&timing_ms[1], ev[1], ev[2]);
  }
  for (auto& e : ev) cudaEventDestroy(e);
  s->len = n_prompt + n_new;
  for (int i = 0; i < produced; ++i)
    if (out_tokens[i] < 0) {
      E->err = "more than 4096 sampling candidates after Top-K: use a Top-K of at most 4096";
      return kUnsupported;
    }
  return produced;
}

int32_t zcu_engine_free_sequence(void* engine, int32_t seq_id) {
  Engine* E = static_cast<Engine*>(engine);
  if (!E) return zc::kBadArgument;
  auto it = E->seqs.find(seq_id);
  if (it == E->seqs.end()) return zc::kOk;
  cudaStreamSynchronize(E->stream);
  // PagedKvCache.FreeSequence (:382-403): pages go back on the free stack in table order
  for (int p : it->second.pages) E->free_stack.push_back(p);
  std::vector<int32_t> none(E->cfg.max_pages_per_seq, -1);
  cudaMemcpy(E->page_table + (size_t)it->second.row * E->cfg.max_pages_per_seq, none.data(), none.size() * 4,
             cudaMemcpyHostToDevice);
  E->free_rows.push_back(it->second.row);
  E->seqs.erase(it);
  return zc::kOk;
}

int32_t zcu_engine_seq_len(void* engine, int32_t seq_id) {
  Engine* E = static_cast<Engine*>(engine);
  if (!E) return zc::kBadArgument;
  auto it = E->seqs.find(seq_id);
  return it == E->seqs.end() ? 0 : it->second.len;
}

int32_t zcu_engine_free_pages(void* engine) {
  Engine* E = static_cast<Engine*>(engine);
  return E ? (int32_t)E->free_stack.size() : zc::kBadArgument;
}

int32_t zcu_engine_page_table(void* engine, int32_t seq_id, int32_t* out, int32_t cap) {
  Engine* E = static_cast<Engine*>(engine);
  if (!E) return zc::kBadArgument;
  auto it = E->seqs.find(seq_id);
  if (it == E->seqs.end()) return 0;
  const int n = (int)it->second.pages.size();
  for (int i = 0; i < n && i < cap; ++i) out[i] = it->second.pages[i];
  return n;
}

// Reads back K (want_value = 0) or V of one token of one layer as fp32 [kv_heads * hd] (PagedKvCache.GetKey/GetValue).
int32_t zcu_engine_get_kv(void* engine, int32_t seq_id, int32_t layer, int32_t token, int32_t want_value, float* out) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !out || layer < 0 || layer >= E->cfg.layers || token < 0) return kBadArgument;
  auto it = E->seqs.find(seq_id);
  if (it == E->seqs.end()) return kBadArgument;
  const int P = E->cfg.page_size;
  if (token / P >= (int)it->second.pages.size()) return kBadArgument;
  const int page = it->second.pages[token / P];
  cudaStreamSynchronize(E->stream);
  std::vector<__half> h((size_t)E->kv_dim);
  const __half* pool = (want_value ? E->vpool : E->kpool) + (size_t)layer * E->layer_pool_elems;
  for (int kh = 0; kh < E->hkv; ++kh) {
    const size_t off = (((size_t)page * E->hkv + kh) * P + token % P) * E->hd;
    if (cudaMemcpy(h.data() + (size_t)kh * E->hd, pool + off, E->hd * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
      return kCudaError;
  }
  float* dst = out + (size_t)E->shard.kv_head_begin * E->hd;
  for (int i = 0; i < E->kv_dim; ++i) dst[i] = __half2float(h[i]);
  return kOk;
}

int32_t zcu_engine_append_kv(void* engine, int32_t seq_id, int32_t layer, int32_t start_pos, int32_t n_tokens,
                             const void* k, const void* v, int32_t kv_dtype) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !k || !v || layer < 0 || layer >= E->cfg.layers || start_pos < 0 || n_tokens < 0 ||
      (kv_dtype != 0 && kv_dtype != 1))
    return kBadArgument;
  E->err.clear();
  if (n_tokens == 0) return kOk;
  E_CUDA(cudaDeviceSynchronize());  // k / v may be device memory written on another stream
  Seq* s = nullptr;
  E_RC(get_seq(E, seq_id, &s));
  E_RC(ensure_pages(E, *s, start_pos + n_tokens));
  // this rank's K/V heads of every token, staged contiguously [n][hkv][hd]
  const size_t esz = kv_dtype ? 2 : 4;
  const size_t full_row = (size_t)E->cfg.kv_heads * E->hd * esz, part = (size_t)E->kv_dim * esz;
  const size_t off = (size_t)E->shard.kv_head_begin * E->hd * esz;
  void* st = nullptr;
  E_RC(stage(E, 2 * part * n_tokens, &st));
  char* sk = static_cast<char*>(st);
  char* sv = sk + part * n_tokens;
  E_CUDA(cudaMemcpy2DAsync(sk, part, static_cast<const char*>(k) + off, full_row, part, n_tokens, cudaMemcpyDefault,
                           E->stream));
  E_CUDA(cudaMemcpy2DAsync(sv, part, static_cast<const char*>(v) + off, full_row, part, n_tokens, cudaMemcpyDefault,
                           E->stream));
  const size_t lo = (size_t)layer * E->layer_pool_elems;
  E_RC(append_kv(sk, sv, kv_dtype, n_tokens, start_pos, E->hkv, E->hd,
                 E->page_table + (size_t)s->row * E->cfg.max_pages_per_seq, E->cfg.max_pages_per_seq,
                 E->cfg.page_size, E->kpool + lo, E->vpool + lo, E->stream));
  E_CUDA(cudaStreamSynchronize(E->stream));
  if (layer == E->cfg.layers - 1) s->len = std::max(s->len, start_pos + n_tokens);
  return kOk;
}

int32_t zcu_engine_generate_batch(void* engine, int32_t batch, const int32_t* seq_ids, const int32_t* tokens,
                                  int32_t n_new, int32_t* out_tokens, float* timing_ms) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || batch <= 0 || !seq_ids || !tokens || n_new < 0 || (n_new > 0 && !out_tokens)) return kBadArgument;
  E->err.clear();
  if (batch > E->cfg.max_batch) {
    E->err = "batch larger than max_batch";
    return kTooLarge;
  }
  if (n_new > E->gen_cap) {
    E->err = "n_new exceeds the per-sequence token capacity";
    return kTooLarge;
  }
  std::vector<int32_t> rows(batch), pos(batch);
  std::vector<Seq*> ss(batch);
  for (int b = 0; b < batch; ++b) {
    E_RC(get_seq(E, seq_ids[b], &ss[b]));
    for (int b2 = 0; b2 < b; ++b2)
      if (ss[b2] == ss[b]) {
        E->err = "a sequence appears twice in the batch";
        return kBadArgument;
      }
    pos[b] = ss[b]->len;
    E_RC(ensure_pages(E, *ss[b], pos[b] + n_new));  // every page up front: no host work between steps
    rows[b] = ss[b]->row;
  }
  const int32_t zero = 0;
  E_CUDA(cudaMemcpyAsync(E->tokens, tokens, batch * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->pos, pos.data(), batch * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->rows, rows.data(), batch * 4, cudaMemcpyHostToDevice, E->stream));
  E_CUDA(cudaMemcpyAsync(E->batch_step, &zero, 4, cudaMemcpyHostToDevice, E->stream));
  auto it = E->batch_graphs.find(batch);
  if (n_new > 0 && it == E->batch_graphs.end()) {
    cudaGraphExec_t ge;
    E_RC(capture_batch_step(E, batch, &ge));
    it = E->batch_graphs.emplace(batch, ge).first;
  }
  if (n_new > 0) E_RC(rank_barrier(E));
  cudaEvent_t ev[2];
  for (auto& e : ev) E_CUDA(cudaEventCreate(&e));
  E_CUDA(cudaEventRecord(ev[0], E->stream));
  for (int i = 0; i < n_new; ++i) E_CUDA(cudaGraphLaunch(it->second, E->stream));
  E_CUDA(cudaEventRecord(ev[1], E->stream));
  std::vector<int32_t> all;
  if (n_new > 0) {
    all.resize((size_t)batch * E->gen_cap);
    E_CUDA(cudaMemcpyAsync(all.data(), E->batch_out, all.size() * 4, cudaMemcpyDeviceToHost, E->stream));
  }
  const int wrc = wait(E);
  if (wrc == kOk && timing_ms) cudaEventElapsedTime(&timing_ms[0], ev[0], ev[1]);
  for (auto& e : ev) cudaEventDestroy(e);
  if (wrc != kOk) return wrc;
  for (int b = 0; b < batch; ++b) {
    for (int i = 0; i < n_new; ++i) out_tokens[(size_t)b * n_new + i] = all[(size_t)b * E->gen_cap + i];
    ss[b]->len = pos[b] + n_new;
  }
  int st = 0;
  cudaMemcpy(&st, E->status, 4, cudaMemcpyDeviceToHost);
  if (st) {
    E->err = "a kernel's bounded wait expired (status " + std::to_string(st) + ")";
    if (E->arp) E->err += "; " + arp_describe(E->arp);
    return kCudaError;
  }
  return n_new;
}

// ---- continuous batching ----

int32_t zcu_engine_submit(void* engine, int32_t seq_id, const int32_t* prompt, int32_t n_prompt, int32_t max_new,
                          const zcu_sampling_config* cfg, uint64_t seed, int32_t eos_token, const int32_t* stop_tokens,
                          int32_t n_stop) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !prompt || !cfg || n_prompt <= 0 || max_new < 0 || n_stop < 0 || (n_stop > 0 && !stop_tokens) ||
      cfg->top_k < 0)
    return kBadArgument;
  E->err.clear();
  if (E->tp_size != 1) {
    E->err = "continuous batching runs on one GPU (each tensor-parallel rank holds a vocabulary slice)";
    return kUnsupported;
  }
  if (n_prompt > E->max_rows) {
    E->err = "prompt longer than max_prefill_tokens";
    return kTooLarge;
  }
  const long long need = (long long)n_prompt + max_new;
  const int P = E->cfg.page_size;
  if (need > (long long)E->cfg.max_pages_per_seq * P || need > E->max_pos ||
      (need + P - 1) / P > E->cfg.total_pages) {
    E->err = "prompt + max_new exceed the sequence capacity (pages, max_pages_per_seq or context length)";
    return kTooLarge;
  }
  if (E->seqs.count(seq_id)) {
    E->err = "sequence id already live";
    return kBadArgument;
  }
  E_RC(serve_init(E));
  Serve* S = E->serve;
  for (const ServeReq& r : S->queue)
    if (r.seq_id == seq_id) {
      E->err = "sequence id already submitted";
      return kBadArgument;
    }
  ServeReq r;
  r.seq_id = seq_id;
  r.prompt.assign(prompt, prompt + n_prompt);
  r.max_new = max_new;
  r.sc = SampleConfig{cfg->temperature, cfg->top_p, cfg->min_p, cfg->top_k, cfg->repetition_penalty};
  r.seed = seed;
  r.eos = eos_token;
  if (n_stop > 0) r.stop.assign(stop_tokens, stop_tokens + n_stop);
  S->queue.push_back(std::move(r));
  return kOk;
}

int32_t zcu_engine_cancel(void* engine, int32_t seq_id) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !E->serve) return kBadArgument;
  Serve* S = E->serve;
  for (auto it = S->queue.begin(); it != S->queue.end(); ++it)
    if (it->seq_id == seq_id) {
      S->queue.erase(it);
      S->cancelled_queued.push_back(seq_id);
      return kOk;
    }
  for (ServeReq& r : S->active)
    if (r.seq_id == seq_id) {
      r.cancel = true;
      return kOk;
    }
  return kBadArgument;
}

int32_t zcu_engine_serve_counts(void* engine, int32_t* active, int32_t* queued) {
  Engine* E = static_cast<Engine*>(engine);
  if (!E) return zc::kBadArgument;
  if (active) *active = E->serve ? (int32_t)E->serve->active.size() : 0;
  if (queued) *queued = E->serve ? (int32_t)E->serve->queue.size() : 0;
  return zc::kOk;
}

int32_t zcu_engine_serve_step(void* engine, zcu_serve_event* events, int32_t cap) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !events) return kBadArgument;
  E->err.clear();
  if (!E->serve) return 0;
  Serve* S = E->serve;
  if (cap < 2 * E->cfg.max_batch + (int)S->cancelled_queued.size()) {
    E->err = "event capacity below 2 * max_batch + pending cancellations";
    return kBadArgument;
  }
  std::vector<zcu_serve_event> ev;
  for (int id : S->cancelled_queued) ev.push_back({id, -1, 1, ZCU_SERVE_CANCELLED});
  S->cancelled_queued.clear();
  auto finish = [&](size_t i) {
    zcu_engine_free_sequence(engine, S->active[i].seq_id);
    S->active.erase(S->active.begin() + (long)i);
  };
  for (size_t i = 0; i < S->active.size();) {
    if (S->active[i].cancel) {
      ev.push_back({S->active[i].seq_id, -1, 1, ZCU_SERVE_CANCELLED});
      finish(i);
    } else {
      ++i;
    }
  }
  const ServeHost h = serve_host(E);
  const int P = E->cfg.page_size;
  // 1. admission, first come first served: a page-table row and the pages of prompt + max_new tokens
  while (!S->queue.empty() && (int)S->active.size() < E->cfg.max_batch && !E->free_rows.empty()) {
    ServeReq& q = S->queue.front();
    const int n = (int)q.prompt.size();
    const int pages = (n + q.max_new + P - 1) / P;
    if ((int)E->free_stack.size() < pages) break;
    ServeReq r = std::move(q);
    S->queue.pop_front();
    Seq* sq = nullptr;
    E_RC(get_seq(E, r.seq_id, &sq));
    E_RC(ensure_pages(E, *sq, n + r.max_new));
    const int row = sq->row;
    E_RC(zcu_engine_prefill(engine, r.seq_id, r.prompt.data(), n, 0, nullptr));  // PrefillPrompt
    if (r.max_new == 0) {  // the reference's loop does not run: nothing is sampled
      ev.push_back({r.seq_id, -1, 1, ZCU_SERVE_MAX_TOKENS});
      zcu_engine_free_sequence(engine, r.seq_id);
      continue;
    }
    // history = the prompt; sample the first token from the prefill's logits
    h.u[0] = serve_uniform(r.seed, 0);
    h.cfg[0] = r.sc;
    const int32_t nn = n;
    E_CUDA(cudaMemcpyAsync(S->past + (size_t)row * S->past_cap, r.prompt.data(), (size_t)n * 4,
                           cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(S->past_len + row, &nn, 4, cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(S->u_dev, h.u, 4, cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(S->cfg_dev, h.cfg, sizeof(SampleConfig), cudaMemcpyHostToDevice, E->stream));
    E_RC(sample_rows_each(E->logits, 1, E->vocab, S->past, S->past_len, S->past_cap, E->rows, S->cfg_dev, S->u_dev,
                          S->out_dev, E->stream));
    E_RC(append_history(S->out_dev, E->rows, 1, S->past, S->past_len, S->past_cap, E->stream));
    E_CUDA(cudaMemcpyAsync(h.out, S->out_dev, 4, cudaMemcpyDeviceToHost, E->stream));
    E_RC(wait(E));
    r.pos = n;
    bool done = false;
    serve_take(r, h.out[0], &ev, &done);
    if (done) {
      zcu_engine_free_sequence(engine, r.seq_id);
      continue;
    }
    S->active.push_back(std::move(r));
  }
  // 2. one decode step of every running request: ForwardToken(pending, pos), then sample
  const int B = (int)S->active.size();
  if (B > 0) {
    for (int b = 0; b < B; ++b) {
      ServeReq& r = S->active[b];
      h.tokens[b] = r.pending;
      h.pos[b] = r.pos;
      h.rows[b] = E->seqs.at(r.seq_id).row;
      h.u[b] = serve_uniform(r.seed, (uint64_t)r.generated);
      h.cfg[b] = r.sc;
    }
    auto it = S->graphs.find(B);
    if (it == S->graphs.end()) {
      cudaGraphExec_t ge;
      E_RC(capture_serve_step(E, B, &ge));
      it = S->graphs.emplace(B, ge).first;
    }
    E_CUDA(cudaMemcpyAsync(E->tokens, h.tokens, (size_t)B * 4, cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(E->pos, h.pos, (size_t)B * 4, cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(E->rows, h.rows, (size_t)B * 4, cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(S->u_dev, h.u, (size_t)B * 4, cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaMemcpyAsync(S->cfg_dev, h.cfg, (size_t)B * sizeof(SampleConfig), cudaMemcpyHostToDevice, E->stream));
    E_CUDA(cudaGraphLaunch(it->second, E->stream));
    E_CUDA(cudaMemcpyAsync(h.out, S->out_dev, (size_t)B * 4, cudaMemcpyDeviceToHost, E->stream));
    E_RC(wait(E));
    int st = 0;
    E_CUDA(cudaMemcpy(&st, E->status, 4, cudaMemcpyDeviceToHost));
    if (st) {
      E->err = "a kernel's bounded wait expired (status " + std::to_string(st) + ")";
      return kCudaError;
    }
    std::vector<char> done(B, 0);
    for (int b = 0; b < B; ++b) {
      ServeReq& r = S->active[b];
      E->seqs.at(r.seq_id).len = r.pos + 1;  // the forwarded token's K/V are in every layer
      r.pos += 1;
      bool d = false;
      serve_take(r, h.out[b], &ev, &d);
      done[b] = d;
    }
    for (int b = B - 1; b >= 0; --b)
      if (done[b]) finish((size_t)b);
  }
  if ((int)ev.size() > cap) {  // cannot happen with cap >= 2 * max_batch + cancellations
    E->err = "event buffer overflow";
    return kTooLarge;
  }
  std::copy(ev.begin(), ev.end(), events);
  return (int32_t)ev.size();
}

}  // extern "C"
