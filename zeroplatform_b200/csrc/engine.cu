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
// B = 1 uses the GEMV kernels with the RmsNorm / SwiGLU prologues fused; B > 1 and batched prefill use the
// tcgen05 GEMM.  Prefill of T > 1 tokens follows PrefillPrompt (:157-315): all T tokens per layer at once,
// K/V appended for all of them, then attention with causal length (l == L-1 ? pos + 1 : pos) per token.
// The reference's causal rule (non-final layers exclude the current token) is on by default; off gives the
// standard rule (pos + 1 everywhere).
// Greedy generation (GenerateStreamAsync, :71-150) runs as replays of one captured CUDA graph per token with
// the sampled token, position and outputs kept on the device (no host round trip per token).

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "../../include/zero_tensor_cuda.h"
#include "common.cuh"
#include "kernels.h"

namespace zc {

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

struct Engine {
  zcu_engine_config cfg{};
  int hd = 0, q_dim = 0, kv_dim = 0, qkv_dim = 0;
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
  float* logits = nullptr;  // [max_batch][vocab]
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
  int gen_cap = 0;

  std::vector<int> free_stack;
  std::vector<int> free_rows;
  std::map<int, Seq> seqs;
  std::map<int, cudaGraphExec_t> step_graphs;  // decode step graphs (B = 1 generation)
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

int attention(Engine* E, int layer, int T, const int32_t* ctx) {
  PagedAttnArgs a{};
  a.q = E->qkv;
  a.k_pool = E->kpool + (size_t)layer * E->layer_pool_elems;
  a.v_pool = E->vpool + (size_t)layer * E->layer_pool_elems;
  a.page_table = E->page_table;
  a.pt_rows = E->rows;
  a.ctx_len = ctx;
  a.out = E->attn;
  a.batch = T;
  a.hq = E->cfg.heads;
  a.hkv = E->cfg.kv_heads;
  a.hd = E->hd;
  a.page_size = E->cfg.page_size;
  a.max_pages = E->cfg.max_pages_per_seq;
  a.num_pages = E->cfg.total_pages;
  a.page_stride = (long long)E->cfg.kv_heads * E->cfg.page_size * E->hd;
  a.slot_stride = E->hd;
  a.head_stride = (long long)E->cfg.page_size * E->hd;
  a.scale = 1.0f / (float)std::sqrt((double)E->hd);  // GqaAttention.cs:45
  a.kv_half = 1;
  a.max_ctx = E->cfg.max_pages_per_seq * E->cfg.page_size;
  a.q_stride = E->qkv_dim;
  a.out_stride = E->q_dim;
  a.workspace = E->attn_ws;
  a.counters = E->attn_ctr;
  a.splits = (T <= E->cfg.max_batch) ? E->attn_splits : 1;
  return paged_attention(a, E->stream);
}

// The forward pass over T activation rows already embedded in E->x, with tokens' positions in E->pos and
// page-table rows in E->rows.  Leaves the last row's logits (or every row's when all_logits) in E->logits.
int forward(Engine* E, int T, bool all_logits) {
  const zcu_engine_config& c = E->cfg;
  const int L = c.layers;
  E_RC(causal_lengths(E->pos, T, E->ctx_ex, E->ctx_in, E->stream));
  for (int l = 0; l < L; ++l) {
    const float* an = E->attn_norm + (size_t)l * c.dim;
    const float* fn = E->ffn_norm + (size_t)l * c.dim;
    if (T == 1) {
      E_RC(gemv_q8_0_rmsnorm(E->wqkv[l].qs, E->wqkv[l].d, E->x, an, c.eps, E->qkv, E->qkv_dim, c.dim, 0, E->stream));
    } else {
      E_RC(rmsnorm(E->x, an, E->xn, T, c.dim, c.eps, E->stream));
      E_RC(linear(E, E->wqkv[l], E->xn, E->qkv, T, 0));
    }
    E_RC(rope_append_kv(E->qkv, T, c.heads, c.kv_heads, E->hd, E->pos, E->rows, E->page_table, c.max_pages_per_seq,
                        c.page_size, E->cos_t, E->sin_t, E->max_pos, E->kpool + (size_t)l * E->layer_pool_elems,
                        E->vpool + (size_t)l * E->layer_pool_elems, E->stream));
    const int32_t* ctx = (c.reference_causal_quirk && l != L - 1) ? E->ctx_ex : E->ctx_in;
    E_RC(attention(E, l, T, ctx));
    E_RC(linear(E, E->wo[l], E->attn, E->x, T, 1));  // x += Wo . attn (MatVecAddQ8_0)
    if (T == 1) {
      E_RC(gemv_q8_0_rmsnorm(E->wgu[l].qs, E->wgu[l].d, E->x, fn, c.eps, E->gu, 2 * c.ffn, c.dim, 0, E->stream));
      E_RC(gemv_q8_0_swiglu(E->wdown[l].qs, E->wdown[l].d, E->gu, E->x, c.dim, c.ffn, 1, E->stream));
    } else {
      E_RC(rmsnorm(E->x, fn, E->xn, T, c.dim, c.eps, E->stream));
      E_RC(linear(E, E->wgu[l], E->xn, E->gu, T, 0));
      E_RC(swiglu_rows(E->gu, E->sw, T, c.ffn, E->stream));
      E_RC(linear(E, E->wdown[l], E->sw, E->x, T, 1));
    }
  }
  if (all_logits && T > 1) {
    E_RC(rmsnorm(E->x, E->final_norm, E->xn, T, c.dim, c.eps, E->stream));
    E_RC(linear(E, E->lm_head, E->xn, E->logits, T, 0));
  } else {  // LM head only for the last row (PrefillPrompt, LlmEngine.cs:307-314)
    const float* xl = E->x + (size_t)(T - 1) * c.dim;
    E_RC(gemv_q8_0_rmsnorm(E->lm_head.qs, E->lm_head.d, xl, E->final_norm, c.eps, E->logits, c.vocab, c.dim, 0,
                           E->stream));
  }
  return kOk;
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

int upload_q8(Engine* E, DevW& dst, size_t row_offset, const void* host, int n, int k) {
  const size_t nb = (size_t)n * (k / QK);
  uint8_t* aos = nullptr;
  if (cudaMalloc(&aos, nb * Q8_BLOCK_BYTES) != cudaSuccess) {
    cudaGetLastError();
    E->err = "staging allocation failed";
    return kOutOfMemory;
  }
  int rc = kOk;
  if (cudaMemcpyAsync(aos, host, nb * Q8_BLOCK_BYTES, cudaMemcpyHostToDevice, E->stream) != cudaSuccess) rc = kCudaError;
  if (rc == kOk)
    rc = repack_q8_0(aos, dst.qs + row_offset * dst.k, dst.d + row_offset * (dst.k / QK), n, k, E->stream);
  if (cudaStreamSynchronize(E->stream) != cudaSuccess) rc = kCudaError;
  cudaFree(aos);
  if (rc != kOk) E->err = "weight upload failed";
  return rc;
}

int capture_gen_step(Engine* E, float penalty, int eos, cudaGraphExec_t* out) {
  cudaGraph_t g;
  E_CUDA(cudaStreamBeginCapture(E->stream, cudaStreamCaptureModeThreadLocal));
  int rc = greedy_sample(E->logits, 1, E->cfg.vocab, E->gen_past, E->gen_past_len, E->gen_cap, penalty, E->tokens,
                         E->stream);
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

}  // namespace

}  // namespace zc

using zc::Engine;

extern "C" {

int32_t zcu_engine_create(const zcu_engine_config* cfg, void* stream, void** out) {
  using namespace zc;
  if (!cfg || !out) return kBadArgument;
  const zcu_engine_config& c = *cfg;
  if (c.vocab <= 0 || c.dim <= 0 || c.layers <= 0 || c.heads <= 0 || c.kv_heads <= 0 || c.ffn <= 0 ||
      c.dim % c.heads || c.heads % c.kv_heads || c.dim % QK || c.ffn % QK || c.total_pages <= 0 || c.page_size <= 0 ||
      c.max_batch <= 0 || c.max_pages_per_seq <= 0 || c.max_prefill_tokens <= 0)
    return kBadArgument;
  const int hd = c.dim / c.heads;
  if (hd % 8 || (hd & (hd - 1)) || hd > 256) return kUnsupported;  // attention kernel head sizes
  Engine* E = new Engine();
  E->cfg = c;
  E->hd = hd;
  E->q_dim = c.heads * hd;
  E->kv_dim = c.kv_heads * hd;
  E->qkv_dim = E->q_dim + 2 * E->kv_dim;
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
  const int L = c.layers;
  step(alloc_weight(E, E->tok_emb, c.vocab, c.dim));
  step(alloc_weight(E, E->lm_head, c.vocab, c.dim));
  E->wqkv.resize(L);
  E->wo.resize(L);
  E->wgu.resize(L);
  E->wdown.resize(L);
  for (int l = 0; l < L && rc == kOk; ++l) {
    step(alloc_weight(E, E->wqkv[l], E->qkv_dim, c.dim));
    step(alloc_weight(E, E->wo[l], c.dim, E->q_dim));
    step(alloc_weight(E, E->wgu[l], 2 * c.ffn, c.dim));
    step(alloc_weight(E, E->wdown[l], c.dim, c.ffn));
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
  E->layer_pool_elems = (size_t)c.total_pages * c.kv_heads * c.page_size * hd;
  step(dalloc(E, &E->kpool, E->layer_pool_elems * L));
  step(dalloc(E, &E->vpool, E->layer_pool_elems * L));
  step(dalloc(E, &E->page_table, (size_t)c.max_batch * c.max_pages_per_seq));
  E->max_rows = std::max(c.max_batch, c.max_prefill_tokens);
  const int R = E->max_rows;
  step(dalloc(E, &E->x, (size_t)R * c.dim));
  step(dalloc(E, &E->xn, (size_t)R * c.dim));
  step(dalloc(E, &E->qkv, (size_t)R * E->qkv_dim));
  step(dalloc(E, &E->attn, (size_t)R * E->q_dim));
  step(dalloc(E, &E->gu, (size_t)R * 2 * c.ffn));
  step(dalloc(E, &E->sw, (size_t)R * c.ffn));
  step(dalloc(E, &E->logits, (size_t)c.max_batch * c.vocab));
  step(dalloc(E, &E->tokens, R));
  step(dalloc(E, &E->pos, R));
  step(dalloc(E, &E->rows, R));
  step(dalloc(E, &E->ctx_ex, R));
  step(dalloc(E, &E->ctx_in, R));
  step(dalloc(E, &E->next, R));
  E->attn_splits = paged_attention_choose_splits(c.max_batch, c.kv_heads, c.max_pages_per_seq * c.page_size,
                                                 c.page_size);
  step(dalloc(E, &E->attn_ws, std::max<size_t>(16, paged_attention_workspace_floats(c.max_batch, c.heads, hd,
                                                                                   E->attn_splits))));
  step(dalloc(E, &E->attn_ctr, (size_t)R * c.heads));
  {  // the largest workspace any batched linear of this engine can ask for
    const int shapes[5][2] = {{E->qkv_dim, c.dim}, {c.dim, E->q_dim}, {2 * c.ffn, c.dim}, {c.dim, c.ffn}, {c.vocab, c.dim}};
    size_t ws = 0;
    for (auto& sh : shapes)
      for (int rows_m : {R, c.max_batch, kGemmMinRows, std::min(R, 128)})
        if (rows_m >= kGemmMinRows) ws = std::max(ws, gemm_q8_0_workspace_bytes(rows_m, sh[0], sh[1]));
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
  if (rc == kOk) {
    cudaMemset(E->attn_ctr, 0, (size_t)R * c.heads * sizeof(int));
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
  if (rc != kOk) {
    for (void* p : E->allocs) cudaFree(p);
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
  cudaStreamSynchronize(E->stream);
  for (auto& kv : E->step_graphs) cudaGraphExecDestroy(kv.second);
  for (void* p : E->allocs) cudaFree(p);
  if (E->own_stream) cudaStreamDestroy(E->stream);
  delete E;
  return zc::kOk;
}

const char* zcu_engine_last_error(void* engine) {
  Engine* E = static_cast<Engine*>(engine);
  return E ? E->err.c_str() : "";
}

int32_t zcu_engine_set_weight(void* engine, int32_t kind, int32_t layer, const void* host, size_t bytes) {
  using namespace zc;
  Engine* E = static_cast<Engine*>(engine);
  if (!E || !host) return kBadArgument;
  E->err.clear();
  const zcu_engine_config& c = E->cfg;
  if (kind >= ZCU_W_ATTN_NORM && (layer < 0 || layer >= c.layers) && kind != ZCU_W_FINAL_NORM) return kBadArgument;
  auto q8bytes = [](size_t n, size_t k) { return n * (k / QK) * Q8_BLOCK_BYTES; };
  auto need = [&](size_t want) { return bytes == want; };
  switch (kind) {
    case ZCU_W_TOK_EMB:
      if (!need(q8bytes(c.vocab, c.dim))) return kBadArgument;
      return upload_q8(E, E->tok_emb, 0, host, c.vocab, c.dim);
    case ZCU_W_LM_HEAD:
      if (!need(q8bytes(c.vocab, c.dim))) return kBadArgument;
      return upload_q8(E, E->lm_head, 0, host, c.vocab, c.dim);
    case ZCU_W_FINAL_NORM:
      if (!need((size_t)c.dim * 4)) return kBadArgument;
      E_CUDA(cudaMemcpy(E->final_norm, host, bytes, cudaMemcpyHostToDevice));
      return kOk;
    case ZCU_W_ATTN_NORM:
    case ZCU_W_FFN_NORM:
      if (!need((size_t)c.dim * 4)) return kBadArgument;
      E_CUDA(cudaMemcpy((kind == ZCU_W_ATTN_NORM ? E->attn_norm : E->ffn_norm) + (size_t)layer * c.dim, host, bytes,
                        cudaMemcpyHostToDevice));
      return kOk;
    case ZCU_W_Q:
      if (!need(q8bytes(E->q_dim, c.dim))) return kBadArgument;
      return upload_q8(E, E->wqkv[layer], 0, host, E->q_dim, c.dim);
    case ZCU_W_K:
      if (!need(q8bytes(E->kv_dim, c.dim))) return kBadArgument;
      return upload_q8(E, E->wqkv[layer], E->q_dim, host, E->kv_dim, c.dim);
    case ZCU_W_V:
      if (!need(q8bytes(E->kv_dim, c.dim))) return kBadArgument;
      return upload_q8(E, E->wqkv[layer], E->q_dim + E->kv_dim, host, E->kv_dim, c.dim);
    case ZCU_W_O:
      if (!need(q8bytes(c.dim, E->q_dim))) return kBadArgument;
      return upload_q8(E, E->wo[layer], 0, host, c.dim, E->q_dim);
    case ZCU_W_GATE:
      if (!need(q8bytes(c.ffn, c.dim))) return kBadArgument;
      return upload_q8(E, E->wgu[layer], 0, host, c.ffn, c.dim);
    case ZCU_W_UP:
      if (!need(q8bytes(c.ffn, c.dim))) return kBadArgument;
      return upload_q8(E, E->wgu[layer], c.ffn, host, c.ffn, c.dim);
    case ZCU_W_DOWN:
      if (!need(q8bytes(c.dim, c.ffn))) return kBadArgument;
      return upload_q8(E, E->wdown[layer], 0, host, c.dim, c.ffn);
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
  E_RC(forward(E, n, false));
  if (logits)
    E_CUDA(cudaMemcpyAsync(logits, E->logits, (size_t)E->cfg.vocab * 4, cudaMemcpyDeviceToHost, E->stream));
  E_CUDA(cudaStreamSynchronize(E->stream));
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
  if (next_tokens) {
    E_RC(greedy_sample(E->logits, batch, E->cfg.vocab, nullptr, nullptr, 0, 1.0f, E->next, E->stream));
    E_CUDA(cudaMemcpyAsync(next_tokens, E->next, batch * 4, cudaMemcpyDeviceToHost, E->stream));
  }
  if (logits)
    E_CUDA(cudaMemcpyAsync(logits, E->logits, (size_t)batch * E->cfg.vocab * 4, cudaMemcpyDeviceToHost, E->stream));
  E_CUDA(cudaStreamSynchronize(E->stream));
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
  E_CUDA(cudaStreamSynchronize(E->stream));
  E_CUDA(cudaEventRecord(ev[1], E->stream));
  if (n_new > 0) {
    // one graph per (penalty, eos) setting; the captured pointers are the engine's fixed buffers
    const int key = (int)(repetition_penalty * 1000.0f) * 1000003 + eos_token;
    auto it = E->step_graphs.find(key);
    if (it == E->step_graphs.end()) {
      cudaGraphExec_t ge;
      E_RC(capture_gen_step(E, repetition_penalty, eos_token, &ge));
      it = E->step_graphs.emplace(key, ge).first;
    }
    for (int i = 0; i < n_new; ++i) E_CUDA(cudaGraphLaunch(it->second, E->stream));
  }
  E_CUDA(cudaEventRecord(ev[2], E->stream));
  int32_t produced = 0;
  E_CUDA(cudaMemcpyAsync(&produced, E->gen_step, 4, cudaMemcpyDeviceToHost, E->stream));
  E_CUDA(cudaStreamSynchronize(E->stream));
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
    E->err = "a kernel's bounded wait expired";
    return kCudaError;
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
  for (int kh = 0; kh < E->cfg.kv_heads; ++kh) {
    const size_t off = (((size_t)page * E->cfg.kv_heads + kh) * P + token % P) * E->hd;
    if (cudaMemcpy(h.data() + (size_t)kh * E->hd, pool + off, E->hd * 2, cudaMemcpyDeviceToHost) != cudaSuccess)
      return kCudaError;
  }
  for (int i = 0; i < E->kv_dim; ++i) out[i] = __half2float(h[i]);
  return kOk;
}

}  // extern "C"
