// moe.cu -- sparse mixture-of-experts FFN layer: SparseMoeLayer.Forward
// (ZeroLlm/src/ZeroLlm.Core/Layers/SparseMoeLayer.cs:32-125) for a batch of tokens, on one GPU or expert-parallel
// over several (one process per GPU, NCCL all-to-all token dispatch).
//
// Per token the reference computes router logits (a MatVec of xNorm with the router weights, or given logits),
// selects the top-k experts (SelectTopK :159-182: repeated arg-max with a strict '>' so ties keep the lowest
// index), takes a softmax over the k selected logits (ComputeSoftmax :184-219, exp in double), runs each
// selected expert's SwiGLU FFN (gate = Wg.x, up = Wu.x, down = Wd.SwiGLU(gate, up)) and adds weight * down to
// the residual in selection order (AddWeightedResidual :247-264, a multiply then an add).
//
// Batched form:
//   route     one warp per token: logits, top-k, softmax; per-expert pair counts (atomics: the order inside an
//             expert does not matter, every result is addressed by its (token, slot) pair)
//   plan      one CTA: per-expert offsets, each (token, slot) pair's row in the expert-sorted order
//   gather    x rows of the pairs in expert order, as fp16 (the GEMM operand)
//   experts   for each expert with rows: [Wgate|Wup] GEMM (Q4_0 or Q8_0 on the tensor cores), SwiGLU to fp16,
//             Wdown GEMM -- rows of one expert at a time; the host reads the per-expert counts once
//   combine   residual[t] = ((residual[t] + w0 * y[row(t,0)]) + w1 * y[row(t,1)]) ..., in slot order
// Expert parallelism (ep_size > 1): expert e lives on rank e / (E / ep_size); every rank routes its own
// tokens, sends each pair's fp16 row to the expert's rank (all-to-all, counts exchanged first), the owner
// runs its experts on what it received and sends the results back along the same routes, and the token's
// rank combines them.  No shared experts (SharedExpertCount = 0, as in the benchmark configuration).

#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/zero_tensor_cuda.h"
#include "collective.h"
#include "common.cuh"
#include "kernels.h"

namespace zc {

void set_last_error(const std::string& msg);

namespace {

constexpr int MOE_MAX_EXPERTS = 256;
constexpr int MOE_MAX_TOPK = 8;

// One warp per token.  Logits: router_logits [T][E] when given, else router_w [E][dim] . x (fp32, lanes split
// dim); E <= MOE_MAX_EXPERTS.  Selection and softmax by lane 0 in the reference's order.
__global__ void moe_route_kernel(const float* __restrict__ x, const float* __restrict__ router_w,
                                 const float* __restrict__ router_logits, int T, int E, int dim, int top_k,
                                 int32_t* __restrict__ sel_idx, float* __restrict__ sel_w, int32_t* __restrict__ counts) {
  pdl_trigger();
  pdl_wait();
  __shared__ float lg[8][MOE_MAX_EXPERTS];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int t = blockIdx.x * 8 + warp;
  if (t >= T) return;
  float* l = lg[warp];
  if (router_logits) {
    for (int e = lane; e < E; e += 32) l[e] = router_logits[(size_t)t * E + e];
  } else if (router_w) {
    const float* xr = x + (size_t)t * dim;
    for (int e = 0; e < E; ++e) {
      const float* wr = router_w + (size_t)e * dim;
      float s = 0.f;
      for (int i = lane; i < dim; i += 32) s = fmaf(xr[i], wr[i], s);
      s = warp_sum(s);
      if (lane == 0) l[e] = s;
    }
  } else {
    for (int e = lane; e < E; e += 32) l[e] = 0.f;  // uniform fallback (ComputeRouterLogits :149-156)
  }
  __syncwarp();
  if (lane != 0) return;
  const int k = min(max(1, top_k), E);
  int idx[MOE_MAX_TOPK];
  float wv[MOE_MAX_TOPK];
  bool picked[MOE_MAX_EXPERTS];
  for (int e = 0; e < E; ++e) picked[e] = false;
  for (int i = 0; i < k; ++i) {
    float mv = -3.40282347e38f;  // float.MinValue
    int mi = 0;
    for (int e = 0; e < E; ++e)
      if (!picked[e] && l[e] > mv) {
        mv = l[e];
        mi = e;
      }
    picked[mi] = true;
    idx[i] = mi;
    wv[i] = mv;
  }
  float mx = wv[0];
  for (int i = 1; i < k; ++i) mx = fmaxf(mx, wv[i]);
  float sum = 0.f;
  for (int i = 0; i < k; ++i) {
    wv[i] = (float)exp((double)(wv[i] - mx));
    sum += wv[i];
  }
  if (sum > 1e-12f) {
    const float inv = 1.0f / sum;
    for (int i = 0; i < k; ++i) wv[i] *= inv;
  } else {
    for (int i = 0; i < k; ++i) wv[i] = 1.0f / k;
  }
  for (int i = 0; i < k; ++i) {
    sel_idx[(size_t)t * k + i] = idx[i];
    sel_w[(size_t)t * k + i] = wv[i];
    // skipped pairs (tiny weight) still get a row: the combine ignores them as the reference skips them
    atomicAdd(counts + idx[i], 1);
  }
}

// One CTA.  offsets[e] = rows of experts < e; row_of[p] = the pair's row in expert order (p = t * k + slot).
__global__ void moe_plan_kernel(const int32_t* __restrict__ sel_idx, int pairs, int E, const int32_t* __restrict__ counts,
                                int32_t* __restrict__ offsets, int32_t* __restrict__ fill, int32_t* __restrict__ row_of) {
  pdl_trigger();
  pdl_wait();
  __shared__ int off[MOE_MAX_EXPERTS + 1];
  __shared__ int cur[MOE_MAX_EXPERTS];
  if (threadIdx.x == 0) {
    int a = 0;
    for (int e = 0; e < E; ++e) {
      off[e] = a;
      a += counts[e];
    }
    off[E] = a;
  }
  __syncthreads();
  for (int e = threadIdx.x; e <= E; e += blockDim.x) offsets[e] = off[e];
  for (int e = threadIdx.x; e < E; e += blockDim.x) cur[e] = 0;
  __syncthreads();
  for (int p = threadIdx.x; p < pairs; p += blockDim.x) {
    const int e = sel_idx[p];
    row_of[p] = off[e] + atomicAdd(&cur[e], 1);
  }
  __syncthreads();
  for (int e = threadIdx.x; e < E; e += blockDim.x) fill[e] = cur[e];
}

// xs[row_of[p]] = x[p / k] as fp16 hi / lo pairs ([hi dim | lo dim] per row) for every pair p.
__global__ void moe_gather_kernel(const float* __restrict__ x, const int32_t* __restrict__ row_of, int pairs, int k,
                                  int dim, __half* __restrict__ xs) {
  pdl_trigger();
  pdl_wait();
  const int n4 = dim / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)pairs * n4;
       i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i / n4), c = (int)(i % n4);
    const float4 v = reinterpret_cast<const float4*>(x + (size_t)(p / k) * dim)[c];
    __half* o = xs + (size_t)row_of[p] * 2 * dim + 4 * c;
    store_hl(o + 0, dim, v.x);
    store_hl(o + 1, dim, v.y);
    store_hl(o + 2, dim, v.z);
    store_hl(o + 3, dim, v.w);
  }
}

// residual[t] += w[t][j] * y[row_of[t*k+j]] for j = 0..k-1 in order (multiply, then add: AddWeightedResidual),
// skipping the pairs the reference skips (invalid expert or |w| < 1e-7).
__global__ void moe_combine_kernel(const float* __restrict__ y, const int32_t* __restrict__ row_of,
                                   const int32_t* __restrict__ sel_idx, const float* __restrict__ sel_w, int T, int k,
                                   int E, int dim, float* __restrict__ residual) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)T * dim;
       i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / dim), c = (int)(i % dim);
    float r = residual[i];
    for (int j = 0; j < k; ++j) {
      const int p = t * k + j;
      const int e = sel_idx[p];
      const float w = sel_w[p];
      if (e < 0 || e >= E || fabsf(w) < 1e-7f) continue;
      r = __fadd_rn(r, __fmul_rn(w, y[(size_t)row_of[p] * dim + c]));
    }
    residual[i] = r;
  }
}

// Row permutation between two orders: dst[map[i]] = src[i] (rows of `cols` fp16 or fp32 elements).
template <typename T>
__global__ void moe_scatter_rows_kernel(const T* __restrict__ src, const int32_t* __restrict__ map, int rows, int cols,
                                        T* __restrict__ dst) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)rows * cols;
       i += (size_t)gridDim.x * blockDim.x) {
    const int r = (int)(i / cols), c = (int)(i % cols);
    dst[(size_t)map[r] * cols + c] = src[i];
  }
}

inline int grid_for(size_t n) {
  size_t g = (n + 255) / 256;
  if (g > 148 * 8) g = 148 * 8;
  return g < 1 ? 1 : (int)g;
}

struct ExpertW {
  uint8_t* qs = nullptr;  // int8 [rows][K] (Q8_0) or nibbles [rows][K/32][16] (Q4_0)
  uint16_t* d = nullptr;  // fp16 [rows][K/32]
};

struct Moe {
  zcu_moe_config cfg{};
  int ep_size = 1, ep_rank = 0;
  int e_begin = 0, e_count = 0;  // experts on this rank
  Comm* comm = nullptr;
  cudaStream_t stream = nullptr;
  bool own_stream = false;
  std::vector<void*> allocs;
  std::vector<ExpertW> w1, w2;  // per local expert: [Wgate | Wup] [2*ffn][dim], Wdown [dim][ffn]
  float* router_w = nullptr;    // [E][dim] fp32 (optional)
  bool has_router = false;
  // routing state for up to max_tokens tokens
  int32_t *sel_idx = nullptr, *counts = nullptr, *offsets = nullptr, *fill = nullptr, *row_of = nullptr;
  float* sel_w = nullptr;
  __half* xs = nullptr;     // gathered rows, expert order [pairs][hi dim | lo dim] (fp16 pairs)
  __half* xr = nullptr;     // rows received for local experts [recv][hi dim | lo dim]
  __half* hbuf = nullptr;   // SwiGLU output [rows][hi ffn | lo ffn]
  float* gu = nullptr;      // gate|up [rows][2*ffn]
  float* yl = nullptr;      // local expert outputs [recv rows][dim]
  float* ys = nullptr;      // outputs back in this rank's pair order [pairs][dim]
  int32_t* perm = nullptr;  // receive order -> local expert order
  int32_t* cnt_all = nullptr;  // [1 + ep_size][E]: this rank's counts, then every rank's (all-gather)
  size_t cap_rows = 0;      // rows the per-expert buffers hold
  void* gemm_ws = nullptr;
  size_t gemm_ws_bytes = 0;
  int* status = nullptr;
  int timeout_ms = 120000;
  std::string err;
};

// Expert-parallel exchange plan of one forward on rank `rank` of W (host only).  counts_all[src * E + e] is the
// number of (token, slot) rows rank src routes to expert e; expert e lives on rank e / (E / W).  A rank's rows
// leave in expert order, so the rows for peer p are one contiguous run (send_rows[p] of them); the rows it
// receives arrive grouped by source and, within a source, by local expert (recv_cnt[src][le]).  perm[i] is the
// position of received row i in the expert-contiguous order [local expert][source][row] that the expert GEMMs
// read; local_cnt[le] is each local expert's row total.
struct EpPlan {
  std::vector<int> send_rows, recv_rows, recv_cnt, local_cnt, perm;
  int total_recv = 0;
};

int moe_ep_plan(int E, int W, int rank, const int32_t* counts_all, EpPlan* p) {
  if (E <= 0 || W <= 0 || E % W || rank < 0 || rank >= W || !counts_all || !p) return kBadArgument;
  const int epr = E / W, e_begin = rank * epr;
  for (size_t i = 0; i < (size_t)W * E; ++i)
    if (counts_all[i] < 0) return kBadArgument;
  p->send_rows.assign(W, 0);
  p->recv_rows.assign(W, 0);
  p->recv_cnt.assign((size_t)W * epr, 0);
  p->local_cnt.assign(epr, 0);
  for (int e = 0; e < E; ++e) p->send_rows[e / epr] += counts_all[(size_t)rank * E + e];
  long long total = 0;
  for (int src = 0; src < W; ++src)
    for (int le = 0; le < epr; ++le) {
      const int n = counts_all[(size_t)src * E + e_begin + le];
      p->recv_cnt[(size_t)src * epr + le] = n;
      p->recv_rows[src] += n;
      p->local_cnt[le] += n;
      total += n;
    }
  if (total > 0x7fffffffLL) return kTooLarge;
  p->total_recv = (int)total;
  p->perm.assign(p->total_recv, 0);
  std::vector<int> base(epr, 0), filled(epr, 0);
  for (int le = 1; le < epr; ++le) base[le] = base[le - 1] + p->local_cnt[le - 1];
  int i = 0;
  for (int src = 0; src < W; ++src)
    for (int le = 0; le < epr; ++le)
      for (int r = 0; r < p->recv_cnt[(size_t)src * epr + le]; ++r) p->perm[i++] = base[le] + filled[le]++;
  return kOk;
}

#define M_CUDA(call)                                             \
  do {                                                           \
    cudaError_t e_ = (call);                                     \
    if (e_ != cudaSuccess) {                                     \
      M->err = std::string(#call ": ") + cudaGetErrorString(e_); \
      return kCudaError;                                         \
    }                                                            \
  } while (0)

#define M_RC(call)                        \
  do {                                    \
    int rc_ = (call);                     \
    if (rc_ != kOk) {                     \
      if (M->err.empty()) M->err = #call; \
      return rc_;                         \
    }                                     \
  } while (0)

template <class T>
int malloc_into(Moe* M, T** p, size_t count) {
  void* v = nullptr;
  if (cudaMalloc(&v, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) {
    cudaGetLastError();
    M->err = "device allocation failed";
    return kOutOfMemory;
  }
  M->allocs.push_back(v);
  *p = static_cast<T*>(v);
  return kOk;
}

int free_one(Moe* M, void* p) {
  auto it = std::find(M->allocs.begin(), M->allocs.end(), p);
  if (it != M->allocs.end()) {
    cudaFree(p);
    M->allocs.erase(it);
  }
  return kOk;
}

// Per-expert row buffers sized for `rows` rows (grown on demand, outside any graph capture).
int ensure_rows(Moe* M, size_t rows) {
  if (rows <= M->cap_rows) return kOk;
  M_CUDA(cudaStreamSynchronize(M->stream));
  for (void* p : {(void*)M->xr, (void*)M->hbuf, (void*)M->gu, (void*)M->yl, (void*)M->perm, M->gemm_ws})
    if (p) free_one(M, p);
  const zcu_moe_config& c = M->cfg;
  M_RC(malloc_into(M, &M->xr, rows * 2 * c.dim));
  M_RC(malloc_into(M, &M->hbuf, rows * 2 * c.ffn));
  M_RC(malloc_into(M, &M->gu, rows * 2 * c.ffn));
  M_RC(malloc_into(M, &M->yl, rows * c.dim));
  M_RC(malloc_into(M, &M->perm, rows));
  const size_t ws = std::max({(size_t)256, gemm_workspace_max((int)rows, 2 * c.ffn, c.dim),
                              gemm_workspace_max((int)rows, c.dim, c.ffn)});
  M_RC(malloc_into(M, reinterpret_cast<uint8_t**>(&M->gemm_ws), ws));
  M->gemm_ws_bytes = ws;
  M->cap_rows = rows;
  return kOk;
}

// x16 rows are [hi k | lo k].
int expert_gemm(Moe* M, const ExpertW& w, const __half* x16, float* y, int rows, int n, int k) {
  if (M->cfg.qtype == 4)
    return gemm_q4_0_tc_h(w.qs, w.d, x16, x16 + k, 2 * k, y, rows, n, k, 0, M->gemm_ws, M->gemm_ws_bytes, M->status,
                          M->stream);
  return gemm_q8_0_tc_h(reinterpret_cast<const int8_t*>(w.qs), w.d, x16, x16 + k, 2 * k, y, rows, n, k, 0,
                        M->gemm_ws, M->gemm_ws_bytes, M->status, M->stream);
}

// Runs the local experts over fp16 hi / lo rows sorted by local expert (counts per local expert on the host).
int run_local_experts(Moe* M, const __half* x16, const std::vector<int>& cnt, float* out) {
  const zcu_moe_config& c = M->cfg;
  int row = 0;
  for (int le = 0; le < M->e_count; ++le) {
    const int n = cnt[le];
    if (n == 0) continue;
    const __half* xe = x16 + (size_t)row * 2 * c.dim;
    M_RC(expert_gemm(M, M->w1[le], xe, M->gu, n, 2 * c.ffn, c.dim));  // [gate | up]
    M_RC(swiglu_rows_h(M->gu, M->hbuf, n, c.ffn, M->stream));
    M_RC(expert_gemm(M, M->w2[le], M->hbuf, out + (size_t)row * c.dim, n, c.dim, c.ffn));
    row += n;
  }
  return kOk;
}

int wait_stream(Moe* M) { return comm_wait(M->comm, M->stream, M->timeout_ms, &M->err); }

}  // namespace
}  // namespace zc

using zc::Moe;

extern "C" {

int32_t zcu_moe_ep_plan(int32_t n_experts, int32_t ep_size, int32_t ep_rank, const int32_t* counts_all,
                        int32_t* send_rows, int32_t* recv_rows, int32_t* recv_cnt, int32_t* perm, int32_t perm_cap) {
  using namespace zc;
  EpPlan p;
  const int rc = moe_ep_plan(n_experts, ep_size, ep_rank, counts_all, &p);
  if (rc != kOk) return rc;
  if (perm_cap < p.total_recv || (p.total_recv > 0 && !perm)) return kTooLarge;
  const int epr = n_experts / ep_size;
  if (send_rows) std::copy(p.send_rows.begin(), p.send_rows.end(), send_rows);
  if (recv_rows) std::copy(p.recv_rows.begin(), p.recv_rows.end(), recv_rows);
  if (recv_cnt) std::copy(p.recv_cnt.begin(), p.recv_cnt.begin() + (size_t)ep_size * epr, recv_cnt);
  if (p.total_recv > 0) std::copy(p.perm.begin(), p.perm.end(), perm);
  return p.total_recv;
}

int32_t zcu_moe_create(const zcu_moe_config* cfg, int32_t ep_size, int32_t ep_rank, const uint8_t* nccl_id,
                       void* stream, void** out) {
  using namespace zc;
  if (!cfg || !out) return kBadArgument;
  const zcu_moe_config& c = *cfg;
  if (c.n_experts <= 0 || c.n_experts > MOE_MAX_EXPERTS || c.top_k <= 0 || c.top_k > MOE_MAX_TOPK ||
      c.top_k > c.n_experts || c.dim <= 0 || c.ffn <= 0 || c.dim % 256 || c.ffn % 256 || c.max_tokens <= 0 ||
      (c.qtype != 4 && c.qtype != 8) || ep_size < 1 || ep_rank < 0 || ep_rank >= ep_size ||
      c.n_experts % ep_size)
    return kBadArgument;
  if (2 * c.ffn < c.dim) return kUnsupported;  // gu rows (2 * ffn floats) double as row scratch of dim floats
  Moe* M = new Moe();
  M->cfg = c;
  M->ep_size = ep_size;
  M->ep_rank = ep_rank;
  M->e_count = c.n_experts / ep_size;
  M->e_begin = ep_rank * M->e_count;
  if (stream) {
    M->stream = reinterpret_cast<cudaStream_t>(stream);
  } else if (cudaStreamCreateWithFlags(&M->stream, cudaStreamNonBlocking) == cudaSuccess) {
    M->own_stream = true;
  } else {
    delete M;
    return kCudaError;
  }
  int rc = kOk;
  auto step = [&](int r) {
    if (rc == kOk) rc = r;
  };
  {
    std::string err;
    step(comm_create(ep_size, ep_rank, nccl_id, &M->comm, &err));
    if (rc != kOk) set_last_error("zcu_moe_create: " + err);
  }
  const size_t pairs = (size_t)c.max_tokens * c.top_k;
  const size_t bpr = c.qtype == 8 ? 1 : 2;  // elements per byte of the quantized rows
  M->w1.resize(M->e_count);
  M->w2.resize(M->e_count);
  for (int le = 0; le < M->e_count && rc == kOk; ++le) {
    step(malloc_into(M, &M->w1[le].qs, (size_t)2 * c.ffn * c.dim / bpr));
    step(malloc_into(M, &M->w1[le].d, (size_t)2 * c.ffn * (c.dim / QK)));
    step(malloc_into(M, &M->w2[le].qs, (size_t)c.dim * c.ffn / bpr));
    step(malloc_into(M, &M->w2[le].d, (size_t)c.dim * (c.ffn / QK)));
  }
  step(malloc_into(M, &M->router_w, (size_t)c.n_experts * c.dim));
  step(malloc_into(M, &M->sel_idx, pairs));
  step(malloc_into(M, &M->sel_w, pairs));
  step(malloc_into(M, &M->row_of, pairs));
  step(malloc_into(M, &M->counts, MOE_MAX_EXPERTS));
  step(malloc_into(M, &M->offsets, MOE_MAX_EXPERTS + 1));
  step(malloc_into(M, &M->fill, MOE_MAX_EXPERTS));
  step(malloc_into(M, &M->xs, pairs * 2 * c.dim));
  step(malloc_into(M, &M->ys, pairs * c.dim));
  step(malloc_into(M, &M->status, 1));
  step(malloc_into(M, &M->cnt_all, (size_t)(ep_size + 1) * c.n_experts));
  if (rc == kOk) rc = ensure_rows(M, std::max<size_t>(pairs, 64));
  if (rc == kOk && cudaMemset(M->status, 0, sizeof(int)) != cudaSuccess) rc = kCudaError;
  if (rc != kOk) {
    for (void* p : M->allocs) cudaFree(p);
    comm_destroy(M->comm);
    if (M->own_stream) cudaStreamDestroy(M->stream);
    delete M;
    cudaGetLastError();
    return rc;
  }
  *out = M;
  return kOk;
}

int32_t zcu_moe_destroy(void* moe) {
  Moe* M = static_cast<Moe*>(moe);
  if (!M) return zc::kBadArgument;
  zc::wait_stream(M);
  zc::comm_destroy(M->comm);
  for (void* p : M->allocs) cudaFree(p);
  if (M->own_stream) cudaStreamDestroy(M->stream);
  delete M;
  return zc::kOk;
}

const char* zcu_moe_last_error(void* moe) {
  Moe* M = static_cast<Moe*>(moe);
  return M ? M->err.c_str() : "";
}

int32_t zcu_moe_set_expert(void* moe, int32_t expert, int32_t which, const void* src, size_t bytes) {
  using namespace zc;
  Moe* M = static_cast<Moe*>(moe);
  if (!M || !src || expert < 0 || expert >= M->cfg.n_experts || which < 0 || which > 2) return kBadArgument;
  M->err.clear();
  const zcu_moe_config& c = M->cfg;
  const size_t blk = c.qtype == 8 ? Q8_BLOCK_BYTES : Q4_BLOCK_BYTES;
  const int rows = which == 2 ? c.dim : c.ffn, cols = which == 2 ? c.ffn : c.dim;
  if (bytes != (size_t)rows * (cols / QK) * blk) {
    M->err = "expert tensor size does not match the configuration";
    return kBadArgument;
  }
  if (expert < M->e_begin || expert >= M->e_begin + M->e_count) return kOk;  // another rank's expert
  const int le = expert - M->e_begin;
  ExpertW& w = which == 2 ? M->w2[le] : M->w1[le];
  const size_t row0 = which == 1 ? (size_t)c.ffn : 0;  // up rows follow the gate rows
  const size_t row_qbytes = c.qtype == 8 ? (size_t)cols : (size_t)cols / 2;
  M_CUDA(cudaDeviceSynchronize());  // a device source may still be written by another stream
  void* aos = nullptr;
  M_CUDA(cudaMalloc(&aos, bytes));
  int rc = cudaMemcpyAsync(aos, src, bytes, cudaMemcpyDefault, M->stream) == cudaSuccess ? kOk : kCudaError;
  if (rc == kOk) {
    rc = c.qtype == 8 ? repack_q8_0(static_cast<const uint8_t*>(aos), reinterpret_cast<int8_t*>(w.qs + row0 * row_qbytes),
                                    w.d + row0 * (cols / QK), rows, cols, M->stream)
                      : repack_q4_0(static_cast<const uint8_t*>(aos), w.qs + row0 * row_qbytes, w.d + row0 * (cols / QK),
                                    rows, cols, M->stream);
  }
  if (cudaStreamSynchronize(M->stream) != cudaSuccess) rc = kCudaError;
  cudaFree(aos);
  if (rc != kOk) M->err = "expert upload failed";
  return rc;
}

int32_t zcu_moe_set_router(void* moe, const float* w, size_t bytes) {
  using namespace zc;
  Moe* M = static_cast<Moe*>(moe);
  if (!M || !w || bytes != (size_t)M->cfg.n_experts * M->cfg.dim * sizeof(float)) return kBadArgument;
  M_CUDA(cudaDeviceSynchronize());
  M_CUDA(cudaMemcpy(M->router_w, w, bytes, cudaMemcpyDefault));
  M->has_router = true;
  return kOk;
}

int32_t zcu_moe_forward(void* moe, const float* xnorm, const float* router_logits, float* residual, int32_t T,
                        int32_t* sel_idx_out, float* sel_w_out) {
  using namespace zc;
  Moe* M = static_cast<Moe*>(moe);
  if (!M || !xnorm || !residual || T < 0) return kBadArgument;
  M->err.clear();
  const zcu_moe_config& c = M->cfg;
  if (T > c.max_tokens) {
    M->err = "more tokens than max_tokens";
    return kTooLarge;
  }
  const int E = c.n_experts, k = c.top_k, P = T * k, W = M->ep_size;
  cudaStream_t s = M->stream;
  if (T > 0) {
    M_CUDA(cudaMemsetAsync(M->counts, 0, E * sizeof(int32_t), s));
    M_CUDA(launch_pdl(moe_route_kernel, dim3((T + 7) / 8), dim3(256), 0, s, xnorm,
                      (const float*)(M->has_router ? M->router_w : nullptr), router_logits, T, E, c.dim, k, M->sel_idx,
                      M->sel_w, M->counts));
    M_CUDA(launch_pdl(moe_plan_kernel, dim3(1), dim3(1024), 0, s, (const int32_t*)M->sel_idx, P, E,
                      (const int32_t*)M->counts, M->offsets, M->fill, M->row_of));
    M_CUDA(launch_pdl(moe_gather_kernel, dim3(grid_for((size_t)P * c.dim / 4)), dim3(256), 0, s, xnorm,
                      (const int32_t*)M->row_of, P, k, c.dim, M->xs));
  }
  std::vector<int> cnt(E, 0);
  if (T > 0) M_CUDA(cudaMemcpyAsync(cnt.data(), M->counts, E * sizeof(int), cudaMemcpyDeviceToHost, s));
  M_RC(wait_stream(M));
  const int epr = M->e_count;
  const size_t row_bytes = (size_t)2 * c.dim * sizeof(__half);  // one hi / lo row
  if (W == 1) {
    std::vector<int> local_cnt(cnt.begin(), cnt.begin() + epr);
    M_RC(ensure_rows(M, std::max<size_t>(P, 1)));
    if (P > 0) M_RC(run_local_experts(M, M->xs, local_cnt, M->ys));
  } else {
    // exchange per-expert counts: every rank learns how many rows of each of its experts each peer sends
    int32_t* dcnt = M->cnt_all;
    M_CUDA(cudaMemcpyAsync(dcnt, cnt.data(), E * sizeof(int32_t), cudaMemcpyHostToDevice, s));
    M_RC(comm_allgather_bytes(M->comm, dcnt, dcnt + E, E * sizeof(int32_t), s, &M->err));
    std::vector<int> all((size_t)W * E);
    M_CUDA(cudaMemcpyAsync(all.data(), dcnt + E, all.size() * sizeof(int32_t), cudaMemcpyDeviceToHost, s));
    M_RC(wait_stream(M));
    EpPlan plan;
    if (moe_ep_plan(E, W, M->ep_rank, all.data(), &plan) != kOk) {
      M->err = "inconsistent expert counts";
      return kBadArgument;
    }
    const int total_recv = plan.total_recv;
    const std::vector<int>& local_cnt = plan.local_cnt;
    const std::vector<int32_t>& perm = plan.perm;
    M_RC(ensure_rows(M, std::max(total_recv, 1)));
    // dispatch: my expert-sorted rows to their owners; received rows land in [source][local expert] order
    std::vector<size_t> sb(W), so(W), rb(W), ro(W);
    size_t a = 0, b = 0;
    for (int p = 0; p < W; ++p) {
      sb[p] = (size_t)plan.send_rows[p] * row_bytes;
      so[p] = a;
      a += sb[p];
      rb[p] = (size_t)plan.recv_rows[p] * row_bytes;
      ro[p] = b;
      b += rb[p];
    }
    M_RC(comm_alltoallv_bytes(M->comm, M->xs, sb.data(), so.data(), M->xr, rb.data(), ro.data(), s, &M->err));
    // [source][local expert] -> [local expert][source] so that each expert's rows are contiguous
    if (total_recv > 0) {
      M_CUDA(cudaMemcpyAsync(M->perm, perm.data(), perm.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
      // xr -> expert-contiguous copy in hbuf's place is not possible (different widths): use gu as scratch
      // (a hi / lo row is dim floats' worth of bytes; gu holds 2 * ffn floats per row)
      __half* xsorted = reinterpret_cast<__half*>(M->gu);
      M_CUDA(launch_pdl(moe_scatter_rows_kernel<__half>, dim3(grid_for((size_t)total_recv * 2 * c.dim)), dim3(256), 0,
                        s, (const __half*)M->xr, (const int32_t*)M->perm, total_recv, 2 * c.dim, xsorted));
      // the expert pass needs gu for gate|up: move the sorted rows back into xr first
      M_CUDA(cudaMemcpyAsync(M->xr, xsorted, (size_t)total_recv * row_bytes, cudaMemcpyDeviceToDevice, s));
      M_RC(run_local_experts(M, M->xr, local_cnt, M->yl));
      // outputs back to [source][local expert] order: yl[perm[i]] -> position i
      float* ysend = M->gu;  // gu holds 2*ffn >= dim floats per row: room for the outputs
      {
        // gather: ysend[i] = yl[perm[i]]
        std::vector<int32_t> inv(total_recv);
        for (int i = 0; i < total_recv; ++i) inv[perm[i]] = i;
        M_CUDA(cudaMemcpyAsync(M->perm, inv.data(), inv.size() * sizeof(int32_t), cudaMemcpyHostToDevice, s));
        M_CUDA(launch_pdl(moe_scatter_rows_kernel<float>, dim3(grid_for((size_t)total_recv * c.dim)), dim3(256), 0, s,
                          (const float*)M->yl, (const int32_t*)M->perm, total_recv, c.dim, ysend));
      }
      M_RC(wait_stream(M));  // the host vectors above must outlive their copies
    }
    // return: the results travel back along the same routes (sizes swapped, fp32 rows)
    const size_t frow = (size_t)c.dim * sizeof(float);
    for (int p = 0; p < W; ++p) {
      std::swap(sb[p], rb[p]);
      std::swap(so[p], ro[p]);
      sb[p] = sb[p] / row_bytes * frow;
      so[p] = so[p] / row_bytes * frow;
      rb[p] = rb[p] / row_bytes * frow;
      ro[p] = ro[p] / row_bytes * frow;
    }
    M_RC(comm_alltoallv_bytes(M->comm, M->gu, sb.data(), so.data(), M->ys, rb.data(), ro.data(), s, &M->err));
  }
  if (T > 0)
    M_CUDA(launch_pdl(moe_combine_kernel, dim3(grid_for((size_t)T * c.dim)), dim3(256), 0, s, (const float*)M->ys,
                      (const int32_t*)M->row_of, (const int32_t*)M->sel_idx, (const float*)M->sel_w, T, k, E, c.dim,
                      residual));
  if (sel_idx_out && T > 0)
    M_CUDA(cudaMemcpyAsync(sel_idx_out, M->sel_idx, (size_t)P * sizeof(int32_t), cudaMemcpyDefault, s));
  if (sel_w_out && T > 0) M_CUDA(cudaMemcpyAsync(sel_w_out, M->sel_w, (size_t)P * sizeof(float), cudaMemcpyDefault, s));
  M_RC(wait_stream(M));
  int st = 0;
  M_CUDA(cudaMemcpy(&st, M->status, sizeof(int), cudaMemcpyDeviceToHost));
  if (st) {
    M->err = "a kernel's bounded wait expired";
    return kCudaError;
  }
  return kOk;
}

}  // extern "C"
