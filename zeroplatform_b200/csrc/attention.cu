// attention.cu -- paged-KV decode attention (one query token per sequence).
//
// Restates GqaAttention.Forward (ZeroLlm/src/ZeroLlm.Core/Layers/GqaAttention.cs:29-130) over a
// KvSequenceView (Memory/PagedKvCache.cs:10-42), and the ZeroTensor operator
// TensorOps.PagedAttention (ZeroTensor/src/ZeroTensor.Core/TensorOps.Neural.cs:2372-2476):
//   out[h] = sum_t softmax_t(q[h] . K[t, h/group] * scale) * V[t, h/group],  t < ctx_len.
// ctx_len == 0 gives zeros (GqaAttention.cs:38-42).  The reference's per-layer causal length
// (non-final layers exclude the current token) is the caller's ctx_len choice.
//
// Design: one CTA per (query-head tile, sequence, split).  A query-head tile holds GT query heads
// that share one KV head, so every K/V row is read once for the whole GQA group.  Inside a CTA,
// LPT = hd/8 lanes cooperate on one token (each lane owns 8 dims and issues one 16-byte load per
// K or V row for fp16 pools), 4 token passes are kept in flight per warp, scores go through a
// shuffle reduction over the LPT lanes, and each token group keeps an online-softmax state
// (max, sum, accumulator) in the exp2 domain.  Token groups merge in shared memory.  Long
// contexts are split across CTAs (flash-decoding); the last CTA of a (sequence, head tile) to
// finish -- found with an atomic arrival counter, no waiting -- merges the split partials.
// Roofline: HBM, bytes = 2 * ctx * hkv * hd * sizeof(kv) per sequence + q/out.

#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int ATT_WARPS = 4;
constexpr int ATT_THREADS = ATT_WARPS * 32;
constexpr int ATT_UNROLL = 4;
// Resident CTAs per SM the register budget is sized for: the q and accumulator registers grow with the query
// heads a CTA serves (GT), so one head (GQA group 1) gets 8 CTAs = 32 warps (<= 64 registers a thread).
// fp32 pools hold twice the raw bytes per token in flight.
__host__ __device__ constexpr int att_min_ctas(int gt, bool half_kv) {
  return half_kv ? (gt == 1 ? 8 : gt == 2 ? 4 : gt == 4 ? 3 : 2) : (gt == 1 ? 4 : gt == 2 ? 3 : 2);
}
constexpr float LOG2E = 1.4426950408889634f;

// Raw K/V words of one lane's 8 dimensions (one 16-byte load for fp16 pools, two for fp32), kept unconverted
// while in flight and converted at use.
template <typename KV>
struct Raw8;
template <>
struct Raw8<__half> {
  int4 v;
};
template <>
struct Raw8<float> {
  int4 a, b;
};

__device__ __forceinline__ void ld_raw(const __half* p, Raw8<__half>& r) { r.v = ld_stream_v4(p); }
__device__ __forceinline__ void ld_raw(const float* p, Raw8<float>& r) {
  r.a = ld_stream_v4(p);
  r.b = ld_stream_v4(p + 4);
}
__device__ __forceinline__ void zero_raw(Raw8<__half>& r) { r.v = make_int4(0, 0, 0, 0); }
__device__ __forceinline__ void zero_raw(Raw8<float>& r) { r.a = r.b = make_int4(0, 0, 0, 0); }

// element pair j (dims 2j, 2j+1) as fp32
__device__ __forceinline__ float2 pair(const Raw8<__half>& r, int j) {
  const int w = j == 0 ? r.v.x : j == 1 ? r.v.y : j == 2 ? r.v.z : r.v.w;
  return __half22float2(*reinterpret_cast<const __half2*>(&w));
}
__device__ __forceinline__ float2 pair(const Raw8<float>& r, int j) {
  const int4& q = j < 2 ? r.a : r.b;
  const int jj = j & 1;
  return make_float2(__int_as_float(jj ? q.z : q.x), __int_as_float(jj ? q.w : q.y));
}

struct AttnDev {
  const float* q;
  const void* k_pool;
  const void* v_pool;
  const int32_t* page_table;
  const int32_t* ctx_len;
  float* out;
  float* ws;
  int* counters;
  int hq, group, page_size, max_pages, num_pages;
  long long page_stride, slot_stride, head_stride;
  long long q_stride, out_stride, pt_stride;
  const int32_t* pt_rows;
  float scale_log2;
  int out_half;  // out is __half hi / lo pairs (lo out_lo_offset elements after hi) instead of float
  long long out_lo_offset;
};

__device__ __forceinline__ void store_out(const AttnDev& a, size_t i, float v) {
  if (a.out_half)
    store_hl(reinterpret_cast<__half*>(a.out) + i, (size_t)a.out_lo_offset, v);
  else
    a.out[i] = v;
}

template <int HD, typename KV, int GT>
__global__ void __launch_bounds__(ATT_THREADS, att_min_ctas(GT, sizeof(KV) == 2)) paged_attn_kernel(AttnDev a) {
  constexpr int LPT = HD / 8;        // lanes per token
  constexpr int TPW = 32 / LPT;      // tokens per warp pass
  constexpr int NG = ATT_WARPS * TPW;  // token groups per CTA
  __shared__ float sm_m[NG][GT];
  __shared__ float sm_l[NG][GT];
  __shared__ float sm_acc[NG][GT][HD];
  __shared__ int s_last;
  pdl_trigger();
  pdl_wait();  // q and the pages come from the previous kernels

  const int split = blockIdx.x, tile = blockIdx.y, b = blockIdx.z;
  const int splits = gridDim.x, tiles = gridDim.y;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int tg = lane / LPT, sub = lane % LPT;
  const int qh0 = tile * GT;
  const int kvh = qh0 / a.group;
  const int ctx = max(0, a.ctx_len[b]);
  const int P = a.page_size;
  const int n_pages = (ctx + P - 1) / P;
  const int pps = (n_pages + splits - 1) / splits;
  const int t_begin = min(ctx, split * pps * P);
  const int t_end = min(ctx, (split + 1) * pps * P);
  const int32_t* pt = a.page_table + (size_t)(a.pt_rows ? a.pt_rows[b] : b) * a.pt_stride;
  const KV* kp = reinterpret_cast<const KV*>(a.k_pool);
  const KV* vp = reinterpret_cast<const KV*>(a.v_pool);

  float2 q[GT][4], acc[GT][4];
  float m[GT], l[GT];
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    const float* qg = a.q + (size_t)b * a.q_stride + (size_t)(qh0 + g) * HD + 8 * sub;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      q[g][j] = make_float2(qg[2 * j] * a.scale_log2, qg[2 * j + 1] * a.scale_log2);
      acc[g][j] = make_float2(0.f, 0.f);
    }
    m[g] = -INFINITY;
    l[g] = 0.f;
  }

  // Each pass: ATT_UNROLL tokens per token group; the online softmax is updated once per pass (the block's
  // maximum first, then one rescale of the running state and the block's exp2 weights).
  for (int t0 = t_begin + warp * TPW * ATT_UNROLL; t0 < t_end; t0 += ATT_WARPS * TPW * ATT_UNROLL) {
    Raw8<KV> kr[ATT_UNROLL], vr[ATT_UNROLL];
    bool valid[ATT_UNROLL];
#pragma unroll
    for (int u = 0; u < ATT_UNROLL; ++u) {
      const int t = t0 + u * TPW + tg;
      const int lp = t / P;
      const int page = (t < t_end && lp < a.max_pages) ? pt[lp] : -1;
      valid[u] = page >= 0 && page < a.num_pages;  // out-of-range page ids are never dereferenced
      if (valid[u]) {
        const long long off = page * a.page_stride + (long long)(t % P) * a.slot_stride +
                              (long long)kvh * a.head_stride + 8 * sub;
        ld_raw(kp + off, kr[u]);
        ld_raw(vp + off, vr[u]);
      } else {
        zero_raw(kr[u]);
        zero_raw(vr[u]);
      }
    }
#pragma unroll
    for (int g = 0; g < GT; ++g) {
      float sc[ATT_UNROLL];
      float mb = -INFINITY;
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; ++u) {
        float2 s2 = make_float2(0.f, 0.f);
#pragma unroll
        for (int j = 0; j < 4; ++j) s2 = __ffma2_rn(q[g][j], pair(kr[u], j), s2);
        float s = s2.x + s2.y;
#pragma unroll
        for (int o = LPT / 2; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        sc[u] = valid[u] ? s : -INFINITY;
        mb = fmaxf(mb, sc[u]);
      }
      const float mn = fmaxf(m[g], mb);
      if (mn == -INFINITY) continue;  // nothing valid yet for this token group
      const float alpha = exp2f(m[g] - mn);
      const float2 a2 = make_float2(alpha, alpha);
      l[g] *= alpha;
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[g][j] = __fmul2_rn(acc[g][j], a2);
#pragma unroll
      for (int u = 0; u < ATT_UNROLL; ++u) {
        const float p = exp2f(sc[u] - mn);  // 0 for invalid tokens
        l[g] += p;
        const float2 p2 = make_float2(p, p);
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[g][j] = __ffma2_rn(p2, pair(vr[u], j), acc[g][j]);
      }
      m[g] = mn;
    }
  }

  const int gi = warp * TPW + tg;
#pragma unroll
  for (int g = 0; g < GT; ++g) {
    if (sub == 0) {
      sm_m[gi][g] = m[g];
      sm_l[gi][g] = l[g];
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      sm_acc[gi][g][8 * sub + 2 * j] = acc[g][j].x;
      sm_acc[gi][g][8 * sub + 2 * j + 1] = acc[g][j].y;
    }
  }
  __syncthreads();

  for (int it = threadIdx.x; it < GT * HD; it += ATT_THREADS) {
    const int g = it / HD, e = it % HD;
    float M = -INFINITY;
    for (int i = 0; i < NG; ++i) M = fmaxf(M, sm_m[i][g]);
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int i = 0; i < NG; ++i) {
        const float mi = sm_m[i][g];
        if (mi == -INFINITY) continue;
        const float w = exp2f(mi - M);
        L = fmaf(sm_l[i][g], w, L);
        O = fmaf(sm_acc[i][g][e], w, O);
      }
    }
    const size_t head = (size_t)b * a.hq + qh0 + g;
    if (splits == 1) {
      store_out(a, (size_t)b * a.out_stride + (size_t)(qh0 + g) * HD + e, L > 0.f ? O / L : 0.f);
    } else {
      float* ws = a.ws + (head * splits + split) * (HD + 2);
      ws[e] = O;
      if (e == 0) {
        ws[HD] = M;
        ws[HD + 1] = L;
      }
    }
  }
  if (splits == 1) return;

  // Split-K merge by the last CTA of this (sequence, head tile) to arrive.
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    int* ctr = a.counters + (size_t)b * tiles + tile;
    s_last = (atomicAdd(ctr, 1) == splits - 1);
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int it = threadIdx.x; it < GT * HD; it += ATT_THREADS) {
    const int g = it / HD, e = it % HD;
    const size_t head = (size_t)b * a.hq + qh0 + g;
    const float* ws = a.ws + head * splits * (HD + 2);
    float M = -INFINITY;
    for (int s = 0; s < splits; ++s) M = fmaxf(M, __ldcg(ws + s * (HD + 2) + HD));
    float L = 0.f, O = 0.f;
    if (M != -INFINITY) {
      for (int s = 0; s < splits; ++s) {
        const float ms = __ldcg(ws + s * (HD + 2) + HD);
        if (ms == -INFINITY) continue;
        const float w = exp2f(ms - M);
        L = fmaf(__ldcg(ws + s * (HD + 2) + HD + 1), w, L);
        O = fmaf(__ldcg(ws + s * (HD + 2) + e), w, O);
      }
    }
    store_out(a, (size_t)b * a.out_stride + (size_t)(qh0 + g) * HD + e, L > 0.f ? O / L : 0.f);
  }
  if (threadIdx.x == 0) a.counters[(size_t)b * tiles + tile] = 0;  // ready for the next call
}

template <int HD, typename KV>
int launch_hd(const AttnDev& d, int batch, int tiles_gt, int gt, int splits, cudaStream_t s) {
  dim3 grid(splits, tiles_gt, batch);
  cudaError_t e;
  switch (gt) {
    case 1: e = launch_pdl(paged_attn_kernel<HD, KV, 1>, grid, dim3(ATT_THREADS), 0, s, d); break;
    case 2: e = launch_pdl(paged_attn_kernel<HD, KV, 2>, grid, dim3(ATT_THREADS), 0, s, d); break;
    case 4: e = launch_pdl(paged_attn_kernel<HD, KV, 4>, grid, dim3(ATT_THREADS), 0, s, d); break;
    case 8: e = launch_pdl(paged_attn_kernel<HD, KV, 8>, grid, dim3(ATT_THREADS), 0, s, d); break;
    default: return kUnsupported;
  }
  return e == cudaSuccess ? kOk : kCudaError;
}

template <typename KV>
int launch_kv(const AttnDev& d, int hd, int batch, int tiles_gt, int gt, int splits, cudaStream_t s) {
  switch (hd) {
    case 8: return launch_hd<8, KV>(d, batch, tiles_gt, gt, splits, s);
    case 16: return launch_hd<16, KV>(d, batch, tiles_gt, gt, splits, s);
    case 32: return launch_hd<32, KV>(d, batch, tiles_gt, gt, splits, s);
    case 64: return launch_hd<64, KV>(d, batch, tiles_gt, gt, splits, s);
    case 128: return launch_hd<128, KV>(d, batch, tiles_gt, gt, splits, s);
    case 256: return launch_hd<256, KV>(d, batch, tiles_gt, gt, splits, s);
    default: return kUnsupported;
  }
}

}  // namespace

size_t paged_attention_workspace_floats(int batch, int hq, int hd, int splits) {
  return splits <= 1 ? 0 : (size_t)batch * hq * splits * (hd + 2);
}

int paged_attention_check(const PagedAttnArgs& a) {
  if (!a.q || !a.k_pool || !a.v_pool || !a.page_table || !a.ctx_len || !a.out) return kBadArgument;
  if (a.batch <= 0 || a.hq <= 0 || a.hkv <= 0 || a.hq % a.hkv || a.page_size <= 0 || a.max_pages <= 0)
    return kBadArgument;
  if ((long long)a.batch * a.hq > 0x7fffffffLL) return kBadArgument;
  switch (a.hd) {
    case 8: case 16: case 32: case 64: case 128: case 256: return kOk;
    default: return a.hd <= 0 ? kBadArgument : kUnsupported;
  }
}

int paged_attention_choose_splits(int batch, int hkv, int max_ctx, int page_size) {
  if (max_ctx <= 0 || page_size <= 0 || batch <= 0 || hkv <= 0) return 1;
  const long long n_pages = ((long long)max_ctx + page_size - 1) / page_size;
  const long long ctas = (long long)batch * hkv;
  // Enough CTAs to keep HBM busy: the fp16 kernel needs about 7 resident CTAs per SM (1000 on 148 SMs) once
  // the batch itself supplies many (a tensor-parallel rank's share of the heads); small batches get at least
  // two CTAs per SM
  const long long target = std::max(2LL * 148, std::min(1000LL, 8 * ctas));
  const long long want = (target + ctas - 1) / ctas;
  long long splits = want < 1 ? 1 : want;
  if (splits > n_pages) splits = n_pages;
  if (splits > 64) splits = 64;
  return splits < 1 ? 1 : (int)splits;
}

int paged_attention(const PagedAttnArgs& a, cudaStream_t s) {
  if (const int rc = paged_attention_check(a)) return rc;
  const int elem = a.kv_half ? 2 : 4;
  const long long vec = 16 / elem;  // elements per 16-byte load
  if (a.page_stride % vec || a.slot_stride % vec || a.head_stride % vec) return kUnsupported;
  if ((reinterpret_cast<uintptr_t>(a.k_pool) | reinterpret_cast<uintptr_t>(a.v_pool)) & 15) return kUnsupported;
  const int group = a.hq / a.hkv;
  int gt = 1;
  for (int c : {8, 4, 2})
    if (group % c == 0) {
      gt = c;
      break;
    }
  int splits = a.splits > 0 ? a.splits : paged_attention_choose_splits(a.batch, a.hkv, a.max_ctx, a.page_size);
  if (splits > 1 && (!a.workspace || !a.counters)) splits = 1;
  AttnDev d;
  d.q = a.q;
  d.k_pool = a.k_pool;
  d.v_pool = a.v_pool;
  d.page_table = a.page_table;
  d.ctx_len = a.ctx_len;
  d.out = a.out;
  d.ws = a.workspace;
  d.counters = a.counters;
  d.hq = a.hq;
  d.group = group;
  d.page_size = a.page_size;
  d.max_pages = a.max_pages;
  d.num_pages = a.num_pages > 0 ? a.num_pages : 0x7fffffff;
  d.page_stride = a.page_stride;
  d.slot_stride = a.slot_stride;
  d.head_stride = a.head_stride;
  d.scale_log2 = a.scale * LOG2E;
  d.q_stride = a.q_stride > 0 ? a.q_stride : (long long)a.hq * a.hd;
  d.out_stride = a.out_stride > 0 ? a.out_stride : (long long)a.hq * a.hd;
  d.pt_stride = a.pt_stride >= 0 ? a.pt_stride : (long long)a.max_pages;
  d.pt_rows = a.pt_rows;
  d.out_half = a.out_half;
  d.out_lo_offset = a.out_lo_offset;
  const int tiles = a.hq / gt;
  return a.kv_half ? launch_kv<__half>(d, a.hd, a.batch, tiles, gt, splits, s)
                   : launch_kv<float>(d, a.hd, a.batch, tiles, gt, splits, s);
}

}  // namespace zc
