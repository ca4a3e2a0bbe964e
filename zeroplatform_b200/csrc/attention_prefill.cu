// attention_prefill.cu -- attention for many query rows of one sequence at once (prompt prefill, and the bridge's
// dense FlashAttention), over the same paged K/V addressing as the decode kernel.
//
// Restates, per query row, TensorOps.FlashAttentionCpu's FlashAttentionComputeRow (ZeroTensor/src/ZeroTensor.Core/
// TensorOps.Neural.cs:670-975): scores q . k * scale over blocks of keys, a running maximum and sum (online softmax),
// the accumulator rescaled as the maximum grows, out = acc / sum -- and, for the engine's prefill, GqaAttention
// .Forward's causal form (ZeroLlm/src/ZeroLlm.Core/Layers/GqaAttention.cs:29-130; LlmEngine.PrefillPrompt's
// per-layer causal length, Engine/LlmEngine.cs:254) through a per-row context length.
//
// Design: one CTA per (tile of PF_BQ query rows, query head, sequence).  The decode kernel reads a sequence's K/V
// once per query row; here a tile reads each key once for PF_BQ rows.  Keys are staged PF_TK at a time as fp32 in
// shared memory (the next block's words are already in registers while the current one is computed), the
// PF_BQ x PF_TK scores come from the tile's pre-scaled q rows (exp2 domain), each row's 16 lanes update its running
// maximum and sum with shuffles, and the thread owning (row, every 8th dim) rescales and accumulates p . V.  Key
// token t sits at page page_table[t / page_size], slot t % page_size, so the same kernel reads the engine's fp16
// page pools and a dense [kv batch][sk][d] fp32 tensor (one page of sk slots).  Tokens at or past a row's context
// length, and pages outside [0, num_pages), contribute nothing.  fp32 arithmetic throughout.

#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int PF_BQ = 32;        // query rows of a tile
constexpr int PF_THREADS = 256;
constexpr int PF_TK = 16;        // key tokens staged at a time

template <typename KV>
__device__ __forceinline__ float kv_at(const KV* p) {
  return (float)*p;
}
template <>
__device__ __forceinline__ float kv_at<__half>(const __half* p) {
  return __half2float(*p);
}

template <int HD, typename KV>
__global__ void __launch_bounds__(PF_THREADS) prefill_attn_kernel(PrefillAttnArgs a) {
  constexpr int QP = HD + 4;                      // padded q row: the two rows a warp reads sit in other banks
  constexpr int KP = HD + 1;                      // padded K row: the 16 tokens a warp reads sit in 16 banks
  constexpr int DPT = HD * PF_BQ / PF_THREADS;    // dims per thread in the V accumulation (HD / 8)
  constexpr int EPT = PF_TK * HD / PF_THREADS;    // K (and V) elements a thread stages per block (HD / 16)
  static_assert(HD % 16 == 0 && EPT >= 1, "head size a multiple of 16");
  __shared__ __align__(16) float sq[PF_BQ][QP];
  __shared__ float sk[PF_TK][KP];
  __shared__ float sv[PF_TK][HD];
  __shared__ float sp[PF_BQ][PF_TK + 1];
  __shared__ float s_m[PF_BQ], s_alpha[PF_BQ];
  __shared__ int sctx[PF_BQ];
  const int tid = threadIdx.x;
  const int tile = blockIdx.x, h = blockIdx.y, z = blockIdx.z;
  const int r0 = tile * PF_BQ;
  const int kvh = h / a.group;
  const float* qz = a.q + (size_t)z * a.q_seq_stride + (size_t)h * a.q_head_stride;
  const KV* kz = reinterpret_cast<const KV*>(a.k) + (size_t)z * a.kv_seq_stride + (size_t)kvh * a.head_stride;
  const KV* vz = reinterpret_cast<const KV*>(a.v) + (size_t)z * a.kv_seq_stride + (size_t)kvh * a.head_stride;
  const int32_t* pt = a.page_table + (size_t)z * a.pt_seq_stride;
  // the tile's q rows (scaled into the exp2 domain) and context lengths
  for (int i = tid; i < PF_BQ * HD; i += PF_THREADS) {
    const int r = i / HD, e = i % HD;
    sq[r][e] = r0 + r < a.rows ? qz[(size_t)(r0 + r) * a.q_row_stride + e] * a.scale_log2 : 0.f;
  }
  if (tid < PF_BQ) {
    const int c = r0 + tid < a.rows ? a.ctx_len[(size_t)z * a.ctx_seq_stride + r0 + tid] : 0;
    sctx[tid] = min(max(c, 0), a.max_pages * a.page_size);
  }
  __syncthreads();
  int max_ctx = 0;
  for (int r = 0; r < PF_BQ; ++r) max_ctx = max(max_ctx, sctx[r]);
  const int n_blocks = (max_ctx + PF_TK - 1) / PF_TK;
  // score role: thread (token st, rows sr and sr + 16); V role: thread (row vr, dims vd + 8 j)
  const int st = tid % PF_TK, sr = tid / PF_TK;
  const int vr = tid / 8, vd = tid % 8;
  float m_run[2] = {-INFINITY, -INFINITY}, l_run[2] = {0.f, 0.f};
  float acc[DPT];
#pragma unroll
  for (int j = 0; j < DPT; ++j) acc[j] = 0.f;
  // stage role: element i = tid + PF_THREADS * u of the block's PF_TK x HD (token i / HD, dim i % HD).  Tokens at
  // or past the tile's longest context, or on pages outside [0, num_pages), stage as zeros (slots never written
  // may hold any bits, and 0 * NaN would reach the sum).
  float kr[EPT], vw[EPT];
  auto load_block = [&](int b) {
#pragma unroll
    for (int u = 0; u < EPT; ++u) {
      const int i = tid + PF_THREADS * u;
      const int tok = b * PF_TK + i / HD, e = i % HD;
      const int page = tok < max_ctx ? pt[tok / a.page_size] : -1;
      const bool ok = page >= 0 && page < a.num_pages;
      const size_t off = (size_t)(ok ? page : 0) * a.page_stride + (size_t)(tok % a.page_size) * a.slot_stride + e;
      kr[u] = ok ? kv_at(kz + off) : 0.f;
      vw[u] = ok ? kv_at(vz + off) : 0.f;
    }
  };
  if (n_blocks > 0) load_block(0);
  for (int b = 0; b < n_blocks; ++b) {
    __syncthreads();  // the previous block's K, V and probabilities are consumed
#pragma unroll
    for (int u = 0; u < EPT; ++u) {
      const int i = tid + PF_THREADS * u;
      sk[i / HD][i % HD] = kr[u];
      sv[i / HD][i % HD] = vw[u];
    }
    __syncthreads();
    if (b + 1 < n_blocks) load_block(b + 1);  // in flight while this block is computed
    const int tok = b * PF_TK + st;
    const int page = tok < max_ctx ? pt[tok / a.page_size] : -1;
    const bool page_ok = page >= 0 && page < a.num_pages;
    float s0 = 0.f, s1 = 0.f;
#pragma unroll 8
    for (int e = 0; e < HD; e += 4) {
      const float4 q0 = *reinterpret_cast<const float4*>(&sq[sr][e]);
      const float4 q1 = *reinterpret_cast<const float4*>(&sq[sr + 16][e]);
      const float k0 = sk[st][e], k1 = sk[st][e + 1], k2 = sk[st][e + 2], k3 = sk[st][e + 3];
      s0 = fmaf(q0.x, k0, s0); s0 = fmaf(q0.y, k1, s0); s0 = fmaf(q0.z, k2, s0); s0 = fmaf(q0.w, k3, s0);
      s1 = fmaf(q1.x, k0, s1); s1 = fmaf(q1.y, k1, s1); s1 = fmaf(q1.z, k2, s1); s1 = fmaf(q1.w, k3, s1);
    }
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int r = sr + 16 * half;
      const float s = (page_ok && tok < sctx[r]) ? (half ? s1 : s0) : -INFINITY;
      // the row's 16 lanes (a half warp): block maximum, then the online update
      float mb = s;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
      const float m_new = fmaxf(m_run[half], mb);
      const float pw = (s == -INFINITY) ? 0.f : exp2f(s - m_new);
      float lb = pw;
#pragma unroll
      for (int o = 8; o > 0; o >>= 1) lb += __shfl_xor_sync(0xffffffffu, lb, o);
      const float alpha = (m_run[half] == -INFINITY) ? 0.f : exp2f(m_run[half] - m_new);
      l_run[half] = l_run[half] * alpha + lb;
      m_run[half] = m_new;
      sp[r][st] = pw;
      if (st == 0) s_alpha[r] = alpha;
    }
    __syncthreads();
    // V role: rescale by the row's alpha, accumulate p . V over the block
    const float al = s_alpha[vr];
#pragma unroll
    for (int j = 0; j < DPT; ++j) acc[j] *= al;
#pragma unroll 4
    for (int t = 0; t < PF_TK; ++t) {
      const float w = sp[vr][t];
#pragma unroll
      for (int j = 0; j < DPT; ++j) acc[j] = fmaf(w, sv[t][vd + 8 * j], acc[j]);
    }
  }
  __syncthreads();
  if (st == 0) {  // each row's sum, published by its first score lane
    s_m[sr] = l_run[0];
    s_m[sr + 16] = l_run[1];
  }
  __syncthreads();
  const int row = r0 + vr;
  if (row < a.rows) {
    const float l = s_m[vr];
    const float inv = l > 0.f ? 1.0f / l : 0.f;  // no attended token: zeros
    const size_t o = (size_t)z * a.out_seq_stride + (size_t)h * a.out_head_stride + (size_t)row * a.out_row_stride + vd;
    if (a.out_half) {
      __half* oh = reinterpret_cast<__half*>(a.out) + o;
#pragma unroll
      for (int j = 0; j < DPT; ++j) store_hl(oh + 8 * j, (size_t)a.out_lo_offset, acc[j] * inv);
    } else {
#pragma unroll
      for (int j = 0; j < DPT; ++j) a.out[o + 8 * j] = acc[j] * inv;
    }
  }
}

template <typename KV>
int launch_pf(const PrefillAttnArgs& a, cudaStream_t s) {
  const dim3 grid((a.rows + PF_BQ - 1) / PF_BQ, a.hq, a.seqs);
  switch (a.hd) {
    case 16: prefill_attn_kernel<16, KV><<<grid, PF_THREADS, 0, s>>>(a); break;
    case 32: prefill_attn_kernel<32, KV><<<grid, PF_THREADS, 0, s>>>(a); break;
    case 64: prefill_attn_kernel<64, KV><<<grid, PF_THREADS, 0, s>>>(a); break;
    case 128: prefill_attn_kernel<128, KV><<<grid, PF_THREADS, 0, s>>>(a); break;
    default: return kUnsupported;
  }
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

}  // namespace

int prefill_attention(const PrefillAttnArgs& a, cudaStream_t s) {
  if (!a.q || !a.k || !a.v || !a.page_table || !a.ctx_len || !a.out) return kBadArgument;
  if (a.rows <= 0 || a.seqs <= 0 || a.hq <= 0 || a.group <= 0 || a.max_pages <= 0 || a.page_size <= 0 ||
      a.num_pages <= 0)
    return kBadArgument;
  if ((long long)a.max_pages * a.page_size > 0x7fffffffLL) return kUnsupported;
  if (a.hd != 16 && a.hd != 32 && a.hd != 64 && a.hd != 128) return kUnsupported;
  if (a.seqs > 65535 || a.hq > 65535) return kUnsupported;
  return a.kv_half ? launch_pf<__half>(a, s) : launch_pf<float>(a, s);
}

}  // namespace zc
