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
//
// Tensor-core form (fp16 K/V, head size 64 or 128: the engine's pools).  One CTA of 8 warps per 64 query rows of a
// head: warps 0-3 take 16 rows each over the even 64-key blocks, warps 4-7 the same rows over the odd blocks (the
// two partial softmaxes merge at the end), keys staged two blocks at a time by cp.async into a double-buffered
// shared-memory ring.  Scores
// S = q . K come from mma.sync m16n8k16 with q carried as an fp16 pair (q_hi = fp16(q), q_lo = fp16(q - q_hi)) and
// K exact in fp16, so S = q_hi K + q_lo K is q . K to ~2^-22; the online softmax runs on the S fragments in fp32
// (exp2 domain), and P . V again takes P as an fp16 pair against exact fp16 V.  Every product is exact and
// accumulates in fp32, so the result matches the fp32 form to summation order.  Warps whose rows have no key in a
// block skip its arithmetic; tiles are issued longest first.

#include <cuda_fp16.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"
#include "sync.cuh"

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

// ---- tensor-core form ----
constexpr int MQ = 64;   // query rows per CTA (16 per warp)
constexpr int MKEYS = 64;  // keys per stage

__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// (x, y) -> fp16 pair (low half = x) and the pair of residuals x - fp16(x), y - fp16(y)
__device__ __forceinline__ void split_pair(float x, float y, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __floats2half2_rn(x, y);
  const float2 f = __half22float2(h);
  const __half2 l = __floats2half2_rn(x - f.x, y - f.y);
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

template <int HD>
__global__ void __launch_bounds__(256) prefill_attn_mma_kernel(PrefillAttnArgs a) {
  constexpr int KSTR = HD + 8;   // halves per staged key row (16-byte pad: ldmatrix rows in distinct banks)
  constexpr int KC = HD / 16;    // 16-wide k-chunks of q . K
  constexpr int DN = HD / 8;     // 8-wide dim tiles of the output
  constexpr int STAGE = MKEYS * KSTR;  // halves per block of K (and of V)
  constexpr int CHUNKS = MKEYS * HD / 8;  // 16-byte pieces per block of K (and of V)
  constexpr int MERGE = DN * 4 + 4;       // floats a thread of the second key group hands over
  extern __shared__ __align__(128) __half pf_smem[];
  __half* sK = pf_smem;              // [2 stages][2 blocks][MKEYS][KSTR]
  __half* sV = pf_smem + 4 * STAGE;  // the same for V
  __shared__ int s_wmax[8];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int rg = warp & 3, kp = warp >> 2;  // row group (16 rows), key group (even / odd blocks)
  const int g = lane >> 2, t4 = lane & 3;
  const int tile = gridDim.x - 1 - blockIdx.x;  // longest (latest) tiles first
  const int h = blockIdx.y, z = blockIdx.z;
  const int rw = tile * MQ + rg * 16;  // the warp's first row
  const int ra = rw + g, rb = rw + g + 8;
  const int kvh = h / a.group;
  const int cap = a.max_pages * a.page_size;
  const int ctx_a = ra < a.rows ? min(max(a.ctx_len[(size_t)z * a.ctx_seq_stride + ra], 0), cap) : 0;
  const int ctx_b = rb < a.rows ? min(max(a.ctx_len[(size_t)z * a.ctx_seq_stride + rb], 0), cap) : 0;
  int wmax = max(ctx_a, ctx_b);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) wmax = max(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
  if (lane == 0) s_wmax[warp] = wmax;
  // q rows as fp16 pairs in A-fragment order (pre-scaled into the exp2 domain)
  uint32_t qh[KC][4], ql[KC][4];
  {
    const float* qz = a.q + (size_t)z * a.q_seq_stride + (size_t)h * a.q_head_stride;
    const float* qa = qz + (size_t)ra * a.q_row_stride;
    const float* qb = qz + (size_t)rb * a.q_row_stride;
#pragma unroll
    for (int kc = 0; kc < KC; ++kc) {
      const int d0 = 16 * kc + 2 * t4;
      float2 v[4] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      if (ra < a.rows) {
        v[0] = *reinterpret_cast<const float2*>(qa + d0);
        v[2] = *reinterpret_cast<const float2*>(qa + d0 + 8);
      }
      if (rb < a.rows) {
        v[1] = *reinterpret_cast<const float2*>(qb + d0);
        v[3] = *reinterpret_cast<const float2*>(qb + d0 + 8);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) split_pair(v[i].x * a.scale_log2, v[i].y * a.scale_log2, qh[kc][i], ql[kc][i]);
    }
  }
  __syncthreads();
  int max_ctx = 0;
#pragma unroll
  for (int w = 0; w < 8; ++w) max_ctx = max(max_ctx, s_wmax[w]);
  const int nb = (max_ctx + MKEYS - 1) / MKEYS;
  const int n_it = (nb + 1) / 2;  // iterations: blocks 2 i (key group 0) and 2 i + 1 (key group 1)
  const __half* kz = reinterpret_cast<const __half*>(a.k) + (size_t)z * a.kv_seq_stride + (size_t)kvh * a.head_stride;
  const __half* vz = reinterpret_cast<const __half*>(a.v) + (size_t)z * a.kv_seq_stride + (size_t)kvh * a.head_stride;
  const int32_t* pt = a.page_table + (size_t)z * a.pt_seq_stride;
  // blocks 2 i and 2 i + 1 of K and V into stage i & 1: token 64 b + key, 16-byte piece `part` of its row; tokens at
  // or past the CTA's longest context, or on pages outside [0, num_pages), arrive as zeros
  auto load_stage = [&](int i) {
#pragma unroll
    for (int c = tid; c < 2 * CHUNKS; c += 256) {
      const int blk = c / CHUNKS, cc = c % CHUNKS;
      const int key = cc / (HD / 8), part = cc % (HD / 8);
      const int tok = (2 * i + blk) * MKEYS + key;
      const int page = tok < max_ctx ? pt[tok / a.page_size] : -1;
      const bool ok = page >= 0 && page < a.num_pages;
      const size_t off =
          (size_t)(ok ? page : 0) * a.page_stride + (size_t)(ok ? tok % a.page_size : 0) * a.slot_stride + 8 * part;
      const int so = ((i & 1) * 2 + blk) * STAGE + key * KSTR + 8 * part;
      cp_async16(smem_u32(sK + so), kz + off, ok);
      cp_async16(smem_u32(sV + so), vz + off, ok);
    }
  };
  float o[DN][4];
#pragma unroll
  for (int i = 0; i < DN; ++i) o[i][0] = o[i][1] = o[i][2] = o[i][3] = 0.f;
  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  if (n_it > 0) load_stage(0);
  cp_async_commit();
  for (int it = 0; it < n_it; ++it) {
    if (it + 1 < n_it) load_stage(it + 1);  // its slots were last read in iteration it - 1 (released by its barrier)
    cp_async_commit();
    cp_async_wait<1>();  // stage it has landed (this thread's copies); the barrier makes it every thread's
    __syncthreads();
    const int b = 2 * it + kp;
    if (b < nb && wmax > b * MKEYS) {  // the warp has at least one key in its block
      const __half* kb = sK + ((it & 1) * 2 + kp) * STAGE;
      const __half* vb = sV + ((it & 1) * 2 + kp) * STAGE;
      float sc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sc[j][0] = sc[j][1] = sc[j][2] = sc[j][3] = 0.f;
#pragma unroll
        for (int kc = 0; kc < KC; kc += 2) {
          uint32_t b0, b1, b2, b3;  // K rows 8 j .. 8 j + 7: dims 16 kc .. 16 kc + 31 as two k-chunks
          ldsm_x4(smem_u32(kb + (8 * j + (lane & 7)) * KSTR + 16 * kc + 8 * (lane >> 3)), b0, b1, b2, b3);
          mma16816(sc[j], qh[kc], b0, b1);
          mma16816(sc[j], ql[kc], b0, b1);
          mma16816(sc[j], qh[kc + 1], b2, b3);
          mma16816(sc[j], ql[kc + 1], b2, b3);
        }
      }
      // mask, block maxima of rows a (values 0, 1) and b (values 2, 3) over the quad's 64 columns
      float mxa = -INFINITY, mxb = -INFINITY;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int k0 = b * MKEYS + 8 * j + 2 * t4;
        if (k0 >= ctx_a) sc[j][0] = -INFINITY;
        if (k0 + 1 >= ctx_a) sc[j][1] = -INFINITY;
        if (k0 >= ctx_b) sc[j][2] = -INFINITY;
        if (k0 + 1 >= ctx_b) sc[j][3] = -INFINITY;
        mxa = fmaxf(mxa, fmaxf(sc[j][0], sc[j][1]));
        mxb = fmaxf(mxb, fmaxf(sc[j][2], sc[j][3]));
      }
#pragma unroll
      for (int off = 1; off <= 2; off <<= 1) {
        mxa = fmaxf(mxa, __shfl_xor_sync(0xffffffffu, mxa, off));
        mxb = fmaxf(mxb, __shfl_xor_sync(0xffffffffu, mxb, off));
      }
      const float na = fmaxf(m_a, mxa), nbm = fmaxf(m_b, mxb);
      const float al_a = m_a == -INFINITY ? 0.f : exp2f(m_a - na);
      const float al_b = m_b == -INFINITY ? 0.f : exp2f(m_b - nbm);
      m_a = na;
      m_b = nbm;
      float sa = 0.f, sb = 0.f;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sc[j][0] = sc[j][0] == -INFINITY ? 0.f : exp2f(sc[j][0] - na);
        sc[j][1] = sc[j][1] == -INFINITY ? 0.f : exp2f(sc[j][1] - na);
        sc[j][2] = sc[j][2] == -INFINITY ? 0.f : exp2f(sc[j][2] - nbm);
        sc[j][3] = sc[j][3] == -INFINITY ? 0.f : exp2f(sc[j][3] - nbm);
        sa += sc[j][0] + sc[j][1];
        sb += sc[j][2] + sc[j][3];
      }
      l_a = l_a * al_a + sa;
      l_b = l_b * al_b + sb;
#pragma unroll
      for (int i = 0; i < DN; ++i) {
        o[i][0] *= al_a;
        o[i][1] *= al_a;
        o[i][2] *= al_b;
        o[i][3] *= al_b;
      }
      // O += P . V, 16 keys at a time; P's A fragment is the S fragment of two key tiles
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t ph[4], pl[4];
        split_pair(sc[2 * kk][0], sc[2 * kk][1], ph[0], pl[0]);
        split_pair(sc[2 * kk][2], sc[2 * kk][3], ph[1], pl[1]);
        split_pair(sc[2 * kk + 1][0], sc[2 * kk + 1][1], ph[2], pl[2]);
        split_pair(sc[2 * kk + 1][2], sc[2 * kk + 1][3], ph[3], pl[3]);
#pragma unroll
        for (int dn = 0; dn < DN; dn += 2) {
          uint32_t b0, b1, b2, b3;  // V rows 16 kk .. 16 kk + 15, dims 8 dn .. 8 dn + 15, transposed
          ldsm_x4_t(smem_u32(vb + (16 * kk + 8 * ((lane >> 3) & 1) + (lane & 7)) * KSTR + 8 * (dn + (lane >> 4))), b0,
                    b1, b2, b3);
          mma16816(o[dn], ph, b0, b1);
          mma16816(o[dn], pl, b0, b1);
          mma16816(o[dn + 1], ph, b2, b3);
          mma16816(o[dn + 1], pl, b2, b3);
        }
      }
    }
    __syncthreads();  // this stage is read by every warp before a later iteration's copy overwrites it
  }
  cp_async_wait<0>();
#pragma unroll
  for (int off = 1; off <= 2; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  // the two key groups of a row group merge: group 1 hands (m, l, O) over through shared memory (the key stages
  // are free: every copy has landed and every warp passed the loop's last barrier)
  __syncthreads();
  float* xch = reinterpret_cast<float*>(pf_smem) + (size_t)(rg * 32 + lane) * MERGE;
  if (kp == 1) {
    xch[0] = m_a;
    xch[1] = m_b;
    xch[2] = l_a;
    xch[3] = l_b;
#pragma unroll
    for (int i = 0; i < DN; ++i) {
      xch[4 + 4 * i] = o[i][0];
      xch[5 + 4 * i] = o[i][1];
      xch[6 + 4 * i] = o[i][2];
      xch[7 + 4 * i] = o[i][3];
    }
  }
  __syncthreads();
  if (kp == 1) return;
  {
    const float m1a = xch[0], m1b = xch[1], l1a = xch[2], l1b = xch[3];
    const float Ma = fmaxf(m_a, m1a), Mb = fmaxf(m_b, m1b);
    const float f0a = m_a == -INFINITY ? 0.f : exp2f(m_a - Ma), f1a = m1a == -INFINITY ? 0.f : exp2f(m1a - Ma);
    const float f0b = m_b == -INFINITY ? 0.f : exp2f(m_b - Mb), f1b = m1b == -INFINITY ? 0.f : exp2f(m1b - Mb);
    l_a = l_a * f0a + l1a * f1a;
    l_b = l_b * f0b + l1b * f1b;
#pragma unroll
    for (int i = 0; i < DN; ++i) {
      o[i][0] = o[i][0] * f0a + xch[4 + 4 * i] * f1a;
      o[i][1] = o[i][1] * f0a + xch[5 + 4 * i] * f1a;
      o[i][2] = o[i][2] * f0b + xch[6 + 4 * i] * f1b;
      o[i][3] = o[i][3] * f0b + xch[7 + 4 * i] * f1b;
    }
  }
  const float ia = l_a > 0.f ? 1.0f / l_a : 0.f, ib = l_b > 0.f ? 1.0f / l_b : 0.f;  // no key: zeros
  const size_t ob = (size_t)z * a.out_seq_stride + (size_t)h * a.out_head_stride;
#pragma unroll
  for (int dn = 0; dn < DN; ++dn) {
    const int d = 8 * dn + 2 * t4;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int row = half ? rb : ra;
      if (row >= a.rows) continue;
      const float inv = half ? ib : ia;
      const float v0 = o[dn][2 * half] * inv, v1 = o[dn][2 * half + 1] * inv;
      const size_t off = ob + (size_t)row * a.out_row_stride + d;
      if (a.out_half) {
        __half* oh = reinterpret_cast<__half*>(a.out) + off;
        store_hl(oh, (size_t)a.out_lo_offset, v0);
        store_hl(oh + 1, (size_t)a.out_lo_offset, v1);
      } else {
        a.out[off] = v0;
        a.out[off + 1] = v1;
      }
    }
  }
}

template <int HD>
int launch_pf_mma(const PrefillAttnArgs& a, cudaStream_t s) {
  constexpr int smem = 8 * MKEYS * (HD + 8) * 2;  // K and V, two stages of two blocks each
  static unsigned long long attr_set = 0;          // devices on which the shared-memory limit was raised
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return kCudaError;
  const unsigned long long bit = 1ull << (dev & 63);
  if (!(attr_set & bit)) {
    if (cudaFuncSetAttribute(prefill_attn_mma_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) !=
        cudaSuccess)
      return kCudaError;
    attr_set |= bit;
  }
  const dim3 grid((a.rows + MQ - 1) / MQ, a.hq, a.seqs);
  prefill_attn_mma_kernel<HD><<<grid, 256, smem, s>>>(a);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

// The tensor-core form needs fp16 K/V whose rows start on 16-byte boundaries and a q row layout that allows
// 8-byte loads.
bool mma_form_ok(const PrefillAttnArgs& a) {
  if (!a.kv_half || (a.hd != 64 && a.hd != 128)) return false;
  if ((reinterpret_cast<uintptr_t>(a.k) | reinterpret_cast<uintptr_t>(a.v)) & 15) return false;
  if ((a.page_stride | a.slot_stride | a.head_stride | a.kv_seq_stride) & 7) return false;
  if ((reinterpret_cast<uintptr_t>(a.q) & 7) || ((a.q_row_stride | a.q_head_stride | a.q_seq_stride) & 1)) return false;
  if ((a.out_row_stride | a.out_head_stride | a.out_seq_stride) & 1) return false;
  return true;
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
  if (mma_form_ok(a)) return a.hd == 64 ? launch_pf_mma<64>(a, s) : launch_pf_mma<128>(a, s);
  return a.kv_half ? launch_pf<__half>(a, s) : launch_pf<float>(a, s);
}

}  // namespace zc
