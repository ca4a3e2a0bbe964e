// decode_fused.cu -- one greedy generation step of a Q8_0 Llama-style model for one sequence as a single
// persistent (cooperative) kernel: LlmSampler.Sample's greedy branch with repetition penalty
// (Sampling/LlmSampler.cs:21-72), the GenerateStreamAsync bookkeeping (Engine/LlmEngine.cs:115-141), the token
// embedding (LlmEngine.cs:317-345) and LlmEngine.ForwardToken (LlmEngine.cs:347-461) over the paged fp16 KV cache.
//
// Why one kernel: at batch 1 a small model's step is a chain of ~80 dependent launches whose weight reads are a
// few hundred KB each, so latency, not HBM, sets the step time.  Here one CTA per SM runs the whole step, and the
// points where a vector must be complete before anyone reads it become grid barriers (an arrival counter plus a
// release flag in global memory; one thread per CTA polls the flag, bounded by a time limit after which every CTA
// stops and the status word records code 41):
//
//   0  sample     each CTA: arg-max of its vocabulary slice of the previous logits, the repetition penalty applied
//                 occurrence by occurrence to the past tokens in the slice                               | barrier
//                 every CTA merges the slices' (value, index) pairs (largest value, lowest index); CTA 0 records
//                 the token (stop token, output, past list); every CTA dequantizes its embedding row
//   per layer:
//   A  qkv        every CTA: RmsNorm of x (redundantly, x in shared memory); its pairs of Wqkv rows; RoPE on q and
//                 k pairs; q -> qbuf, k and v -> the layer's fp16 pages at the token's slot                | barrier
//   B  attention  CTA (head h, split s): softmax partial over its slice of the context (the reference's causal
//                 rule: non-final layers attend to [0, pos)); the last split of a head to arrive (atomic counter)
//                 merges the partials in split order and multiplies the head's output by its 32-block columns of
//                 Wo: P[h] = Wo[:, head h] . attn_h                                                          | barrier
//   C  ffn up     every CTA: x += sum over h of P[h] (head order; the same in every CTA), RmsNorm, its units of
//                 Wgate and Wup, SwiGLU -> hbuf                                                               | barrier
//   D  ffn down   every CTA: its rows of x_new = x + Wdown . hbuf -> global x                                  | barrier
//   LM head       every CTA: RmsNorm with the final norm, its rows of the LM head -> logits; CTA 0 advances pos
//
// Memory: every weight byte is read once per step.  A CTA's rows of Wqkv, Wgate|Wup, Wdown and the LM head are
// contiguous, so one thread bulk-copies them (cp.async.bulk with mbarrier completion, no multicast) into shared
// memory well before they are used -- a layer's rows right after the previous layer consumed that region -- and the
// GEMVs read shared memory.  Wo, read by columns of a head in phase B, is prefetched into L2 by row shares.  Loads
// that depend on a barrier (K/V, partials, Wo slices, the heads' partial sums) are issued all at once.  Data
// written in this kernel by another CTA (qbuf, K/V pages, partials, P, hbuf, x, pairs) is read through L2
// (ld.global.cg); weights through the non-coherent path.  The staged projections take their activations as int16
// per 32-block (each value within 2^-16 of its block's largest, the form of the 4096-column slab GEMV) and sum exact
// int32 block products; Wo (in phase B) takes fp32 activations.  Wo is summed per head and then over heads, another
// fp32 order than one MatVecAdd over all columns.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "sync.cuh"

namespace zc {

namespace {

constexpr int FS_THREADS = 512;
constexpr int FS_WARPS = FS_THREADS / 32;
constexpr uint64_t FS_WAIT_NS = 2000000000ull;  // a grid barrier that waits longer than 2 s gives up
constexpr float FS_LOG2E = 1.4426950408889634f;
constexpr int FS_WAVE = 4096;  // floats of the attention reduction area (tokens of a wave x hd)

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ int4 ldcg4(const void* p) { return __ldcg(reinterpret_cast<const int4*>(p)); }

// One arrival with release semantics at GPU scope: after the CTA's __syncthreads, every write the CTA made
// before it is visible to a thread that observes the count with ld.acquire.gpu (no separate full fence).
__device__ __forceinline__ void red_release_gpu(unsigned* p, unsigned v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// Grid barrier number k (1, 2, ...): ctl[0] counts arrivals; one thread per CTA adds its arrival (release, after
// the CTA's __syncthreads) and polls the count (acquire) until it reaches k * grid; the closing __syncthreads
// passes the acquired view on to the CTA.  Returns false when the wait ran out or another CTA gave up (ctl[1]).
__device__ __forceinline__ bool grid_sync(unsigned* ctl, unsigned& k, int* status, volatile int* sh_ok) {
  __syncthreads();
  ++k;
  if (threadIdx.x == 0) {
    int ok = 1;
    red_release_gpu(ctl, 1u);
    const unsigned target = k * gridDim.x;
    const uint64_t t0 = global_ns();
    uint32_t polls = 0;
    while (ld_acquire_gpu(ctl) < target) {
      if ((++polls & 31) == 0) {
        if (*reinterpret_cast<volatile unsigned*>(ctl + 1)) {
          ok = 0;
          break;
        }
        if (global_ns() - t0 > FS_WAIT_NS) {
          atomicExch(ctl + 1, 1u);
          atomicExch(status, 41);
          ok = 0;
          break;
        }
      }
    }
    *sh_ok = ok;
  }
  __syncthreads();
  return *sh_ok != 0;
}

// units [b, e) of `n` balanced over the grid
__device__ __forceinline__ void share(int n, int& b, int& e) {
  b = (int)((long long)n * blockIdx.x / gridDim.x);
  e = (int)((long long)n * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ uint32_t row_bytes(int K, int r0, int r1) {
  return r1 > r0 ? (uint32_t)(r1 - r0) * (uint32_t)(K + K / 16) : 0u;
}

// One thread: bulk-copies rows [r0, r1) of a Q8_0 matrix (K columns) into shared memory (int8 rows at dst_q,
// fp16 scales at dst_d), completion counted on `bar` (armed by the caller with the byte count).
__device__ __forceinline__ void copy_rows(uint8_t* dst_q, uint16_t* dst_d, const int8_t* qs, const uint16_t* d, int K,
                                          int r0, int r1, uint32_t bar) {
  if (r1 <= r0) return;
  const uint32_t n = (uint32_t)(r1 - r0);
  bulk_g2s(smem_u32(dst_q), qs + (size_t)r0 * K, n * (uint32_t)K, bar);
  bulk_g2s(smem_u32(dst_d), d + (size_t)r0 * (K / QK), n * (uint32_t)(K / 16), bar);
}

__device__ __forceinline__ void prefetch_rows(const int8_t* qs, const uint16_t* d, int K, int r0, int r1) {
  if (r1 <= r0) return;
  const uint32_t n = (uint32_t)(r1 - r0);
  bulk_prefetch_l2(qs + (size_t)r0 * K, n * (uint32_t)K);
  bulk_prefetch_l2(d + (size_t)r0 * (K / QK), n * (uint32_t)(K / 16));
}

// 16 int8 weights . 16 fp32 activations (shared memory), exact conversion, packed FMAs
__device__ __forceinline__ float dot16_s(const int4& w, const float* xs) {
  const float2 bias = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  const uint32_t* wv = reinterpret_cast<const uint32_t*>(&w);
  const float4* x4 = reinterpret_cast<const float4*>(xs);
  float2 s = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t b = wv[j] ^ 0x80808080u;
    const float4 xv = x4[j];
    const float2 p01 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7650)),
                                              __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7651))),
                                  bias);
    const float2 p23 = __fadd2_rn(make_float2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7652)),
                                              __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7653))),
                                  bias);
    s = __ffma2_rn(p01, make_float2(xv.x, xv.y), s);
    s = __ffma2_rn(p23, make_float2(xv.z, xv.w), s);
  }
  return s.x + s.y;
}

// GEMV of rows staged in shared memory against x in shared memory.  Each lane owns CPL 16-value chunks of the K
// columns (chunk c = lane-in-group + G * k) and keeps them in registers as int16 with a per-32-block scale
// (q = rint(x * 32767 / max|x|): every value within 2^-16 of its block's largest), read and quantized once per
// call; per row a lane then reads only its 16-byte weight chunks and the block scales from shared memory, and a
// chunk is 8 DP2A instructions (two int16 x int8 products each, exact in int32), one conversion and one FMA.  G
// lanes per row (G * CPL = K / 16), so a warp holds 32 / G row groups; the loop is uniform over the warp (a
// missing row computes zeros) so the full-warp shuffles always have all 32 lanes.  emit(local row, value) runs on
// the group's first lane.
template <int CPL>
struct XChunks {
  int v[CPL][8];
  float s[CPL];
};

template <int G, int CPL>
__device__ __forceinline__ void quantize_chunks(const float* xs, XChunks<CPL>& xq) {
  const int li = threadIdx.x % G;
#pragma unroll
  for (int k = 0; k < CPL; ++k) {
    const float4* x4 = reinterpret_cast<const float4*>(xs + (li + G * k) * 16);
    float v[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 f = x4[j];
      v[4 * j] = f.x;
      v[4 * j + 1] = f.y;
      v[4 * j + 2] = f.z;
      v[4 * j + 3] = f.w;
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(v[j]));
    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));  // the other half of the 32-block
    const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
    xq.s[k] = amax * (1.0f / 32767.0f);
    const float2 inv2 = make_float2(inv, inv), mg2 = make_float2(12582912.0f, 12582912.0f);  // 1.5 * 2^23
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float2 r = __ffma2_rn(make_float2(v[2 * j], v[2 * j + 1]), inv2, mg2);
      xq.v[k][j] = (int)__byte_perm(__float_as_uint(r.x), __float_as_uint(r.y), 0x5410);
    }
  }
}

template <int G, int CPL, class Emit>
__device__ __forceinline__ void gemv_q(const uint8_t* sq, const uint16_t* sd, const float* xs, int nrows, Emit emit) {
  constexpr int K = G * CPL * 16, KB = K / QK, RPW = 32 / G;
  XChunks<CPL> xq;
  quantize_chunks<G, CPL>(xs, xq);
  const int li = threadIdx.x % G, sub = (threadIdx.x & 31) / G, warp = threadIdx.x >> 5;
  for (int base = RPW * warp; base < nrows; base += RPW * (FS_THREADS / 32)) {
    const int r = base + sub;
    const bool valid = r < nrows;
    const uint8_t* wr = sq + (size_t)(valid ? r : 0) * K;
    const uint16_t* dr = sd + (size_t)(valid ? r : 0) * KB;
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < CPL; ++k) {
      const int c = li + G * k;
      const int4 w = *reinterpret_cast<const int4*>(wr + (size_t)c * 16);
      int d = __dp2a_lo(xq.v[k][0], w.x, 0);
      d = __dp2a_hi(xq.v[k][1], w.x, d);
      d = __dp2a_lo(xq.v[k][2], w.y, d);
      d = __dp2a_hi(xq.v[k][3], w.y, d);
      d = __dp2a_lo(xq.v[k][4], w.z, d);
      d = __dp2a_hi(xq.v[k][5], w.z, d);
      d = __dp2a_lo(xq.v[k][6], w.w, d);
      d = __dp2a_hi(xq.v[k][7], w.w, d);
      acc = fmaf(h2f(dr[c >> 1]) * xq.s[k], (float)d, acc);
    }
#pragma unroll
    for (int o = G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (valid && li == 0) emit(r, acc);
  }
}

// K-dispatch of gemv_q (the K values fused_step_plan admits)
template <class Emit>
__device__ __forceinline__ void gemv_smem(const uint8_t* sq, const uint16_t* sd, int K, const float* xs, int nrows,
                                          Emit emit) {
  switch (K) {
    case 512: gemv_q<16, 2>(sq, sd, xs, nrows, emit); break;
    case 768: gemv_q<16, 3>(sq, sd, xs, nrows, emit); break;
    case 1024: gemv_q<16, 4>(sq, sd, xs, nrows, emit); break;
    case 2048: gemv_q<32, 4>(sq, sd, xs, nrows, emit); break;
    case 2560: gemv_q<32, 5>(sq, sd, xs, nrows, emit); break;
    case 3072: gemv_q<32, 6>(sq, sd, xs, nrows, emit); break;
    case 4096: gemv_q<32, 8>(sq, sd, xs, nrows, emit); break;
    default: break;
  }
}

__host__ __device__ constexpr bool fused_k_ok(int K) {
  return K == 512 || K == 768 || K == 1024 || K == 2048 || K == 2560 || K == 3072 || K == 4096;
}

// xn = RmsNorm(x) * w (RmsNorm.Forward, Layers/RmsNorm.cs:14-59): mean of squares in fp32,
// 1 / (float)sqrt((double)(ms + eps)), then (x * inv) * w
__device__ __forceinline__ void rmsnorm_s(const float* x, const float* __restrict__ w, float* xn, int n, float eps,
                                          float* red) {
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += FS_THREADS) ss = fmaf(x[i], x[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x == 0) {
    float t = 0.f;
    for (int i = 0; i < FS_WARPS; ++i) t += red[i];
    red[FS_WARPS] = 1.0f / (float)sqrt((double)(t / (float)n + eps));
  }
  __syncthreads();
  const float inv = red[FS_WARPS];
  for (int i = threadIdx.x; i < n; i += FS_THREADS) xn[i] = __fmul_rn(__fmul_rn(x[i], inv), w[i]);
  __syncthreads();
}

__device__ __forceinline__ bool better(float v, int i, float best, int bi) { return v > best || (v == best && i < bi); }

// 8 fp16 values (one 16-byte word) to fp32
__device__ __forceinline__ void h8(const int4& w, float (&f)[8]) {
  const __half2* h = reinterpret_cast<const __half2*>(&w);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 v = __half22float2(h[j]);
    f[2 * j] = v.x;
    f[2 * j + 1] = v.y;
  }
}

__global__ void __launch_bounds__(FS_THREADS, 1) fused_step_kernel(FusedStepArgs a) {
  extern __shared__ __align__(128) float sm[];
  float* xs = sm;                        // residual x [dim_pad]
  float* xn = xs + a.dim_pad;            // normed x, SwiGLU input [vec_pad]
  float* rowbuf = xn + a.vec_pad;        // projection results of this CTA [row_cap]
  float* scores = rowbuf + a.row_cap;    // attention probabilities [score_cap]; sampling counts reuse it
  float* red = scores + a.score_cap;     // reductions [64]
  float* qh = red + 64;                  // one query head, pre-scaled [128]
  float* cs = qh + 128;                  // cos [0, 64) and sin [64, 128) of the step's position
  float* wave = cs + 128;                // attention reductions [FS_WAVE]
  int32_t* pts = reinterpret_cast<int32_t*>(wave + FS_WAVE);  // the sequence's page-table row [pt_pad]
  uint8_t* wts = reinterpret_cast<uint8_t*>(pts + a.pt_pad);  // staged weight rows
  __shared__ __align__(8) uint64_t bars[4];                   // staging of A, C, D, LM head
  __shared__ volatile int sh_ok;
  __shared__ volatile int sh_abort;
  __shared__ int sh_tok;
  __shared__ int sh_last;
  unsigned k_bar = 0;
  const int tid = threadIdx.x;
  const int pos = *reinterpret_cast<volatile int32_t*>(a.pos);
  const int row_pt = a.rows[0];
  const int L = a.layers;
  const int half = a.hd / 2;

  // this CTA's share of every phase
  int u0, u1, j0, j1, n0, n1, v0, v1;
  share(a.qkv_dim / 2, u0, u1);  // pairs of Wqkv rows
  share(a.ffn, j0, j1);          // FFN units
  share(a.dim, n0, n1);          // rows of Wdown (and of Wo, prefetched into L2)
  share(a.vocab, v0, v1);        // rows of the LM head
  const int nA = 2 * (u1 - u0), nC = j1 - j0, nD = n1 - n0, nV = v1 - v0;
  // staging regions: A | C (gate rows, up rows, gate scales, up scales) | D;  the LM head's rows reuse them all
  uint8_t* wA = wts;
  uint8_t* wC = wA + (size_t)nA * (a.dim + a.dim / 16);
  uint8_t* wD = wC + (size_t)2 * nC * (a.dim + a.dim / 16);
  const uint32_t bA = smem_u32(&bars[0]), bC = smem_u32(&bars[1]), bD = smem_u32(&bars[2]), bL = smem_u32(&bars[3]);
  auto stage_A = [&](int l) {
    const FusedLayerW W = a.lw[l];
    mbar_arrive_tx(bA, row_bytes(a.dim, 2 * u0, 2 * u1));
    copy_rows(wA, reinterpret_cast<uint16_t*>(wA + (size_t)nA * a.dim), W.qkv_qs, W.qkv_d, a.dim, 2 * u0, 2 * u1,
              bA);
  };
  auto stage_C = [&](int l) {
    const FusedLayerW W = a.lw[l];
    mbar_arrive_tx(bC, 2 * row_bytes(a.dim, j0, j1));
    uint16_t* dC = reinterpret_cast<uint16_t*>(wC + (size_t)2 * nC * a.dim);
    copy_rows(wC, dC, W.gu_qs, W.gu_d, a.dim, j0, j1, bC);
    copy_rows(wC + (size_t)nC * a.dim, dC + (size_t)nC * (a.dim / QK), W.gu_qs, W.gu_d, a.dim, a.ffn + j0,
              a.ffn + j1, bC);
  };
  auto stage_D = [&](int l) {
    const FusedLayerW W = a.lw[l];
    mbar_arrive_tx(bD, row_bytes(a.ffn, n0, n1));
    copy_rows(wD, reinterpret_cast<uint16_t*>(wD + (size_t)nD * a.ffn), W.dn_qs, W.dn_d, a.ffn, n0, n1, bD);
  };
  if (tid == 0) {
    sh_abort = 0;
    for (int i = 0; i < 4; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
    stage_A(0);
    stage_C(0);
    stage_D(0);
    prefetch_rows(a.lw[0].o_qs, a.lw[0].o_d, a.q_dim, n0, n1);
  }
  // the step's constants: the sequence's page-table row, RoPE angles of its position
  for (int i = tid; i < a.max_pages; i += FS_THREADS) pts[i] = a.page_table[(size_t)row_pt * a.max_pages + i];
  {
    const int pc = min(max(pos, 0), a.max_pos - 1);
    for (int i = tid; i < half; i += FS_THREADS) {
      cs[i] = a.cos_t[(size_t)pc * half + i];
      cs[64 + i] = a.sin_t[(size_t)pc * half + i];
    }
  }
  // parity of each staging barrier's next phase, and whether that phase is armed and not yet waited for; a CTA
  // that stops early first waits (bounded) for those copies
  uint32_t parA = 0, parC = 0, parD = 0;
  bool pA = true, pC = true, pD = true, pL = false;
  auto drain = [&]() {
    const uint32_t bs[4] = {bA, bC, bD, bL};
    const uint32_t pars[4] = {parA, parC, parD, 0u};
    const bool pend[4] = {pA, pC, pD, pL};
    for (int i = 0; i < 4; ++i) {
      if (!pend[i]) continue;
      const uint32_t par = pars[i];
      const uint64_t t0 = global_ns();
      while (!mbar_try(bs[i], par) && global_ns() - t0 < 100000000ull) {
      }
    }
  };

  // ---------------- 0: sample the previous step's logits ----------------
  {
    int* cnt = reinterpret_cast<int*>(scores);  // occurrences of each token of the slice in the past list
    const bool pen = a.penalty > 1.0f && a.past_len;
    __syncthreads();
    if (pen) {
      for (int i = tid; i < nV; i += FS_THREADS) cnt[i] = 0;
      __syncthreads();
      const int n = min(*a.past_len, a.past_cap);
      for (int i = tid; i < n; i += FS_THREADS) {
        const int t = a.past[i];
        if (t >= v0 && t < v1) atomicAdd(&cnt[t - v0], 1);
      }
      __syncthreads();
    }
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = v0 + tid; i < v1; i += FS_THREADS) {
      float v = a.logits[i];
      if (pen)
        for (int c = cnt[i - v0]; c > 0; --c) v = v > 0 ? v / a.penalty : v * a.penalty;
      if (better(v, i, best, bi)) {
        best = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (better(ob, oi, best, bi)) {
        best = ob;
        bi = oi;
      }
    }
    int* redi = reinterpret_cast<int*>(red + 32);
    if ((tid & 31) == 0) {
      red[tid >> 5] = best;
      redi[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float b = red[0];
      int i0 = redi[0];
      for (int w = 1; w < FS_WARPS; ++w)
        if (better(red[w], redi[w], b, i0)) {
          b = red[w];
          i0 = redi[w];
        }
      a.pairs[blockIdx.x] = make_int2(__float_as_int(b), i0);
    }
  }
  if (!grid_sync(a.ctl, k_bar, a.status, &sh_ok)) return drain();
  {
    // every CTA merges the pairs: lanes of warp 0 take strided shares, then a shuffle merge (value, then index)
    if (tid < 32) {
      float b = -INFINITY;
      int bi = 0x7fffffff;
      for (int q = tid; q < (int)gridDim.x; q += 32) {
        const int2 p = __ldcg(a.pairs + q);
        if (p.y != 0x7fffffff && better(__int_as_float(p.x), p.y, b, bi)) {
          b = __int_as_float(p.x);
          bi = p.y;
        }
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        const float ob = __shfl_xor_sync(0xffffffffu, b, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (oi != 0x7fffffff && better(ob, oi, b, bi)) {
          b = ob;
          bi = oi;
        }
      }
      if (tid == 0) {
        const int tok = bi == 0x7fffffff ? 0 : bi;  // an all-NaN row keeps index 0, as the reference's scan does
        sh_tok = tok;
        if (blockIdx.x == 0) {
          a.tokens[0] = tok;
          if (!*a.done) {
            if (a.eos >= 0 && tok == a.eos) {
              *a.done = 1;
            } else {
              a.gen_out[*a.gen_step] = tok;
              if (*a.past_len < a.past_cap) a.past[*a.past_len] = tok;
              *a.past_len += 1;
              *a.gen_step += 1;
            }
          }
        }
      }
    }
    __syncthreads();
    int tok = sh_tok;
    if (tok < 0 || tok >= a.vocab) tok = 0;  // unknown ids read row 0 (LlmEngine.cs:321)
    const int8_t* er = a.emb_qs + (size_t)tok * a.dim;
    const uint16_t* ed = a.emb_d + (size_t)tok * (a.dim / QK);
    for (int i = tid; i < a.dim; i += FS_THREADS) xs[i] = (float)er[i] * h2f(ed[i / QK]);
  }

  const int group = a.hq / a.hkv;
  const int S = a.splits;
  const int lp_pos = pos / a.page_size;
  const int page_pos = (pos >= 0 && lp_pos < a.max_pages) ? pts[lp_pos] : -1;
  for (int l = 0; l < L; ++l) {
    const FusedLayerW W = a.lw[l];
    __half* kpool = a.kpool + (size_t)l * a.layer_pool_elems;
    __half* vpool = a.vpool + (size_t)l * a.layer_pool_elems;
    // ---------------- A: RmsNorm, Wqkv, RoPE, K/V append ----------------
    rmsnorm_s(xs, a.attn_norm + (size_t)l * a.dim, xn, a.dim, a.eps, red);
    if (!mbar_wait(bA, parA, &sh_abort, a.status, 42)) {
      atomicExch(a.ctl + 1, 1u);
      return drain();
    }
    pA = false;
    parA ^= 1;
    gemv_smem(wA, reinterpret_cast<const uint16_t*>(wA + (size_t)nA * a.dim), a.dim, xn, nA,
              [&](int r, float v) { rowbuf[r] = v; });
    __syncthreads();
    for (int p = u0 + tid; p < u1; p += FS_THREADS) {
      const int row = 2 * p;
      float x0 = rowbuf[row - 2 * u0], x1 = rowbuf[row + 1 - 2 * u0];
      const int pi = (row % a.hd) / 2;
      if (row < a.q_dim + a.kv_dim) {  // RoPE.ApplyInplace on q and k
        const float c = cs[pi], s = cs[64 + pi];
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        x0 = y0;
        x1 = y1;
      }
      if (row < a.q_dim) {
        *reinterpret_cast<float2*>(a.qbuf + row) = make_float2(x0, x1);
        continue;
      }
      const bool is_k = row < a.q_dim + a.kv_dim;
      const int r = is_k ? row - a.q_dim : row - a.q_dim - a.kv_dim;
      if (page_pos < 0 || page_pos >= a.num_pages) continue;
      const size_t off =
          (((size_t)page_pos * a.hkv + r / a.hd) * a.page_size + (pos % a.page_size)) * a.hd + (r % a.hd);
      *reinterpret_cast<__half2*>((is_k ? kpool : vpool) + off) = __floats2half2_rn(x0, x1);
    }
    if (!grid_sync(a.ctl, k_bar, a.status, &sh_ok)) return drain();
    if (l + 1 < L) pA = true;
    if (tid == 0 && l + 1 < L) {  // region A is free: the next layer's Wqkv rows; its Wo share into L2
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      stage_A(l + 1);
      prefetch_rows(a.lw[l + 1].o_qs, a.lw[l + 1].o_d, a.q_dim, n0, n1);
    }

    // ---------------- B: attention partials, merge, per-head Wo ----------------
    if ((int)blockIdx.x < a.hq * S) {
      const int h = blockIdx.x / S, s = blockIdx.x % S;
      const int kvh = h / group;
      const int n = (a.quirk && l != L - 1) ? pos : pos + 1;  // LlmEngine.cs:254, PagedKvCache.cs:139-142
      const int t0 = (int)((long long)n * s / S), t1 = (int)((long long)n * (s + 1) / S);
      for (int i = tid; i < a.hd; i += FS_THREADS) qh[i] = ldcg(a.qbuf + (size_t)h * a.hd + i) * a.scale_log2;
      __syncthreads();
      // waves of W tokens: TPT threads per token, 8 dims (one 16-byte word of K and of V) each
      const int TPT = a.hd / 8, Wt = FS_THREADS / TPT;
      const int tw = tid / TPT, g = tid % TPT;
      const bool one_wave = t1 - t0 <= Wt;
      float vreg[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int w0 = t0; w0 < t1; w0 += Wt) {
        const int t = w0 + tw;
        int4 kw = make_int4(0, 0, 0, 0), vw = make_int4(0, 0, 0, 0);
        bool ok = false;
        if (t < t1) {
          const int page = pts[t / a.page_size];
          if (page >= 0 && page < a.num_pages) {
            const size_t off = (((size_t)page * a.hkv + kvh) * a.page_size + (t % a.page_size)) * a.hd + 8 * g;
            kw = ldcg4(kpool + off);
            if (one_wave) vw = ldcg4(vpool + off);
            ok = true;
          }
        }
        float kf[8];
        h8(kw, kf);
        float part = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) part = fmaf(qh[8 * g + j], kf[j], part);
        for (int o = TPT / 2; o > 0; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
        if (t < t1 && g == 0) scores[t - t0] = ok ? part : -INFINITY;
        if (one_wave) h8(vw, vreg);
      }
      __syncthreads();
      const int warp = tid >> 5, lane = tid & 31;
      float m = -INFINITY;
      for (int i = tid; i < t1 - t0; i += FS_THREADS) m = fmaxf(m, scores[i]);
      m = warp_max(m);
      if (lane == 0) red[warp] = m;
      __syncthreads();
      m = red[0];
      for (int w = 1; w < FS_WARPS; ++w) m = fmaxf(m, red[w]);
      __syncthreads();
      float lsum = 0.f;
      for (int i = tid; i < t1 - t0; i += FS_THREADS) {
        const float p = m == -INFINITY ? 0.f : exp2f(scores[i] - m);
        scores[i] = p;
        lsum += p;
      }
      lsum = warp_sum(lsum);
      if (lane == 0) red[warp] = lsum;
      __syncthreads();
      lsum = 0.f;
      for (int w = 0; w < FS_WARPS; ++w) lsum += red[w];
      // o[d] = sum_t p_t v_t[d]: a wave's p * v words go to `wave` [Wt][hd]; thread (block b, dim d) sums 8 tokens
      // of the wave, and the blocks' sums are added in order
      float o_acc = 0.f;  // threads d < hd
      const int blocks = FS_THREADS / a.hd, per = Wt / blocks;
      const int dd = tid % a.hd, bb = tid / a.hd;
      for (int w0 = t0; w0 < t1; w0 += Wt) {
        const int t = w0 + tw;
        float pv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        if (t < t1) {
          const float p = scores[t - t0];
          if (!one_wave) {
            const int page = pts[t / a.page_size];
            int4 vw = make_int4(0, 0, 0, 0);
            if (page >= 0 && page < a.num_pages)
              vw = ldcg4(vpool + (((size_t)page * a.hkv + kvh) * a.page_size + (t % a.page_size)) * a.hd + 8 * g);
            h8(vw, vreg);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) pv[j] = p * vreg[j];
        }
        __syncthreads();  // the previous wave's block sums have been read
#pragma unroll
        for (int j = 0; j < 8; ++j) wave[tw * a.hd + 8 * g + j] = pv[j];
        __syncthreads();
        float ps = 0.f;
        for (int i = 0; i < per; ++i) ps += wave[(bb * per + i) * a.hd + dd];
        __syncthreads();
        wave[bb * a.hd + dd] = ps;
        __syncthreads();
        if (tid < a.hd) {
          float ws = 0.f;
          for (int q = 0; q < blocks; ++q) ws += wave[q * a.hd + tid];
          o_acc += ws;
        }
      }
      float* part = a.part + ((size_t)h * S + s) * (a.hd + 2);
      if (tid < a.hd) part[2 + tid] = o_acc;
      if (tid == 0) {
        part[0] = m;
        part[1] = lsum;
      }
      // this split's Wo items (row, 16-column chunk of head h): the first batch's loads go out before the wait,
      // since the weights do not depend on the attention
      const int cpr = a.hd / 16, kb = a.q_dim / QK;
      const int rw0 = (int)((long long)a.dim * s / S), rw1 = (int)((long long)a.dim * (s + 1) / S);
      const int items = (rw1 - rw0) * cpr;
      int4 w[8];
      float sc[8];
      auto load_wo = [&](int it0) {
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int it = it0 + j * FS_THREADS + tid;
          const int row = rw0 + it / cpr, c = it % cpr;
          const bool ok = it < items;
          w[j] = ok ? ld_stream_v4(W.o_qs + (size_t)row * a.q_dim + (size_t)h * a.hd + c * 16) : make_int4(0, 0, 0, 0);
          sc[j] = ok ? h2f(__ldg(W.o_d + (size_t)row * kb + (size_t)h * (a.hd / QK) + (c >> 1))) : 0.f;
        }
      };
      load_wo(0);
      // every split of head h waits (bounded) for the head's S partials -- all CTAs of a cooperative launch are
      // resident, so the wait ends -- then merges them and computes its share of the head's Wo rows
      __syncthreads();
      if (tid == 0) {
        red_release_gpu(a.ctl + 3 + h, 1u);
        const unsigned want = (unsigned)S * (unsigned)(l + 1);
        const uint64_t tw0 = global_ns();
        uint32_t polls = 0;
        int ok = 1;
        while (ld_acquire_gpu(a.ctl + 3 + h) < want) {
          if ((++polls & 31) == 0 &&
              (*reinterpret_cast<volatile unsigned*>(a.ctl + 1) || global_ns() - tw0 > FS_WAIT_NS)) {
            atomicExch(a.ctl + 1, 1u);
            atomicExch(a.status, 41);
            ok = 0;
            break;
          }
        }
        sh_last = ok;
      }
      __syncthreads();
      if (!sh_last) return drain();
      // merge the S partials in split order (exp2 domain): out = sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M)
      const float* phd = a.part + (size_t)h * S * (a.hd + 2);
      for (int i = tid; i < S * (a.hd + 2); i += FS_THREADS) wave[i] = ldcg(phd + i);
      __syncthreads();
      float* attn = scores;  // [hd]
      for (int i = tid; i < a.hd; i += FS_THREADS) {
        float M = -INFINITY;
        for (int q = 0; q < S; ++q) M = fmaxf(M, wave[q * (a.hd + 2)]);
        float num = 0.f, den = 0.f;
        if (M != -INFINITY)
          for (int q = 0; q < S; ++q) {
            const float* pq = wave + q * (a.hd + 2);
            if (pq[0] == -INFINITY) continue;
            const float f = exp2f(pq[0] - M);
            den = fmaf(pq[1], f, den);
            num = fmaf(pq[2 + i], f, num);
          }
        attn[i] = den > 0.f ? num / den : 0.f;  // ctx 0 gives zeros (GqaAttention.cs:38-42)
      }
      __syncthreads();
      // P[h][row] = Wo[row, head h's hd columns] . attn_h for this split's rows: items (row, 16-column chunk), a
      // batch's loads all in flight; the cpr chunks of a row are adjacent lanes and meet in a shuffle reduction
      for (int it0 = 0; it0 < items; it0 += 8 * FS_THREADS) {
        if (it0 > 0) load_wo(it0);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const int it = it0 + j * FS_THREADS + tid;
          const int c = it % cpr;
          float v = it < items ? sc[j] * dot16_s(w[j], attn + c * 16) : 0.f;
          for (int o = cpr / 2; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
          if (it < items && c == 0) a.P[(size_t)h * a.dim + rw0 + it / cpr] = v;
        }
      }
    }
    if (!grid_sync(a.ctl, k_bar, a.status, &sh_ok)) return drain();

    // ---------------- C: x += Wo . attn (summed over heads), RmsNorm, Wgate / Wup, SwiGLU ----------------
    for (int i = tid; i < a.dim; i += FS_THREADS) {
      float acc = 0.f;
      for (int h0 = 0; h0 < a.hq; h0 += 16) {
        float v[16];
#pragma unroll
        for (int u = 0; u < 16; ++u) v[u] = h0 + u < a.hq ? ldcg(a.P + (size_t)(h0 + u) * a.dim + i) : 0.f;
#pragma unroll
        for (int u = 0; u < 16; ++u)
          if (h0 + u < a.hq) acc = (h0 + u == 0) ? v[u] : acc + v[u];
      }
      xs[i] = xs[i] + acc;
    }
    __syncthreads();
    rmsnorm_s(xs, a.ffn_norm + (size_t)l * a.dim, xn, a.dim, a.eps, red);
    if (!mbar_wait(bC, parC, &sh_abort, a.status, 42)) {
      atomicExch(a.ctl + 1, 1u);
      return drain();
    }
    pC = false;
    parC ^= 1;
    const uint16_t* dC = reinterpret_cast<const uint16_t*>(wC + (size_t)2 * nC * a.dim);
    gemv_smem(wC, dC, a.dim, xn, 2 * nC, [&](int r, float v) { rowbuf[r] = v; });  // gate rows, then up rows
    __syncthreads();
    for (int j = tid; j < nC; j += FS_THREADS) {  // SwiGLU.Forward (Layers/SwiGLU.cs:13-51)
      const float g = rowbuf[j], u = rowbuf[nC + j];
      const float sg = 1.0f / (1.0f + expf(-g));
      a.hbuf[j0 + j] = __fmul_rn(__fmul_rn(g, sg), u);
    }
    if (!grid_sync(a.ctl, k_bar, a.status, &sh_ok)) return drain();
    if (l + 1 < L) pC = true;
    if (tid == 0 && l + 1 < L) {  // region C is free: the next layer's Wgate / Wup rows
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      stage_C(l + 1);
    }

    // ---------------- D: x_new = x + Wdown . SwiGLU (MatVecAddQ8_0), this CTA's rows ----------------
    for (int i0 = 0; i0 < a.ffn; i0 += 4 * FS_THREADS) {
      float v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * FS_THREADS + tid;
        v[u] = i < a.ffn ? ldcg(a.hbuf + i) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int i = i0 + u * FS_THREADS + tid;
        if (i < a.ffn) xn[i] = v[u];
      }
    }
    __syncthreads();
    if (!mbar_wait(bD, parD, &sh_abort, a.status, 42)) {
      atomicExch(a.ctl + 1, 1u);
      return drain();
    }
    pD = false;
    parD ^= 1;
    gemv_smem(wD, reinterpret_cast<const uint16_t*>(wD + (size_t)nD * a.ffn), a.ffn, xn, nD,
              [&](int r, float v) { a.x[n0 + r] = xs[n0 + r] + v; });
    if (!grid_sync(a.ctl, k_bar, a.status, &sh_ok)) return drain();
    if (l + 1 < L) pD = true;
    else pL = true;
    if (tid == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      if (l + 1 < L) {
        stage_D(l + 1);
      } else {  // after the last layer every region is free: the LM head's rows
        mbar_arrive_tx(bL, row_bytes(a.dim, v0, v1));
        copy_rows(wts, reinterpret_cast<uint16_t*>(wts + (size_t)nV * a.dim), a.lm_qs, a.lm_d, a.dim, v0, v1, bL);
      }
    }
    for (int i = tid; i < a.dim; i += FS_THREADS) xs[i] = ldcg(a.x + i);
    __syncthreads();
  }

  // ---------------- LM head ----------------
  rmsnorm_s(xs, a.final_norm, xn, a.dim, a.eps, red);
  if (!mbar_wait(bL, 0, &sh_abort, a.status, 42)) {
    atomicExch(a.ctl + 1, 1u);
    return drain();
  }
  gemv_smem(wts, reinterpret_cast<const uint16_t*>(wts + (size_t)nV * a.dim), a.dim, xn, nV,
            [&](int r, float v) { a.logits[v0 + r] = v; });
  if (blockIdx.x == 0 && tid == 0) *a.pos = pos + 1;
}

}  // namespace

int fused_step_plan(FusedStepArgs& a, int sms, int max_ctx, size_t* smem, const char** why) {
  auto no = [&](const char* m) {
    if (why) *why = m;
    return kUnsupported;
  };
  if (a.hd != 64 && a.hd != 128) return no("head size must be 64 or 128");
  if (a.dim % 256 || a.ffn % 256 || a.q_dim % 256) return no("dim, ffn and q_dim must be multiples of 256");
  if (!fused_k_ok(a.dim) || !fused_k_ok(a.ffn)) return no("dim and ffn must be 512, 768, 1024, 2048, 2560, 3072 or 4096");
  if (a.hq % a.hkv || a.hq > sms) return no("heads must divide by kv heads and fit the grid");
  if (a.page_size <= 0 || max_ctx <= 0 || a.max_pages <= 0) return no("no context capacity");
  if (a.max_pages > 4096) return no("page-table row above 4096 pages");
  a.splits = std::max(1, sms / a.hq);
  if (a.splits * (a.hd + 2) > FS_WAVE) return no("too many attention splits for the merge area");
  const int score_cap = (max_ctx + a.splits - 1) / a.splits + 1;
  const int vocab_share = (a.vocab + sms - 1) / sms + 1;
  a.score_cap = (std::max(score_cap, std::max(vocab_share, a.hd)) + 3) / 4 * 4;
  a.dim_pad = (a.dim + 3) / 4 * 4;
  a.vec_pad = (std::max(a.dim, a.ffn) + 3) / 4 * 4;
  const int qkv_rows = 2 * ((a.qkv_dim / 2 + sms - 1) / sms);
  const int ffn_units = (a.ffn + sms - 1) / sms;
  const int down_rows = (a.dim + sms - 1) / sms;
  const int lm_rows = (a.vocab + sms - 1) / sms;
  a.row_cap = (std::max(qkv_rows, 2 * ffn_units) + 3) / 4 * 4;
  a.pt_pad = (a.max_pages + 3) / 4 * 4;
  const size_t rb_dim = (size_t)a.dim + a.dim / 16, rb_ffn = (size_t)a.ffn + a.ffn / 16;
  const size_t layer_bytes = (size_t)qkv_rows * rb_dim + (size_t)2 * ffn_units * rb_dim + (size_t)down_rows * rb_ffn;
  const size_t wt_bytes = std::max(layer_bytes, (size_t)lm_rows * rb_dim);
  if (wt_bytes >= (1u << 20)) return no("a CTA's staged rows above 1 MB");
  const size_t floats = (size_t)a.dim_pad + a.vec_pad + a.row_cap + a.score_cap + 64 + 128 + 128 + FS_WAVE + a.pt_pad;
  const size_t bytes = floats * sizeof(float) + (wt_bytes + 15) / 16 * 16;
  if (bytes > 220 * 1024) return no("shared-memory plan above 220 KB");
  a.scale_log2 = (1.0f / (float)std::sqrt((double)a.hd)) * FS_LOG2E;
  *smem = bytes;
  return kOk;
}

size_t fused_step_scratch_floats(const FusedStepArgs& a, int sms) {
  // part [hq][S][hd + 2], P [hq][dim], qbuf [q_dim], hbuf [ffn], x [dim], pairs [sms] (int2)
  return (size_t)a.hq * a.splits * (a.hd + 2) + (size_t)a.hq * a.dim + a.q_dim + a.ffn + a.dim + 2 * (size_t)sms + 64;
}

int fused_step_launch(const FusedStepArgs& a, int sms, size_t smem, cudaStream_t s) {
  // per device (the attribute belongs to the current device's context); a host call of about a microsecond
  if (cudaFuncSetAttribute(fused_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
    return kCudaError;
  if (cudaMemsetAsync(a.ctl, 0, (3 + a.hq) * sizeof(unsigned), s) != cudaSuccess) return kCudaError;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(sms);
  cfg.blockDim = dim3(FS_THREADS);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;  // every CTA resident at once: the grid barriers rely on it
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, fused_step_kernel, a) == cudaSuccess ? kOk : kCudaError;
}

}  // namespace zc
