// decode_fused.cu -- one greedy generation step of a Q8_0 Llama-style model for one sequence as a single
// persistent (cooperative) kernel: LlmSampler.Sample's greedy branch with repetition penalty
// (Sampling/LlmSampler.cs:21-72), the GenerateStreamAsync bookkeeping (Engine/LlmEngine.cs:115-141), the token
// embedding (LlmEngine.cs:317-345) and LlmEngine.ForwardToken (LlmEngine.cs:347-461) over the paged fp16 KV cache.
//
// Why one kernel: at batch 1 a small model's step is a chain of ~80 dependent launches whose weight reads are a
// few hundred KB each, so the chain's latency, not HBM, sets the step time.  Here one CTA per SM runs the whole
// step, and the points where a vector must be complete before anyone reads it become grid barriers (an arrival
// counter in global memory, polled by one thread per CTA, bounded by a time limit after which every CTA stops and
// the status word records code 41):
//
//   0  sample     each CTA: arg-max of its vocabulary slice of the previous logits, with the repetition penalty
//                 applied occurrence by occurrence to the past tokens in the slice  -> pairs   | barrier
//                 every CTA merges the pairs (largest value, lowest index); CTA 0 records the token (eos, output,
//                 past list); every CTA dequantizes the token's embedding row into shared memory
//   per layer:
//   A  qkv        every CTA: RmsNorm of x (redundantly, x in shared memory); its pairs of Wqkv rows; RoPE on q and
//                 k pairs; q -> qbuf, k and v -> the layer's fp16 pages at the token's slot          | barrier
//   B  attention  CTA (head h, split s) for h < hq, s < S: online-softmax partial over its slice of the context
//                 (the reference's causal rule: non-final layers attend to [0, pos)); the last split of a head to
//                 arrive (atomic counter) merges the partials in split order and multiplies the head's output by
//                 its 32-block columns of Wo: P[h] = Wo[:, head h] . attn_h                       | barrier
//   C  ffn up     every CTA: x += sum over h of P[h] (head order; the same in every CTA), RmsNorm, its units of
//                 Wgate and Wup, SwiGLU -> hbuf                                                     | barrier
//   D  ffn down   every CTA: its rows of x_new = x + Wdown . hbuf -> global x                        | barrier
//   LM head       every CTA: RmsNorm with the final norm, its rows of the LM head -> logits; CTA 0 advances pos
//
// Every weight byte is read once per step.  While a phase runs, each CTA asks L2 (cp.async.bulk.prefetch.L2) for
// the weight rows it needs in later phases, so the barrier waits overlap the HBM reads.  Data written in this
// kernel by another CTA (qbuf, K/V pages, partials, P, hbuf, x, pairs) is read through L2 (ld.global.cg); weights
// through the non-coherent path.  Projections compute in fp32 on exactly converted int8 values (as the GEMV's
// fp32 forms); Wo is summed per head and then over heads, another fp32 order than one MatVecAdd over all columns.

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int FS_THREADS = 512;
constexpr int FS_WARPS = FS_THREADS / 32;
constexpr int FS_G = 16;                      // lanes per weight row
constexpr int FS_ROWS_PER_PASS = FS_THREADS / FS_G;
constexpr uint64_t FS_WAIT_NS = 2000000000ull;  // a grid barrier that waits longer than 2 s gives up
constexpr float FS_LOG2E = 1.4426950408889634f;

__device__ __forceinline__ uint64_t fs_now() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ unsigned ld_acquire_gpu(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Grid barrier: every CTA arrives once; `target` counts arrivals expected so far.  Returns false when the wait
// ran out or another CTA gave up (then every thread of the CTA returns from the kernel).
__device__ __forceinline__ bool grid_sync(unsigned* ctl, unsigned& target, int* status, int* sh_ok) {
  __syncthreads();
  target += gridDim.x;
  if (threadIdx.x == 0) {
    int ok = 1;
    __threadfence();
    atomicAdd(ctl, 1u);
    const uint64_t t0 = fs_now();
    uint32_t polls = 0;
    while (ld_acquire_gpu(ctl) < target) {
      if (*reinterpret_cast<volatile unsigned*>(ctl + 1)) {
        ok = 0;
        break;
      }
      if ((++polls & 63) == 0 && fs_now() - t0 > FS_WAIT_NS) {
        atomicExch(ctl + 1, 1u);
        atomicExch(status, 41);
        ok = 0;
        break;
      }
    }
    __threadfence();
    *sh_ok = ok;
  }
  __syncthreads();
  return *sh_ok != 0;
}

__device__ __forceinline__ float ldcg(const float* p) { return __ldcg(p); }

// units [b, e) of `n` balanced over the grid
__device__ __forceinline__ void share(int n, int& b, int& e) {
  b = (int)((long long)n * blockIdx.x / gridDim.x);
  e = (int)((long long)n * (blockIdx.x + 1) / gridDim.x);
}

__device__ __forceinline__ void prefetch_rows(const int8_t* qs, const uint16_t* d, int K, int r0, int r1) {
  if (r1 <= r0) return;
  const size_t n = (size_t)(r1 - r0);
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(qs + (size_t)r0 * K), "r"((unsigned)(n * K))
               : "memory");
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(d + (size_t)r0 * (K / QK)),
               "r"((unsigned)(n * (K / QK) * 2))
               : "memory");
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

// Rows [r0, r1) of a Q8_0 matrix (SoA, K columns) times x (shared memory): FS_G lanes per row, chunks strided
// over the lanes, a shuffle reduction over the FS_G lanes; emit(row, value) runs on the group's first lane.
template <class Emit>
__device__ __forceinline__ void gemv_rows(const int8_t* __restrict__ qs, const uint16_t* __restrict__ d, int K,
                                          const float* xs, int r0, int r1, Emit emit) {
  const int gi = threadIdx.x / FS_G, li = threadIdx.x % FS_G;
  const int warp = threadIdx.x >> 5, sub = gi & 1;  // a warp holds two row groups
  const int nch = K / 16, kb = K / QK;
  // the loop is uniform over the warp (both groups iterate together, a missing row computes zeros), so the
  // full-warp shuffles below always have all 32 lanes
  for (int base = r0 + 2 * warp; base < r1; base += FS_ROWS_PER_PASS) {
    const int row = base + sub;
    const bool valid = row < r1;
    const int8_t* wr = qs + (size_t)(valid ? row : r0) * K;
    const uint16_t* dr = d + (size_t)(valid ? row : r0) * kb;
    float acc = 0.f;
    for (int c0 = li; c0 < nch; c0 += 4 * FS_G) {
      int4 w[4];
      float sc[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * FS_G;
        w[u] = c < nch ? ld_stream_v4(wr + (size_t)c * 16) : make_int4(0, 0, 0, 0);
        sc[u] = c < nch ? h2f(__ldg(dr + (c >> 1))) : 0.f;
      }
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const int c = c0 + u * FS_G;
        if (c < nch) acc = fmaf(sc[u], dot16_s(w[u], xs + c * 16), acc);
      }
    }
#pragma unroll
    for (int o = FS_G / 2; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (valid && li == 0) emit(row, acc);
  }
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

__global__ void __launch_bounds__(FS_THREADS, 1) fused_step_kernel(FusedStepArgs a) {
  extern __shared__ __align__(16) float sm[];
  float* xs = sm;                         // residual x [dim]
  float* xn = xs + a.dim_pad;             // normed x / attention output [max(dim, ffn) padded]
  float* rowbuf = xn + a.vec_pad;         // projection results of this CTA [row_cap]
  float* scores = rowbuf + a.row_cap;     // attention probabilities [score_cap]; sampling counts reuse it
  float* red = scores + a.score_cap;      // reductions [64]
  float* qh = red + 64;                   // one query head, pre-scaled [128]
  __shared__ int sh_ok;
  __shared__ int sh_tok;
  unsigned target = 0;
  const int tid = threadIdx.x;
  const int pos = *reinterpret_cast<volatile int32_t*>(a.pos);
  const int row_pt = a.rows[0];
  const int L = a.layers;

  // ---------------- 0: sample the previous step's logits ----------------
  {
    int v0, v1;
    share(a.vocab, v0, v1);
    int* cnt = reinterpret_cast<int*>(scores);  // occurrences of each token of the slice in the past list
    const bool pen = a.penalty > 1.0f && a.past_len;
    if (pen) {
      for (int i = tid; i < v1 - v0; i += FS_THREADS) cnt[i] = 0;
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
  if (!grid_sync(a.ctl, target, a.status, &sh_ok)) return;
  if (tid == 0) {
    float b = -INFINITY;
    int bi = 0x7fffffff;
    for (int k = 0; k < (int)gridDim.x; ++k) {
      const int2 p = __ldcg(a.pairs + k);
      if (p.y == 0x7fffffff) continue;
      if (better(__int_as_float(p.x), p.y, b, bi)) {
        b = __int_as_float(p.x);
        bi = p.y;
      }
    }
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
  __syncthreads();
  {
    int tok = sh_tok;
    if (tok < 0 || tok >= a.vocab) tok = 0;  // unknown ids read row 0 (LlmEngine.cs:321)
    const int8_t* er = a.emb_qs + (size_t)tok * a.dim;
    const uint16_t* ed = a.emb_d + (size_t)tok * (a.dim / QK);
    for (int i = tid; i < a.dim; i += FS_THREADS) xs[i] = (float)er[i] * h2f(ed[i / QK]);
  }

  const int half = a.hd / 2;
  const int group = a.hq / a.hkv;
  const int S = a.splits;
  for (int l = 0; l < L; ++l) {
    const FusedLayerW W = a.lw[l];
    __half* kpool = a.kpool + (size_t)l * a.layer_pool_elems;
    __half* vpool = a.vpool + (size_t)l * a.layer_pool_elems;
    int u0, u1, j0, j1, n0, n1;
    share(a.qkv_dim / 2, u0, u1);  // pairs of Wqkv rows
    share(a.ffn, j0, j1);          // FFN units
    share(a.dim, n0, n1);          // rows of Wdown
    // L2 prefetch of this CTA's later rows: Wo (a contiguous share, read column-wise in B), Wgate/Wup, Wdown
    if (tid == 0) {
      prefetch_rows(W.o_qs, W.o_d, a.q_dim, n0, n1);
      prefetch_rows(W.gu_qs, W.gu_d, a.dim, j0, j1);
      prefetch_rows(W.gu_qs, W.gu_d, a.dim, a.ffn + j0, a.ffn + j1);
      prefetch_rows(W.dn_qs, W.dn_d, a.ffn, n0, n1);
    }
    // ---------------- A: RmsNorm, Wqkv, RoPE, K/V append ----------------
    rmsnorm_s(xs, a.attn_norm + (size_t)l * a.dim, xn, a.dim, a.eps, red);
    const int r0 = 2 * u0, r1 = 2 * u1;
    gemv_rows(W.qkv_qs, W.qkv_d, a.dim, xn, r0, r1, [&](int row, float v) { rowbuf[row - r0] = v; });
    __syncthreads();
    for (int p = u0 + tid; p < u1; p += FS_THREADS) {
      const int row = 2 * p;
      float x0 = rowbuf[row - r0], x1 = rowbuf[row + 1 - r0];
      const int pi = (row % a.hd) / 2;
      if (row < a.q_dim + a.kv_dim) {  // RoPE.ApplyInplace on q and k
        const int pc = min(max(pos, 0), a.max_pos - 1);
        const float c = a.cos_t[(size_t)pc * half + pi], s = a.sin_t[(size_t)pc * half + pi];
        const float y0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
        const float y1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
        x0 = y0;
        x1 = y1;
      }
      if (row < a.q_dim) {
        a.qbuf[row] = x0;
        a.qbuf[row + 1] = x1;
        continue;
      }
      const bool is_k = row < a.q_dim + a.kv_dim;
      const int r = is_k ? row - a.q_dim : row - a.q_dim - a.kv_dim;
      const int kvh = r / a.hd;
      const int lp = pos / a.page_size;
      if (pos < 0 || lp >= a.max_pages) continue;
      const int page = a.page_table[(size_t)row_pt * a.max_pages + lp];
      if (page < 0 || page >= a.num_pages) continue;
      const size_t off = (((size_t)page * a.hkv + kvh) * a.page_size + (pos % a.page_size)) * a.hd + (r % a.hd);
      *reinterpret_cast<__half2*>((is_k ? kpool : vpool) + off) = __floats2half2_rn(x0, x1);
    }
    if (!grid_sync(a.ctl, target, a.status, &sh_ok)) return;

    // ---------------- B: attention partials, merge, per-head Wo ----------------
    if ((int)blockIdx.x < a.hq * S) {
      const int h = blockIdx.x / S, s = blockIdx.x % S;
      const int kvh = h / group;
      const int n = (a.quirk && l != L - 1) ? pos : pos + 1;  // LlmEngine.cs:254, PagedKvCache.cs:139-142
      const int t0 = (int)((long long)n * s / S), t1 = (int)((long long)n * (s + 1) / S);
      float* ob = xn;   // per-group output partials [groups][hd]
      for (int i = tid; i < a.hd; i += FS_THREADS) qh[i] = ldcg(a.qbuf + (size_t)h * a.hd + i) * a.scale_log2;
      __syncthreads();
      // scores: one warp per token, lanes over the dimensions
      const int warp = tid >> 5, lane = tid & 31;
      const int dpl = a.hd / 32;  // 2 or 4 dims per lane
      for (int t = t0 + warp; t < t1; t += FS_WARPS) {
        const int lp = t / a.page_size;
        const int page = a.page_table[(size_t)row_pt * a.max_pages + lp];
        float sc = -INFINITY;
        if (page >= 0 && page < a.num_pages) {
          const __half* kr = kpool + (((size_t)page * a.hkv + kvh) * a.page_size + (t % a.page_size)) * a.hd;
          float part = 0.f;
          for (int e = 0; e < dpl; e += 2) {
            const int dd = lane * dpl + e;
            const unsigned raw = __ldcg(reinterpret_cast<const unsigned*>(kr + dd));
            const float2 kv = __half22float2(*reinterpret_cast<const __half2*>(&raw));
            part = fmaf(qh[dd], kv.x, part);
            part = fmaf(qh[dd + 1], kv.y, part);
          }
          sc = warp_sum(part);
        }
        if (lane == 0) scores[t - t0] = sc;
      }
      __syncthreads();
      float m = -INFINITY;
      for (int i = tid; i < t1 - t0; i += FS_THREADS) m = fmaxf(m, scores[i]);
      m = warp_max(m);
      __shared__ float wred[FS_WARPS];
      if (lane == 0) wred[warp] = m;
      __syncthreads();
      m = wred[0];
      for (int w = 1; w < FS_WARPS; ++w) m = fmaxf(m, wred[w]);
      __syncthreads();
      float lsum = 0.f;
      for (int i = tid; i < t1 - t0; i += FS_THREADS) {
        const float p = m == -INFINITY ? 0.f : exp2f(scores[i] - m);
        scores[i] = p;
        lsum += p;
      }
      lsum = warp_sum(lsum);
      if (lane == 0) wred[warp] = lsum;
      __syncthreads();
      lsum = 0.f;
      for (int w = 0; w < FS_WARPS; ++w) lsum += wred[w];
      // o[d] = sum_t p_t v_t[d]: token groups of hd threads, then a sum over the groups in order
      const int ng = FS_THREADS / a.hd, g = tid / a.hd, dd = tid % a.hd;
      float o = 0.f;
      for (int t = t0 + g; t < t1; t += ng) {
        const int lp = t / a.page_size;
        const int page = a.page_table[(size_t)row_pt * a.max_pages + lp];
        const float p = scores[t - t0];
        if (page < 0 || page >= a.num_pages || p == 0.f) continue;
        const __half* vr = vpool + (((size_t)page * a.hkv + kvh) * a.page_size + (t % a.page_size)) * a.hd;
        const unsigned short raw = __ldcg(reinterpret_cast<const unsigned short*>(vr + dd));
        o = fmaf(p, __half2float(__ushort_as_half(raw)), o);
      }
      ob[g * a.hd + dd] = o;
      __syncthreads();
      float* part = a.part + ((size_t)h * S + s) * (a.hd + 2);
      for (int i = tid; i < a.hd; i += FS_THREADS) {
        float acc = 0.f;
        for (int gg = 0; gg < ng; ++gg) acc += ob[gg * a.hd + i];
        part[2 + i] = acc;
      }
      if (tid == 0) {
        part[0] = m;
        part[1] = lsum;
      }
      __threadfence();
      __syncthreads();
      __shared__ int last;
      if (tid == 0) last = atomicAdd(a.ctl + 2 + h, 1u) == (unsigned)(S - 1);
      __syncthreads();
      if (last) {
        if (tid == 0) a.ctl[2 + h] = 0;
        __threadfence();
        // merge the S partials in split order (exp2 domain): out = sum_s o_s 2^(m_s - M) / sum_s l_s 2^(m_s - M)
        float* attn = scores;  // [hd]
        const float* ph = a.part + (size_t)h * S * (a.hd + 2);
        for (int i = tid; i < a.hd; i += FS_THREADS) {
          float M = -INFINITY;
          for (int q = 0; q < S; ++q) M = fmaxf(M, ldcg(ph + (size_t)q * (a.hd + 2)));
          float num = 0.f, den = 0.f;
          if (M != -INFINITY)
            for (int q = 0; q < S; ++q) {
              const float* pq = ph + (size_t)q * (a.hd + 2);
              const float mq = ldcg(pq);
              if (mq == -INFINITY) continue;
              const float f = exp2f(mq - M);
              den = fmaf(ldcg(pq + 1), f, den);
              num = fmaf(ldcg(pq + 2 + i), f, num);
            }
          attn[i] = den > 0.f ? num / den : 0.f;  // ctx 0 gives zeros (GqaAttention.cs:38-42)
        }
        __syncthreads();
        // P[h][row] = Wo[row, head h's columns] . attn_h: hd / 16 chunks and hd / 32 scales per row
        const int cpr = a.hd / 16, kb = a.q_dim / QK;
        for (int row = tid; row < a.dim; row += FS_THREADS) {
          const int8_t* wr = W.o_qs + (size_t)row * a.q_dim + (size_t)h * a.hd;
          const uint16_t* dr = W.o_d + (size_t)row * kb + (size_t)h * (a.hd / QK);
          float acc = 0.f;
          for (int c = 0; c < cpr; ++c) acc = fmaf(h2f(__ldg(dr + (c >> 1))), dot16_s(ld_stream_v4(wr + c * 16), attn + c * 16), acc);
          a.P[(size_t)h * a.dim + row] = acc;
        }
      }
    }
    if (!grid_sync(a.ctl, target, a.status, &sh_ok)) return;

    // ---------------- C: x += Wo . attn (summed over heads), RmsNorm, Wgate / Wup, SwiGLU ----------------
    for (int i = tid; i < a.dim; i += FS_THREADS) {
      float acc = ldcg(a.P + i);
      for (int h = 1; h < a.hq; ++h) acc += ldcg(a.P + (size_t)h * a.dim + i);
      xs[i] = xs[i] + acc;
    }
    __syncthreads();
    rmsnorm_s(xs, a.ffn_norm + (size_t)l * a.dim, xn, a.dim, a.eps, red);
    if (l + 1 < L && tid == 0) {  // the next layer's Wqkv pairs of this CTA
      const FusedLayerW Wn = a.lw[l + 1];
      prefetch_rows(Wn.qkv_qs, Wn.qkv_d, a.dim, 2 * u0, 2 * u1);
    } else if (tid == 0) {
      int v0, v1;
      share(a.vocab, v0, v1);
      prefetch_rows(a.lm_qs, a.lm_d, a.dim, v0, v1);
    }
    const int nu = j1 - j0;
    gemv_rows(W.gu_qs, W.gu_d, a.dim, xn, j0, j1, [&](int row, float v) { rowbuf[row - j0] = v; });
    gemv_rows(W.gu_qs, W.gu_d, a.dim, xn, a.ffn + j0, a.ffn + j1,
              [&](int row, float v) { rowbuf[nu + row - a.ffn - j0] = v; });
    __syncthreads();
    for (int j = tid; j < nu; j += FS_THREADS) {  // SwiGLU.Forward (Layers/SwiGLU.cs:13-51)
      const float g = rowbuf[j], u = rowbuf[nu + j];
      const float sg = 1.0f / (1.0f + expf(-g));
      a.hbuf[j0 + j] = __fmul_rn(__fmul_rn(g, sg), u);
    }
    if (!grid_sync(a.ctl, target, a.status, &sh_ok)) return;

    // ---------------- D: x_new = x + Wdown . SwiGLU (MatVecAddQ8_0), this CTA's rows ----------------
    for (int i = tid; i < a.ffn; i += FS_THREADS) xn[i] = ldcg(a.hbuf + i);
    __syncthreads();
    gemv_rows(W.dn_qs, W.dn_d, a.ffn, xn, n0, n1, [&](int row, float v) { a.x[row] = xs[row] + v; });
    if (!grid_sync(a.ctl, target, a.status, &sh_ok)) return;
    for (int i = tid; i < a.dim; i += FS_THREADS) xs[i] = ldcg(a.x + i);
    __syncthreads();
  }

  // ---------------- LM head ----------------
  rmsnorm_s(xs, a.final_norm, xn, a.dim, a.eps, red);
  int v0, v1;
  share(a.vocab, v0, v1);
  gemv_rows(a.lm_qs, a.lm_d, a.dim, xn, v0, v1, [&](int row, float v) { a.logits[row] = v; });
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
  if (a.hq % a.hkv || a.hq > sms) return no("heads must divide by kv heads and fit the grid");
  if ((long long)a.hq * a.dim > 65536) return no("heads x dim above 65536");
  if (a.page_size <= 0 || max_ctx <= 0) return no("no context capacity");
  a.splits = std::max(1, sms / a.hq);
  const int score_cap = (max_ctx + a.splits - 1) / a.splits + 1;
  const int vocab_share = (a.vocab + sms - 1) / sms + 1;
  a.score_cap = (std::max(score_cap, std::max(vocab_share, a.hd)) + 3) / 4 * 4;
  a.dim_pad = (a.dim + 3) / 4 * 4;
  a.vec_pad = (std::max(a.dim, std::max(a.ffn, (FS_THREADS / a.hd) * a.hd)) + 3) / 4 * 4;
  const int qkv_rows = 2 * ((a.qkv_dim / 2 + sms - 1) / sms);
  const int ffn_rows = 2 * ((a.ffn + sms - 1) / sms);
  a.row_cap = (std::max(qkv_rows, ffn_rows) + 3) / 4 * 4;
  const size_t bytes = (size_t)(a.dim_pad + a.vec_pad + a.row_cap + a.score_cap + 64 + 128) * sizeof(float);
  if (bytes > 200 * 1024) return no("shared-memory plan above 200 KB");
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
  if (cudaMemsetAsync(a.ctl, 0, (2 + a.hq) * sizeof(unsigned), s) != cudaSuccess) return kCudaError;
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
