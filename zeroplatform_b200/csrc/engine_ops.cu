// engine_ops.cu -- small kernels of the device decode step (LlmEngine.ForwardToken / PrefillPrompt pieces).
//
//   rope_append_kv   RoPE.ApplyInplace on q and k (Layers/RoPE.cs:131-163) + PagedKvCache.AppendToken /
//                    AppendTokenAt (Memory/PagedKvCache.cs:237-316) into fp16 pages [page][kv head][slot][hd]
//   swiglu_rows      SwiGLU.Forward (Layers/SwiGLU.cs:13-51) on [T][gate | up] rows
//   greedy_sample    LlmSampler.Sample greedy branch with repetition penalty (Sampling/LlmSampler.cs:21-72)
//   causal_lengths   per-layer causal context lengths (LlmEngine.cs:254, PagedKvCache.cs:139-142)
//   advance_generation  GenerateStreamAsync bookkeeping between steps (Engine/LlmEngine.cs:115-141)

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

// Element e of a projection's output: qkv[e] itself, or (part != nullptr) the sum of the GEMM's split-K partials
// part[s * stride + e] in split order -- the order splitk_reduce_kernel adds them in, so the values are the same.
__device__ __forceinline__ float split_sum(const float* __restrict__ y, const float* __restrict__ part, int splits,
                                           size_t stride, size_t e) {
  if (!part) return y[e];
  float v = part[e];
  for (int s = 1; s < splits; ++s) v += part[(size_t)s * stride + e];
  return v;
}

__global__ void rope_append_kernel(float* __restrict__ qkv, const float* __restrict__ part, int splits, size_t stride,
                                   int T, int hq, int hkv, int hd,
                                   const int32_t* __restrict__ pos, const int32_t* __restrict__ rows,
                                   const int32_t* __restrict__ page_table, int max_pages, int page_size,
                                   const float* __restrict__ cos_t, const float* __restrict__ sin_t, int max_pos,
                                   __half* __restrict__ k_pool, __half* __restrict__ v_pool) {
  pdl_trigger();
  pdl_wait();
  const int half = hd / 2;
  const int q_dim = hq * hd, kv_dim = hkv * hd;
  const int row_len = q_dim + 2 * kv_dim;
  const int heads = hq + 2 * hkv;  // q heads, k heads, v heads
  const size_t total = (size_t)T * heads * half;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % half);
    const int h = (int)((i / half) % heads);
    const int t = (int)(i / ((size_t)half * heads));
    const int ps = pos[t];
    float* row = qkv + (size_t)t * row_len;
    float* v = row + (size_t)h * hd + 2 * p;  // q, k and v heads are consecutive in the row
    const size_t e = (size_t)(v - qkv);
    float x0 = split_sum(qkv, part, splits, stride, e), x1 = split_sum(qkv, part, splits, stride, e + 1);
    if (h < hq + hkv) {  // rotate q and k
      const int pc = min(max(ps, 0), max_pos - 1);
      const float c = cos_t[(size_t)pc * half + p], s = sin_t[(size_t)pc * half + p];
      const float r0 = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
      const float r1 = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
      x0 = r0;
      x1 = r1;
      if (h < hq) {
        v[0] = x0;
        v[1] = x1;
        continue;
      }
    }
    if (part) {  // the row holds the projection (v unrotated) as the separate reduction would have left it
      v[0] = x0;
      v[1] = x1;
    }
    // k or v head: append to the page pool
    const int lp = ps / page_size;
    if (ps < 0 || lp >= max_pages) continue;
    const int page = page_table[(size_t)rows[t] * max_pages + lp];
    if (page < 0) continue;
    const int kvh = h < hq + hkv ? h - hq : h - hq - hkv;
    __half* pool = h < hq + hkv ? k_pool : v_pool;
    const size_t off = (((size_t)page * hkv + kvh) * page_size + (ps % page_size)) * hd + 2 * p;
    *reinterpret_cast<__half2*>(pool + off) = __floats2half2_rn(x0, x1);
    if (h < hq + hkv) {  // the rotated k is also kept in the row (used by nothing downstream, kept for tests)
      v[0] = x0;
      v[1] = x1;
    }
  }
}

template <typename OutT>
__global__ void swiglu_rows_kernel(const float* __restrict__ gu, const float* __restrict__ part, int splits,
                                   size_t stride, OutT* __restrict__ out, int T, int ffn) {
  pdl_trigger();
  pdl_wait();
  const size_t total = (size_t)T * ffn;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int t = (int)(i / ffn), j = (int)(i % ffn);
    const float g = split_sum(gu, part, splits, stride, (size_t)t * 2 * ffn + j);
    const float u = split_sum(gu, part, splits, stride, (size_t)t * 2 * ffn + ffn + j);
    const float sg = 1.0f / (1.0f + expf(-g));
    constexpr int kPlanes = sizeof(OutT) == 2 ? 2 : 1;  // __half: rows [hi ffn | lo ffn]
    store_act(out + (size_t)t * ffn * kPlanes + j, (size_t)ffn, __fmul_rn(__fmul_rn(g, sg), u));
  }
}

// One CTA per row.  The penalty is applied occurrence by occurrence, in order, as the reference loops over
// pastTokens (a token seen c times is divided c times); only thread 0 touches the penalised logits.
// With a vocabulary split over ranks (vocab_offset = first token id of this rank's logits), the penalty
// touches the past tokens that fall in this rank's range, and `pairs` receives (best value, global index) per
// row for greedy_merge instead of a token in `out`.
__global__ void greedy_kernel(float* __restrict__ logits, int vocab, const int32_t* __restrict__ past,
                              const int32_t* __restrict__ past_len, int past_cap, float penalty,
                              int32_t* __restrict__ out, int vocab_offset, int2* __restrict__ pairs) {
  pdl_trigger();
  pdl_wait();
  float* lg = logits + (size_t)blockIdx.x * vocab;
  if (penalty > 1.0f && past && past_len) {
    if (threadIdx.x == 0) {
      const int n = min(past_len[blockIdx.x], past_cap);
      const int32_t* pt = past + (size_t)blockIdx.x * past_cap;
      for (int i = 0; i < n; ++i) {
        const unsigned tok = (unsigned)(pt[i] - vocab_offset);
        if (pt[i] >= vocab_offset && tok < (unsigned)vocab) lg[tok] = lg[tok] > 0 ? lg[tok] / penalty : lg[tok] * penalty;
      }
    }
    __syncthreads();
  }
  float best = -INFINITY;
  int idx = 0x7fffffff;
  for (int i = threadIdx.x; i < vocab; i += blockDim.x) {
    const float v = lg[i];
    if (v > best || (v == best && i < idx)) {
      best = v;
      idx = i;
    }
  }
  __shared__ float sb[32];
  __shared__ int si[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ob = __shfl_xor_sync(0xffffffffu, best, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ob > best || (ob == best && oi < idx)) {
      best = ob;
      idx = oi;
    }
  }
  if ((threadIdx.x & 31) == 0) {
    sb[threadIdx.x >> 5] = best;
    si[threadIdx.x >> 5] = idx;
  }
  __syncthreads();
  if (threadIdx.x == 0) {
    float b = sb[0];
    int bi = si[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w)
      if (sb[w] > b || (sb[w] == b && si[w] < bi)) {
        b = sb[w];
        bi = si[w];
      }
    if (pairs) {
      pairs[blockIdx.x] = make_int2(__float_as_int(b), bi == 0x7fffffff ? bi : bi + vocab_offset);
    } else {
      // all-NaN rows keep index 0, as the reference's scan does
      out[blockIdx.x] = bi == 0x7fffffff ? 0 : bi;
    }
  }
}

// pairs [ranks][rows] of (value bits, global index) -> the row's token: largest value, lowest index on ties.
__global__ void greedy_merge_kernel(const int2* __restrict__ pairs, int ranks, int rows, int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  for (int r = blockIdx.x * blockDim.x + threadIdx.x; r < rows; r += gridDim.x * blockDim.x) {
    float best = -INFINITY;
    int idx = 0x7fffffff;
    for (int k = 0; k < ranks; ++k) {
      const int2 p = pairs[(size_t)k * rows + r];
      const float v = __int_as_float(p.x);
      if (p.y == 0x7fffffff) continue;
      if (v > best || (v == best && p.y < idx)) {
        best = v;
        idx = p.y;
      }
    }
    out[r] = idx == 0x7fffffff ? 0 : idx;
  }
}

// Batched generation bookkeeping: every sequence's sampled token becomes its next input and is recorded.
__global__ void batch_advance_kernel(const int32_t* __restrict__ next, int32_t* __restrict__ tokens,
                                     int32_t* __restrict__ pos, int32_t* __restrict__ out, int out_stride,
                                     int32_t* __restrict__ step, int B) {
  pdl_trigger();
  pdl_wait();
  const int st = *step;
  for (int b = threadIdx.x; b < B; b += blockDim.x) {
    const int t = next[b];
    if (st < out_stride) out[(size_t)b * out_stride + st] = t;
    tokens[b] = t;
    pos[b] += 1;
  }
  __syncthreads();
  if (threadIdx.x == 0) *step = st + 1;
}

// PagedKvCache.AppendTokenAt for a run of tokens: src rows [n][kvh][hd] (fp32 or fp16) to the fp16 pools.
template <class T>
__global__ void append_kv_kernel(const T* __restrict__ k, const T* __restrict__ v, int n, int start, int kvh, int hd,
                                 const int32_t* __restrict__ pt_row, int max_pages, int page_size,
                                 __half* __restrict__ k_pool, __half* __restrict__ v_pool) {
  const size_t total = (size_t)n * kvh * hd;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int e = (int)(i % hd);
    const int h = (int)((i / hd) % kvh);
    const int t = (int)(i / ((size_t)hd * kvh));
    const int p = start + t;
    const int lp = p / page_size;
    if (lp >= max_pages) continue;
    const int page = pt_row[lp];
    if (page < 0) continue;
    const size_t off = (((size_t)page * kvh + h) * page_size + (p % page_size)) * hd + e;
    k_pool[off] = __float2half_rn((float)k[i]);
    v_pool[off] = __float2half_rn((float)v[i]);
  }
}

__global__ void causal_kernel(const int32_t* __restrict__ pos, int B, int32_t* __restrict__ ex,
                              int32_t* __restrict__ in) {
  pdl_trigger();
  pdl_wait();
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < B) {
    ex[b] = pos[b];
    in[b] = pos[b] + 1;
  }
}

__global__ void advance_kernel(const int32_t* __restrict__ tok, int32_t* __restrict__ pos, int32_t* __restrict__ out,
                               int32_t* __restrict__ step, int32_t* __restrict__ past, int32_t* __restrict__ past_len,
                               int past_cap, int eos, int32_t* __restrict__ done) {
  pdl_trigger();
  pdl_wait();
  if (threadIdx.x != 0 || blockIdx.x != 0) return;
  if (*done) return;
  const int t = tok[0];
  if (eos >= 0 && t == eos) {
    *done = 1;
    return;
  }
  out[*step] = t;
  if (*past_len < past_cap) past[*past_len] = t;
  *past_len += 1;
  *step += 1;
}

inline int grid_for(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

inline int launched() { return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError; }

}  // namespace

int rope_append_kv(float* qkv, int T, int hq, int hkv, int hd, const int32_t* pos, const int32_t* rows,
                   const int32_t* page_table, int max_pages, int page_size, const float* cos_t, const float* sin_t,
                   int max_pos, __half* k_pool, __half* v_pool, cudaStream_t s) {
  if (!qkv || !pos || !rows || !page_table || !cos_t || !sin_t || !k_pool || !v_pool || (hd & 1)) return kBadArgument;
  if (T <= 0) return kOk;
  const size_t n = (size_t)T * (hq + 2 * hkv) * (hd / 2);
  return launch_pdl(rope_append_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, qkv, (const float*)nullptr, 1,
                    (size_t)0, T, hq, hkv, hd, pos, rows, page_table, max_pages, page_size, cos_t, sin_t, max_pos,
                    k_pool, v_pool) == cudaSuccess
             ? kOk
             : kCudaError;
}

int rope_append_kv_parts(const float* part, int splits, float* qkv, int T, int hq, int hkv, int hd,
                         const int32_t* pos, const int32_t* rows, const int32_t* page_table, int max_pages,
                         int page_size, const float* cos_t, const float* sin_t, int max_pos, __half* k_pool,
                         __half* v_pool, cudaStream_t s) {
  if (!part || splits < 1 || !qkv || !pos || !rows || !page_table || !cos_t || !sin_t || !k_pool || !v_pool ||
      (hd & 1))
    return kBadArgument;
  if (T <= 0) return kOk;
  const size_t n = (size_t)T * (hq + 2 * hkv) * (hd / 2);
  const size_t stride = (size_t)T * (hq + 2 * hkv) * hd;
  return launch_pdl(rope_append_kernel, dim3(grid_for(n, 256)), dim3(256), 0, s, qkv, part, splits, stride, T, hq,
                    hkv, hd, pos, rows, page_table, max_pages, page_size, cos_t, sin_t, max_pos, k_pool,
                    v_pool) == cudaSuccess
             ? kOk
             : kCudaError;
}

int swiglu_rows(const float* gu, float* out, int T, int ffn, cudaStream_t s) {
  if (!gu || !out) return kBadArgument;
  if (T <= 0) return kOk;
  return launch_pdl(swiglu_rows_kernel<float>, dim3(grid_for((size_t)T * ffn, 256)), dim3(256), 0, s, gu,
                    (const float*)nullptr, 1, (size_t)0, out, T, ffn) == cudaSuccess
             ? kOk
             : kCudaError;
}

int swiglu_rows_h(const float* gu, __half* out, int T, int ffn, cudaStream_t s) {
  if (!gu || !out) return kBadArgument;
  if (T <= 0) return kOk;
  return launch_pdl(swiglu_rows_kernel<__half>, dim3(grid_for((size_t)T * ffn, 256)), dim3(256), 0, s, gu,
                    (const float*)nullptr, 1, (size_t)0, out, T, ffn) == cudaSuccess
             ? kOk
             : kCudaError;
}

int swiglu_rows_h_parts(const float* part, int splits, __half* out, int T, int ffn, cudaStream_t s) {
  if (!part || splits < 1 || !out) return kBadArgument;
  if (T <= 0) return kOk;
  return launch_pdl(swiglu_rows_kernel<__half>, dim3(grid_for((size_t)T * ffn, 256)), dim3(256), 0, s, part, part,
                    splits, (size_t)T * 2 * ffn, out, T, ffn) == cudaSuccess
             ? kOk
             : kCudaError;
}

int greedy_sample(float* logits, int rows, int vocab, const int32_t* past, const int32_t* past_len, int past_cap,
                  float penalty, int32_t* out, cudaStream_t s) {
  if (!logits || !out || rows <= 0 || vocab <= 0) return kBadArgument;
  return launch_pdl(greedy_kernel, dim3(rows), dim3(1024), 0, s, logits, vocab, past, past_len, past_cap, penalty, out,
                    0, (int2*)nullptr) == cudaSuccess
             ? kOk
             : kCudaError;
}

int greedy_partial(float* logits, int rows, int vocab, int vocab_offset, const int32_t* past, const int32_t* past_len,
                   int past_cap, float penalty, int2* pairs, cudaStream_t s) {
  if (!logits || !pairs || rows <= 0 || vocab <= 0) return kBadArgument;
  return launch_pdl(greedy_kernel, dim3(rows), dim3(1024), 0, s, logits, vocab, past, past_len, past_cap, penalty,
                    (int32_t*)nullptr, vocab_offset, pairs) == cudaSuccess
             ? kOk
             : kCudaError;
}

int greedy_merge(const int2* pairs, int ranks, int rows, int32_t* out, cudaStream_t s) {
  if (!pairs || !out || ranks <= 0 || rows <= 0) return kBadArgument;
  return launch_pdl(greedy_merge_kernel, dim3((rows + 255) / 256), dim3(256), 0, s, pairs, ranks, rows, out) ==
                 cudaSuccess
             ? kOk
             : kCudaError;
}

int batch_advance(const int32_t* next, int32_t* tokens, int32_t* pos, int32_t* out, int out_stride, int32_t* step,
                  int B, cudaStream_t s) {
  if (!next || !tokens || !pos || !out || !step || B <= 0) return kBadArgument;
  return launch_pdl(batch_advance_kernel, dim3(1), dim3(1024), 0, s, next, tokens, pos, out, out_stride, step, B) ==
                 cudaSuccess
             ? kOk
             : kCudaError;
}

int append_kv(const void* k, const void* v, int half_input, int n, int start, int kvh, int hd, const int32_t* pt_row,
              int max_pages, int page_size, __half* k_pool, __half* v_pool, cudaStream_t s) {
  if (!k || !v || !pt_row || !k_pool || !v_pool || n < 0 || start < 0) return kBadArgument;
  if (n == 0) return kOk;
  const size_t total = (size_t)n * kvh * hd;
  if (half_input)
    append_kv_kernel<__half><<<grid_for(total, 256), 256, 0, s>>>(static_cast<const __half*>(k),
                                                                 static_cast<const __half*>(v), n, start, kvh, hd,
                                                                 pt_row, max_pages, page_size, k_pool, v_pool);
  else
    append_kv_kernel<float><<<grid_for(total, 256), 256, 0, s>>>(static_cast<const float*>(k),
                                                                static_cast<const float*>(v), n, start, kvh, hd,
                                                                pt_row, max_pages, page_size, k_pool, v_pool);
  return launched();
}

int causal_lengths(const int32_t* pos, int B, int32_t* ctx_excl, int32_t* ctx_incl, cudaStream_t s) {
  if (!pos || !ctx_excl || !ctx_incl) return kBadArgument;
  if (B <= 0) return kOk;
  return launch_pdl(causal_kernel, dim3((B + 255) / 256), dim3(256), 0, s, pos, B, ctx_excl, ctx_incl) == cudaSuccess
             ? kOk
             : kCudaError;
}

int advance_generation(const int32_t* tok, int32_t* pos, int32_t* out, int32_t* step, int32_t* past,
                       int32_t* past_len, int past_cap, int eos, int32_t* done, cudaStream_t s) {
  return launch_pdl(advance_kernel, dim3(1), dim3(32), 0, s, tok, pos, out, step, past, past_len, past_cap, eos,
                    done) == cudaSuccess
             ? kOk
             : kCudaError;
}

}  // namespace zc
