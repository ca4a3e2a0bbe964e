// sampler.cu -- LlmSampler.Sample on the device (ZeroLlm/src/ZeroLlm.Core/Sampling/LlmSampler.cs:21-172), every
// branch, so that no logits leave the GPU whatever the SamplingConfig:
//
//   1  repetition penalty, occurrence by occurrence in past-list order (:39-57), in place
//   2  greedy (Temperature <= 0.001 or TopK == 1): the first maximum, index 0 when logits[0] is NaN (:60-73)
//   3  temperature: logits *= 1 / T, in place (:76-80)
//   4  softmax: max, exp in double rounded to float, sum, probabilities in place (:83-101)
//   5  candidates p > 1e-6 by probability descending (:104-113); Top-K (:116-119), Min-P (:122-132), Top-P
//      cumulative cutoff (:135-150), renormalisation (:153-155), and the CDF walk with the supplied draw (:158-171)
//
// One CTA of 1024 threads per row.  Steps 1-4 are block-parallel (the softmax sum is a tree, not the reference's
// left-to-right float sum: probabilities agree to a few ulp).  The candidate pool is cut to its Top-K without a full
// sort: a 4-pass radix select on the probability bits finds the K-th largest value, the candidates above it and the
// lowest-index ones equal to it are gathered into shared memory, and a bitonic sort orders them by probability
// descending, lower token id first among equal ones (.NET's List.Sort leaves that order unspecified).  Min-P, Top-P,
// the renormalisation and the CDF walk then run in the reference's sequential order on the sorted prefix.  Pools
// above SAMPLE_MAX_CAND candidates after Top-K (TopK 0 over a flat distribution) are refused: the row's token is -1.

#include <cuda_runtime.h>
#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

constexpr int SAMPLE_THREADS = 1024;
constexpr int SAMPLE_WARPS = SAMPLE_THREADS / 32;

__device__ __forceinline__ bool greater_key(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* red, Op op) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    T w = red[threadIdx.x];  // SAMPLE_WARPS == 32
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) w = op(w, __shfl_xor_sync(0xffffffffu, w, o));
    if (threadIdx.x == 0) red[0] = w;
  }
  __syncthreads();
  const T r = red[0];
  __syncthreads();
  return r;
}

__global__ void __launch_bounds__(SAMPLE_THREADS) sample_kernel(float* __restrict__ logits, int vocab,
                                                                  const int32_t* __restrict__ past,
                                                                  const int32_t* __restrict__ past_len, int past_cap,
                                                                  const int32_t* __restrict__ past_rows,
                                                                  SampleConfig cfg0,
                                                                  const SampleConfig* __restrict__ row_cfg,
                                                                  const float* __restrict__ uniforms,
                                                                  int32_t* __restrict__ out, int32_t* cand_idx,
                                                                  float* cand_p, int32_t* n_cand, int cand_cap) {
  pdl_trigger();
  pdl_wait();
  const SampleConfig cfg = row_cfg ? row_cfg[blockIdx.x] : cfg0;
  const int prow = past_rows ? past_rows[blockIdx.x] : (int)blockIdx.x;  // this row's history
  __shared__ float redf[32];
  __shared__ int redi[32];
  __shared__ unsigned hist[256];
  __shared__ float sv[SAMPLE_MAX_CAND];
  __shared__ int si[SAMPLE_MAX_CAND];
  __shared__ int s_count;
  __shared__ unsigned s_prefix;
  __shared__ int s_remaining;
  __shared__ int s_base;
  const int row = blockIdx.x, tid = threadIdx.x;
  float* lg = logits + (size_t)row * vocab;
  // 1. repetition penalty (thread 0, the reference's order)
  if (cfg.penalty > 1.0f && past && past_len && tid == 0) {
    const int n = min(past_len[prow], past_cap);
    const int32_t* pt = past + (size_t)prow * past_cap;
    for (int i = 0; i < n; ++i) {
      const unsigned t = (unsigned)pt[i];
      if (t < (unsigned)vocab) lg[t] = lg[t] > 0 ? lg[t] / cfg.penalty : lg[t] * cfg.penalty;
    }
  }
  __syncthreads();
  // 2. greedy
  if (cfg.temperature <= 0.001f || cfg.top_k == 1) {
    float best = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
      const float v = lg[i];
      if (greater_key(v, i, best, bi)) {  // NaN never compares greater
        best = v;
        bi = i;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (greater_key(ob, oi, best, bi)) {
        best = ob;
        bi = oi;
      }
    }
    if ((tid & 31) == 0) {
      redf[tid >> 5] = best;
      redi[tid >> 5] = bi;
    }
    __syncthreads();
    if (tid == 0) {
      float b = redf[0];
      int i0 = redi[0];
      for (int w = 1; w < SAMPLE_WARPS; ++w)
        if (greater_key(redf[w], redi[w], b, i0)) {
          b = redf[w];
          i0 = redi[w];
        }
      // the reference starts from logits[0]: a NaN there compares false against everything and index 0 stays
      out[row] = (isnan(lg[0]) || i0 == 0x7fffffff || !(b > lg[0] || i0 == 0)) ? 0 : i0;
      if (n_cand) n_cand[row] = 0;
    }
    return;
  }
  // 3. temperature, 4. softmax (in place, as the reference)
  const float inv_temp = 1.0f / cfg.temperature;
  float mx = -INFINITY;
  for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
    const float v = lg[i] * inv_temp;
    lg[i] = v;
    if (v > mx) mx = v;
  }
  mx = block_reduce(mx, redf, [](float a, float b) { return b > a ? b : a; });
  float sum = 0.f;
  for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
    const float e = (float)exp((double)(lg[i] - mx));
    lg[i] = e;
    sum += e;
  }
  sum = block_reduce(sum, redf, [](float a, float b) { return a + b; });
  const float inv_sum = sum > 0 ? 1.0f / sum : 0.0f;
  int cnt = 0;
  for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
    const float p = lg[i] * inv_sum;
    lg[i] = p;
    cnt += p > 1e-6f;
  }
  cnt = block_reduce(cnt, redi, [](int a, int b) { return a + b; });
  const int want = cfg.top_k > 0 ? min(cfg.top_k, cnt) : cnt;
  if (want > SAMPLE_MAX_CAND) {
    if (tid == 0) {
      out[row] = -1;
      if (n_cand) n_cand[row] = -1;
    }
    return;
  }
  // 5a. radix select: the want-th largest probability among the candidates (positive floats order as their bits)
  if (tid == 0) {
    s_prefix = 0;
    s_remaining = want;
  }
  __syncthreads();
  unsigned mask = 0;
  for (int shift = 24; shift >= 0 && want > 0; shift -= 8) {
    for (int b = tid; b < 256; b += SAMPLE_THREADS) hist[b] = 0;
    __syncthreads();
    const unsigned prefix = s_prefix;
    for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
      const float p = lg[i];
      if (!(p > 1e-6f)) continue;
      const unsigned key = __float_as_uint(p);
      if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & 255u], 1u);
    }
    __syncthreads();
    if (tid == 0) {
      int rem = s_remaining;
      for (int b = 255; b >= 0; --b) {
        const int h = (int)hist[b];
        if (h >= rem) {
          s_prefix = prefix | ((unsigned)b << shift);
          break;
        }
        rem -= h;
      }
      s_remaining = rem;
    }
    mask |= 255u << shift;
    __syncthreads();
  }
  // 5b. gather: every candidate above the threshold, and the lowest-index ones equal to it (index order)
  const unsigned thr = s_prefix;
  const int need_eq = s_remaining;  // how many candidates equal to the threshold are taken
  if (tid == 0) {
    s_count = 0;
    s_base = 0;
  }
  __syncthreads();
  if (want > 0) {
    for (int i = tid; i < vocab; i += SAMPLE_THREADS) {
      const float p = lg[i];
      if (p > 1e-6f && __float_as_uint(p) > thr) {
        const int slot = atomicAdd(&s_count, 1);
        sv[slot] = p;
        si[slot] = i;
      }
    }
    __syncthreads();
    const int n_gt = s_count;
    for (int i0 = 0; i0 < vocab && s_base < need_eq; i0 += SAMPLE_THREADS) {  // s_base: equal ones taken so far
      const int i = i0 + tid;
      const bool eq = i < vocab && lg[i] > 1e-6f && __float_as_uint(lg[i]) == thr;
      // block exclusive scan of eq in index order
      const unsigned ballot = __ballot_sync(0xffffffffu, eq);
      const int lane = tid & 31, warp = tid >> 5;
      if (lane == 0) redi[warp] = __popc(ballot);
      __syncthreads();
      int before = 0;
      for (int w = 0; w < warp; ++w) before += redi[w];
      before += __popc(ballot & ((1u << lane) - 1u));
      const int base = s_base;
      if (eq && base + before < need_eq) {
        sv[n_gt + base + before] = lg[i];
        si[n_gt + base + before] = i;
      }
      __syncthreads();
      if (tid == 0) {
        int tot = 0;
        for (int w = 0; w < SAMPLE_WARPS; ++w) tot += redi[w];
        s_base = base + tot;
      }
      __syncthreads();
    }
  }
  // 5c. bitonic sort of the want items (probability descending, lower index first); padding sorts last
  int n2 = 1;
  while (n2 < want) n2 <<= 1;
  for (int i = want + tid; i < n2; i += SAMPLE_THREADS) {
    sv[i] = -1.0f;
    si[i] = 0x7fffffff;
  }
  __syncthreads();
  for (int k = 2; k <= n2; k <<= 1)
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = tid; i < n2; i += SAMPLE_THREADS) {
        const int l = i ^ j;
        if (l > i) {
          const bool up = (i & k) == 0;  // this run is ordered "greater first"
          const bool swap = up ? greater_key(sv[l], si[l], sv[i], si[i]) : greater_key(sv[i], si[i], sv[l], si[l]);
          if (swap) {
            const float tv = sv[i];
            sv[i] = sv[l];
            sv[l] = tv;
            const int ti = si[i];
            si[i] = si[l];
            si[l] = ti;
          }
        }
      }
      __syncthreads();
    }
  // 5d. Min-P, Top-P, renormalisation, CDF walk: the reference's sequential order on the sorted prefix
  if (tid == 0) {
    int n = want;
    if (cfg.min_p > 0.0f && n > 0) {
      const float thr_p = sv[0] * cfg.min_p;
      int keep = 1;
      while (keep < n && !(sv[keep] < thr_p)) ++keep;
      n = keep;
    }
    float cumulative = 0.0f;
    for (int i = 0; i < n; ++i) {
      cumulative += sv[i];
      if (cumulative >= cfg.top_p) {
        n = i + 1;
        break;
      }
    }
    float total = 0.0f;
    for (int i = 0; i < n; ++i) total += sv[i];
    const float inv_total = total > 0 ? 1.0f / total : 1.0f;
    const float u = uniforms[row];
    float running = 0.0f;
    int tok = n > 0 ? si[0] : 0;
    for (int i = 0; i < n; ++i) {
      running += sv[i] * inv_total;
      if (u <= running) {
        tok = si[i];
        break;
      }
    }
    out[row] = tok;
    if (n_cand) n_cand[row] = n;
    if (cand_idx && cand_p)
      for (int i = 0; i < n && i < cand_cap; ++i) {
        cand_idx[(size_t)row * cand_cap + i] = si[i];
        cand_p[(size_t)row * cand_cap + i] = sv[i] * inv_total;
      }
  }
}

// u[row] = the top 24 bits of SplitMix64(seed + counter + row), scaled to [0, 1); counter += rows.
__global__ void uniform_kernel(uint64_t seed, int32_t* counter, int rows, float* u) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  const uint64_t c = (uint64_t)(uint32_t)*counter;
  __syncthreads();
  if (r < rows) u[r] = splitmix_uniform(seed + c + (uint64_t)r);
  if (r == 0 && blockIdx.x == 0) {
    // every thread of block 0 read *counter before the update (the __syncthreads above); rows <= blockDim.x
    *counter = (int32_t)(c + (uint64_t)rows);
  }
}

}  // namespace

int sample_rows(float* logits, int rows, int vocab, const int32_t* past, const int32_t* past_len, int past_cap,
                const SampleConfig& cfg, const float* uniforms, int32_t* out, int32_t* cand_idx, float* cand_p,
                int32_t* n_cand, int cand_cap, cudaStream_t s) {
  if (!logits || !out || rows <= 0 || vocab <= 0) return kBadArgument;
  const bool greedy = cfg.temperature <= 0.001f || cfg.top_k == 1;
  if (!greedy && !uniforms) return kBadArgument;
  if (cfg.top_k < 0) return kBadArgument;
  return launch_pdl(sample_kernel, dim3(rows), dim3(SAMPLE_THREADS), 0, s, logits, vocab, past, past_len, past_cap,
                    (const int32_t*)nullptr, cfg, (const SampleConfig*)nullptr, uniforms, out, cand_idx, cand_p,
                    n_cand, cand_cap) == cudaSuccess
             ? kOk
             : kCudaError;
}

int sample_rows_each(float* logits, int rows, int vocab, const int32_t* past, const int32_t* past_len, int past_cap,
                     const int32_t* past_rows, const SampleConfig* row_cfg, const float* uniforms, int32_t* out,
                     cudaStream_t s) {
  if (!logits || !out || !row_cfg || !uniforms || rows <= 0 || vocab <= 0) return kBadArgument;
  return launch_pdl(sample_kernel, dim3(rows), dim3(SAMPLE_THREADS), 0, s, logits, vocab, past, past_len, past_cap,
                    past_rows, SampleConfig{}, row_cfg, uniforms, out, (int32_t*)nullptr, (float*)nullptr,
                    (int32_t*)nullptr, 0) == cudaSuccess
             ? kOk
             : kCudaError;
}

namespace {
// past[past_rows[r]][past_len[past_rows[r]]++] = tok[r] while the row has room (past_cap).
__global__ void append_history_kernel(const int32_t* tok, const int32_t* past_rows, int rows, int32_t* past,
                                      int32_t* past_len, int past_cap) {
  pdl_trigger();
  pdl_wait();
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= rows) return;
  const int p = past_rows[r];
  const int n = past_len[p];
  if (n < past_cap) {
    past[(size_t)p * past_cap + n] = tok[r];
    past_len[p] = n + 1;
  }
}
}  // namespace

int append_history(const int32_t* tok, const int32_t* past_rows, int rows, int32_t* past, int32_t* past_len,
                   int past_cap, cudaStream_t s) {
  if (!tok || !past_rows || !past || !past_len || rows <= 0 || past_cap <= 0) return kBadArgument;
  return launch_pdl(append_history_kernel, dim3((rows + 127) / 128), dim3(128), 0, s, tok, past_rows, rows, past,
                    past_len, past_cap) == cudaSuccess
             ? kOk
             : kCudaError;
}

int draw_uniforms(uint64_t seed, int32_t* counter, int rows, float* u, cudaStream_t s) {
  if (!counter || !u || rows <= 0 || rows > 1024) return kBadArgument;
  return launch_pdl(uniform_kernel, dim3(1), dim3(rows < 32 ? 32 : rows), 0, s, seed, counter, rows, u) == cudaSuccess
             ? kOk
             : kCudaError;
}

}  // namespace zc
