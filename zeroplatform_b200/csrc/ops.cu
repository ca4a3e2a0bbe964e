// ops.cu -- the small operators between the quantized GEMVs of a decode step.
//
//   rmsnorm    RmsNorm.Forward           (ZeroLlm/src/ZeroLlm.Core/Layers/RmsNorm.cs:14-59)
//   rope       RoPE.ApplyInplace         (Layers/RoPE.cs:131-163), interleaved pairs (2i, 2i+1),
//              cos/sin tables computed on the host in double exactly as RoPE.EnsureCache (:83-125)
//   swiglu     SwiGLU.Forward            (Layers/SwiGLU.cs:13-51): (g * sigmoid(g)) * up
//   silu       TensorOps SiLU            (ZeroTensor bridge zc_silu_f32)
//   embed      LlmEngine.LookupTokenEmbedding for Q8_0 tables (Engine/LlmEngine.cs:317-345)
//   copy_words the host-pointer entries' zero-copy transfers (pinned, mapped host buffers)
// All are HBM/latency bound element-wise kernels.

#include <math.h>

#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

// One CTA per row.  OutT = float, or __half when the row feeds the tensor-core GEMM directly: then out rows are
// [hi n | lo n] (store_hl).  Launched with programmatic dependent launch: it waits for the previous kernel
// before reading x.
template <typename OutT>
__global__ void rmsnorm_kernel(const float* __restrict__ x, const float* __restrict__ w, OutT* __restrict__ out,
                               int n, float eps) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const float* xr = x + (size_t)blockIdx.x * n;
  constexpr int kPlanes = sizeof(OutT) == 2 ? 2 : 1;
  OutT* orow = out + (size_t)blockIdx.x * n * kPlanes;
  float ss = 0.f;
  for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float mean_sq = red[0] / (float)n;
  const float inv = 1.0f / (float)sqrt((double)(mean_sq + eps));
  for (int i = threadIdx.x; i < n; i += blockDim.x) store_act(orow + i, (size_t)n, xr[i] * inv * w[i]);
}

__global__ void swiglu_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                              size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float gv = g[i];
    const float s = 1.0f / (1.0f + expf(-gv));
    out[i] = (gv * s) * u[i];
  }
}

__global__ void silu_kernel(const float* __restrict__ x, float* __restrict__ out, size_t n) {
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
    const float v = x[i];
    out[i] = v / (1.0f + expf(-v));
  }
}

__global__ void rope_kernel(float* __restrict__ x, int rows, int heads, int hd, const int32_t* __restrict__ pos,
                            int pos0, const float* __restrict__ cos_t, const float* __restrict__ sin_t,
                            int max_pos) {
  const int half = hd / 2;
  const size_t total = (size_t)rows * heads * half;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % half);
    const size_t rh = i / half;
    const int row = (int)(rh / heads);
    int ps = pos ? pos[row] : pos0 + row;
    ps = min(max(ps, 0), max_pos - 1);
    const float c = cos_t[(size_t)ps * half + p], s = sin_t[(size_t)ps * half + p];
    float* v = x + rh * hd + 2 * p;
    const float x0 = v[0], x1 = v[1];
    // separate roundings, no contraction: the reference computes x0*c - x1*s with two products
    v[0] = __fsub_rn(__fmul_rn(x0, c), __fmul_rn(x1, s));
    v[1] = __fadd_rn(__fmul_rn(x0, s), __fmul_rn(x1, c));
  }
}

__global__ void embed_q8_0_kernel(const int8_t* __restrict__ qs, const uint16_t* __restrict__ d,
                                  const int32_t* __restrict__ tokens, int vocab, int dim, float* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  int tok = tokens[blockIdx.x];
  if (tok < 0 || tok >= vocab) tok = 0;  // unknown ids map to 0 (LlmEngine.cs:321)
  const int8_t* row = qs + (size_t)tok * dim;
  const uint16_t* dr = d + (size_t)tok * (dim / QK);
  float* o = out + (size_t)blockIdx.x * dim;
  for (int i = threadIdx.x; i < dim; i += blockDim.x) o[i] = (float)row[i] * h2f(dr[i / QK]);
}


// TensorOps.ApplyRoPEInPlace, interleaved branch (ZeroTensor/src/ZeroTensor.Core/TensorOps.Neural.cs:1246-1366):
// x [heads][seq][hd]; invFreq = 1 / (float)pow(theta, 2i/hd) in float, angle = pos * invFreq in float,
// cos/sin evaluated in double and rounded to float.
__global__ void rope_tensorops_kernel(float* __restrict__ x, int heads, int seq, int hd, int pos0, float theta) {
  const int half = hd / 2;
  const size_t total = (size_t)heads * seq * half;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(i % half);
    const size_t hs = i / half;
    const int s = (int)(hs % seq);
    const float inv_freq = 1.0f / (float)pow((double)theta, (2.0 * p) / hd);
    const float angle = __fmul_rn((float)(pos0 + s), inv_freq);
    const float c = (float)cos((double)angle), sn = (float)sin((double)angle);
    float* v = x + hs * hd + 2 * p;
    const float x1 = v[0], x2 = v[1];
    v[0] = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, sn));
    v[1] = __fadd_rn(__fmul_rn(x2, c), __fmul_rn(x1, sn));
  }
}

// fp32 GEMM for the zc_gemm_f32 bridge entry (TensorBlas.cs:138): C = alpha*A*B + beta*C, all row-major
// and contiguous (the host entry packs strided operands).  Plain 32x32-tiled SIMT kernel: this entry is
// not on the quantized hot path.
__global__ void sgemm_kernel(int m, int n, int k, float alpha, const float* __restrict__ A,
                             const float* __restrict__ B, float beta, float* __restrict__ C) {
  __shared__ float As[32][33];
  __shared__ float Bs[32][33];
  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;  // 32 x 8 threads, 4 rows each
  const int row0 = blockIdx.y * 32, col = blockIdx.x * 32 + tx;
  float acc[4] = {0.f, 0.f, 0.f, 0.f};
  for (int k0 = 0; k0 < k; k0 += 32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int r = ty + 8 * j;
      As[r][tx] = (row0 + r < m && k0 + tx < k) ? A[(size_t)(row0 + r) * k + k0 + tx] : 0.f;
      Bs[r][tx] = (k0 + r < k && col < n) ? B[(size_t)(k0 + r) * n + col] : 0.f;
    }
    __syncthreads();
#pragma unroll 8
    for (int kk = 0; kk < 32; ++kk) {
      const float b = Bs[kk][tx];
#pragma unroll
      for (int j = 0; j < 4; ++j) acc[j] = fmaf(As[ty + 8 * j][kk], b, acc[j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int r = row0 + ty + 8 * j;
    if (r < m && col < n) {
      float* cp = C + (size_t)r * n + col;
      *cp = beta == 0.f ? alpha * acc[j] : alpha * acc[j] + beta * *cp;
    }
  }
}

__global__ void dot_i8_kernel(const int8_t* __restrict__ a, const int8_t* __restrict__ b, size_t n,
                              int32_t* __restrict__ out) {
  __shared__ int red[32];
  int s = 0;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
    s += (int)a[i] * (int)b[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    atomicAdd(out, t);  // integer addition: the result is exact and order independent
  }
}

inline int grid_for(size_t n, int threads) {
  size_t g = (n + threads - 1) / threads;
  if (g > 148 * 16) g = 148 * 16;
  return g < 1 ? 1 : (int)g;
}

inline int launched() { return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError; }

}  // namespace

namespace {

// dst[0, bytes) = src[0, bytes): 16-byte words, then the 4-byte tail.  Either side may be pinned host memory
// mapped into the device's address space (the host-pointer entries' zero-copy activations and results).
__global__ void copy_words_kernel(const int4* __restrict__ src, int4* __restrict__ dst, size_t n16,
                                  const uint32_t* __restrict__ tsrc, uint32_t* __restrict__ tdst, int ntail) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x)
    dst[i] = src[i];
  if (blockIdx.x == 0 && (int)threadIdx.x < ntail) tdst[threadIdx.x] = tsrc[threadIdx.x];
}

}  // namespace

int copy_words(const void* src, void* dst, size_t bytes, cudaStream_t s) {
  if (!src || !dst || bytes % 4 || (reinterpret_cast<uintptr_t>(src) & 15) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return kBadArgument;
  if (bytes == 0) return kOk;
  const size_t n16 = bytes / 16;
  const int ntail = (int)(bytes % 16) / 4;
  const unsigned grid = (unsigned)std::max<size_t>(1, std::min<size_t>((n16 + 127) / 128, 148));
  return launch_pdl(copy_words_kernel, dim3(grid), dim3(128), 0, s, static_cast<const int4*>(src),
                    static_cast<int4*>(dst), n16, static_cast<const uint32_t*>(src) + n16 * 4,
                    static_cast<uint32_t*>(dst) + n16 * 4, ntail) == cudaSuccess
             ? kOk
             : kCudaError;
}

int rmsnorm(const float* x, const float* w, float* out, int rows, int n, float eps, cudaStream_t s) {
  if (!x || !w || !out || rows < 0 || n <= 0) return kBadArgument;
  if (rows == 0) return kOk;
  int threads = n >= 1024 ? 512 : (n >= 256 ? 256 : 128);
  return launch_pdl(rmsnorm_kernel<float>, dim3(rows), dim3(threads), 0, s, x, w, out, n, eps) == cudaSuccess
             ? kOk
             : kCudaError;
}

int rmsnorm_h(const float* x, const float* w, __half* out, int rows, int n, float eps, cudaStream_t s) {
  if (!x || !w || !out || rows < 0 || n <= 0) return kBadArgument;
  if (rows == 0) return kOk;
  int threads = n >= 1024 ? 512 : (n >= 256 ? 256 : 128);
  return launch_pdl(rmsnorm_kernel<__half>, dim3(rows), dim3(threads), 0, s, x, w, out, n, eps) == cudaSuccess
             ? kOk
             : kCudaError;
}

int swiglu(const float* gate, const float* up, float* out, size_t n, cudaStream_t s) {
  if (!gate || !up || !out) return kBadArgument;
  if (n == 0) return kOk;
  swiglu_kernel<<<grid_for(n, 256), 256, 0, s>>>(gate, up, out, n);
  return launched();
}

int silu(const float* x, float* out, size_t n, cudaStream_t s) {
  if (!x || !out) return kBadArgument;
  if (n == 0) return kOk;
  silu_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, out, n);
  return launched();
}

int rope(float* x, int rows, int heads, int hd, const int32_t* pos, int pos0, const float* cos_t, const float* sin_t,
         int max_pos, cudaStream_t s) {
  if (!x || !cos_t || !sin_t || rows < 0 || heads <= 0 || hd <= 0 || (hd & 1) || max_pos <= 0) return kBadArgument;
  if (rows == 0) return kOk;
  size_t n = (size_t)rows * heads * (hd / 2);
  rope_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, rows, heads, hd, pos, pos0, cos_t, sin_t, max_pos);
  return launched();
}

int embed_q8_0(const int8_t* qs, const uint16_t* d, const int32_t* tokens, int n_tokens, int vocab, int dim,
               float* out, cudaStream_t s) {
  if (!qs || !d || !tokens || !out || n_tokens < 0 || vocab <= 0 || dim <= 0 || dim % QK) return kBadArgument;
  if (n_tokens == 0) return kOk;
  return launch_pdl(embed_q8_0_kernel, dim3(n_tokens), dim3(256), 0, s, qs, d, tokens, vocab, dim, out) == cudaSuccess
             ? kOk
             : kCudaError;
}

int rope_tensorops(float* x, int heads, int seq, int hd, int pos0, float theta, cudaStream_t s) {
  if (!x || heads < 0 || seq < 0 || hd <= 0 || (hd & 1)) return kBadArgument;
  size_t n = (size_t)heads * seq * (hd / 2);
  if (n == 0) return kOk;
  rope_tensorops_kernel<<<grid_for(n, 256), 256, 0, s>>>(x, heads, seq, hd, pos0, theta);
  return launched();
}

int sgemm(int m, int n, int k, float alpha, const float* a, const float* b, float beta, float* c, cudaStream_t s) {
  if (!a || !b || !c || m < 0 || n < 0 || k < 0) return kBadArgument;
  if (m == 0 || n == 0) return kOk;
  dim3 grid((n + 31) / 32, (m + 31) / 32);
  sgemm_kernel<<<grid, 256, 0, s>>>(m, n, k, alpha, a, b, beta, c);
  return launched();
}

int dot_i8(const int8_t* a, const int8_t* b, size_t n, int32_t* out, cudaStream_t s) {
  if (!out || (n > 0 && (!a || !b))) return kBadArgument;
  if (cudaMemsetAsync(out, 0, sizeof(int32_t), s) != cudaSuccess) return kCudaError;
  if (n == 0) return kOk;
  dot_i8_kernel<<<grid_for(n, 256), 256, 0, s>>>(a, b, n, out);
  return launched();
}

}  // namespace zc
