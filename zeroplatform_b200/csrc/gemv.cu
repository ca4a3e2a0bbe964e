// gemv.cu -- block-quantized decode GEMV (y = W x, y += W x) for Q8_0 and Q4_0 weights.
//
// Restates QuantizedKernels.MatVecMulQ8_0 / MatVecAddQ8_0 / ...Q4_0
// (ZeroLlm/src/ZeroLlm.Core/Quantization/QuantizedKernels.cs:190-349) and the ZeroTensor
// streaming twin GgufDequantizer.GemvQ8_0 / GemvQ4_0 (ZeroTensor/src/ZeroTensor.Core/
// Serialization/GgufFormat.cs:333-516): y[n] = sum_b d[n,b] * sum_i x[32b+i] * q[n,b,i].
//
// Device layout ("SoA", produced once per weight by the repack kernels below):
//   Q8_0: qs int8 [N][K]            d fp16 [N][K/32]
//   Q4_0: qs u8   [N][K/32][16]     d fp16 [N][K/32]   (byte j = elem j | elem j+16 << 4, as in BlockQ4_0)
// so every row of quantized values is 16-byte aligned and streams with 128-bit loads; the reference's
// 34/18-byte array-of-structs blocks are not 16-byte aligned.
//
// Kernel shape: one warp owns R rows; each lane streams 16-byte chunks of those rows with
// L1-bypassing 128-bit loads (all of a row's chunks in flight at once), the activation vector is
// staged once per CTA in shared memory (XOR-swizzled so that the 128-bit shared loads of a warp are
// bank-conflict free), int8/nibble -> fp32 conversion is exact (PRMT + FADD), per-chunk sums are
// scaled by the block scale, and a warp-shuffle reduction finishes each row.
// The HBM roofline: bytes = N*K (Q8) or N*K/2 (Q4) + N*K/32*2 (scales) + 4K + 4N.

#include "common.cuh"
#include "kernels.h"

namespace zc {

// ------------------------------------------------------------------------------------------
// AoS -> SoA repack (one thread per 32-element block; blocks are 2-byte aligned in AoS).
// ------------------------------------------------------------------------------------------
__global__ void repack_q8_0_kernel(const uint8_t* __restrict__ aos, int8_t* __restrict__ qs,
                                   uint16_t* __restrict__ d, size_t nblocks) {
  size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(aos + b * Q8_BLOCK_BYTES);
  d[b] = src[0];
  uint32_t w[8];
#pragma unroll
  for (int i = 0; i < 8; ++i) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
  int4* dst = reinterpret_cast<int4*>(qs + b * QK);
  dst[0] = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
  dst[1] = make_int4((int)w[4], (int)w[5], (int)w[6], (int)w[7]);
}

__global__ void repack_q4_0_kernel(const uint8_t* __restrict__ aos, uint8_t* __restrict__ qs,
                                   uint16_t* __restrict__ d, size_t nblocks) {
  size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const uint16_t* src = reinterpret_cast<const uint16_t*>(aos + b * Q4_BLOCK_BYTES);
  d[b] = src[0];
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = (uint32_t)src[1 + 2 * i] | ((uint32_t)src[2 + 2 * i] << 16);
  *reinterpret_cast<int4*>(qs + b * 16) = make_int4((int)w[0], (int)w[1], (int)w[2], (int)w[3]);
}

// ------------------------------------------------------------------------------------------
// Activation staging policies (applied once per CTA while the weight loads are in flight).
// ------------------------------------------------------------------------------------------
struct XPlain {  // x as given
  const float* x;
  __device__ __forceinline__ void prepare(float*) const {}
  __device__ __forceinline__ float get(int i, const float*) const { return x[i]; }
};

// x = RmsNorm(x_raw) * w, fused: RmsNorm.Forward (Layers/RmsNorm.cs:14-59) computed per CTA -- mean of
// squares in fp32, 1 / (float)sqrt((double)(ms + eps)), then (x * inv) * w as the reference orders it.
struct XRmsNorm {
  const float* x;
  const float* w;
  float eps;
  int n;
  __device__ __forceinline__ void prepare(float* red) const {
    float ss = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) ss = fmaf(x[i], x[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x == 0) {
      float t = 0.f;
      for (int i = 0; i < (int)(blockDim.x >> 5); ++i) t += red[i];
      red[blockDim.x >> 5] = 1.0f / (float)sqrt((double)(t / (float)n + eps));
    }
    __syncthreads();
  }
  __device__ __forceinline__ float get(int i, const float* red) const {
    return __fmul_rn(__fmul_rn(x[i], red[blockDim.x >> 5]), w[i]);
  }
};

// x = SwiGLU(gate, up) with gate = gu[0:ffn], up = gu[ffn:2ffn] (SwiGLU.Forward, Layers/SwiGLU.cs:13-51).
struct XSwiGLU {
  const float* gu;
  int ffn;
  __device__ __forceinline__ void prepare(float*) const {}
  __device__ __forceinline__ float get(int i, const float*) const {
    const float g = gu[i];
    const float sg = 1.0f / (1.0f + expf(-g));
    return __fmul_rn(__fmul_rn(g, sg), gu[ffn + i]);
  }
};

// Chunk geometry: Q8 chunks hold 16 values (4 float4), Q4 chunks hold 32 values (8 float4).
template <int F4_PER_CHUNK>
__device__ __forceinline__ int swz(int chunk, int j) {
  // Logical float4 j of chunk `chunk` -> physical float4 slot (conflict-free for 8-lane phases).
  if (F4_PER_CHUNK == 4) return chunk * 4 + (j ^ ((chunk >> 1) & 3));
  return chunk * 8 + (j ^ (chunk & 7));
}

template <int F4_PER_CHUNK, class XP>
__device__ __forceinline__ void stage_x(float4* sx, const XP& xp, int k0, int len, float* red) {
  xp.prepare(red);
  const int nf4 = len / 4;
  for (int f = threadIdx.x; f < nf4; f += blockDim.x) {
    int chunk = f / F4_PER_CHUNK, j = f % F4_PER_CHUNK;
    int e = k0 + 4 * f;
    sx[swz<F4_PER_CHUNK>(chunk, j)] = make_float4(xp.get(e, red), xp.get(e + 1, red), xp.get(e + 2, red),
                                                  xp.get(e + 3, red));
  }
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
constexpr int SEG_Q8 = 8192;   // activations staged per K segment (32 KB of shared memory)
constexpr int SEG_Q4 = 8192;
constexpr int UNROLL = 8;      // chunks in flight per lane per row (Q4_0)

// Loads one batch of UNROLL chunks per row (and the block scales they need) for lane `lane`.
template <int R, int U, int CHUNK_BYTES, int CHUNKS_PER_BLOCK>
__device__ __forceinline__ void load_batch(int4 (&w)[R][U], float (&sc)[R][U], const uint8_t* __restrict__ qs,
                                           const uint16_t* __restrict__ dsc, size_t row_bytes, int kb,
                                           int row0, int N, int seg_chunk0, int seg_blk0, int cb, int nch,
                                           int lane) {
#pragma unroll
  for (int r = 0; r < R; ++r)
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int c = cb + lane + 32 * u;
      const int row = row0 + r;
      const bool ok = c < nch && row < N;
      w[r][u] = ok ? ld_stream_v4(qs + (size_t)row * row_bytes + (size_t)(seg_chunk0 + c) * CHUNK_BYTES)
                   : make_int4(0, 0, 0, 0);
      sc[r][u] = ok ? h2f(__ldg(dsc + (size_t)row * kb + seg_blk0 + c / CHUNKS_PER_BLOCK)) : 0.f;
    }
}

template <int R, int U, class XP>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_q8_0_kernel(const int8_t* __restrict__ qs,
                                                                 const uint16_t* __restrict__ dsc, XP xp,
                                                                 float* __restrict__ y, int N, int K,
                                                                 int accumulate) {
  extern __shared__ float4 sx[];
  __shared__ float red[GEMV_WARPS + 1];
  static_assert(GEMV_THREADS / 32 == GEMV_WARPS, "red[] holds one partial per warp plus the result");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * GEMV_WARPS + warp) * R;
  const int kb = K / QK;
  const uint8_t* q = reinterpret_cast<const uint8_t*>(qs);
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  int4 w[R][U];
  float sc[R][U];

  for (int k0 = 0; k0 < K; k0 += SEG_Q8) {
    const int len = min(SEG_Q8, K - k0);
    const int nch = len / 16;  // 16-value chunks (half a block)
    // The first batch of weight loads is issued before x is staged so both are in flight together; the
    // weights do not depend on the previous kernel, so they are issued before the dependency wait.
    if (k0 == 0) pdl_trigger();
    load_batch<R, U, 16, 2>(w, sc, q, dsc, (size_t)K, kb, row0, N, k0 / 16, k0 / QK, 0, nch, lane);
    if (k0 == 0) pdl_wait();
    if (k0 > 0) __syncthreads();
    stage_x<4>(sx, xp, k0, len, red);
    __syncthreads();
    for (int cb = 0; cb < nch; cb += 32 * U) {
      if (cb > 0) load_batch<R, U, 16, 2>(w, sc, q, dsc, (size_t)K, kb, row0, N, k0 / 16, k0 / QK, cb, nch, lane);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cb + lane + 32 * u;
        if (c >= nch) break;
        float4 xv[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xv[j] = sx[swz<4>(c, j)];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t* wv = reinterpret_cast<const uint32_t*>(&w[r][u]);
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float f0, f1, f2, f3;
            s8x4_to_f32(wv[j], f0, f1, f2, f3);
            s = fmaf(f0, xv[j].x, s);
            s = fmaf(f1, xv[j].y, s);
            s = fmaf(f2, xv[j].z, s);
            s = fmaf(f3, xv[j].w, s);
          }
          acc[r] = fmaf(sc[r][u], s, acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float v = warp_sum(acc[r]);
    if (lane == 0 && row0 + r < N) y[row0 + r] = accumulate ? y[row0 + r] + v : v;
  }
}

template <int R, class XP>
__global__ void __launch_bounds__(GEMV_THREADS) gemv_q4_0_kernel(const uint8_t* __restrict__ qs,
                                                                 const uint16_t* __restrict__ dsc, XP xp,
                                                                 float* __restrict__ y, int N, int K,
                                                                 int accumulate) {
  extern __shared__ float4 sx[];
  __shared__ float red[GEMV_WARPS + 1];
  constexpr int U = UNROLL / 2;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * GEMV_WARPS + warp) * R;
  const int kb = K / QK;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  int4 w[R][U];
  float sc[R][U];

  for (int k0 = 0; k0 < K; k0 += SEG_Q4) {
    const int len = min(SEG_Q4, K - k0);
    const int nch = len / QK;  // one chunk = one 32-value block = 16 bytes
    if (k0 == 0) pdl_trigger();
    load_batch<R, U, 16, 1>(w, sc, qs, dsc, (size_t)K / 2, kb, row0, N, k0 / QK, k0 / QK, 0, nch, lane);
    if (k0 == 0) pdl_wait();
    if (k0 > 0) __syncthreads();
    stage_x<8>(sx, xp, k0, len, red);
    __syncthreads();
    for (int cb = 0; cb < nch; cb += 32 * U) {
      if (cb > 0) load_batch<R, U, 16, 1>(w, sc, qs, dsc, (size_t)K / 2, kb, row0, N, k0 / QK, k0 / QK, cb, nch, lane);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cb + lane + 32 * u;
        if (c >= nch) break;
        float4 xv[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) xv[j] = sx[swz<8>(c, j)];
#pragma unroll
        for (int r = 0; r < R; ++r) {
          const uint32_t* wv = reinterpret_cast<const uint32_t*>(&w[r][u]);
          float s = 0.f;
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float f0, f1, f2, f3;
            u4x4_to_f32(wv[j] & 0x0F0F0F0Fu, f0, f1, f2, f3);  // elements 4j..4j+3
            s = fmaf(f0, xv[j].x, s);
            s = fmaf(f1, xv[j].y, s);
            s = fmaf(f2, xv[j].z, s);
            s = fmaf(f3, xv[j].w, s);
            u4x4_to_f32((wv[j] >> 4) & 0x0F0F0F0Fu, f0, f1, f2, f3);  // elements 16+4j..16+4j+3
            s = fmaf(f0, xv[4 + j].x, s);
            s = fmaf(f1, xv[4 + j].y, s);
            s = fmaf(f2, xv[4 + j].z, s);
            s = fmaf(f3, xv[4 + j].w, s);
          }
          acc[r] = fmaf(sc[r][u], s, acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    float v = warp_sum(acc[r]);
    if (lane == 0 && row0 + r < N) y[row0 + r] = accumulate ? y[row0 + r] + v : v;
  }
}

// ------------------------------------------------------------------------------------------
// Launchers
// ------------------------------------------------------------------------------------------
int repack_q8_0(const uint8_t* aos, int8_t* qs, uint16_t* d, size_t n, size_t k, cudaStream_t s) {
  if (!aos || !qs || !d || k % QK) return kBadArgument;
  size_t nb = n * (k / QK);
  if (nb == 0) return kOk;
  repack_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(aos, qs, d, nb);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

int repack_q4_0(const uint8_t* aos, uint8_t* qs, uint16_t* d, size_t n, size_t k, cudaStream_t s) {
  if (!aos || !qs || !d || k % QK) return kBadArgument;
  size_t nb = n * (k / QK);
  if (nb == 0) return kOk;
  repack_q4_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(aos, qs, d, nb);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

template <class Kern>
static int set_smem(Kern k, int bytes) {
  if (bytes > 48 * 1024) {
    if (cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes) != cudaSuccess)
      return kCudaError;
  }
  return kOk;
}

constexpr int Q4_R = 4;

// Rows per warp (R) and 16-byte chunks per lane per row (U) for a row of K int8 values: R * U stays at 16
// loads in flight per lane, so short rows (K = 768: 48 chunks) still keep ~8 KB per warp in flight.
template <class XP>
static int launch_q8(const int8_t* qs, const uint16_t* d, const XP& xp, float* y, int n, int k, int accumulate,
                     cudaStream_t s) {
  if (!qs || !d || !y || n < 0 || k <= 0 || k % QK) return kBadArgument;
  if (n == 0) return kOk;
  const int smem = min(k, SEG_Q8) * 4;
  const int chunks = min(k, SEG_Q8) / 16;
  auto go = [&](auto kern, int r) -> int {
    if (set_smem(kern, smem) != kOk) return kCudaError;
    const int rows_per_cta = GEMV_WARPS * r;
    const int grid = (n + rows_per_cta - 1) / rows_per_cta;
    return launch_pdl(kern, dim3(grid), dim3(GEMV_THREADS), smem, s, qs, d, xp, y, n, k, accumulate) == cudaSuccess
               ? kOk
               : kCudaError;
  };
  if (chunks > 64) return go(gemv_q8_0_kernel<2, 8, XP>, 2);  // K >= 1056
  if (chunks > 32) return go(gemv_q8_0_kernel<8, 2, XP>, 8);  // K in (512, 1024]
  return go(gemv_q8_0_kernel<16, 1, XP>, 16);                 // K <= 512
}

int gemv_q8_0(const int8_t* qs, const uint16_t* d, const float* x, float* y, int n, int k, int accumulate,
              cudaStream_t s) {
  if (!x) return kBadArgument;
  return launch_q8(qs, d, XPlain{x}, y, n, k, accumulate, s);
}

int gemv_q8_0_rmsnorm(const int8_t* qs, const uint16_t* d, const float* x, const float* norm_w, float eps, float* y,
                      int n, int k, int accumulate, cudaStream_t s) {
  if (!x || !norm_w) return kBadArgument;
  return launch_q8(qs, d, XRmsNorm{x, norm_w, eps, k}, y, n, k, accumulate, s);
}

int gemv_q8_0_swiglu(const int8_t* qs, const uint16_t* d, const float* gate_up, float* y, int n, int k,
                     int accumulate, cudaStream_t s) {
  if (!gate_up) return kBadArgument;
  return launch_q8(qs, d, XSwiGLU{gate_up, k}, y, n, k, accumulate, s);
}

int gemv_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, int n, int k, int accumulate,
              cudaStream_t s) {
  if (!qs || !d || !x || !y || n < 0 || k <= 0 || k % QK) return kBadArgument;
  if (n == 0) return kOk;
  const int rows_per_cta = GEMV_WARPS * Q4_R;
  const int grid = (n + rows_per_cta - 1) / rows_per_cta;
  const int smem = min(k, SEG_Q4) * 4;
  auto kern = gemv_q4_0_kernel<Q4_R, XPlain>;
  if (set_smem(kern, smem) != kOk) return kCudaError;
  return launch_pdl(kern, dim3(grid), dim3(GEMV_THREADS), smem, s, qs, d, XPlain{x}, y, n, k, accumulate) == cudaSuccess
             ? kOk
             : kCudaError;
}

}  // namespace zc
