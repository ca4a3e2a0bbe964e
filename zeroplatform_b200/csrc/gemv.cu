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
// Forms: the slab form (Q8_0, K = 4096: activations in registers, 7 rows a CTA split between registers and
// bulk copies), the direct form below for the other decode shapes, and the streaming form (int16 activations,
// DP2A, L2 prefetch) for >= 64 MB of weights.  Direct form: one warp owns R rows; each lane keeps 8
// L1-bypassing 128-bit weight loads in flight (U chunks of each of the R rows), the activation vector is
// staged once per CTA in shared memory
// (XOR-swizzled so that the 128-bit shared loads of a warp are bank-conflict free), int8/nibble -> fp32
// conversion is exact (PRMT + packed FADD), products accumulate in packed fp32x2 FMAs, per-chunk sums are
// scaled by the block scale, and a warp-shuffle reduction finishes each row.  At most 64 registers a
// thread: four CTAs share an SM, so consecutive GEMVs overlap under programmatic dependent launch.
// The HBM roofline: bytes = N*K (Q8) or N*K/2 (Q4) + N*K/32*2 (scales) + 4K + 4N.

#include <algorithm>

#include "common.cuh"
#include "kernels.h"
#include "sync.cuh"

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
  // values i .. i+3 (i a multiple of 4); one 128-bit load when x is 16-byte aligned
  __device__ __forceinline__ float4 get4(int i, const float*) const {
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) return __ldg(reinterpret_cast<const float4*>(x + i));
    return make_float4(x[i], x[i + 1], x[i + 2], x[i + 3]);
  }
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
  __device__ __forceinline__ float4 get4(int i, const float* red) const {
    return make_float4(get(i, red), get(i + 1, red), get(i + 2, red), get(i + 3, red));
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
  __device__ __forceinline__ float4 get4(int i, const float* red) const {
    return make_float4(get(i, red), get(i + 1, red), get(i + 2, red), get(i + 3, red));
  }
};

// ------------------------------------------------------------------------------------------
// Activations as int16 per 32-value block.
//
// Each CTA stages its K-segment of x once: block b gets the scale s_b = max|x| / 32767 and the values
// q = rint(x / s_b) in [-32767, 32767] (|x - s_b q| <= s_b / 2: a relative error of at most 2^-16 of the
// block's largest value).  A block's 32 int8 (or nibble) weights then meet their activations in DP2A
// instructions -- two int16 x int8 products summed into an int32 each -- so a 16-value chunk costs 8 integer
// dot-product instructions instead of 16 conversions and 16 FMAs, and the int32 block sums are exact.  One
// int -> float conversion and the two scales finish a chunk:  y += d_w * s_b * sum_i q_i w_i.
//
// Shared layout: the int16 values in 16-byte units, chunk by chunk (a Q8_0 chunk = 16 values = 2 units, a
// Q4_0 chunk = one 32-value block = 4 units), with the units of chunk c XOR-swizzled so that the 8 lanes of
// a 128-bit load phase (chunks c .. c+7) hit distinct banks; then the block scales (fp32) and, for Q4_0, the
// block sums of q (int32, for the -8 nibble offset).
// ------------------------------------------------------------------------------------------
template <int UPC>  // 16-byte units per chunk: 2 (Q8_0) or 4 (Q4_0)
__device__ __forceinline__ int xunit(int chunk, int u) {
  if (UPC == 2) return chunk * 2 + (u ^ ((chunk >> 2) & 1));
  return chunk * 4 + (u ^ ((chunk >> 1) & 3));
}

// Stages x[k0, k0 + len) as int16 blocks in two steps: (A) global -> shared fp32 with 128-bit loads, one
// pass; (B) shared fp32 -> shared int16, one thread per half block (16 values).  The two halves of a block are
// adjacent lanes and agree on the block maximum with one shuffle.  Rounding uses the magic number
// 1.5 * 2^23: v * inv + 1.5 * 2^23 (one packed FMA for two values, a single round-to-nearest-even) leaves
// rint(v * inv) in the low bits of the float's encoding, and one PRMT packs two of those 16-bit integers.
template <int UPC, class XP>
__device__ __forceinline__ void stage_xq(float4* xf, int4* xq, float* xs, int* xsum, const XP& xp, int k0, int len,
                                         float* red) {
  xp.prepare(red);
  for (int f = threadIdx.x; f < len / 4; f += blockDim.x) xf[f] = xp.get4(k0 + 4 * f, red);
  __syncthreads();
  const float magic = 12582912.0f;  // 1.5 * 2^23
  const int halves = len / 16;
  for (int h = threadIdx.x; h < halves; h += blockDim.x) {  // halves is even: partners iterate together
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {  // pass 1 over shared memory: the block maximum
      const float4 v = xf[4 * h + i];
      amax = fmaxf(amax, fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w))));
    }
    amax = fmaxf(amax, __shfl_xor_sync(__activemask(), amax, 1));
    const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
    const float2 inv2 = make_float2(inv, inv), mg2 = make_float2(magic, magic);
    const int c = UPC == 2 ? h : h >> 1;  // chunk and first unit of this half block
    const int u0 = UPC == 2 ? 0 : 2 * (h & 1);
    float part = 0.f;  // sum of the 16 integers, exact in fp32
#pragma unroll
    for (int half = 0; half < 2; ++half) {  // pass 2: 8 values -> one 16-byte unit of int16
      int wv[4];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const float4 v = xf[4 * h + 2 * half + i];
        const float2 a = __ffma2_rn(make_float2(v.x, v.y), inv2, mg2);
        const float2 b = __ffma2_rn(make_float2(v.z, v.w), inv2, mg2);
        wv[2 * i] = (int)__byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x5410);
        wv[2 * i + 1] = (int)__byte_perm(__float_as_uint(b.x), __float_as_uint(b.y), 0x5410);
        if (xsum) part += ((a.x - magic) + (a.y - magic)) + ((b.x - magic) + (b.y - magic));
      }
      xq[xunit<UPC>(c, u0 + half)] = make_int4(wv[0], wv[1], wv[2], wv[3]);
    }
    if (xsum) part += __shfl_xor_sync(__activemask(), part, 1);
    if ((h & 1) == 0) {
      xs[h >> 1] = amax * (1.0f / 32767.0f);
      if (xsum) xsum[h >> 1] = (int)part;
    }
  }
}

__device__ __forceinline__ int dp2a_lo(int x2, int w4, int c) { return __dp2a_lo(x2, w4, c); }
__device__ __forceinline__ int dp2a_hi(int x2, int w4, int c) { return __dp2a_hi(x2, w4, c); }

// sum over the 16 values of a Q8_0 chunk: w = 16 int8, x0 / x1 = the chunk's 16 int16 (logical units 0, 1).
__device__ __forceinline__ int dot16_q8(const int4& w, const int4& x0, const int4& x1) {
  int s = dp2a_lo(x0.x, w.x, 0);
  s = dp2a_hi(x0.y, w.x, s);
  s = dp2a_lo(x0.z, w.y, s);
  s = dp2a_hi(x0.w, w.y, s);
  s = dp2a_lo(x1.x, w.z, s);
  s = dp2a_hi(x1.y, w.z, s);
  s = dp2a_lo(x1.z, w.w, s);
  return dp2a_hi(x1.w, w.w, s);
}

// sum over the 32 nibbles u of a Q4_0 block (byte j = value j | value j+16 << 4) with x0..x3 = values 0..31.
__device__ __forceinline__ int dot32_q4(const int4& w, const int4& x0, const int4& x1, const int4& x2,
                                        const int4& x3) {
  const int m = 0x0F0F0F0F;
  const int l0 = w.x & m, l1 = w.y & m, l2 = w.z & m, l3 = w.w & m;                      // values 0..15
  const int h0 = (w.x >> 4) & m, h1 = (w.y >> 4) & m, h2 = (w.z >> 4) & m, h3 = (w.w >> 4) & m;  // 16..31
  int s = dp2a_lo(x0.x, l0, 0);
  s = dp2a_hi(x0.y, l0, s);
  s = dp2a_lo(x0.z, l1, s);
  s = dp2a_hi(x0.w, l1, s);
  s = dp2a_lo(x1.x, l2, s);
  s = dp2a_hi(x1.y, l2, s);
  s = dp2a_lo(x1.z, l3, s);
  s = dp2a_hi(x1.w, l3, s);
  s = dp2a_lo(x2.x, h0, s);
  s = dp2a_hi(x2.y, h0, s);
  s = dp2a_lo(x2.z, h1, s);
  s = dp2a_hi(x2.w, h1, s);
  s = dp2a_lo(x3.x, h2, s);
  s = dp2a_hi(x3.y, h2, s);
  s = dp2a_lo(x3.z, h3, s);
  return dp2a_hi(x3.w, h3, s);
}

// fp32 activations (the decode-chain form): staged in a swizzled float4 layout, products accumulate in packed
// fp32x2 FMAs after an exact int8 / nibble -> fp32 conversion (PRMT + packed FADD).
template <int F4_PER_CHUNK>
__device__ __forceinline__ int swz(int chunk, int j) {
  // logical float4 j of chunk `chunk` -> physical float4 slot (conflict-free for 8-lane phases)
  if (F4_PER_CHUNK == 4) return chunk * 4 + (j ^ ((chunk >> 1) & 3));
  return chunk * 8 + (j ^ (chunk & 7));
}

__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }

__device__ __forceinline__ void bytes_to_f2(uint32_t b, float2 bias, float2& p01, float2& p23) {
  p01 = __fadd2_rn(f2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7650)),
                      __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7651))), bias);
  p23 = __fadd2_rn(f2(__uint_as_float(__byte_perm(b, 0x4B000000u, 0x7652)),
                      __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7653))), bias);
}

// sum over a Q8_0 chunk (16 values) with x in fp32: chunk c of the swizzled layout
__device__ __forceinline__ float dotf_q8(const int4& w, const float4* sx, int c) {
  const float2 bias = f2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
  const uint32_t* wv = reinterpret_cast<const uint32_t*>(&w);
  float2 s = f2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 xv = sx[swz<4>(c, j)];
    float2 p01, p23;
    bytes_to_f2(wv[j] ^ 0x80808080u, bias, p01, p23);
    s = __ffma2_rn(p01, f2(xv.x, xv.y), s);
    s = __ffma2_rn(p23, f2(xv.z, xv.w), s);
  }
  return s.x + s.y;
}

// sum over a Q4_0 block (32 values) with x in fp32
__device__ __forceinline__ float dotf_q4(const int4& w, const float4* sx, int c) {
  const float2 bias = f2(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
  const uint32_t* wv = reinterpret_cast<const uint32_t*>(&w);
  float2 s = f2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float4 xl = sx[swz<8>(c, j)], xh = sx[swz<8>(c, 4 + j)];
    float2 l01, l23, h01, h23;
    bytes_to_f2(wv[j] & 0x0F0F0F0Fu, bias, l01, l23);
    bytes_to_f2((wv[j] >> 4) & 0x0F0F0F0Fu, bias, h01, h23);
    s = __ffma2_rn(l01, f2(xl.x, xl.y), s);
    s = __ffma2_rn(l23, f2(xl.z, xl.w), s);
    s = __ffma2_rn(h01, f2(xh.x, xh.y), s);
    s = __ffma2_rn(h23, f2(xh.z, xh.w), s);
  }
  return s.x + s.y;
}

constexpr int GEMV_THREADS = 256;
constexpr int GEMV_WARPS = GEMV_THREADS / 32;
// Four CTAs of 256 threads per SM (at most 64 registers a thread): the CTAs of the next GEMV in the stream fit
// beside this one's and issue their weight loads -- before griddepcontrol.wait, weights never depend on the
// previous kernel -- while this one finishes.
constexpr int GEMV_MIN_CTAS = 4;
constexpr int GEMV_STREAM_CTAS_PER_SM = 4;          // grid of the streaming form (contiguous row ranges)
constexpr size_t GEMV_STREAM_BYTES = 64ull << 20;  // weights from which a GEMV uses the streaming form
constexpr int SEG = 8192;   // activations staged per K segment: 32 KB fp32 + 16 KB int16 + 2 KB scales / sums
// 16-byte weight chunks in flight per lane (R rows x U chunks): 8 for Q8_0 (16 values each), 4 for Q4_0
// (32 values each: twice the arithmetic per byte, and the registers the nibble unpacking needs)
__host__ __device__ constexpr int loads_per_lane(int qt) { return qt == 8 ? 8 : 4; }

__host__ __device__ constexpr int seg_smem_bytes(int len) { return len * 4 + len * 2 + (len / QK) * 8; }

// Loads one batch of U chunks per row (and the block scales they need) for lane `lane`.
template <int R, int U, int CHUNKS_PER_BLOCK>
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
      w[r][u] = ok ? ld_stream_v4(qs + (size_t)row * row_bytes + (size_t)(seg_chunk0 + c) * 16)
                   : make_int4(0, 0, 0, 0);
      sc[r][u] = ok ? h2f(__ldg(dsc + (size_t)row * kb + seg_blk0 + c / CHUNKS_PER_BLOCK)) : 0.f;
    }
}

// Bulk prefetch of the 16-byte units wholly inside [p, p + bytes) into L2 (a hint: nothing outside the range is
// touched, no completion is awaited).
__device__ __forceinline__ void prefetch_l2(const void* p, size_t bytes) {
  const uintptr_t a = (reinterpret_cast<uintptr_t>(p) + 15) & ~(uintptr_t)15;
  const uintptr_t e = (reinterpret_cast<uintptr_t>(p) + bytes) & ~(uintptr_t)15;
  for (uintptr_t o = a; o < e; o += 0x40000000u) {
    const uint32_t n = (uint32_t)((e - o) < 0x40000000u ? (e - o) : 0x40000000u);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(o), "r"(n) : "memory");
  }
}

// acc[r] += d_w * s_x * (chunk c of row r . x) for the int16 activation layout (the u-th loaded chunk).
template <int QT, int R, int U>
__device__ __forceinline__ void chunk_dot(float (&acc)[R], const int4 (&w)[R][U], const float (&sc)[R][U], int u,
                                          int c, const int4* xq, const float* xs, const int* xsum) {
  const int b = QT == 8 ? c >> 1 : c;
  const float s_x = xs[b];
  if (QT == 8) {
    const int4 x0 = xq[xunit<2>(c, 0)], x1 = xq[xunit<2>(c, 1)];
#pragma unroll
    for (int r = 0; r < R; ++r) acc[r] = fmaf(sc[r][u] * s_x, (float)dot16_q8(w[r][u], x0, x1), acc[r]);
  } else {
    const int4 x0 = xq[xunit<4>(c, 0)], x1 = xq[xunit<4>(c, 1)], x2 = xq[xunit<4>(c, 2)], x3 = xq[xunit<4>(c, 3)];
    const int off = 8 * xsum[b];  // the nibbles carry +8
#pragma unroll
    for (int r = 0; r < R; ++r)
      acc[r] = fmaf(sc[r][u] * s_x, (float)(dot32_q4(w[r][u], x0, x1, x2, x3) - off), acc[r]);
  }
}

template <int F4_PER_CHUNK, class XP>
__device__ __forceinline__ void stage_xf_scalar(float4* sx, const XP& xp, int k0, int len, float* red) {
  xp.prepare(red);
  for (int f = threadIdx.x; f < len / 4; f += blockDim.x) {
    const int e = k0 + 4 * f;
    sx[swz<F4_PER_CHUNK>(f / F4_PER_CHUNK, f % F4_PER_CHUNK)] =
        make_float4(xp.get(e, red), xp.get(e + 1, red), xp.get(e + 2, red), xp.get(e + 3, red));
  }
}

// Decode-chain form: one batch of R rows per warp (the grid covers every row), so a CTA issues all of its
// weight loads before griddepcontrol.wait; fp32 activations staged per K segment of SEG values.
template <int QT, int R, int U, class XP>
__global__ void __launch_bounds__(GEMV_THREADS, R == 1 ? GEMV_MIN_CTAS : GEMV_MIN_CTAS - 1)
    gemv_direct_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, XP xp,
                       float* __restrict__ y, int N, int K, int accumulate) {
  constexpr int VPC = QT == 8 ? 16 : 32;
  constexpr int CPB = QT == 8 ? 2 : 1;
  static_assert(R * U == loads_per_lane(QT), "R rows x U chunks = the loads in flight per lane");
  extern __shared__ float4 sxf[];
  __shared__ float red[GEMV_WARPS + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row0 = (blockIdx.x * GEMV_WARPS + warp) * R;
  const int kb = K / QK;
  const size_t row_bytes = QT == 8 ? (size_t)K : (size_t)K / 2;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  int4 w[R][U];
  float sc[R][U];
  for (int k0 = 0; k0 < K; k0 += SEG) {
    const int len = min(SEG, K - k0);
    const int nch = len / VPC;
    if (k0 == 0) pdl_trigger();
    load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, row0, N, k0 / VPC, k0 / QK, 0, nch, lane);
    if (k0 == 0) pdl_wait();  // x (and y when accumulating) may come from the previous kernel
    if (k0 > 0) __syncthreads();
    stage_xf_scalar<QT == 8 ? 4 : 8>(sxf, xp, k0, len, red);
    __syncthreads();
    for (int cb = 0; cb < nch; cb += 32 * U) {
      if (cb > 0) load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, row0, N, k0 / VPC, k0 / QK, cb, nch, lane);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cb + lane + 32 * u;
        if (c >= nch) break;
#pragma unroll
        for (int r = 0; r < R; ++r)
          acc[r] = fmaf(sc[r][u], QT == 8 ? dotf_q8(w[r][u], sxf, c) : dotf_q4(w[r][u], sxf, c), acc[r]);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0 && row0 + r < N) y[row0 + r] = accumulate ? y[row0 + r] + v : v;
  }
}

// Error word of the slab form's bounded waits (0 = healthy); read and cleared through gemv_wait_status().
__device__ int g_gemv_status;

// Sum over the 32 lanes of each of 8 values with 9 shuffles (a transposed butterfly: each level halves the
// values a lane carries).  Lane l ends with the sum of value (l >> 4 & 1) * 4 + (l >> 3 & 1) * 2 + (l >> 2 & 1).
__device__ __forceinline__ float transposed_sum8(const float (&p)[8], int lane) {
  const bool b4 = lane & 16, b3 = lane & 8, b2 = lane & 4;
  float q4[4], q2[2];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float send = b4 ? p[i] : p[i + 4], keep = b4 ? p[i + 4] : p[i];
    q4[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const float send = b3 ? q4[i] : q4[i + 2], keep = b3 ? q4[i + 2] : q4[i];
    q2[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
  }
  float q1 = (b2 ? q2[1] : q2[0]) + __shfl_xor_sync(0xffffffffu, b2 ? q2[0] : q2[1], 4);
  q1 += __shfl_xor_sync(0xffffffffu, q1, 2);
  return q1 + __shfl_xor_sync(0xffffffffu, q1, 1);
}

// This lane's 16 activations as int16, packed two to a register (element 2j in the low half), with the scale
// of their 32-value block: lanes 2i and 2i + 1 hold the two halves of one block and agree on its maximum with one
// shuffle.  q = rint(x * 32767 / max|x|), so |x - s q| <= s / 2 with s = max|x| / 32767 (2^-16 of the block's
// largest value).  Rounding uses the magic number 1.5 * 2^23: v * inv + 1.5 * 2^23 (one packed FMA for two values,
// a single round-to-nearest-even) leaves rint(v * inv) in the low 16 bits of the float's encoding, and one PRMT
// packs two of them.
struct XLane16 {
  int v[8];
  float s;
};

__device__ __forceinline__ void lane_quantize16(const float (&x)[16], XLane16& r) {
  float amax = 0.f;
#pragma unroll
  for (int j = 0; j < 16; ++j) amax = fmaxf(amax, fabsf(x[j]));
  amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
  const float inv = amax > 0.f ? 32767.0f / amax : 0.f;
  r.s = amax * (1.0f / 32767.0f);
  const float2 inv2 = f2(inv, inv), mg2 = f2(12582912.0f, 12582912.0f);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 a = __ffma2_rn(f2(x[2 * j], x[2 * j + 1]), inv2, mg2);
    r.v[j] = (int)__byte_perm(__float_as_uint(a.x), __float_as_uint(a.y), 0x5410);
  }
}

// 16 int8 weights . this lane's 16 int16 activations, exact in int32 (DP2A: two int16 x int8 products a step)
__device__ __forceinline__ int dot16_i16(const int4& w, const XLane16& x) {
  int s = dp2a_lo(x.v[0], w.x, 0);
  s = dp2a_hi(x.v[1], w.x, s);
  s = dp2a_lo(x.v[2], w.y, s);
  s = dp2a_hi(x.v[3], w.y, s);
  s = dp2a_lo(x.v[4], w.z, s);
  s = dp2a_hi(x.v[5], w.z, s);
  s = dp2a_lo(x.v[6], w.w, s);
  return dp2a_hi(x.v[7], w.w, s);
}

// Slab form of the decode-chain Q8_0 GEMV for K == 4096 (d_model of the 7B-class shapes).  Warp w owns the
// columns [512 w, 512 w + 512) of every row of its CTA, so each lane keeps its 16 activations in registers (x is
// never staged in shared memory), as int16 with a per-block scale (lane_quantize16).  A CTA owns SLAB_ROWS = 7
// rows: SLAB_REG = 4 stream into registers (one 16-byte load per lane and row) and SLAB_SMEM = 3 are bulk-copied
// into shared memory by one thread, all issued before griddepcontrol.wait.  Each row chunk is 8 DP2A
// instructions, one conversion and one multiply by d_w * s_x: about a third of the instructions of the fp32 form,
// and the work after the wait is what bounds back-to-back launches (the next launch's weight stream starts only
// as this one's CTAs retire).  Row sums leave each warp through the transposed butterfly and the 8 warps' slab
// sums are added in warp order in shared memory.  At most 64 registers: four CTAs per SM.
constexpr int SLAB_K = 4096, SLAB_REG = 4, SLAB_SMEM = 3, SLAB_ROWS = SLAB_REG + SLAB_SMEM;

template <class XP>
__global__ void __launch_bounds__(GEMV_THREADS, 4)
    gemv_slab_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, XP xp, float* __restrict__ y,
                     int N, int accumulate) {
  constexpr int K = SLAB_K, KB = K / QK;
  static_assert(GEMV_WARPS * 32 * 16 == K, "one 16-value chunk per lane covers a row");
  __shared__ __align__(128) uint8_t srow[SLAB_SMEM][K];
  __shared__ __align__(16) uint16_t ssc[SLAB_SMEM][KB];
  __shared__ __align__(8) uint64_t bar;
  __shared__ float red[GEMV_WARPS][8];
  __shared__ float xred[GEMV_WARPS + 1];
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int c = warp * 32 + lane;  // this lane's chunk: columns [16 c, 16 c + 16)
  const int r0 = blockIdx.x * SLAB_ROWS;
  const int nrows = min(SLAB_ROWS, N - r0);
  const int nreg = min(SLAB_REG, nrows), nsm = nrows - nreg;
  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(smem_u32(&bar), 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_trigger();
  if (threadIdx.x == 0) {
    mbar_arrive_tx(smem_u32(&bar), (uint32_t)nsm * (K + KB * 2));
    for (int j = 0; j < nsm; ++j) {
      const size_t row = (size_t)(r0 + nreg + j);
      bulk_g2s(smem_u32(srow[j]), qs + row * K, K, smem_u32(&bar));
      bulk_g2s(smem_u32(ssc[j]), dsc + row * KB, KB * 2, smem_u32(&bar));
    }
  }
  int4 w[SLAB_REG];
  float sc[SLAB_REG];
#pragma unroll
  for (int r = 0; r < SLAB_REG; ++r) {
    const bool ok = r < nreg;
    w[r] = ok ? ld_stream_v4(qs + (size_t)(r0 + r) * K + (size_t)c * 16) : make_int4(0, 0, 0, 0);
    sc[r] = ok ? h2f(__ldg(dsc + (size_t)(r0 + r) * KB + (c >> 1))) : 0.f;
  }
  pdl_wait();  // x (and y when accumulating) may come from the previous kernel
  xp.prepare(xred);
  XLane16 xq;
  {
    float xv[16];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 v = xp.get4(c * 16 + 4 * j, xred);
      xv[4 * j] = v.x;
      xv[4 * j + 1] = v.y;
      xv[4 * j + 2] = v.z;
      xv[4 * j + 3] = v.w;
    }
    lane_quantize16(xv, xq);
  }
  float p[8];
#pragma unroll
  for (int r = 0; r < SLAB_REG; ++r) p[r] = (sc[r] * xq.s) * (float)dot16_i16(w[r], xq);
  const bool ok = nsm == 0 || mbar_wait(smem_u32(&bar), 0, &abort_flag, &g_gemv_status, 31);
#pragma unroll
  for (int j = 0; j < SLAB_SMEM; ++j) {
    p[SLAB_REG + j] = 0.f;
    if (ok && j < nsm)
      p[SLAB_REG + j] =
          (h2f(ssc[j][c >> 1]) * xq.s) * (float)dot16_i16(*reinterpret_cast<const int4*>(&srow[j][c * 16]), xq);
  }
#pragma unroll
  for (int r = SLAB_ROWS; r < 8; ++r) p[r] = 0.f;
  const float v = transposed_sum8(p, lane);
  const int row = ((lane >> 4) & 1) * 4 + ((lane >> 3) & 1) * 2 + ((lane >> 2) & 1);
  if ((lane & 3) == 0 && row < SLAB_ROWS) red[warp][row] = v;
  __syncthreads();
  if ((int)threadIdx.x < nrows && ok) {
    float t = 0.f;
#pragma unroll
    for (int q = 0; q < GEMV_WARPS; ++q) t += red[q][threadIdx.x];
    float* yo = y + r0 + threadIdx.x;
    *yo = accumulate ? *yo + t : t;
  }
}

// QT = 8: Q8_0 rows (K bytes, 16-value chunks); QT = 4: Q4_0 rows (K / 2 bytes, one 32-value block per chunk).
// CTA c owns the contiguous rows [c * N / G, (c + 1) * N / G) (G = grid size).  When K fits one staged
// segment each warp walks the CTA's rows in batches of R rows, x is staged once, and the first batch is
// loaded before griddepcontrol.wait -- with a grid of one batch per warp that is every weight byte of the
// CTA; with the small streaming grid (`prefetch` set) the CTA also asks L2 for its whole row range at once.
// Longer rows are split into K segments and the grid has one batch per warp.
template <int QT, int R, int U, class XP>
__global__ void __launch_bounds__(GEMV_THREADS, R == 1 ? GEMV_MIN_CTAS : GEMV_MIN_CTAS - 1)
    gemv_kernel(const uint8_t* __restrict__ qs, const uint16_t* __restrict__ dsc, XP xp, float* __restrict__ y, int N,
                int K, int accumulate, int prefetch) {
  constexpr int VPC = QT == 8 ? 16 : 32;  // values per chunk
  constexpr int UPC = VPC / 8;            // 16-byte int16 units per chunk
  constexpr int CPB = QT == 8 ? 2 : 1;    // chunks per block
  static_assert(R * U == loads_per_lane(QT), "R rows x U chunks = the loads in flight per lane");
  extern __shared__ int4 smem_x[];
  __shared__ float red[GEMV_WARPS + 1];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // rows of this CTA: a balanced share of N (K <= SEG, warps loop over it) or exactly one batch per warp
  const bool looped = K <= SEG;
  const int r0 = looped ? (int)((long long)blockIdx.x * N / gridDim.x) : blockIdx.x * GEMV_WARPS * R;
  const int nrows = looped ? (int)((long long)(blockIdx.x + 1) * N / gridDim.x) - r0 : min(GEMV_WARPS * R, N - r0);
  const int kb = K / QK;
  const size_t row_bytes = QT == 8 ? (size_t)K : (size_t)K / 2;
  int4 w[R][U];
  float sc[R][U];
  pdl_trigger();
  if (looped) {
    const int nch = K / VPC;
    if (prefetch && threadIdx.x == 0) {
      prefetch_l2(qs + (size_t)r0 * row_bytes, (size_t)nrows * row_bytes);
      prefetch_l2(dsc + (size_t)r0 * kb, (size_t)nrows * kb * 2);
    }
    int rb = warp * R;  // first row (relative to r0) of this warp's current batch
    load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, r0 + rb, r0 + nrows, 0, 0, 0, nch, lane);
    float4* xf = reinterpret_cast<float4*>(smem_x);
    int4* xq = smem_x + K / 4;
    float* xs = reinterpret_cast<float*>(xq + K / 8);
    int* xsum = QT == 4 ? reinterpret_cast<int*>(xs + kb) : nullptr;
    pdl_wait();  // x (and y when accumulating) may come from the previous kernel
    stage_xq<UPC>(xf, xq, xs, xsum, xp, 0, K, red);
    __syncthreads();
    for (; rb < nrows; rb += GEMV_WARPS * R) {
      float acc[R];
#pragma unroll
      for (int r = 0; r < R; ++r) acc[r] = 0.f;
      for (int cb = 0; cb < nch; cb += 32 * U) {
        if (cb > 0) load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, r0 + rb, r0 + nrows, 0, 0, cb, nch, lane);
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int c = cb + lane + 32 * u;
          if (c >= nch) break;
          chunk_dot<QT, R, U>(acc, w, sc, u, c, xq, xs, xsum);
        }
      }
      // next batch of this warp: issue its loads before reducing this one
      const int nb = rb + GEMV_WARPS * R;
      if (nb < nrows) load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, r0 + nb, r0 + nrows, 0, 0, 0, nch, lane);
#pragma unroll
      for (int r = 0; r < R; ++r) {
        const float v = warp_sum(acc[r]);
        const int row = r0 + rb + r;
        if (lane == 0 && rb + r < nrows) y[row] = accumulate ? y[row] + v : v;
      }
    }
    return;
  }
  // K > SEG: one batch of R rows per warp, K in segments (x staged per segment)
  const int row0 = r0 + warp * R;
  float acc[R];
#pragma unroll
  for (int r = 0; r < R; ++r) acc[r] = 0.f;
  for (int k0 = 0; k0 < K; k0 += SEG) {
    const int len = min(SEG, K - k0);
    const int nch = len / VPC;
    float4* xf = reinterpret_cast<float4*>(smem_x);
    int4* xq = smem_x + len / 4;
    float* xs = reinterpret_cast<float*>(xq + len / 8);
    int* xsum = QT == 4 ? reinterpret_cast<int*>(xs + len / QK) : nullptr;
    load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, row0, r0 + nrows, k0 / VPC, k0 / QK, 0, nch, lane);
    if (k0 == 0) pdl_wait();
    if (k0 > 0) __syncthreads();
    stage_xq<UPC>(xf, xq, xs, xsum, xp, k0, len, red);
    __syncthreads();
    for (int cb = 0; cb < nch; cb += 32 * U) {
      if (cb > 0) load_batch<R, U, CPB>(w, sc, qs, dsc, row_bytes, kb, row0, r0 + nrows, k0 / VPC, k0 / QK, cb, nch, lane);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int c = cb + lane + 32 * u;
        if (c >= nch) break;
        chunk_dot<QT, R, U>(acc, w, sc, u, c, xq, xs, xsum);
      }
    }
  }
#pragma unroll
  for (int r = 0; r < R; ++r) {
    const float v = warp_sum(acc[r]);
    if (lane == 0 && row0 + r < r0 + nrows) y[row0 + r] = accumulate ? y[row0 + r] + v : v;
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

static int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

// Shape of the per-lane load batch: U chunks of each of R rows, R * U = loads_per_lane.  A row of nch chunks
// takes U = loads_per_lane when it spans a whole warp pass; shorter rows give each warp more rows, so every
// lane keeps the same number of loads in flight (Q8_0, K = 768: 48 chunks, U = 2, R = 4).
template <int QT, class XP>
static int launch_gemv(const uint8_t* qs, const uint16_t* d, const XP& xp, float* y, int n, int k, int accumulate,
                       cudaStream_t s) {
  if (!qs || !d || !y || n < 0 || k <= 0 || k % QK) return kBadArgument;
  if (n == 0) return kOk;
  const int len = min(k, SEG);
  const int nch = len / (QT == 8 ? 16 : 32);
  const int smem = seg_smem_bytes(len);
  // Streaming shapes (at least 64 MB of weights, K in one segment): int16 activations + DP2A, a grid of
  // GEMV_STREAM_CTAS_PER_SM CTAs per SM walking contiguous row ranges that are prefetched into L2.  Smaller
  // weights (the decode chain's GEMVs, whose time is set by the dependency on the previous kernel): fp32
  // activations, one batch per warp, every weight load issued before griddepcontrol.wait, no prefetch.
  const size_t weight_bytes = (QT == 8 ? (size_t)n * k : (size_t)n * k / 2) + (size_t)n * (k / QK) * 2;
  const bool stream = k <= SEG && weight_bytes >= GEMV_STREAM_BYTES;
  auto go = [&](auto kern, int r, int sm_bytes) -> int {  // streaming form (looped, prefetching)
    if (set_smem(kern, sm_bytes) != kOk) return kCudaError;
    const int rows_per_cta = GEMV_WARPS * r;
    const int grid = std::min((n + rows_per_cta - 1) / rows_per_cta, GEMV_STREAM_CTAS_PER_SM * sm_count());
    return launch_pdl(kern, dim3(grid), dim3(GEMV_THREADS), sm_bytes, s, qs, d, xp, y, n, k, accumulate, 1) ==
                   cudaSuccess
               ? kOk
               : kCudaError;
  };
  auto go_direct = [&](auto kern, int r, int sm_bytes) -> int {  // decode-chain form
    if (set_smem(kern, sm_bytes) != kOk) return kCudaError;
    const int rows_per_cta = GEMV_WARPS * r;
    const int grid = (n + rows_per_cta - 1) / rows_per_cta;
    return launch_pdl(kern, dim3(grid), dim3(GEMV_THREADS), sm_bytes, s, qs, d, xp, y, n, k, accumulate) ==
                   cudaSuccess
               ? kOk
               : kCudaError;
  };
  const int fsmem = len * 4;
  if constexpr (QT == 8) {
    const bool aligned = !(reinterpret_cast<uintptr_t>(qs) & 15) && !(reinterpret_cast<uintptr_t>(d) & 15);
    if (!stream && k == SLAB_K && aligned)
      return launch_pdl(gemv_slab_kernel<XP>, dim3((n + SLAB_ROWS - 1) / SLAB_ROWS), dim3(GEMV_THREADS), 0, s, qs, d,
                        xp, y, n, accumulate) == cudaSuccess
                 ? kOk
                 : kCudaError;
    if (stream) {
      if (nch > 128) return go(gemv_kernel<QT, 1, 8, XP>, 1, smem);
      if (nch > 64) return go(gemv_kernel<QT, 2, 4, XP>, 2, smem);
      if (nch > 32) return go(gemv_kernel<QT, 4, 2, XP>, 4, smem);
      return go(gemv_kernel<QT, 8, 1, XP>, 8, smem);
    }
    if (nch > 128) return go_direct(gemv_direct_kernel<QT, 1, 8, XP>, 1, fsmem);
    if (nch > 64) return go_direct(gemv_direct_kernel<QT, 2, 4, XP>, 2, fsmem);
    if (nch > 32) return go_direct(gemv_direct_kernel<QT, 4, 2, XP>, 4, fsmem);
    return go_direct(gemv_direct_kernel<QT, 8, 1, XP>, 8, fsmem);
  } else {
  if (stream) {
    if (nch > 64) return go(gemv_kernel<QT, 1, 4, XP>, 1, smem);
    if (nch > 32) return go(gemv_kernel<QT, 2, 2, XP>, 2, smem);
    return go(gemv_kernel<QT, 4, 1, XP>, 4, smem);
  }
  if (nch > 64) return go_direct(gemv_direct_kernel<QT, 1, 4, XP>, 1, fsmem);
  if (nch > 32) return go_direct(gemv_direct_kernel<QT, 2, 2, XP>, 2, fsmem);
  return go_direct(gemv_direct_kernel<QT, 4, 1, XP>, 4, fsmem);
  }
}

template <class XP>
static int launch_q8(const int8_t* qs, const uint16_t* d, const XP& xp, float* y, int n, int k, int accumulate,
                     cudaStream_t s) {
  return launch_gemv<8>(reinterpret_cast<const uint8_t*>(qs), d, xp, y, n, k, accumulate, s);
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

int gemv_wait_status(int reset) {
  int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_gemv_status, sizeof(int)) != cudaSuccess) return kCudaError;
  if (reset && v) {
    const int zero = 0;
    cudaMemcpyToSymbol(g_gemv_status, &zero, sizeof(int));
  }
  return v;
}

int gemv_q4_0(const uint8_t* qs, const uint16_t* d, const float* x, float* y, int n, int k, int accumulate,
              cudaStream_t s) {
  if (!x) return kBadArgument;
  return launch_gemv<4>(qs, d, XPlain{x}, y, n, k, accumulate, s);
}

}  // namespace zc
