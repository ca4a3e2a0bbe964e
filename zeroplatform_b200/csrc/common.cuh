// common.cuh -- shared device helpers for the ZeroLlm B200 kernels (sm_100a only).
#pragma once

#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <utility>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "zeroplatform_b200 kernels are written for sm_100a (B200) only"
#endif

namespace zc {

// Status codes shared by every entry point (0 = handled, as the reference bridge expects).
enum Status : int {
  kOk = 0,
  kNotHandled = -1,      // caller should run its own (managed) path
  kBadArgument = -2,     // sizes / alignment / null pointers
  kCudaError = -3,       // a CUDA runtime call failed; details in zc_cuda_last_error()
  kUnsupported = -4,     // a shape this library does not cover
  kOutOfMemory = -5,     // device allocation failed
  kTooLarge = -6,        // exceeds a fixed-capacity buffer
};

constexpr int QK = 32;            // elements per Q8_0 / Q4_0 block
constexpr int Q8_BLOCK_BYTES = 34;
constexpr int Q4_BLOCK_BYTES = 18;

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 128-bit streaming load that bypasses L1 allocation: weights are read exactly once per call.
__device__ __forceinline__ int4 ld_stream_v4(const void* p) {
  int4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.s32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

// Programmatic dependent launch: let the next kernel in the stream start its prologue now, and wait until the
// previous kernel's memory is visible before touching anything it produced.  Both are no-ops when the kernel
// was launched without the programmatic-serialization attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ float4 ld_f4(const float* p) { return __ldg(reinterpret_cast<const float4*>(p)); }

__device__ __forceinline__ float h2f(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// v as the pair of fp16 values the tensor-core GEMM takes for an activation: hi = fp16(v) at p[0] and
// lo = fp16(v - hi) at p[lo_off] (v - hi is exact in fp32; hi + lo holds v to about 2^-22 relative).
__device__ __forceinline__ void store_hl(__half* p, size_t lo_off, float v) {
  const __half h = __float2half_rn(v);
  p[0] = h;
  p[lo_off] = __float2half_rn(v - __half2float(h));
}

__device__ __forceinline__ void store_act(float* p, size_t, float v) { *p = v; }
__device__ __forceinline__ void store_act(__half* p, size_t lo_off, float v) { store_hl(p, lo_off, v); }

// Exact int8 -> fp32 for the four signed bytes of w: byte i becomes the float 2^23 + (q_i + 128),
// from which one subtraction recovers q_i exactly (PRMT + FADD instead of a conversion unit op).
__device__ __forceinline__ void s8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t b = w ^ 0x80808080u;
  const float bias = 8388736.0f;  // 2^23 + 128
  f0 = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7650)) - bias;
  f1 = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7651)) - bias;
  f2 = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7652)) - bias;
  f3 = __uint_as_float(__byte_perm(b, 0x4B000000u, 0x7653)) - bias;
}

// Exact nibble -> fp32 with the Q4_0 offset: byte i of v (each 0..15) becomes (v_i - 8).
__device__ __forceinline__ void u4x4_to_f32(uint32_t v, float& f0, float& f1, float& f2, float& f3) {
  const float bias = 8388616.0f;  // 2^23 + 8
  f0 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7650)) - bias;
  f1 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7651)) - bias;
  f2 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7652)) - bias;
  f3 = __uint_as_float(__byte_perm(v, 0x4B000000u, 0x7653)) - bias;
}

// SplitMix64 (Steele, Lea and Flood, "Fast splittable pseudorandom number generators", OOPSLA 2014) of x, its top
// 24 bits as a float in [0, 1): the counter-based draw of the device sampler (one per generated token).
__host__ __device__ inline float splitmix_uniform(uint64_t x) {
  uint64_t z = x + 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  z ^= z >> 31;
  return (float)(z >> 40) * (1.0f / 16777216.0f);
}

// Launches `kernel` with programmatic stream serialization, so it may overlap the tail of the previous
// kernel in the stream (the kernel itself calls pdl_wait() before reading that kernel's outputs).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s,
                              Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

}  // namespace zc
