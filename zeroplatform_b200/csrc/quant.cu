// quant.cu -- fp32 -> GGML Q8_0 / Q4_0 block quantizers on the device.
//
// Restates BlockQ8_0.Quantize (ZeroLlm/src/ZeroLlm.Core/Quantization/BlockQ8_0.cs:43-71) and
// BlockQ4_0.Quantize (BlockQ4_0.cs:120-150) as driven by LlmQuantizer.QuantizeToQ8_0 / QuantizeToQ4_0
// (LlmQuantizer.cs:20-57).  Every step is an IEEE-exact operation (division, reciprocal and product
// rounded to nearest, Math.Round = rint, (Half)f = __float2half_rn), so the blocks are bit-identical
// to the reference's.  Output is the reference's packed AoS layout (34 / 18 bytes per block).

#include <math.h>

#include "common.cuh"
#include "kernels.h"

namespace zc {

namespace {

__global__ void quantize_q8_0_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst, size_t nblocks) {
  const size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float4* s4 = reinterpret_cast<const float4*>(src + b * QK);
  float v[QK];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 t = s4[i];
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < QK; ++i) {
    const float a = fabsf(v[i]);
    if (a > amax) amax = a;
  }
  const float d = __fdiv_rn(amax, 127.0f);
  const float id = d > 1e-15f ? __frcp_rn(d) : 0.0f;
  uint16_t* out = reinterpret_cast<uint16_t*>(dst + b * Q8_BLOCK_BYTES);
  out[0] = __half_as_ushort(__float2half_rn(d));
#pragma unroll
  for (int i = 0; i < QK; i += 2) {
    int q0 = (int)rintf(__fmul_rn(v[i], id));
    int q1 = (int)rintf(__fmul_rn(v[i + 1], id));
    q0 = min(127, max(-127, q0));
    q1 = min(127, max(-127, q1));
    out[1 + i / 2] = (uint16_t)((q0 & 0xFF) | ((q1 & 0xFF) << 8));
  }
}

__global__ void quantize_q4_0_kernel(const float* __restrict__ src, uint8_t* __restrict__ dst, size_t nblocks) {
  const size_t b = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
  if (b >= nblocks) return;
  const float4* s4 = reinterpret_cast<const float4*>(src + b * QK);
  float v[QK];
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    float4 t = s4[i];
    v[4 * i] = t.x;
    v[4 * i + 1] = t.y;
    v[4 * i + 2] = t.z;
    v[4 * i + 3] = t.w;
  }
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < QK; ++i) {
    const float a = fabsf(v[i]);
    if (a > amax) amax = a;
  }
  const float d = __fdiv_rn(amax, 8.0f);
  const float id = d != 0.0f ? __frcp_rn(d) : 0.0f;
  uint16_t* out = reinterpret_cast<uint16_t*>(dst + b * Q4_BLOCK_BYTES);
  out[0] = __half_as_ushort(__float2half_rn(d));
  uint32_t bytes[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    const int q0 = min(15, max(0, (int)rintf(__fmul_rn(v[i], id)) + 8));
    const int q1 = min(15, max(0, (int)rintf(__fmul_rn(v[i + 16], id)) + 8));
    bytes[i] = (uint32_t)((q0 & 0x0F) | ((q1 & 0x0F) << 4));
  }
#pragma unroll
  for (int i = 0; i < 16; i += 2) out[1 + i / 2] = (uint16_t)(bytes[i] | (bytes[i + 1] << 8));
}

}  // namespace

int quantize_q8_0(const float* src, uint8_t* dst, size_t n, cudaStream_t s) {
  if (!src || !dst || n % QK) return kBadArgument;
  if (reinterpret_cast<uintptr_t>(src) & 15) return kUnsupported;
  const size_t nb = n / QK;
  if (nb == 0) return kOk;
  quantize_q8_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(src, dst, nb);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

int quantize_q4_0(const float* src, uint8_t* dst, size_t n, cudaStream_t s) {
  if (!src || !dst || n % QK) return kBadArgument;
  if (reinterpret_cast<uintptr_t>(src) & 15) return kUnsupported;
  const size_t nb = n / QK;
  if (nb == 0) return kOk;
  quantize_q4_0_kernel<<<(unsigned)((nb + 255) / 256), 256, 0, s>>>(src, dst, nb);
  return cudaPeekAtLastError() == cudaSuccess ? kOk : kCudaError;
}

}  // namespace zc
