/*
 * zero_tensor.h -- the ZeroTensor native-bridge C ABI, implemented on B200 by libzero_tensor.so.
 *
 * These are exactly the exports that ZeroTensorNativeBridge resolves
 * (ZeroTensor/src/ZeroTensor.Core/Native/ZeroTensorNativeBridge.cs:93-108, :144-185) and calls through
 * `delegate* unmanaged[Cdecl]` pointers (:255-389).  The bridge marks the library available only
 * when the first six resolve (:157).  C# `nuint` is size_t, `nint` is intptr_t.
 *
 * Contract (same as the reference):
 *   - every pointer is HOST memory owned by the caller (pinned by `fixed` for the call);
 *   - the call is synchronous: results are in the output buffer when it returns;
 *   - return 0 = handled; any other value = not handled, and the C# caller silently runs its
 *     managed path (GgufFormat.cs:343-349, :441-447; TensorOps.Neural.cs:2408-2413).
 *     Codes: -1 not handled, -2 bad argument, -3 CUDA error (message in zc_cuda_last_error()),
 *     -4 unsupported shape, -5 out of device memory;
 *   - calls are re-entrant: each host thread gets its own CUDA stream and staging buffers
 *     (LlmEngine.PrefillPrompt calls the kernels from Parallel.For workers, LlmEngine.cs:208,252).
 * The work runs on the calling thread's current CUDA device.  There is no CPU fallback inside
 * the library: when no usable GPU is present every compute entry returns -3.
 */
#ifndef ZERO_TENSOR_H
#define ZERO_TENSOR_H

#include <stddef.h>
#include <stdint.h>

#ifndef ZC_API
#if defined(__GNUC__)
#define ZC_API __attribute__((visibility("default")))
#else
#define ZC_API
#endif
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* zc_version -> uint (ZeroTensorNativeBridge.cs:93,144). Encoded as major<<16 | minor<<8 | patch. */
ZC_API uint32_t zc_version(void);

/* zc_is_simd_supported -> int (ZeroTensorNativeBridge.cs:94,146): 1 when a B200-class GPU
 * (compute capability 10.x) is visible, else 0. */
ZC_API int32_t zc_is_simd_supported(void);

/* zc_gemm_f32 (ZeroTensorNativeBridge.cs:95,276-287; caller TensorBlas.cs:138):
 * C = alpha * A(m,k) * B(k,n) + beta * C with arbitrary element strides (row stride, column stride). */
ZC_API int32_t zc_gemm_f32(size_t m, size_t n, size_t k, float alpha, const float* a, intptr_t rsa, intptr_t csa,
                    const float* b, intptr_t rsb, intptr_t csb, float beta, float* c, intptr_t rsc, intptr_t csc,
                    int32_t parallel);

/* zc_flash_attention_f32 (ZeroTensorNativeBridge.cs:96,290-302; caller TensorOps.Neural.cs:1062-1080):
 * TensorOps.FlashAttentionCpu on the device.  q [batch][sq][d], k [kv batch][sk][d], v [kv batch][sk][dv], out
 * [batch][sq][dv]; kv batch of b = is_gqa ? (b / hq) * hkv + (b % hq) / group : b.  Handles mask == NULL, dv == d,
 * d one of 16 / 32 / 64 / 128; returns -1 (not handled: the managed FlashAttention runs) for a mask, whose broadcast
 * extent the ABI does not carry, and for other shapes.  sk == 0 gives zeros. */
ZC_API int32_t zc_flash_attention_f32(size_t batch, size_t sq, size_t sk, size_t d, size_t dv, float scale, int32_t is_gqa,
                               size_t hq, size_t hkv, size_t group, const float* q, const float* k, const float* v,
                               const float* mask, float* out);

/* zc_gemv_q4_0 (ZeroTensorNativeBridge.cs:97,305-309; caller GgufDequantizer.GemvQ4_0,
 * GgufFormat.cs:333-349): y[n_rows] = W x for W the raw GGML Q4_0 blocks (18 B each, row-major,
 * k_cols/32 blocks per row) and x[k_cols].  k_cols must be a multiple of 32. */
ZC_API int32_t zc_gemv_q4_0(const uint8_t* w, const float* x, float* y, size_t n_rows, size_t k_cols);

/* zc_gemv_q8_0 (ZeroTensorNativeBridge.cs:98,311-316; caller GgufDequantizer.GemvQ8_0,
 * GgufFormat.cs:431-447): as zc_gemv_q4_0 with Q8_0 blocks (34 B each). */
ZC_API int32_t zc_gemv_q8_0(const uint8_t* w, const float* x, float* y, size_t n_rows, size_t k_cols);

/* zc_rmsnorm_f32 (ZeroTensorNativeBridge.cs:99,255-259; caller TensorOps.Neural.cs:165):
 * dst = x / sqrt(mean(x^2) + eps) * w over n elements. */
ZC_API int32_t zc_rmsnorm_f32(size_t n, const float* x, const float* w, float* dst, float eps);

/* zc_silu_f32 (ZeroTensorNativeBridge.cs:100,261-266): dst = src / (1 + exp(-src)). */
ZC_API int32_t zc_silu_f32(size_t n, const float* src, float* dst);

/* zc_swiglu_f32 (ZeroTensorNativeBridge.cs:101,268-273; caller TensorOps.Neural.cs:465):
 * dst = silu(gate) * up. */
ZC_API int32_t zc_swiglu_f32(size_t n, const float* gate, const float* up, float* dst);

/* zc_rope_f32 (ZeroTensorNativeBridge.cs:104,332-337; caller TensorOps.Neural.cs:1273, interleaved
 * mode): x is [num_heads][seq_len][head_dim]; pair (2i, 2i+1) of position pos_offset + s rotates by
 * pos * (1 / (float)pow(theta_base, 2i/head_dim)), as the managed ApplyRoPEInPlace computes it. */
ZC_API int32_t zc_rope_f32(size_t num_heads, size_t seq_len, size_t head_dim, size_t pos_offset, float theta_base, float* x);

/* zc_paged_attention_f32 (ZeroTensorNativeBridge.cs:105,340-348; caller TensorOps.PagedAttention,
 * TensorOps.Neural.cs:2372-2416): q/out [hq][hd]; k_cache/v_cache pools [num_blocks][block_size][hkv][hd]
 * fp32; block_table[ceil(ctx_len/block_size)] physical block ids. The pool extent is not part of the
 * ABI: the blocks referenced by the table are what is read. */
ZC_API int32_t zc_paged_attention_f32(size_t hq, size_t hkv, size_t hd, size_t block_size, size_t ctx_len, float scale,
                               const float* q, const float* k_cache, const float* v_cache, const int32_t* block_table,
                               float* out);

/* zc_dot_i8 (ZeroTensorNativeBridge.cs:108,385-389): *out = sum a[i]*b[i] with int32 accumulation. */
ZC_API int32_t zc_dot_i8(size_t n, const int8_t* a, const int8_t* b, int32_t* out);

/* Weight residency (not in the reference ABI).  Registers a read-only quantized weight tensor that lives
 * in host memory -- e.g. a tensor inside the memory-mapped GGUF file that GgufArchive.MatMulQuantized
 * streams from (GgufFormat.cs:164-247) -- so that later zc_gemv_q8_0 / zc_gemv_q4_0 calls with the same
 * pointer, shape and type on the same device use a device-resident copy: only x and y cross PCIe.
 * ggml_type uses the GGML ids the reference uses (GgufFormat.cs:41 GgmlType): 8 = Q8_0, 2 = Q4_0.
 * The caller promises that the bytes do not change until zc_unregister_weights (true for a read-only
 * mmap).  Registering an already registered pointer replaces the copy. */
ZC_API int32_t zc_register_weights(int32_t ggml_type, const uint8_t* w, size_t n_rows, size_t k_cols);
ZC_API int32_t zc_unregister_weights(const uint8_t* w);

/* Message of the last failure on the calling thread ("" if none). Not in the reference ABI. */
ZC_API const char* zc_cuda_last_error(void);

#ifdef __cplusplus
}
#endif
#endif
