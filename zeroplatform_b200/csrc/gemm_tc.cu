// gemm_tc.cu -- batched / prefill quantized GEMM on the 5th-generation tensor cores (tcgen05, sm_100a).
//
// Y[m, n] (=|+=) sum_k X[m, k] * dequant(W)[n, k] for X fp32 [M][K], W Q8_0 (SoA: int8 [N][K] + fp16
// scales [N][K/32]) or Q4_0 (SoA: nibbles [N][K/32][16] + fp16 scales), Y fp32 [M][N].  This is LlmEngine.PrefillPrompt's token-parallel loop of
// QuantizedKernels.MatVecMulQ8_0 / MatVecAddQ8_0 (ZeroLlm/src/ZeroLlm.Core/Engine/LlmEngine.cs:208-304,
// Quantization/QuantizedKernels.cs:190-308) executed as one contraction.
//
// Numerics: both operands enter the tensor core as pairs of fp16 values.  Weights: a_hi = fp16(q * d) (the
// exact product rounded once) and a_lo = fp16(q * d - a_hi) (one fused multiply-add: the residual rounded
// once); activations: x_hi = fp16(x) and x_lo = fp16(x - x_hi).  Each 16-wide k-step accumulates three products
// in fp32 TMEM -- a_hi x_hi + a_hi x_lo + a_lo x_hi, two instructions since the x_hi and x_lo tiles form one
// operand of twice the width -- and the products are exact, so the result carries both operands to about 2^-22 (the dropped a_lo x_lo term is below 2^-22) and differs from the fp32
// reference only by summation order.  A single fp16(q * d) x fp16(x) product misses the 1e-3 bound on
// 4096-wide layers.  (An int8 MMA cannot apply the per-32-value fp16 block scales inside the tensor core, and a
// CUDA-core epilogue per block would run several times slower than the MMA itself.)
//
// Structure (one persistent CTA per SM, 16 warps):
//   warp 0      TMA producer: raw int8 W tiles [128 rows x 256 k] into a shared-memory ring (2-6 deep)
//   warp 1      MMA issuer: one thread issues 4 x 2 tcgen05.mma.kind::f16 (M=128, N=2 BN and BN, K=16) per stage
//   warp 2      TMA producer: activation tiles (fp16, pre-converted) [BN tokens x 64 k], 128B swizzle
//   warps 4-11  dequantizers: int8 W tile (shared memory) x fp16 block scales -> fp16 hi / lo planes of q*d,
//               either in shared memory in the UMMA K-major 128B-swizzled layout (fence.proxy.async before
//               signalling the MMA warp) or, for tiles of at most 64 tokens and Q8_0 tiles of 128, in TMEM
//               (tcgen05.st, one weight row per lane; the MMA then reads A from TMEM)
//   warps 12-15 epilogue: tcgen05.ld 32 TMEM columns at a time, coalesced fp32 stores of Y (or of the
//               split-K partials, summed afterwards in split order by splitk_reduce_kernel)
// The accumulator is double-buffered in TMEM (2 x 2 BN columns: the x_hi and x_lo halves) so the epilogue of
// one tile overlaps the MMAs of the next.  Every mbarrier wait is bounded: on time-out the CTA records an error code in
// `status`, stops issuing work, drains what it issued and frees its TMEM before returning.
//
// Roofline: tensor (fp16 dense), flops = 2 * M * N * K.

#include <cuda.h>

#include "common.cuh"
#include "kernels.h"
#include "sync.cuh"

namespace zc {

namespace {

constexpr int BM = 128;                   // weight rows per tile = MMA M = TMEM lanes
constexpr int BK = 64;                    // k per stage: 64 fp16 = one 128-byte swizzle row
constexpr int MAX_STAGES = 8;             // ring depth limit (barrier arrays are sized for it)
constexpr int DQ_WARPS = 8;               // weight dequantizer warps (two per SM sub-partition)
constexpr int DQ_THREADS = DQ_WARPS * 32;
constexpr int DQ_ITEMS = BM * BK / 16 / DQ_THREADS;  // 16-value chunks per dequantizer thread per stage
constexpr int EPI_WARP0 = 4 + DQ_WARPS;       // first of the four epilogue warps
constexpr int GEMM_THREADS = (EPI_WARP0 + 4) * 32;
constexpr int A_PLANE_BYTES = BM * BK * 2;      // 16 KB: one fp16 plane (hi or lo) of A
constexpr int A_STAGE_BYTES = 2 * A_PLANE_BYTES;  // a stage holds both planes
constexpr int W_SUB = 4;                    // k-stages per int8 weight tile (one TMA box of 256 bytes x 128 rows)
constexpr int S_TILE_BYTES = BM * BK * W_SUB / QK * 2;  // fp16 block scales of a weight tile (8 per row)
// Quantized bytes of a weight tile [128 rows x 256 k]: 32 KB of int8 (Q8_0) or 16 KB of nibbles (Q4_0).
__host__ __device__ constexpr int w_tile_bytes(int qt) { return qt == 8 ? BM * BK * W_SUB : BM * BK * W_SUB / 2; }
__host__ __device__ constexpr int w_stage_bytes(int qt) { return w_tile_bytes(qt) + S_TILE_BYTES; }
__host__ __device__ constexpr int w_row_bytes(int qt) { return w_tile_bytes(qt) / BM; }  // 256 or 128
constexpr int MAX_SPLITS = 8;               // split-K ranges per output tile at most
// Tensor-memory A (tile widths BN <= 64, and Q8_0 tiles of BN = 128 with a single accumulator; TMA'd scales):
// the dequantizers store the fp16 hi / lo planes of each k-stage into TMEM columns after the accumulators (64
// columns a stage: 32 hi, 32 lo), so A never occupies shared memory or its bandwidth.  The weight tile then arrives 128B-swizzled (128-byte boxes) so that
// one-row-per-lane reads are conflict free.
constexpr int TMEM_COLS = 512;
constexpr int A_TMEM_STAGE_COLS = 64;
constexpr int AT_MAX_BN = 64;

struct GemmParams {
  const uint16_t* d;
  float* y;         // output [M][N]
  float* part;      // split partials [splits][M][N] (splits > 1)
  int* status;
  int M, N, K;
  int accumulate;
  int bn;           // tokens per tile (MMA N): 32, 64, 128 or 256
  int ab_stages;    // A/B pipeline depth
  int w_stages;     // int8 weight ring depth
  int n_tok_tiles;
  int n_tiles;      // output tiles
  int splits;       // K ranges per tile (split-K); work units = n_tiles * splits
  int kb_per_split;  // a multiple of W_SUB
  int scale_tma;     // 1: block scales arrive by TMA with their weight tile (K % 256 == 0), 0: loaded per item
  int x_merged;      // 1: x_map is 3-D (k, token, hi / lo plane): one TMA box brings both activation tiles
  int acc_bufs;      // TMEM accumulators: 2 (the epilogue of a tile overlaps the next tile's MMAs), or 1 for
                     // 128-token tiles with A in TMEM (their 2 x 128 accumulator columns leave room for 4 A stages)
};

__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
      : "memory");
}

// UMMA shared-memory descriptor: K-major operand, 128-byte swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t addr) {
  uint64_t desc = 0;
  desc |= (uint64_t)((addr & 0x3FFFFu) >> 4);  // start address
  desc |= (uint64_t)1u << 16;                   // leading byte offset (unused for swizzled K-major)
  desc |= (uint64_t)(1024u >> 4) << 32;         // stride byte offset between 8-row core groups
  desc |= (uint64_t)1u << 46;                   // descriptor version for tcgen05
  desc |= (uint64_t)2u << 61;                   // layout: SWIZZLE_128B
  return desc;
}

// Instruction descriptor for kind::f16: A = B = fp16, D = fp32, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(a), "l"(b), "r"(idesc), "r"(acc));
}

// The same with A read from tensor memory at column address a_tmem (rows on lanes, two fp16 per column).
__device__ __forceinline__ void umma_f16_ta(uint32_t tmem_d, uint32_t a_tmem, uint64_t b, uint32_t idesc,
                                            uint32_t acc) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
      "r"(a_tmem), "l"(b), "r"(idesc), "r"(acc));
}

// 16 consecutive 32-bit columns of this thread's TMEM lane (the warp's lane quadrant) from registers.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
      "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive 32-bit columns of this thread's TMEM lane.  The registers are operands of the wait as well, so
// no read of them can be scheduled before the load has completed.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]),
                 "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

// q (exact fp16 pair) times the block scale -> (hi, lo) = (fp16(q d), fp16(q d - hi)): the fused multiply-add
// forms q d - hi exactly before its single rounding.
__device__ __forceinline__ void scale_hl(__half2 q, __half2 d2, uint32_t& hi, uint32_t& lo) {
  const __half2 h = __hmul2_rn(q, d2);
  const __half2 l = __hfma2(q, d2, __hneg2(h));
  hi = *reinterpret_cast<const uint32_t*>(&h);
  lo = *reinterpret_cast<const uint32_t*>(&l);
}

// 16 int8 weights (one int4) times the fp16 block scale -> 16 hi and 16 lo fp16 values, as 16-byte chunks of
// values 0-7 (h0, l0) and 8-15 (h1, l1).
__device__ __forceinline__ void dequant16(int4 w, __half2 d2, uint4& h0, uint4& h1, uint4& l0, uint4& l1) {
  const uint32_t* wv = reinterpret_cast<const uint32_t*>(&w);
  uint32_t oh[8], ol[8];
  const __half2 bias = __halves2half2(__ushort_as_half(0x6480), __ushort_as_half(0x6480));  // 1024 + 128
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t b = wv[j] ^ 0x80808080u;  // q + 128 in each byte
    // halves 0x64XX = 1024 + XX (exact), pairs (byte0, byte1) and (byte2, byte3)
    const uint32_t p01 = __byte_perm(b, 0x64646464u, 0x5140);
    const uint32_t p23 = __byte_perm(b, 0x64646464u, 0x7362);
    scale_hl(__hsub2(*reinterpret_cast<const __half2*>(&p01), bias), d2, oh[2 * j], ol[2 * j]);  // exact q first
    scale_hl(__hsub2(*reinterpret_cast<const __half2*>(&p23), bias), d2, oh[2 * j + 1], ol[2 * j + 1]);
  }
  h0 = make_uint4(oh[0], oh[1], oh[2], oh[3]);
  h1 = make_uint4(oh[4], oh[5], oh[6], oh[7]);
  l0 = make_uint4(ol[0], ol[1], ol[2], ol[3]);
  l1 = make_uint4(ol[4], ol[5], ol[6], ol[7]);
}

// Four nibbles (one per byte, 0..15) -> two half2 of (u - 8) * d, hi and lo.
__device__ __forceinline__ void nib4(uint32_t u, __half2 d2, uint32_t& h0, uint32_t& h1, uint32_t& l0, uint32_t& l1) {
  const __half2 bias = __halves2half2(__ushort_as_half(0x6408), __ushort_as_half(0x6408));  // 1024 + 8
  const uint32_t a = __byte_perm(u, 0x64646464u, 0x5140);
  const uint32_t b = __byte_perm(u, 0x64646464u, 0x7362);
  scale_hl(__hsub2(*reinterpret_cast<const __half2*>(&a), bias), d2, h0, l0);  // exact u - 8, then * d
  scale_hl(__hsub2(*reinterpret_cast<const __half2*>(&b), bias), d2, h1, l1);
}

// One Q4_0 block (16 bytes: byte j = value j | value j+16 << 4) times its scale -> 32 hi and 32 lo fp16 values
// as four 16-byte chunks each (values 0-7, 8-15, 16-23, 24-31).
__device__ __forceinline__ void dequant32_q4(int4 w, __half2 d2, uint4 (&ch)[4], uint4 (&cl)[4]) {
  const uint32_t m = 0x0F0F0F0Fu;
  const uint32_t wv[4] = {(uint32_t)w.x, (uint32_t)w.y, (uint32_t)w.z, (uint32_t)w.w};
  uint32_t oh[16], ol[16];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    nib4(wv[j] & m, d2, oh[2 * j], oh[2 * j + 1], ol[2 * j], ol[2 * j + 1]);  // values 4j .. 4j+3
    nib4((wv[j] >> 4) & m, d2, oh[8 + 2 * j], oh[8 + 2 * j + 1], ol[8 + 2 * j], ol[8 + 2 * j + 1]);  // 16+4j ..
  }
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    ch[q] = make_uint4(oh[4 * q], oh[4 * q + 1], oh[4 * q + 2], oh[4 * q + 3]);
    cl[q] = make_uint4(ol[4 * q], ol[4 * q + 1], ol[4 * q + 2], ol[4 * q + 3]);
  }
}

// QT = 8: Q8_0 weights (int8 tiles); QT = 4: Q4_0 weights (nibble tiles, one 32-value block per dequant item).
// AT: A in tensor memory (see TMEM_COLS); otherwise A in shared memory.
template <int QT, bool AT>
__global__ void __launch_bounds__(GEMM_THREADS, 1)
    gemm_q8_0_tc_kernel(const __grid_constant__ CUtensorMap x_map, const __grid_constant__ CUtensorMap xl_map,
                        const __grid_constant__ CUtensorMap w_map, const __grid_constant__ CUtensorMap s_map,
                        GemmParams p) {
  constexpr int W_STAGE_BYTES = w_stage_bytes(QT);
  constexpr int W_TILE_BYTES = w_tile_bytes(QT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int bn = p.bn;
  const int AST = p.ab_stages;
  const int WSTAGES = p.w_stages;
  const int b_tile_bytes = bn * BK * 2;         // one fp16 activation tile (hi or lo)
  const int b_stage_bytes = 2 * b_tile_bytes;   // hi tile, then lo tile
  uint8_t* a_st = smem;                                  // AST x 2 x 16 KB (fp16 A hi, lo planes; SW128); none if AT
  uint8_t* b_st = AT ? smem : a_st + AST * A_STAGE_BYTES;  // AST x 2 x bn*128 B (fp16 X hi, lo; SW128 by TMA)
  uint8_t* w_st = b_st + AST * b_stage_bytes;            // WSTAGES x 8 KB (int8 W, TMA, unswizzled)
  uint64_t* bars = reinterpret_cast<uint64_t*>(w_st + WSTAGES * W_STAGE_BYTES);
  uint64_t* ab_full = bars;                            // [AST]: DQ_THREADS dequant arrivals + 1 X TMA (tx)
  uint64_t* ab_empty = bars + MAX_STAGES;              // [AST]: MMA commit
  uint64_t* w_full = bars + 2 * MAX_STAGES;            // [WSTAGES]: W TMA (tx)
  uint64_t* w_empty = bars + 3 * MAX_STAGES;           // [WSTAGES]: DQ_THREADS dequant arrivals
  uint64_t* tfull = bars + 4 * MAX_STAGES;             // [2]
  uint64_t* tempty = tfull + 2;                  // [2]
  uint64_t* drain = tempty + 2;                  // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nk = (p.K + BK - 1) / BK;
  const int n_units = p.n_tiles * p.splits;

  if (threadIdx.x == 0) {
    for (int s = 0; s < AST; ++s) {
      mbar_init(smem_u32(&ab_full[s]), DQ_THREADS + 1);
      mbar_init(smem_u32(&ab_empty[s]), 1);
    }
    for (int s = 0; s < WSTAGES; ++s) {
      mbar_init(smem_u32(&w_full[s]), 1);
      mbar_init(smem_u32(&w_empty[s]), DQ_THREADS);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(smem_u32(&tfull[a]), 1);
      mbar_init(smem_u32(&tempty[a]), 128);
    }
    mbar_init(smem_u32(drain), 1);
    *abort_flag = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {  // 2 accumulators of 2 bn fp32 columns: [x_hi sums | x_lo sums] (power of two >= 128),
                    // with A's stages after them when AT
    const uint32_t ncols = AT ? (uint32_t)TMEM_COLS : 4u * (uint32_t)bn;
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(tmem_slot)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;
  // Programmatic dependent launch: the next kernel may be scheduled now.  Weights never depend on the
  // previous kernel, so the weight producer and the dequantizers start at once; the activation producer and
  // the epilogue wait for the previous kernel (its X is read, and Y may still be read by it) first.
  pdl_trigger();

  // Work unit u -> output tile u / splits (weight tile major), K range (u % splits).
  auto unit_tile = [&](int u) { return u / p.splits; };
  auto unit_kb0 = [&](int u) { return (u % p.splits) * p.kb_per_split; };
  auto unit_kb1 = [&](int u) { return min(nk, (u % p.splits + 1) * p.kb_per_split); };

  if (warp == 0) {
    // ---------------- TMA producer: raw int8 weight tiles [128 rows x 64 k] ----------------
    if (lane == 0) {
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
        const int row0 = (unit_tile(u) / p.n_tok_tiles) * BM;
        for (int kb = unit_kb0(u); kb < unit_kb1(u); kb += W_SUB) {  // one box covers W_SUB k-stages
          if (!mbar_wait(smem_u32(&w_empty[s]), ph ^ 1, abort_flag, p.status, 1)) break;
          mbar_arrive_tx(smem_u32(&w_full[s]), (uint32_t)(p.scale_tma ? W_STAGE_BYTES : W_TILE_BYTES));
          tma_load_2d(smem_u32(w_st + s * W_STAGE_BYTES), &w_map, QT == 8 ? kb * BK : kb * BK / 2, row0,
                      smem_u32(&w_full[s]));
          if (AT && QT == 8)  // the second 128-byte half of the 256-byte rows
            tma_load_2d(smem_u32(w_st + s * W_STAGE_BYTES + BM * 128), &w_map, kb * BK + 128, row0,
                        smem_u32(&w_full[s]));
          if (p.scale_tma)  // the 8 scales per row of these 256 k (x = kb * 2, a multiple of 8 scales = 16 bytes)
            tma_load_2d(smem_u32(w_st + s * W_STAGE_BYTES + W_TILE_BYTES), &s_map, kb * (BK / QK), row0,
                        smem_u32(&w_full[s]));
          if (++s == WSTAGES) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (*abort_flag) __nanosleep(20000);  // let issued loads land before the CTA can exit
    }
  } else if (warp == 2) {
    // ---------------- TMA producer: fp16 activation tiles [bn tokens x 64 k] ----------------
    if (lane == 0) {
      pdl_wait();
      int s = 0;
      uint32_t ph = 0;
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
        const int tok0 = (unit_tile(u) % p.n_tok_tiles) * bn;
        for (int kb = unit_kb0(u); kb < unit_kb1(u); ++kb) {
          if (!mbar_wait(smem_u32(&ab_empty[s]), ph ^ 1, abort_flag, p.status, 6)) break;
          mbar_arrive_tx(smem_u32(&ab_full[s]), (uint32_t)b_stage_bytes);
          if (p.x_merged) {  // [plane][token][64 k]: the hi tile, then the lo tile, in one instruction
            tma_load_3d(smem_u32(b_st + s * b_stage_bytes), &x_map, kb * BK, tok0, 0, smem_u32(&ab_full[s]));
          } else {
            tma_load_2d(smem_u32(b_st + s * b_stage_bytes), &x_map, kb * BK, tok0, smem_u32(&ab_full[s]));
            tma_load_2d(smem_u32(b_st + s * b_stage_bytes + b_tile_bytes), &xl_map, kb * BK, tok0,
                        smem_u32(&ab_full[s]));
          }
          if (++s == AST) {
            s = 0;
            ph ^= 1;
          }
        }
      }
      if (*abort_flag) __nanosleep(20000);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      // Per 16-wide k-step two MMAs: a_hi x [x_hi | x_lo] (N = 2 bn: the hi and lo activation tiles are adjacent
      // rows of the B stage) into accumulator columns [0, 2 bn), then a_lo x x_hi (N = bn) added into [0, bn); the
      // epilogue adds column c + bn to column c.  Shared-memory descriptors advance by address / 16, so they are
      // formed once and offset per stage and k-step.
      const uint32_t idesc2 = idesc_f16(BM, 2 * bn), idesc1 = idesc_f16(BM, bn);
      const uint64_t adesc0 = umma_desc_sw128(smem_u32(a_st)), bdesc0 = umma_desc_sw128(smem_u32(b_st));
      int s = 0;
      uint32_t ph = 0;
      int it = 0;
      for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x, ++it) {
        const int acc = it % p.acc_bufs;
        const uint32_t acc_ph = (uint32_t)(it / p.acc_bufs) & 1;
        if (!mbar_wait(smem_u32(&tempty[acc]), acc_ph ^ 1, abort_flag, p.status, 2)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + (uint32_t)(acc * 2 * bn);
        bool ok = true;
        const int kb0 = unit_kb0(u);
        for (int kb = kb0; kb < unit_kb1(u); ++kb) {
          if (!mbar_wait(smem_u32(&ab_full[s]), ph, abort_flag, p.status, 3)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t bd = bdesc0 + (uint64_t)(s * (b_stage_bytes >> 4));
          if constexpr (AT) {  // A stage s: TMEM columns [2 acc_bufs bn + 64 s, +32) hi, [+32, +64) lo; 8 per k16
            const uint32_t at = tmem_base + (uint32_t)(2 * p.acc_bufs * bn + s * A_TMEM_STAGE_COLS);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {
              umma_f16_ta(d_tmem, at + 8 * kk, bd + 2 * kk, idesc2, (kb != kb0 || kk != 0) ? 1u : 0u);
              umma_f16_ta(d_tmem, at + 32 + 8 * kk, bd + 2 * kk, idesc1, 1u);
            }
          } else {
            const uint64_t ad = adesc0 + (uint64_t)(s * (A_STAGE_BYTES >> 4));
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk) {  // +32 bytes of K per step = +2 in the descriptor
              umma_f16(d_tmem, ad + 2 * kk, bd + 2 * kk, idesc2, (kb != kb0 || kk != 0) ? 1u : 0u);  // a_hi x [hi|lo]
              umma_f16(d_tmem, ad + (A_PLANE_BYTES >> 4) + 2 * kk, bd + 2 * kk, idesc1, 1u);          // a_lo x x_hi
            }
          }
          umma_commit(smem_u32(&ab_empty[s]));  // frees the A/B stage once these MMAs have read it
          if (++s == AST) {
            s = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(smem_u32(&tfull[acc]));  // accumulator complete
      }
      // Every MMA issued above has finished once this commit's barrier flips (bounded on an abort).
      umma_commit(smem_u32(drain));
      uint64_t t0 = global_ns();
      while (!mbar_try(smem_u32(drain), 0) && global_ns() - t0 < WAIT_NS) {
      }
    }
  } else if (warp >= 4 && warp < EPI_WARP0) {
    // ---------------- W dequantizers: int8 tile in smem -> fp16(q*d) in the SW128 layout ----------------
    const int tid = threadIdx.x - 128;  // 0..DQ_THREADS-1
    int ws = 0, as = 0;
    uint32_t wph = 0, aph = 0;
    for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x) {
      const int row0 = (unit_tile(u) / p.n_tok_tiles) * BM;
      const int kb0 = unit_kb0(u), kb1 = unit_kb1(u);
      bool stop = false;
      for (int kb = kb0; kb < kb1 && !stop; ++kb) {
        const int sub = (kb - kb0) % W_SUB;  // which 64-byte column block of the current weight tile
        if (sub == 0 && !mbar_wait(smem_u32(&w_full[ws]), wph, abort_flag, p.status, 4)) break;
        if constexpr (AT) {
          // One weight row per lane (row 32 * (warp % 4) + lane: the warp's TMEM lane quadrant), 32 values per
          // lane per stage: warps 4-7 take values [0, 32) of the stage, warps 8-11 values [32, 64).
          const int g = (warp - 4) >> 2, r = 32 * (warp & 3) + lane;
          const uint8_t* tile = w_st + ws * W_STAGE_BYTES;
          const uint16_t* ssrc = reinterpret_cast<const uint16_t*>(tile + W_TILE_BYTES);
          int4 w0, w1 = make_int4(0, 0, 0, 0);
          if (QT == 8) {  // bytes [64 sub + 32 g, +32) of the row: 128-byte box o >> 7, chunks XOR-swizzled by r % 8
            const int o = sub * 64 + g * 32;
            const uint8_t* rowp = tile + (o >> 7) * (BM * 128) + r * 128;
            const int c0 = (o & 127) >> 4;
            w0 = *reinterpret_cast<const int4*>(rowp + ((c0 ^ (r & 7)) << 4));
            w1 = *reinterpret_cast<const int4*>(rowp + (((c0 + 1) ^ (r & 7)) << 4));
          } else {  // one 16-byte Q4_0 block at byte 32 sub + 16 g of the 128-byte row
            const int c0 = sub * 2 + g;
            w0 = *reinterpret_cast<const int4*>(tile + r * 128 + ((c0 ^ (r & 7)) << 4));
          }
          const __half h = __ushort_as_half(ssrc[r * (W_SUB * BK / QK) + sub * (BK / QK) + g]);
          const __half2 d2 = __halves2half2(h, h);
          if (sub == W_SUB - 1 || kb == kb1 - 1) {  // last use of this tile: release it to the TMA producer
            mbar_arrive(smem_u32(&w_empty[ws]));
            if (++ws == WSTAGES) {
              ws = 0;
              wph ^= 1;
            }
          }
          if (!mbar_wait(smem_u32(&ab_empty[as]), aph ^ 1, abort_flag, p.status, 5)) {
            stop = true;
            break;
          }
          tc_fence_after();  // the MMAs that read this A stage have completed (their commit released it)
          uint32_t hv[16], lv[16];  // column c of the lane's 16 holds values (2c, 2c + 1), low half first
          if (QT == 8) {
            uint4 h0, h1, l0, l1;
            dequant16(w0, d2, h0, h1, l0, l1);
            hv[0] = h0.x, hv[1] = h0.y, hv[2] = h0.z, hv[3] = h0.w, hv[4] = h1.x, hv[5] = h1.y, hv[6] = h1.z, hv[7] = h1.w;
            lv[0] = l0.x, lv[1] = l0.y, lv[2] = l0.z, lv[3] = l0.w, lv[4] = l1.x, lv[5] = l1.y, lv[6] = l1.z, lv[7] = l1.w;
            dequant16(w1, d2, h0, h1, l0, l1);
            hv[8] = h0.x, hv[9] = h0.y, hv[10] = h0.z, hv[11] = h0.w, hv[12] = h1.x, hv[13] = h1.y, hv[14] = h1.z,
            hv[15] = h1.w;
            lv[8] = l0.x, lv[9] = l0.y, lv[10] = l0.z, lv[11] = l0.w, lv[12] = l1.x, lv[13] = l1.y, lv[14] = l1.z,
            lv[15] = l1.w;
          } else {
            uint4 qh[4], ql[4];
            dequant32_q4(w0, d2, qh, ql);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              hv[4 * q] = qh[q].x, hv[4 * q + 1] = qh[q].y, hv[4 * q + 2] = qh[q].z, hv[4 * q + 3] = qh[q].w;
              lv[4 * q] = ql[q].x, lv[4 * q + 1] = ql[q].y, lv[4 * q + 2] = ql[q].z, lv[4 * q + 3] = ql[q].w;
            }
          }
          const uint32_t ta = tmem_base + ((uint32_t)(32 * (warp & 3)) << 16) +
                              (uint32_t)(2 * p.acc_bufs * bn + as * A_TMEM_STAGE_COLS + 16 * g);
          tmem_st16(ta, hv);
          tmem_st16(ta + 32, lv);
          tmem_st_wait();
          tc_fence_before();
          mbar_arrive(smem_u32(&ab_full[as]));
          if (++as == AST) {
            as = 0;
            aph ^= 1;
          }
          continue;
        }
        // Q8_0: DQ_ITEMS items of 16 values (row r, 16-value chunk c); Q4_0: one item of one 32-value block
        // (row r, block b of the stage) per thread.
        constexpr int ITEMS = QT == 8 ? DQ_ITEMS : BM * BK / 32 / DQ_THREADS;
        int4 cw[ITEMS];
        __half2 cd[ITEMS];
        const uint8_t* wsrc = w_st + ws * W_STAGE_BYTES + sub * (QT == 8 ? BK : BK / 2);
        const uint16_t* ssrc = reinterpret_cast<const uint16_t*>(w_st + ws * W_STAGE_BYTES + W_TILE_BYTES);
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
          const int item = tid + DQ_THREADS * j;
          const int r = QT == 8 ? item >> 2 : item >> 1;
          const int c = QT == 8 ? item & 3 : item & 1;  // 16-value chunk (Q8_0) or block (Q4_0) of the stage
          cw[j] = *reinterpret_cast<const int4*>(wsrc + r * w_row_bytes(QT) + c * 16);
          const int blk = QT == 8 ? c >> 1 : c;  // block of this k-stage (two per stage)
          __half h;
          if (p.scale_tma) {
            h = __ushort_as_half(ssrc[r * (W_SUB * BK / QK) + sub * (BK / QK) + blk]);
          } else {  // K not a multiple of 256: scales straight from global memory
            const int row = row0 + r, k = kb * BK + blk * QK;
            h = __ushort_as_half((row < p.N && k < p.K) ? __ldg(p.d + (size_t)row * (p.K / QK) + (k >> 5))
                                                        : (unsigned short)0);
          }
          cd[j] = __halves2half2(h, h);
        }
        if (sub == W_SUB - 1 || kb == kb1 - 1) {  // last use of this tile: release it to the TMA producer
          mbar_arrive(smem_u32(&w_empty[ws]));
          if (++ws == WSTAGES) {
            ws = 0;
            wph ^= 1;
          }
        }
        if (!mbar_wait(smem_u32(&ab_empty[as]), aph ^ 1, abort_flag, p.status, 5)) {
          stop = true;
          break;
        }
        uint8_t* a = a_st + as * A_STAGE_BYTES;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
          const int item = tid + DQ_THREADS * j;
          const int r = QT == 8 ? item >> 2 : item >> 1;
          // row r of the tile: 128-byte line in its 1024-byte group, 16-byte chunks XOR-swizzled by r % 8
          uint8_t* line = a + (r >> 3) * 1024 + (r & 7) * 128;
          if (QT == 8) {
            const int c = item & 3;
            uint4 h0, h1, l0, l1;
            dequant16(cw[j], cd[j], h0, h1, l0, l1);
            const int o0 = ((2 * c) ^ (r & 7)) << 4, o1 = ((2 * c + 1) ^ (r & 7)) << 4;
            *reinterpret_cast<uint4*>(line + o0) = h0;
            *reinterpret_cast<uint4*>(line + o1) = h1;
            *reinterpret_cast<uint4*>(line + A_PLANE_BYTES + o0) = l0;
            *reinterpret_cast<uint4*>(line + A_PLANE_BYTES + o1) = l1;
          } else {
            const int b = item & 1;
            uint4 qh[4], ql[4];
            dequant32_q4(cw[j], cd[j], qh, ql);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              const int o = ((4 * b + q) ^ (r & 7)) << 4;
              *reinterpret_cast<uint4*>(line + o) = qh[q];
              *reinterpret_cast<uint4*>(line + A_PLANE_BYTES + o) = ql[q];
            }
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive(smem_u32(&ab_full[as]));
        if (++as == AST) {
          as = 0;
          aph ^= 1;
        }
      }
    }
  } else if (warp >= EPI_WARP0) {
    // ---------------- epilogue (4 warps -> TMEM lane quadrants warp % 4) ----------------
    pdl_wait();
    const int quad = warp & 3;
    const int row_in_tile = quad * 32 + lane;
    int it = 0;
    for (int u = blockIdx.x; u < n_units && !*abort_flag; u += gridDim.x, ++it) {
      const int acc = it % p.acc_bufs;
      const uint32_t acc_ph = (uint32_t)(it / p.acc_bufs) & 1;
      if (!mbar_wait(smem_u32(&tfull[acc]), acc_ph, abort_flag, p.status, 7)) break;
      tc_fence_after();
      const int t = unit_tile(u);
      const int row = (t / p.n_tok_tiles) * BM + row_in_tile;
      const int tok0 = (t % p.n_tok_tiles) * bn;
      const size_t mn = (size_t)p.M * p.N;
      float* out = p.splits > 1 ? p.part + (size_t)(u % p.splits) * mn : p.y;
      const bool acc_mode = p.splits == 1 && p.accumulate;
      for (int c0 = 0; c0 < bn; c0 += 32) {
        uint32_t r[32];
        uint32_t rl[32];
        const uint32_t tcol = tmem_base + ((uint32_t)(quad * 32) << 16) + (uint32_t)(acc * 2 * bn + c0);
        tmem_ld32(tcol, r);                  // a_hi x_hi + a_lo x_hi
        tmem_ld32(tcol + (uint32_t)bn, rl);  // a_hi x_lo
        if (row < p.N) {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const int m = tok0 + c0 + j;
            if (m < p.M) {
              float* yp = out + (size_t)m * p.N + row;
              const float v = __uint_as_float(r[j]) + __uint_as_float(rl[j]);
              *yp = acc_mode ? *yp + v : v;
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&tempty[acc]));
    }
  }

  // Drain: TMEM is idle once the MMA thread's drain commit flipped (or timed out); free it.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(AT ? (uint32_t)TMEM_COLS : 4u * (uint32_t)bn));
  }
}

// Split-K reduction in a fixed order (deterministic): y (=|+=) sum_s part[s].
__global__ void splitk_reduce_kernel(const float* __restrict__ part, float* __restrict__ y, size_t mn, int splits,
                                     int accumulate) {
  pdl_trigger();
  pdl_wait();
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < mn; i += (size_t)gridDim.x * blockDim.x) {
    float v = part[i];
    for (int s = 1; s < splits; ++s) v += part[(size_t)s * mn + i];
    y[i] = accumulate ? y[i] + v : v;
  }
}

// x [m][k] fp32 -> y [m][hi k | lo k] fp16 with hi = fp16(x), lo = fp16(x - hi).
__global__ void f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y, int m, int k) {
  pdl_trigger();
  pdl_wait();
  const int k4 = k / 4;
  for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < (size_t)m * k4; i += (size_t)gridDim.x * blockDim.x) {
    const size_t r = i / k4, c = i % k4;
    const float4 v = reinterpret_cast<const float4*>(x + r * k)[c];
    __half2 a = __floats2half2_rn(v.x, v.y), b = __floats2half2_rn(v.z, v.w);
    const float2 fa = __half22float2(a), fb = __half22float2(b);
    __half2 la = __floats2half2_rn(v.x - fa.x, v.y - fa.y), lb = __floats2half2_rn(v.z - fb.x, v.w - fb.y);
    __half2* hi = reinterpret_cast<__half2*>(y + r * 2 * k + 4 * c);
    __half2* lo = reinterpret_cast<__half2*>(y + r * 2 * k + k + 4 * c);
    hi[0] = a;
    hi[1] = b;
    lo[0] = la;
    lo[1] = lb;
  }
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

int num_sms() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

struct GemmConfig {
  int bn, splits, kb_per, ab_stages, w_stages, n_tok_tiles, n_tiles;
};

constexpr int SMEM_LIMIT = 232448;  // 227 KB of dynamic shared memory per CTA
constexpr int SMEM_FIXED = 1024 + 512;  // alignment slack + barriers, TMEM slot, abort flag

// Ring depths from the shared-memory budget: the A/B ring (fp16 A + fp16 X per stage) as deep as fits after
// the int8 weight ring, at most MAX_STAGES.  Deep rings keep several stages in flight across the
// dequantize -> MMA -> commit round trip.
static void ring_depths(int qt, int bn, int& ab, int& w) {
  w = bn <= 64 ? 3 : 2;
  if (qt == 4) ++w;  // nibble tiles are half the size
  ab = (SMEM_LIMIT - SMEM_FIXED - w * w_stage_bytes(qt)) / (A_STAGE_BYTES + 2 * bn * BK * 2);
  if (ab > MAX_STAGES) ab = MAX_STAGES;
}

// Ring depths with A in tensor memory: as many A stages as TMEM holds after the accumulators (at most
// MAX_STAGES), the weight ring as deep as shared memory allows (2 .. 4 tiles, 6 for the half-size Q4_0 tiles).
static int acc_bufs_at(int bn) { return bn <= AT_MAX_BN ? 2 : 1; }
static void ring_depths_at(int qt, int bn, int& ab, int& w) {
  ab = std::min(MAX_STAGES, (TMEM_COLS - 2 * acc_bufs_at(bn) * bn) / A_TMEM_STAGE_COLS);
  w = qt == 8 ? 4 : 6;
  while (w > 2 && SMEM_FIXED + ab * 2 * bn * BK * 2 + w * w_stage_bytes(qt) > SMEM_LIMIT) --w;
}

// A tile width is usable when its A/B ring is at least double-buffered (dequantizing one stage while the
// tensor core reads the other).
static bool ring_ok(int qt, int bn) {
  int ab, w;
  ring_depths(qt, bn, ab, w);
  return ab >= 2;
}

// Tile width and split-K for an M x N x K problem.  Cost model: waves of work units on the SMs, each unit
// costing (its k-stages) x (bn + 64) (the 64 stands for the A-operand traffic every stage pays whatever bn
// is), plus a small charge per extra split for the partial-sum traffic.  Split-K only when M <= 128 (small
// decode batches), where the partials are small.
static GemmConfig choose_config(int m, int n, int k, int qt = 8) {
  const int sms = num_sms();
  const int nk = (k + BK - 1) / BK;
  GemmConfig best{};
  double best_cost = 1e30;
  const int bns[4] = {32, 64, 128, 256};
  for (int bn : bns) {
    if (bn > 32 && m <= bn / 2) continue;  // a narrower tile already covers every token
    if (!ring_ok(qt, bn)) continue;
    const int tok_tiles = (m + bn - 1) / bn;
    const int tiles = ((n + BM - 1) / BM) * tok_tiles;
    const int max_s = m <= 128 ? MAX_SPLITS : 1;
    for (int sp = 1; sp <= max_s; ++sp) {
      const int kb_per = ((nk + sp - 1) / sp + W_SUB - 1) / W_SUB * W_SUB;  // whole weight tiles per split
      if (sp > 1 && kb_per < 8) break;
      const int real_sp = (nk + kb_per - 1) / kb_per;
      const int units = tiles * real_sp;
      const int waves = (units + sms - 1) / sms;
      const double cost = (double)waves * kb_per * (bn + 64) + (real_sp > 1 ? 0.02 * real_sp * nk * (bn + 64) : 0.0);
      if (cost < best_cost - 1e-9) {
        best_cost = cost;
        int ab, w;
        ring_depths(qt, bn, ab, w);
        best = GemmConfig{bn, real_sp, kb_per, ab, w, tok_tiles, tiles};
      }
    }
  }
  return best;
}

static size_t align256(size_t b) { return (b + 255) & ~size_t(255); }

// Workspace: [fp16 X][split partials].

}  // namespace

size_t gemm_q8_0_workspace_bytes(int m, int n, int k) {
  const GemmConfig c = choose_config(m, n, k);
  size_t b = align256((size_t)m * k * 4);  // fp16 [m][hi k | lo k]
  // split partials; up to M = 128 (decode batches) room for one even without split-K: gemm_*_tc_h_partials
  // leaves a single-split result there
  if (c.splits > 1 || m <= 128) b += (size_t)std::max(c.splits, 1) * m * n * sizeof(float);
  return b;
}

size_t gemm_workspace_max(int m_max, int n, int k) {
  // split-K is chosen only up to M = 128 (and the partials grow with M there), beyond it the size grows with M
  size_t b = gemm_q8_0_workspace_bytes(std::max(m_max, 1), n, k);
  for (int m = 1; m <= std::min(m_max, 129); ++m) b = std::max(b, gemm_q8_0_workspace_bytes(m, n, k));
  return b;
}

// Core launcher on fp16 activations x16 [m][k] (16-byte aligned rows); QT = 8 (Q8_0) or 4 (Q4_0) weights.
// partials != nullptr: no reduction -- the products stay in the workspace as *nsplit partials [m][n]
// (*partials, one or more, summed in split order by the caller); y and accumulate are then unused.
template <int QT>
static int launch_gemm(const void* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx, float* y,
                       int m, int n, int k, int accumulate, char* ws, int* status, cudaStream_t s,
                       float** partials = nullptr, int* nsplit = nullptr) {
  EncodeTiledFn enc = encode_fn();
  if (!enc) return kCudaError;
  GemmConfig c = choose_config(m, n, k, QT);
  // Block scales [N][K/32] fp16 by TMA, 8 per row per weight tile (needs a 16-byte row pitch: K % 256 == 0).
  const int scale_tma = (k % 256 == 0) ? 1 : 0;
  // A in tensor memory: tiles of up to 64 tokens (double-buffered accumulators), and 128-token Q8_0 tiles with a
  // single accumulator (measured: 512 x 11008 x 4096 140.7 -> 123.9 us; Q4_0 tiles of 128 ran 6 % slower)
  const bool at = (c.bn <= AT_MAX_BN || (c.bn == 128 && QT == 8)) && scale_tma;
  if (at) ring_depths_at(QT, c.bn, c.ab_stages, c.w_stages);
  float* part = reinterpret_cast<float*>(ws + align256((size_t)m * k * 4));
  if (partials) {
    if (m > 128 && c.splits == 1) return kUnsupported;  // no partial space reserved (see the workspace rule)
    *partials = part;
    *nsplit = c.splits;
    if (c.splits == 1) {  // the single split writes its result straight into the partial slot
      y = part;
      accumulate = 0;
    }
  }
  CUtensorMap xmap, xlmap, wmap;
  for (int half = 0; half < 2; ++half) {  // the hi and the lo values of x: [m][k] each, row pitch ldx elements
    cuuint64_t gdim[2] = {(cuuint64_t)k, (cuuint64_t)m};
    cuuint64_t gstride[1] = {(cuuint64_t)ldx * 2};
    cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)c.bn};
    cuuint32_t estride[2] = {1, 1};
    if (enc(half ? &xlmap : &xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(half ? x_lo : x_hi), gdim,
            gstride, box, estride, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return kCudaError;
  }
  // The hi and lo tiles of a stage as one 3-D box (k, token, plane) when the lo values sit a whole number of
  // 16-byte units after the hi ones: one TMA instruction per stage instead of two (each instruction costs the
  // issuing SM a few hundred cycles whatever its size).  Shared memory receives [plane][token][64 k], the layout
  // of the two separate tiles.
  int x_merged = 0;
  CUtensorMap xmap3;
  {
    const long long off = (long long)(x_lo - x_hi);  // elements from a hi value to its lo value
    if (off > 0 && (off * 2) % 16 == 0) {
      cuuint64_t gdim[3] = {(cuuint64_t)k, (cuuint64_t)m, 2};
      cuuint64_t gstride[2] = {(cuuint64_t)ldx * 2, (cuuint64_t)off * 2};
      cuuint32_t box[3] = {(cuuint32_t)BK, (cuuint32_t)c.bn, 2};
      cuuint32_t estride[3] = {1, 1, 1};
      if (enc(&xmap3, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<__half*>(x_hi), gdim, gstride, box, estride,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS) {
        xmap = xmap3;
        x_merged = 1;
      }
    }
  }
  {
    // weight tiles: whole 256- (Q8_0) or 128-byte (Q4_0) rows unswizzled, or with A in TMEM 128-byte boxes
    // with the 128B swizzle (a Q8_0 tile is then two boxes)
    const cuuint64_t row_bytes = QT == 8 ? (cuuint64_t)k : (cuuint64_t)k / 2;
    cuuint64_t gdim[2] = {row_bytes, (cuuint64_t)n};
    cuuint64_t gstride[1] = {row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(at ? 128 : w_row_bytes(QT)), (cuuint32_t)BM};
    cuuint32_t estride[2] = {1, 1};
    if (enc(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(qs), gdim, gstride, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, at ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return kCudaError;
  }

  CUtensorMap smap = wmap;
  if (scale_tma) {
    cuuint64_t gdim[2] = {(cuuint64_t)(k / QK), (cuuint64_t)n};
    cuuint64_t gstride[1] = {(cuuint64_t)(k / QK) * 2};
    cuuint32_t box[2] = {(cuuint32_t)(BK * W_SUB / QK), (cuuint32_t)BM};
    cuuint32_t estride[2] = {1, 1};
    if (enc(&smap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<uint16_t*>(d), gdim, gstride, box, estride,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return kCudaError;
  }

  GemmParams p;
  p.d = d;
  p.scale_tma = scale_tma;
  p.x_merged = x_merged;
  p.acc_bufs = at ? acc_bufs_at(c.bn) : 2;
  p.y = y;
  p.part = part;
  p.status = status;
  p.M = m;
  p.N = n;
  p.K = k;
  p.accumulate = accumulate;
  p.bn = c.bn;
  p.ab_stages = c.ab_stages;
  p.w_stages = c.w_stages;
  p.n_tok_tiles = c.n_tok_tiles;
  p.n_tiles = c.n_tiles;
  p.splits = c.splits;
  p.kb_per_split = c.kb_per;
  const int smem = SMEM_FIXED + c.ab_stages * ((at ? 0 : A_STAGE_BYTES) + 2 * c.bn * BK * 2) +
                   c.w_stages * w_stage_bytes(QT);
  auto kern = at ? gemm_q8_0_tc_kernel<QT, true> : gemm_q8_0_tc_kernel<QT, false>;
  if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) return kCudaError;
  const int grid = std::min(c.n_tiles * c.splits, num_sms());
  if (launch_pdl(kern, dim3(grid), dim3(GEMM_THREADS), (size_t)smem, s, xmap, xlmap, wmap, smap, p) != cudaSuccess)
    return kCudaError;
  if (c.splits > 1 && !partials) {
    const size_t mn = (size_t)m * n;
    if (launch_pdl(splitk_reduce_kernel, dim3((unsigned)std::min<size_t>((mn + 255) / 256, 148 * 8)), dim3(256), 0,
                   s, (const float*)part, y, mn, c.splits, accumulate) != cudaSuccess)
      return kCudaError;
  }
  return kOk;
}

static int check_gemm_args(const void* qs, const void* d, const void* x, const void* y, int m, int n, int k,
                           const void* workspace, size_t workspace_bytes, const int* status) {
  if (!qs || !d || !x || !y || !status || m <= 0 || n <= 0 || k <= 0 || k % QK) return kBadArgument;
  if (k % 16) return kUnsupported;  // TMA row pitches (fp16 activations, int8 weights) must be 16-byte multiples
  if (!workspace || workspace_bytes < gemm_q8_0_workspace_bytes(m, n, k)) return kBadArgument;
  if (reinterpret_cast<uintptr_t>(workspace) & 255 || reinterpret_cast<uintptr_t>(x) & 15 ||
      reinterpret_cast<uintptr_t>(qs) & 15 || reinterpret_cast<uintptr_t>(d) & 15)
    return kUnsupported;
  return kOk;
}

static int convert_x(const float* x, char* ws, int m, int k, cudaStream_t s) {
  const size_t n4 = (size_t)m * k / 4;
  return launch_pdl(f32_to_f16_kernel, dim3((unsigned)std::min<size_t>((n4 + 255) / 256, 148 * 8)), dim3(256), 0, s, x,
                    reinterpret_cast<__half*>(ws), m, k) == cudaSuccess
             ? kOk
             : kCudaError;
}

int gemm_q8_0_tc(const int8_t* qs, const uint16_t* d, const float* x, float* y, int m, int n, int k, int accumulate,
                 void* workspace, size_t workspace_bytes, int* status, cudaStream_t s) {
  const int rc = check_gemm_args(qs, d, x, y, m, n, k, workspace, workspace_bytes, status);
  if (rc != kOk) return rc;
  char* ws = static_cast<char*>(workspace);
  if (convert_x(x, ws, m, k, s) != kOk) return kCudaError;
  const __half* x16 = reinterpret_cast<const __half*>(ws);
  return launch_gemm<8>(qs, d, x16, x16 + k, 2 * k, y, m, n, k, accumulate, ws, status, s);
}

int gemm_q8_0_tc_h(const int8_t* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx, float* y,
                   int m, int n, int k, int accumulate, void* workspace, size_t workspace_bytes, int* status,
                   cudaStream_t s) {
  const int rc = check_gemm_args(qs, d, x_hi, y, m, n, k, workspace, workspace_bytes, status);
  if (rc != kOk) return rc;
  if ((reinterpret_cast<uintptr_t>(x_lo) & 15) || (ldx * 2) % 16) return kUnsupported;
  return launch_gemm<8>(qs, d, x_hi, x_lo, ldx, y, m, n, k, accumulate, static_cast<char*>(workspace), status, s);
}

int gemm_q4_0_tc(const uint8_t* qs, const uint16_t* d, const float* x, float* y, int m, int n, int k, int accumulate,
                 void* workspace, size_t workspace_bytes, int* status, cudaStream_t s) {
  const int rc = check_gemm_args(qs, d, x, y, m, n, k, workspace, workspace_bytes, status);
  if (rc != kOk) return rc;
  if (k % 32) return kUnsupported;  // nibble rows (K / 2 bytes) must be 16-byte multiples
  char* ws = static_cast<char*>(workspace);
  if (convert_x(x, ws, m, k, s) != kOk) return kCudaError;
  const __half* x16 = reinterpret_cast<const __half*>(ws);
  return launch_gemm<4>(qs, d, x16, x16 + k, 2 * k, y, m, n, k, accumulate, ws, status, s);
}

int gemm_q8_0_tc_h_partials(const int8_t* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx,
                            int m, int n, int k, void* workspace, size_t workspace_bytes, int* status, cudaStream_t s,
                            float** partials, int* nsplit) {
  if (!partials || !nsplit) return kBadArgument;
  const int rc = check_gemm_args(qs, d, x_hi, x_hi, m, n, k, workspace, workspace_bytes, status);
  if (rc != kOk) return rc;
  if ((reinterpret_cast<uintptr_t>(x_lo) & 15) || (ldx * 2) % 16) return kUnsupported;
  return launch_gemm<8>(qs, d, x_hi, x_lo, ldx, nullptr, m, n, k, 0, static_cast<char*>(workspace), status, s,
                        partials, nsplit);
}

int gemm_q4_0_tc_h(const uint8_t* qs, const uint16_t* d, const __half* x_hi, const __half* x_lo, int ldx, float* y,
                   int m, int n, int k, int accumulate, void* workspace, size_t workspace_bytes, int* status,
                   cudaStream_t s) {
  const int rc = check_gemm_args(qs, d, x_hi, y, m, n, k, workspace, workspace_bytes, status);
  if (rc != kOk) return rc;
  if ((reinterpret_cast<uintptr_t>(x_lo) & 15) || (ldx * 2) % 16) return kUnsupported;
  return launch_gemm<4>(qs, d, x_hi, x_lo, ldx, y, m, n, k, accumulate, static_cast<char*>(workspace), status, s);
}

}  // namespace zc
