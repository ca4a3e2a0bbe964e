// oracle.cpp -- CPU restatement of ZeroLlm's quantized-linear + paged-KV decode path.
//
// TEST INFRASTRUCTURE ONLY (parity checker and timed CPU baseline); see oracle.h for the
// conventions.  Every function cites the C# it restates (paths relative to the reference root).
// Built with -ffp-contract=off so that only the explicit fmaf / _mm256_fmadd_ps calls fuse,
// exactly where the C# calls Fma.MultiplyAdd.

#include "oracle.h"

#include <immintrin.h>

#include <algorithm>
#include <limits>
#include <atomic>
#include <cmath>
#include <condition_variable>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <mutex>
#include <thread>
#include <vector>

namespace {

// ------------------------------------------------------------------------------------------
// Host thread pool standing in for .NET Parallel.For (dynamic chunked scheduling).
// A parallel_for issued from inside a running region executes serially, as nested
// Parallel.For bodies effectively do once every worker is busy.
// ------------------------------------------------------------------------------------------
class Pool {
 public:
  explicit Pool(int n) : nthreads_(n < 1 ? 1 : n) {
    for (int i = 1; i < nthreads_; ++i) workers_.emplace_back([this] { loop(); });
  }
  ~Pool() {
    {
      std::lock_guard<std::mutex> g(mu_);
      stop_ = true;
      ++gen_;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return nthreads_; }

  void parallel_for(size_t n, size_t grain, int max_threads, const std::function<void(size_t)>& f) {
    if (in_region_ || n <= grain || nthreads_ <= 1 || max_threads == 1) {
      for (size_t i = 0; i < n; ++i) f(i);
      return;
    }
    std::lock_guard<std::mutex> call_guard(call_mu_);
    {
      std::lock_guard<std::mutex> g(mu_);
      job_ = &f;
      n_ = n;
      grain_ = grain < 1 ? 1 : grain;
      next_.store(0);
      pending_ = static_cast<int>(workers_.size());
      ++gen_;
    }
    cv_.notify_all();
    in_region_ = true;
    work();
    in_region_ = false;
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void work() {
    for (;;) {
      size_t begin = next_.fetch_add(grain_);
      if (begin >= n_) return;
      size_t end = std::min(n_, begin + grain_);
      for (size_t i = begin; i < end; ++i) (*job_)(i);
    }
  }
  void loop() {
    in_region_ = true;
    uint64_t seen = 0;
    for (;;) {
      std::unique_lock<std::mutex> lk(mu_);
      cv_.wait(lk, [&] { return gen_ != seen; });
      seen = gen_;
      if (stop_) return;
      lk.unlock();
      work();
      lk.lock();
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }

  int nthreads_;
  std::vector<std::thread> workers_;
  std::mutex mu_, call_mu_;
  std::condition_variable cv_, done_cv_;
  const std::function<void(size_t)>* job_ = nullptr;
  size_t n_ = 0, grain_ = 1;
  std::atomic<size_t> next_{0};
  int pending_ = 0;
  uint64_t gen_ = 0;
  bool stop_ = false;
  static thread_local bool in_region_;
};
thread_local bool Pool::in_region_ = false;

Pool& pool() {
  static Pool p([] {
    const char* env = std::getenv("ORC_THREADS");
    int n = env ? std::atoi(env) : 0;
    if (n <= 0) n = static_cast<int>(std::thread::hardware_concurrency());
    return n < 1 ? 1 : n;
  }());
  return p;
}

// .NET 8 Vector256<float>.Sum on AVX: lower128 + upper128, then two horizontal adds.
inline float net_sum256(__m256 v) {
  __m128 lo = _mm256_castps256_ps128(v);
  __m128 hi = _mm256_extractf128_ps(v, 1);
  __m128 a = _mm_add_ps(lo, hi);
  a = _mm_hadd_ps(a, a);
  a = _mm_hadd_ps(a, a);
  return _mm_cvtss_f32(a);
}

// .NET 8 Vector.Dot(Vector<float>, Vector<float>) on AVX: per-128-bit-lane dpps, then lower + upper.
inline float net_dot256(__m256 a, __m256 b) {
  __m256 d = _mm256_dp_ps(a, b, 0xF1);
  return _mm_cvtss_f32(_mm256_castps256_ps128(d)) + _mm_cvtss_f32(_mm256_extractf128_ps(d, 1));
}

constexpr int QK = 32;
constexpr size_t Q8_BYTES = 34;
constexpr size_t Q4_BYTES = 18;

inline float block_scale(const uint8_t* blk) {
  uint16_t h;
  std::memcpy(&h, blk, 2);
  return orc_f16_to_f32(h);
}

}  // namespace

extern "C" {

// ---- HalfHelper (HalfHelper.cs:13-75; .NET 8 branch = IEEE binary16, round to nearest even) ----
uint16_t orc_f32_to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) {  // inf / nan
    if (ax > 0x7f800000u) return static_cast<uint16_t>(sign | 0x7e00u | ((ax >> 13) & 0x3ffu));
    return static_cast<uint16_t>(sign | 0x7c00u);
  }
  if (ax >= 0x477ff000u) return static_cast<uint16_t>(sign | 0x7c00u);  // >= 65520 rounds to inf
  if (ax >= 0x38800000u) {                                              // normal binary16 range
    uint32_t mant = ax & 0x7fffffu;
    uint32_t exp = (ax >> 23) - 127 + 15;
    uint32_t h = (exp << 10) | (mant >> 13);
    uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;  // carries into the exponent correctly
    return static_cast<uint16_t>(sign | h);
  }
  // Subnormal binary16 (or zero): count of 2^-24 units, rounded half-to-even. The scaling is exact.
  float a;
  std::memcpy(&a, &ax, 4);
  uint32_t h = static_cast<uint32_t>(std::rint(a * 16777216.0f));
  return static_cast<uint16_t>(sign | h);
}

float orc_f16_to_f32(uint16_t h) {
  uint32_t sign = static_cast<uint32_t>(h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1fu;
  uint32_t mant = h & 0x3ffu;
  uint32_t out;
  if (exp == 0) {
    if (mant == 0) {
      out = sign;
    } else {  // subnormal: mant * 2^-24, exact in binary32
      float v = static_cast<float>(mant) * (1.0f / 16777216.0f);
      std::memcpy(&out, &v, 4);
      out |= sign;
    }
  } else if (exp == 31) {
    out = sign | 0x7f800000u | (mant << 13);
  } else {
    out = sign | ((exp - 15 + 127) << 23) | (mant << 13);
  }
  float f;
  std::memcpy(&f, &out, 4);
  return f;
}

void orc_f32_to_f16_array(const float* src, uint16_t* dst, size_t n) {
  for (size_t i = 0; i < n; ++i) dst[i] = orc_f32_to_f16(src[i]);
}

// ---- BlockQ8_0.Quantize (BlockQ8_0.cs:43-71) via LlmQuantizer.QuantizeToQ8_0 (LlmQuantizer.cs:20-36) ----
void orc_quantize_q8_0(const float* src, size_t n, uint8_t* dst) {
  size_t nb = n / QK;
  for (size_t b = 0; b < nb; ++b) {
    const float* s = src + b * QK;
    uint8_t* blk = dst + b * Q8_BYTES;
    float amax = 0.0f;
    for (int i = 0; i < QK; ++i) {
      float v = std::fabs(s[i]);
      if (v > amax) amax = v;
    }
    float d = amax / 127.0f;
    float id = d > 1e-15f ? 1.0f / d : 0.0f;
    uint16_t hd = orc_f32_to_f16(d);
    std::memcpy(blk, &hd, 2);
    for (int i = 0; i < QK; ++i) {
      float v0 = s[i] * id;
      int q = static_cast<int>(std::rint(static_cast<double>(v0)));
      if (q > 127) q = 127;
      if (q < -127) q = -127;
      blk[2 + i] = static_cast<uint8_t>(static_cast<int8_t>(q));
    }
  }
}

// ---- BlockQ4_0.Quantize (BlockQ4_0.cs:47-76) via LlmQuantizer.QuantizeToQ4_0 (LlmQuantizer.cs:42-57) ----
void orc_quantize_q4_0(const float* src, size_t n, uint8_t* dst) {
  size_t nb = n / QK;
  for (size_t b = 0; b < nb; ++b) {
    const float* s = src + b * QK;
    uint8_t* blk = dst + b * Q4_BYTES;
    float amax = 0.0f;
    for (int i = 0; i < QK; ++i) {
      float v = std::fabs(s[i]);
      if (v > amax) amax = v;
    }
    float d = amax / 8.0f;
    float id = d != 0.0f ? 1.0f / d : 0.0f;
    uint16_t hd = orc_f32_to_f16(d);
    std::memcpy(blk, &hd, 2);
    for (int i = 0; i < 16; ++i) {
      float x0 = s[i] * id;
      float x1 = s[i + 16] * id;
      double r0 = std::rint(static_cast<double>(x0)) + 8.0;
      double r1 = std::rint(static_cast<double>(x1)) + 8.0;
      int q0 = static_cast<int>(std::min(15.0, std::max(0.0, r0)));
      int q1 = static_cast<int>(std::min(15.0, std::max(0.0, r1)));
      blk[2 + i] = static_cast<uint8_t>((q0 & 0x0F) | ((q1 & 0x0F) << 4));
    }
  }
}

// ---- BlockQ8_0.Dequantize (BlockQ8_0.cs:25-38) ----
void orc_dequantize_q8_0(const uint8_t* blocks, size_t n, float* dst) {
  for (size_t b = 0; b < n / QK; ++b) {
    const uint8_t* blk = blocks + b * Q8_BYTES;
    float d = block_scale(blk);
    for (int i = 0; i < QK; ++i) dst[b * QK + i] = static_cast<float>(static_cast<int8_t>(blk[2 + i])) * d;
  }
}

// ---- BlockQ4_0.Dequantize (BlockQ4_0.cs:25-42) ----
void orc_dequantize_q4_0(const uint8_t* blocks, size_t n, float* dst) {
  for (size_t b = 0; b < n / QK; ++b) {
    const uint8_t* blk = blocks + b * Q4_BYTES;
    float d = block_scale(blk);
    for (int i = 0; i < 16; ++i) {
      uint8_t v = blk[2 + i];
      dst[b * QK + i] = static_cast<float>((v & 0x0F) - 8) * d;
      dst[b * QK + i + 16] = static_cast<float>((v >> 4) - 8) * d;
    }
  }
}

// ---- QuantizedKernels.DotProductQ8_0 (QuantizedKernels.cs:21-78) ----
float orc_dot_q8_0(const float* x, const uint8_t* w, size_t nblocks, int path) {
  float total = 0.0f;
  if (path == 0) {  // AVX2/FMA branch (:26-53)
    for (size_t b = 0; b < nblocks; ++b) {
      const uint8_t* blk = w + b * Q8_BYTES;
      float scale = block_scale(blk);
      const float* bx = x + b * QK;
      const int8_t* qs = reinterpret_cast<const int8_t*>(blk + 2);
      __m128i r0, r1, r2, r3;
      std::memcpy(&r0, qs, 8);
      std::memcpy(&r1, qs + 8, 8);
      std::memcpy(&r2, qs + 16, 8);
      std::memcpy(&r3, qs + 24, 8);
      __m256 w0 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(r0));
      __m256 w1 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(r1));
      __m256 w2 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(r2));
      __m256 w3 = _mm256_cvtepi32_ps(_mm256_cvtepi8_epi32(r3));
      __m256 d0 = _mm256_mul_ps(w0, _mm256_loadu_ps(bx));
      __m256 d1 = _mm256_mul_ps(w1, _mm256_loadu_ps(bx + 8));
      __m256 d2 = _mm256_fmadd_ps(w2, _mm256_loadu_ps(bx + 16), d0);
      __m256 d3 = _mm256_fmadd_ps(w3, _mm256_loadu_ps(bx + 24), d1);
      total += net_sum256(_mm256_add_ps(d2, d3)) * scale;
    }
    return total;
  }
  for (size_t b = 0; b < nblocks; ++b) {  // scalar branch (:56-77)
    const uint8_t* blk = w + b * Q8_BYTES;
    float scale = block_scale(blk);
    const float* bx = x + b * QK;
    const int8_t* q = reinterpret_cast<const int8_t*>(blk + 2);
    float s[4];
    for (int g = 0; g < 4; ++g) {
      const float* xx = bx + 8 * g;
      const int8_t* qq = q + 8 * g;
      float acc = xx[0] * qq[0];
      for (int i = 1; i < 8; ++i) acc = acc + xx[i] * qq[i];
      s[g] = acc;
    }
    total += ((s[0] + s[1]) + (s[2] + s[3])) * scale;
  }
  return total;
}

// ---- QuantizedKernels.DotProductQ4_0 (QuantizedKernels.cs:101-168) ----
float orc_dot_q4_0(const float* x, const uint8_t* w, size_t nblocks, int path) {
  float total = 0.0f;
  if (path == 0) {  // AVX2/FMA branch (:106-135)
    const __m256i mask = _mm256_set1_epi32(0x0F);
    const __m256i off = _mm256_set1_epi32(8);
    for (size_t b = 0; b < nblocks; ++b) {
      const uint8_t* blk = w + b * Q4_BYTES;
      float scale = block_scale(blk);
      const float* bx = x + b * QK;
      const uint8_t* qs = blk + 2;
      __m128i a0, a1;
      std::memcpy(&a0, qs, 8);
      std::memcpy(&a1, qs + 8, 8);
      __m256i raw0 = _mm256_cvtepu8_epi32(a0);
      __m256i raw1 = _mm256_cvtepu8_epi32(a1);
      __m256 w00 = _mm256_cvtepi32_ps(_mm256_sub_epi32(_mm256_and_si256(raw0, mask), off));
      __m256 w10 = _mm256_cvtepi32_ps(_mm256_sub_epi32(_mm256_and_si256(_mm256_srli_epi32(raw0, 4), mask), off));
      __m256 w01 = _mm256_cvtepi32_ps(_mm256_sub_epi32(_mm256_and_si256(raw1, mask), off));
      __m256 w11 = _mm256_cvtepi32_ps(_mm256_sub_epi32(_mm256_and_si256(_mm256_srli_epi32(raw1, 4), mask), off));
      __m256 d0 = _mm256_mul_ps(w00, _mm256_loadu_ps(bx));
      __m256 d1 = _mm256_mul_ps(w01, _mm256_loadu_ps(bx + 8));
      __m256 d2 = _mm256_fmadd_ps(w10, _mm256_loadu_ps(bx + 16), d0);
      __m256 d3 = _mm256_fmadd_ps(w11, _mm256_loadu_ps(bx + 24), d1);
      total += net_sum256(_mm256_add_ps(d2, d3)) * scale;
    }
    return total;
  }
  for (size_t b = 0; b < nblocks; ++b) {  // scalar branch (:138-167)
    const uint8_t* blk = w + b * Q4_BYTES;
    float scale = block_scale(blk);
    const float* bx = x + b * QK;
    const uint8_t* q = blk + 2;
    float s[4];
    for (int g = 0; g < 4; ++g) {
      float acc = 0.0f;
      for (int j = 0; j < 4; ++j) {
        int i = 4 * g + j;
        float lo = bx[i] * static_cast<float>((q[i] & 0x0F) - 8);
        float hi = bx[i + 16] * static_cast<float>((q[i] >> 4) - 8);
        acc = (j == 0) ? (lo + hi) : (acc + lo) + hi;
      }
      s[g] = acc;
    }
    total += ((s[0] + s[1]) + (s[2] + s[3])) * scale;
  }
  return total;
}

// ---- MatVecMulQ8_0 / MatVecAddQ8_0 / ...Q4_0 (QuantizedKernels.cs:190-349) ----
static void matvec_impl(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols, int accumulate,
                        int threads, bool q8) {
  size_t bpr = cols / QK;
  size_t row_bytes = bpr * (q8 ? Q8_BYTES : Q4_BYTES);
  auto body = [&](size_t r) {
    const uint8_t* wr = w + r * row_bytes;
    float v = q8 ? orc_dot_q8_0(x, wr, bpr, 0) : orc_dot_q4_0(x, wr, bpr, 0);
    if (accumulate)
      y[r] += v;
    else
      y[r] = v;
  };
  if (rows >= 1024)
    pool().parallel_for(rows, 16, threads, body);
  else
    for (size_t r = 0; r < rows; ++r) body(r);
}

void orc_matvec_q8_0(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols, int accumulate,
                     int threads) {
  matvec_impl(w, x, y, rows, cols, accumulate, threads, true);
}
void orc_matvec_q4_0(const uint8_t* w, const float* x, float* y, size_t rows, size_t cols, int accumulate,
                     int threads) {
  matvec_impl(w, x, y, rows, cols, accumulate, threads, false);
}

static void matmul_impl(const uint8_t* w, const float* x, float* y, size_t m, size_t rows, size_t cols,
                        int accumulate, int threads, bool q8) {
  pool().parallel_for(m, 1, threads, [&](size_t t) {
    matvec_impl(w, x + t * cols, y + t * rows, rows, cols, accumulate, 1, q8);
  });
}
void orc_matmul_q8_0(const uint8_t* w, const float* x, float* y, size_t m, size_t rows, size_t cols, int accumulate,
                     int threads) {
  matmul_impl(w, x, y, m, rows, cols, accumulate, threads, true);
}
void orc_matmul_q4_0(const uint8_t* w, const float* x, float* y, size_t m, size_t rows, size_t cols, int accumulate,
                     int threads) {
  matmul_impl(w, x, y, m, rows, cols, accumulate, threads, false);
}

// ---- TensorBlas.GemmInt8 (TensorBlas.Quantized.cs:39-154): int32 accumulation, same sum ----
void orc_gemm_i8(const int8_t* a, const int8_t* b, int32_t* c, size_t m, size_t n, size_t k) {
  std::memset(c, 0, m * n * sizeof(int32_t));
  pool().parallel_for(m, 1, 0, [&](size_t i) {
    for (size_t p = 0; p < k; ++p) {
      int32_t av = a[i * k + p];
      if (av == 0) continue;
      for (size_t j = 0; j < n; ++j) c[i * n + j] += av * static_cast<int32_t>(b[p * n + j]);
    }
  });
}

int32_t orc_dot_i8(const int8_t* a, const int8_t* b, size_t n) {
  int32_t s = 0;
  for (size_t i = 0; i < n; ++i) s += static_cast<int32_t>(a[i]) * static_cast<int32_t>(b[i]);
  return s;
}

void orc_block_dots_i8(const int8_t* xq, const uint8_t* w, int32_t* p, size_t m, size_t rows, size_t cols) {
  size_t bpr = cols / QK;
  pool().parallel_for(m, 1, 0, [&](size_t t) {
    for (size_t r = 0; r < rows; ++r)
      for (size_t b = 0; b < bpr; ++b) {
        const int8_t* q = reinterpret_cast<const int8_t*>(w + (r * bpr + b) * Q8_BYTES + 2);
        const int8_t* xx = xq + t * cols + b * QK;
        int32_t s = 0;
        for (int i = 0; i < QK; ++i) s += static_cast<int32_t>(xx[i]) * static_cast<int32_t>(q[i]);
        p[(t * rows + r) * bpr + b] = s;
      }
  });
}

// ---- LlmEngine.DotProductSimd (LlmEngine.cs:463-500), Vector<float> = 8 lanes ----
float orc_dot_f32(const float* a, const float* b, int len) {
  const int vs = 8, step4 = 32;
  int limit4 = len - (len % step4);
  int limit1 = len - (len % vs);
  __m256 acc0 = _mm256_setzero_ps(), acc1 = acc0, acc2 = acc0, acc3 = acc0;
  int i = 0;
  for (; i < limit4; i += step4) {
    acc0 = _mm256_add_ps(acc0, _mm256_mul_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i)));
    acc1 = _mm256_add_ps(acc1, _mm256_mul_ps(_mm256_loadu_ps(a + i + 8), _mm256_loadu_ps(b + i + 8)));
    acc2 = _mm256_add_ps(acc2, _mm256_mul_ps(_mm256_loadu_ps(a + i + 16), _mm256_loadu_ps(b + i + 16)));
    acc3 = _mm256_add_ps(acc3, _mm256_mul_ps(_mm256_loadu_ps(a + i + 24), _mm256_loadu_ps(b + i + 24)));
  }
  acc0 = _mm256_add_ps(_mm256_add_ps(acc0, acc1), _mm256_add_ps(acc2, acc3));
  for (; i < limit1; i += vs) acc0 = _mm256_add_ps(acc0, _mm256_mul_ps(_mm256_loadu_ps(a + i), _mm256_loadu_ps(b + i)));
  float sum = net_dot256(acc0, _mm256_set1_ps(1.0f));
  for (; i < len; ++i) sum += a[i] * b[i];
  return sum;
}

// ---- RmsNorm.Forward (RmsNorm.cs:14-59) ----
void orc_rmsnorm(const float* x, const float* w, float* out, size_t n, float eps) {
  size_t simd = n - (n % 8);
  __m256 ss = _mm256_setzero_ps();
  for (size_t i = 0; i < simd; i += 8) {
    __m256 v = _mm256_loadu_ps(x + i);
    ss = _mm256_add_ps(ss, _mm256_mul_ps(v, v));
  }
  float sum_sq = net_dot256(ss, _mm256_set1_ps(1.0f));
  for (size_t i = simd; i < n; ++i) sum_sq += x[i] * x[i];
  float mean_sq = sum_sq / static_cast<float>(n);
  float inv_rms = 1.0f / static_cast<float>(std::sqrt(static_cast<double>(mean_sq + eps)));
  for (size_t i = 0; i < n; ++i) out[i] = x[i] * inv_rms * w[i];
}

// ---- RoPE.EnsureCache (RoPE.cs:83-125) ----
void orc_rope_table(int max_pos, int head_dim, float freq_base, float* cos_t, float* sin_t) {
  int half = head_dim / 2;
  std::vector<double> freqs(half);
  for (int i = 0; i < half; ++i) {
    double exponent = 2.0 * i / head_dim;
    freqs[i] = 1.0 / std::pow(static_cast<double>(freq_base), exponent);
  }
  for (int p = 0; p < max_pos; ++p)
    for (int i = 0; i < half; ++i) {
      double theta = p * freqs[i];
      cos_t[static_cast<size_t>(p) * half + i] = static_cast<float>(std::cos(theta));
      sin_t[static_cast<size_t>(p) * half + i] = static_cast<float>(std::sin(theta));
    }
}

// ---- RoPE.ApplyInplace (RoPE.cs:131-163), table path ----
void orc_rope_apply(float* v, int pos, int head_dim, const float* cos_t, const float* sin_t) {
  int half = head_dim / 2;
  const float* c = cos_t + static_cast<size_t>(pos) * half;
  const float* s = sin_t + static_cast<size_t>(pos) * half;
  for (int i = 0; i < half; ++i) {
    float x0 = v[2 * i], x1 = v[2 * i + 1];
    v[2 * i] = x0 * c[i] - x1 * s[i];
    v[2 * i + 1] = x0 * s[i] + x1 * c[i];
  }
}

// ---- SwiGLU.Forward (SwiGLU.cs:13-51) ----
void orc_swiglu(const float* gate, const float* up, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    float g = gate[i];
    float s = 1.0f / (1.0f + static_cast<float>(std::exp(-static_cast<double>(g))));
    out[i] = (g * s) * up[i];
  }
}

// ---- GqaAttention.Forward (GqaAttention.cs:29-130) ----
void orc_gqa_attention(const float* q, const float* kpool, const float* vpool, const int32_t* page_table,
                       int page_size, size_t page_stride, int seq_len, int hq, int hkv, int hd, float* out) {
  if (seq_len <= 0) {
    std::memset(out, 0, sizeof(float) * static_cast<size_t>(hq) * hd);
    return;
  }
  int group = hq / hkv;
  float scale = 1.0f / static_cast<float>(std::sqrt(static_cast<double>(hd)));
  size_t token_stride = static_cast<size_t>(hkv) * hd;
  std::vector<float> scores(seq_len);
  int simd = hd - (hd % 8);
  auto row = [&](const float* pool_base, int t) {
    return pool_base + static_cast<size_t>(page_table[t / page_size]) * page_stride +
           static_cast<size_t>(t % page_size) * token_stride;
  };
  for (int qh = 0; qh < hq; ++qh) {
    int kvh = qh / group;
    const float* qv = q + static_cast<size_t>(qh) * hd;
    float* o = out + static_cast<size_t>(qh) * hd;
    std::memset(o, 0, sizeof(float) * hd);
    float max_score = -INFINITY;
    for (int t = 0; t < seq_len; ++t) {
      float dot = orc_dot_f32(qv, row(kpool, t) + static_cast<size_t>(kvh) * hd, hd);
      float s = dot * scale;
      scores[t] = s;
      if (s > max_score) max_score = s;
    }
    float sum_exp = 0.0f;
    for (int t = 0; t < seq_len; ++t) {
      float e = static_cast<float>(std::exp(static_cast<double>(scores[t] - max_score)));
      scores[t] = e;
      sum_exp += e;
    }
    float inv_sum = sum_exp > 0 ? 1.0f / sum_exp : 0.0f;
    for (int t = 0; t < seq_len; ++t) {
      float weight = scores[t] * inv_sum;
      if (weight <= 0.0f) continue;
      const float* vv = row(vpool, t) + static_cast<size_t>(kvh) * hd;
      for (int d = 0; d < simd; ++d) o[d] += weight * vv[d];
      for (int d = simd; d < hd; ++d) o[d] += weight * vv[d];
    }
  }
}

// ---- TensorOps.FlashAttentionCpu (TensorOps.Neural.cs:983-1180; row kernel :670-975) ----
void orc_flash_attention(size_t batch, int sq, int sk, int d, int dv, float scale, int is_gqa, int hq, int hkv,
                         int group, const float* q, const float* k, const float* v, const float* mask,
                         size_t mask_batches, float* out) {
  const int kBc = 32;
  const size_t mask_stride = static_cast<size_t>(sq) * sk;
  auto row = [&](size_t b, int i) {
    const size_t bkv = is_gqa ? (b / hq) * hkv + (b % hq) / group : b;
    const float* qi = q + (b * sq + i) * static_cast<size_t>(d);
    const float* kb = k + bkv * static_cast<size_t>(sk) * d;
    const float* vb = v + bkv * static_cast<size_t>(sk) * dv;
    const float* mrow =
        mask ? mask + (mask_stride > 0 ? (b % mask_batches) * mask_stride + static_cast<size_t>(i) * sk : 0) : nullptr;
    float* o = out + (b * sq + i) * static_cast<size_t>(dv);
    std::vector<float> acc(dv, 0.0f);
    float scores[kBc], weights[kBc];
    float max_score = -INFINITY, sum_exp = 0.0f;
    for (int j0 = 0; j0 < sk; j0 += kBc) {
      const int n = std::min(kBc, sk - j0);
      for (int t = 0; t < n; ++t) scores[t] = orc_dot_f32(qi, kb + static_cast<size_t>(j0 + t) * d, d) * scale;
      if (mrow)
        for (int t = 0; t < n; ++t) scores[t] += mrow[j0 + t];
      float m_block = -INFINITY;
      for (int t = 0; t < n; ++t)
        if (scores[t] > m_block) m_block = scores[t];
      if (m_block == -INFINITY) continue;
      float l_block = 0.0f;
      for (int t = 0; t < n; ++t) {
        if (scores[t] == -INFINITY) {
          weights[t] = 0.0f;
        } else {
          weights[t] = static_cast<float>(std::exp(static_cast<double>(scores[t] - m_block)));
          l_block += weights[t];
        }
      }
      const float m_new = std::max(max_score, m_block);
      const float alpha =
          max_score == -INFINITY ? 0.0f : static_cast<float>(std::exp(static_cast<double>(max_score - m_new)));
      const float beta = static_cast<float>(std::exp(static_cast<double>(m_block - m_new)));
      sum_exp = sum_exp * alpha + l_block * beta;
      max_score = m_new;
      if (alpha != 1.0f)
        for (int c = 0; c < dv; ++c) acc[c] *= alpha;
      for (int t = 0; t < n; ++t) {
        const float w = weights[t] * beta;
        if (w == 0.0f) continue;
        const float* vt = vb + static_cast<size_t>(j0 + t) * dv;
        for (int c = 0; c < dv; ++c) acc[c] = std::fmaf(w, vt[c], acc[c]);
      }
    }
    const float inv = sum_exp > 0.0f ? 1.0f / sum_exp : 0.0f;
    for (int c = 0; c < dv; ++c) o[c] = acc[c] * inv;
  };
  pool().parallel_for(batch * sq, 1, 0, [&](size_t r) { row(r / sq, static_cast<int>(r % sq)); });
}

// ---- TensorOps.PagedAttention fallback (TensorOps.Neural.cs:2418-2473) ----
void orc_paged_attention(const float* q, const float* kc, const float* vc, const int32_t* block_table, int hq,
                         int hkv, int hd, int block_size, int context_len, float scale, float* out) {
  int ratio = hq / hkv;
  int nlb = (context_len + block_size - 1) / block_size;
  for (int h = 0; h < hq; ++h) {
    int kvh = h / ratio;
    const float* qh = q + static_cast<size_t>(h) * hd;
    float* oh = out + static_cast<size_t>(h) * hd;
    for (int d = 0; d < hd; ++d) oh[d] = 0.0f;
    float m_prev = -INFINITY, l_prev = 0.0f;
    for (int lb = 0; lb < nlb; ++lb) {
      int phys = block_table[lb];
      int tib = std::min(block_size, context_len - lb * block_size);
      for (int bo = 0; bo < tib; ++bo) {
        size_t off = ((static_cast<size_t>(phys) * block_size + bo) * hkv + kvh) * hd;
        const float* kv = kc + off;
        const float* vv = vc + off;
        float dot = 0.0f;
        for (int d = 0; d < hd; ++d) dot += qh[d] * kv[d];
        float score = dot * scale;
        float m_cur = std::max(m_prev, score);
        float alpha = static_cast<float>(std::exp(static_cast<double>(m_prev - m_cur)));
        float beta = static_cast<float>(std::exp(static_cast<double>(score - m_cur)));
        l_prev = l_prev * alpha + beta;
        for (int d = 0; d < hd; ++d) oh[d] = oh[d] * alpha + beta * vv[d];
        m_prev = m_cur;
      }
    }
    if (l_prev > 0.0f) {
      float inv = 1.0f / l_prev;
      for (int d = 0; d < hd; ++d) oh[d] *= inv;
    }
  }
}

// ---- SparseMoeLayer.Forward (SparseMoeLayer.cs:32-125, SelectTopK :159-182, ComputeSoftmax :184-219) ----
void orc_moe_forward(const float* xnorm, const float* router_w, const float* router_logits, int n_experts, int top_k,
                     int qtype, const uint8_t* eg, const uint8_t* eu, const uint8_t* ed, int dim, int ffn,
                     float* residual, int32_t* sel_idx, float* sel_w) {
  if (n_experts <= 0) return;
  int k = std::min(std::max(1, top_k), n_experts);
  std::vector<float> logits(n_experts);
  if (router_logits) {
    for (int e = 0; e < n_experts; ++e) logits[e] = router_logits[e];
  } else if (router_w) {
    for (int e = 0; e < n_experts; ++e) logits[e] = orc_dot_f32(xnorm, router_w + static_cast<size_t>(e) * dim, dim);
  } else {
    for (int e = 0; e < n_experts; ++e) logits[e] = 0.0f;
  }
  std::vector<int> idx(k);
  std::vector<float> wts(k);
  std::vector<char> picked(n_experts, 0);
  for (int i = 0; i < k; ++i) {
    float max_val = -3.40282347e38f;  // float.MinValue
    int max_idx = 0;
    for (int j = 0; j < n_experts; ++j)
      if (!picked[j] && logits[j] > max_val) {
        max_val = logits[j];
        max_idx = j;
      }
    picked[max_idx] = 1;
    idx[i] = max_idx;
    wts[i] = max_val;
  }
  {
    float mx = wts[0];
    for (int i = 1; i < k; ++i)
      if (wts[i] > mx) mx = wts[i];
    float sum = 0.0f;
    for (int i = 0; i < k; ++i) {
      float e = static_cast<float>(std::exp(static_cast<double>(wts[i] - mx)));
      wts[i] = e;
      sum += e;
    }
    if (sum > 1e-12f) {
      float inv = 1.0f / sum;
      for (int i = 0; i < k; ++i) wts[i] *= inv;
    } else {
      for (int i = 0; i < k; ++i) wts[i] = 1.0f / k;
    }
  }
  size_t blk = qtype == 8 ? Q8_BYTES : Q4_BYTES;
  size_t up_bytes = static_cast<size_t>(ffn) * (dim / QK) * blk;
  size_t down_bytes = static_cast<size_t>(dim) * (ffn / QK) * blk;
  std::vector<float> gate(ffn), up(ffn), sw(ffn), down(dim);
  for (int i = 0; i < k; ++i) {
    if (sel_idx) sel_idx[i] = idx[i];
    if (sel_w) sel_w[i] = wts[i];
    int e = idx[i];
    float w = wts[i];
    if (e < 0 || e >= n_experts || std::fabs(w) < 1e-7f) continue;
    if (qtype == 8) {
      orc_matvec_q8_0(eg + e * up_bytes, xnorm, gate.data(), ffn, dim, 0, 0);
      orc_matvec_q8_0(eu + e * up_bytes, xnorm, up.data(), ffn, dim, 0, 0);
      orc_swiglu(gate.data(), up.data(), sw.data(), ffn);
      orc_matvec_q8_0(ed + e * down_bytes, sw.data(), down.data(), dim, ffn, 0, 0);
    } else {
      orc_matvec_q4_0(eg + e * up_bytes, xnorm, gate.data(), ffn, dim, 0, 0);
      orc_matvec_q4_0(eu + e * up_bytes, xnorm, up.data(), ffn, dim, 0, 0);
      orc_swiglu(gate.data(), up.data(), sw.data(), ffn);
      orc_matvec_q4_0(ed + e * down_bytes, sw.data(), down.data(), dim, ffn, 0, 0);
    }
    for (int d = 0; d < dim; ++d) residual[d] += w * down[d];  // AddWeightedResidual (:247-264)
  }
}

// ---- LlmSampler.Sample greedy branch (LlmSampler.cs:21-72) ----
int32_t orc_sample_greedy(float* logits, size_t vocab, const int32_t* past, size_t n_past, float penalty) {
  if (penalty > 1.0f && n_past > 0) {
    for (size_t i = 0; i < n_past; ++i) {
      uint32_t tok = static_cast<uint32_t>(past[i]);
      if (tok < vocab) {
        if (logits[tok] > 0)
          logits[tok] /= penalty;
        else
          logits[tok] *= penalty;
      }
    }
  }
  size_t best = 0;
  float best_val = logits[0];
  for (size_t i = 1; i < vocab; ++i)
    if (logits[i] > best_val) {
      best_val = logits[i];
      best = i;
    }
  return static_cast<int32_t>(best);
}

// ---- LlmSampler.Sample, all branches (LlmSampler.cs:21-172), the random draw given as u ----
int32_t orc_sample(float* logits, size_t vocab, const int32_t* past, size_t n_past, float temperature, float top_p,
                   float min_p, int32_t top_k, float penalty, float u, int32_t* cand_idx, float* cand_p,
                   int32_t* n_cand, int32_t cap) {
  if (n_cand) *n_cand = 0;
  if (vocab == 0) return 0;
  if (penalty > 1.0f && n_past > 0) {  // 1. repetition penalty, occurrence by occurrence (:39-57)
    for (size_t i = 0; i < n_past; ++i) {
      uint32_t tok = static_cast<uint32_t>(past[i]);
      if (tok < vocab) {
        if (logits[tok] > 0)
          logits[tok] /= penalty;
        else
          logits[tok] *= penalty;
      }
    }
  }
  if (temperature <= 0.001f || top_k == 1) {  // 2. greedy (:60-73)
    size_t best = 0;
    float best_val = logits[0];
    for (size_t i = 1; i < vocab; ++i)
      if (logits[i] > best_val) {
        best_val = logits[i];
        best = i;
      }
    return static_cast<int32_t>(best);
  }
  const float inv_temp = 1.0f / temperature;  // 3. temperature (:76-80)
  for (size_t i = 0; i < vocab; ++i) logits[i] *= inv_temp;
  float max_logit = -std::numeric_limits<float>::infinity();  // 4. softmax (:83-101)
  for (size_t i = 0; i < vocab; ++i)
    if (logits[i] > max_logit) max_logit = logits[i];
  float sum_exp = 0.0f;
  for (size_t i = 0; i < vocab; ++i) {
    const float e = static_cast<float>(std::exp(static_cast<double>(logits[i] - max_logit)));
    logits[i] = e;
    sum_exp += e;
  }
  const float inv_sum = sum_exp > 0 ? 1.0f / sum_exp : 0.0f;
  for (size_t i = 0; i < vocab; ++i) logits[i] *= inv_sum;
  std::vector<std::pair<int, float>> cand;  // 5. candidates p > 1e-6, by probability descending (:104-113)
  for (size_t i = 0; i < vocab; ++i)
    if (logits[i] > 1e-6f) cand.emplace_back(static_cast<int>(i), logits[i]);
  std::stable_sort(cand.begin(), cand.end(), [](const std::pair<int, float>& a, const std::pair<int, float>& b) {
    return a.second > b.second;
  });
  if (top_k > 0 && cand.size() > static_cast<size_t>(top_k)) cand.resize(top_k);  // Top-K (:116-119)
  if (min_p > 0.0f && !cand.empty()) {                                               // Min-P (:122-132)
    const float thr = cand[0].second * min_p;
    for (size_t i = cand.size(); i-- > 1;)
      if (cand[i].second < thr) cand.erase(cand.begin() + static_cast<long>(i));
  }
  float cumulative = 0.0f;  // Top-P (:135-150)
  size_t cutoff = cand.size();
  for (size_t i = 0; i < cand.size(); ++i) {
    cumulative += cand[i].second;
    if (cumulative >= top_p) {
      cutoff = i + 1;
      break;
    }
  }
  if (cutoff < cand.size()) cand.resize(cutoff);
  float total = 0.0f;  // renormalise (:153-155)
  for (const auto& c : cand) total += c.second;
  const float inv_total = total > 0 ? 1.0f / total : 1.0f;
  if (cand_idx && cand_p && n_cand) {
    const int n = static_cast<int>(std::min<size_t>(cand.size(), static_cast<size_t>(std::max(cap, 0))));
    for (int i = 0; i < n; ++i) {
      cand_idx[i] = cand[i].first;
      cand_p[i] = cand[i].second * inv_total;
    }
    *n_cand = static_cast<int32_t>(cand.size());
  }
  float running = 0.0f;  // 6. CDF walk (:158-171)
  for (const auto& c : cand) {
    running += c.second * inv_total;
    if (u <= running) return c.first;
  }
  return cand.empty() ? 0 : cand[0].first;
}

int orc_num_threads(void) { return pool().size(); }

}  // extern "C"

// ==========================================================================================
// Engine: LlmEngine (LlmEngine.cs:157-461) over PagedKvCache (PagedKvCache.cs:47-286).
// ==========================================================================================
namespace {

struct Engine {
  orc_model m;
  int hd, qdim, kvdim, page_size, total_pages, threads;
  bool kv16;
  size_t token_stride, layer_stride, page_stride;  // floats
  std::vector<float> kstore, vstore;               // [page][layer][slot][kvdim] (KvBlock.cs:16-36)
  std::vector<int> refcount;
  std::vector<int> free_stack;  // Stack<int>: pushed 0..N-1, Pop() takes the last
  std::map<int, std::vector<int>> tables;
  std::map<int, int> lens;
  std::vector<float> cos_t, sin_t;
  int max_pos = 0;
  size_t q8_row(int cols) const { return static_cast<size_t>(cols / QK) * Q8_BYTES; }

  void ensure_rope(int pos) {
    if (pos < max_pos) return;
    int np = std::max({1024, m.context_length, pos + 1});
    np = std::max(np, max_pos * 2);
    cos_t.assign(static_cast<size_t>(np) * (hd / 2), 0.0f);
    sin_t.assign(static_cast<size_t>(np) * (hd / 2), 0.0f);
    orc_rope_table(np, hd, m.rope_base, cos_t.data(), sin_t.data());
    max_pos = np;
  }

  void reset_block(int b) {
    refcount[b] = 0;
    size_t n = static_cast<size_t>(m.layers) * layer_stride;
    std::fill(kstore.begin() + b * n, kstore.begin() + (b + 1) * n, 0.0f);
    std::fill(vstore.begin() + b * n, vstore.begin() + (b + 1) * n, 0.0f);
  }

  // PagedKvCache.AppendTokenAt (:281-316) / AppendToken (:237-276). advance: AppendToken rule.
  bool write_kv(int seq, int layer, int token, const float* k, const float* v, bool append_rule) {
    auto it = tables.find(seq);
    if (it == tables.end()) {
      it = tables.emplace(seq, std::vector<int>()).first;
      lens[seq] = 0;
    }
    std::vector<int>& table = it->second;
    int bi = token / page_size, slot = token % page_size;
    while (static_cast<int>(table.size()) <= bi) {
      if (free_stack.empty()) return false;
      int nb = free_stack.back();
      free_stack.pop_back();
      refcount[nb] = 1;
      table.push_back(nb);
    }
    size_t off = static_cast<size_t>(table[bi]) * page_stride + static_cast<size_t>(layer) * layer_stride +
                 static_cast<size_t>(slot) * token_stride;
    for (int i = 0; i < kvdim; ++i) {
      float kk = k[i], vv = v[i];
      if (kv16) {
        kk = orc_f16_to_f32(orc_f32_to_f16(kk));
        vv = orc_f16_to_f32(orc_f32_to_f16(vv));
      }
      kstore[off + i] = kk;
      vstore[off + i] = vv;
    }
    if (layer == m.layers - 1) {
      if (append_rule)
        lens[seq] = lens[seq] + 1;
      else if (token + 1 > lens[seq])
        lens[seq] = token + 1;
    }
    return true;
  }

  void free_sequence(int seq) {  // PagedKvCache.FreeSequence (:382-403)
    auto it = tables.find(seq);
    if (it == tables.end()) return;
    for (int b : it->second) {
      refcount[b]--;
      if (refcount[b] <= 0) {
        reset_block(b);
        free_stack.push_back(b);
      }
    }
    tables.erase(it);
    lens.erase(seq);
  }

  void embed(int token, float* x) {  // LookupTokenEmbedding (:317-345)
    int safe = (token >= 0 && token < m.vocab) ? token : 0;
    orc_dequantize_q8_0(m.tok_emb + static_cast<size_t>(safe) * q8_row(m.dim), m.dim, x);
  }

  void attend(int seq, int layer, int seq_len, const float* q, float* out) {
    static const std::vector<int> empty;
    auto it = tables.find(seq);
    const std::vector<int>& table = it == tables.end() ? empty : it->second;
    if (it == tables.end()) seq_len = 0;
    orc_gqa_attention(q, kstore.data() + static_cast<size_t>(layer) * layer_stride,
                      vstore.data() + static_cast<size_t>(layer) * layer_stride, table.data(), page_size, page_stride,
                      seq_len, m.heads, m.kv_heads, hd, out);
  }

  // One token's pre-attention part: rmsnorm, q/k/v projections, RoPE.
  void qkv(int l, const float* x, float* xn, float* q, float* k, float* v, int pos, int thr) {
    orc_rmsnorm(x, m.attn_norm + static_cast<size_t>(l) * m.dim, xn, m.dim, m.eps);
    orc_matvec_q8_0(m.wq + static_cast<size_t>(l) * qdim * q8_row(m.dim), xn, q, qdim, m.dim, 0, thr);
    orc_matvec_q8_0(m.wk + static_cast<size_t>(l) * kvdim * q8_row(m.dim), xn, k, kvdim, m.dim, 0, thr);
    orc_matvec_q8_0(m.wv + static_cast<size_t>(l) * kvdim * q8_row(m.dim), xn, v, kvdim, m.dim, 0, thr);
    for (int h = 0; h < m.heads; ++h) orc_rope_apply(q + h * hd, pos, hd, cos_t.data(), sin_t.data());
    for (int h = 0; h < m.kv_heads; ++h) orc_rope_apply(k + h * hd, pos, hd, cos_t.data(), sin_t.data());
  }

  // Post-attention part: Wo + residual, FFN rmsnorm, gate/up, SwiGLU, Wdown + residual.
  void ffn_part(int l, float* x, float* xn, const float* attn, float* gate, float* up, float* sw, int thr) {
    orc_matvec_q8_0(m.wo + static_cast<size_t>(l) * m.dim * q8_row(qdim), attn, x, m.dim, qdim, 1, thr);
    orc_rmsnorm(x, m.ffn_norm + static_cast<size_t>(l) * m.dim, xn, m.dim, m.eps);
    orc_matvec_q8_0(m.wgate + static_cast<size_t>(l) * m.ffn * q8_row(m.dim), xn, gate, m.ffn, m.dim, 0, thr);
    orc_matvec_q8_0(m.wup + static_cast<size_t>(l) * m.ffn * q8_row(m.dim), xn, up, m.ffn, m.dim, 0, thr);
    orc_swiglu(gate, up, sw, m.ffn);
    orc_matvec_q8_0(m.wdown + static_cast<size_t>(l) * m.dim * q8_row(m.ffn), sw, x, m.dim, m.ffn, 1, thr);
  }

  void head(const float* x, float* xn, float* logits, int thr) {
    orc_rmsnorm(x, m.final_norm, xn, m.dim, m.eps);
    orc_matvec_q8_0(m.lm_head, xn, logits, m.vocab, m.dim, 0, thr);
  }

  int forward_token(int seq, int token, int pos, float* logits) {  // ForwardToken (:347-461)
    ensure_rope(pos);
    std::vector<float> x(m.dim), xn(m.dim), q(qdim), k(kvdim), v(kvdim), attn(qdim), gate(m.ffn), up(m.ffn),
        sw(m.ffn);
    embed(token, x.data());
    for (int l = 0; l < m.layers; ++l) {
      qkv(l, x.data(), xn.data(), q.data(), k.data(), v.data(), pos, threads);
      if (!write_kv(seq, l, lens.count(seq) ? lens[seq] : 0, k.data(), v.data(), true)) return -1;
      attend(seq, l, lens[seq], q.data(), attn.data());
      ffn_part(l, x.data(), xn.data(), attn.data(), gate.data(), up.data(), sw.data(), threads);
    }
    head(x.data(), xn.data(), logits, threads);
    return 0;
  }

  int prefill(int seq, const int32_t* tokens, int n, int start, float* logits) {  // PrefillPrompt (:157-315)
    if (n <= 0) return 0;
    if (n == 1) return forward_token(seq, tokens[0], start, logits);
    ensure_rope(start + n);
    size_t T = static_cast<size_t>(n);
    std::vector<float> xb(T * m.dim), xnb(T * m.dim), qb(T * qdim), kb(T * kvdim), vb(T * kvdim), ab(T * qdim),
        gb(T * m.ffn), ub(T * m.ffn), sb(T * m.ffn);
    pool().parallel_for(T, 1, threads, [&](size_t t) { embed(tokens[t], xb.data() + t * m.dim); });
    for (int l = 0; l < m.layers; ++l) {
      pool().parallel_for(T, 1, threads, [&](size_t t) {
        qkv(l, xb.data() + t * m.dim, xnb.data() + t * m.dim, qb.data() + t * qdim, kb.data() + t * kvdim,
            vb.data() + t * kvdim, start + static_cast<int>(t), 1);
      });
      for (size_t t = 0; t < T; ++t)
        if (!write_kv(seq, l, start + static_cast<int>(t), kb.data() + t * kvdim, vb.data() + t * kvdim, false))
          return -1;
      pool().parallel_for(T, 1, threads, [&](size_t t) {
        int causal = (l == m.layers - 1) ? (start + static_cast<int>(t) + 1) : (start + static_cast<int>(t));
        attend(seq, l, causal, qb.data() + t * qdim, ab.data() + t * qdim);
        ffn_part(l, xb.data() + t * m.dim, xnb.data() + t * m.dim, ab.data() + t * qdim, gb.data() + t * m.ffn,
                 ub.data() + t * m.ffn, sb.data() + t * m.ffn, 1);
      });
    }
    head(xb.data() + (T - 1) * m.dim, xnb.data() + (T - 1) * m.dim, logits, threads);
    return 0;
  }
};

}  // namespace

extern "C" {

void* orc_engine_create(const orc_model* m, int total_pages, int page_size, int kv_fp16, int threads) {
  if (!m || total_pages <= 0 || page_size <= 0) return nullptr;
  Engine* e = new Engine();
  e->m = *m;
  e->hd = m->dim / m->heads;
  e->qdim = m->heads * e->hd;
  e->kvdim = m->kv_heads * e->hd;
  e->page_size = page_size;
  e->total_pages = total_pages;
  e->threads = threads;
  e->kv16 = kv_fp16 != 0;
  e->token_stride = static_cast<size_t>(e->kvdim);
  e->layer_stride = static_cast<size_t>(page_size) * e->token_stride;
  e->page_stride = static_cast<size_t>(m->layers) * e->layer_stride;
  e->kstore.assign(static_cast<size_t>(total_pages) * e->page_stride, 0.0f);
  e->vstore.assign(static_cast<size_t>(total_pages) * e->page_stride, 0.0f);
  e->refcount.assign(total_pages, 0);
  for (int i = 0; i < total_pages; ++i) e->free_stack.push_back(i);
  e->ensure_rope(0);
  return e;
}

void orc_engine_destroy(void* e) { delete static_cast<Engine*>(e); }

int orc_engine_prefill(void* e, int seq, const int32_t* tokens, int n, int start, float* logits) {
  return static_cast<Engine*>(e)->prefill(seq, tokens, n, start, logits);
}
int orc_engine_forward_token(void* e, int seq, int token, int pos, float* logits) {
  return static_cast<Engine*>(e)->forward_token(seq, token, pos, logits);
}
int orc_engine_seq_len(void* e, int seq) {
  auto* E = static_cast<Engine*>(e);
  auto it = E->lens.find(seq);
  return it == E->lens.end() ? 0 : it->second;
}
int orc_engine_free_blocks(void* e) { return static_cast<int>(static_cast<Engine*>(e)->free_stack.size()); }
void orc_engine_free_sequence(void* e, int seq) { static_cast<Engine*>(e)->free_sequence(seq); }

int orc_engine_get_kv(void* e, int seq, int layer, int token, int want_value, float* out) {
  auto* E = static_cast<Engine*>(e);
  auto it = E->tables.find(seq);
  if (it == E->tables.end()) return -1;
  int bi = token / E->page_size;
  if (bi >= static_cast<int>(it->second.size())) return -1;
  size_t off = static_cast<size_t>(it->second[bi]) * E->page_stride + static_cast<size_t>(layer) * E->layer_stride +
               static_cast<size_t>(token % E->page_size) * E->token_stride;
  const std::vector<float>& st = want_value ? E->vstore : E->kstore;
  std::memcpy(out, st.data() + off, sizeof(float) * E->kvdim);
  return 0;
}

int orc_engine_page_table(void* e, int seq, int32_t* out, int cap) {
  auto* E = static_cast<Engine*>(e);
  auto it = E->tables.find(seq);
  if (it == E->tables.end()) return 0;
  int n = static_cast<int>(it->second.size());
  for (int i = 0; i < n && i < cap; ++i) out[i] = it->second[i];
  return n;
}

int orc_engine_append_token(void* e, int seq, int layer, const float* k, const float* v) {
  auto* E = static_cast<Engine*>(e);
  int len = E->lens.count(seq) ? E->lens[seq] : 0;
  return E->write_kv(seq, layer, len, k, v, true) ? 0 : -1;
}

}  // extern "C"
