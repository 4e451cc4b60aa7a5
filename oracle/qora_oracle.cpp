// qora_oracle.cpp — TEST INFRASTRUCTURE ONLY (the parity checker and the timed CPU
// baseline). A restatement, in C++, of the reference CPU decode path of the Rust crate
// `qora`; each function names the reference lines it follows. Compiled with
// -O3 -ffp-contract=off (see Makefile) so that no multiply/add pair is fused unless
// the reference fuses it explicitly. Nothing shipped links this file.
#include "qora_oracle.h"

#include <immintrin.h>
#include <atomic>
#include <condition_variable>
#include <functional>
#include <mutex>
#include <thread>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <string>
#include <vector>

namespace {

constexpr size_t kGroup = 32;                  // Q4_GROUP_SIZE (src/gemv.rs:20)
constexpr size_t kParallelThreshold = 4000000; // k*n cut-over (src/gemv.rs:541, :651, :684)

int g_threads = 1;
int g_avx512 = -1;  // -1: not yet detected

// Persistent worker pool standing in for rayon's global pool. parallel_for(count, f)
// runs f(i) for every i in [0, count) on up to g_threads threads (the caller works
// too). Each index is computed independently, so results never depend on scheduling.
class Pool {
 public:
  ~Pool() { stop(); }
  void run(long count, const std::function<void(long)>& f, int threads) {
    if (count <= 0) return;
    if (threads <= 1 || count == 1) {
      for (long i = 0; i < count; ++i) f(i);
      return;
    }
    std::lock_guard<std::mutex> serial(run_mu_);
    ensure(threads - 1);
    {
      std::lock_guard<std::mutex> lk(mu_);
      job_ = &f;
      count_ = count;
      next_.store(0);
      active_ = (int)std::min<long>(threads - 1, (long)workers_.size());
      pending_ = active_;
      ++epoch_;
    }
    cv_.notify_all();
    drain();
    std::unique_lock<std::mutex> lk(mu_);
    done_cv_.wait(lk, [&] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void drain() {
    for (;;) {
      const long i = next_.fetch_add(1);
      if (i >= count_) break;
      (*job_)(i);
    }
  }
  void ensure(int n) {
    while ((int)workers_.size() < n) {
      const int id = (int)workers_.size();
      workers_.emplace_back([this, id] { loop(id); });
    }
  }
  void loop(int id) {
    uint64_t seen = 0;
    for (;;) {
      {
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return quit_ || (epoch_ != seen && id < active_); });
        if (quit_) return;
        seen = epoch_;
      }
      drain();
      std::lock_guard<std::mutex> lk(mu_);
      if (--pending_ == 0) done_cv_.notify_one();
    }
  }
  void stop() {
    {
      std::lock_guard<std::mutex> lk(mu_);
      quit_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
    workers_.clear();
  }
  std::mutex run_mu_, mu_;
  std::condition_variable cv_, done_cv_;
  std::vector<std::thread> workers_;
  const std::function<void(long)>* job_ = nullptr;
  long count_ = 0;
  std::atomic<long> next_{0};
  int active_ = 0, pending_ = 0;
  uint64_t epoch_ = 0;
  bool quit_ = false;
};

Pool& pool() {
  static Pool p;
  return p;
}

void parallel_for(long count, bool enabled, const std::function<void(long)>& f) {
  pool().run(count, f, enabled ? g_threads : 1);
}

bool host_avx512() { return __builtin_cpu_supports("avx512f"); }
bool use_avx512() {
  if (g_avx512 < 0) g_avx512 = host_avx512() ? 1 : 0;
  return g_avx512 == 1;
}

// Exact IEEE binary16 -> binary32 (the `half` crate's to_f32 is exact).
inline float h2f(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1Fu;
  const uint32_t m = h & 0x3FFu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else {
      float f = std::ldexp((float)m, -24);  // subnormal: m * 2^-24, exact in f32
      std::memcpy(&bits, &f, 4);
      bits |= sign;
    }
  } else if (e == 31) {
    bits = sign | 0x7F800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float out;
  std::memcpy(&out, &bits, 4);
  return out;
}

// Nearest IEEE binary16 value of x (ties to even), returned as f32. From the format's
// definition: the quantum of |x| is 2^(e-10) for binade e >= -14 and 2^-24 below
// (subnormals); |x| >= 65520 (halfway between 65504 and 2^16) overflows to inf.
// Scaling by a power of two is exact in double, and nearbyint rounds to nearest even.
inline float round_f16(float x) {
  uint32_t b;
  std::memcpy(&b, &x, 4);
  const uint32_t a = b & 0x7FFFFFFFu;
  if (a >= 0x7F800000u) return x;  // inf, nan
  const bool neg = (b >> 31) != 0;
  if (a >= 0x477FF000u) return neg ? -INFINITY : INFINITY;
  const int e = (int)(a >> 23) - 127;  // f32 subnormals give -127: they round to 0 or 2^-24 steps
  const int qexp = std::max(e - 10, -24);
  const double v = std::nearbyint(std::ldexp((double)std::fabs(x), -qexp));
  const float r = (float)std::ldexp(v, qexp);
  return neg ? -r : r;
}

// ---------------------------------------------------------------- Q4 row kernels
// gemv_q4_inner scalar path (src/gemv.rs:605-640): per input row ki, s = scale*x,
// a 16-entry table s*(q-8), and out[j] += table[nibble] in element order.
void q4_rows_scalar(const float* x, const uint8_t* packed, const uint16_t* scales,
                    size_t n, size_t k0, size_t k1, float* out) {
  const size_t gpr = n / kGroup;
  for (size_t ki = k0; ki < k1; ++ki) {
    const float xv = x[ki];
    if (xv == 0.0f) continue;
    for (size_t g = 0; g < gpr; ++g) {
      const float s = h2f(scales[ki * gpr + g]) * xv;
      if (s == 0.0f) continue;
      float table[16];
      for (int q = 0; q < 16; ++q) table[q] = (q == 8) ? 0.0f : s * (float)(q - 8);
      const uint8_t* src = packed + (ki * gpr + g) * 16;
      float* dst = out + g * kGroup;
      for (int b = 0; b < 16; ++b) {
        dst[2 * b] += table[src[b] & 0x0F];
        dst[2 * b + 1] += table[src[b] >> 4];
      }
    }
  }
}

// Same arithmetic as gemv_q4_avx512 (src/simd.rs:44-83): identical products
// factor*s and identical per-element additions, vectorised 16 elements at a time.
__attribute__((target("avx512f"))) void q4_rows_avx512(const float* x,
                                                       const uint8_t* packed,
                                                       const uint16_t* scales, size_t n,
                                                       size_t k0, size_t k1, float* out) {
  const size_t gpr = n / kGroup;
  const __m512 factors = _mm512_setr_ps(-8, -7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7);
  const __m512i shift = _mm512_setr_epi32(0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4);
  const __m512i low4 = _mm512_set1_epi32(0x0F);
  for (size_t ki = k0; ki < k1; ++ki) {
    const float xv = x[ki];
    if (xv == 0.0f) continue;
    for (size_t g = 0; g < gpr; ++g) {
      const float s = h2f(scales[ki * gpr + g]) * xv;
      if (s == 0.0f) continue;
      const __m512 table = _mm512_mul_ps(factors, _mm512_set1_ps(s));
      const __m128i bytes = _mm_loadu_si128((const __m128i*)(packed + (ki * gpr + g) * 16));
      // each byte twice: b0 b0 b1 b1 ... so lane 2i holds the low nibble, 2i+1 the high
      const __m512i e0 = _mm512_cvtepu8_epi32(_mm_unpacklo_epi8(bytes, bytes));
      const __m512i e1 = _mm512_cvtepu8_epi32(_mm_unpackhi_epi8(bytes, bytes));
      const __m512i i0 = _mm512_and_si512(_mm512_srlv_epi32(e0, shift), low4);
      const __m512i i1 = _mm512_and_si512(_mm512_srlv_epi32(e1, shift), low4);
      float* dst = out + g * kGroup;
      _mm512_storeu_ps(dst, _mm512_add_ps(_mm512_loadu_ps(dst), _mm512_permutexvar_ps(i0, table)));
      _mm512_storeu_ps(dst + 16,
                       _mm512_add_ps(_mm512_loadu_ps(dst + 16), _mm512_permutexvar_ps(i1, table)));
    }
  }
}

void q4_rows(const float* x, const uint8_t* packed, const uint16_t* scales, size_t n,
             size_t k0, size_t k1, float* out) {
  if (use_avx512())
    q4_rows_avx512(x, packed, scales, n, k0, k1, out);
  else
    q4_rows_scalar(x, packed, scales, n, k0, k1, out);
}

// One (row, group) update of the AVX-512 gate/up chunk: table = factors*s, then the 32
// elements added in order (the per-matrix body of src/simd.rs:112-143).
__attribute__((target("avx512f"))) inline void q4_group_avx512(const uint8_t* src, float s,
                                                              float* dst) {
  const __m512 factors = _mm512_setr_ps(-8, -7, -6, -5, -4, -3, -2, -1, 0, 1, 2, 3, 4, 5, 6, 7);
  const __m512i shift = _mm512_setr_epi32(0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4, 0, 4);
  const __m512i low4 = _mm512_set1_epi32(0x0F);
  const __m512 table = _mm512_mul_ps(factors, _mm512_set1_ps(s));
  const __m128i bytes = _mm_loadu_si128((const __m128i*)src);
  const __m512i i0 = _mm512_and_si512(
      _mm512_srlv_epi32(_mm512_cvtepu8_epi32(_mm_unpacklo_epi8(bytes, bytes)), shift), low4);
  const __m512i i1 = _mm512_and_si512(
      _mm512_srlv_epi32(_mm512_cvtepu8_epi32(_mm_unpackhi_epi8(bytes, bytes)), shift), low4);
  _mm512_storeu_ps(dst, _mm512_add_ps(_mm512_loadu_ps(dst), _mm512_permutexvar_ps(i0, table)));
  _mm512_storeu_ps(dst + 16,
                   _mm512_add_ps(_mm512_loadu_ps(dst + 16), _mm512_permutexvar_ps(i1, table)));
}

// fused_gate_up_q4 AVX-512 chunk (src/simd.rs:87-147)
__attribute__((target("avx512f"))) void gate_up_rows_avx512(
    const float* x, const uint8_t* gp, const uint16_t* gsc, const uint8_t* up,
    const uint16_t* usc, size_t n, size_t k0, size_t k1, float* gout, float* uout) {
  const size_t gpr = n / kGroup;
  for (size_t ki = k0; ki < k1; ++ki) {
    const float xv = x[ki];
    if (xv == 0.0f) continue;
    for (size_t g = 0; g < gpr; ++g) {
      const float gs = h2f(gsc[ki * gpr + g]) * xv;
      const float us = h2f(usc[ki * gpr + g]) * xv;
      if (gs == 0.0f && us == 0.0f) continue;
      const size_t off = (ki * gpr + g) * 16;
      if (gs != 0.0f) q4_group_avx512(gp + off, gs, gout + g * kGroup);
      if (us != 0.0f) q4_group_avx512(up + off, us, uout + g * kGroup);
    }
  }
}

// fused_gate_up_q4 scalar chunk (src/gemv.rs:439-480)
void gate_up_rows_scalar(const float* x, const uint8_t* gp, const uint16_t* gsc,
                         const uint8_t* up, const uint16_t* usc, size_t n, size_t k0,
                         size_t k1, float* gout, float* uout) {
  const size_t gpr = n / kGroup;
  for (size_t ki = k0; ki < k1; ++ki) {
    const float xv = x[ki];
    if (xv == 0.0f) continue;
    for (size_t g = 0; g < gpr; ++g) {
      const float gs = h2f(gsc[ki * gpr + g]) * xv;
      const float us = h2f(usc[ki * gpr + g]) * xv;
      if (gs == 0.0f && us == 0.0f) continue;
      float gt[16], ut[16];
      for (int q = 0; q < 16; ++q) {
        gt[q] = (q == 8) ? 0.0f : gs * (float)(q - 8);
        ut[q] = (q == 8) ? 0.0f : us * (float)(q - 8);
      }
      const size_t off = (ki * gpr + g) * 16;
      float* gd = gout + g * kGroup;
      float* ud = uout + g * kGroup;
      for (int b = 0; b < 16; ++b) {
        gd[2 * b] += gt[gp[off + b] & 0x0F];
        gd[2 * b + 1] += gt[gp[off + b] >> 4];
        ud[2 * b] += ut[up[off + b] & 0x0F];
        ud[2 * b + 1] += ut[up[off + b] >> 4];
      }
    }
  }
}

// gemv_f16_avx512 (src/simd.rs:151-176): FMA on 16-wide blocks, scalar mul+add tail.
__attribute__((target("avx512f,f16c"))) void f16_rows_avx512(const float* x, const uint16_t* w,
                                                             size_t k, size_t n, float* out) {
  const size_t n16 = n / 16 * 16;
  for (size_t ki = 0; ki < k; ++ki) {
    const float v = x[ki];
    if (v == 0.0f) continue;
    const __m512 vv = _mm512_set1_ps(v);
    const uint16_t* row = w + ki * n;
    size_t j = 0;
    for (; j < n16; j += 16) {
      const __m512 wf = _mm512_cvtph_ps(_mm256_loadu_si256((const __m256i*)(row + j)));
      _mm512_storeu_ps(out + j, _mm512_fmadd_ps(vv, wf, _mm512_loadu_ps(out + j)));
    }
    for (; j < n; ++j) out[j] += v * h2f(row[j]);
  }
}

// gemv_f16 scalar path (src/gemv.rs:558-566): no zero skip, no FMA.
void f16_rows_scalar(const float* x, const uint16_t* w, size_t k, size_t n, float* out) {
  for (size_t ki = 0; ki < k; ++ki) {
    const float v = x[ki];
    const uint16_t* row = w + ki * n;
    for (size_t j = 0; j < n; ++j) out[j] += v * h2f(row[j]);
  }
}

// Ordered k-split (src/gemv.rs:655-673): T chunks of ceil(k/T) rows, each into its own
// zeroed partial, chunks past k skipped, partials summed into a zero vector in order.
template <typename Chunk>
void ksplit(size_t k, size_t n, int parts, std::vector<std::vector<float>>& partials,
            Chunk chunk) {
  const size_t T = (size_t)std::max(1, parts);
  const size_t ck = (k + T - 1) / T;
  partials.assign(T, std::vector<float>());
  parallel_for((long)T, true, [&](long t) {
    const size_t k0 = (size_t)t * ck;
    if (k0 >= k) return;
    const size_t k1 = std::min(k, ((size_t)t + 1) * ck);
    partials[t].assign(n, 0.0f);
    chunk(k0, k1, partials[t].data());
  });
}

// ---------------------------------------------------------------- model containers
struct Mat {
  bool q4 = true;
  uint64_t k = 0, n = 0;
  std::vector<uint8_t> packed;
  std::vector<uint16_t> scales;
  std::vector<uint16_t> data;
};

struct Layer {
  Mat w[7];  // q k v o gate up down (src/save.rs:242-248 order)
  std::vector<uint16_t> g_in, g_post;
  uint32_t num_heads = 0, num_kv_heads = 0, head_dim = 0, num_kv_groups = 0;
};

}  // namespace

struct orc_model {
  uint32_t format = 1;
  uint32_t num_layers = 0, vocab = 0, hidden = 0, half_dim = 0;
  std::vector<uint8_t> use_rope;
  std::vector<Layer> layers;
  Mat embed;
  std::vector<uint16_t> final_norm;
  std::vector<float> cos_t, sin_t;
};

struct orc_kv {
  uint32_t kv_stride = 0;  // kv_heads * head_dim
  std::vector<std::vector<float>> k, v;
  std::vector<uint32_t> len;
  bool f16 = false;        // opt-in binary16 cache (values rounded as they enter)
};

namespace {

void gemv(const float* x, const Mat& w, float* y);

void gemv_q4_impl(const float* x, const uint8_t* p, const uint16_t* s, size_t k, size_t n,
                  float* y) {
  if (k * n < kParallelThreshold) {
    std::fill(y, y + n, 0.0f);
    q4_rows(x, p, s, n, 0, k, y);
    return;
  }
  std::vector<std::vector<float>> parts;
  ksplit(k, n, g_threads, parts, [&](size_t k0, size_t k1, float* out) {
    q4_rows(x, p, s, n, k0, k1, out);
  });
  std::fill(y, y + n, 0.0f);
  for (auto& pt : parts)
    if (!pt.empty())
      for (size_t j = 0; j < n; ++j) y[j] += pt[j];
}

void gemv_f16_impl(const float* x, const uint16_t* w, size_t k, size_t n, float* y) {
  if (use_avx512()) {
    if (k * n < kParallelThreshold) {
      std::fill(y, y + n, 0.0f);
      f16_rows_avx512(x, w, k, n, y);
      return;
    }
    std::vector<std::vector<float>> parts;
    ksplit(k, n, g_threads, parts, [&](size_t k0, size_t k1, float* out) {
      f16_rows_avx512(x + k0, w + k0 * n, k1 - k0, n, out);
    });
    std::fill(y, y + n, 0.0f);
    for (auto& pt : parts)
      if (!pt.empty())
        for (size_t j = 0; j < n; ++j) y[j] += pt[j];
    return;
  }
  std::fill(y, y + n, 0.0f);
  f16_rows_scalar(x, w, k, n, y);
}

void gemv(const float* x, const Mat& w, float* y) {
  if (w.q4)
    gemv_q4_impl(x, w.packed.data(), w.scales.data(), w.k, w.n, y);
  else
    gemv_f16_impl(x, w.data.data(), w.k, w.n, y);
}

inline float silu_mul(float g, float u) {  // src/gemv.rs:497-499
  const float s = g / (1.0f + std::exp(-g));
  return s * u;
}

void fused_gate_up_q4_impl(const float* x, const uint8_t* gp, const uint16_t* gs,
                           const uint8_t* up, const uint16_t* us, size_t k, size_t n,
                           float* out) {
  const size_t T = (size_t)std::max(1, g_threads);
  const size_t ck = (k + T - 1) / T;
  std::vector<std::vector<float>> gpart(T), upart(T);
  const bool avx = use_avx512();
  parallel_for((long)T, true, [&](long t) {
    const size_t k0 = (size_t)t * ck;
    if (k0 >= k) return;
    const size_t k1 = std::min(k, ((size_t)t + 1) * ck);
    gpart[t].assign(n, 0.0f);
    upart[t].assign(n, 0.0f);
    if (avx)
      gate_up_rows_avx512(x, gp, gs, up, us, n, k0, k1, gpart[t].data(), upart[t].data());
    else
      gate_up_rows_scalar(x, gp, gs, up, us, n, k0, k1, gpart[t].data(), upart[t].data());
  });
  std::vector<float> gsum(n, 0.0f), usum(n, 0.0f);
  for (size_t t = 0; t < T; ++t) {
    if (gpart[t].empty()) continue;
    for (size_t j = 0; j < n; ++j) {
      gsum[j] += gpart[t][j];
      usum[j] += upart[t][j];
    }
  }
  for (size_t j = 0; j < n; ++j) out[j] = silu_mul(gsum[j], usum[j]);
}

// fused_gate_up_gemv (src/gemv.rs:392-409)
void fused_gate_up(const float* x, const Mat& g, const Mat& u, float* out) {
  if (g.q4 && u.q4) {
    fused_gate_up_q4_impl(x, g.packed.data(), g.scales.data(), u.packed.data(),
                          u.scales.data(), g.k, g.n, out);
    return;
  }
  std::vector<float> gv(g.n), uv(u.n);
  gemv(x, g, gv.data());
  gemv(x, u, uv.data());
  for (size_t j = 0; j < g.n; ++j) out[j] = silu_mul(gv[j], uv[j]);
}

void rms_norm(const float* x, const uint16_t* gamma, size_t size, float* out) {
  float sum_sq = 0.0f;
  for (size_t i = 0; i < size; ++i) sum_sq += x[i] * x[i];
  const float inv = 1.0f / std::sqrt(sum_sq / (float)size + 1e-6f);
  for (size_t i = 0; i < size; ++i) out[i] = x[i] * inv * h2f(gamma[i]);
}

void rope(float* d, size_t heads, size_t hd, const float* ct, const float* st, size_t half,
          size_t pos) {
  const size_t off = pos * half;
  for (size_t h = 0; h < heads; ++h) {
    float* base = d + h * hd;
    for (size_t i = 0; i < half; ++i) {
      const float a = base[i], b = base[half + i];
      const float c = ct[off + i], s = st[off + i];
      base[i] = a * c - b * s;
      base[half + i] = b * c + a * s;
    }
  }
}

void softmax(float* s, size_t n) {
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i) mx = std::fmax(mx, s[i]);
  float sum = 0.0f;
  for (size_t i = 0; i < n; ++i) {
    s[i] = std::exp(s[i] - mx);
    sum += s[i];
  }
  const float inv = 1.0f / sum;
  for (size_t i = 0; i < n; ++i) s[i] *= inv;
}

void embed_q4(const uint8_t* packed, const uint16_t* scales, size_t n, size_t row, float* out) {
  const size_t gpr = n / kGroup;
  for (size_t g = 0; g < gpr; ++g) {
    const float sc = h2f(scales[row * gpr + g]);
    const uint8_t* src = packed + (row * gpr + g) * 16;
    for (int b = 0; b < 16; ++b) {
      out[g * kGroup + 2 * b] = sc * (float)((int)(src[b] & 0x0F) - 8);
      out[g * kGroup + 2 * b + 1] = sc * (float)((int)((src[b] >> 4) & 0x0F) - 8);
    }
  }
}

void embed(const orc_model* m, size_t token, float* out) {  // src/gemv.rs:515-526
  if (m->embed.q4) {
    embed_q4(m->embed.packed.data(), m->embed.scales.data(), m->hidden, token, out);
  } else {
    const uint16_t* row = m->embed.data.data() + token * m->hidden;
    for (size_t i = 0; i < m->hidden; ++i) out[i] = h2f(row[i]);
  }
}

void lm_head_q4(const float* x, const uint8_t* packed, const uint16_t* scales, size_t vocab,
                size_t hidden, float* logits) {
  const size_t gpr = hidden / kGroup;
  const size_t chunks = (vocab + 255) / 256;
  parallel_for((long)chunks, true, [&](long c) {
    const size_t v1 = std::min(vocab, (size_t)(c + 1) * 256);
    for (size_t v = (size_t)c * 256; v < v1; ++v) {
      float dot = 0.0f;
      for (size_t g = 0; g < gpr; ++g) {
        const float sc = h2f(scales[v * gpr + g]);
        if (sc == 0.0f) continue;
        float table[16];
        for (int q = 0; q < 16; ++q) table[q] = (q == 8) ? 0.0f : sc * (float)(q - 8);
        const uint8_t* src = packed + (v * gpr + g) * 16;
        const float* xi = x + g * kGroup;
        for (int b = 0; b < 16; ++b) {
          dot += xi[2 * b] * table[src[b] & 0x0F];
          dot += xi[2 * b + 1] * table[src[b] >> 4];
        }
      }
      logits[v] = dot;
    }
  });
}

void lm_head_f16(const float* x, const uint16_t* w, size_t vocab, size_t hidden, float* logits) {
  const size_t chunks = (vocab + 255) / 256;
  parallel_for((long)chunks, true, [&](long c) {
    const size_t v1 = std::min(vocab, (size_t)(c + 1) * 256);
    for (size_t v = (size_t)c * 256; v < v1; ++v) {
      const uint16_t* row = w + v * hidden;
      float sum = 0.0f;
      for (size_t j = 0; j < hidden; ++j) sum += x[j] * h2f(row[j]);
      logits[v] = sum;
    }
  });
}

void lm_head(const orc_model* m, const float* x, float* logits) {
  if (m->embed.q4)
    lm_head_q4(x, m->embed.packed.data(), m->embed.scales.data(), m->vocab, m->hidden, logits);
  else
    lm_head_f16(x, m->embed.data.data(), m->vocab, m->hidden, logits);
}

// attention of one query head over kv_len cached rows (src/gemv.rs:922-948)
void attend_head(const float* q, const float* K, const float* V, size_t kv_len,
                 size_t kv_stride, size_t kvh, size_t hd, float scale, float* out) {
  std::vector<float> scores(kv_len);
  for (size_t s = 0; s < kv_len; ++s) {
    const float* kr = K + s * kv_stride + kvh * hd;
    float dot = 0.0f;
    for (size_t d = 0; d < hd; ++d) dot += q[d] * kr[d];
    scores[s] = dot * scale;
  }
  softmax(scores.data(), kv_len);
  for (size_t s = 0; s < kv_len; ++s) {
    const float* vr = V + s * kv_stride + kvh * hd;
    const float p = scores[s];
    for (size_t d = 0; d < hd; ++d) out[d] += p * vr[d];
  }
}

void gemm(const float* x, size_t seq, const Mat& w, float* y);

void gemm_q4_impl(const float* x, size_t seq, const uint8_t* p, const uint16_t* s, size_t k,
                  size_t n, float* y) {
  const bool par = !(seq <= 1 || k * n < kParallelThreshold);
  parallel_for((long)seq, par, [&](long t) {
    float* row = y + (size_t)t * n;
    std::fill(row, row + n, 0.0f);
    q4_rows(x + (size_t)t * k, p, s, n, 0, k, row);
  });
}

void gemm_f16_impl(const float* x, size_t seq, const uint16_t* w, size_t k, size_t n, float* y) {
  // scalar, single-threaded, no FMA (src/gemv.rs:571-588)
  for (size_t t = 0; t < seq; ++t) {
    float* row = y + t * n;
    std::fill(row, row + n, 0.0f);
    const float* xr = x + t * k;
    for (size_t ki = 0; ki < k; ++ki) {
      const float v = xr[ki];
      const uint16_t* wr = w + ki * n;
      for (size_t j = 0; j < n; ++j) row[j] += v * h2f(wr[j]);
    }
  }
}

void gemm(const float* x, size_t seq, const Mat& w, float* y) {
  if (w.q4)
    gemm_q4_impl(x, seq, w.packed.data(), w.scales.data(), w.k, w.n, y);
  else
    gemm_f16_impl(x, seq, w.data.data(), w.k, w.n, y);
}

// ---------------------------------------------------------------- .qora reader
struct Reader {
  FILE* f = nullptr;
  std::string err;
  bool ok = true;
  void need(void* dst, size_t n) {
    if (!ok) return;
    if (n && std::fread(dst, 1, n, f) != n) {
      ok = false;
      err = "short read";
    }
  }
  uint32_t u32() { uint32_t v = 0; need(&v, 4); return v; }
  uint64_t u64() { uint64_t v = 0; need(&v, 8); return v; }
  uint8_t u8() { uint8_t v = 0; need(&v, 1); return v; }
  template <typename T>
  void vec(std::vector<T>& out) {  // u64 length prefix then raw elements
    const uint64_t len = u64();
    if (!ok) return;
    if (len > (1ull << 36)) { ok = false; err = "implausible vector length"; return; }
    out.resize(len);
    need(out.data(), len * sizeof(T));
  }
};

bool read_mat(Reader& r, uint8_t fmt, Mat& m) {  // read_weight_data (src/save.rs:217-238)
  m.k = r.u64();
  m.n = r.u64();
  if (fmt == 0) {
    m.q4 = false;
    r.vec(m.data);
    if (r.ok && m.data.size() != m.k * m.n) { r.ok = false; r.err = "f16 weight size mismatch"; }
  } else if (fmt == 1) {
    m.q4 = true;
    r.vec(m.packed);
    r.vec(m.scales);
    if (r.ok && (m.n % kGroup != 0 || m.packed.size() != m.k * m.n / 2 ||
                 m.scales.size() != m.k * m.n / kGroup)) {
      r.ok = false;
      r.err = "q4 weight size mismatch";
    }
  } else {
    r.ok = false;
    r.err = "Unknown format id " + std::to_string(fmt);
  }
  return r.ok;
}

void set_err(char* err, size_t len, const std::string& s) {
  if (err && len) std::snprintf(err, len, "%s", s.c_str());
}

void copy_mat(const qora_matrix_view& v, uint32_t fmt, Mat& m) {
  m.k = v.k;
  m.n = v.n;
  m.q4 = fmt == QORA_FORMAT_Q4;
  if (m.q4) {
    m.packed.assign(v.packed, v.packed + v.k * v.n / 2);
    m.scales.assign(v.scales, v.scales + v.k * v.n / kGroup);
  } else {
    m.data.assign(v.data, v.data + v.k * v.n);
  }
}

}  // namespace

// ================================================================ C ABI
extern "C" {

void orc_set_threads(int t) { g_threads = t < 1 ? 1 : t; }
int orc_get_threads(void) { return g_threads; }
void orc_set_avx512(int on) { g_avx512 = (on && host_avx512()) ? 1 : 0; }
int orc_get_avx512(void) { return use_avx512() ? 1 : 0; }
int orc_host_has_avx512(void) { return host_avx512() ? 1 : 0; }

float orc_f16_to_f32(uint16_t h) { return h2f(h); }

orc_model* orc_model_load(const char* path, char* err, size_t errlen) {
  Reader r;
  r.f = std::fopen(path, "rb");
  if (!r.f) { set_err(err, errlen, std::string("cannot open ") + path); return nullptr; }
  std::setvbuf(r.f, nullptr, _IOFBF, 8 << 20);
  auto* m = new orc_model();
  char magic[4] = {0, 0, 0, 0};
  r.need(magic, 4);
  if (r.ok && std::memcmp(magic, "QOR3", 4) != 0) { r.ok = false; r.err = "Invalid magic bytes"; }
  uint32_t version = r.u32();
  if (r.ok && version != 1) { r.ok = false; r.err = "Unsupported version " + std::to_string(version) + ", expected 1"; }
  const uint8_t fmt = r.u8();
  m->format = fmt;
  m->num_layers = r.u32();
  m->vocab = r.u32();
  m->hidden = r.u32();
  m->half_dim = r.u32();
  r.vec(m->use_rope);
  if (r.ok && m->num_layers > 4096) { r.ok = false; r.err = "implausible layer count"; }
  if (r.ok) m->layers.resize(m->num_layers);
  for (uint32_t i = 0; r.ok && i < m->num_layers; ++i) {  // read_layer_weights (:241-262)
    Layer& L = m->layers[i];
    for (int w = 0; w < 7 && r.ok; ++w) read_mat(r, fmt, L.w[w]);
    r.vec(L.g_in);
    r.vec(L.g_post);
    L.num_heads = r.u32();
    L.num_kv_heads = r.u32();
    L.head_dim = r.u32();
    L.num_kv_groups = r.u32();
  }
  if (r.ok) read_mat(r, fmt, m->embed);
  r.vec(m->final_norm);
  r.vec(m->cos_t);
  r.vec(m->sin_t);
  std::fclose(r.f);
  if (!r.ok) { set_err(err, errlen, r.err); delete m; return nullptr; }
  if (m->use_rope.size() != m->num_layers) {
    set_err(err, errlen, "no_rope_layers length != num_layers");
    delete m;
    return nullptr;
  }
  return m;
}

orc_model* orc_model_from_view(const qora_weights_view* v, char* err, size_t errlen) {
  if (!v || (v->format != QORA_FORMAT_Q4 && v->format != QORA_FORMAT_F16)) {
    set_err(err, errlen, "bad view");
    return nullptr;
  }
  auto* m = new orc_model();
  m->format = v->format;
  m->num_layers = v->num_layers;
  m->vocab = v->vocab;
  m->hidden = v->hidden;
  m->half_dim = v->rope_half_dim;
  m->use_rope.assign(v->no_rope_layers, v->no_rope_layers + v->num_layers);
  m->layers.resize(v->num_layers);
  for (uint32_t i = 0; i < v->num_layers; ++i) {
    const qora_layer_view& lv = v->layers[i];
    Layer& L = m->layers[i];
    const qora_matrix_view* mats[7] = {&lv.q_proj, &lv.k_proj, &lv.v_proj, &lv.o_proj,
                                       &lv.gate_proj, &lv.up_proj, &lv.down_proj};
    for (int w = 0; w < 7; ++w) copy_mat(*mats[w], v->format, L.w[w]);
    L.g_in.assign(lv.input_norm_gamma, lv.input_norm_gamma + v->hidden);
    L.g_post.assign(lv.post_attn_norm_gamma, lv.post_attn_norm_gamma + v->hidden);
    L.num_heads = lv.num_heads;
    L.num_kv_heads = lv.num_kv_heads;
    L.head_dim = lv.head_dim;
    L.num_kv_groups = lv.num_kv_groups;
  }
  copy_mat(v->embed, v->format, m->embed);
  m->final_norm.assign(v->final_norm_gamma, v->final_norm_gamma + v->hidden);
  const size_t tl = v->rope_rows * v->rope_half_dim;
  m->cos_t.assign(v->rope_cos, v->rope_cos + tl);
  m->sin_t.assign(v->rope_sin, v->rope_sin + tl);
  return m;
}

void orc_model_free(orc_model* m) { delete m; }
uint32_t orc_model_vocab(const orc_model* m) { return m->vocab; }
uint32_t orc_model_hidden(const orc_model* m) { return m->hidden; }
uint32_t orc_model_layers(const orc_model* m) { return m->num_layers; }
uint32_t orc_model_format(const orc_model* m) { return m->format; }

orc_kv* orc_kv_new(const orc_model* m) {
  auto* kv = new orc_kv();
  const Layer& L0 = m->layers.at(0);
  kv->kv_stride = L0.num_kv_heads * L0.head_dim;
  kv->k.resize(m->num_layers);
  kv->v.resize(m->num_layers);
  kv->len.assign(m->num_layers, 0);
  for (uint32_t i = 0; i < m->num_layers; ++i) {  // empty_kv_cache capacity (src/gemv.rs:162)
    kv->k[i].reserve((size_t)kv->kv_stride * 512);
    kv->v[i].reserve((size_t)kv->kv_stride * 512);
  }
  return kv;
}
void orc_kv_free(orc_kv* kv) { delete kv; }
uint32_t orc_kv_len(const orc_kv* kv, uint32_t layer) { return kv->len.at(layer); }
int orc_kv_import(orc_kv* kv, uint32_t layer, const float* k, const float* v, uint32_t seq_len) {
  if (layer >= kv->len.size()) return 1;
  const size_t n = (size_t)seq_len * kv->kv_stride;
  kv->k[layer].assign(k, k + n);
  kv->v[layer].assign(v, v + n);
  if (kv->f16) {
    for (float& x : kv->k[layer]) x = round_f16(x);
    for (float& x : kv->v[layer]) x = round_f16(x);
  }
  kv->len[layer] = seq_len;
  return 0;
}
int orc_kv_set_f16(orc_kv* kv, int on) {
  for (uint32_t n : kv->len)
    if (n) return 1;
  kv->f16 = on != 0;
  return 0;
}
void orc_round_f16(const float* x, float* out, size_t n) {
  for (size_t i = 0; i < n; ++i) out[i] = round_f16(x[i]);
}
int orc_kv_export(const orc_kv* kv, uint32_t layer, float* k, float* v, uint32_t seq_len) {
  if (layer >= kv->len.size() || seq_len > kv->len[layer]) return 1;
  const size_t n = (size_t)seq_len * kv->kv_stride;
  std::memcpy(k, kv->k[layer].data(), n * 4);
  std::memcpy(v, kv->v[layer].data(), n * 4);
  return 0;
}

void orc_gemv_q4(const float* x, const uint8_t* packed, const uint16_t* scales, size_t k,
                 size_t n, float* y) {
  gemv_q4_impl(x, packed, scales, k, n, y);
}
void orc_gemv_q4_rows(const float* x, const uint8_t* packed, const uint16_t* scales, size_t n,
                      size_t k0, size_t k1, float* y) {
  std::fill(y, y + n, 0.0f);
  q4_rows(x, packed, scales, n, k0, k1, y);
}
void orc_fused_gate_up_q4(const float* x, const uint8_t* gp, const uint16_t* gs,
                          const uint8_t* up, const uint16_t* us, size_t k, size_t n,
                          float* out) {
  fused_gate_up_q4_impl(x, gp, gs, up, us, k, n, out);
}
void orc_gemv_f16(const float* x, const uint16_t* w, size_t k, size_t n, float* y) {
  gemv_f16_impl(x, w, k, n, y);
}
void orc_gemm_q4(const float* x, size_t seq, const uint8_t* packed, const uint16_t* scales,
                 size_t k, size_t n, float* y) {
  gemm_q4_impl(x, seq, packed, scales, k, n, y);
}
void orc_gemm_f16(const float* x, size_t seq, const uint16_t* w, size_t k, size_t n, float* y) {
  gemm_f16_impl(x, seq, w, k, n, y);
}
void orc_embed_q4(const uint8_t* packed, const uint16_t* scales, size_t n, size_t row, float* out) {
  embed_q4(packed, scales, n, row, out);
}
void orc_dequant_q4_rows(const uint8_t* packed, const uint16_t* scales, size_t n, size_t row0,
                         size_t rows, float* out) {
  for (size_t r = 0; r < rows; ++r) embed_q4(packed, scales, n, row0 + r, out + r * n);
}
void orc_rms_norm(const float* x, const uint16_t* gamma, size_t size, float* out) {
  rms_norm(x, gamma, size, out);
}
void orc_rope(float* data, size_t heads, size_t head_dim, const float* cos_t,
              const float* sin_t, size_t half_dim, size_t pos) {
  rope(data, heads, head_dim, cos_t, sin_t, half_dim, pos);
}
void orc_softmax(float* s, size_t n) { softmax(s, n); }
void orc_lm_head_q4(const float* x, const uint8_t* packed, const uint16_t* scales, size_t vocab,
                    size_t hidden, float* logits) {
  lm_head_q4(x, packed, scales, vocab, hidden, logits);
}
void orc_lm_head_f16(const float* x, const uint16_t* w, size_t vocab, size_t hidden,
                     float* logits) {
  lm_head_f16(x, w, vocab, hidden, logits);
}
uint32_t orc_argmax(const float* logits, size_t n) {
  size_t best = 0;
  float mx = -INFINITY;
  for (size_t i = 0; i < n; ++i)
    if (logits[i] > mx) { mx = logits[i]; best = i; }
  return (uint32_t)best;
}

// Rng::next_f32 (src/generate.rs:54-60): xorshift64, top 24 bits / 2^24
float orc_rng_next_f32(uint64_t* state) {
  uint64_t s = *state;
  s ^= s << 13;
  s ^= s >> 7;
  s ^= s << 17;
  *state = s;
  return (float)(s >> 40) / 16777216.0f;
}

// apply_repetition_penalty (src/generate.rs:64-79): every occurrence in the last 64
// history tokens, in order
void orc_repetition_penalty(float* logits, size_t n, const uint32_t* hist, size_t nh, float penalty) {
  if (penalty <= 1.0f) return;
  const size_t window = std::min<size_t>(nh, 64);
  for (size_t i = nh - window; i < nh; ++i) {
    const size_t idx = hist[i];
    if (idx < n) {
      if (logits[idx] > 0.0f)
        logits[idx] /= penalty;
      else
        logits[idx] *= penalty;
    }
  }
}

// apply_presence_penalty (src/generate.rs:82-92): once per distinct history token
void orc_presence_penalty(float* logits, size_t n, const uint32_t* hist, size_t nh, float penalty) {
  if (penalty <= 0.0f || nh == 0) return;
  std::vector<bool> seen(n, false);
  for (size_t i = 0; i < nh; ++i)
    if (hist[i] < n) seen[hist[i]] = true;
  for (size_t i = 0; i < n; ++i)
    if (seen[i]) logits[i] -= penalty;
}

// sample_token_top_k (src/generate.rs:345-394): greedy when temperature <= 0, else
// top-k by a stable descending sort, softmax at 1/temperature against the global
// maximum, top-p cut on the cumulative sum, one draw of the generator.
uint32_t orc_sample_top_k(const float* logits, size_t n, float temperature, float top_p, size_t top_k,
                          uint64_t* state) {
  if (temperature <= 0.0f) return orc_argmax(logits, n);
  const float inv_temp = 1.0f / temperature;
  float max_logit = -INFINITY;
  for (size_t i = 0; i < n; ++i) max_logit = std::fmax(max_logit, logits[i]);
  std::vector<std::pair<uint32_t, float>> idx(n);
  for (size_t i = 0; i < n; ++i) idx[i] = {(uint32_t)i, logits[i]};
  std::stable_sort(idx.begin(), idx.end(), [](const std::pair<uint32_t, float>& a,
                                              const std::pair<uint32_t, float>& b) { return a.second > b.second; });
  const size_t k = top_k > 0 ? std::min(top_k, n) : n;
  std::vector<std::pair<uint32_t, float>> probs(k);
  for (size_t i = 0; i < k; ++i) probs[i] = {idx[i].first, std::exp((idx[i].second - max_logit) * inv_temp)};
  float sum = 0.0f;
  for (auto& p : probs) sum += p.second;
  if (sum <= 0.0f) return probs[0].first;
  const float inv = 1.0f / sum;
  for (auto& p : probs) p.second *= inv;
  float cumsum = 0.0f;
  size_t cutoff = probs.size();
  for (size_t i = 0; i < probs.size(); ++i) {
    cumsum += probs[i].second;
    if (cumsum >= top_p) {
      cutoff = i + 1;
      break;
    }
  }
  float total = 0.0f;
  for (size_t i = 0; i < cutoff; ++i) total += probs[i].second;
  if (total <= 0.0f) return probs[0].first;
  const float rand_val = orc_rng_next_f32(state) * total;
  float accum = 0.0f;
  for (size_t i = 0; i < cutoff; ++i) {
    accum += probs[i].second;
    if (accum >= rand_val) return probs[i].first;
  }
  return probs[0].first;
}

// One sampling step of the generation loop (src/generate.rs:216-235, final-answer branch
// and the thinking branch's banned token): penalties on a copy, then sample_token_top_k.
uint32_t orc_sample(const float* logits, size_t n, const uint32_t* hist, size_t nh, float temperature, float top_p,
                    size_t top_k, float repetition_penalty, float presence_penalty, int64_t ban, uint64_t* state) {
  std::vector<float> l(logits, logits + n);
  orc_repetition_penalty(l.data(), n, hist, nh, repetition_penalty);
  orc_presence_penalty(l.data(), n, hist, nh, presence_penalty);
  if (ban >= 0 && (size_t)ban < n) l[ban] = -INFINITY;
  return orc_sample_top_k(l.data(), n, temperature, top_p, top_k, state);
}

int orc_layer_forward(const orc_model* m, uint32_t li, float* x, orc_kv* kv) {
  if (li >= m->num_layers) return 1;
  const Layer& L = m->layers[li];
  const size_t H = m->hidden;
  const size_t nh = L.num_heads, nkv = L.num_kv_heads, hd = L.head_dim, grp = L.num_kv_groups;
  const size_t kv_stride = nkv * hd;
  std::vector<float> xn(H), q(L.w[0].n), kn(L.w[1].n), vn(L.w[2].n);
  rms_norm(x, L.g_in.data(), H, xn.data());
  gemv(xn.data(), L.w[0], q.data());
  gemv(xn.data(), L.w[1], kn.data());
  gemv(xn.data(), L.w[2], vn.data());
  const size_t pos = kv->len[li];
  if (m->use_rope[li]) {
    if ((pos + 1) * m->half_dim > m->cos_t.size()) return 2;
    rope(q.data(), nh, hd, m->cos_t.data(), m->sin_t.data(), m->half_dim, pos);
    rope(kn.data(), nkv, hd, m->cos_t.data(), m->sin_t.data(), m->half_dim, pos);
  }
  if (kv->f16) {
    for (float& t : kn) t = round_f16(t);
    for (float& t : vn) t = round_f16(t);
  }
  kv->k[li].insert(kv->k[li].end(), kn.begin(), kn.end());
  kv->v[li].insert(kv->v[li].end(), vn.begin(), vn.end());
  kv->len[li] = (uint32_t)(pos + 1);
  const size_t kv_len = pos + 1;
  const float scale = 1.0f / std::sqrt((float)hd);
  std::vector<float> attn(nh * hd, 0.0f);
  const float* K = kv->k[li].data();
  const float* V = kv->v[li].data();
  // heads in parallel once kv_len >= 64 (src/gemv.rs:918); each head is independent,
  // so the result does not depend on the split
  parallel_for((long)nh, kv_len >= 64, [&](long h) {
    attend_head(q.data() + h * hd, K, V, kv_len, kv_stride, (size_t)h / grp, hd, scale,
                attn.data() + h * hd);
  });
  std::vector<float> o(L.w[3].n);
  gemv(attn.data(), L.w[3], o.data());
  for (size_t j = 0; j < H; ++j) x[j] += o[j];
  rms_norm(x, L.g_post.data(), H, xn.data());
  std::vector<float> inter(L.w[4].n);
  fused_gate_up(xn.data(), L.w[4], L.w[5], inter.data());
  std::vector<float> mlp(L.w[6].n);
  gemv(inter.data(), L.w[6], mlp.data());
  for (size_t j = 0; j < H; ++j) x[j] += mlp[j];
  return 0;
}

int orc_forward_decode(const orc_model* m, uint32_t token, orc_kv* kv, float* logits) {
  if (token >= m->vocab) return 1;
  std::vector<float> x(m->hidden);
  embed(m, token, x.data());
  for (uint32_t i = 0; i < m->num_layers; ++i) {
    const int rc = orc_layer_forward(m, i, x.data(), kv);
    if (rc) return rc;
  }
  std::vector<float> xn(m->hidden);
  rms_norm(x.data(), m->final_norm.data(), m->hidden, xn.data());
  lm_head(m, xn.data(), logits);
  return 0;
}

int orc_prefill(const orc_model* m, const uint32_t* ids, size_t n, orc_kv* kv, float* logits) {
  if (n == 0) return 1;
  const size_t H = m->hidden;
  std::vector<float> x(n * H);
  for (size_t t = 0; t < n; ++t) {
    if (ids[t] >= m->vocab) return 1;
    embed(m, ids[t], x.data() + t * H);
  }
  std::vector<float> xn(n * H);
  for (uint32_t li = 0; li < m->num_layers; ++li) {
    const Layer& L = m->layers[li];
    const size_t nh = L.num_heads, nkv = L.num_kv_heads, hd = L.head_dim, grp = L.num_kv_groups;
    const size_t qs = nh * hd, ks = nkv * hd;
    for (size_t t = 0; t < n; ++t) rms_norm(x.data() + t * H, L.g_in.data(), H, xn.data() + t * H);
    std::vector<float> qa(n * L.w[0].n), ka(n * L.w[1].n), va(n * L.w[2].n);
    gemm(xn.data(), n, L.w[0], qa.data());
    gemm(xn.data(), n, L.w[1], ka.data());
    gemm(xn.data(), n, L.w[2], va.data());
    if (m->use_rope[li]) {
      if (n * m->half_dim > m->cos_t.size()) return 2;
      for (size_t t = 0; t < n; ++t) {
        rope(qa.data() + t * qs, nh, hd, m->cos_t.data(), m->sin_t.data(), m->half_dim, t);
        rope(ka.data() + t * ks, nkv, hd, m->cos_t.data(), m->sin_t.data(), m->half_dim, t);
      }
    }
    if (kv->f16) {  // every position attends to the cached (rounded) keys and values
      for (float& t : ka) t = round_f16(t);
      for (float& t : va) t = round_f16(t);
    }
    const float scale = 1.0f / std::sqrt((float)hd);
    std::vector<float> attn(n * qs, 0.0f);
    parallel_for((long)nh, true, [&](long h) {
      std::vector<float> head(hd);
      for (size_t t1 = 0; t1 < n; ++t1) {
        std::fill(head.begin(), head.end(), 0.0f);
        attend_head(qa.data() + t1 * qs + h * hd, ka.data(), va.data(), t1 + 1, ks,
                    (size_t)h / grp, hd, scale, head.data());
        std::memcpy(attn.data() + t1 * qs + h * hd, head.data(), hd * 4);
      }
    });
    std::vector<float> o(n * L.w[3].n);
    gemm(attn.data(), n, L.w[3], o.data());
    for (size_t j = 0; j < n * H; ++j) x[j] += o[j];
    for (size_t t = 0; t < n; ++t) rms_norm(x.data() + t * H, L.g_post.data(), H, xn.data() + t * H);
    const size_t I = L.w[4].n;
    std::vector<float> g(n * I), u(n * I), inter(n * I);
    gemm(xn.data(), n, L.w[4], g.data());
    gemm(xn.data(), n, L.w[5], u.data());
    for (size_t j = 0; j < n * I; ++j) inter[j] = silu_mul(g[j], u[j]);
    std::vector<float> d(n * L.w[6].n);
    gemm(inter.data(), n, L.w[6], d.data());
    for (size_t j = 0; j < n * H; ++j) x[j] += d[j];
    kv->k[li] = std::move(ka);
    kv->v[li] = std::move(va);
    kv->len[li] = (uint32_t)n;
  }
  std::vector<float> last(H);
  rms_norm(x.data() + (n - 1) * H, m->final_norm.data(), H, last.data());
  lm_head(m, last.data(), logits);
  return 0;
}

static float top2_margin(const float* l, size_t n) {
  float a = -INFINITY, b = -INFINITY;
  for (size_t i = 0; i < n; ++i) {
    if (l[i] > a) { b = a; a = l[i]; }
    else if (l[i] > b) b = l[i];
  }
  return a - b;
}

int orc_generate_greedy(const orc_model* m, const uint32_t* prompt, size_t n_prompt,
                        size_t n_new, orc_kv* kv, uint32_t* tokens, float* margins) {
  std::vector<float> logits(m->vocab);
  int rc = orc_prefill(m, prompt, n_prompt, kv, logits.data());
  if (rc) return rc;
  for (size_t i = 0; i < n_new; ++i) {
    if (i > 0) {
      rc = orc_forward_decode(m, tokens[i - 1], kv, logits.data());
      if (rc) return rc;
    }
    tokens[i] = orc_argmax(logits.data(), m->vocab);
    if (margins) margins[i] = top2_margin(logits.data(), m->vocab);
  }
  return 0;
}

}  // extern "C"
