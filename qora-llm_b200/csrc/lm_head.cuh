// lm_head.cuh — tied-embedding lm_head over the Q4 [vocab][hidden] table as row dot
// products (lm_head_parallel_q4, src/gemv.rs:825-864) with the greedy argmax fused in
// (src/generate.rs:346-352: first maximum wins). Optional final RMSNorm prologue
// (src/gemv.rs:1015). Rows are split into equal contiguous ranges, one per CTA; a warp
// owns a row at a time, each lane GPL consecutive groups of it.
//
// Per group g: sum_e x_e (q_e - 8) scale_g = scale_g * (sum_e x_e q_e - 8 * X_g), with
// X_g = sum of the group's inputs computed once. The nibble is taken as the subnormal
// q * 2^(p - 149) (see q4_gemv.cuh) and the input pre-scaled by 2^(85 - p), so every
// product is x * q * 2^-64 whatever the nibble position.
#pragma once

#include "common.cuh"

namespace qora {

constexpr int kLmThreads = 256;
constexpr int kLmWarps = kLmThreads / 32;

struct LmArgs {
  const float* x;        // [hidden] input (pre-norm if gamma != nullptr)
  const float* gamma;    // final norm gains (f32) or nullptr
  const uint8_t* packed; // row r packed nibbles at packed + r*row_stride_p (hidden/2 bytes)
  const uint8_t* scales; // row r f16 scales at scales + r*row_stride_s (hidden/32 values)
  long long row_stride_p, row_stride_s;
  int vocab;
  float* logits;         // [vocab] or nullptr
  unsigned* argmax_out;  // one value
  float* part_v;         // [gridDim.x]
  unsigned* part_i;      // [gridDim.x]
  unsigned* counter;     // one value, zero between launches
};

template <int GPL>
__global__ void __launch_bounds__(kLmThreads, 2) lm_head_kernel(const LmArgs a) {
  constexpr int H = GPL * 32 * 32;  // hidden
  constexpr int EPL = GPL * 32;     // elements per lane
  __shared__ float xn[H];
  __shared__ float red[kLmWarps];
  __shared__ float bv[kLmWarps];
  __shared__ unsigned bi[kLmWarps];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  float inv = 1.0f;
  if (a.gamma) inv = rms_inv(a.x, H, red);
  for (int i = tid; i < H; i += kLmThreads)
    xn[i] = a.gamma ? __fmul_rn(__fmul_rn(a.x[i], inv), a.gamma[i]) : a.x[i];
  __syncthreads();

  // lane's inputs, pre-scaled per nibble position, and per-group sums
  float2 xs[EPL / 2];
  float xg[GPL];
#pragma unroll
  for (int g = 0; g < GPL; ++g) {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const float v = xn[lane * EPL + g * 32 + e];
      s += v;
      const int m = e & 7;
      const int p = (m < 5) ? 4 * m : 4 * m - 12;
      const float f = __fmul_rn(v, __int_as_float((127 + 85 - p) << 23));
      if (e & 1) xs[(g * 32 + e) / 2].y = f; else xs[(g * 32 + e) / 2].x = f;
    }
    xg[g] = s * 8.0f;
  }

  const long long r0 = (long long)blockIdx.x * a.vocab / gridDim.x;
  const long long r1 = (long long)(blockIdx.x + 1) * a.vocab / gridDim.x;
  float best = -INFINITY;
  unsigned besti = 0xFFFFFFFFu;
  const float k64 = 18446744073709551616.0f;  // 2^64

  for (long long r = r0 + warp; r < r1; r += kLmWarps) {
    const uint4* wp = reinterpret_cast<const uint4*>(a.packed + r * a.row_stride_p) + lane * GPL;
    const unsigned short* sp = reinterpret_cast<const unsigned short*>(a.scales + r * a.row_stride_s) + lane * GPL;
    uint4 w[GPL];
    unsigned short sc[GPL];
#pragma unroll
    for (int g = 0; g < GPL; ++g) {
      w[g] = __ldg(wp + g);
      sc[g] = __ldg(sp + g);
    }
    float acc = 0.0f;
#pragma unroll
    for (int g = 0; g < GPL; ++g) {
      float2 d = make_float2(0.0f, 0.0f);
      const uint32_t ws[4] = {w[g].x, w[g].y, w[g].z, w[g].w};
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t u = ws[i], b = u >> 12;
        const int base = (g * 32 + i * 8) / 2;
        d = __ffma2_rn(make_float2(__uint_as_float(u & 0xFu), __uint_as_float(u & 0xF0u)), xs[base + 0], d);
        d = __ffma2_rn(make_float2(__uint_as_float(u & 0xF00u), __uint_as_float(u & 0xF000u)), xs[base + 1], d);
        d = __ffma2_rn(make_float2(__uint_as_float(u & 0xF0000u), __uint_as_float(b & 0xF00u)), xs[base + 2], d);
        d = __ffma2_rn(make_float2(__uint_as_float(b & 0xF000u), __uint_as_float(b & 0xF0000u)), xs[base + 3], d);
      }
      const float dot = __fmaf_rn(d.x + d.y, k64, -xg[g]);
      acc = __fmaf_rn(__half2float(__ushort_as_half(sc[g])), dot, acc);
    }
    acc = warp_sum(acc);
    if (lane == 0 && a.logits) a.logits[r] = acc;
    if (better(acc, (unsigned)r, best, besti)) {
      best = acc;
      besti = (unsigned)r;
    }
  }

  if (lane == 0) {
    bv[warp] = best;
    bi[warp] = besti;
  }
  __syncthreads();
  if (tid == 0) {
    float b = bv[0];
    unsigned i0 = bi[0];
    for (int w = 1; w < kLmWarps; ++w)
      if (better(bv[w], bi[w], b, i0)) { b = bv[w]; i0 = bi[w]; }
    __stcg(a.part_v + blockIdx.x, b);
    __stcg(a.part_i + blockIdx.x, i0);
    __threadfence();
    s_last = (atomicAdd(a.counter, 1u) == gridDim.x - 1);
  }
  __syncthreads();
  if (!s_last) return;
  if (tid == 0) {
    __threadfence();
    float b = -INFINITY;
    unsigned i0 = 0xFFFFFFFFu;
    for (unsigned k = 0; k < gridDim.x; ++k) {
      const float v = __ldcg(a.part_v + k);
      const unsigned ii = __ldcg(a.part_i + k);
      if (better(v, ii, b, i0)) { b = v; i0 = ii; }
    }
    *a.argmax_out = (i0 == 0xFFFFFFFFu) ? 0u : i0;  // all NaN / -inf: index 0 like the reference
    *a.counter = 0u;
  }
}

}  // namespace qora
