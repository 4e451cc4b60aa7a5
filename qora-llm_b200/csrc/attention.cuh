// attention.cuh — GQA decode attention over the f32 KV cache (src/gemv.rs:914-989,
// softmax_raw :782-793), split over the sequence ("flash-decoding"): CTA (j, c) handles
// KV head j and the c-th chunk of the filled positions for the kGrp query heads that
// share it, producing an unnormalised partial (running max m, sum l, o = sum e^(s-m) v).
// The last CTA of head j merges the chunk partials in chunk order (deterministic).
#pragma once

#include "common.cuh"

namespace qora {

constexpr int kAttnThreads = 128;   // one thread per head dim in the P.V phase
constexpr int kAttnMaxChunk = 2048; // positions per CTA (score buffer capacity)
constexpr int kGrp = 4;             // query heads per KV head (num_kv_groups)

struct AttnArgs {
  const float* q;      // [nh * 128] (RoPE applied)
  const float* kc;     // layer K cache, head-major [nkv][max_seq][128]
  const float* vc;
  long long hs;        // head stride (max_seq * 128)
  float* out;          // [nh * 128]
  const StepState* st; // length = st->pos + 1 (the row appended by this step included)
  int nkv;             // KV heads in this cache
  int nc;              // chunks (gridDim.y)
  float scale;         // 1/sqrt(head_dim)
  float* part_o;       // [nkv][nc][kGrp][128]
  float* part_ml;      // [nkv][nc][kGrp][2]
  unsigned* counters;  // [nkv]
};

__global__ void __launch_bounds__(kAttnThreads) attn_decode_kernel(const AttnArgs a) {
  __shared__ float qs[kGrp][kHeadDim];
  __shared__ float sc[kGrp][kAttnMaxChunk];
  __shared__ float s_m[kGrp], s_l[kGrp];
  __shared__ int s_last;

  const int j = blockIdx.x, c = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = a.st->pos + 1;
  const int chunk = (len + a.nc - 1) / a.nc;
  const int s0 = min(len, c * chunk);
  const int s1 = min(len, s0 + chunk);
  const int n = s1 - s0;

  for (int i = tid; i < kGrp * kHeadDim; i += kAttnThreads)
    qs[i / kHeadDim][i % kHeadDim] = a.q[(j * kGrp) * kHeadDim + i];
  __syncthreads();

  // scores: warp w takes positions s0+w, s0+w+4, ...; lane covers dims 4*lane..4*lane+3
  for (int s = s0 + warp; s < s1; s += kAttnThreads / 32) {
    const float4 k4 = __ldg(reinterpret_cast<const float4*>(a.kc + j * a.hs + (long long)s * kHeadDim) + lane);
#pragma unroll
    for (int h = 0; h < kGrp; ++h) {
      const float4 q4 = *reinterpret_cast<const float4*>(&qs[h][lane * 4]);
      float d = q4.x * k4.x;
      d = __fmaf_rn(q4.y, k4.y, d);
      d = __fmaf_rn(q4.z, k4.z, d);
      d = __fmaf_rn(q4.w, k4.w, d);
      d = warp_sum(d);
      if (lane == 0) sc[h][s - s0] = __fmul_rn(d, a.scale);
    }
  }
  __syncthreads();

  // chunk-local softmax numerators: warp h owns query head h
  {
    const int h = warp;
    float m = -INFINITY;
    for (int i = lane; i < n; i += 32) m = fmaxf(m, sc[h][i]);
    m = warp_max(m);
    float l = 0.0f;
    for (int i = lane; i < n; i += 32) {
      const float e = expf(sc[h][i] - m);
      sc[h][i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      s_m[h] = (n > 0) ? m : -INFINITY;
      s_l[h] = (n > 0) ? l : 0.0f;
    }
  }
  __syncthreads();

  // P.V: thread d accumulates dim d for the kGrp heads
  {
    const int d = tid;
    float o[kGrp] = {0.0f, 0.0f, 0.0f, 0.0f};
    const float* vp = a.vc + j * a.hs + (long long)s0 * kHeadDim + d;
    for (int i = 0; i < n; ++i) {
      const float v = __ldg(vp + (long long)i * kHeadDim);
#pragma unroll
      for (int h = 0; h < kGrp; ++h) o[h] = __fmaf_rn(sc[h][i], v, o[h]);
    }
    const long long base = ((long long)j * a.nc + c) * kGrp;
#pragma unroll
    for (int h = 0; h < kGrp; ++h) __stcg(a.part_o + (base + h) * kHeadDim + d, o[h]);
    if (d < kGrp) {
      __stcg(a.part_ml + (base + d) * 2 + 0, s_m[d]);
      __stcg(a.part_ml + (base + d) * 2 + 1, s_l[d]);
    }
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_last = (atomicAdd(a.counters + j, 1u) == (unsigned)(a.nc - 1));
  __syncthreads();
  if (!s_last) return;
  __threadfence();

  // merge the nc chunk partials of KV head j (chunk order)
  const int d = tid;
#pragma unroll
  for (int h = 0; h < kGrp; ++h) {
    float M = -INFINITY;
    for (int k = 0; k < a.nc; ++k) {
      const long long b = ((long long)j * a.nc + k) * kGrp + h;
      M = fmaxf(M, __ldcg(a.part_ml + b * 2));
    }
    float L = 0.0f, O = 0.0f;
    for (int k = 0; k < a.nc; ++k) {
      const long long b = ((long long)j * a.nc + k) * kGrp + h;
      const float l = __ldcg(a.part_ml + b * 2 + 1);
      if (l == 0.0f) continue;
      const float w = expf(__ldcg(a.part_ml + b * 2) - M);
      L = __fmaf_rn(l, w, L);
      O = __fmaf_rn(__ldcg(a.part_o + b * kHeadDim + d), w, O);
    }
    a.out[(j * kGrp + h) * kHeadDim + d] = __fmul_rn(O, __fdiv_rn(1.0f, L));
  }
  if (tid == 0) a.counters[j] = 0u;
}

}  // namespace qora
