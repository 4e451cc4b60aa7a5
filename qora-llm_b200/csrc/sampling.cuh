// sampling.cuh — one token from a row of logits on the device: the reference's
// sampling step (src/generate.rs:216-235) without copying the logits to the host.
//
//   penalties   apply_repetition_penalty (every occurrence among the last 64 history
//               tokens, in order; src/generate.rs:64-79), apply_presence_penalty (once
//               per distinct history token; :82-92), an optional banned token (-inf)
//   greedy      temperature <= 0: first maximum (:346-352)
//   top-k       the k best (value descending, lower index first — the order of the
//               reference's stable sort) by k rounds of a block-wide "next best" search
//   top-p       softmax at 1/temperature against the global maximum over the k, then
//               the cumulative cut, the xorshift64 draw and the scan, sequentially in
//               the reference's order (:355-394)
//
// One CTA of 1024 threads per call; k <= kMaxTopK. The generator state is passed in
// and the advanced state written back, so the host's sequence of draws matches the
// reference's (a draw happens only when the scan is reached).
#pragma once

#include "common.cuh"

namespace qora {
namespace smp {

constexpr int kThreads = 1024;
constexpr int kMaxTopK = 1024;
constexpr int kMaxVocabBits = 1 << 18;  // presence bitmap capacity (tokens)

struct Params {
  float temperature;
  float top_p;
  int top_k;               // 1..kMaxTopK (already clamped to the vocabulary)
  float repetition_penalty;
  float presence_penalty;
  int ban;                 // -1: none
};

struct Out {
  unsigned token;
  unsigned pad;
  unsigned long long state;
};

// strict "a before b" in the reference's sorted order: larger value, then lower index
QORA_DEV bool before(float va, unsigned ia, float vb, unsigned ib) { return va > vb || (va == vb && ia < ib); }

// block-wide best (value, index) under `before`; every thread gets the result
QORA_DEV void block_best(float& v, unsigned& i, float* sv, unsigned* si) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const unsigned oi = __shfl_xor_sync(0xffffffffu, i, o);
    if (before(ov, oi, v, i)) {
      v = ov;
      i = oi;
    }
  }
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = i;
  }
  __syncthreads();
  if (warp == 0) {
    v = sv[lane];
    i = si[lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const unsigned oi = __shfl_xor_sync(0xffffffffu, i, o);
      if (before(ov, oi, v, i)) {
        v = ov;
        i = oi;
      }
    }
    if (lane == 0) {
      sv[0] = v;
      si[0] = i;
    }
  }
  __syncthreads();
  v = sv[0];
  i = si[0];
  __syncthreads();
}

// work: [V] scratch (the penalised copy of the logits)
__global__ void __launch_bounds__(kThreads) sample_kernel(const float* logits, int V, const unsigned* hist, int nh,
                                                          Params p, unsigned long long state, float* work,
                                                          Out* out) {
  __shared__ unsigned seen[kMaxVocabBits / 32];
  __shared__ float sv[32];
  __shared__ unsigned si[32];
  __shared__ float cv[kMaxTopK];
  __shared__ unsigned ci[kMaxTopK];
  __shared__ int s_found;
  const int tid = threadIdx.x;
  for (int i = tid; i < V; i += kThreads) work[i] = logits[i];
  const bool presence = p.presence_penalty > 0.0f && nh > 0;
  if (presence)
    for (int w = tid; w < (V + 31) / 32; w += kThreads) seen[w] = 0u;
  __syncthreads();
  if (presence)
    for (int i = tid; i < nh; i += kThreads)
      if (hist[i] < (unsigned)V) atomicOr(&seen[hist[i] >> 5], 1u << (hist[i] & 31));
  if (tid == 0 && p.repetition_penalty > 1.0f) {  // in history order: duplicates compound
    const int window = nh < 64 ? nh : 64;
    for (int k = nh - window; k < nh; ++k) {
      const unsigned idx = hist[k];
      if (idx < (unsigned)V) {
        const float x = work[idx];
        work[idx] = x > 0.0f ? __fdiv_rn(x, p.repetition_penalty) : __fmul_rn(x, p.repetition_penalty);
      }
    }
  }
  __syncthreads();
  if (presence)
    for (int i = tid; i < V; i += kThreads)
      if (seen[i >> 5] & (1u << (i & 31))) work[i] = __fsub_rn(work[i], p.presence_penalty);
  __syncthreads();
  if (tid == 0 && p.ban >= 0 && p.ban < V) work[p.ban] = -INFINITY;
  __syncthreads();

  if (p.temperature <= 0.0f) {  // greedy: first strict maximum, index 0 if none
    float bv = -INFINITY;
    unsigned bi = 0xFFFFFFFFu;
    for (int i = tid; i < V; i += kThreads)
      if (better(work[i], (unsigned)i, bv, bi)) {
        bv = work[i];
        bi = (unsigned)i;
      }
    block_best(bv, bi, sv, si);
    if (tid == 0) {
      out->token = bi == 0xFFFFFFFFu ? 0u : bi;
      out->state = state;
    }
    return;
  }
  // global maximum (NaN ignored, as f32::max does)
  float mx = -INFINITY;
  for (int i = tid; i < V; i += kThreads) mx = fmaxf(mx, work[i]);
  {
    float m2 = mx;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
    if ((tid & 31) == 0) sv[tid >> 5] = m2;
    __syncthreads();
    if (tid < 32) {
      m2 = sv[tid];
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) m2 = fmaxf(m2, __shfl_xor_sync(0xffffffffu, m2, o));
      if (tid == 0) sv[0] = m2;
    }
    __syncthreads();
    mx = sv[0];
    __syncthreads();
  }
  // the k best in the reference's order: each round, the best element strictly after the
  // previous pick
  float lv = INFINITY;
  unsigned li = 0u;
  bool first = true;
  if (tid == 0) s_found = 0;
  for (int r = 0; r < p.top_k; ++r) {
    float bv = -INFINITY;
    unsigned bi = 0xFFFFFFFFu;
    for (int i = tid; i < V; i += kThreads) {
      const float x = work[i];
      if (x != x) continue;  // NaN never ranks
      const bool after = first || before(lv, li, x, (unsigned)i);
      if (after && (bi == 0xFFFFFFFFu || before(x, (unsigned)i, bv, bi))) {
        bv = x;
        bi = (unsigned)i;
      }
    }
    block_best(bv, bi, sv, si);
    if (bi == 0xFFFFFFFFu) break;
    if (tid == 0) {
      cv[r] = bv;
      ci[r] = bi;
      s_found = r + 1;
    }
    lv = bv;
    li = bi;
    first = false;
  }
  __syncthreads();
  if (tid == 0) {
    // candidates found (fewer than top_k only when the row has fewer non-NaN entries)
    const int kk = s_found;
    if (kk == 0) {
      out->token = 0u;
      out->state = state;
      return;
    }
    const float inv_temp = __fdiv_rn(1.0f, p.temperature);
    float sum = 0.0f;
    for (int j = 0; j < kk; ++j) {
      cv[j] = expf(__fmul_rn(__fsub_rn(cv[j], mx), inv_temp));
      sum = __fadd_rn(sum, cv[j]);
    }
    unsigned tok = ci[0];
    unsigned long long s = state;
    if (sum > 0.0f) {
      const float inv = __fdiv_rn(1.0f, sum);
      for (int j = 0; j < kk; ++j) cv[j] = __fmul_rn(cv[j], inv);
      float cumsum = 0.0f;
      int cutoff = kk;
      for (int j = 0; j < kk; ++j) {
        cumsum = __fadd_rn(cumsum, cv[j]);
        if (cumsum >= p.top_p) {
          cutoff = j + 1;
          break;
        }
      }
      float total = 0.0f;
      for (int j = 0; j < cutoff; ++j) total = __fadd_rn(total, cv[j]);
      if (total > 0.0f) {
        s ^= s << 13;  // Rng::next_f32 (src/generate.rs:54-60)
        s ^= s >> 7;
        s ^= s << 17;
        const float rnd = __fmul_rn(__fdiv_rn((float)(s >> 40), 16777216.0f), total);
        float accum = 0.0f;
        for (int j = 0; j < cutoff; ++j) {
          accum = __fadd_rn(accum, cv[j]);
          if (accum >= rnd) {
            tok = ci[j];
            break;
          }
        }
      }
    }
    out->token = tok;
    out->state = s;
  }
}

}  // namespace smp
}  // namespace qora
