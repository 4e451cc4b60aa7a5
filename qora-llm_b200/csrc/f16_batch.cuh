// f16_batch.cuh — the per-row kernels of F16-weight decode and prefill for M "rows" at
// once (batched decode of independent sequences; prompt prefill). A
// row is one token of one sequence at one position; a batched decode step has one row
// per sequence, a prefill chunk one row per prompt token of a sequence. Per layer:
//
//   umma::norm_split_tiled  RMSNorm (optional) of each row into the tensor-core operand
//   umma::umma_gemm_kernel  q|k|v, o, gate|up, down and the tied lm_head on tcgen05
//   umma::reduce_tiles      partial slots summed (+ residual, or SwiGLU)
//   rope_kv                 RoPE on q/k at each row's position, k/v appended to its cache
//   attention_rows          causal attention of each row over its sequence's cache prefix
//   argmax_rows             first maximum per row
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "umma_gemm.cuh"

namespace qora {
namespace f16b {

constexpr int kMaxRows = umma::kMaxRows;  // rows per step (prefill chunk / batch)

// ---------------------------------------------------------------- per-row helpers
// Row table in device memory (one per KV cache): seq | pos | token, kMaxRows ints each,
// then the greedy step counter and an error flag. Kernels read it at run time, so one
// captured graph serves every step.
struct RowInfo {
  int* seq;    // [M] sequence of each row
  int* pos;    // [M] position of each row
  int* token;  // [M] token id of each row (embedding)
  int* step;   // greedy step counter (ring row)
  int* error;  // nonzero: a token id was out of range
};
constexpr int kRowInts = 3 * kMaxRows + 2;
__host__ __device__ inline RowInfo row_info(int* base) {
  return RowInfo{base, base + kMaxRows, base + 2 * kMaxRows, base + 3 * kMaxRows, base + 3 * kMaxRows + 1};
}

// x[m] = f32(E[token[m]]) (embed_lookup, src/gemv.rs:515-526), read from the tiled
// embedding (umma tile layout, n = vocab, k = hidden). One CTA per row.
__global__ void embed_rows_kernel(const uint8_t* emb_t, int H, int vocab, RowInfo ri, float* x) {
  const int m = blockIdx.x;
  const int tok = ri.token[m];
  if (tok < 0 || tok >= vocab) {  // the host validates ids; this keeps the read in bounds
    if (threadIdx.x == 0) *ri.error = 1;
    return;
  }
  const int chunks = H / umma::kChunkK, t = tok / umma::kTileN, o = tok % umma::kTileN;
  for (int g = threadIdx.x; g < H / 8; g += blockDim.x) {
    const int k = g * 8;
    const uint8_t* p = emb_t + ((size_t)t * chunks + k / umma::kChunkK) * umma::kATile + umma::tile_off(o, k % umma::kChunkK);
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const __half* h = reinterpret_cast<const __half*>(&v);
#pragma unroll
    for (int i = 0; i < 8; ++i) x[(long long)m * H + k + i] = __half2float(h[i]);
  }
}

// End of a batched greedy step: each row's greedy token becomes its next input, its
// position advances, and the token is recorded at ring[step][m].
__global__ void advance_rows_kernel(int M, RowInfo ri, const unsigned* am, unsigned* ring, int ring_rows) {
  const int m = threadIdx.x;
  const int s = *ri.step;
  if (m < M) {
    if (ring && s >= 0 && s < ring_rows) ring[(long long)s * M + m] = am[m];
    ri.token[m] = (int)am[m];
    ri.pos[m] += 1;
  }
  __syncthreads();
  if (m == 0) *ri.step = s + 1;
}

// RoPE on q and k of each row at its position (layers with the flag; src/gemv.rs:757-778),
// then k and v appended to the row's sequence cache, head-major [kvh][max_seq][128] per
// sequence (sequence stride seq_stride floats).
__global__ void rope_kv_kernel(float* qkv, int nq, int nkvw, int rope, const float* cos_t, const float* sin_t,
                               RowInfo ri, float* kc, float* vc, long long seq_stride, long long head_stride) {
  const int m = blockIdx.x, pos = ri.pos[m];
  float* row = qkv + (long long)m * (nq + 2 * nkvw);
  const int pairs = (nq + nkvw) / 2;  // (d, d+64) pairs of the q and k heads
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const int h = i / kHalfDim, d = i % kHalfDim, c = h * kHeadDim + d;
    float* p = row + c;
    const float x1 = p[0], x2 = p[kHalfDim];
    float y1 = x1, y2 = x2;
    if (rope) {
      const float cs = cos_t[(long long)pos * kHalfDim + d], sn = sin_t[(long long)pos * kHalfDim + d];
      y1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      y2 = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
    }
    p[0] = y1;
    p[kHalfDim] = y2;
  }
  __syncthreads();
  float* kd = kc + (long long)ri.seq[m] * seq_stride;
  float* vd = vc + (long long)ri.seq[m] * seq_stride;
  for (int i = threadIdx.x; i < nkvw; i += blockDim.x) {
    const int j = i / kHeadDim, d = i % kHeadDim;
    kd[j * head_stride + (long long)pos * kHeadDim + d] = row[nq + i];
    vd[j * head_stride + (long long)pos * kHeadDim + d] = row[nq + nkvw + i];
  }
}

// Attention of row m's query heads of KV head j over positions [0, pos[m]] of its
// sequence (decode attention, src/gemv.rs:914-989; softmax_raw :782-793): scores in
// chunks of 256 with a running maximum, normalised at the end. One CTA per (j, m).
constexpr int kAttnRowThreads = 128;
__global__ void __launch_bounds__(kAttnRowThreads)
    attention_rows_kernel(const float* qkv, int nq, int nkvw, int grp, RowInfo ri, const float* kc,
                          const float* vc, long long seq_stride, long long head_stride, float* out) {
  __shared__ float qs[4][kHeadDim];
  __shared__ float sc[4][256];
  __shared__ float s_m[4], s_l[4], s_a[4];
  const int j = blockIdx.x, m = blockIdx.y;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = ri.pos[m] + 1;
  const float* q = qkv + (long long)m * (nq + 2 * nkvw) + (long long)j * grp * kHeadDim;
  const float* K = kc + (long long)ri.seq[m] * seq_stride + j * head_stride;
  const float* V = vc + (long long)ri.seq[m] * seq_stride + j * head_stride;
  const float scale = 0.08838834764831845f;  // 1/sqrt(128): the f32 quotient of 1 and f32 sqrt(128)
  for (int i = tid; i < grp * kHeadDim; i += kAttnRowThreads) qs[i / kHeadDim][i % kHeadDim] = q[i];
  if (tid < 4) {
    s_m[tid] = -INFINITY;
    s_l[tid] = 0.0f;
  }
  float o[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  __syncthreads();
  for (int s0 = 0; s0 < len; s0 += 256) {
    const int n = min(256, len - s0);
    // scores: warp w takes positions s0+w, +4, ...; lanes split the 128 dims
    for (int s = warp; s < n; s += 4) {
      const float4 k4 = reinterpret_cast<const float4*>(K + (long long)(s0 + s) * kHeadDim)[lane];
      for (int h = 0; h < grp; ++h) {
        const float4 q4 = reinterpret_cast<const float4*>(qs[h])[lane];
        float d = q4.x * k4.x;
        d = __fmaf_rn(q4.y, k4.y, d);
        d = __fmaf_rn(q4.z, k4.z, d);
        d = __fmaf_rn(q4.w, k4.w, d);
        d = warp_sum(d);
        if (lane == 0) sc[h][s] = __fmul_rn(d, scale);
      }
    }
    __syncthreads();
    // running softmax per head (warp h)
    if (warp < grp) {
      const int h = warp;
      float mx = s_m[h];
      for (int i = lane; i < n; i += 32) mx = fmaxf(mx, sc[h][i]);
      mx = warp_max(mx);
      float l = 0.0f;
      for (int i = lane; i < n; i += 32) {
        const float e = expf(sc[h][i] - mx);
        sc[h][i] = e;
        l += e;
      }
      l = warp_sum(l);
      if (lane == 0) {
        const float a = expf(s_m[h] - mx);  // rescale of what was accumulated so far
        s_a[h] = a;
        s_l[h] = __fmaf_rn(s_l[h], a, l);
        s_m[h] = mx;
      }
    }
    __syncthreads();
    // P.V: thread d accumulates dim d of the grp heads
    {
      const int d = tid;
      for (int h = 0; h < grp; ++h) o[h] = __fmul_rn(o[h], s_a[h]);
      for (int i = 0; i < n; ++i) {
        const float v = V[(long long)(s0 + i) * kHeadDim + d];
        for (int h = 0; h < grp; ++h) o[h] = __fmaf_rn(sc[h][i], v, o[h]);
      }
    }
    __syncthreads();
  }
  float* dst = out + (long long)m * nq + (long long)j * grp * kHeadDim;
  for (int h = 0; h < grp; ++h) dst[h * kHeadDim + tid] = __fmul_rn(o[h], __fdiv_rn(1.0f, s_l[h]));
}

// First maximum of each row of logits (src/generate.rs:346-352); one CTA per row.
__global__ void argmax_rows_kernel(const float* logits, int V, unsigned* out) {
  __shared__ float bv[8];
  __shared__ unsigned bi[8];
  const int m = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const float* row = logits + (long long)m * V;
  float best = -INFINITY;
  unsigned besti = 0xFFFFFFFFu;
  for (int v = tid; v < V; v += blockDim.x)
    if (better(row[v], (unsigned)v, best, besti)) {
      best = row[v];
      besti = (unsigned)v;
    }
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, best, o);
    const unsigned oi = __shfl_xor_sync(0xffffffffu, besti, o);
    if (better(ov, oi, best, besti)) {
      best = ov;
      besti = oi;
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
    for (int w = 1; w < (int)(blockDim.x / 32); ++w)
      if (better(bv[w], bi[w], b, i0)) {
        b = bv[w];
        i0 = bi[w];
      }
    out[m] = (i0 == 0xFFFFFFFFu) ? 0u : i0;
  }
}

}  // namespace f16b
}  // namespace qora
