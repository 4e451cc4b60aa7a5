// f16_batch.cuh — the per-row kernels of F16-weight decode and prefill for M "rows" at
// once (benchmark config 5: batched decode of independent sequences; prompt prefill). A
// row is one token of one sequence at one position; a batched decode step has one row
// per sequence, a prefill chunk one row per prompt token of a sequence. Per layer:
//
//   umma::fused_gemm  RMSNorm + q|k|v GEMM + RoPE + KV-cache append
//   attention_split   causal attention of each row over its sequence's cache prefix
//   umma::fused_gemm  o_proj GEMM + residual
//   umma::fused_gemm  RMSNorm + gate|up GEMM + SwiGLU
//   umma::fused_gemm  down_proj GEMM + residual
// and per step: embed_rows at the start, umma::fused_gemm (final RMSNorm + tied lm_head
// + greedy argmax) at the end, advance_rows between greedy steps.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "umma_gemm.cuh"

namespace qora {
namespace f16b {

constexpr int kMaxRows = umma::kMaxRows;  // rows per step (prefill chunk / batch)
using umma::RowInfo;
using umma::kRowInts;
using umma::row_info;

// x[m] = f32(E[token[m]]) (embed_lookup, src/gemv.rs:515-526), read from the tiled
// embedding (n = vocab, k = hidden), with the per-128-channel statistics (sum of squares,
// max |x|) the first RMSNorm reads; also advances the forward-pass counter. Grid
// (hidden / 128, M), 128 threads.
__global__ void __launch_bounds__(128) embed_rows_kernel(const uint8_t* emb_t, int H, int vocab, RowInfo ri,
                                                          float* x, float* st_ss, float* st_mx, unsigned* epoch) {
  __shared__ float red[2][4];
  const int t = blockIdx.x, m = blockIdx.y, i = threadIdx.x;
  if (t == 0 && m == 0 && i == 0) *epoch += 1u;  // a new forward pass (exchange tags)
  const int tok = ri.token[m];
  if (tok < 0 || tok >= vocab) {  // the host validates ids; this keeps the read in bounds
    if (i == 0 && t == 0) *ri.error = 1;
    return;
  }
  const int chunks = H / umma::kChunkK, k = t * umma::kTileN + i;
  const uint8_t* p = emb_t + ((size_t)(tok / umma::kTileN) * chunks + k / umma::kChunkK) * umma::kATile +
                     umma::tile_off(tok % umma::kTileN, k % umma::kChunkK);
  const float v = __half2float(*reinterpret_cast<const __half*>(p));
  x[(size_t)m * H + k] = v;
  float ss = warp_sum(__fmul_rn(v, v)), mx = warp_max(fabsf(v));
  if ((i & 31) == 0) {
    red[0][i >> 5] = ss;
    red[1][i >> 5] = mx;
  }
  __syncthreads();
  if (i == 0) {
    st_ss[(size_t)t * kMaxRows + m] = __fadd_rn(__fadd_rn(red[0][0], red[0][1]), __fadd_rn(red[0][2], red[0][3]));
    st_mx[(size_t)t * kMaxRows + m] = fmaxf(fmaxf(red[1][0], red[1][1]), fmaxf(red[1][2], red[1][3]));
  }
}

// Q4 weights: x[m] = E[token[m]] from the row-interleaved Q4 table (row r: hidden/2 nibble
// bytes, the low nibble the even element, then hidden/32 f16 scales), each element
// scale * (q - 8) as embed_q4 does (src/gemv.rs:515-526), with the same statistics and
// counter update as embed_rows_kernel. Grid (hidden / 128, M), 128 threads.
__global__ void __launch_bounds__(128) embed_rows_q4_kernel(const uint8_t* table, long long row_bytes, int H, int vocab,
                                                             RowInfo ri, float* x, float* st_ss, float* st_mx,
                                                             unsigned* epoch) {
  __shared__ float red[2][4];
  const int t = blockIdx.x, m = blockIdx.y, i = threadIdx.x;
  if (t == 0 && m == 0 && i == 0) *epoch += 1u;
  const int tok = ri.token[m];
  if (tok < 0 || tok >= vocab) {  // the host validates ids; this keeps the read in bounds
    if (i == 0 && t == 0) *ri.error = 1;
    return;
  }
  const int k = t * umma::kTileN + i;
  const uint8_t* row = table + (size_t)tok * row_bytes;
  const int q = (row[k >> 1] >> (4 * (k & 1))) & 0xF;
  const float sc = __half2float(reinterpret_cast<const __half*>(row + H / 2)[k / 32]);
  const float v = __fmul_rn(sc, (float)(q - 8));
  x[(size_t)m * H + k] = v;
  float ss = warp_sum(__fmul_rn(v, v)), mx = warp_max(fabsf(v));
  if ((i & 31) == 0) {
    red[0][i >> 5] = ss;
    red[1][i >> 5] = mx;
  }
  __syncthreads();
  if (i == 0) {
    st_ss[(size_t)t * kMaxRows + m] = __fadd_rn(__fadd_rn(red[0][0], red[0][1]), __fadd_rn(red[0][2], red[0][3]));
    st_mx[(size_t)t * kMaxRows + m] = fmaxf(fmaxf(red[1][0], red[1][1]), fmaxf(red[1][2], red[1][3]));
  }
}

// End of a batched greedy step: each row's greedy token becomes its next input, its
// position advances, and the token is recorded at ring[step][m].
__global__ void advance_rows_kernel(int M, umma::RowInfo ri, const unsigned* am, unsigned* ring, int ring_rows) {
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

// Attention of row m's 4 query heads of KV head j over positions [0, pos[m]] of its
// sequence (q rows [M][nq] after RoPE; the K/V cache rows already hold position pos[m]).
// Decode attention of the reference (src/gemv.rs:914-989, softmax_raw :782-793), split
// over positions: CTA (j, m, p) takes chunk p of the row's positions (chunk = a multiple
// of 64 sized so that a row has at most kAttSplits chunks) and keeps a running maximum
// over 64-position blocks; the last chunk to finish (per-(m, j) counter, self-resetting)
// merges the chunks in order and writes the normalised output and the row's max |out|
// (the o_proj operand's scale). Grid (kv heads, M, kAttSplits), 128 threads.
constexpr int kAttThreads = 128;
constexpr int kAttSplits = 16;
constexpr int kAttBlock = 64;

struct AttnRowsArgs {
  const float* q;       // [M][nq]
  int nq, nkv;
  int hpk;              // query heads per KV head held here (4; 2 on a rank of 8-way TP)
  RowInfo rows;
  const float* kc;      // this layer's caches [batch][kv heads][max_seq][128]
  const float* vc;
  long long seq_stride, head_stride;
  float* out;           // [M][nq]
  float* st_mx;         // [kv heads][kMaxRows]
  float* o_part;        // [kMaxRows][nkv][kAttSplits][4][128] chunk partials
  float* ml_part;       // [kMaxRows][nkv][kAttSplits][4][2] chunk (max, sum)
  unsigned* cnt;        // [kMaxRows][nkv] arrivals
};

__global__ void __launch_bounds__(kAttThreads) attention_split_kernel(const AttnRowsArgs a) {
  __shared__ __align__(16) float qs[4][kHeadDim];
  __shared__ float sc[4][kAttBlock];
  __shared__ __align__(16) float s_o[4][4][kHeadDim];  // per-warp P.V partials [warp][head][dim]
  __shared__ float s_a[4], s_red[4];
  __shared__ int s_last;
  const int j = blockIdx.x, m = blockIdx.y, p = blockIdx.z;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int len = a.rows.pos[m] + 1;
  const int per = kAttSplits * kAttBlock;
  const int cs = kAttBlock * ((len + per - 1) / per);  // chunk length (multiple of 64)
  const int n = (len + cs - 1) / cs;                    // chunks of this row
  if (p >= n) return;
  const int sb = p * cs, se = min(len, sb + cs);
  const float* K = a.kc + (long long)a.rows.seq[m] * a.seq_stride + j * a.head_stride;
  const float* V = a.vc + (long long)a.rows.seq[m] * a.seq_stride + j * a.head_stride;
  const float scale = 0.08838834764831845f;  // 1/sqrt(128): the f32 quotient of 1 and f32 sqrt(128)
  {
    const float* q = a.q + (size_t)m * a.nq + (size_t)j * a.hpk * kHeadDim;
    for (int i = tid; i < 4 * kHeadDim; i += kAttThreads) qs[i / kHeadDim][i % kHeadDim] = i / kHeadDim < a.hpk ? q[i] : 0.0f;
  }
  float mrun = -INFINITY, lrun = 0.0f;  // held by warp h = head h
  // P.V accumulators: warp w sums its 16 positions of each block, lane l owns dims 4l..4l+3
  float4 o4[4];
#pragma unroll
  for (int h = 0; h < 4; ++h) o4[h] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  __syncthreads();
  const int pi = 16 * warp + (lane & 15), half = lane >> 4;
  for (int s0 = sb; s0 < se; s0 += kAttBlock) {
    const int nn = min(kAttBlock, se - s0);
    // scores: lane -> position s0 + pi, dims [64 half, 64 half + 64); halves combined
    float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    if (pi < nn) {
      const float4* kr = reinterpret_cast<const float4*>(K + (long long)(s0 + pi) * kHeadDim + half * 64);
      float4 kv[16];
#pragma unroll
      for (int i = 0; i < 16; ++i) kv[i] = kr[i];
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float4* qh = reinterpret_cast<const float4*>(&qs[h][half * 64]);
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float4 qv = qh[i];
          acc[h] = __fmaf_rn(qv.x, kv[i].x, acc[h]);
          acc[h] = __fmaf_rn(qv.y, kv[i].y, acc[h]);
          acc[h] = __fmaf_rn(qv.z, kv[i].z, acc[h]);
          acc[h] = __fmaf_rn(qv.w, kv[i].w, acc[h]);
        }
      }
    }
#pragma unroll
    for (int h = 0; h < 4; ++h) acc[h] = __fadd_rn(acc[h], __shfl_xor_sync(0xffffffffu, acc[h], 16));
    if (pi < nn && half == 0) {
#pragma unroll
      for (int h = 0; h < 4; ++h) sc[h][pi] = __fmul_rn(acc[h], scale);
    }
    __syncthreads();
    {  // running softmax of head h = warp
      const int h = warp;
      const float v0 = lane < nn ? sc[h][lane] : -INFINITY, v1 = lane + 32 < nn ? sc[h][lane + 32] : -INFINITY;
      const float mx = warp_max(fmaxf(v0, v1));
      const float mnew = fmaxf(mrun, mx);
      const float e0 = lane < nn ? expf(v0 - mnew) : 0.0f, e1 = lane + 32 < nn ? expf(v1 - mnew) : 0.0f;
      if (lane < nn) sc[h][lane] = e0;
      if (lane + 32 < nn) sc[h][lane + 32] = e1;
      const float l = warp_sum(__fadd_rn(e0, e1));
      const float al = expf(mrun - mnew);  // 0 on the first block
      lrun = __fmaf_rn(lrun, al, l);
      mrun = mnew;
      if (lane == 0) s_a[h] = al;
    }
    __syncthreads();
    {  // P.V: warp w takes positions 16w..16w+15 of the block (loads all in flight)
#pragma unroll
      for (int h = 0; h < 4; ++h) {
        const float al = s_a[h];
        o4[h] = make_float4(__fmul_rn(o4[h].x, al), __fmul_rn(o4[h].y, al), __fmul_rn(o4[h].z, al),
                            __fmul_rn(o4[h].w, al));
      }
      const float4* vr = reinterpret_cast<const float4*>(V + (long long)(s0 + 16 * warp) * kHeadDim) + lane;
      float4 v[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        v[i] = 16 * warp + i < nn ? vr[i * (kHeadDim / 4)] : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll
      for (int i = 0; i < 16; ++i) {
        if (16 * warp + i < nn) {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            const float pw = sc[h][16 * warp + i];
            o4[h].x = __fmaf_rn(pw, v[i].x, o4[h].x);
            o4[h].y = __fmaf_rn(pw, v[i].y, o4[h].y);
            o4[h].z = __fmaf_rn(pw, v[i].z, o4[h].z);
            o4[h].w = __fmaf_rn(pw, v[i].w, o4[h].w);
          }
        }
      }
    }
    __syncthreads();
  }
  // the four warps' partial sums, added in warp order: thread = dim d
#pragma unroll
  for (int h = 0; h < 4; ++h) *reinterpret_cast<float4*>(&s_o[warp][h][4 * lane]) = o4[h];
  __syncthreads();
  float o[4];
#pragma unroll
  for (int h = 0; h < 4; ++h)
    o[h] = __fadd_rn(__fadd_rn(__fadd_rn(s_o[0][h][tid], s_o[1][h][tid]), s_o[2][h][tid]), s_o[3][h][tid]);
  const size_t slot = ((size_t)m * a.nkv + j) * kAttSplits;
  float* dst = a.out + (size_t)m * a.nq + (size_t)j * a.hpk * kHeadDim;
  float mxo = 0.0f;
  if (n == 1) {
    if (lane == 0) s_red[warp] = lrun;  // warp h holds head h's sum
    __syncthreads();
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      const float r = __fmul_rn(o[h], __fdiv_rn(1.0f, s_red[h]));
      if (h < a.hpk) {
        dst[h * kHeadDim + tid] = r;
        mxo = fmaxf(mxo, fabsf(r));
      }
    }
  } else {
#pragma unroll
    for (int h = 0; h < 4; ++h) a.o_part[((slot + p) * 4 + h) * kHeadDim + tid] = o[h];
    if (lane == 0) {
      a.ml_part[((slot + p) * 4 + warp) * 2] = mrun;
      a.ml_part[((slot + p) * 4 + warp) * 2 + 1] = lrun;
    }
    __syncthreads();
    if (tid == 0) {
      __threadfence();
      const unsigned old = atomicAdd(&a.cnt[(size_t)m * a.nkv + j], 1u);
      const bool last = old == (unsigned)(n - 1);
      if (last) {
        a.cnt[(size_t)m * a.nkv + j] = 0u;
        __threadfence();
      }
      s_last = last ? 1 : 0;
    }
    __syncthreads();
    if (!s_last) return;
    // merge the chunks in order
#pragma unroll
    for (int h = 0; h < 4; ++h) {
      float mg = -INFINITY;
      for (int c = 0; c < n; ++c) mg = fmaxf(mg, __ldcg(&a.ml_part[((slot + c) * 4 + h) * 2]));
      float l = 0.0f, acc = 0.0f;
      for (int c = 0; c < n; ++c) {
        const float w = expf(__ldcg(&a.ml_part[((slot + c) * 4 + h) * 2]) - mg);
        l = __fmaf_rn(__ldcg(&a.ml_part[((slot + c) * 4 + h) * 2 + 1]), w, l);
        acc = __fmaf_rn(__ldcg(&a.o_part[((slot + c) * 4 + h) * kHeadDim + tid]), w, acc);
      }
      const float r = __fmul_rn(acc, __fdiv_rn(1.0f, l));
      if (h < a.hpk) {
        dst[h * kHeadDim + tid] = r;
        mxo = fmaxf(mxo, fabsf(r));
      }
    }
  }
  // max |out| of this (row, kv head): the o_proj operand's row scale
  mxo = warp_max(mxo);
  __syncthreads();
  if (lane == 0) s_red[warp] = mxo;
  __syncthreads();
  if (tid == 0) a.st_mx[(size_t)j * kMaxRows + m] = fmaxf(fmaxf(s_red[0], s_red[1]), fmaxf(s_red[2], s_red[3]));
}

}  // namespace f16b
}  // namespace qora
