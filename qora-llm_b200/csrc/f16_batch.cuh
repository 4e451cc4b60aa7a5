// f16_batch.cuh — F16-weight decode and prefill for M "rows" at once (
// batched decode of independent sequences; prompt prefill). A row is one token of one
// sequence at one position; a batched decode step has one row per sequence, a prefill
// chunk one row per prompt token of a sequence. The same per-layer kernels serve both:
//
//   norm_split      RMSNorm (optional) of each row, written as two f16 terms (hi, lo)
//   gemm_f16        P = [hi|lo](rows) . W on the tensor cores (mma.sync m16n8k16, f16 in,
//                   f32 accumulate), split over K into deterministic partial slots
//   reduce          Y = sum of the slots (slot order), + residual, or SwiGLU
//   rope_kv         RoPE on q/k at each row's position, k/v appended to its sequence's cache
//   attention_rows  causal attention of each row over its sequence's cache prefix
//   argmax_rows     first maximum per row
//
// Precision. The reference multiplies f32 activations by f16 weights in f32
// (gemv_f16 / gemm_f16, src/gemv.rs:534-588; FMA on the AVX-512 path). Here each
// activation x is split into hi = f16(x) and lo = f16(x - hi); both products with the
// f16 weight are exact in the tensor core's f32 accumulator, so the result carries ~22
// bits of x (absolute error below 2^-24 |x|, plus f16 subnormal spacing 2^-24 for tiny
// values) — far inside the logits bar — at 2 MMAs per weight tile.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"

namespace qora {
namespace f16b {

constexpr int kMaxRows = 128;      // rows per step (prefill chunk / batch)
constexpr int kTileN = 64;         // outputs per CTA
constexpr int kChunkK = 64;        // K rows per shared-memory stage
constexpr int kThreads = 128;      // 4 warps, 16 outputs each
constexpr int kPitch = kChunkK + 8;  // f16 per shared row (144 bytes: conflict-free ldmatrix)

// ---------------------------------------------------------------- activations -> f16 pairs
// xh[m][k] = f16(y), xl[m][k] = f16(y - xh) with y = x[m][k] (* inv_rms(x[m]) * gamma[k] if
// gamma != nullptr; rms_norm_f16, src/gemv.rs:744-753, eps 1e-6). Also writes y to yf when
// given. One CTA per row.
__global__ void __launch_bounds__(256) norm_split_kernel(const float* x, const float* gamma, int K,
                                                         __half* xh, __half* xl, float* yf) {
  __shared__ float red[8];
  const int m = blockIdx.x;
  const float* xr = x + (long long)m * K;
  float inv = 1.0f;
  if (gamma) inv = rms_inv(xr, K, red);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float y = gamma ? __fmul_rn(__fmul_rn(xr[k], inv), gamma[k]) : xr[k];
    const __half h = __float2half_rn(y);
    const __half l = __float2half_rn(__fsub_rn(y, __half2float(h)));
    xh[(long long)m * K + k] = h;
    xl[(long long)m * K + k] = l;
    if (yf) yf[(long long)m * K + k] = y;
  }
}

// ---------------------------------------------------------------- tensor-core GEMM
QORA_DEV void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
QORA_DEV void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
QORA_DEV void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

QORA_DEV void ldsm_x4(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(s));
}
QORA_DEV void ldsm_x4_t(const void* p, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3) : "r"(s));
}
QORA_DEV void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

struct GemmArgs {
  const __half* w;     // weights: N-major [K][ldw] (projections) or K-major [N][ldw] (lm_head)
  long long ldw;       // elements between consecutive K rows (N-major) / output rows (K-major)
  const __half* xh;    // activations hi [M][K]
  const __half* xl;    // activations lo [M][K]
  int M, K, N;         // rows, reduction length, outputs (N % 64 == 0, K % 64 == 0)
  int splits;          // K slices (gridDim.y)
  float* out;          // [splits][M][N] partials (out + s*M*N)
};

// One CTA: 64 outputs x all M rows x one K slice. Warp w: outputs [16w, 16w+16); per 16
// of K one ldmatrix of the weight tile (transposed for N-major storage) and, per 8 rows,
// one ldmatrix of the hi and of the lo activations, two MMAs.
template <bool kKMajorW, int MT>  // MT = row tiles of 8 (M <= 8*MT)
__global__ void __launch_bounds__(kThreads) gemm_f16_kernel(const GemmArgs g) {
  extern __shared__ __align__(16) __half sm[];
  __half* ws = sm;                                   // [2][64][kPitch]
  __half* xs = sm + 2 * 64 * kPitch;                 // [2][2][8*MT][kPitch]
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int n0 = blockIdx.x * kTileN;
  const int chunks = g.K / kChunkK;
  const int c0 = (int)((long long)blockIdx.y * chunks / g.splits);
  const int c1 = (int)((long long)(blockIdx.y + 1) * chunks / g.splits);
  const int M = g.M, MP = 8 * MT;

  auto load = [&](int c, int buf) {
    const int k0 = c * kChunkK;
    __half* wd = ws + buf * 64 * kPitch;
    // 64 rows x 128 bytes of weights: rows are K (N-major) or outputs (K-major)
    for (int i = tid; i < 64 * 8; i += kThreads) {
      const int r = i >> 3, q = (i & 7) * 8;
      const __half* src = kKMajorW ? g.w + (long long)(n0 + r) * g.ldw + k0 + q : g.w + (long long)(k0 + r) * g.ldw + n0 + q;
      cp_async16(wd + r * kPitch + q, src);
    }
    __half* xd = xs + buf * 2 * MP * kPitch;
    for (int i = tid; i < 2 * M * 8; i += kThreads) {
      const int hl = i / (M * 8), rem = i - hl * M * 8, m = rem >> 3, q = (rem & 7) * 8;
      cp_async16(xd + (hl * MP + m) * kPitch + q, (hl ? g.xl : g.xh) + (long long)m * g.K + k0 + q);
    }
    cp_async_commit();
  };

  float acc[MT][4];
#pragma unroll
  for (int t = 0; t < MT; ++t)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[t][j] = 0.0f;

  // rows >= M of the activation tile read zeros
  for (int i = tid; i < 2 * 2 * (MP - M) * kPitch; i += kThreads) {
    const int per = (MP - M) * kPitch, b = i / (2 * per), rem = i - b * 2 * per, hl = rem / per, r = rem - hl * per;
    xs[(b * 2 + hl) * MP * kPitch + M * kPitch + r] = __float2half_rn(0.0f);
  }
  if (c0 < c1) load(c0, 0);
  for (int c = c0; c < c1; ++c) {
    const int buf = (c - c0) & 1;
    if (c + 1 < c1) {
      load(c + 1, buf ^ 1);
      cp_async_wait<1>();
    } else {
      cp_async_wait<0>();
    }
    __syncthreads();
    const __half* wb = ws + buf * 64 * kPitch;
    const __half* xb = xs + buf * 2 * MP * kPitch;
#pragma unroll
    for (int kk = 0; kk < kChunkK; kk += 16) {
      uint32_t a0, a1, a2, a3;
      const int mi = lane >> 3, ri = lane & 7;  // ldmatrix: matrix mi, row ri
      if (kKMajorW) {
        // smem rows = outputs: matrix (rows n 0-7|8-15, cols k 0-7|8-15)
        const __half* p = wb + (warp * 16 + (mi & 1) * 8 + ri) * kPitch + kk + (mi >> 1) * 8;
        ldsm_x4(p, a0, a1, a2, a3);
      } else {
        // smem rows = K: matrix mi holds k rows (mi>>1)*8 + ri, outputs (mi&1)*8 .. +7
        const __half* p = wb + (kk + (mi >> 1) * 8 + ri) * kPitch + warp * 16 + (mi & 1) * 8;
        ldsm_x4_t(p, a0, a1, a2, a3);
      }
#pragma unroll
      for (int t = 0; t < MT; ++t) {
        // hi and lo activations of rows 8t..8t+7: (rows, k 0-7) and (rows, k 8-15) each
        uint32_t bh0, bh1, bl0, bl1;
        const int hl = mi >> 1;  // lanes 0-15: hi, 16-31: lo
        const __half* p = xb + (hl * MP + 8 * t + ri) * kPitch + kk + (mi & 1) * 8;
        ldsm_x4(p, bh0, bh1, bl0, bl1);
        mma16816(acc[t], a0, a1, a2, a3, bh0, bh1);
        mma16816(acc[t], a0, a1, a2, a3, bl0, bl1);
      }
    }
    __syncthreads();
  }
  // D fragment: (output g / g+8, row 2t / 2t+1) -> out[slot][row][n]
  float* out = g.out + (long long)blockIdx.y * M * g.N;
  const int gq = lane >> 2, tq = lane & 3;
#pragma unroll
  for (int t = 0; t < MT; ++t) {
    const int m0 = 8 * t + 2 * tq;
    const int n = n0 + warp * 16 + gq;
    if (m0 < M) {
      out[(long long)m0 * g.N + n] = acc[t][0];
      out[(long long)m0 * g.N + n + 8] = acc[t][2];
    }
    if (m0 + 1 < M) {
      out[(long long)(m0 + 1) * g.N + n] = acc[t][1];
      out[(long long)(m0 + 1) * g.N + n + 8] = acc[t][3];
    }
  }
}

constexpr size_t gemm_smem_bytes(int MT) { return (size_t)(2 * 64 + 2 * 2 * 8 * MT) * kPitch * sizeof(__half); }

// ---------------------------------------------------------------- split-K reduction
// mode 0: y = sum;  1: y = res + sum (residual add, y may alias res);  2: SwiGLU,
// h[m][j] = silu(sum[m][j]) * sum[m][I + j] for j < I = N/2 (gate|up concatenated).
__global__ void reduce_kernel(const float* part, int splits, int M, int N, int mode, const float* res, float* y) {
  const int cols = mode == 2 ? N / 2 : N;
  const long long total = (long long)M * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / cols), n = (int)(i - (long long)m * cols);
    float s = 0.0f;
    for (int k = 0; k < splits; ++k) s = __fadd_rn(s, part[((long long)k * M + m) * N + n]);
    if (mode == 2) {
      float u = 0.0f;
      for (int k = 0; k < splits; ++k) u = __fadd_rn(u, part[((long long)k * M + m) * N + cols + n]);
      y[(long long)m * cols + n] = __fmul_rn(__fdiv_rn(s, __fadd_rn(1.0f, expf(-s))), u);
    } else {
      y[(long long)m * N + n] = mode == 1 ? __fadd_rn(res[(long long)m * N + n], s) : s;
    }
  }
}

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

// x[m] = f32(E[token[m]]) (embed_lookup, src/gemv.rs:515-526)
__global__ void embed_rows_kernel(const __half* emb, int H, int vocab, RowInfo ri, float* x) {
  const int m = blockIdx.x;
  const int tok = ri.token[m];
  if (tok < 0 || tok >= vocab) {  // the host validates ids; this keeps the read in bounds
    if (threadIdx.x == 0) *ri.error = 1;
    return;
  }
  const __half* row = emb + (long long)tok * H;
  for (int k = threadIdx.x; k < H; k += blockDim.x) x[(long long)m * H + k] = __half2float(row[k]);
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
