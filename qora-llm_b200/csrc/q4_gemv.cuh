// q4_gemv.cuh — batch-1 Q4 GEMV on CUDA cores, HBM-streaming.
//
// y[j] = sum_ki x[ki] * (q[ki][j] - 8) * scale[ki][j/32]   (gemv_q4, src/gemv.rs:596-675)
//
// Work decomposition. The matrix is cut into column tiles of 8 groups (256 outputs).
// The (tile, row) space, tile-major, is split into `ctas` equal contiguous ranges, one
// per CTA, so every CTA streams the same number of bytes whatever the shape. A CTA walks
// its range as one or more segments (tile t, rows [r0, r1)); per segment each lane owns
// one 16-byte group chunk per row (8 lanes across the tile's groups, 4 rows per warp
// step), accumulates its 32 outputs in registers, and the CTA writes one 256-float
// partial. The last CTA to finish a tile (atomic arrival counter) adds the tile's
// partials in slot order — a fixed order, so results are deterministic — and runs the
// fused epilogue (store / RoPE + KV append / residual add / SwiGLU).
//
// Dequantisation without shifts. For a 32-bit word w holding nibbles e0..e7 (bits
// 4m..4m+3), the float whose bits are (w & (0xF << 4m)) is the subnormal
// q * 2^(4m - 149), exactly; nibbles 5..7 come from w >> 12 the same way. FFMA (which
// keeps subnormal operands) multiplies it by c = scale * x * 2^64, so each element costs
// one LOP3 and half an FFMA2. The power of two per nibble position and the "-8" offset
// (8 * sum c, one add per group) are applied once per output at the end:
//   y = acc * 2^(85 - p_m) - 8 * sum(c) * 2^-64,  p_m = {0,4,8,12,16,8,12,16}[m].
#pragma once

#include "common.cuh"

namespace qora {

constexpr int kTileGroups = 8;                 // groups per column tile
constexpr int kTileCols = kTileGroups * kGroup; // 256 outputs
constexpr int kGemvThreads = 256;
constexpr int kGemvWarps = kGemvThreads / 32;
constexpr int kRowsPerStep = kGemvWarps * 4;   // rows covered by one CTA step
constexpr int kTiledRowBytes = kTileGroups * 16 + kTileGroups * 2;  // 144: 8 chunks + 8 scales

// Location of a Q4 matrix's bytes. Byte address of group-chunk (tile t, lane group gi,
// row r): p[sel] + t*tile_stride_p + gl*16 + r*row_stride_p, scale at
// s[sel] + t*tile_stride_s + gl*2 + r*row_stride_s, where with split == 0: sel = 0,
// gl = gi; with split == 4 (gate/up given as two matrices): sel = gi >= 4, gl = gi & 3.
struct Q4Src {
  const uint8_t* p[2];
  const uint8_t* s[2];
  long long tile_stride_p, tile_stride_s;
  long long row_stride_p, row_stride_s;
  int split;   // 0 or 4
  int K;       // rows (input dim)
  int G;       // valid groups per source (per matrix for split == 4)
  int tiles;
};

struct SplitPlan {
  int ctas;
  long long total;     // tiles * K
  int max_slots;
  float* partials;     // [tiles][max_slots][kTileCols]
  unsigned* counters;  // [tiles], zero between launches
};

// CTA whose range contains linear row index p (ranges are [c*T/C, (c+1)*T/C)).
QORA_DEV int owner_cta(long long p, long long total, int ctas) {
  return (int)(((p + 1) * (long long)ctas - 1) / total);
}

QORA_DEV float q4_scale_of_pos(int m) {
  // 2^(85 - p_m)
  const int p = (m < 5) ? 4 * m : 4 * m - 12;
  return __int_as_float((127 + 85 - p) << 23);
}

// Accumulate one row's 32 elements of a group: acc[i] holds the pair (2i, 2i+1).
QORA_DEV void q4_fma_chunk(const uint4 w, const float c, float2 (&acc)[16]) {
  const float2 cc = make_float2(c, c);
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t a = ws[i];
    const uint32_t b = a >> 12;
    acc[4 * i + 0] = __ffma2_rn(make_float2(__uint_as_float(a & 0xFu), __uint_as_float(a & 0xF0u)),
                                cc, acc[4 * i + 0]);
    acc[4 * i + 1] = __ffma2_rn(make_float2(__uint_as_float(a & 0xF00u), __uint_as_float(a & 0xF000u)),
                                cc, acc[4 * i + 1]);
    acc[4 * i + 2] = __ffma2_rn(make_float2(__uint_as_float(a & 0xF0000u), __uint_as_float(b & 0xF00u)),
                                cc, acc[4 * i + 2]);
    acc[4 * i + 3] = __ffma2_rn(make_float2(__uint_as_float(b & 0xF000u), __uint_as_float(b & 0xF0000u)),
                                cc, acc[4 * i + 3]);
  }
}

// ---------------------------------------------------------------- prologues
// Input of the GEMV: value of input row r (before the 2^64 pre-scale).
struct ProPlain {  // o_proj (attention output), down_proj (SwiGLU output), plain GEMV
  const float* x;
  QORA_DEV float prepare(float*) const { return 1.0f; }
  QORA_DEV float load(int r, float) const { return x[r]; }
};

struct ProNorm {  // RMSNorm fused in front of q/k/v and gate/up (every CTA recomputes it)
  const float* x;
  const float* gamma;  // f32 copy of the f16 gains
  int n;
  QORA_DEV float prepare(float* red) const { return rms_inv(x, n, red); }
  QORA_DEV float load(int r, float inv) const {
    return __fmul_rn(__fmul_rn(x[r], inv), gamma[r]);  // x * inv_rms * gamma (src/gemv.rs:750)
  }
};

// ---------------------------------------------------------------- epilogues
// Called by all threads of the last-arriving CTA of tile t with the tile's 256 sums in
// y (shared memory).
struct EpiStore {
  float* out;
  int n;
  QORA_DEV void operator()(int t, const float* y) const {
    for (int o = threadIdx.x; o < kTileCols; o += blockDim.x) {
      const int c = t * kTileCols + o;
      if (c < n) out[c] = y[o];
    }
  }
};

struct EpiResidual {  // x += W.in  (src/gemv.rs:995-997, :1009-1011)
  float* x;
  int n;
  QORA_DEV void operator()(int t, const float* y) const {
    for (int o = threadIdx.x; o < kTileCols; o += blockDim.x) {
      const int c = t * kTileCols + o;
      if (c < n) x[c] = __fadd_rn(x[c], y[o]);
    }
  }
};

// Fused gate/up tile: columns [0,128) are gate outputs t*128.., [128,256) the matching up
// outputs. silu(g) * u with silu(g) = g / (1 + exp(-g)) (src/gemv.rs:494-500).
struct EpiSwiGLU {
  float* h;
  int n;  // intermediate size
  QORA_DEV void operator()(int t, const float* y) const {
    for (int o = threadIdx.x; o < kTileCols / 2; o += blockDim.x) {
      const int c = t * (kTileCols / 2) + o;
      if (c < n) {
        const float g = y[o];
        const float s = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
        h[c] = __fmul_rn(s, y[o + kTileCols / 2]);
      }
    }
  }
};

// Fused q|k|v tile (q: [0,nq), k: [nq,nq+nkv), v: after). RoPE (src/gemv.rs:757-778) on
// q and k when `rope`, at position st->pos; k and v rows appended to the KV cache at
// that position (src/gemv.rs:909-911).
struct EpiQKV {
  float* q;
  float* kc;  // this layer's K cache, head-major [kv head][max_seq][128]
  float* vc;
  long long hs;  // head stride of the cache (max_seq * 128)
  const StepState* st;
  const float* cos_t;
  const float* sin_t;
  int nq, nkv, rope, max_pos;
  QORA_DEV void store(int c, float v, int pos) const {
    if (c < nq) {
      q[c] = v;
    } else {
      const int j = (c < nq + nkv) ? c - nq : c - nq - nkv;  // within k or v
      float* dst = (c < nq + nkv) ? kc : vc;
      dst[(j / kHeadDim) * hs + (long long)pos * kHeadDim + (j % kHeadDim)] = v;
    }
  }
  QORA_DEV void operator()(int t, const float* y) const {
    const int pos = st->pos;
    if (pos < 0 || pos >= max_pos) return;  // host guarantees capacity
    for (int o = threadIdx.x; o < kTileCols; o += blockDim.x) {
      const int c = t * kTileCols + o;
      if (c >= nq + 2 * nkv) continue;
      const int d = c & (kHeadDim - 1);
      if (rope && c < nq + nkv) {
        if (d < kHalfDim) {
          const float x1 = y[o], x2 = y[o + kHalfDim];
          const float cs = cos_t[(long long)pos * kHalfDim + d];
          const float sn = sin_t[(long long)pos * kHalfDim + d];
          store(c, __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn)), pos);
          store(c + kHalfDim, __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn)), pos);
        }
      } else {
        store(c, y[o], pos);
      }
    }
  }
};

// ---------------------------------------------------------------- the kernel
// Dynamic shared memory: `seg_cap` floats for the segment's pre-scaled inputs.
template <class Pro, class Epi>
__global__ void __launch_bounds__(kGemvThreads, 2)
    q4_gemv_kernel(const Q4Src src, const SplitPlan plan, const Pro pro, const Epi epi) {
  extern __shared__ float xs[];
  __shared__ float red[kGemvWarps][kTileGroups][kGroup + 1];
  __shared__ float ybuf[kTileCols];
  __shared__ float nred[kGemvWarps];
  __shared__ int s_last;

  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int gi = lane & 7, sub = lane >> 3;
  const int c = blockIdx.x;
  const long long lin0 = (long long)c * plan.total / plan.ctas;
  const long long lin1 = (long long)(c + 1) * plan.total / plan.ctas;
  const float inv = pro.prepare(nred);
  const int K = src.K;
  const int sel = src.split ? (gi >= 4) : 0;
  const int gl = src.split ? (gi & 3) : gi;
  const float kX = 18446744073709551616.0f;  // 2^64

  for (long long p = lin0; p < lin1;) {
    const int t = (int)(p / K);
    const int r0 = (int)(p - (long long)t * K);
    const long long pe = min(lin1, (long long)(t + 1) * K);
    const int r1 = (int)(pe - (long long)t * K);
    p = pe;

    __syncthreads();  // xs reuse across segments
    for (int i = tid; i < r1 - r0; i += kGemvThreads) xs[i] = pro.load(r0 + i, inv) * kX;
    __syncthreads();

    const int gtile = src.split ? (kTileGroups / 2) : kTileGroups;
    const bool valid = (t * gtile + gl) < src.G;
    const uint8_t* pb = (sel ? src.p[1] : src.p[0]) + (long long)t * src.tile_stride_p + gl * 16;
    const uint8_t* sb = (sel ? src.s[1] : src.s[0]) + (long long)t * src.tile_stride_s + gl * 2;

    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
    float csum = 0.0f;

    if (valid) {
      int r = r0 + warp * 4 + sub;
      for (; r + 3 * kRowsPerStep < r1; r += 4 * kRowsPerStep) {
        uint4 w[4];
        uint16_t sc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const long long rr = r + u * kRowsPerStep;
          w[u] = __ldg(reinterpret_cast<const uint4*>(pb + rr * src.row_stride_p));
          sc[u] = __ldg(reinterpret_cast<const unsigned short*>(sb + rr * src.row_stride_s));
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float cf = __half2float(__ushort_as_half(sc[u])) * xs[r + u * kRowsPerStep - r0];
          csum += cf;
          q4_fma_chunk(w[u], cf, acc);
        }
      }
      for (; r < r1; r += kRowsPerStep) {
        const uint4 w = __ldg(reinterpret_cast<const uint4*>(pb + (long long)r * src.row_stride_p));
        const uint16_t sc = __ldg(reinterpret_cast<const unsigned short*>(sb + (long long)r * src.row_stride_s));
        const float cf = __half2float(__ushort_as_half(sc)) * xs[r - r0];
        csum += cf;
        q4_fma_chunk(w, cf, acc);
      }
    }

    // finalize this lane's 32 outputs, then add the 4 row-lanes of each group
    const float bias = csum * 4.3368086899420177e-19f;  // 8 * 2^-64
    float yv[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int e0 = 2 * i, e1 = 2 * i + 1;
      yv[e0] = __fmaf_rn(acc[i].x, q4_scale_of_pos(e0 & 7), -bias);
      yv[e1] = __fmaf_rn(acc[i].y, q4_scale_of_pos(e1 & 7), -bias);
    }
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      yv[e] += __shfl_xor_sync(0xffffffffu, yv[e], 8);
      yv[e] += __shfl_xor_sync(0xffffffffu, yv[e], 16);
    }
    if (sub == 0) {
#pragma unroll
      for (int e = 0; e < 32; ++e) red[warp][gi][e] = yv[e];
    }
    __syncthreads();

    const int slot_first = owner_cta((long long)t * K, plan.total, plan.ctas);
    const int slot_last = owner_cta((long long)(t + 1) * K - 1, plan.total, plan.ctas);
    const int slot = c - slot_first, nslots = slot_last - slot_first + 1;
    float* part = plan.partials + ((long long)t * plan.max_slots) * kTileCols;
    {
      const int o = tid;  // kGemvThreads == kTileCols
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kGemvWarps; ++w) s += red[w][o >> 5][o & 31];
      __stcg(part + (long long)slot * kTileCols + o, s);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
      const unsigned prev = atomicAdd(plan.counters + t, 1u);
      s_last = (prev == (unsigned)(nslots - 1));
    }
    __syncthreads();
    if (s_last) {
      __threadfence();
      {
        const int o = tid;
        float s = 0.0f;
        for (int k = 0; k < nslots; ++k) s += __ldcg(part + (long long)k * kTileCols + o);
        ybuf[o] = s;
      }
      __syncthreads();
      epi(t, ybuf);
      if (tid == 0) plan.counters[t] = 0u;
    }
  }
}

}  // namespace qora
