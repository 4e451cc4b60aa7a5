// umma_gemm.cuh — F16-weight GEMM on the 5th-generation tensor cores (tcgen05 + TMEM)
// for the batched paths: Y[rows][N] = X[rows][K] . W[K][N] with W f16 and X f32.
//
// Operands. W is re-tiled once at load into 128-channel x 64-k tiles of 16 KB, each in
// the UMMA "K-major, no swizzle" canonical layout (8x8 core matrices of 128 contiguous
// bytes; 8-row groups 1024 B apart, k-groups 128 B apart), stored tile-major so one
// 16 KB bulk copy moves one tile chunk. X is written by its producer (norm_split_tiled)
// in the same layout per 64-k chunk, as 2R rows: rows 0..R-1 the f16 "hi" terms of the
// rows (after a per-row power-of-two scale), rows R..2R-1 the f16 "lo" terms
// (x - hi). One MMA (M=128 channels, N=2R, K=16) multiplies both; the epilogue adds
// the hi and lo columns in f32 and undoes the row scale, so each product carries ~22
// bits of x, and the weights are exact.
//
// Work split. The (tile, k-chunk) units of one GEMM are cut into gridDim.x equal
// contiguous ranges (one persistent CTA per SM). A CTA's range covers a few "segments"
// (one tile's chunk run each); each segment accumulates in TMEM and is written to its
// own partial slot [R][128]. reduce_tiles_kernel then sums a tile's slots in CTA order
// (deterministic) and applies the epilogue (residual add / SwiGLU).
//
// Roles (192 threads): warp 0 lane 0 issues the bulk copies into an S-stage ring; warp 1
// owns the TMEM allocation and its lane 0 issues the MMAs (tcgen05.commit releases each
// stage and signals each finished accumulator); warps 2-5 drain the double-buffered
// accumulators (tcgen05.ld) to the partial slots. Every wait is bounded (globaltimer):
// on a timeout the CTA sets *err, stops issuing, waits for its copies and MMAs in
// flight, frees its TMEM and returns.
#pragma once

#include <cuda_fp16.h>

#include "common.cuh"
#include "ptx.cuh"

namespace qora {
namespace umma {

constexpr int kTileN = 128;                  // output channels per tile (UMMA M)
constexpr int kChunkK = 64;                  // k per pipeline stage
constexpr int kATile = kTileN * kChunkK * 2;  // 16 KB of weights per stage
constexpr int kThreads = 192;
constexpr int kMaxRows = 128;                // R <= 128 (N = 2R <= 256)
constexpr int kSmemBudget = 200 * 1024;

// byte offset of element (r, k) of a [rows][64] f16 chunk tile
__host__ __device__ constexpr int tile_off(int r, int k) {
  return (r >> 3) * 1024 + (k >> 3) * 128 + (r & 7) * 16 + (k & 7) * 2;
}

__host__ __device__ inline long long range_begin(long long c, long long T, long long G) { return c * T / G; }

// CTA whose range holds unit u
__device__ inline int owner_of(long long u, long long T, int G) {
  int c = (int)(u * G / T);
  while (c + 1 < G && range_begin(c + 1, T, G) <= u) ++c;
  while (c > 0 && range_begin(c, T, G) > u) --c;
  return c;
}

// ---------------------------------------------------------------- tcgen05 wrappers
QORA_DEV void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(ptx::smem_addr(slot)),
               "r"(ncols)
               : "memory");
}
QORA_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
QORA_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
QORA_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
QORA_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem] . B[smem]^T, kind::f16, issued by one thread
QORA_DEV void mma_f16(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive on `bar` once every tcgen05 operation this thread issued so far has completed
QORA_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   ptx::smem_addr(bar))
               : "memory");
}
// 8 consecutive 32-bit columns of this thread's TMEM lane
QORA_DEV void tmem_ld8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7])
               : "r"(taddr)
               : "memory");
}
QORA_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// shared-memory matrix descriptor: K-major, no swizzle, k-groups 128 B apart (leading
// byte offset), 8-row groups 1024 B apart (stride byte offset), descriptor version 1
QORA_DEV uint64_t smem_desc(uint32_t saddr) {
  return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)(128 >> 4) << 16) | ((uint64_t)(1024 >> 4) << 32) |
         (1ull << 46);
}
// instruction descriptor: f32 accumulate, A = B = f16, both K-major, M = 128, N = n
__host__ __device__ constexpr uint32_t instr_desc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTileN >> 4) << 24);
}

// bounded mbarrier wait; false (and the CTA's abort flag set) after limit_ns
QORA_DEV bool wait_bar(uint64_t* bar, uint32_t parity, unsigned long long limit_ns, volatile int* abort) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = ptx::globaltimer();
  for (;;) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (ptx::globaltimer() - t0 > limit_ns) {
      *abort = 1;
      return false;
    }
  }
}

struct GemmArgs {
  const uint8_t* w;         // tiled weights [tiles][chunks][16 KB]
  const uint8_t* x;         // tiled activations [chunks][R * 256 B]
  const float* row_inv;     // [R] power-of-two unscale of each row
  float* part;              // [gridDim.x][maxseg][R][128] partial slots
  int tiles, chunks, R, stages, maxseg;
  int* err;                 // set to 1 when a wait timed out
  unsigned long long timeout_ns;
};

__host__ __device__ constexpr uint32_t stage_bytes(int R) { return (uint32_t)kATile + (uint32_t)R * 256u; }
__host__ __device__ constexpr uint32_t tmem_cols(int R) {
  return 4 * R <= 32 ? 32u : 4 * R <= 64 ? 64u : 4 * R <= 128 ? 128u : 4 * R <= 256 ? 256u : 512u;
}
inline size_t gemm_smem(int R, int stages) { return (size_t)stages * stage_bytes(R) + (2 * stages + 5) * 8 + 16; }
inline int gemm_stages(int R) {
  const int s = (int)((kSmemBudget - 128) / stage_bytes(R));
  return s < 2 ? 2 : (s > 8 ? 8 : s);
}

__global__ void __launch_bounds__(kThreads, 1) umma_gemm_kernel(const GemmArgs a) {
  extern __shared__ __align__(1024) uint8_t smem[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort;
  const int S = a.stages, R = a.R, C = a.chunks;
  const uint32_t SB = stage_bytes(R);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * SB);
  uint64_t* empty = full + S;
  uint64_t* accf = empty + S;  // [2] accumulator ready
  uint64_t* acce = accf + 2;   // [2] accumulator drained
  uint64_t* fin = acce + 2;    // all MMAs complete
  volatile int* abort = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ncols = tmem_cols(R);

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
    }
    ptx::mbar_init(&accf[0], 1);
    ptx::mbar_init(&accf[1], 1);
    ptx::mbar_init(&acce[0], 4);
    ptx::mbar_init(&acce[1], 4);
    ptx::mbar_init(fin, 1);
    ptx::fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(&s_tmem, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  const long long T = (long long)a.tiles * C, G = gridDim.x;
  const long long b0 = range_begin(blockIdx.x, T, G), b1 = range_begin(blockIdx.x + 1, T, G);
  const unsigned long long lim = a.timeout_ns;

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: bulk copies of weight + activation chunks into the ring
      long long issued = 0;
      for (long long u = b0; u < b1 && !*abort; ++u, ++issued) {
        const int s = (int)(issued % S);
        const uint32_t k = (uint32_t)(issued / S);
        if (k > 0 && !wait_bar(&empty[s], (k - 1) & 1, lim, abort)) break;
        const long long t = u / C, c = u % C;
        uint8_t* st = smem + (size_t)s * SB;
        ptx::mbar_arrive_expect_tx(&full[s], SB);
        ptx::bulk_g2s(st, a.w + ((size_t)t * C + c) * kATile, kATile, &full[s]);
        ptx::bulk_g2s(st + kATile, a.x + (size_t)c * R * 256, (uint32_t)R * 256, &full[s]);
      }
      // copies still in flight land before the CTA can exit
      const long long first = issued > S ? issued - S : 0;
      for (long long i = first; i < issued; ++i) {
        volatile int no_abort = 0;
        wait_bar(&full[i % S], (uint32_t)(i / S) & 1, lim, &no_abort);
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // ---- MMA issuer
      const uint32_t idesc = instr_desc(2 * R);
      const uint32_t sbase = ptx::smem_addr(smem);
      long long i = 0, u = b0;
      int seg = 0;
      while (u < b1 && !*abort) {
        const long long t = u / C, e = (t + 1) * C < b1 ? (t + 1) * C : b1;
        const int buf = seg & 1;
        if (seg >= 2 && !wait_bar(&acce[buf], ((seg >> 1) - 1) & 1, lim, abort)) break;
        tc_fence_after();
        const uint32_t d = tmem + (uint32_t)(buf * 2 * R);
        bool ok = true;
        for (const long long u0 = u; u < e; ++u, ++i) {
          const int s = (int)(i % S);
          if (!wait_bar(&full[s], (uint32_t)(i / S) & 1, lim, abort)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + (uint32_t)s * SB, sb = sa + kATile;
#pragma unroll
          for (int k16 = 0; k16 < kChunkK / 16; ++k16)
            mma_f16(d, smem_desc(sa + k16 * 256), smem_desc(sb + k16 * 256), idesc, (u > u0 || k16 > 0) ? 1u : 0u);
          mma_commit(&empty[s]);
        }
        if (!ok) break;
        mma_commit(&accf[buf]);
        ++seg;
      }
      mma_commit(fin);
      volatile int no_abort = 0;
      wait_bar(fin, 0, lim, &no_abort);
    }
  } else {
    // ---- epilogue: accumulator (128 channels x [hi | lo] columns) -> partial slot
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31 = channels of this warp
    long long u = b0;
    int seg = 0;
    while (u < b1 && !*abort) {
      const long long t = u / C, e = (t + 1) * C < b1 ? (t + 1) * C : b1;
      u = e;
      const int buf = seg & 1;
      // every lane waits; the warp leaves together (tcgen05.ld is warp-collective)
      const bool ok = wait_bar(&accf[buf], (seg >> 1) & 1, lim, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      const uint32_t base = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * 2 * R);
      float* dst = a.part + ((size_t)(blockIdx.x * a.maxseg + seg) * R) * kTileN + q * 32 + lane;
      for (int j = 0; j < R; j += 8) {
        uint32_t h[8], l[8];
        tmem_ld8(base + j, h);
        tmem_ld8(base + R + j, l);
        tmem_wait_ld();
#pragma unroll
        for (int r = 0; r < 8; ++r)
          dst[(size_t)(j + r) * kTileN] = __fmul_rn(__fadd_rn(__uint_as_float(h[r]), __uint_as_float(l[r])),
                                                    a.row_inv[j + r]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acce[buf]);
      ++seg;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && s_abort) atomicExch(a.err, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// ---------------------------------------------------------------- producers / consumers
// Row m of X (RMSNorm'd with gamma when given, rms_norm_f16 src/gemv.rs:744-753) into the
// tiled hi|lo operand for R padded rows: y is scaled by 2^e (e puts max|y| in
// [2^13, 2^14)), hi = f16(y'), lo = f16(y' - hi); row_inv[m] = 2^-e. Rows M..R-1 are
// zero. One CTA per padded row.
__global__ void __launch_bounds__(256) norm_split_tiled_kernel(const float* x, const float* gamma, int K, int M,
                                                                int R, uint8_t* xt, float* row_inv) {
  __shared__ float red[8];
  const int m = blockIdx.x;
  const int nk8 = K / 8;
  if (m >= M) {
    for (int g = threadIdx.x; g < nk8; g += blockDim.x) {
      const int k = g * 8, c = k / kChunkK, kk = k % kChunkK;
      uint8_t* base = xt + (size_t)c * R * 256;
      *reinterpret_cast<uint4*>(base + tile_off(m, kk)) = make_uint4(0, 0, 0, 0);
      *reinterpret_cast<uint4*>(base + tile_off(R + m, kk)) = make_uint4(0, 0, 0, 0);
    }
    if (threadIdx.x == 0) row_inv[m] = 0.0f;
    return;
  }
  const float* xr = x + (size_t)m * K;
  float inv = 1.0f;
  if (gamma) inv = rms_inv(xr, K, red);
  float mx = 0.0f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const float y = gamma ? __fmul_rn(__fmul_rn(xr[k], inv), gamma[k]) : xr[k];
    mx = fmaxf(mx, fabsf(y));
  }
  mx = warp_max(mx);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  mx = 0.0f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) mx = fmaxf(mx, red[w]);
  int e = 0;
  if (mx > 0.0f && mx < INFINITY) {
    int ex;
    frexpf(mx, &ex);  // mx in [2^(ex-1), 2^ex)
    e = min(100, max(-100, 14 - ex));
  }
  const float sc = ldexpf(1.0f, e);
  for (int g = threadIdx.x; g < nk8; g += blockDim.x) {
    const int k = g * 8, c = k / kChunkK, kk = k % kChunkK;
    __align__(16) __half hv[8], lv[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float y = gamma ? __fmul_rn(__fmul_rn(xr[k + i], inv), gamma[k + i]) : xr[k + i];
      const float ys = __fmul_rn(y, sc);
      hv[i] = __float2half_rn(ys);
      lv[i] = __float2half_rn(__fsub_rn(ys, __half2float(hv[i])));
    }
    uint8_t* base = xt + (size_t)c * R * 256;
    *reinterpret_cast<uint4*>(base + tile_off(m, kk)) = *reinterpret_cast<const uint4*>(hv);
    *reinterpret_cast<uint4*>(base + tile_off(R + m, kk)) = *reinterpret_cast<const uint4*>(lv);
  }
  if (threadIdx.x == 0) row_inv[m] = ldexpf(1.0f, -e);
}

struct ReduceArgs {
  const float* part;
  int tiles, chunks, R, M, maxseg, G;
  int N;            // GEMM outputs (tiles * 128)
  int mode;         // 0: y = sum; 1: y = res + sum; 2: SwiGLU over gate|up halves
  const float* res;
  float* y;         // [M][N] (mode 2: [M][N/2])
  int ldy;
};

__device__ inline float tile_sum(const ReduceArgs& a, int m, int n) {
  const int t = n / kTileN, o = n % kTileN;
  const long long T = (long long)a.tiles * a.chunks;
  const int c0 = owner_of((long long)t * a.chunks, T, a.G), c1 = owner_of((long long)(t + 1) * a.chunks - 1, T, a.G);
  float s = 0.0f;
  for (int c = c0; c <= c1; ++c) {
    const int seg = t - (int)(range_begin(c, T, a.G) / a.chunks);
    s = __fadd_rn(s, a.part[((size_t)(c * a.maxseg + seg) * a.R + m) * kTileN + o]);
  }
  return s;
}

__global__ void reduce_tiles_kernel(const ReduceArgs a) {
  const int cols = a.mode == 2 ? a.N / 2 : a.N;
  const long long total = (long long)a.M * cols;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total; i += (long long)gridDim.x * blockDim.x) {
    const int m = (int)(i / cols), n = (int)(i - (long long)m * cols);
    const float s = tile_sum(a, m, n);
    float v;
    if (a.mode == 2) {
      const float u = tile_sum(a, m, n + cols);
      v = __fmul_rn(__fdiv_rn(s, __fadd_rn(1.0f, expf(-s))), u);
    } else {
      v = a.mode == 1 ? __fadd_rn(a.res[(size_t)m * a.ldy + n], s) : s;
    }
    a.y[(size_t)m * a.ldy + n] = v;
  }
}

// One-time re-tiling of an f16 matrix into [tiles][chunks][16 KB] UMMA tiles. src is
// N-major [K][ld] (columns col0..col0+N-1 taken) or K-major [N][ld]; the N channels land
// in tiles t0.. of a matrix with `chunks` = K/64 chunks per tile.
__global__ void tile_weights_kernel(const __half* src, long long ld, int kmajor, int K, int N, int col0,
                                    int t0, uint8_t* dst) {
  const long long units = (long long)N * (K / 8);  // 16-byte output units: 8 k of one channel
  const int chunks = K / kChunkK;
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < units; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int k8 = (int)(i / N);
    const int k = k8 * 8;
    __align__(16) __half v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = kmajor ? src[(long long)n * ld + k + j] : src[(long long)(k + j) * ld + col0 + n];
    const int t = t0 + n / kTileN, o = n % kTileN, c = k / kChunkK;
    uint8_t* tile = dst + ((size_t)t * chunks + c) * kATile;
    *reinterpret_cast<uint4*>(tile + tile_off(o, k % kChunkK)) = *reinterpret_cast<const uint4*>(v);
  }
}

}  // namespace umma
}  // namespace qora
