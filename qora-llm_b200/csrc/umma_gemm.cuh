// umma_gemm.cuh — F16-weight GEMMs of the batched paths on the 5th-generation tensor
// cores (tcgen05 + TMEM), with the surrounding per-row work fused in:
//   Y[rows][N] = op( prologue(X)[rows][K] . W[K][N] )
//
// Operands. W is re-tiled once at load into 128-channel x 64-k tiles of 16 KB, each in
// the UMMA "K-major, no swizzle" canonical layout (8x8 core matrices of 128 contiguous
// bytes; 8-row groups 1024 B apart, k-groups 128 B apart), stored tile-major so one
// 16 KB bulk copy moves one tile chunk. The activation operand is built by the GEMM's
// own prologue: every CTA writes a slice of it (per row: optional RMSNorm with the row's
// inverse RMS from the producer's per-tile statistics, a power-of-two row scale, then
// f16 hi = f16(y) and lo = f16(y - hi)) into a global staging buffer in the same tile
// layout as 2R rows (hi rows, then lo rows); a grid barrier (cooperative launch) then
// opens the activation copies, while the weight copies of the first ring stages are
// already in flight. One MMA (M=128 channels, N=2R, K=16) multiplies both halves; the
// drain adds the hi and lo columns in f32 and undoes the row scale, so every product
// carries ~22 bits of x, and the weights are exact.
//
// Work split. The (tile, k-chunk) units are cut into gridDim.x equal contiguous ranges
// (one persistent CTA per SM). A CTA's range covers a few segments (one tile's chunk run
// each); each segment accumulates in TMEM (double-buffered) and is drained to its own
// partial slot [R][128]. The CTA that completes a tile's last slot (per-tile counter,
// self-resetting) sums the slots in CTA order (deterministic) and applies the fused
// epilogue: store; q|k|v with RoPE and the KV-cache append; residual add with the
// row statistics the next RMSNorm needs; SwiGLU of the tile's gate|up halves; logits
// with the greedy argmax (64-bit atomic max of ordered keys, finished by the last tile).
//
// Roles (192 threads): all warps build the operand slice; then warp 0 lane 0 issues the
// bulk copies into an S-stage ring, warp 1 owns the TMEM allocation and its lane 0 issues
// the MMAs (tcgen05.commit releases each stage and signals each finished accumulator),
// warps 2-5 drain the accumulators and finish tiles. Every wait is bounded (globaltimer):
// on a timeout the CTA sets *err, stops issuing, waits for its copies and MMAs in flight,
// frees its TMEM and returns.
//
// Q4 weights (the Q4 prompt pass, gemm_q4 of src/gemv.rs:680-706). The weights stay Q4
// in HBM (0.5625 B per weight): each stage's bulk copy brings a 4.5 KB chunk of nibbles
// and f16 scales, and four more warps (320 threads) dequantise it into two f16 tiles in
// shared memory, hi = f16((q - 8) * s) and lo = (q - 8) * s - hi. The product of a 4-bit
// integer and an f16 scale has at most 15 significant bits, so hi + lo is the weight
// exactly (lo is a multiple of the scale's ulp, which f16 holds down to its subnormals);
// the MMA issuer runs both tiles against the same operand, so the accumulator receives
// (hi + lo) . x with x to ~22 bits, as for f16 weights.
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
// Q4 weights: one chunk (128 channels x 64 k) = nibble words [1024] (word p holds the 8 k
// of the 16-byte unit p of the f16 tile, see q4_unit) + f16 scales [4 channel groups of
// 32][64 k]
constexpr int kQ4Words = kTileN * kChunkK / 8;
constexpr int kQ4Chunk = kQ4Words * 4 + 4 * kChunkK * 2;
constexpr int kQ4Slot = 5 * 1024;            // its stage slot (stages stay 1 KB aligned)
constexpr int kQ4DqWarps = 4;                // dequantising warps of the Q4 kernel
constexpr int kQ4Threads = kThreads + 32 * kQ4DqWarps;

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


// Per-row table of the batched F16 steps (device memory, one per KV cache): seq | pos |
// token (kMaxRows ints each), then the greedy step counter and an error flag.
struct RowInfo {
  int* seq;
  int* pos;
  int* token;
  int* step;
  int* error;
};
constexpr int kRowInts = 3 * kMaxRows + 2;
__host__ __device__ inline RowInfo row_info(int* base) {
  return RowInfo{base, base + kMaxRows, base + 2 * kMaxRows, base + 3 * kMaxRows, base + 3 * kMaxRows + 1};
}

enum : int { kEpStore = 0, kEpQKV = 1, kEpResidual = 2, kEpSwiGLU = 3, kEpLogits = 4 };

struct FusedArgs {
  // weights and work split
  const uint8_t* w;          // tiled weights [tiles][chunks][16 KB]
  int tiles, chunks, M, R, stages, maxseg;
  // activation operand: xin rows [M][ldx] f32; RMSNorm with gamma (f32 [K]) when set
  const float* xin;
  int ldx;
  const float* gamma;
  float gmax;                // max |gamma|
  const float* st_ss;        // producer statistics of xin: [st_n][kMaxRows] sum of squares
  const float* st_mx;        //                               [st_n][kMaxRows] max |x|
  int st_n;
  uint8_t* xt;               // staged operand [chunks][R * 256 B]
  float* part;               // partial slots [gridDim.x][maxseg][R][128]
  unsigned* tile_cnt;        // [tiles] arrivals (self-resetting)
  unsigned* sync;            // [0] grid barrier count, [1] generation, [2] tiles finished (logits)
  // epilogue
  int ep;
  float* y;                  // output rows, row stride ldy
  int ldy;
  const float* res;          // kEpResidual: residual rows (may alias y)
  float* o_ss;               // output statistics [tiles][kMaxRows] (residual: ss and mx; SwiGLU: mx)
  float* o_mx;
  int q_tiles, k_tiles, rope;  // kEpQKV: q heads, k heads (v heads follow), RoPE on/off
  const float* cos_t;
  const float* sin_t;
  RowInfo rows;
  float* kc;                 // KV caches of this layer: [batch][kv_heads][max_seq][128]
  float* vc;
  long long seq_stride, head_stride;
  unsigned long long* am_key;  // kEpLogits: [M] ordered keys (zero between launches)
  unsigned* am_out;          //            [M] greedy token of each row
  int col0;                  // kEpLogits: global column of local tile 0 (vocab split)
  // tensor parallelism: the residual GEMMs (o_proj, down) exchange their partial tiles
  // and the lm_head its row candidates (and logits) with every rank over NVLink
  int tp, rank;
  const unsigned* epoch;     // forward-pass counter; tag = epoch * 128 + tag_slot
  int tag_slot;
  unsigned long long* xr_peer[8];   // every rank's receive block [T][tiles][kMaxRows][128] words
  float* lg_peer[8];                // every rank's full logits [kMaxRows][ldy]
  unsigned long long* key_peer[8];  // every rank's candidates [T][kMaxRows][2] (key, tag)
  int* err;
  unsigned long long timeout_ns;
};

// Stage of the f16 kernel: weight tile [kATile] | operand [R * 256]. Stage of the Q4
// kernel: weight tile hi [kATile] | lo [kATile] | operand [R * 256] | Q4 chunk [kQ4Chunk]
// (the chunk and the operand arrive by bulk copy; the dequantising warps fill hi and lo).
__host__ __device__ constexpr uint32_t stage_bytes(int R, bool q4 = false) {
  return q4 ? 2u * kATile + (uint32_t)R * 256u + (uint32_t)kQ4Slot : (uint32_t)kATile + (uint32_t)R * 256u;
}
__host__ __device__ constexpr uint32_t tmem_cols(int R) {
  return 4 * R <= 32 ? 32u : 4 * R <= 64 ? 64u : 4 * R <= 128 ? 128u : 4 * R <= 256 ? 256u : 512u;
}
inline size_t gemm_smem(int R, int stages, bool q4 = false) {
  return (size_t)stages * stage_bytes(R, q4) + ((q4 ? 3 : 2) * stages + 5) * 8 + 16;
}
inline int gemm_stages(int R, bool q4 = false) {
  const int s = (int)((kSmemBudget - 128) / stage_bytes(R, q4));
  return s < 2 ? 2 : (s > 8 ? 8 : s);
}

QORA_DEV void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

// ordered key: larger value wins, ties go to the lower index, NaN never wins
QORA_DEV unsigned long long am_key(float v, unsigned idx) {
  if (v != v) return 0ull;
  const unsigned b = __float_as_uint(v);
  const unsigned o = (b & 0x80000000u) ? ~b : (b | 0x80000000u);
  return ((unsigned long long)o << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}

// Grid-wide barrier of a cooperative launch (count + generation, self-resetting).
QORA_DEV void grid_sync(unsigned* sync, unsigned long long limit_ns, volatile int* abort) {
  __syncthreads();
  if (threadIdx.x == 0) {
    volatile unsigned* gen = sync + 1;
    const unsigned g0 = *gen;
    __threadfence();
    const unsigned old = atomicAdd(sync, 1u);
    if (old == gridDim.x - 1) {
      atomicExch(sync, 0u);
      __threadfence();
      atomicAdd(sync + 1, 1u);
    } else {
      const uint64_t t0 = ptx::globaltimer();
      while (*gen == g0) {
        if (ptx::globaltimer() - t0 > limit_ns) {
          *abort = 1;
          break;
        }
      }
    }
    __threadfence();
  }
  __syncthreads();
}

// half-warp reductions (lanes 0-15 and 16-31 each hold one row)
QORA_DEV float hw_sum(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = __fadd_rn(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
QORA_DEV float hw_max(float v) {
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Tensor parallelism: this rank's partial of (tile t, row m, channels j0..j0+3 and +64)
// goes to every rank as tagged 64-bit words (tag << 32 | f32 bits, one single-copy-atomic
// store each); then the T ranks' partials are read back from this rank's block and summed
// in rank order, so every rank gets the same bits. Waits are bounded (the CTA's error
// flag is set and zeros are used on expiry).
QORA_DEV void tp_sum_partials(const FusedArgs& a, int t, int m, int j0, float (&s0)[4], float (&s1)[4]) {
  const unsigned tag = *a.epoch * 128u + (unsigned)a.tag_slot;
  const size_t mine = (((size_t)a.rank * a.tiles + t) * kMaxRows + m) * kTileN + j0;
  for (int p = 0; p < a.tp; ++p) {
    unsigned long long* dst = a.xr_peer[p] + mine;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      ptx::st_relaxed_sys_b64(reinterpret_cast<uint64_t*>(dst + i),
                              ((uint64_t)tag << 32) | __float_as_uint(s0[i]));
      ptx::st_relaxed_sys_b64(reinterpret_cast<uint64_t*>(dst + 64 + i),
                              ((uint64_t)tag << 32) | __float_as_uint(s1[i]));
    }
  }
  float u0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, u1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  const unsigned long long* own = a.xr_peer[a.rank];
  for (int p = 0; p < a.tp; ++p) {
    const uint64_t* src =
        reinterpret_cast<const uint64_t*>(own + (((size_t)p * a.tiles + t) * kMaxRows + m) * kTileN + j0);
    uint64_t w[8];
    const uint64_t t0 = ptx::globaltimer();
    for (;;) {
      bool ok = true;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        w[i] = ptx::ld_relaxed_sys_b64(src + i);
        w[4 + i] = ptx::ld_relaxed_sys_b64(src + 64 + i);
      }
#pragma unroll
      for (int i = 0; i < 8; ++i) ok &= (unsigned)(w[i] >> 32) == tag;
      if (ok) break;
      if (ptx::globaltimer() - t0 > a.timeout_ns) {
        atomicExch(a.err, 1);
        break;
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      u0[i] = __fadd_rn(u0[i], __uint_as_float((unsigned)w[i]));
      u1[i] = __fadd_rn(u1[i], __uint_as_float((unsigned)w[4 + i]));
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    s0[i] = u0[i];
    s1[i] = u1[i];
  }
}

// Epilogue of row m, channels j0..j0+3 and j0+64..j0+67 of tile t (s0 / s1: the summed
// partials). Called by all lanes; rows are held by half-warps (q = lane % 16 picks j0 =
// 4q), `act` false for rows past M. Statistics are reduced within the half-warp.
QORA_DEV void finish_quad(const FusedArgs& a, int t, int m, int q, bool act, float (&s0)[4], float (&s1)[4]) {
  const int j0 = 4 * q;
  if (a.ep == kEpStore) {
    if (act) {
      float* yr = a.y + (size_t)m * a.ldy + t * kTileN + j0;
      *reinterpret_cast<float4*>(yr) = make_float4(s0[0], s0[1], s0[2], s0[3]);
      *reinterpret_cast<float4*>(yr + 64) = make_float4(s1[0], s1[1], s1[2], s1[3]);
    }
  } else if (a.ep == kEpQKV) {
    if (act) {
      const int pos = a.rows.pos[m];
      const bool isv = t >= a.q_tiles + a.k_tiles;
      float y0[4], y1[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        y0[i] = s0[i];
        y1[i] = s1[i];
        if (a.rope && !isv) {  // apply_rope_raw (src/gemv.rs:757-778)
          const float cs = a.cos_t[(size_t)pos * kHalfDim + j0 + i], sn = a.sin_t[(size_t)pos * kHalfDim + j0 + i];
          y0[i] = __fsub_rn(__fmul_rn(s0[i], cs), __fmul_rn(s1[i], sn));
          y1[i] = __fadd_rn(__fmul_rn(s1[i], cs), __fmul_rn(s0[i], sn));
        }
      }
      float* dst;
      if (t < a.q_tiles) {
        dst = a.y + (size_t)m * a.ldy + t * kTileN;
      } else {
        const int kh = isv ? t - a.q_tiles - a.k_tiles : t - a.q_tiles;
        dst = (isv ? a.vc : a.kc) + (long long)a.rows.seq[m] * a.seq_stride + kh * a.head_stride +
              (long long)pos * kHeadDim;
      }
      *reinterpret_cast<float4*>(dst + j0) = make_float4(y0[0], y0[1], y0[2], y0[3]);
      *reinterpret_cast<float4*>(dst + j0 + 64) = make_float4(y1[0], y1[1], y1[2], y1[3]);
    }
  } else if (a.ep == kEpResidual) {
    float ss = 0.0f, mx = 0.0f;
    if (act && a.tp > 1) tp_sum_partials(a, t, m, j0, s0, s1);
    if (act) {
      float* yr = a.y + (size_t)m * a.ldy + t * kTileN + j0;
      const float* rr = a.res + (size_t)m * a.ldy + t * kTileN + j0;
      const float4 r0 = *reinterpret_cast<const float4*>(rr), r1 = *reinterpret_cast<const float4*>(rr + 64);
      const float v0[4] = {__fadd_rn(r0.x, s0[0]), __fadd_rn(r0.y, s0[1]), __fadd_rn(r0.z, s0[2]), __fadd_rn(r0.w, s0[3])};
      const float v1[4] = {__fadd_rn(r1.x, s1[0]), __fadd_rn(r1.y, s1[1]), __fadd_rn(r1.z, s1[2]), __fadd_rn(r1.w, s1[3])};
      *reinterpret_cast<float4*>(yr) = make_float4(v0[0], v0[1], v0[2], v0[3]);
      *reinterpret_cast<float4*>(yr + 64) = make_float4(v1[0], v1[1], v1[2], v1[3]);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        ss = __fmaf_rn(v0[i], v0[i], ss);
        ss = __fmaf_rn(v1[i], v1[i], ss);
        mx = fmaxf(mx, fmaxf(fabsf(v0[i]), fabsf(v1[i])));
      }
    }
    ss = hw_sum(ss);
    mx = hw_max(mx);
    if (act && q == 0) {
      a.o_ss[(size_t)t * kMaxRows + m] = ss;
      a.o_mx[(size_t)t * kMaxRows + m] = mx;
    }
  } else if (a.ep == kEpSwiGLU) {  // fused_gate_up_gemv's silu(g) * u (src/gemv.rs:497-499)
    float mx = 0.0f;
    if (act) {
      float h[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        h[i] = __fmul_rn(__fdiv_rn(s0[i], __fadd_rn(1.0f, expf(-s0[i]))), s1[i]);
        mx = fmaxf(mx, fabsf(h[i]));
      }
      *reinterpret_cast<float4*>(a.y + (size_t)m * a.ldy + t * 64 + j0) = make_float4(h[0], h[1], h[2], h[3]);
    }
    mx = hw_max(mx);
    if (act && q == 0) a.o_mx[(size_t)t * kMaxRows + m] = mx;
  } else {  // kEpLogits
    unsigned long long k = 0ull;
    if (act) {
      const size_t col = (size_t)a.col0 + t * kTileN + j0;
      float* yr = a.y + (size_t)m * a.ldy + col;
      *reinterpret_cast<float4*>(yr) = make_float4(s0[0], s0[1], s0[2], s0[3]);
      *reinterpret_cast<float4*>(yr + 64) = make_float4(s1[0], s1[1], s1[2], s1[3]);
      for (int p = 0; p < a.tp; ++p) {  // every other rank's copy of the full logits
        if (p == a.rank) continue;
        float* pr = a.lg_peer[p] + (size_t)m * a.ldy + col;
        *reinterpret_cast<float4*>(pr) = make_float4(s0[0], s0[1], s0[2], s0[3]);
        *reinterpret_cast<float4*>(pr + 64) = make_float4(s1[0], s1[1], s1[2], s1[3]);
      }
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const unsigned long long k0 = am_key(s0[i], (unsigned)(col + i));
        const unsigned long long k1 = am_key(s1[i], (unsigned)(col + 64 + i));
        if (k0 > k) k = k0;
        if (k1 > k) k = k1;
      }
    }
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      const unsigned long long ok = __shfl_xor_sync(0xffffffffu, k, o);
      if (ok > k) k = ok;
    }
    if (act && q == 0) atomicMax(&a.am_key[m], k);
  }
}

constexpr int kMaxContrib = 160;  // >= CTAs of a launch (one per SM)

// Finish tile t (all its slots are written): 128 epilogue threads, 16 per row (thread q
// of a row owns channels 4q..4q+3 and 64+4q..64+4q+3), 16 rows per round (two rows per
// thread); each channel's slots are summed in CTA order, eight contributors' loads for
// both rows in flight at a time.
QORA_DEV void finish_tile(const FusedArgs& a, int t, long long* s_cb) {
  const int e = threadIdx.x - 64, q = e & 15, rsub = e >> 4;
  const long long T = (long long)a.tiles * a.chunks;
  const int G = gridDim.x;
  const int c0 = owner_of((long long)t * a.chunks, T, G), c1 = owner_of((long long)(t + 1) * a.chunks - 1, T, G);
  const int nc = c1 - c0 + 1;
  for (int i = e; i < nc; i += 128) {
    const int c = c0 + i, seg = t - (int)(range_begin(c, T, G) / a.chunks);
    s_cb[i] = (long long)(c * a.maxseg + seg) * a.R * kTileN;
  }
  ptx::named_bar(1, 128);
  // two row passes per round: every contributor's loads of 16 rows in flight together
  for (int m0 = 0; m0 < a.M; m0 += 16) {
    const int mA = m0 + rsub, mB = m0 + 8 + rsub;
    const bool actA = mA < a.M, actB = mB < a.M;
    float sA0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sA1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    float sB0[4] = {0.0f, 0.0f, 0.0f, 0.0f}, sB1[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    for (int i0 = 0; i0 < nc; i0 += 8) {
      float4 a0[8], a1[8], b0[8], b1[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const bool in = i0 + k < nc;
        const float* p = a.part + s_cb[in ? i0 + k : i0] + 4 * q;
        const float4 z = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        a0[k] = in && actA ? __ldcg(reinterpret_cast<const float4*>(p + (size_t)mA * kTileN)) : z;
        a1[k] = in && actA ? __ldcg(reinterpret_cast<const float4*>(p + (size_t)mA * kTileN + 64)) : z;
        b0[k] = in && actB ? __ldcg(reinterpret_cast<const float4*>(p + (size_t)mB * kTileN)) : z;
        b1[k] = in && actB ? __ldcg(reinterpret_cast<const float4*>(p + (size_t)mB * kTileN + 64)) : z;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (i0 + k < nc) {
          sA0[0] = __fadd_rn(sA0[0], a0[k].x);
          sA0[1] = __fadd_rn(sA0[1], a0[k].y);
          sA0[2] = __fadd_rn(sA0[2], a0[k].z);
          sA0[3] = __fadd_rn(sA0[3], a0[k].w);
          sA1[0] = __fadd_rn(sA1[0], a1[k].x);
          sA1[1] = __fadd_rn(sA1[1], a1[k].y);
          sA1[2] = __fadd_rn(sA1[2], a1[k].z);
          sA1[3] = __fadd_rn(sA1[3], a1[k].w);
          sB0[0] = __fadd_rn(sB0[0], b0[k].x);
          sB0[1] = __fadd_rn(sB0[1], b0[k].y);
          sB0[2] = __fadd_rn(sB0[2], b0[k].z);
          sB0[3] = __fadd_rn(sB0[3], b0[k].w);
          sB1[0] = __fadd_rn(sB1[0], b1[k].x);
          sB1[1] = __fadd_rn(sB1[1], b1[k].y);
          sB1[2] = __fadd_rn(sB1[2], b1[k].z);
          sB1[3] = __fadd_rn(sB1[3], b1[k].w);
        }
    }
    finish_quad(a, t, mA, q, actA, sA0, sA1);
    if (m0 + 8 < a.M) finish_quad(a, t, mB, q, actB, sB0, sB1);
  }
  ptx::named_bar(1, 128);  // s_cb is free again
  if (a.ep == kEpLogits) {
    int* s_flag = reinterpret_cast<int*>(s_cb);  // s_cb is free: reuse one word as a flag
    if (e == 0) {
      if (a.tp > 1)
        __threadfence_system();  // this CTA's peer logits stores before its arrival
      else
        __threadfence();
      const unsigned old = atomicAdd(a.sync + 2, 1u);
      const bool last = old == (unsigned)a.tiles - 1;
      if (last) __threadfence_system();
      *s_flag = last ? 1 : 0;
    }
    ptx::named_bar(1, 128);
    const bool last = *s_flag != 0;
    ptx::named_bar(1, 128);
    if (last) {
      // every tile of this rank is done: its row candidates (and, under tensor
      // parallelism, the exchange of candidates: release after this rank's logits, the
      // first maximum over ranks in rank order — the same on every rank)
      const unsigned tag = a.tp > 1 ? *a.epoch * 128u + (unsigned)a.tag_slot : 0u;
      for (int m = e; m < a.M; m += 128) {
        unsigned long long k = atomicExch(&a.am_key[m], 0ull);
        if (a.tp > 1) {
          for (int p = 0; p < a.tp; ++p) {
            uint64_t* slot = reinterpret_cast<uint64_t*>(a.key_peer[p] + ((size_t)a.rank * kMaxRows + m) * 2);
            ptx::st_relaxed_sys_b64(slot, k);
            ptx::st_release_sys_b64(slot + 1, tag);
          }
          unsigned long long best = 0ull;
          for (int p = 0; p < a.tp; ++p) {
            const uint64_t* slot =
                reinterpret_cast<const uint64_t*>(a.key_peer[a.rank] + ((size_t)p * kMaxRows + m) * 2);
            const uint64_t t0 = ptx::globaltimer();
            while (ptx::ld_acquire_sys_b64(slot + 1) != tag) {
              if (ptx::globaltimer() - t0 > a.timeout_ns) {
                atomicExch(a.err, 1);
                break;
              }
            }
            const unsigned long long kp = ptx::ld_relaxed_sys_b64(slot);
            if (kp > best) best = kp;
          }
          k = best;
        }
        a.am_out[m] = k ? 0xFFFFFFFFu - (unsigned)(k & 0xFFFFFFFFull) : 0u;
      }
      if (e == 0) atomicExch(a.sync + 2, 0u);
    }
  }
}

QORA_DEV __half2 u32_h2(uint32_t v) {
  __half2 h;
  memcpy(&h, &v, 4);
  return h;
}
QORA_DEV uint32_t h2_u32(__half2 h) {
  uint32_t v;
  memcpy(&v, &h, 4);
  return v;
}

// Unit p (0..1023) of a Q4 chunk: the 16-byte row segment at byte 16p of the f16 tile,
// i.e. channel o = 8 (p >> 6) + (p & 7), k = 8 ((p >> 3) & 7) + [0, 8). Its nibbles are
// word p (bits 4j..4j+3: k = 2j, bits 16+4j..16+4j+3: k = 2j+1, so one mask per pair
// gives a half2), its scales the 8 f16 of channel group p >> 8 at those k. 1024 + q is
// exact in f16 (0x6400 | q), and so is q - 8; hi is the f16 rounding of (q - 8) s (one
// rounding, no contraction) and lo = (q - 8) s - hi comes exact out of one fused
// multiply-add.
QORA_DEV void q4_unit(const uint8_t* chunk, int p, uint4& hv, uint4& lv) {
  const uint32_t w = reinterpret_cast<const uint32_t*>(chunk)[p];
  const uint4 sv = *reinterpret_cast<const uint4*>(chunk + kQ4Words * 4 + (p >> 8) * 128 + ((p >> 3) & 7) * 16);
  const uint32_t sw[4] = {sv.x, sv.y, sv.z, sv.w};
  const __half2 bias = u32_h2(0x64086408u);  // 1032
  uint32_t h[4], l[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const __half2 q = __hsub2(u32_h2(((w >> (4 * j)) & 0x000F000Fu) | 0x64006400u), bias);
    const __half2 s = u32_h2(sw[j]);
    const __half2 hi = __hmul2_rn(q, s);
    h[j] = h2_u32(hi);
    l[j] = h2_u32(__hfma2(q, s, __hneg2(hi)));
  }
  hv = make_uint4(h[0], h[1], h[2], h[3]);
  lv = make_uint4(l[0], l[1], l[2], l[3]);
}

template <bool Q4>
__global__ void __launch_bounds__(Q4 ? kQ4Threads : kThreads, 1) fused_gemm_kernel(const FusedArgs a) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ uint32_t s_tmem;
  __shared__ int s_abort, s_last, s_eok[4];
  __shared__ float s_inv[kMaxRows], s_sc[kMaxRows], s_rowinv[kMaxRows];
  __shared__ long long s_cb[kMaxContrib];
  const int S = a.stages, R = a.R, C = a.chunks, M = a.M;
  const int K = C * kChunkK;
  const uint32_t SB = stage_bytes(R, Q4);
  // stage layout: weights (f16: the tile; Q4: hi and lo tiles) | operand | (Q4 chunk)
  const uint32_t OFF_B = Q4 ? 2u * kATile : (uint32_t)kATile;
  const uint32_t OFF_W = Q4 ? OFF_B + (uint32_t)R * 256u : 0u;  // where the weight copy lands
  const uint32_t WB = Q4 ? (uint32_t)kQ4Chunk : (uint32_t)kATile;  // weight bytes per unit
  const uint32_t CB = WB + (uint32_t)R * 256u;                      // bytes copied per stage
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)S * SB);
  uint64_t* empty = full + S;
  uint64_t* dq = empty + S;             // Q4: [S] tiles dequantised (one arrival per dequantising warp)
  uint64_t* accf = dq + (Q4 ? S : 0);  // [2] accumulator ready
  uint64_t* acce = accf + 2;            // [2] accumulator drained
  uint64_t* fin = acce + 2;             // all MMAs complete
  volatile int* abort = &s_abort;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ncols = tmem_cols(R);
  const unsigned long long lim = a.timeout_ns;

  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int s = 0; s < S; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], 1);
      if (Q4) ptx::mbar_init(&dq[s], kQ4DqWarps);
    }
    ptx::mbar_init(&accf[0], 1);
    ptx::mbar_init(&accf[1], 1);
    ptx::mbar_init(&acce[0], 4);
    ptx::mbar_init(&acce[1], 4);
    ptx::mbar_init(fin, 1);
    ptx::fence_mbar_init();
  }
  // row constants: inverse RMS (rms_norm_f16, src/gemv.rs:744-747) from the producer's
  // per-tile sums of squares, and a power-of-two scale that puts the row's largest
  // operand value in [2^13, 2^14) (from a bound: max|x| * inv * max|gamma|)
  for (int m = threadIdx.x; m < R; m += blockDim.x) {
    float inv = 1.0f, sc = 0.0f, ri = 0.0f;
    if (m < M) {
      float mx = 0.0f;
#pragma unroll 8
      for (int t = 0; t < a.st_n; ++t) mx = fmaxf(mx, a.st_mx[(size_t)t * kMaxRows + m]);
      float bound = mx;
      if (a.gamma) {
        float ss = 0.0f;
#pragma unroll 8
        for (int t = 0; t < a.st_n; ++t) ss = __fadd_rn(ss, a.st_ss[(size_t)t * kMaxRows + m]);
        inv = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)K), 1e-6f)));
        bound = mx * inv * a.gmax;
      }
      int e = 0;
      if (bound > 0.0f && bound < INFINITY) {
        int ex;
        frexpf(bound, &ex);
        e = min(100, max(-100, 14 - ex));
      }
      sc = ldexpf(1.0f, e);
      ri = ldexpf(1.0f, -e);
    }
    s_inv[m] = inv;
    s_sc[m] = sc;
    s_rowinv[m] = ri;
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
  const long long n_units = b1 - b0;
  const int pre = (int)(n_units < S ? n_units : S);

  // weight copies of the first ring stages go out before the operand exists
  if (threadIdx.x == 0) {
    for (int i = 0; i < pre; ++i) {
      const long long u = b0 + i, t = u / C, c = u % C;
      ptx::mbar_arrive_expect_tx(&full[i], CB);
      ptx::bulk_g2s(smem + (size_t)i * SB + OFF_W, a.w + ((size_t)t * C + c) * WB, WB, &full[i]);
    }
  }
  // this CTA's slice of the operand: units (chunk c, row r, 8 k) in that order
  {
    const long long U = (long long)C * R * 8;
    const long long u0 = range_begin(blockIdx.x, U, G), u1 = range_begin(blockIdx.x + 1, U, G);
    for (long long u = u0 + threadIdx.x; u < u1; u += blockDim.x) {
      const int g = (int)(u & 7), r = (int)((u >> 3) % R), c = (int)(u / (8LL * R));
      const int k = c * kChunkK + g * 8;
      uint8_t* base = a.xt + (size_t)c * R * 256;
      uint4 hv = make_uint4(0, 0, 0, 0), lv = make_uint4(0, 0, 0, 0);
      if (r < M) {
        const float4* xp = reinterpret_cast<const float4*>(a.xin + (size_t)r * a.ldx + k);
        const float4 x0 = xp[0], x1 = xp[1];
        float v[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
        if (a.gamma) {
          const float4* gp = reinterpret_cast<const float4*>(a.gamma + k);
          const float4 g0 = gp[0], g1 = gp[1];
          const float gv[8] = {g0.x, g0.y, g0.z, g0.w, g1.x, g1.y, g1.z, g1.w};
#pragma unroll
          for (int i = 0; i < 8; ++i) v[i] = __fmul_rn(__fmul_rn(v[i], s_inv[r]), gv[i]);
        }
        __align__(16) __half h[8], l[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float ys = __fmul_rn(v[i], s_sc[r]);
          h[i] = __float2half_rn(ys);
          l[i] = __float2half_rn(__fsub_rn(ys, __half2float(h[i])));
        }
        hv = *reinterpret_cast<const uint4*>(h);
        lv = *reinterpret_cast<const uint4*>(l);
      }
      *reinterpret_cast<uint4*>(base + tile_off(r, g * 8)) = hv;
      *reinterpret_cast<uint4*>(base + tile_off(R + r, g * 8)) = lv;
    }
  }
  grid_sync(a.sync, lim, abort);

  if (warp == 0) {
    if (lane == 0) {
      // ---- producer: activation copies of the pre-issued stages, then both per stage
      fence_proxy_async_global();
      long long issued = pre;
      for (int i = 0; i < pre; ++i) {  // issued even after an abort, so those stages complete
        const long long c = (b0 + i) % C;
        ptx::bulk_g2s(smem + (size_t)i * SB + OFF_B, a.xt + (size_t)c * R * 256, (uint32_t)R * 256, &full[i]);
      }
      for (long long u = b0 + pre; u < b1 && !*abort; ++u, ++issued) {
        const int s = (int)(issued % S);
        const uint32_t k = (uint32_t)(issued / S);
        if (!wait_bar(&empty[s], (k - 1) & 1, lim, abort)) break;
        const long long t = u / C, c = u % C;
        uint8_t* st = smem + (size_t)s * SB;
        ptx::mbar_arrive_expect_tx(&full[s], CB);
        ptx::bulk_g2s(st + OFF_W, a.w + ((size_t)t * C + c) * WB, WB, &full[s]);
        ptx::bulk_g2s(st + OFF_B, a.xt + (size_t)c * R * 256, (uint32_t)R * 256, &full[s]);
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
          const uint32_t ph = (uint32_t)(i / S) & 1;
          // Q4: the operand copy (full) and the dequantised tiles (dq) both
          if (!wait_bar(&full[s], ph, lim, abort) || (Q4 && !wait_bar(&dq[s], ph, lim, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = sbase + (uint32_t)s * SB, sb = sa + OFF_B;
#pragma unroll
          for (int k16 = 0; k16 < kChunkK / 16; ++k16) {
            mma_f16(d, smem_desc(sa + k16 * 256), smem_desc(sb + k16 * 256), idesc, (u > u0 || k16 > 0) ? 1u : 0u);
            if (Q4) mma_f16(d, smem_desc(sa + kATile + k16 * 256), smem_desc(sb + k16 * 256), idesc, 1u);
          }
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
  } else if (Q4 && warp >= 6) {
    // ---- dequantisers (Q4): chunk of each landed stage -> f16 hi and lo tiles. A stage's
    // tiles are free when its copies land: the producer reissued the stage only after the
    // MMAs that read them had committed.
    const int dw = warp - 6;
    long long i = 0;
    for (long long u = b0; u < b1; ++u, ++i) {
      const int s = (int)(i % S);
      const bool ok = wait_bar(&full[s], (uint32_t)(i / S) & 1, lim, abort);
      if (!__all_sync(0xffffffffu, ok)) break;
      uint8_t* st = smem + (size_t)s * SB;
      const uint8_t* chunk = st + OFF_W;
#pragma unroll 2
      for (int p = dw * 32 + lane; p < kQ4Words; p += 32 * kQ4DqWarps) {
        uint4 hv, lv;
        q4_unit(chunk, p, hv, lv);
        *reinterpret_cast<uint4*>(st + 16 * p) = hv;
        *reinterpret_cast<uint4*>(st + kATile + 16 * p) = lv;
      }
      ptx::fence_proxy_async();  // the tiles are read by the tensor cores (async proxy)
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&dq[s]);
    }
  } else {
    // ---- epilogue: accumulator (128 channels x [hi | lo] columns) -> partial slot, then
    // the CTA that completes a tile finishes it
    const int q = warp & 3;  // TMEM lanes 32q .. 32q+31 = channels of this warp
    const int e = threadIdx.x - 64;
    long long u = b0;
    int seg = 0;
    while (u < b1) {
      const long long t = u / C, end = (t + 1) * C < b1 ? (t + 1) * C : b1;
      u = end;
      const int buf = seg & 1;
      // every lane waits; the four warps agree before any of them goes on, so that they
      // all take the same named barriers (and tcgen05.ld stays warp-collective)
      const bool ok = wait_bar(&accf[buf], (seg >> 1) & 1, lim, abort);
      const bool wok = __all_sync(0xffffffffu, ok);
      if (lane == 0) s_eok[q] = wok ? 1 : 0;
      ptx::named_bar(1, 128);
      if (!(s_eok[0] && s_eok[1] && s_eok[2] && s_eok[3])) break;
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
          dst[(size_t)(j + r) * kTileN] =
              __fmul_rn(__fadd_rn(__uint_as_float(h[r]), __uint_as_float(l[r])), s_rowinv[j + r]);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) ptx::mbar_arrive(&acce[buf]);
      ++seg;
      // tile bookkeeping: contributors are the CTAs whose ranges meet tile t
      const int c0 = owner_of(t * C, T, (int)G), c1 = owner_of((t + 1) * C - 1, T, (int)G);
      ptx::named_bar(1, 128);  // this CTA's slot is written
      bool last = true;
      if (c1 > c0) {
        if (e == 0) {
          __threadfence();
          const unsigned old = atomicAdd(&a.tile_cnt[t], 1u);
          const bool l = old == (unsigned)(c1 - c0);
          if (l) {
            a.tile_cnt[t] = 0u;
            __threadfence();
          }
          s_last = l ? 1 : 0;
        }
        ptx::named_bar(1, 128);
        last = s_last != 0;
      }
      if (last) finish_tile(a, (int)t, s_cb);
    }
  }
  // lanes 1-31 of warps 0 and 1 wait here for their role lane: every warp reaches the
  // block barrier converged, so it counts each warp once
  __syncwarp();
  tc_fence_before();
  __syncthreads();
  if (threadIdx.x == 0 && s_abort) atomicExch(a.err, 1);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
}

// Per-row statistics of rows stored flat [M][K] for the generic GEMM entry: max |x|
// over the row (one statistics tile, no RMSNorm).
__global__ void row_max_kernel(const float* x, int K, float* mx) {
  __shared__ float red[8];
  const int m = blockIdx.x;
  float v = 0.0f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) v = fmaxf(v, fabsf(x[(size_t)m * K + k]));
  v = warp_max(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x == 0) {
    float r = 0.0f;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) r = fmaxf(r, red[w]);
    mx[m] = r;
  }
}

// One-time re-tiling of an f16 matrix into [tiles][chunks][16 KB] UMMA tiles. src is
// N-major [K][ld] (columns col0..col0+N-1 taken) or K-major [N][ld] (rows = channels).
// Channel n lands in tile t0 + n / group at row o0 + n % group (group 128: whole tiles;
// group 64: one half of each tile, for the interleaved gate|up matrix); `chunks` is the
// destination's chunks per tile (>= K/64; k beyond K stays as the destination holds it).
__global__ void tile_weights_kernel(const __half* src, long long ld, int kmajor, int K, int N, int col0,
                                    int t0, int group, int o0, int chunks, uint8_t* dst) {
  const long long units = (long long)N * (K / 8);  // 16-byte output units: 8 k of one channel
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < units; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int k8 = (int)(i / N);
    const int k = k8 * 8;
    __align__(16) __half v[8];
#pragma unroll
    for (int j = 0; j < 8; ++j)
      v[j] = kmajor ? src[(long long)n * ld + k + j] : src[(long long)(k + j) * ld + col0 + n];
    const int t = t0 + n / group, o = o0 + n % group, c = k / kChunkK;
    uint8_t* tile = dst + ((size_t)t * chunks + c) * kATile;
    *reinterpret_cast<uint4*>(tile + tile_off(o, k % kChunkK)) = *reinterpret_cast<const uint4*>(v);
  }
}

// One-time re-tiling of a Q4 matrix in the file's layout (nibbles [K][ld/2], the low
// nibble of a byte the even column; f16 scales [K][ld/32]) into [tiles][chunks][kQ4Chunk]
// chunks for the Q4 kernel. Column col0 + n lands in tile t0 + n / group at channel
// o0 + n % group, as in tile_weights_kernel; col0, group and o0 are multiples of 32, so a
// tile's 32-channel blocks each take one scale group.
__global__ void tile_q4_kernel(const uint8_t* packed, const uint16_t* scales, long long ld, int K, int N, int col0,
                               int t0, int group, int o0, int chunks, uint8_t* dst) {
  const long long units = (long long)N * (K / 8);  // one nibble word: 8 k of one channel
  for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < units; i += (long long)gridDim.x * blockDim.x) {
    const int n = (int)(i % N);
    const int k = (int)(i / N) * 8;
    const int col = col0 + n;
    const int t = t0 + n / group, o = o0 + n % group, c = k / kChunkK, kk = k % kChunkK;
    uint32_t w = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t q = (packed[(long long)(k + j) * (ld / 2) + col / 2] >> (4 * (col & 1))) & 0xFu;
      w |= q << ((j & 1) ? 16 + 4 * (j >> 1) : 4 * (j >> 1));
    }
    uint8_t* chunk = dst + ((size_t)t * chunks + c) * kQ4Chunk;
    const int p = (o >> 3) * 64 + (kk >> 3) * 8 + (o & 7);
    reinterpret_cast<uint32_t*>(chunk)[p] = w;
    if ((o & 31) == 0) {
      uint16_t* sc = reinterpret_cast<uint16_t*>(chunk + kQ4Words * 4 + (o >> 5) * 128) + kk;
#pragma unroll
      for (int j = 0; j < 8; ++j) sc[j] = scales[(long long)(k + j) * (ld / 32) + col / 32];
    }
  }
}

}  // namespace umma
}  // namespace qora
