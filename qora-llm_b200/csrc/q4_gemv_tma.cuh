// q4_gemv_tma.cuh — the per-operation Q4 GEMV (benchmark config 1: gemv_q4,
// src/gemv.rs:596-675, on the reference's own F1 layout) as a Blackwell TMA stream.
//
// y[j] = sum_ki x[ki] * (q[ki][j] - 8) * scale[ki][j/32]
//
// The matrix is read where it lies: packed nibbles [K][n/2] bytes and f16 scales
// [K][n/32], both row-major (the .qora arrays as loaded). Column tiles of 256 outputs are
// 128 bytes of every packed row plus 16 bytes of every scale row, so a tile's rows form a
// 2-D box of each array: two tensor maps (cuTensorMapEncodeTiled) describe them, and one
// cp.async.bulk.tensor load moves 128 rows x 128 bytes (16 KB) of nibbles, another the
// 128 rows x 16 bytes of their scales, into shared memory.
//
// Work decomposition: the (tile, row) space, tile-major, is cut into one equal contiguous
// range per CTA (one CTA per SM, every CTA streams the same bytes). A CTA issues every box
// of its range at once (about 86 KB for config 1: all of its bytes in flight from the
// first cycle), then computes each box as it lands: lane (sub, gi) takes group gi of 4
// rows per warp pass, with the shift-free dequantisation of q4_gemv.cuh. A range covers
// one or two tiles (segments); each segment's sums are one split-K partial, published as
// tagged 64-bit words ((1 << 32) | f32 bits, single-copy atomic: no fence, no arrival
// counter). Once a CTA has published all of its partials, it finishes the tiles whose last
// slot it holds: it reads every slot of the tile (re-reading, bounded, the words not yet
// tagged), adds them in slot order (deterministic), stores y and puts the words back to
// zero for the next launch. Nobody waits before publishing its own partials, and the
// CTAs a finisher waits for hold lower slots, so no wait can go round in a circle.
//
// Back-to-back GEMVs overlap: launched with programmatic stream serialisation, a kernel
// issues its weight loads (read-only inputs) before griddepcontrol.wait, and only reads x
// and touches the shared split-K scratch and y after the previous kernel has completed.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "ptx.cuh"
#include "q4_gemv.cuh"

namespace qora {
namespace g1 {

// Two CTAs fit one SM (registers and shared memory), so that the next launch's CTA on an
// SM issues its weight loads while this launch's CTA there still computes and finishes.
constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kBoxRows = 64;                   // rows per box (CTA ranges are whole boxes)
constexpr int kPackBox = kBoxRows * 128;       // nibble bytes per box (256 outputs per row)
constexpr int kScaleBox = kBoxRows * 16;       // scale bytes per box (8 groups per row)
constexpr int kBoxBytes = kPackBox + kScaleBox;
constexpr int kMaxBoxes = 11;                  // rows per CTA <= kMaxBoxes * kBoxRows
constexpr int kMaxRows = kMaxBoxes * kBoxRows;
constexpr float kTwo64 = 18446744073709551616.0f;
constexpr unsigned long long kTimeoutNs = 2000000000ull;

struct Args {
  const float* x;
  float* y;
  uint64_t* partials;  // tagged [tiles][slots][256], zero between launches
  int K, n, tiles, slots;
};

// shared memory: boxes [kMaxBoxes][kBoxBytes] | xs [kMaxRows] | red [kWarps][256] |
// spare [256] | full barriers [kMaxBoxes] | spare word
constexpr int kOffXs = kMaxBoxes * kBoxBytes;
constexpr int kOffRed = kOffXs + kMaxRows * 4;
constexpr int kOffY = kOffRed + kWarps * kTileCols * 4;
constexpr int kOffBar = kOffY + kTileCols * 4;
constexpr size_t kSmemBytes = kOffBar + kMaxBoxes * 8 + 16;

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          ptx::smem_addr(dst)),
      "l"(map), "r"(x), "r"(y), "r"(ptx::smem_addr(bar))
      : "memory");
}

// ---- split geometry (host and device; tests/cpp/gemv_split_check.cu checks it)
// CTA c of G owns boxes [c*B/G, (c+1)*B/G) of the B = tiles * K / kBoxRows flattened row
// boxes (tile-major): rows [*l0, *l1) of the flattened (tile, row) space
__host__ __device__ inline void range_of(int c, int G, unsigned boxes, int* l0, int* l1) {
  *l0 = (int)((unsigned)c * boxes / (unsigned)G) * kBoxRows;
  *l1 = (int)((unsigned)(c + 1) * boxes / (unsigned)G) * kBoxRows;
}
// the CTAs holding rows of tile t: [*first, *last] (the owner of box p is ((p + 1) G - 1) / B)
__host__ __device__ inline void tile_ctas(int t, int K, int G, unsigned boxes, int* first, int* last) {
  const unsigned K1 = (unsigned)(K / kBoxRows);
  *first = (int)((((unsigned)t * K1 + 1u) * (unsigned)G - 1u) / boxes);
  *last = (int)((((unsigned)(t + 1) * K1) * (unsigned)G - 1u) / boxes);
}
// shapes the kernel takes on G CTAs: 256-column tiles, whole boxes of rows, at least one
// and at most kMaxBoxes boxes per CTA, no more boxes per CTA than a tile has (so a range
// touches at most two tiles: the kernel's two segments), 32-bit split arithmetic
__host__ __device__ inline bool shape_ok(long long k, long long n, int G) {
  if (k <= 0 || n <= 0 || n % kTileCols || k % kBoxRows) return false;
  const long long boxes = (n / kTileCols) * (k / kBoxRows), per = (boxes + G - 1) / G;
  return boxes >= G && boxes * G < (1ll << 32) && per <= kMaxBoxes && per <= k / kBoxRows;
}
// host: split-K slots per tile to allocate (every CTA owns at least floor(B / G) boxes)
__host__ __device__ inline int slots_bound(int K, long long boxes, int G) {
  const long long per = boxes / G > 0 ? boxes / G : 1;
  return (int)((K / kBoxRows) / per) + 2;
}

// the CTA's segments (tile, first row, end row) of the flattened range [l0, l1)
struct Segs {
  int n, t[2], r0[2], r1[2];
};
__host__ __device__ __forceinline__ Segs segs_of(int l0, int l1, int K) {
  Segs s;
  s.n = 0;
  for (int p = l0; p < l1 && s.n < 2; ++s.n) {
    const int t = p / K, pe = min(l1, (t + 1) * K);
    s.t[s.n] = t;
    s.r0[s.n] = p - t * K;
    s.r1[s.n] = pe - t * K;
    p = pe;
  }
  return s;
}

__global__ void __launch_bounds__(kThreads, 2)
    q4_gemv_tma_kernel(const __grid_constant__ CUtensorMap mp, const __grid_constant__ CUtensorMap ms, const Args a) {
  extern __shared__ __align__(128) uint8_t sm[];
  float* xs = reinterpret_cast<float*>(sm + kOffXs);
  float* red = reinterpret_cast<float*>(sm + kOffRed);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + kOffBar);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, gi = lane & 7, sub = lane >> 3;
  const int c = blockIdx.x, G = gridDim.x, K = a.K;
  // whole boxes per CTA (host: K % kBoxRows == 0, B >= G, B * G < 2^32)
  const unsigned total = (unsigned)a.tiles * (unsigned)(K / kBoxRows);
  int l0, l1;
  range_of(c, G, total, &l0, &l1);
  const Segs sg = segs_of(l0, l1, K);

  if (tid == 0) {  // every box of the range at once
    int b = 0;
    for (int s = 0; s < sg.n; ++s)
      for (int r = sg.r0[s]; r < sg.r1[s]; r += kBoxRows, ++b) ptx::mbar_init(&bars[b], 1);
    ptx::fence_mbar_init();
    b = 0;
    for (int s = 0; s < sg.n; ++s)
      for (int r = sg.r0[s]; r < sg.r1[s]; r += kBoxRows, ++b) {
        uint8_t* box = sm + (size_t)b * kBoxBytes;
        ptx::mbar_arrive_expect_tx(&bars[b], kBoxBytes);
        tma_load_2d(box, &mp, sg.t[s] * 128, r, &bars[b]);
        tma_load_2d(box + kPackBox, &ms, sg.t[s] * 8, r, &bars[b]);
      }
  }
  // the next GEMV in the stream may start its own weight loads on SMs this grid leaves
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // x, the split-K scratch and y are shared with the previous kernel of the stream
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int i = tid; i < l1 - l0; i += kThreads) {
    const int n0 = sg.r1[0] - sg.r0[0];
    xs[i] = a.x[i < n0 ? sg.r0[0] + i : sg.r0[1] + (i - n0)] * kTwo64;
  }
  __syncthreads();

  int b = 0, off = 0;
  int fin_t[2], fin_n[2], nfin = 0;  // tiles this CTA finishes (it holds their last slot)
  for (int s = 0; s < sg.n; ++s) {
    const int t = sg.t[s], r0 = sg.r0[s], r1 = sg.r1[s];
    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
    float cs = 0.0f;
    for (int rb = r0; rb < r1; rb += kBoxRows, ++b) {
      bool ok = ptx::mbar_try_wait(&bars[b], 0);
      if (!ok) {  // bounded: a box that never lands leaves this CTA's sums at zero
        const uint64_t t0 = ptx::globaltimer();
        while (!(ok = ptx::mbar_try_wait(&bars[b], 0)) && ptx::globaltimer() - t0 < kTimeoutNs) {
        }
      }
      const int R = min(kBoxRows, r1 - rb);
      const uint8_t* pk = sm + (size_t)b * kBoxBytes;
      const uint8_t* sc = pk + kPackBox;
      const float* xr = xs + off + (rb - r0);
      if (ok) {
        uint4 w[2];
        float cf[2];
#pragma unroll
        for (int k = 0; k < 2; ++k) {  // rows warp*4 + sub and 32 later: loads first
          const int i = warp * 4 + sub + k * 32, j = i < R ? i : 0;
          w[k] = *reinterpret_cast<const uint4*>(pk + j * 128 + gi * 16);
          const uint16_t sv = *reinterpret_cast<const uint16_t*>(sc + j * 16 + gi * 2);
          cf[k] = i < R ? __half2float(__ushort_as_half(sv)) * xr[j] : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          if (warp * 4 + k * 32 < R) {  // warp-uniform skip of passes past the box's rows
            cs += cf[k];
            q4_fma_chunk(w[k], cf[k], acc);
          }
        }
      }
    }
    off += r1 - r0;
    // lane (sub, gi) holds 32 outputs of group gi: transposing reduction over the 4 lanes
    // of the group (masks 16, 8) leaves it outputs sub*8 + [0, 8)
    const float bias = cs * 4.3368086899420177e-19f;  // 8 * 2^-64
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[2 * i] = __fmaf_rn(acc[i].x, q4_scale_of_pos((2 * i) & 7), -bias);
      v[2 * i + 1] = __fmaf_rn(acc[i].y, q4_scale_of_pos((2 * i + 1) & 7), -bias);
    }
#pragma unroll
    for (int msk = 16; msk >= 8; msk >>= 1) {
      const bool hi = (lane & msk) != 0;
#pragma unroll
      for (int e2 = 0; e2 < msk; ++e2) {
        const float send = hi ? v[e2] : v[msk + e2];
        const float keep = hi ? v[msk + e2] : v[e2];
        v[e2] = keep + __shfl_xor_sync(0xffffffffu, send, msk);
      }
    }
#pragma unroll
    for (int e2 = 0; e2 < 8; ++e2) red[warp * kTileCols + gi * 32 + sub * 8 + e2] = v[e2];
    __syncthreads();
    // this segment's partial (slot = CTA - first CTA of the tile), published tagged
    int slot_first, slot_last;
    tile_ctas(t, K, G, total, &slot_first, &slot_last);
    const int slot = c - slot_first, nslots = slot_last - slot_first + 1;
    if (tid < kTileCols) {
      float y = 0.0f;
      for (int w = 0; w < kWarps; ++w) y += red[w * kTileCols + tid];
      ptx::st_relaxed_b64(a.partials + ((size_t)t * a.slots + slot) * kTileCols + tid,
                          (1ull << 32) | __float_as_uint(y));
    }
    if (slot == nslots - 1) {
      fin_t[nfin] = t;
      fin_n[nfin] = nslots;
      ++nfin;
    }
    __syncthreads();  // red is rewritten by the next segment
  }
  // finish the tiles whose last slot is ours: every slot's word of column tid, eight loads
  // in flight, stale ones re-read (bounded: a partial that never arrives counts as 0)
  for (int f = 0; f < nfin && tid < kTileCols; ++f) {
    uint64_t* part = a.partials + (size_t)fin_t[f] * a.slots * kTileCols + tid;
    const int ns = fin_n[f];
    float y = 0.0f;
    for (int k0 = 0; k0 < ns; k0 += 8) {
      uint64_t v[8];
      const uint64_t t0 = ptx::globaltimer();
      for (;;) {
        bool ok = true;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          v[k] = k0 + k < ns ? ptx::ld_relaxed_b64(part + (size_t)(k0 + k) * kTileCols) : (1ull << 32);
          ok &= (v[k] >> 32) == 1ull;
        }
        if (ok || ptx::globaltimer() - t0 > kTimeoutNs) break;
      }
#pragma unroll
      for (int k = 0; k < 8; ++k)
        if (k0 + k < ns && (v[k] >> 32) == 1ull) y += __uint_as_float((uint32_t)v[k]);
    }
    const int col = fin_t[f] * kTileCols + tid;
    if (col < a.n) a.y[col] = y;
    for (int k = 0; k < ns; ++k) ptx::st_relaxed_b64(part + (size_t)k * kTileCols, 0ull);
  }
}

}  // namespace g1
}  // namespace qora
