// megakernel.cuh — the whole batch-1 decode step (embedding, every layer, final norm,
// lm_head, greedy argmax, state advance) as ONE persistent kernel: one CTA per SM.
//
// Why: at batch 1 every projection is a ~2-25 MB HBM stream, and a kernel per operation
// pays launch gaps plus the drain/fill of the memory pipeline at each boundary. Here the
// weight stream never stops: each CTA's producer warp walks the CTA's fixed list of
// weight byte ranges for the whole step (they do not depend on activations) and copies
// them with bulk (TMA) copies into a ring of shared-memory stages; the consumer warps
// walk the same list, waiting for (a) the stage to land and (b) the activation the phase
// needs, published by other CTAs through gpu-scope release/acquire counters. While
// consumers wait on a dependency the producer keeps filling the ring.
//
// Per layer (CTA subsets in brackets; split-K partials in global memory):
//   QKV  [last 48 CTAs] fused RMSNorm + q|k|v GEMV -> partials          (qkv_parts)
//   ATTN [units]  each unit reduces the q (and, for the unit holding the new position,
//        k/v) partials itself, applies RoPE, appends the KV row, attends over its
//        chunk of positions (cached K/V rows stream through the ring) -> (m, l, o)
//   O    [32 CTAs] merge the attention partials of the rows it needs, GEMV -> partials
//   GU   [all] x_mid = x_in + sum of O partials (each CTA, full vector), RMSNorm,
//        gate|up GEMV -> partials per tile                                (gu_arr[t])
//   DOWN [all] SwiGLU of the rows it needs from the gate/up partials, GEMV; the last
//        CTA of an output tile adds x_in + O partials + down partials -> x_out (dn_done)
// then lm_head rows (a contiguous slice per CTA) with a fused first-maximum argmax.
// QKV and O run on small disjoint subsets so that their few partials can be reduced by
// the consumers directly, which removes a reduction hop from each of them.
//
// Every wait (dependency counter, stage barrier, ring slot) is bounded by a timeout; on
// expiry the CTA records QORA_ERR_TIMEOUT in the step state, stops computing, drains the
// copies it has in flight and exits. No form of multicast is used.
#pragma once

#include "common.cuh"
#include "ptx.cuh"
#include "q4_gemv.cuh"

namespace qora {
namespace mk {

// 15 consumer warps + 1 producer warp = 4 warps per SM sub-partition, which leaves a
// 128-register budget per thread
constexpr int kCW = 15;                // consumer warps
constexpr int kCT = kCW * 32;          // consumer threads
constexpr int kThreads = kCT + 32;     // + one producer warp
constexpr int kStageBytes = 17280;     // 120 tiled rows of 144 B = 15 embedding rows
constexpr int kStageRows = kStageBytes / kTiledRowBytes;
constexpr int kStages = 11;
constexpr int kMaxVItems = 2;          // (kv head, dim) items per thread in the P.V pass
constexpr int kMaxAttnChunk = 192;
constexpr int kMinAttnChunk = 16;
constexpr int kMaxUnits = 256;         // attention units per step (merge weights buffer)
constexpr int kBar = 1;                // named barrier of the consumer warps
// shared scratch (floats): XS = inputs of this CTA's GEMV segments; B = x copy / merge
// weights / cross-warp reduction; Y = a tile's 256 sums; MISC = small reductions
constexpr int kXsCap = 1536;
constexpr int kBFloats = kCW * kTileCols;       // 3840
constexpr int kOffB = kXsCap;
constexpr int kOffY = kOffB + kBFloats;
constexpr int kOffMisc = kOffY + kTileCols;
constexpr int kScratchFloats = 6272;            // 24.5 KB
// attention layout: q [2048] | scores [16][kMaxAttnChunk] | (m,l) [16][2] | new k,v rows
constexpr int kAttQ = 0, kAttS = 2048, kAttML = kAttS + 16 * kMaxAttnChunk, kAttKV = kAttML + 32;
static_assert(kOffMisc + 256 <= kScratchFloats, "scratch layout");
static_assert(kAttKV + 1024 <= kScratchFloats, "attention scratch");
static_assert(8 * kMaxUnits + 8 <= kBFloats, "merge weights");

constexpr size_t smem_bytes() {
  return (size_t)kStages * kStageBytes + (size_t)kScratchFloats * 4 + 2 * kStages * 8 + 64;
}

enum Mat { QKV = 0, OPR = 1, GU = 2, DOWN = 3 };

struct Layer {
  const uint8_t* w[4];  // tile-major Q4: q|k|v, o, gate/up (interleaved per 128), down
  const float* g_in;
  const float* g_post;
  float* kc;            // K cache [max_seq][nkvw]
  float* vc;
  int rope;
  int pad;
};

struct Args {
  const Layer* layers;
  int L;
  int K[4], tiles[4], slots[4];
  int sub0[4], subn[4];       // CTA subset [sub0, sub0+subn) that runs each matrix
  int segs[4];                // segments (CTA x tile pieces) of each matrix
  int H, I, nq, nkvw, nh, nkvh, grp, vocab;
  int lm_row_bytes, lm_rows_per_stage;
  const uint8_t* lm;          // [vocab][H/2 packed | H/16 scales]
  const float* final_gamma;
  const float* cos_t;
  const float* sin_t;
  int max_pos;                // positions the KV cache (and RoPE table) can hold
  float* xbuf;                // [L+1][H] residual stream (x_0 = embedding, x_{L+1} = out)
  float* logits;              // [vocab]
  float* part[4];             // split-K partials [tiles][slots][256]
  float* att_o;               // [max_units][nh][128]
  float* att_ml;              // [max_units][nh][2]
  int max_units;
  unsigned* cnt;              // dependency counters, zero between launches
  int cpl;                    // counters per layer
  int n_cnt;
  float* lm_v;                // [gridDim.x]
  unsigned* lm_i;
  StepState* st;
  unsigned* ring;
  int ring_cap;
  unsigned long long timeout_ns;
  unsigned long long* trace;  // optional phase timestamps, or nullptr
};

// Trace layout: per CTA kTracePerCta u64 globaltimer stamps written by consumer thread 0:
// [0] start, [1] after embedding, then per layer L at 2 + 8L + {0: x ready, 1: QKV done,
// 2: attention done, 3: attention partials ready, 4: O done, 5: x_mid ready, 6: GU done,
// 7: DOWN done}, then [2+8*kTraceLayers] lm start, [+1] end. Then, per CTA, one stamp per
// layer when the producer has issued that layer's last copy; then kTraceFine stamps of
// layer 1 at finer points (stages, barriers) per CTA.
constexpr int kTraceLayers = 64;
constexpr int kTracePerCta = 2 + 8 * kTraceLayers + 2;
constexpr int kTraceFine = 64;
QORA_DEV void stamp(const Args& a, int c, int idx) {
  if (a.trace && threadIdx.x == 0) a.trace[(long long)c * kTracePerCta + idx] = ptx::globaltimer();
}

// ---- counter layout (per layer L) ----
QORA_DEV int c_qkv_parts(const Args& a, int L) { return L * a.cpl + 0; }
QORA_DEV int c_att(const Args& a, int L) { return L * a.cpl + 1; }
QORA_DEV int c_o_parts(const Args& a, int L) { return L * a.cpl + 2; }
QORA_DEV int c_gu_arr(const Args& a, int L, int t) { return L * a.cpl + 3 + t; }
QORA_DEV int c_dn_arr(const Args& a, int L, int t) { return L * a.cpl + 3 + a.tiles[GU] + t; }
QORA_DEV int c_dn_done(const Args& a, int L) { return L * a.cpl + 3 + a.tiles[GU] + a.tiles[DOWN]; }
QORA_DEV int c_lm(const Args& a) { return a.L * a.cpl; }

QORA_DEV void attn_plan(int len, int G, int& chunk, int& nu) {
  chunk = (len + G - 1) / G;
  chunk = max(kMinAttnChunk, min(kMaxAttnChunk, chunk));
  nu = (len + chunk - 1) / chunk;
}

// split-K slots of tile t of matrix m (its subset's CTAs whose range touches the tile)
QORA_DEV int nslots(const Args& a, int m, int t) {
  const long long K = a.K[m], total = (long long)a.tiles[m] * K;
  const int g = a.subn[m];
  return owner_cta((long long)(t + 1) * K - 1, total, g) - owner_cta((long long)t * K, total, g) + 1;
}

// Sum of the split-K partials of output o of tile t (slot order: deterministic).
QORA_DEV float sum_slots(const Args& a, int m, int t, int o) {
  const float* p = a.part[m] + (long long)t * a.slots[m] * kTileCols + o;
  const int ns = nslots(a, m, t);
  float s = 0.0f;
#pragma unroll 4
  for (int k = 0; k < ns; ++k) s += __ldcg(p + (long long)k * kTileCols);
  return s;
}

// Shared state of one CTA.
struct Smem {
  uint8_t* ring;
  float* scratch;
  uint64_t* full;
  uint64_t* empty;
  volatile int* flags;  // [0] abort, [1] last-arriver, [3] chunks issued, [4] producer done
};

QORA_DEV Smem carve(uint8_t* base) {
  Smem s;
  s.ring = base;
  s.scratch = reinterpret_cast<float*>(base + (size_t)kStages * kStageBytes);
  s.full = reinterpret_cast<uint64_t*>(base + (size_t)kStages * kStageBytes + kScratchFloats * 4);
  s.empty = s.full + kStages;
  s.flags = reinterpret_cast<volatile int*>(s.empty + kStages);
  return s;
}

// Segments of CTA c in the flattened (tile, row) space of matrix m: f(t, r0, r1, slot).
template <class F>
QORA_DEV void for_each_segment(const Args& a, int m, int c, F&& f) {
  const int lc = c - a.sub0[m], g = a.subn[m];
  if (lc < 0 || lc >= g) return;
  const long long K = a.K[m], total = (long long)a.tiles[m] * K;
  const long long lin0 = (long long)lc * total / g, lin1 = (long long)(lc + 1) * total / g;
  for (long long p = lin0; p < lin1;) {
    const long long t = p / K, r0 = p - t * K;
    const long long pe = min(lin1, (t + 1) * K);
    const int slot = lc - owner_cta(t * K, total, g);
    f((int)t, (int)r0, (int)(pe - t * K), slot);
    p = pe;
  }
}

// ------------------------------------------------------------------ the chunk sequence
// The producer walks exactly this sequence of (source, bytes) copies; the consumers
// consume the same sequence in the same order (see the phases below).
template <class F, class E>
QORA_DEV void for_each_chunk(const Args& a, int c, int G, int pos, F&& f, E&& layer_end) {
  const int len = pos + 1;
  int chunk, nu;
  attn_plan(len, G, chunk, nu);
  const int kvrow = a.nkvw * 4;
  const int kv_rows_stage = kStageBytes / kvrow;
  auto gemv = [&](int m, int L) {
    const uint8_t* base = a.layers[L].w[m];
    const long long K = a.K[m];
    for_each_segment(a, m, c, [&](int t, int r0, int r1, int) {
      for (int r = r0; r < r1; r += kStageRows) {
        const int n = min(kStageRows, r1 - r);
        f(base + ((long long)t * K + r) * kTiledRowBytes, (uint32_t)(n * kTiledRowBytes));
      }
    });
  };
  for (int L = 0; L < a.L; ++L) {
    gemv(QKV, L);
    for (int u = c; u < nu; u += G) {
      const int s0 = u * chunk, s1 = min(len, s0 + chunk), sc1 = min(s1, pos);
      for (int kvs = 0; kvs < 2; ++kvs) {
        const float* src = kvs ? a.layers[L].vc : a.layers[L].kc;
        for (int s = s0; s < sc1; s += kv_rows_stage) {
          const int n = min(kv_rows_stage, sc1 - s);
          f(reinterpret_cast<const uint8_t*>(src + (long long)s * a.nkvw), (uint32_t)(n * kvrow));
        }
      }
    }
    gemv(OPR, L);
    gemv(GU, L);
    gemv(DOWN, L);
    layer_end(L);
  }
  const long long v0 = (long long)c * a.vocab / G, v1 = (long long)(c + 1) * a.vocab / G;
  for (long long r = v0; r < v1; r += a.lm_rows_per_stage) {
    const long long n = min((long long)a.lm_rows_per_stage, v1 - r);
    f(a.lm + r * a.lm_row_bytes, (uint32_t)(n * a.lm_row_bytes));
  }
}

// ------------------------------------------------------------------ consumer helpers
struct Cons {
  const Args& a;
  Smem sm;
  int c, G, tid, lane, warp, pos, token;
  int layer = 0;
  int fine = 0;
  uint32_t chunk = 0;
  uint32_t stage_idx = 0;
  bool stage_ok = false;  // warp-uniform: the current stage landed and the CTA is healthy

  // consistent across the consumer warps between named barriers
  QORA_DEV bool aborted() const { return sm.flags[0] != 0; }
  // uniform within the calling warp at any point
  QORA_DEV bool aborted_w() const { return __shfl_sync(0xffffffffu, sm.flags[0] != 0, 0); }

  QORA_DEV void set_abort(int code) {
    sm.flags[0] = 1;
    atomicExch(&a.st->error, code);
  }

  QORA_DEV void bar() { ptx::named_bar(kBar, kCT); }

  // barrier that also agrees on the abort state: every consumer gets the same answer, so
  // it may gate code that contains further barriers (the producer can raise the flag at
  // any time, so a plain read after a barrier is not enough)
  QORA_DEV bool sync_aborted() {
    const int v = sm.flags[0] != 0;
    int r;
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.s32 p, %1, 0;\n bar.red.or.pred p, 1, %2, p;\n"
        " selp.s32 %0, 1, 0, p;\n}\n"
        : "=r"(r)
        : "r"(v), "r"(kCT)
        : "memory");
    return r != 0;
  }

  QORA_DEV void fstamp() {
    if (a.trace && layer == 1 && tid == 0 && fine < kTraceFine)
      a.trace[(long long)G * (kTracePerCta + kTraceLayers) + (long long)c * kTraceFine + fine] =
          ptx::globaltimer();
    if (layer == 1) ++fine;
  }

  // thread 0 spins (bounded) until *p >= target; no barrier
  QORA_DEV void spin_ge(const unsigned* p, unsigned target) {
    if (aborted()) return;
    if (ptx::ld_acquire(p) >= target) return;
    const uint64_t t0 = ptx::globaltimer();
    while (ptx::ld_acquire(p) < target) {
      if (ptx::globaltimer() - t0 > a.timeout_ns) {
        set_abort(2);
        return;
      }
    }
  }

  // thread 0 waits until *p >= target; all consumers then see the outcome
  QORA_DEV void wait_ge(const unsigned* p, unsigned target) {
    if (tid == 0) spin_ge(p, target);
    bar();
  }

  // next stage of the ring (every consumer warp calls this for every chunk, in order).
  // Once the CTA has aborted, stages are skipped without waiting (see drain()).
  QORA_DEV const uint8_t* acquire_stage() {
    stage_idx = chunk % kStages;
    const uint32_t parity = (chunk / kStages) & 1u;
    if (aborted_w()) {
      stage_ok = false;
      return sm.ring;
    }
    bool timed_out = false;
    if (!ptx::mbar_try_wait(&sm.full[stage_idx], parity)) {
      const uint64_t t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&sm.full[stage_idx], parity)) {
        if (ptx::globaltimer() - t0 > a.timeout_ns) {
          timed_out = true;
          break;
        }
      }
    }
    stage_ok = __all_sync(0xffffffffu, !timed_out);
    if (!stage_ok && lane == 0) set_abort(2);
    return sm.ring + (size_t)stage_idx * kStageBytes;
  }

  QORA_DEV void release_stage() {
    __syncwarp();
    if (lane == 0 && stage_ok) ptx::mbar_arrive(&sm.empty[stage_idx]);
    ++chunk;
  }

  // After an abort: wait (bounded) for the producer to stop and for the copies it issued
  // last to land, so that no bulk copy targets this CTA's shared memory after it exits.
  QORA_DEV void drain() {
    bar();
    if (tid == 0 && aborted()) {
      const uint64_t t0 = ptx::globaltimer();
      while (sm.flags[4] == 0 && ptx::globaltimer() - t0 < a.timeout_ns) {
      }
      const uint32_t issued = (uint32_t)sm.flags[3];
      const uint32_t first = issued > (uint32_t)kStages ? issued - kStages : 0u;
      for (uint32_t j = first; j < issued; ++j) {
        const uint64_t t1 = ptx::globaltimer();
        while (!ptx::mbar_try_wait(&sm.full[j % kStages], (j / kStages) & 1u) &&
               ptx::globaltimer() - t1 < a.timeout_ns) {
        }
      }
    }
    bar();
  }

  // block sum over consumer threads (fixed order), result in every thread
  QORA_DEV float csum(float v) {
    float* red = sm.scratch + kOffMisc;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    bar();
    float t = 0.0f;
    for (int w = 0; w < kCW; ++w) t += red[w];
    bar();
    return t;
  }

  // publish: every consumer's prior global writes, then a release increment
  QORA_DEV void publish(unsigned* ctr) {
    bar();
    if (tid == 0) ptx::red_add_release(ctr, 1u);
  }
};

QORA_DEV void load_vec(Cons& C, float* dst, const float* src, int n) {
  for (int i = C.tid; i < n; i += kCT) dst[i] = __ldcg(src + i);
}

QORA_DEV float rms_inv_of(Cons& C, const float* sx, int H) {
  float s = 0.0f;
  for (int i = C.tid; i < H; i += kCT) s = __fmaf_rn(sx[i], sx[i], s);
  const float tot = C.csum(s);
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, (float)H), 1e-6f)));
}

// x_mid = x_in + (sum of the O partials) for every column, into shared memory sx
QORA_DEV void build_x_mid(Cons& C, float* sx, const float* x_in, int H) {
  const Args& a = C.a;
  for (int i = C.tid; i < H; i += kCT) {
    const float xi = __ldcg(x_in + i);
    sx[i] = __fadd_rn(xi, sum_slots(a, OPR, i / kTileCols, i % kTileCols));
  }
}

// One GEMV phase for this CTA (nothing if the CTA is outside the matrix's subset).
// pro(t, r0, r1, xs) fills xs[0..r1-r0) with the inputs of rows r0..r1 of one segment
// (it may wait and use barriers; every consumer calls it); all segments' inputs are
// prepared before streaming. After each segment's partial is stored, done(t, slot)
// runs on every consumer (it publishes the partial / detects the last arriver).
template <class Pro, class Done>
QORA_DEV void gemv_phase(Cons& C, int m, int L, Pro&& pro, Done&& done) {
  const Args& a = C.a;
  float* xs = C.sm.scratch;
  float* red = C.sm.scratch + kOffB;
  const int gi = C.lane & 7, sub = C.lane >> 3;
  const float kX = 18446744073709551616.0f;  // 2^64

  // 1) inputs of every segment
  int n_in = 0;
  for_each_segment(a, m, C.c, [&](int t, int r0, int r1, int) {
    C.fstamp();
    if (!C.sync_aborted()) pro(t, r0, r1, xs + n_in);
    n_in += r1 - r0;
  });
  if (n_in == 0) return;  // CTA not in this matrix's subset (uniform)
  C.bar();
  for (int i = C.tid; i < n_in; i += kCT) xs[i] *= kX;
  C.bar();
  C.fstamp();

  // 2) stream and accumulate
  int off = 0;
  for_each_segment(a, m, C.c, [&](int t, int r0, int r1, int slot) {
    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
    float cs = 0.0f;
    for (int cr = r0; cr < r1; cr += kStageRows) {
      const uint8_t* stg = C.acquire_stage();
      const int R = min(kStageRows, r1 - cr);
      if (C.stage_ok) {
        const float* xr = xs + off + (cr - r0);
        // two rows per lane per stage, both rows' loads issued before the math
        const int i0 = C.warp * 4 + sub, i1 = i0 + kCW * 4;
        const bool v0 = i0 < R, v1 = i1 < R;
        const uint8_t* row0 = stg + (v0 ? i0 : 0) * kTiledRowBytes;
        const uint8_t* row1 = stg + (v1 ? i1 : 0) * kTiledRowBytes;
        const uint4 w0 = *reinterpret_cast<const uint4*>(row0 + gi * 16);
        const uint4 w1 = *reinterpret_cast<const uint4*>(row1 + gi * 16);
        const uint16_t s0 = *reinterpret_cast<const uint16_t*>(row0 + kTileGroups * 16 + gi * 2);
        const uint16_t s1 = *reinterpret_cast<const uint16_t*>(row1 + kTileGroups * 16 + gi * 2);
        const float c0 = v0 ? __half2float(__ushort_as_half(s0)) * xr[i0] : 0.0f;
        const float c1 = v1 ? __half2float(__ushort_as_half(s1)) * xr[i1] : 0.0f;
        cs += c0 + c1;
        q4_fma_chunk(w0, c0, acc);
        q4_fma_chunk(w1, c1, acc);
      }
      C.release_stage();
      C.fstamp();
    }
    off += r1 - r0;

    // finalize this lane's 32 outputs, then a transposing reduction over the 4 row
    // lanes of each group: afterwards lane (sub, gi) holds 8 summed outputs
    const float bias = cs * 4.3368086899420177e-19f;  // 8 * 2^-64
    float yv[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      yv[2 * i] = __fmaf_rn(acc[i].x, q4_scale_of_pos((2 * i) & 7), -bias);
      yv[2 * i + 1] = __fmaf_rn(acc[i].y, q4_scale_of_pos((2 * i + 1) & 7), -bias);
    }
    const bool hi16 = (sub & 2) != 0, hi8 = (sub & 1) != 0;
    float h[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float send = hi16 ? yv[e] : yv[16 + e];
      const float keep = hi16 ? yv[16 + e] : yv[e];
      h[e] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
    }
    float q8[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float send = hi8 ? h[e] : h[8 + e];
      const float keep = hi8 ? h[8 + e] : h[e];
      q8[e] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
    }
    {
      const int base = C.warp * kTileCols + gi * kGroup + (hi16 ? 16 : 0) + (hi8 ? 8 : 0);
      float4* dst = reinterpret_cast<float4*>(red + base);
      dst[0] = make_float4(q8[0], q8[1], q8[2], q8[3]);
      dst[1] = make_float4(q8[4], q8[5], q8[6], q8[7]);
    }
    C.bar();
    float* part = a.part[m] + ((long long)t * a.slots[m] + slot) * kTileCols;
    if (C.tid < kTileCols) {
      const int o = C.tid;
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) s += red[w * kTileCols + o];
      __stcg(part + o, s);
    }
    C.bar();
    C.fstamp();
    done(t, slot);
    C.fstamp();
  });
}

// ------------------------------------------------------------------ the kernel
template <int GPL>
__global__ void __launch_bounds__(kThreads, 1) decode_megakernel(const Args a) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  Smem sm = carve(smem_raw);
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x, G = gridDim.x;
  const int pos = a.st->pos;
  const int token = a.st->token;

  if (tid == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&sm.full[s], 1);
      ptx::mbar_init(&sm.empty[s], kCW);
    }
    sm.flags[0] = (token < 0 || token >= a.vocab || pos < 0 || pos >= a.max_pos) ? 1 : 0;
    sm.flags[1] = 0;
    sm.flags[3] = 0;
    sm.flags[4] = 0;
    ptx::fence_mbar_init();
  }
  __syncthreads();  // last block-wide barrier: the producer warp leaves below

  if (warp == kCW) {
    // ---------------- producer: stream this CTA's bytes in consumption order
    if (lane == 0) {
      uint32_t chunk = 0;
      bool dead = sm.flags[0] != 0;
      for_each_chunk(
          a, c, G, pos,
          [&](const uint8_t* src, uint32_t bytes) {
            if (dead) return;
            const uint32_t s = chunk % kStages;
            const uint32_t parity = ((chunk / kStages) & 1u) ^ 1u;
            if (!ptx::mbar_try_wait(&sm.empty[s], parity)) {
              const uint64_t t0 = ptx::globaltimer();
              while (!ptx::mbar_try_wait(&sm.empty[s], parity)) {
                if (sm.flags[0] != 0) {  // consumers gave up: stop issuing
                  dead = true;
                  return;
                }
                if (ptx::globaltimer() - t0 > a.timeout_ns) {
                  dead = true;
                  sm.flags[0] = 1;
                  atomicExch(&a.st->error, 2);
                  return;
                }
              }
            }
            ptx::mbar_arrive_expect_tx(&sm.full[s], bytes);
            ptx::bulk_g2s(sm.ring + (size_t)s * kStageBytes, src, bytes, &sm.full[s]);
            ++chunk;
          },
          [&](int L) {
            if (a.trace && L < kTraceLayers)
              a.trace[(long long)G * kTracePerCta + (long long)c * kTraceLayers + L] = ptx::globaltimer();
          });
      sm.flags[3] = (int)chunk;
      __threadfence_block();
      sm.flags[4] = 1;
    }
    return;
  }

  // ---------------- consumers
  stamp(a, c, 0);
  Cons C{a, sm, c, G, tid, lane, warp, pos, token};
  if (sm.flags[0] && tid == 0) atomicExch(&a.st->error, 1);
  const int H = a.H;
  float* sB = sm.scratch + kOffB;  // x copy for the norms
  float* sMisc = sm.scratch + kOffMisc;

  // embedding row (embed_lookup_q4, src/gemv.rs:710-736): every CTA builds x_0 locally
  if (!C.aborted()) {
    const uint8_t* row = a.lm + (long long)token * a.lm_row_bytes;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(row + H / 2);
    for (int e = tid; e < H; e += kCT) {
      const uint8_t b = row[e >> 1];
      const int q = ((e & 1) ? (b >> 4) : (b & 0xF)) - 8;
      const float v = __fmul_rn(__half2float(__ushort_as_half(sc[e / kGroup])), (float)q);
      sB[e] = v;
      if (c == 0) a.xbuf[e] = v;
    }
  }
  C.bar();
  stamp(a, c, 1);

  int chunk_sz, nu;
  attn_plan(pos + 1, G, chunk_sz, nu);
  const float att_scale = __fdiv_rn(1.0f, __fsqrt_rn((float)kHeadDim));

  for (int L = 0; L < a.L; ++L) {
    const Layer& ly = a.layers[L];
    C.layer = L;
    const float* x_in = a.xbuf + (long long)L * H;
    float* x_out = a.xbuf + (long long)(L + 1) * H;
    const int tb = 2 + 8 * min(L, kTraceLayers - 1);

    // ===== QKV (subset): RMSNorm(x_in) . Wqkv -> partials
    const bool in_qkv = (c >= a.sub0[QKV] && c < a.sub0[QKV] + a.subn[QKV]);
    if (in_qkv) {
      if (L > 0) {
        C.wait_ge(a.cnt + c_dn_done(a, L - 1), (unsigned)a.tiles[DOWN]);
        if (!C.aborted()) load_vec(C, sB, x_in, H);
        C.bar();
      }
      stamp(a, c, tb + 0);
      const float inv = C.sync_aborted() ? 1.0f : rms_inv_of(C, sB, H);
      gemv_phase(
          C, QKV, L,
          [&](int, int r0, int r1, float* xs) {
            for (int i = C.tid; i < r1 - r0; i += kCT)
              xs[i] = __fmul_rn(__fmul_rn(sB[r0 + i], inv), __ldg(ly.g_in + r0 + i));
          },
          [&](int, int) { C.publish(a.cnt + c_qkv_parts(a, L)); });
    }
    stamp(a, c, tb + 1);

    // ===== ATTN (units of `chunk_sz` positions, all query heads)
    {
      const int kvrow = a.nkvw * 4;
      const int rps = kStageBytes / kvrow;
      float* sq = sm.scratch + kAttQ;    // [nh][128] (RoPE applied)
      float* sc = sm.scratch + kAttS;    // [nh][kMaxAttnChunk]
      float* sml = sm.scratch + kAttML;  // [nh][2]
      float* skv = sm.scratch + kAttKV;  // new k row [nkvw] | new v row [nkvw]
      const int gq = lane >> 3, li = lane & 7;  // K pass: 4 row groups x 8 lanes of 16 dims
      const int nv = a.nkvh * kHeadDim;         // P.V items: (kv head, dim)
      bool ready = false;
      for (int u = c; u < nu; u += G) {
        const int s0 = u * chunk_sz, s1 = min(pos + 1, s0 + chunk_sz), sc1 = min(s1, pos);
        const int n = s1 - s0;
        const bool has_pos = pos >= s0 && pos < s1;
        if (!ready) {
          C.wait_ge(a.cnt + c_qkv_parts(a, L), (unsigned)a.segs[QKV]);
          C.fstamp();
          // q (and k|v for the unit holding the new position) from the QKV partials,
          // RoPE on q and k (src/gemv.rs:757-778); k|v appended to the cache
          if (!C.aborted()) {
            const int ncols = a.nq + 2 * a.nkvw;
            for (int i = tid; i < ncols / 2; i += kCT) {
              // pair (col, col + 64) within one head: i -> head hh, dim d < 64
              const int hh = i / kHalfDim, d = i % kHalfDim;
              const int col = hh * kHeadDim + d;
              if (col >= a.nq && !has_pos) continue;
              const float x1 = sum_slots(a, QKV, col / kTileCols, col % kTileCols);
              const float x2 = sum_slots(a, QKV, (col + kHalfDim) / kTileCols, (col + kHalfDim) % kTileCols);
              float y1 = x1, y2 = x2;
              if (ly.rope && col < a.nq + a.nkvw) {
                const float cs = a.cos_t[(long long)pos * kHalfDim + d];
                const float sn = a.sin_t[(long long)pos * kHalfDim + d];
                y1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
                y2 = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
              }
              if (col < a.nq) {
                sq[col] = y1;
                sq[col + kHalfDim] = y2;
              } else {
                const int kc = col - a.nq;  // within k|v
                skv[kc] = y1;
                skv[kc + kHalfDim] = y2;
                float* dst = (kc < a.nkvw) ? ly.kc + (long long)pos * a.nkvw + kc
                                           : ly.vc + (long long)pos * a.nkvw + (kc - a.nkvw);
                dst[0] = y1;
                dst[kHalfDim] = y2;
              }
            }
          }
          C.bar();
          ready = true;
        }
        // one K row per 8-lane group; every lane of the warp executes the shuffles
        auto score = [&](int hq, const float* krow, int idx, bool valid) {
          float acc = 0.0f;
          if (valid) {
            const float4* kp = reinterpret_cast<const float4*>(krow + (hq / a.grp) * kHeadDim + li * 16);
            const float4* qp = reinterpret_cast<const float4*>(sq + hq * kHeadDim + li * 16);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 k4 = kp[j];
              const float4 q4 = qp[j];
              acc = __fmaf_rn(q4.x, k4.x, acc);
              acc = __fmaf_rn(q4.y, k4.y, acc);
              acc = __fmaf_rn(q4.z, k4.z, acc);
              acc = __fmaf_rn(q4.w, k4.w, acc);
            }
          }
          acc += __shfl_xor_sync(0xffffffffu, acc, 1);
          acc += __shfl_xor_sync(0xffffffffu, acc, 2);
          acc += __shfl_xor_sync(0xffffffffu, acc, 4);
          if (valid && li == 0) sc[hq * kMaxAttnChunk + idx] = __fmul_rn(acc, att_scale);
        };
        for (int s = s0; s < sc1; s += rps) {
          const uint8_t* stg = C.acquire_stage();
          const int nr = min(rps, sc1 - s);
          if (C.stage_ok) {  // warp-uniform
            for (int hq = warp; hq < a.nh; hq += kCW)
              for (int ib = 0; ib < nr; ib += 4) {
                const int i = ib + gq;
                score(hq, reinterpret_cast<const float*>(stg + min(i, nr - 1) * kvrow), s - s0 + i, i < nr);
              }
          }
          C.release_stage();
          C.fstamp();
        }
        if (!C.aborted_w() && has_pos)  // warp-uniform: the new row, from shared memory
          for (int hq = warp; hq < a.nh; hq += kCW) score(hq, skv, pos - s0, gq == 0);
        C.bar();
        // chunk softmax numerators: query heads spread over warps
        if (!C.aborted_w()) {
          for (int hq = warp; hq < a.nh; hq += kCW) {
            float* row = sc + hq * kMaxAttnChunk;
            float mx = -INFINITY;
            for (int i = lane; i < n; i += 32) mx = fmaxf(mx, row[i]);
            mx = warp_max(mx);
            float l = 0.0f;
            for (int i = lane; i < n; i += 32) {
              const float e = expf(row[i] - mx);
              row[i] = e;
              l += e;
            }
            l = warp_sum(l);
            if (lane == 0) {
              sml[hq * 2] = mx;
              sml[hq * 2 + 1] = l;
            }
          }
        }
        C.bar();
        C.fstamp();
        // P.V: item (kv head g, dim d) accumulates the grp query heads that share g
        float o[kMaxVItems][4];
#pragma unroll
        for (int k = 0; k < kMaxVItems; ++k)
#pragma unroll
          for (int j = 0; j < 4; ++j) o[k][j] = 0.0f;
        for (int s = s0; s < sc1; s += rps) {
          const uint8_t* stg = C.acquire_stage();
          const int nr = min(rps, sc1 - s);
          if (C.stage_ok) {
#pragma unroll
            for (int k = 0; k < kMaxVItems; ++k) {
              const int it = tid + k * kCT;
              if (it < nv) {
                const int g = it / kHeadDim, d = it % kHeadDim;
                for (int i = 0; i < nr; ++i) {
                  const float v = reinterpret_cast<const float*>(stg + i * kvrow)[g * kHeadDim + d];
                  const int idx = s - s0 + i;
#pragma unroll
                  for (int j = 0; j < 4; ++j)
                    if (j < a.grp) o[k][j] = __fmaf_rn(sc[(g * a.grp + j) * kMaxAttnChunk + idx], v, o[k][j]);
                }
              }
            }
          }
          C.release_stage();
          C.fstamp();
        }
        if (!C.aborted()) {
#pragma unroll
          for (int k = 0; k < kMaxVItems; ++k) {
            const int it = tid + k * kCT;
            if (it < nv) {
              const int g = it / kHeadDim, d = it % kHeadDim;
              if (has_pos) {
                const float v = skv[a.nkvw + g * kHeadDim + d];
#pragma unroll
                for (int j = 0; j < 4; ++j)
                  if (j < a.grp) o[k][j] = __fmaf_rn(sc[(g * a.grp + j) * kMaxAttnChunk + (pos - s0)], v, o[k][j]);
              }
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if (j < a.grp) __stcg(a.att_o + ((long long)u * a.nh + g * a.grp + j) * kHeadDim + d, o[k][j]);
            }
          }
          if (tid < a.nh) {
            __stcg(a.att_ml + ((long long)u * a.nh + tid) * 2, sml[tid * 2]);
            __stcg(a.att_ml + ((long long)u * a.nh + tid) * 2 + 1, sml[tid * 2 + 1]);
          }
        }
        C.publish(a.cnt + c_att(a, L));
        C.bar();
      }
    }
    stamp(a, c, tb + 2);

    // ===== O projection (subset): merge attention partials for the rows it needs
    const bool in_o = (c >= a.sub0[OPR] && c < a.sub0[OPR] + a.subn[OPR]);
    if (in_o) {
      C.wait_ge(a.cnt + c_att(a, L), (unsigned)nu);
      stamp(a, c, tb + 3);
      float* mw = sm.scratch + kOffB;  // [<=8 heads][kMaxUnits] weights, then 1/L per head
      gemv_phase(
          C, OPR, L,
          [&](int, int r0, int r1, float* xs) {
            const int h0 = r0 / kHeadDim, h1 = (r1 - 1) / kHeadDim;
            const int nhs = h1 - h0 + 1;  // <= 8 (host checks the segment length)
            // per head: M = max m_u, w_u = exp(m_u - M), 1/L with L = sum l_u w_u
            if (warp < nhs) {
              const int h = h0 + warp;
              float mx = -INFINITY;
              for (int u = lane; u < nu; u += 32) mx = fmaxf(mx, __ldcg(a.att_ml + ((long long)u * a.nh + h) * 2));
              mx = warp_max(mx);
              float l = 0.0f;
              for (int u = lane; u < nu; u += 32) {
                const float2 ml = __ldcg(reinterpret_cast<const float2*>(a.att_ml + ((long long)u * a.nh + h) * 2));
                const float w = expf(ml.x - mx);
                mw[warp * kMaxUnits + u] = w;
                l = __fmaf_rn(ml.y, w, l);
              }
              l = warp_sum(l);
              if (lane == 0) mw[8 * kMaxUnits + warp] = __fdiv_rn(1.0f, l);
            }
            C.bar();
            for (int i = C.tid; i < r1 - r0; i += kCT) {
              const int r = r0 + i, h = r / kHeadDim, dd = r % kHeadDim, j = h - h0;
              const float* op = a.att_o + (long long)h * kHeadDim + dd;
              float acc = 0.0f;
#pragma unroll 4
              for (int u = 0; u < nu; ++u)
                acc = __fmaf_rn(__ldcg(op + (long long)u * a.nh * kHeadDim), mw[j * kMaxUnits + u], acc);
              xs[i] = __fmul_rn(acc, mw[8 * kMaxUnits + j]);
            }
            C.bar();
          },
          [&](int, int) { C.publish(a.cnt + c_o_parts(a, L)); });
    }
    stamp(a, c, tb + 4);

    // ===== gate/up (all): x_mid = x_in + O partials, RMSNorm, GEMV -> partials per tile
    C.wait_ge(a.cnt + c_o_parts(a, L), (unsigned)a.segs[OPR]);
    stamp(a, c, tb + 5);
    {
      if (!C.aborted()) build_x_mid(C, sB, x_in, H);
      C.bar();
      const float inv2 = C.sync_aborted() ? 1.0f : rms_inv_of(C, sB, H);
      gemv_phase(
          C, GU, L,
          [&](int, int r0, int r1, float* xs) {
            for (int i = C.tid; i < r1 - r0; i += kCT)
              xs[i] = __fmul_rn(__fmul_rn(sB[r0 + i], inv2), __ldg(ly.g_post + r0 + i));
          },
          [&](int t, int) { C.publish(a.cnt + c_gu_arr(a, L, t)); });
    }
    stamp(a, c, tb + 6);

    // ===== down (all): SwiGLU of the rows it needs from the gate/up partials; the last
    // CTA of each output tile writes x_out = x_in + O + down for the tile
    gemv_phase(
        C, DOWN, L,
        [&](int, int r0, int r1, float* xs) {
          const int t0 = r0 / (kTileCols / 2), t1 = (r1 - 1) / (kTileCols / 2);
          if (C.tid == 0)
            for (int tg = t0; tg <= t1; ++tg) C.spin_ge(a.cnt + c_gu_arr(a, L, tg), (unsigned)nslots(a, GU, tg));
          if (C.sync_aborted()) return;
          for (int i = C.tid; i < r1 - r0; i += kCT) {
            const int r = r0 + i, tg = r / (kTileCols / 2), o = r % (kTileCols / 2);
            const float g = sum_slots(a, GU, tg, o);
            const float u = sum_slots(a, GU, tg, kTileCols / 2 + o);
            const float sg = __fdiv_rn(g, __fadd_rn(1.0f, expf(-g)));
            xs[i] = __fmul_rn(sg, u);
          }
        },
        [&](int t, int) {
          if (C.tid == 0) {
            const unsigned prev = ptx::atom_add_acqrel(a.cnt + c_dn_arr(a, L, t), 1u);
            C.sm.flags[1] = (prev == (unsigned)(nslots(a, DOWN, t) - 1));
          }
          C.bar();
          if (C.sm.flags[1]) {
            if (C.tid < kTileCols) {
              const int col = t * kTileCols + C.tid;
              if (col < H) {
                const float xm = __fadd_rn(__ldcg(x_in + col), sum_slots(a, OPR, t, C.tid));
                x_out[col] = __fadd_rn(xm, sum_slots(a, DOWN, t, C.tid));
              }
            }
            C.publish(a.cnt + c_dn_done(a, L));
          }
          C.bar();
        });
    stamp(a, c, tb + 7);
  }

  // ===== final norm + lm_head + argmax
  C.wait_ge(a.cnt + c_dn_done(a, a.L - 1), (unsigned)a.tiles[DOWN]);
  stamp(a, c, 2 + 8 * kTraceLayers);
  const float* x_fin = a.xbuf + (long long)a.L * H;
  if (!C.aborted()) load_vec(C, sB, x_fin, H);
  C.bar();
  {
    const float inv = C.sync_aborted() ? 1.0f : rms_inv_of(C, sB, H);
    for (int i = tid; i < H; i += kCT) sB[i] = __fmul_rn(__fmul_rn(sB[i], inv), a.final_gamma[i]);
  }
  C.bar();
  constexpr int EPL = GPL * 32;
  float2 xs2[EPL / 2];
  float xg[GPL];
#pragma unroll
  for (int g = 0; g < GPL; ++g) {
    float s = 0.0f;
#pragma unroll
    for (int e = 0; e < 32; ++e) {
      const float v = sB[lane * EPL + g * 32 + e];
      s += v;
      const int mm = e & 7;
      const int p = (mm < 5) ? 4 * mm : 4 * mm - 12;
      const float f = __fmul_rn(v, __int_as_float((127 + 85 - p) << 23));
      if (e & 1) xs2[(g * 32 + e) / 2].y = f; else xs2[(g * 32 + e) / 2].x = f;
    }
    xg[g] = s * 8.0f;
  }
  float best = -INFINITY;
  unsigned besti = 0xFFFFFFFFu;
  {
    const long long v0 = (long long)c * a.vocab / G, v1 = (long long)(c + 1) * a.vocab / G;
    const float k64 = 18446744073709551616.0f;
    for (long long r = v0; r < v1; r += a.lm_rows_per_stage) {
      const uint8_t* stg = C.acquire_stage();
      const int nr = (int)min((long long)a.lm_rows_per_stage, v1 - r);
      if (C.stage_ok) {
        for (int i = warp; i < nr; i += kCW) {
          const uint8_t* row = stg + (size_t)i * a.lm_row_bytes;
          const uint4* wp = reinterpret_cast<const uint4*>(row) + lane * GPL;
          const uint16_t* sp = reinterpret_cast<const uint16_t*>(row + H / 2) + lane * GPL;
          float acc = 0.0f;
#pragma unroll
          for (int g = 0; g < GPL; ++g) {
            const uint4 w = wp[g];
            float2 dd = make_float2(0.0f, 0.0f);
            const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              const uint32_t uu = ws[k], bb = uu >> 12;
              const int base = (g * 32 + k * 8) / 2;
              dd = __ffma2_rn(make_float2(__uint_as_float(uu & 0xFu), __uint_as_float(uu & 0xF0u)), xs2[base + 0], dd);
              dd = __ffma2_rn(make_float2(__uint_as_float(uu & 0xF00u), __uint_as_float(uu & 0xF000u)), xs2[base + 1], dd);
              dd = __ffma2_rn(make_float2(__uint_as_float(uu & 0xF0000u), __uint_as_float(bb & 0xF00u)), xs2[base + 2], dd);
              dd = __ffma2_rn(make_float2(__uint_as_float(bb & 0xF000u), __uint_as_float(bb & 0xF0000u)), xs2[base + 3], dd);
            }
            const float dot = __fmaf_rn(dd.x + dd.y, k64, -xg[g]);
            acc = __fmaf_rn(__half2float(__ushort_as_half(sp[g])), dot, acc);
          }
          acc = warp_sum(acc);
          const unsigned vi = (unsigned)(r + i);
          if (lane == 0) a.logits[vi] = acc;
          if (better(acc, vi, best, besti)) {
            best = acc;
            besti = vi;
          }
        }
      }
      C.release_stage();
    }
  }
  stamp(a, c, 2 + 8 * kTraceLayers + 1);
  C.drain();
  // CTA argmax -> global partial -> last CTA finishes the step
  float* bvs = sMisc;
  unsigned* bis = reinterpret_cast<unsigned*>(sMisc + kCW);
  if (lane == 0) {
    bvs[warp] = best;
    bis[warp] = besti;
  }
  C.bar();
  if (tid == 0) {
    float b = bvs[0];
    unsigned bi = bis[0];
    for (int w = 1; w < kCW; ++w)
      if (better(bvs[w], bis[w], b, bi)) { b = bvs[w]; bi = bis[w]; }
    __stcg(a.lm_v + c, b);
    __stcg(a.lm_i + c, bi);
    const unsigned prev = ptx::atom_add_acqrel(a.cnt + c_lm(a), 1u);
    sm.flags[1] = (prev == (unsigned)(G - 1));
  }
  C.bar();
  if (!sm.flags[1]) return;
  if (tid == 0) {
    float b = -INFINITY;
    unsigned bi = 0xFFFFFFFFu;
    for (int k = 0; k < G; ++k) {
      const float v = __ldcg(a.lm_v + k);
      const unsigned ii = __ldcg(a.lm_i + k);
      if (better(v, ii, b, bi)) { b = v; bi = ii; }
    }
    const unsigned am = (bi == 0xFFFFFFFFu) ? 0u : bi;
    StepState* st = a.st;
    st->argmax = am;
    const int s = st->step;
    if (a.ring && s >= 0 && s < a.ring_cap) a.ring[s] = am;
    st->step = s + 1;
    st->token = (int)am;
    st->pos = pos + 1;
  }
  // every CTA has arrived: reset the dependency counters for the next launch
  for (int i = tid; i < a.n_cnt; i += kCT) a.cnt[i] = 0u;
}

}  // namespace mk
}  // namespace qora
