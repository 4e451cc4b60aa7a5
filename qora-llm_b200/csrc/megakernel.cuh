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
// Per layer (CTA sets in brackets):
//   QKV  [one CTA per 32-column group of q|k|v] RMSNorm(x) . W over all rows -> final
//        q|k|v values (before RoPE), no split-K
//   ATTN [one CTA per (kv head, chunk of positions)] RoPE on its 4 query heads (and,
//        for the chunk holding the new position, on k, which it appends with v to the
//        head-major cache), scores, softmax numerators, P.V -> (m, l, o); the last unit
//        of a KV head (atomic arrival count) merges the chunks and publishes the heads'
//        normalised output (one chunk: the unit publishes o / l itself)
//   O    [one CTA per 32-column group of o_proj] the merged attention output of all
//        heads, GEMV over all rows, x_mid = x + o for its columns
//   GU   [all] RMSNorm(x_mid) . [gate|up], split-K over 256-column tiles -> partials
//   DOWN [all] SwiGLU of its rows from the gate/up partials, split-K GEMV with every
//        CTA's rows inside one output tile; the last CTA of a tile (atomic arrival
//        count) writes x_next = x_mid + down for it
// then lm_head rows (a contiguous slice per CTA) with a fused first-maximum argmax.
//
// Hand-off between CTAs: every value one CTA passes to another (q|k|v, attention
// partials, x_mid, gate/up partials, x_next) travels as a 64-bit word (tag << 32 | f32
// bits) written and read with single-copy-atomic relaxed accesses; the tag names the
// launch and the layer. A reader first polls one word per producer (warp 0), then loads
// its values and re-reads any whose tag is not yet the current one. No release fence or
// counter sits between a producer and its consumers.
//
// Instruction-cache discipline: B200's per-SM instruction cache holds ~60 KB of code
// (measured: straight-line code runs at ~2.7 cycles per instruction up to 61 KB and
// 4-11 beyond 76 KB), and a layer executes every phase once, so the code of one layer
// must stay below that. Every phase is a separate non-inlined function taking only
// scalars (the consumer state is rebuilt in registers; nothing lives in local memory,
// whose L1 is a few KB next to this kernel's shared memory), all GEMVs share two
// streaming loops, and non-critical loops are not unrolled. Every dependent global read
// of a phase is issued as one batch, so a phase costs one L2 round trip, not one per
// value; counters are polled with relaxed loads and one acquire fence.
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
constexpr int kStageBytes = 34560;     // 1920 one-group rows = 240 eight-group rows = 30 embedding rows
constexpr int kStages = 5;
constexpr int kBar = 1;                // named barrier of the consumer warps
constexpr int kKVRows = kStageBytes / (kHeadDim * 4);  // f32 K or V rows of one head per stage (67)
constexpr int kKVRows16 = kStageBytes / (kHeadDim * 2);  // f16 rows (135)
constexpr int kMinAttnChunk = 64;
constexpr int kMaxAttnChunk = 1024;
constexpr int kMaxUnits = 256;         // attention units (kv head x chunk); units <= CTAs
constexpr int kHeadsPerKV = 4;         // query heads per KV head (SmolLM3-3B: 16 / 4)
// shared scratch (floats): XS = inputs of this CTA's GEMV (pre-scaled by 2^64); B = x
// copy / cross-warp reduction / merge weights / epilogue parts; Y = a segment's reduced
// sums; MISC = small reductions and tables; TAB = split-K slots per tile
constexpr int kXsCap = 2048;
constexpr int kXsPer = (kXsCap + kCT - 1) / kCT;  // xs entries per thread (5)
constexpr int kOffB = kXsCap;
constexpr int kBFloats = kCW * 256;
constexpr int kOffY = kOffB + kBFloats;
constexpr int kOffMisc = kOffY + 256;
constexpr int kOffTab = kOffMisc + 64;
constexpr int kMaxTabTiles = 128;
constexpr int kScratchFloats = kOffTab + kMaxTabTiles;
// attention (overlaps XS and B): q [4][128] | scores [4][kMaxAttnChunk] | (m,l) [4][2] | new k,v
constexpr int kAttQ = 0, kAttS = 512, kAttML = kAttS + 4 * kMaxAttnChunk, kAttKV = kAttML + 8;
constexpr int kDnParts = 7;            // down epilogue: partial sums of the slots, [7][64] float4
static_assert(kAttKV + 256 <= kOffY, "attention scratch");
static_assert(kDnParts * 64 * 4 <= kBFloats && kDnParts * 64 <= kCT, "down epilogue");
constexpr float kTwo64 = 18446744073709551616.0f;

enum Mat { QKV = 0, OPR = 1, GU = 2, DOWN = 3 };

struct Layer {
  const uint8_t* w[4];  // QKV, OPR: one-group tiles [group][K/8][8 rows x 16 B | 8 scales];
                        // GU, DOWN: eight-group tiles [tile][K][8 groups x 16 B | 8 scales]
  const float* g_in;
  const float* g_post;
  float* kc;            // K cache, head-major [kv head][max_seq][128]
  float* vc;
  int rope;
  int pad;
};

struct Args {
  const Layer* layers;
  int L;
  int K[4], tiles[4], slots[4];
  int sub0[4], subn[4];       // CTA set [sub0, sub0+subn) that runs each matrix
  int H, nq, nkvw, nh, nkvh, vocab;
  int lm_row_bytes, lm_rows_per_stage;
  long long head_stride;      // elements between KV heads of a layer's cache (max_seq * 128)
  int kv16;                   // 1: the cache holds IEEE binary16 K/V (opt-in), 0: f32
  int kv_pad;
  const uint8_t* lm;          // [vocab][H/2 packed | H/16 scales]
  const float* final_gamma;
  const float* cos_t;
  const float* sin_t;
  int max_pos;                // positions the KV cache (and RoPE table) can hold
  uint64_t* xbuf;             // tagged [L+1][H] residual stream into each layer (x_0 = embedding)
  uint64_t* xmid;             // tagged [L][H] residual after attention
  uint64_t* qkv;              // tagged [nq + 2 nkvw] this step's q|k|v (before RoPE)
  float* logits;              // [vocab]
  uint64_t* gu_part;          // tagged gate/up split-K partials [tiles][slots][256]
  float* dn_part;             // down split-K partials [tiles][slots][256]
  uint64_t* att_o;            // tagged [kMaxUnits][4][128]
  uint64_t* att_ml;           // tagged [kMaxUnits][4][2]
  uint64_t* att_fin;          // tagged [nh][128] merged attention output of the layer
  unsigned* epoch;            // launches so far (the tag base); advanced by the last CTA
  unsigned* cnt;              // down arrival counters [L][tiles] + the final arrival, zero between launches
  int cpl;                    // counters per layer
  int n_cnt;
  float* lm_v;                // [gridDim.x]
  unsigned* lm_i;
  StepState* st;
  unsigned* ring;
  int ring_cap;
  unsigned long long timeout_ns;
  unsigned long long* trace;  // optional phase timestamps, or nullptr
  // tensor parallelism (tp = 1: none): this rank's shard, its lm_head vocab rows
  // [v0, v1), and every rank's receive buffers (own included), written over NVLink
  int tp, rank, hpk;          // hpk: query heads per local KV head
  int v0, v1;
  int want_logits;            // tp > 1: assemble the full logits on every rank (else only
                              // the (value, index) candidates cross NVLink)
  int pad2;
  uint64_t* peer_o[8];        // tagged o_proj partials [L][tp][H]
  uint64_t* peer_d[8];        // tagged down partials [L][tp][H]
  uint64_t* peer_lm[8];       // tagged lm_head bests [tp][2] (value, index)
  float* peer_logits[8];      // full logits [vocab]
};

constexpr size_t smem_bytes() {
  return (size_t)kStages * kStageBytes + (size_t)kScratchFloats * 4 + 2 * kStages * 8 + 64 +
         ((sizeof(Args) + 15) / 16) * 16;
}

// Dynamic shared memory: ring | scratch | full[kStages] | empty[kStages] | flags[16] | Args
extern __shared__ __align__(128) uint8_t g_mk_smem[];
QORA_DEV float* sm_scratch() { return reinterpret_cast<float*>(g_mk_smem + (size_t)kStages * kStageBytes); }
QORA_DEV uint64_t* sm_full() { return reinterpret_cast<uint64_t*>(sm_scratch() + kScratchFloats); }
QORA_DEV uint64_t* sm_empty() { return sm_full() + kStages; }
QORA_DEV volatile int* sm_flags() { return reinterpret_cast<volatile int*>(sm_empty() + kStages); }
QORA_DEV Args* sm_args() { return reinterpret_cast<Args*>(reinterpret_cast<uint8_t*>(sm_empty() + kStages) + 64); }
// flags: [0] abort, [1] last-arriver, [2] pos, [3] chunks issued, [4] producer done,
// [5] token, [6] fine-trace counter, [7] current layer, [8] tag base (epoch * 64)

// Trace layout: per CTA kTracePerCta u64 globaltimer stamps written by consumer thread 0:
// [0] start, [1] after embedding, then per layer L at 2 + 8L + {0: x ready (QKV CTAs),
// 1: QKV done, 2: attention done, 3: attention partials ready (O CTAs), 4: O done,
// 5: x_mid ready, 6: GU done, 7: DOWN done}, then [2+8*kTraceLayers] lm start, [+1] end.
// Then, per CTA, one stamp per layer when the producer has issued that layer's last
// copy; then kTraceFine stamps of layer 1 at finer points (phase steps) per CTA.
constexpr int kTraceLayers = 64;
constexpr int kTracePerCta = 2 + 8 * kTraceLayers + 2;
constexpr int kTraceFine = 64;

// After this long in one bounded wait, the waiter also polls the step's error word, so
// that a timeout recorded by any CTA (or an earlier launch) stops the whole grid without
// every dependent CTA running into its own full timeout.
constexpr unsigned long long kGridCheckNs = 100000ull;
QORA_DEV bool grid_failed(const Args& a) {
  return ptx::ld_relaxed(reinterpret_cast<const unsigned*>(&a.st->error)) != 0u;
}

// ---- counter layout: down arrivals per (layer, output tile), then the final arrival
QORA_DEV int c_dn_arr(const Args& a, int L, int t) { return L * a.cpl + t; }
// attention arrivals per (layer, kv head) after the down counters of the layer
QORA_DEV int c_att(const Args& a, int L, int g) { return L * a.cpl + a.tiles[DOWN] + g; }
QORA_DEV int c_lm(const Args& a) { return a.L * a.cpl; }

// Attention units: (kv head, chunk of `chunk` positions), about one unit per CTA.
// Attention units run on the CTAs from the end of the grid (the q|k|v CTAs) so that the
// o_proj CTAs at the front keep their o_proj weights queued in the ring behind nothing.
QORA_DEV int attn_unit_of(int c, int G) { return G - 1 - c; }

QORA_DEV void attn_plan(int len, int G, int nkvh, int& chunk, int& nch) {
  chunk = (len * nkvh + G - 1) / G;
  chunk = max(kMinAttnChunk, min(kMaxAttnChunk, chunk));
  nch = (len + chunk - 1) / chunk;
}

// ---- split-K geometry (32-bit: the host checks set size x tiles x K < 2^31)
// CTA lc of a g-CTA set owns rows [lc*T/g, (lc+1)*T/g) of the tiles*K flattened rows
QORA_DEV int owner32(unsigned p, unsigned total, unsigned g) { return (int)(((p + 1u) * g - 1u) / total); }

struct Span {
  int lin0, n;
};
// Tile-aligned split-K (down_proj): tile t of T runs on CTAs [al_first(t), al_first(t+1))
// of a g-CTA set (g >= T, so every tile gets floor or ceil of g/T CTAs), and CTA j of
// the n on tile t owns its rows [j*K/n, (j+1)*K/n). No CTA crosses a tile boundary, so
// none streams two partial segments or finishes two tiles.
// (32-bit: the host checks tiles * g and g * K below 2^31)
__host__ __device__ inline int al_first(int t, int g, int T) { return (int)((unsigned)(t * g) / (unsigned)T); }
__host__ __device__ inline int al_tile(int lc, int g, int T) {  // the tile CTA lc works on
  int t = (int)((unsigned)(lc * T) / (unsigned)g);
  while (t + 1 < T && al_first(t + 1, g, T) <= lc) ++t;
  while (t > 0 && al_first(t, g, T) > lc) --t;
  return t;
}

// this CTA's span and first-CTA index of the tile-aligned matrix, computed once per launch
// (al_span) and kept after the slot table: the phases read two words instead of carrying
// the tile search
QORA_DEV int al_slot_words(const Args& a) { return a.tiles[GU] + a.tiles[DOWN]; }
__host__ __device__ __forceinline__ void al_span(const Args& a, int m, int lc, int* out) {  // out: lin0, n, first CTA of the tile
  const int g = a.subn[m], T = a.tiles[m], K = a.K[m], t = al_tile(lc, g, T);
  const int f0 = al_first(t, g, T), n = al_first(t + 1, g, T) - f0, j = lc - f0;
  const int r0 = (int)((unsigned)(j * K) / (unsigned)n), r1 = (int)((unsigned)((j + 1) * K) / (unsigned)n);
  out[0] = t * K + r0;
  out[1] = r1 - r0;
  out[2] = f0;
}

QORA_DEV Span span_of(const Args& a, int m, int c) {
  const int lc = c - a.sub0[m];
  const unsigned g = (unsigned)a.subn[m];
  if (lc < 0 || lc >= (int)g) return Span{0, 0};
  if (m == DOWN) {  // tile-aligned: the calling CTA's own span (every caller passes blockIdx.x)
    const int* w = reinterpret_cast<const int*>(sm_scratch() + kOffTab) + al_slot_words(a);
    return Span{w[0], w[1]};
  }
  const unsigned total = (unsigned)a.tiles[m] * (unsigned)a.K[m];
  const unsigned l0 = (unsigned)lc * total / g, l1 = (unsigned)(lc + 1) * total / g;
  return Span{(int)l0, (int)(l1 - l0)};
}

// the set-local index of the first CTA contributing to tile t (for the aligned matrix:
// the calling CTA's own tile)
QORA_DEV int slot0(const Args& a, int m, int t) {
  if (m == DOWN) return reinterpret_cast<const int*>(sm_scratch() + kOffTab)[al_slot_words(a) + 2];
  const unsigned K = (unsigned)a.K[m], total = (unsigned)a.tiles[m] * K;
  return owner32((unsigned)t * K, total, (unsigned)a.subn[m]);
}

QORA_DEV int nslots(const Args& a, int m, int t) {
  if (m == DOWN) return al_first(t + 1, a.subn[m], a.tiles[m]) - al_first(t, a.subn[m], a.tiles[m]);
  const unsigned K = (unsigned)a.K[m], total = (unsigned)a.tiles[m] * K, g = (unsigned)a.subn[m];
  return owner32((unsigned)(t + 1) * K - 1u, total, g) - owner32((unsigned)t * K, total, g) + 1;
}

QORA_DEV int row_bytes(int m) { return m < GU ? 18 : 144; }

// tile pieces of CTA c's span: f(t, r0, r1)
template <class F>
QORA_DEV void for_each_seg(const Args& a, int m, int c, F&& f) {
  const Span sp = span_of(a, m, c);
  const int K = a.K[m];
  for (int p = sp.lin0, e = sp.lin0 + sp.n; p < e;) {
    const int t = p / K, r0 = p - t * K, pe = min(e, (t + 1) * K);
    f(t, r0, pe - t * K);
    p = pe;
  }
}

QORA_DEV float4 f4add(float4 a, float4 b) {
  return make_float4(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y), __fadd_rn(a.z, b.z), __fadd_rn(a.w, b.w));
}
QORA_DEV float4 ldcg4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// ------------------------------------------------------------------ the producer
// The producer walks exactly this sequence of (source, bytes) copies; the consumers
// consume the same sequence in the same order (see the phases below).
constexpr uint32_t kDead = 0xFFFFFFFFu;  // producer state after an abort: issue nothing

// one bulk copy into the next ring slot (bounded wait for the slot to be released);
// returns the next chunk index, or kDead once the CTA has given up
__device__ __noinline__ uint32_t issue(const uint8_t* src, uint32_t bytes, uint32_t chunk) {
  if (chunk == kDead) return kDead;
  volatile int* flags = sm_flags();
  uint64_t* full = sm_full();
  uint64_t* empty = sm_empty();
  const uint32_t s = chunk % kStages;
  const uint32_t parity = ((chunk / kStages) & 1u) ^ 1u;
  if (!ptx::mbar_try_wait(&empty[s], parity)) {
    const uint64_t t0 = ptx::globaltimer();
    while (!ptx::mbar_try_wait(&empty[s], parity)) {
      if (flags[0] != 0) return kDead;  // consumers gave up: stop issuing
      const uint64_t dt = ptx::globaltimer() - t0;
      if (dt > sm_args()->timeout_ns) {
        flags[0] = 1;
        atomicExch(&sm_args()->st->error, 2);
        return kDead;
      }
      if (dt > kGridCheckNs && grid_failed(*sm_args())) {
        flags[0] = 1;
        return kDead;
      }
    }
  }
  ptx::mbar_arrive_expect_tx(&full[s], bytes);
  ptx::bulk_g2s(g_mk_smem + (size_t)s * kStageBytes, src, bytes, &full[s]);
  flags[3] = (int)(chunk + 1);  // copies issued (drain() waits for the last ones)
  return chunk + 1;
}

__device__ __noinline__ uint32_t produce_gemv(int m, int L, uint32_t chunk) {
  const Args& a = *sm_args();
  const uint8_t* base = a.layers[L].w[m];
  const int rb = row_bytes(m), rps = kStageBytes / rb;
  const long long K = a.K[m];
  for_each_seg(a, m, blockIdx.x, [&](int t, int r0, int r1) {
#pragma unroll 1
    for (int r = r0; r < r1; r += rps)
      chunk = issue(base + ((long long)t * K + r) * rb, (uint32_t)(min(rps, r1 - r) * rb), chunk);
  });
  return chunk;
}

// the cached K rows, then V rows, of this CTA's attention unit (if it has one)
__device__ __noinline__ uint32_t produce_kv(int L, uint32_t chunk) {
  const Args& a = *sm_args();
  const int c = blockIdx.x, pos = sm_flags()[2], len = pos + 1;
  int csz, nch;
  attn_plan(len, gridDim.x, a.nkvh, csz, nch);
  const int u = attn_unit_of(c, gridDim.x);
  if (u >= a.nkvh * nch) return chunk;
  const int g = u % a.nkvh, s0 = (u / a.nkvh) * csz, sc1 = min(min(len, s0 + csz), pos);
  const int esz = a.kv16 ? 2 : 4, rps = a.kv16 ? kKVRows16 : kKVRows;
#pragma unroll 1
  for (int kvs = 0; kvs < 2; ++kvs) {
    const uint8_t* src = reinterpret_cast<const uint8_t*>(kvs ? a.layers[L].vc : a.layers[L].kc) +
                         g * a.head_stride * esz;
#pragma unroll 1
    for (int s = s0; s < sc1; s += rps)
      chunk = issue(src + (long long)s * kHeadDim * esz, (uint32_t)(min(rps, sc1 - s) * kHeadDim * esz), chunk);
  }
  return chunk;
}

__device__ __noinline__ uint32_t produce_lm(uint32_t chunk) {
  const Args& a = *sm_args();
  const int c = blockIdx.x, G = gridDim.x, nv = a.v1 - a.v0;  // this rank's vocab rows
  const int v0 = a.v0 + (int)((unsigned)(c * nv) / (unsigned)G), v1 = a.v0 + (int)((unsigned)((c + 1) * nv) / (unsigned)G);
#pragma unroll 1
  for (int r = v0; r < v1; r += a.lm_rows_per_stage)
    chunk = issue(a.lm + (long long)r * a.lm_row_bytes,
                  (uint32_t)(min(a.lm_rows_per_stage, v1 - r) * a.lm_row_bytes), chunk);
  return chunk;
}

// ------------------------------------------------------------------ consumer state
struct Cons {
  const Args* ap;         // shared-memory copy of the kernel arguments
  uint8_t* ring;
  float* scratch;
  uint64_t* full;
  uint64_t* empty;
  volatile int* flags;
  int c, G, tid, lane, warp, pos;
  uint32_t chunk;
  uint32_t stage_idx;
  bool stage_ok;          // warp-uniform: the current stage landed and the CTA is healthy

  QORA_DEV const Args& a() const { return *ap; }
  QORA_DEV int ns(int m, int t) const {  // split-K slots of tile t (GU, DOWN)
    return reinterpret_cast<const int*>(scratch + kOffTab)[(m == GU ? 0 : ap->tiles[GU]) + t];
  }
  // consistent across the consumer warps between named barriers
  QORA_DEV bool aborted() const { return flags[0] != 0; }
  // uniform within the calling warp at any point
  QORA_DEV bool aborted_w() const { return __shfl_sync(0xffffffffu, flags[0] != 0, 0); }

  QORA_DEV void set_abort(int code) {
    flags[0] = 1;
    atomicExch(&ap->st->error, code);
  }

  QORA_DEV void bar() const { ptx::named_bar(kBar, kCT); }

  QORA_DEV void stamp(int idx) {
    if (ap->trace && tid == 0) ap->trace[(long long)c * kTracePerCta + idx] = ptx::globaltimer();
  }

  QORA_DEV void fstamp() {  // fine-grained trace stamp of layer 1 (thread 0, tracing enabled)
    if (tid == 0 && flags[7] == 1 && ap->trace) {
      const int fine = flags[6];
      if (fine < kTraceFine)
        ap->trace[(long long)G * (kTracePerCta + kTraceLayers) + (long long)c * kTraceFine + fine] =
            ptx::globaltimer();
      flags[6] = fine + 1;
    }
  }

  // next stage of the ring (every consumer warp calls this for every chunk, in order).
  // Once the CTA has aborted, stages are skipped without waiting (see drain()).
  QORA_DEV const uint8_t* acquire_stage() {
    stage_idx = chunk % kStages;
    const uint32_t parity = (chunk / kStages) & 1u;
    if (aborted_w()) {
      stage_ok = false;
      return ring;
    }
    bool timed_out = false;
    if (!ptx::mbar_try_wait(&full[stage_idx], parity)) {
      const uint64_t t0 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&full[stage_idx], parity)) {
        if (ptx::globaltimer() - t0 > ap->timeout_ns) {
          timed_out = true;
          break;
        }
      }
    }
    stage_ok = __all_sync(0xffffffffu, !timed_out);
    if (!stage_ok && lane == 0) set_abort(2);
    return ring + (size_t)stage_idx * kStageBytes;
  }

  QORA_DEV void release_stage() {
    __syncwarp();
    if (lane == 0 && stage_ok) ptx::mbar_arrive(&empty[stage_idx]);
    ++chunk;
  }

  // block sum over consumer threads (fixed order), result in every thread
  QORA_DEV float csum(float v) {
    float* red = scratch + kOffMisc;
    v = warp_sum(v);
    if (lane == 0) red[warp] = v;
    bar();
    float t = 0.0f;
    for (int w = 0; w < kCW; ++w) t += red[w];
    bar();
    return t;
  }

};

// the consumer view of this CTA, rebuilt in registers by every phase (phases take only
// scalars: nothing of the consumer state lives in local memory)
QORA_DEV Cons make_cons(uint32_t chunk) {
  Cons C;
  C.ap = sm_args();
  C.ring = g_mk_smem;
  C.scratch = sm_scratch();
  C.full = sm_full();
  C.empty = sm_empty();
  C.flags = sm_flags();
  C.c = blockIdx.x;
  C.G = gridDim.x;
  C.tid = threadIdx.x;
  C.lane = threadIdx.x & 31;
  C.warp = threadIdx.x >> 5;
  C.pos = C.flags[2];
  C.chunk = chunk;
  C.stage_idx = 0;
  C.stage_ok = false;
  return C;
}

__device__ __noinline__ float rms_inv_from(float sumsq, int H) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)H), 1e-6f)));
}

// ---- tagged hand-off values: (tag << 32) | f32 bits
QORA_DEV uint32_t tag_of(const Cons& C, int L) { return (uint32_t)C.flags[8] + (uint32_t)L + 1u; }
QORA_DEV void st_tagged(uint64_t* p, float v, uint32_t tag) {
  ptx::st_relaxed_b64(p, ((uint64_t)tag << 32) | __float_as_uint(v));
}
QORA_DEV bool tag_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
QORA_DEV float tag_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

// Retry control for a batch of tagged loads that found a stale tag (the producer's
// store had not arrived yet): true = give up (abort set, or the CTA already aborted).
QORA_DEV bool retry_stop(const Cons& C, uint64_t& t0, int it) {
  if (it == 0) {
    t0 = ptx::globaltimer();
    return false;
  }
  if (C.aborted()) return true;
  const uint64_t dt = ptx::globaltimer() - t0;
  if (dt > C.ap->timeout_ns) {
    C.flags[0] = 1;
    atomicExch(&C.ap->st->error, 2);
    return true;
  }
  if (dt > kGridCheckNs && grid_failed(*C.ap)) {  // another CTA gave up: its code stands
    C.flags[0] = 1;
    return true;
  }
  return false;
}

// Warp 0 polls the sentinel words addr(0..n-1) until each carries `tag` (bounded; abort
// on timeout), then every consumer thread passes the barrier.
template <class Addr>
QORA_DEV void await_tags(const Cons& C, int n, uint32_t tag, Addr&& addr) {
  if (C.warp == 0 && !C.aborted_w()) {
    const uint64_t t0 = ptx::globaltimer();
#pragma unroll 1
    for (;;) {
      bool mine = true;
#pragma unroll 1
      for (int i = C.lane; i < n; i += 32) mine &= tag_ok(ptx::ld_relaxed_b64(addr(i)), tag);
      if (__all_sync(0xffffffffu, mine)) break;
      int stop = 0;
      if (C.lane == 0) {
        const uint64_t dt = ptx::globaltimer() - t0;
        stop = C.aborted() ? 1 : dt > C.ap->timeout_ns ? 2 : (dt > kGridCheckNs && grid_failed(*C.ap)) ? 3 : 0;
      }
      stop = __shfl_sync(0xffffffffu, stop, 0);
      if (stop) {
        if (stop >= 2 && C.lane == 0) {
          C.flags[0] = 1;
          if (stop == 2) atomicExch(&C.ap->st->error, 2);
        }
        break;
      }
    }
  }
  C.bar();
}

// tagged x (H <= 2048 values) -> sB (shared), returns this thread's sum of squares
QORA_DEV float load_x(const Cons& C, float* sB, const uint64_t* x, int H, uint32_t tag) {
  constexpr int kPairs = (2048 / 2 + kCT - 1) / kCT;
  uint64_t w[kPairs][2];
  uint64_t t0 = 0;
#pragma unroll 1
  for (int it = 0;; ++it) {
    bool ok = true;
#pragma unroll
    for (int j = 0; j < kPairs; ++j) {
      const int b = C.tid + j * kCT;
      if (b < H / 2) {
        ptx::ld_relaxed_v2_b64(x + 2 * b, w[j][0], w[j][1]);
        ok &= tag_ok(w[j][0], tag) & tag_ok(w[j][1], tag);
      }
    }
    if (ok || retry_stop(C, t0, it)) break;
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kPairs; ++j) {
    const int b = C.tid + j * kCT;
    if (b < H / 2) {
      const float v0 = tag_val(w[j][0]), v1 = tag_val(w[j][1]);
      sB[2 * b] = v0;
      sB[2 * b + 1] = v1;
      ss = __fmaf_rn(v0, v0, ss);
      ss = __fmaf_rn(v1, v1, ss);
    }
  }
  return ss;
}

// one tagged value, re-read until it carries `tag` (bounded)
QORA_DEV float ld_checked(const Cons& C, const uint64_t* p, uint32_t tag) {
  uint64_t w, t0 = 0;
#pragma unroll 1
  for (int it = 0;; ++it) {
    w = ptx::ld_relaxed_b64(p);
    if (tag_ok(w, tag) || retry_stop(C, t0, it)) break;
  }
  return tag_val(w);
}

// Rows of this thread's xs entries i = tid + j*kCT of a span: (lin0 + i) mod K, stepped
// without a division when kCT < K (every matrix of the full-size model).
QORA_DEV int row_next(int r, int K) {
  r += kCT;
  if (r >= K) r -= K;
  return r >= K ? r % K : r;
}

QORA_DEV void prefetch_gains(const Cons& C, const float* g, Span sp, int K, float (&gam)[kXsPer]) {
  int r = (sp.lin0 + C.tid) % K;
#pragma unroll
  for (int j = 0; j < kXsPer; ++j, r = row_next(r, K)) gam[j] = (C.tid + j * kCT < sp.n) ? __ldg(g + r) : 0.0f;
}

// xs[i] = x[row] * inv * gamma[row] * 2^64 for the span's rows (gains prefetched)
QORA_DEV void fill_norm_inputs(const Cons& C, const float* sB, float inv, const float (&gam)[kXsPer], Span sp,
                               int K) {
  float* xs = C.scratch;
  int r = (sp.lin0 + C.tid) % K;
#pragma unroll
  for (int j = 0; j < kXsPer; ++j, r = row_next(r, K)) {
    const int i = C.tid + j * kCT;
    if (i < sp.n) xs[i] = __fmul_rn(__fmul_rn(sB[r], inv), gam[j]) * kTwo64;
  }
}

// Tensor parallelism: this rank's partial value v of column `col` goes to every rank's
// receive buffer bufs[p][(L*tp + rank)*H + col]; the sum over ranks (rank order, the same
// on every rank) comes back once all tp partials of the column have arrived (bounded).
QORA_DEV void tp_push(const Cons& C, uint64_t* const* bufs, int L, int col, float v, uint32_t tag) {
  const Args& a = C.a();
  const long long o = ((long long)L * a.tp + a.rank) * a.H + col;
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  for (int p = 0; p < a.tp; ++p) ptx::st_relaxed_sys_b64(bufs[p] + o, w);
}
QORA_DEV float tp_sum(const Cons& C, const uint64_t* own, int L, int col, uint32_t tag) {
  const Args& a = C.a();
  const uint64_t* q = own + (long long)L * a.tp * a.H + col;
  float s = 0.0f;
  uint64_t t0 = 0;
#pragma unroll 1
  for (int it = 0;; ++it) {
    bool ok = true;
    s = 0.0f;
#pragma unroll 1
    for (int p = 0; p < a.tp; ++p) {
      const uint64_t w = ptx::ld_relaxed_sys_b64(q + (long long)p * a.H);
      ok &= tag_ok(w, tag);
      s = __fadd_rn(s, tag_val(w));
    }
    if (ok || retry_stop(C, t0, it)) break;
  }
  return s;
}

// ------------------------------------------------------------------ phases
__device__ __noinline__ void seg_store(int m, int L, int t, int slot);
__device__ __noinline__ void gemv_finish(int m, int L, int t);

// Stream this CTA's segments of matrix m (TG groups per tile) through the ring and
// reduce each segment's 32*TG sums into Y, then store and publish them. xs holds the (pre-scaled)
// inputs of all segments back to back. Lane (sub, gi) takes group gi of rows sub and
// sub + 15*(32/TG) of each warp's share of a stage.
template <int TG>
__device__ __noinline__ uint32_t gemv_stream(int m, int L, uint32_t chunk) {
  constexpr int W = 32 / TG;        // rows per warp pass
  constexpr int RPS = kStageBytes / (18 * TG);  // rows per stage
  constexpr int NP = RPS / (kCW * W);            // rows per lane per stage
  static_assert(TG == 1 || TG == 8, "tile width");
  static_assert(NP * kCW * W == RPS, "stage rows");
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const float* xs = C.scratch;
  float* red = C.scratch + kOffB;
  float* y = C.scratch + kOffY;
  const int gi = C.lane % TG, sub = C.lane / TG;
  const Span sp = span_of(a, m, C.c);
  const int K = a.K[m], lc = C.c - a.sub0[m];
  int off = 0;
#pragma unroll 1
  for (int p = sp.lin0, e = sp.lin0 + sp.n; p < e;) {
    const int t = p / K, r0 = p - t * K, r1 = min(e, (t + 1) * K) - t * K;
    const int slot = lc - slot0(a, m, t);
    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
    float cs = 0.0f;
#pragma unroll 1
    for (int cr = r0; cr < r1; cr += RPS) {
      const uint8_t* stg = C.acquire_stage();
      const int R = min(RPS, r1 - cr);
      if (C.stage_ok) {
        // NP rows per lane, all loads issued before the math; 144-byte blocks: TG == 8
        // one row of 8 groups, TG == 1 eight rows of one group
        const float* xr = xs + off + (cr - r0);
        uint4 w[NP];
        float cf[NP];
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          const int i = C.warp * W + sub + k * kCW * W;
          const bool ok = i < R;
          const int j = ok ? i : 0;
          const uint8_t* blk = stg + (TG == 8 ? j : j >> 3) * 144;
          const int q = TG == 8 ? gi : (j & 7);
          w[k] = *reinterpret_cast<const uint4*>(blk + q * 16);
          const uint16_t sv = *reinterpret_cast<const uint16_t*>(blk + 128 + q * 2);
          cf[k] = ok ? __half2float(__ushort_as_half(sv)) * xr[j] : 0.0f;
        }
        // passes whose rows all lie past the stage's end are skipped (warp-uniform)
        const int base = C.warp * W;
#pragma unroll
        for (int k = 0; k < NP; ++k) {
          if (base + k * kCW * W < R) {
            cs += cf[k];
            q4_fma_chunk(w[k], cf[k], acc);
          }
        }
      }
      C.release_stage();
    }
    off += r1 - r0;

    // this lane's 32 outputs, then a transposing reduction over the W lanes of each
    // group (masks 16 .. TG): afterwards lane (sub, gi) holds outputs sub*TG + [0, TG)
    const float bias = cs * 4.3368086899420177e-19f;  // 8 * 2^-64
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[2 * i] = __fmaf_rn(acc[i].x, q4_scale_of_pos((2 * i) & 7), -bias);
      v[2 * i + 1] = __fmaf_rn(acc[i].y, q4_scale_of_pos((2 * i + 1) & 7), -bias);
    }
#pragma unroll
    for (int msk = 16; msk >= TG; msk >>= 1) {
      const bool hi = (C.lane & msk) != 0;
#pragma unroll
      for (int e2 = 0; e2 < msk; ++e2) {
        const float send = hi ? v[e2] : v[msk + e2];
        const float keep = hi ? v[msk + e2] : v[e2];
        v[e2] = keep + __shfl_xor_sync(0xffffffffu, send, msk);
      }
    }
    float* dst = red + C.warp * (32 * TG) + gi * 32 + sub * TG;
#pragma unroll
    for (int e2 = 0; e2 < TG; ++e2) dst[e2] = v[e2];
    C.bar();
    if (C.tid < 32 * TG) {
      float s = 0.0f;
#pragma unroll
      for (int w = 0; w < kCW; ++w) s += red[w * 32 * TG + C.tid];
      y[C.tid] = s;
    }
    C.bar();
    C.fstamp();
    seg_store(m, L, t, slot);
    gemv_finish(m, L, t);
    C.fstamp();
    p += r1 - r0;
  }
  return C.chunk;
}

// A finished segment's sums (Y): q|k|v and o_proj results are final (one group per
// CTA) and go out tagged; gate/up partials go out tagged; down partials are plain
// floats, published by the arrival count in gemv_finish.
__device__ __noinline__ void seg_store(int m, int L, int t, int slot) {
  Cons C = make_cons(0);
  const Args& a = C.a();
  const float* y = C.scratch + kOffY;
  const uint32_t tag = tag_of(C, L);
  if (m == QKV) {
    if (C.tid < 32) st_tagged(a.qkv + t * 32 + C.tid, y[C.tid], tag);
  } else if (m == OPR) {
    if (C.tid < 32) {
      const long long col = (long long)L * a.H + t * 32 + C.tid;
      float o = y[C.tid];
      if (a.tp > 1) {  // row-split o_proj: sum the ranks' partials of this column
        tp_push(C, a.peer_o, L, t * 32 + C.tid, o, tag);
        o = tp_sum(C, a.peer_o[a.rank], L, t * 32 + C.tid, tag);
      }
      st_tagged(a.xmid + col, __fadd_rn(ld_checked(C, a.xbuf + col, tag), o), tag);
    }
  } else if (C.tid < 256) {
    const long long o = ((long long)t * a.slots[m] + slot) * 256 + C.tid;
    if (m == GU) st_tagged(a.gu_part + o, y[C.tid], tag);
    else __stcg(a.dn_part + o, y[C.tid]);
  }
}

// Down: count this segment's arrival at tile t; the last arriver writes the tile's next
// residual x_{L+1} = x_mid + (down partials summed over the slots).
__device__ __noinline__ void gemv_finish(int m, int L, int t) {
  if (m != DOWN) return;
  Cons C = make_cons(0);
  const Args& a = C.a();
  const int H = a.H;
  C.bar();
  if (C.tid == 0) {
    const unsigned prev = ptx::atom_add_acqrel(a.cnt + c_dn_arr(a, L, t), 1u);
    C.flags[1] = (prev == (unsigned)(C.ns(DOWN, t) - 1));
  }
  C.bar();
  if (C.flags[1]) {
    const uint32_t tag = tag_of(C, L);
    float4* parts = reinterpret_cast<float4*>(C.scratch + kOffB);  // [kDnParts][64]
    const int b = C.tid & 63, p = C.tid >> 6;
    const long long col = (long long)L * H + t * 256 + 4 * b;
    uint64_t xw[4] = {0, 0, 0, 0};
    if (C.tid < 64) {
      uint64_t t0 = 0;
#pragma unroll 1
      for (int it = 0;; ++it) {
        ptx::ld_relaxed_v2_b64(a.xmid + col, xw[0], xw[1]);
        ptx::ld_relaxed_v2_b64(a.xmid + col + 2, xw[2], xw[3]);
        const bool ok = tag_ok(xw[0], tag) & tag_ok(xw[1], tag) & tag_ok(xw[2], tag) & tag_ok(xw[3], tag);
        if (ok || retry_stop(C, t0, it)) break;
      }
    }
    if (p < kDnParts) {
      const int ns = C.ns(DOWN, t);
      const float* pd = a.dn_part + (long long)t * a.slots[DOWN] * 256 + 4 * b;
      float4 s = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 1
      for (int k0 = p; k0 < ns; k0 += 4 * kDnParts) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = (k0 + j * kDnParts < ns) ? ldcg4(pd + (k0 + j * kDnParts) * 256) : s;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (k0 + j * kDnParts < ns) s = f4add(s, v[j]);
      }
      parts[p * 64 + b] = s;
    }
    C.bar();
    if (C.tid < 64) {
      float4 d = parts[b];
#pragma unroll 1
      for (int q = 1; q < kDnParts; ++q) d = f4add(d, parts[q * 64 + b]);
      float dv[4] = {d.x, d.y, d.z, d.w};
      if (a.tp > 1) {  // row-split down: sum the ranks' partials of these columns
        const int c0 = t * 256 + 4 * b;
#pragma unroll
        for (int j = 0; j < 4; ++j) tp_push(C, a.peer_d, L, c0 + j, dv[j], tag);
#pragma unroll
        for (int j = 0; j < 4; ++j) dv[j] = tp_sum(C, a.peer_d[a.rank], L, c0 + j, tag);
      }
      const uint32_t tn = tag + 1u;  // x_{L+1} carries layer L+1's tag
#pragma unroll
      for (int j = 0; j < 4; ++j)
        st_tagged(a.xbuf + col + H + j, __fadd_rn(tag_val(xw[j]), dv[j]), tn);
    }
  }
  C.bar();
}

// QKV: RMSNorm(x) . W for this CTA's 32-column group, all rows
__device__ __noinline__ uint32_t qkv_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const Span sp = span_of(a, QKV, C.c);
  if (sp.n == 0) return chunk;
  const int H = a.H;
  float* sB = C.scratch + kOffB;
  float gam[kXsPer];
  prefetch_gains(C, a.layers[L].g_in, sp, H, gam);
  float ss = 0.0f;
  if (L > 0) {
    const uint32_t tag = tag_of(C, L);
    const uint64_t* x = a.xbuf + (long long)L * H;
    await_tags(C, a.tiles[DOWN], tag, [&](int i) { return x + i * 256; });  // one word per down tile
    ss = load_x(C, sB, x, H, tag);
  } else {
#pragma unroll 1
    for (int i = C.tid; i < H; i += kCT) ss = __fmaf_rn(sB[i], sB[i], ss);
  }
  C.stamp(2 + 8 * min(L, kTraceLayers - 1) + 0);
  const float inv = rms_inv_from(C.csum(ss), H);
  fill_norm_inputs(C, sB, inv, gam, sp, H);
  C.bar();
  C.fstamp();
  return gemv_stream<1>(QKV, L, C.chunk);
}

// 4 query heads . one K row (8 lanes per row, 16 dims each); lane li == 0 writes
QORA_DEV void kscore(const float* sq, const float* krow, float* sc, int idx, bool valid, int li) {
  float d[kHeadsPerKV] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (valid) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float4 k4 = reinterpret_cast<const float4*>(krow + li * 16)[j];
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h) {
        const float4 q4 = reinterpret_cast<const float4*>(sq + h * kHeadDim + li * 16)[j];
        d[h] = __fmaf_rn(q4.x, k4.x, d[h]);
        d[h] = __fmaf_rn(q4.y, k4.y, d[h]);
        d[h] = __fmaf_rn(q4.z, k4.z, d[h]);
        d[h] = __fmaf_rn(q4.w, k4.w, d[h]);
      }
    }
  }
  const float scale = 0.08838834764831845f;  // 1/sqrt(128): the f32 quotient of 1 and f32 sqrt(128)
#pragma unroll
  for (int h = 0; h < kHeadsPerKV; ++h) {
    float v = d[h];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    if (valid && li == 0) sc[h * kMaxAttnChunk + idx] = __fmul_rn(v, scale);
  }
}

// Attention merge, run by the last of the nch units of KV head g to arrive (acq_rel
// arrival count): per query head, M = max_ch m, w_ch = exp(m_ch - M), l = sum_ch l_ch w_ch,
// out = (sum_ch o_ch w_ch, chunk order) * (1 / l), published tagged for o_proj.
__device__ __noinline__ void attn_merge(int L, int g, int nch) {
  Cons C = make_cons(0);
  const Args& a = C.a();
  const int hpk = a.hpk, nkvh = a.nkvh;
  C.bar();  // every partial of this unit is stored
  if (C.tid == 0) {
    const unsigned prev = ptx::atom_add_acqrel(a.cnt + c_att(a, L, g), 1u);
    C.flags[1] = (prev == (unsigned)(nch - 1));
  }
  C.bar();
  if (!C.flags[1] || C.aborted()) return;
  const uint32_t tag = tag_of(C, L);
  float* mw = C.scratch + kOffB;            // [hpk][nch] chunk weights
  float* invl = mw + kHeadsPerKV * nch;     // [hpk]
  const long long ustride = (long long)nkvh * kHeadsPerKV * 2;         // (m, l): next chunk, same head
  const long long ostride = (long long)nkvh * kHeadsPerKV * kHeadDim;  // o: next chunk, same head
  if (C.warp < hpk) {  // one warp per query head, lane = chunk
    const int h = C.warp;
    const uint64_t* ml = a.att_ml + ((long long)g * kHeadsPerKV + h) * 2;
    float mx = -INFINITY;
#pragma unroll 1
    for (int ch = C.lane; ch < nch; ch += 32) mx = fmaxf(mx, ld_checked(C, ml + ch * ustride, tag));
    mx = warp_max(mx);
    float l = 0.0f;
    if (C.lane < nch) {
      const float w = expf(ld_checked(C, ml + C.lane * ustride, tag) - mx);
      mw[h * nch + C.lane] = w;
      l = __fmul_rn(ld_checked(C, ml + C.lane * ustride + 1, tag), w);
    }
#pragma unroll 1
    for (int ch = C.lane + 32; ch < nch; ch += 32) {
      const float w = expf(ld_checked(C, ml + ch * ustride, tag) - mx);
      mw[h * nch + ch] = w;
      l = __fmaf_rn(ld_checked(C, ml + ch * ustride + 1, tag), w, l);
    }
    l = warp_sum(l);
    if (C.lane == 0) invl[h] = __fdiv_rn(1.0f, l);
  }
  C.bar();
  const uint64_t* o0 = a.att_o + (long long)g * kHeadsPerKV * kHeadDim;
#pragma unroll 1
  for (int r = C.tid; r < hpk * kHeadDim; r += kCT) {
    const int h = r / kHeadDim;
    float acc = 0.0f;
#pragma unroll 1
    for (int c0 = 0; c0 < nch; c0 += 4) {  // four chunks' values in flight
      uint64_t v[4], t0 = 0;
#pragma unroll 1
      for (int it = 0;; ++it) {
        bool ok = true;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const bool in = c0 + k < nch;
          v[k] = in ? ptx::ld_relaxed_b64(o0 + (c0 + k) * ostride + r) : 0ull;
          ok &= !in || tag_ok(v[k], tag);
        }
        if (ok || retry_stop(C, t0, it)) break;
      }
#pragma unroll
      for (int k = 0; k < 4; ++k)
        if (c0 + k < nch) acc = __fmaf_rn(tag_val(v[k]), mw[h * nch + c0 + k], acc);
    }
    st_tagged(a.att_fin + (long long)(g * hpk) * kHeadDim + r, __fmul_rn(acc, invl[h]), tag);
  }
}

// kscore for a binary16 K row (opt-in f16 cache): lane li takes dims [8li, 8li+8) and
// [64+8li, 64+8li+8) as two 16-byte loads (conflict-free across the 8 lanes of a row)
QORA_DEV void kscore16(const float* sq, const __half* krow, float* sc, int idx, bool valid, int li) {
  float d[kHeadsPerKV] = {0.0f, 0.0f, 0.0f, 0.0f};
  if (valid) {
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const uint4 raw = *reinterpret_cast<const uint4*>(krow + j * kHalfDim + li * 8);
      const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
      float kf[8];
#pragma unroll
      for (int t = 0; t < 4; ++t) {
        const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[t]));
        kf[2 * t] = f.x;
        kf[2 * t + 1] = f.y;
      }
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h) {
        const float4 qa = *reinterpret_cast<const float4*>(sq + h * kHeadDim + j * kHalfDim + li * 8);
        const float4 qb = *reinterpret_cast<const float4*>(sq + h * kHeadDim + j * kHalfDim + li * 8 + 4);
        d[h] = __fmaf_rn(qa.x, kf[0], d[h]);
        d[h] = __fmaf_rn(qa.y, kf[1], d[h]);
        d[h] = __fmaf_rn(qa.z, kf[2], d[h]);
        d[h] = __fmaf_rn(qa.w, kf[3], d[h]);
        d[h] = __fmaf_rn(qb.x, kf[4], d[h]);
        d[h] = __fmaf_rn(qb.y, kf[5], d[h]);
        d[h] = __fmaf_rn(qb.z, kf[6], d[h]);
        d[h] = __fmaf_rn(qb.w, kf[7], d[h]);
      }
    }
  }
  const float scale = 0.08838834764831845f;
#pragma unroll
  for (int h = 0; h < kHeadsPerKV; ++h) {
    float v = d[h];
    v += __shfl_xor_sync(0xffffffffu, v, 1);
    v += __shfl_xor_sync(0xffffffffu, v, 2);
    v += __shfl_xor_sync(0xffffffffu, v, 4);
    if (valid && li == 0) sc[h * kMaxAttnChunk + idx] = __fmul_rn(v, scale);
  }
}

// one cached V element as f32
QORA_DEV float kv_elem(const float* p) { return *p; }
QORA_DEV float kv_elem(const __half* p) { return __half2float(*p); }

// ATTN: unit u = c = (kv head g = u % nkvh, chunk u / nkvh) for the 4 query heads of g
// (src/gemv.rs:914-989, softmax_raw :782-793; RoPE src/gemv.rs:757-778). KV is float
// (the reference's f32 cache) or __half (the opt-in binary16 cache: the new k and v are
// rounded to nearest-even as they enter the cache, and the new position's score and P.V
// use the rounded values, exactly as if they were read back from it).
template <class KV>
__device__ __noinline__ uint32_t attention_phase_t(int L, uint32_t chunk) {
  constexpr bool kF16 = sizeof(KV) == 2;
  constexpr int kRows = kF16 ? kKVRows16 : kKVRows;
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const int pos = C.pos, len = pos + 1, tid = C.tid, lane = C.lane, warp = C.warp;
  int csz, nch;
  attn_plan(len, C.G, a.nkvh, csz, nch);
  const int u = attn_unit_of(C.c, C.G);
  if (u >= a.nkvh * nch) return chunk;
  const int g = u % a.nkvh;
  const int s0 = (u / a.nkvh) * csz, s1 = min(len, s0 + csz), sc1 = min(s1, pos), n = s1 - s0;
  const bool has_pos = pos < s1;
  const Layer& ly = a.layers[L];
  KV* kc = reinterpret_cast<KV*>(ly.kc) + g * a.head_stride;
  KV* vc = reinterpret_cast<KV*>(ly.vc) + g * a.head_stride;
  float* sq = C.scratch + kAttQ;
  float* sc = C.scratch + kAttS;
  float* sml = C.scratch + kAttML;
  float* skv = C.scratch + kAttKV;
  // RoPE pairs (d, d+64): threads 0..64*hpk-1 the query heads of g, 256..319 k;
  // 320..447 copy v
  const int hpk = a.hpk;
  const bool rope = ly.rope != 0;
  float cs = 1.0f, sn = 0.0f;
  if (rope && tid < 320) {  // the tables do not depend on this step's activations
    cs = __ldg(a.cos_t + (long long)pos * kHalfDim + (tid & 63));
    sn = __ldg(a.sin_t + (long long)pos * kHalfDim + (tid & 63));
  }
  // one sentinel per producing group: the 4*hpk q groups of g's query heads, then the 4
  // k and 4 v groups of head g
  const uint32_t tag = tag_of(C, L);
  const int nqg = 4 * hpk;
  const int gq0 = g * nqg, gk0 = a.nq / 32 + g * 4, gv0 = (a.nq + a.nkvw) / 32 + g * 4;
  await_tags(C, nqg + 8, tag,
             [&](int i) { return a.qkv + 32 * (i < nqg ? gq0 + i : i < nqg + 4 ? gk0 + i - nqg : gv0 + i - nqg - 4); });
  C.fstamp();
  if (tid < 320 && (tid < 64 * hpk || (tid >= 256 && has_pos))) {
    const bool isk = tid >= 256;
    const int hh = (tid >> 6) & 3, d = tid & 63;
    const uint64_t* src = isk ? a.qkv + a.nq + g * kHeadDim : a.qkv + (g * hpk + hh) * kHeadDim;
    uint64_t w1, w2, t0 = 0;
#pragma unroll 1
    for (int it = 0;; ++it) {
      w1 = ptx::ld_relaxed_b64(src + d);
      w2 = ptx::ld_relaxed_b64(src + d + kHalfDim);
      if ((tag_ok(w1, tag) & tag_ok(w2, tag)) || retry_stop(C, t0, it)) break;
    }
    const float x1 = tag_val(w1), x2 = tag_val(w2);
    float y1 = x1, y2 = x2;
    if (rope) {
      y1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      y2 = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
    }
    if (!isk) {
      sq[hh * kHeadDim + d] = y1;
      sq[hh * kHeadDim + d + kHalfDim] = y2;
    } else if constexpr (kF16) {
      const __half h1 = __float2half_rn(y1), h2 = __float2half_rn(y2);
      skv[d] = __half2float(h1);
      skv[d + kHalfDim] = __half2float(h2);
      kc[(long long)pos * kHeadDim + d] = h1;
      kc[(long long)pos * kHeadDim + d + kHalfDim] = h2;
    } else {
      skv[d] = y1;
      skv[d + kHalfDim] = y2;
      kc[(long long)pos * kHeadDim + d] = y1;
      kc[(long long)pos * kHeadDim + d + kHalfDim] = y2;
    }
  } else if (tid >= 320 && tid < 448 && has_pos) {
    const int d = tid - 320;
    const float v = ld_checked(C, a.qkv + a.nq + a.nkvw + g * kHeadDim + d, tag);
    if constexpr (kF16) {
      const __half hv = __float2half_rn(v);
      skv[kHeadDim + d] = __half2float(hv);
      vc[(long long)pos * kHeadDim + d] = hv;
    } else {
      skv[kHeadDim + d] = v;
      vc[(long long)pos * kHeadDim + d] = v;
    }
  }
  C.bar();
  C.fstamp();
  // scores: 4 rows per warp pass (8 lanes each), 60 rows per CTA pass
  const int li = lane & 7, ri = warp * 4 + (lane >> 3);
#pragma unroll 1
  for (int s = s0; s < sc1; s += kRows) {
    const uint8_t* stg = C.acquire_stage();
    const int nr = min(kRows, sc1 - s);
    if (C.stage_ok) {
#pragma unroll 1
      for (int rb = 0; rb < nr; rb += kCW * 4) {
        const int i = rb + ri;
        const KV* krow = reinterpret_cast<const KV*>(stg) + min(i, nr - 1) * kHeadDim;
        if constexpr (kF16) kscore16(sq, krow, sc, s - s0 + i, i < nr, li);
        else kscore(sq, krow, sc, s - s0 + i, i < nr, li);
      }
    }
    C.release_stage();
  }
  if (has_pos && warp == 0 && !C.aborted_w()) kscore(sq, skv, sc, pos - s0, (lane >> 3) == 0, li);
  C.bar();
  C.fstamp();
  // chunk softmax numerators, one warp per query head
  if (warp < hpk && !C.aborted_w()) {
    float* row = sc + warp * kMaxAttnChunk;
    float mx = -INFINITY;
#pragma unroll 1
    for (int i = lane; i < n; i += 32) mx = fmaxf(mx, row[i]);
    mx = warp_max(mx);
    float l = 0.0f;
#pragma unroll 1
    for (int i = lane; i < n; i += 32) {
      const float e = expf(row[i] - mx);
      row[i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (lane == 0) {
      sml[warp * 2] = mx;
      sml[warp * 2 + 1] = l;
    }
  }
  C.bar();
  C.fstamp();
  // P.V: three groups of 128 threads (warps 0-3, 4-7, 8-11) take rows grp, grp + 3, ...
  // of each stage, four rows per step with their loads issued together; thread d of a
  // group accumulates dim d of the 4 heads; the groups' sums are added in group order
  const int grp = tid >> 7, dd = tid & (kHeadDim - 1);
  float o[kHeadsPerKV] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll 1
  for (int s = s0; s < sc1; s += kRows) {
    const uint8_t* stg = C.acquire_stage();
    const int nr = min(kRows, sc1 - s);
    if (C.stage_ok && grp < 3) {
      const KV* vr = reinterpret_cast<const KV*>(stg) + dd;
      const float* pr = sc + (s - s0);
      int i = grp;
#pragma unroll 1
      for (; i + 9 < nr; i += 12) {
        float v[4];
#pragma unroll
        for (int r = 0; r < 4; ++r) v[r] = kv_elem(vr + (i + 3 * r) * kHeadDim);
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int h = 0; h < kHeadsPerKV; ++h) o[h] = __fmaf_rn(pr[h * kMaxAttnChunk + i + 3 * r], v[r], o[h]);
      }
#pragma unroll 1
      for (; i < nr; i += 3) {
        const float v = kv_elem(vr + i * kHeadDim);
#pragma unroll
        for (int h = 0; h < kHeadsPerKV; ++h) o[h] = __fmaf_rn(pr[h * kMaxAttnChunk + i], v, o[h]);
      }
    }
    C.release_stage();
  }
  float ppos[kHeadsPerKV] = {0.0f, 0.0f, 0.0f, 0.0f};  // the new position's probabilities
  if (has_pos && tid < kHeadDim) {
#pragma unroll
    for (int h = 0; h < kHeadsPerKV; ++h) ppos[h] = sc[h * kMaxAttnChunk + pos - s0];
  }
  C.bar();  // every read of the probabilities is done: groups 1 and 2 park their sums there
  if ((grp == 1 || grp == 2) && !C.aborted()) {
#pragma unroll
    for (int h = 0; h < kHeadsPerKV; ++h) sc[(grp - 1) * kHeadsPerKV * kHeadDim + h * kHeadDim + dd] = o[h];
  }
  C.bar();
  if (tid < kHeadDim && !C.aborted()) {
#pragma unroll
    for (int h = 0; h < kHeadsPerKV; ++h)
      o[h] = __fadd_rn(__fadd_rn(o[h], sc[h * kHeadDim + tid]), sc[kHeadsPerKV * kHeadDim + h * kHeadDim + tid]);
    if (has_pos) {
      const float v = skv[kHeadDim + tid];
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h) o[h] = __fmaf_rn(ppos[h], v, o[h]);
    }
    if (nch == 1) {  // the whole context: publish o / l (exp(m - max) = 1 for the one chunk)
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h)
        if (h < hpk)
          st_tagged(a.att_fin + (long long)(g * hpk + h) * kHeadDim + tid,
                    __fmul_rn(o[h], __fdiv_rn(1.0f, sml[h * 2 + 1])), tag);
    } else {
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h)
        if (h < hpk) st_tagged(a.att_o + ((long long)u * kHeadsPerKV + h) * kHeadDim + tid, o[h], tag);
      if (tid < 2 * hpk) st_tagged(a.att_ml + (long long)u * 2 * kHeadsPerKV + tid, sml[tid], tag);
    }
  }
  if (nch > 1) attn_merge(L, g, nch);
  return C.chunk;
}

__device__ __noinline__ uint32_t attention_phase(int L, uint32_t chunk) {
  return sm_args()->kv16 ? attention_phase_t<__half>(L, chunk) : attention_phase_t<float>(L, chunk);
}

// O: the merged attention output of every head (tagged, one sentinel word per head), GEMV
// over all rows for this CTA's 32 columns, x_mid = x + o
__device__ __noinline__ uint32_t o_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const Span sp = span_of(a, OPR, C.c);
  if (sp.n == 0) return chunk;
  const int K = a.K[OPR];
  const uint32_t tag = tag_of(C, L);
  await_tags(C, a.nh, tag, [&](int i) { return a.att_fin + (long long)i * kHeadDim; });
  C.stamp(2 + 8 * min(L, kTraceLayers - 1) + 3);
  C.fstamp();
  // xs = att * 2^64: each thread scales the pairs it loaded itself
  float* xs = C.scratch;
  load_x(C, xs, a.att_fin, K, tag);
  constexpr int kPairs = (2048 / 2 + kCT - 1) / kCT;
#pragma unroll
  for (int j = 0; j < kPairs; ++j) {
    const int b = C.tid + j * kCT;
    if (b < K / 2) {
      xs[2 * b] *= kTwo64;
      xs[2 * b + 1] *= kTwo64;
    }
  }
  C.bar();
  C.fstamp();
  return gemv_stream<1>(OPR, L, C.chunk);
}

// GU (all): RMSNorm(x_mid) . [gate|up] -> split-K partials per tile
__device__ __noinline__ uint32_t gu_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const Span sp = span_of(a, GU, C.c);
  const int H = a.H;
  float* sB = C.scratch + kOffB;
  float gam[kXsPer];
  prefetch_gains(C, a.layers[L].g_post, sp, a.K[GU], gam);
  const uint32_t tag = tag_of(C, L);
  const uint64_t* xm = a.xmid + (long long)L * H;
  await_tags(C, H / 32, tag, [&](int i) { return xm + i * 32; });  // one word per o_proj group
  C.stamp(2 + 8 * min(L, kTraceLayers - 1) + 5);
  const float ss = load_x(C, sB, xm, H, tag);
  const float inv = rms_inv_from(C.csum(ss), H);
  fill_norm_inputs(C, sB, inv, gam, sp, a.K[GU]);
  C.bar();
  C.fstamp();
  return gemv_stream<8>(GU, L, C.chunk);
}

// DOWN (all): SwiGLU of the rows it needs from the gate/up partials (src/gemv.rs:412-502),
// split-K GEMV
__device__ __noinline__ uint32_t down_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const Span sp = span_of(a, DOWN, C.c);
  const int K = a.K[DOWN];
  constexpr int kHalfTile = 128;  // gate (then up) outputs per gate/up tile
  // gate/up tiles of this CTA's rows: one range per segment (the host checks <= 2)
  int tr[4] = {0, -1, 0, -1};
  {
    int k = 0;
    for_each_seg(a, DOWN, C.c, [&](int, int r0, int r1) {
      if (k < 2) {
        tr[2 * k] = r0 / kHalfTile;
        tr[2 * k + 1] = (r1 - 1) / kHalfTile;
      }
      ++k;
    });
  }
  // one sentinel per (gate/up tile, split-K slot) this CTA reads
  const uint32_t tag = tag_of(C, L);
  {
    const int S = a.slots[GU], n0 = tr[1] - tr[0] + 1, n1 = tr[3] - tr[2] + 1;
    await_tags(C, (n0 + n1) * S, tag, [&](int i) {
      const int k = i / S, t = k < n0 ? tr[0] + k : tr[2] + (k - n0);
      return a.gu_part + ((long long)t * S + min(i % S, C.ns(GU, t) - 1)) * 256;
    });
  }
  // rows i = tid, tid + kCT: both rows' gate and up partials (4 slots each) in flight
  {
    float* xs = C.scratch;
    int r = (sp.lin0 + C.tid) % K;
#pragma unroll 1
    for (int i = C.tid; i < sp.n; i += 2 * kCT) {
      const int r2 = row_next(r, K);
      const bool two = i + kCT < sp.n;
      const int t1 = r / kHalfTile, t2 = r2 / kHalfTile;
      const int n1 = C.ns(GU, t1), n2 = two ? C.ns(GU, t2) : 0;
      const uint64_t* p1 = a.gu_part + (long long)t1 * a.slots[GU] * 256 + r % kHalfTile;
      const uint64_t* p2 = a.gu_part + (long long)t2 * a.slots[GU] * 256 + r2 % kHalfTile;
      float g1 = 0.0f, u1 = 0.0f, g2 = 0.0f, u2 = 0.0f;
#pragma unroll 1
      for (int k0 = 0; k0 < max(n1, n2); k0 += 4) {
        uint64_t v[4][4], t0 = 0;
#pragma unroll 1
        for (int it = 0;; ++it) {
          bool ok = true;
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const bool ok1 = k0 + k < n1, ok2 = k0 + k < n2;
            v[0][k] = ok1 ? ptx::ld_relaxed_b64(p1 + (k0 + k) * 256) : 0ull;
            v[1][k] = ok1 ? ptx::ld_relaxed_b64(p1 + (k0 + k) * 256 + kHalfTile) : 0ull;
            v[2][k] = ok2 ? ptx::ld_relaxed_b64(p2 + (k0 + k) * 256) : 0ull;
            v[3][k] = ok2 ? ptx::ld_relaxed_b64(p2 + (k0 + k) * 256 + kHalfTile) : 0ull;
            ok &= (!ok1 || (tag_ok(v[0][k], tag) & tag_ok(v[1][k], tag))) &&
                  (!ok2 || (tag_ok(v[2][k], tag) & tag_ok(v[3][k], tag)));
          }
          if (ok || retry_stop(C, t0, it)) break;
        }
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          if (k0 + k < n1) {
            g1 = __fadd_rn(g1, tag_val(v[0][k]));
            u1 = __fadd_rn(u1, tag_val(v[1][k]));
          }
          if (k0 + k < n2) {
            g2 = __fadd_rn(g2, tag_val(v[2][k]));
            u2 = __fadd_rn(u2, tag_val(v[3][k]));
          }
        }
      }
      xs[i] = __fmul_rn(__fdiv_rn(g1, __fadd_rn(1.0f, expf(-g1))), u1) * kTwo64;
      if (two) xs[i + kCT] = __fmul_rn(__fdiv_rn(g2, __fadd_rn(1.0f, expf(-g2))), u2) * kTwo64;
      r = row_next(r2, K);
    }
  }
  C.bar();
  C.fstamp();
  return gemv_stream<8>(DOWN, L, C.chunk);
}

// Drain after an abort: wait (bounded) for the producer to stop and for the copies it
// issued last to land, so that no bulk copy targets this CTA's shared memory after it
// exits.
__device__ __noinline__ void drain() {
  Cons C = make_cons(0);
  C.bar();
  if (C.tid == 0 && C.aborted()) {
    const uint64_t t0 = ptx::globaltimer();
    while (C.flags[4] == 0 && ptx::globaltimer() - t0 < C.ap->timeout_ns) {
    }
    const uint32_t issued = (uint32_t)C.flags[3];
    const uint32_t first = issued > (uint32_t)kStages ? issued - kStages : 0u;
    for (uint32_t j = first; j < issued; ++j) {
      const uint64_t t1 = ptx::globaltimer();
      while (!ptx::mbar_try_wait(&C.full[j % kStages], (j / kStages) & 1u) &&
             ptx::globaltimer() - t1 < C.ap->timeout_ns) {
      }
    }
  }
  C.bar();
}

// final RMSNorm + lm_head rows of this CTA (src/gemv.rs:825-864, 1015) with the greedy
// first-maximum argmax (src/generate.rs:346-352); per-warp bests into MISC
template <int GPL>
__device__ __noinline__ void lm_phase(uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const int H = a.H, lane = C.lane, warp = C.warp;
  float* sB = C.scratch + kOffB;
  const uint32_t tag = tag_of(C, a.L);
  const uint64_t* x = a.xbuf + (long long)a.L * H;
  await_tags(C, a.tiles[DOWN], tag, [&](int i) { return x + i * 256; });
  C.stamp(2 + 8 * kTraceLayers);
  const float ss = load_x(C, sB, x, H, tag);
  const float inv = rms_inv_from(C.csum(ss), H);
  for (int i = C.tid; i < H; i += kCT) sB[i] = __fmul_rn(__fmul_rn(sB[i], inv), a.final_gamma[i]);
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
  const int nv = a.v1 - a.v0;  // this rank's vocab rows
  const int v0 = a.v0 + (int)((unsigned)(C.c * nv) / (unsigned)C.G), v1 = a.v0 + (int)((unsigned)((C.c + 1) * nv) / (unsigned)C.G);
#pragma unroll 1
  for (int r = v0; r < v1; r += a.lm_rows_per_stage) {
    const uint8_t* stg = C.acquire_stage();
    const int nr = min(a.lm_rows_per_stage, v1 - r);
    if (C.stage_ok) {
#pragma unroll 1
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
          const float dot = __fmaf_rn(dd.x + dd.y, kTwo64, -xg[g]);
          acc = __fmaf_rn(__half2float(__ushort_as_half(sp[g])), dot, acc);
        }
        acc = warp_sum(acc);
        const unsigned vi = (unsigned)(r + i);
        if (lane == 0) {
          if (a.tp > 1) {  // every rank holds the full logits, when the caller wants them
            if (a.want_logits)
              for (int p = 0; p < a.tp; ++p) a.peer_logits[p][vi] = acc;
          } else {
            a.logits[vi] = acc;
          }
        }
        if (better(acc, vi, best, besti)) {
          best = acc;
          besti = vi;
        }
      }
    }
    C.release_stage();
  }
  if (lane == 0) {
    C.scratch[kOffMisc + 16 + warp] = best;
    reinterpret_cast<unsigned*>(C.scratch + kOffMisc + 32)[warp] = besti;
  }
}

// ------------------------------------------------------------------ the kernel
template <int GPL>
__global__ void __launch_bounds__(kThreads, 1) decode_megakernel(const Args args) {
  float* scratch = sm_scratch();
  uint64_t* full = sm_full();
  uint64_t* empty = sm_empty();
  volatile int* flags = sm_flags();
  Args* sa = sm_args();
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int c = blockIdx.x, G = gridDim.x;

  if (tid == 0) {
    *sa = args;
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], kCW);
    }
    const int pos0 = args.st->pos, tok0 = args.st->token;
    // an error left by an earlier launch of this step sequence (a timeout, a rejected
    // token) stops this one at once: the host reads the first error after the sequence
    flags[0] = (tok0 < 0 || tok0 >= args.vocab || pos0 < 0 || pos0 >= args.max_pos || args.st->error != 0) ? 1 : 0;
    flags[1] = 0;
    flags[2] = pos0;
    flags[3] = 0;
    flags[4] = 0;
    flags[5] = tok0;
    flags[6] = 0;
    flags[7] = 0;
    flags[8] = (int)(*args.epoch * 64u);  // tags of this launch: tag base + layer + 1
    ptx::fence_mbar_init();
  }
  {  // split-K slots per tile of gate/up, then down
    int* tab = reinterpret_cast<int*>(scratch + kOffTab);
    for (int t = tid; t < args.tiles[GU]; t += kThreads) tab[t] = nslots(args, GU, t);
    for (int t = tid; t < args.tiles[DOWN]; t += kThreads) tab[args.tiles[GU] + t] = nslots(args, DOWN, t);
    const int lc = c - args.sub0[DOWN];
    if (tid == 0 && lc >= 0 && lc < args.subn[DOWN])
      al_span(args, DOWN, lc, tab + args.tiles[GU] + args.tiles[DOWN]);
  }
  __syncthreads();  // last block-wide barrier: the producer warp leaves below
  const Args& a = *sa;
  const int pos = flags[2];
  const int token = flags[5];

  if (warp == kCW) {
    // ---------------- producer: stream this CTA's bytes in consumption order
    if (lane == 0) {
      uint32_t chunk = flags[0] ? kDead : 0u;
#pragma unroll 1
      for (int L = 0; L < a.L; ++L) {
        chunk = produce_gemv(QKV, L, chunk);
        chunk = produce_kv(L, chunk);
        chunk = produce_gemv(OPR, L, chunk);
        chunk = produce_gemv(GU, L, chunk);
        chunk = produce_gemv(DOWN, L, chunk);
        if (a.trace && L < kTraceLayers)
          a.trace[(long long)G * kTracePerCta + (long long)c * kTraceLayers + L] = ptx::globaltimer();
      }
      produce_lm(chunk);
      __threadfence_block();
      flags[4] = 1;
    }
    return;
  }

  // ---------------- consumers
  Cons C = make_cons(0);
  C.stamp(0);
  if (flags[0] && tid == 0) atomicCAS(&a.st->error, 0, 1);  // keep an earlier code (2: timeout)
  const int H = a.H;
  float* sB = scratch + kOffB;  // x copy for the norms

  // embedding row (embed_lookup_q4, src/gemv.rs:710-736): every CTA builds x_0 locally
  if (!C.aborted()) {
    const uint8_t* row = a.lm + (long long)token * a.lm_row_bytes;
    const uint16_t* sc = reinterpret_cast<const uint16_t*>(row + H / 2);
    for (int e = tid; e < H; e += kCT) {
      const uint8_t b = row[e >> 1];
      const int q = ((e & 1) ? (b >> 4) : (b & 0xF)) - 8;
      const float v = __fmul_rn(__half2float(__ushort_as_half(sc[e / kGroup])), (float)q);
      sB[e] = v;
      if (c == 0) st_tagged(a.xbuf + e, v, tag_of(C, 0));
    }
  }
  C.bar();
  C.stamp(1);

  uint32_t chunk = 0;
#pragma unroll 1
  for (int L = 0; L < a.L; ++L) {
    if (tid == 0) flags[7] = L;
    const int tb = 2 + 8 * min(L, kTraceLayers - 1);
    chunk = qkv_phase(L, chunk);
    C.stamp(tb + 1);
    chunk = attention_phase(L, chunk);
    C.stamp(tb + 2);
    chunk = o_phase(L, chunk);
    C.stamp(tb + 4);
    chunk = gu_phase(L, chunk);
    C.stamp(tb + 6);
    chunk = down_phase(L, chunk);
    C.stamp(tb + 7);
  }
  if (tid == 0) flags[7] = -1;

  lm_phase<GPL>(chunk);
  C.stamp(2 + 8 * kTraceLayers + 1);
  drain();
  // CTA argmax -> global partial -> last CTA finishes the step
  const float* bvs = scratch + kOffMisc + 16;
  const unsigned* bis = reinterpret_cast<const unsigned*>(scratch + kOffMisc + 32);
  if (tid == 0) {
    float b = bvs[0];
    unsigned bi = bis[0];
    for (int w = 1; w < kCW; ++w)
      if (better(bvs[w], bis[w], b, bi)) { b = bvs[w]; bi = bis[w]; }
    __stcg(a.lm_v + c, b);
    __stcg(a.lm_i + c, bi);
    const unsigned prev = ptx::atom_add_acqrel(a.cnt + c_lm(a), 1u);
    flags[1] = (prev == (unsigned)(G - 1));
  }
  C.bar();
  if (!flags[1]) return;
  if (tid == 0) {
    float b = -INFINITY;
    unsigned bi = 0xFFFFFFFFu;
    for (int k = 0; k < G; ++k) {
      const float v = __ldcg(a.lm_v + k);
      const unsigned ii = __ldcg(a.lm_i + k);
      if (better(v, ii, b, bi)) { b = v; bi = ii; }
    }
    if (a.tp > 1) {
      // cross-rank first maximum: each rank releases its (value, index) to every rank
      // (the release also covers this rank's logits stores), then reads all of them
      const uint32_t tag = tag_of(C, a.L);
      for (int p = 0; p < a.tp; ++p) {
        ptx::st_release_sys_b64(a.peer_lm[p] + 2 * a.rank, ((uint64_t)tag << 32) | __float_as_uint(b));
        ptx::st_release_sys_b64(a.peer_lm[p] + 2 * a.rank + 1, ((uint64_t)tag << 32) | bi);
      }
      const uint64_t* mine = a.peer_lm[a.rank];
      b = -INFINITY;
      bi = 0xFFFFFFFFu;
      for (int p = 0; p < a.tp; ++p) {
        uint64_t wv = 0, wi = 0, t0 = 0;
        for (int it = 0;; ++it) {
          wv = ptx::ld_acquire_sys_b64(mine + 2 * p);
          wi = ptx::ld_acquire_sys_b64(mine + 2 * p + 1);
          if ((tag_ok(wv, tag) & tag_ok(wi, tag)) || retry_stop(C, t0, it)) break;
        }
        if (better(tag_val(wv), (unsigned)wi, b, bi)) {
          b = tag_val(wv);
          bi = (unsigned)wi;
        }
      }
    }
    const unsigned am = (bi == 0xFFFFFFFFu) ? 0u : bi;
    StepState* st = a.st;
    st->argmax = am;
    const int s = st->step;
    if (a.ring && s >= 0 && s < a.ring_cap) a.ring[s] = am;
    st->step = s + 1;
    st->token = (int)am;
    st->pos = pos + 1;
    *a.epoch = *a.epoch + 1u;  // next launch's tags
  }
  // every CTA has arrived: reset the arrival counters for the next launch
  for (int i = tid; i < a.n_cnt; i += kCT) a.cnt[i] = 0u;
}

}  // namespace mk
}  // namespace qora
