// megakernel.cuh — the whole batch-1 decode step (embedding, every layer, final norm,
// lm_head, greedy argmax, state advance) as ONE persistent kernel: one CTA per SM.
//
// Why: at batch 1 every projection is a ~2-25 MB HBM stream, and a kernel per operation
// pays launch gaps plus the drain/fill of the memory pipeline at each boundary. Here the
// weight stream never stops: each CTA's producer warp walks the CTA's fixed list of
// weight byte ranges for the whole step (they do not depend on activations) and copies
// them with bulk (TMA) copies into a ring of shared-memory stages; the consumer warps
// walk the same list, waiting for (a) the stage to land and (b) the activation the phase
// needs, published by other CTAs as tagged words. While consumers wait on a dependency
// the producer keeps filling the ring.
//
// Per layer (CTA sets in brackets):
//   QKV  [one CTA per 32-column group of q|k|v] RMSNorm(x) . W over all rows -> final
//        q|k|v values (before RoPE), no split-K
//   ATTN [one CTA per (kv head, chunk of positions)] RoPE on its query heads (and, for
//        the chunk holding the new position, on k, which it appends with v to the
//        head-major cache), scores, softmax numerators, P.V -> (m, l, o); with several
//        chunks per KV head every unit of the head then merges one slice of the head's
//        outputs from all chunks' partials (one chunk: the unit publishes o / l itself)
//   O    [one CTA per 32-column group of o_proj] the merged attention output of all
//        heads, GEMV over all rows, x_mid = x + o for its columns
//   GU   [all] RMSNorm(x_mid) . [gate|up], split-K over 256-column tiles -> partials
//   DOWN [all] SwiGLU of its rows from the gate/up partials, split-K GEMV with every
//        CTA's rows inside one output tile; then each CTA of a tile sums one slice of
//        the tile's columns over all its split-K partials: x_next = x_mid + down
// then lm_head rows (a contiguous slice per CTA) with a fused first-maximum argmax.
//
// Hand-off between CTAs: every value one CTA passes to another travels as a 64-bit word
// (tag << 32 | f32 bits) written and read with single-copy-atomic relaxed accesses; the
// tag names the launch and the layer. A reader loads its words directly and re-reads
// (after a short sleep) only those whose tag is not yet the current one: one L2 round
// trip once the data is there, no separate flag, fence or arrival counter.
//
// Instruction-cache discipline: B200's per-SM instruction cache holds ~60 KB of code
// (a straight-line probe runs at ~2.7 cycles per instruction up to 61 KB and 4-11
// beyond 76 KB) and every layer executes each phase once, so code a layer runs beyond
// that is fetched again from L2 every layer (measured: phase prologues of ~150
// instructions taking 1.3-2 us while each layer ran ~150 KB of code). So the code a
// layer executes is kept small: one GEMV routine serves all four matrices (the tile
// width is a runtime parameter), the attention unit and the hand-off helpers exist once,
// out of line, and only the GEMV's inner loop is unrolled. Nothing of the consumer state
// lives in local memory.
//
// Every wait (tagged word, stage barrier, ring slot) is bounded by a timeout; on expiry
// the CTA records QORA_ERR_TIMEOUT in the step state, stops computing, drains the copies
// it has in flight and exits; long waits also watch the step's error word, so that one
// CTA's timeout stops the grid. No form of multicast is used.
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
// K or V rows of one head per stage: multiples of 4 (the P.V reads four rows'
// probabilities as one float4), one score pass each (see score_rows: one row per lane
// group for f32, two for binary16); chunks are whole multiples of 60 rows
constexpr int kKVRows = 60;     // f32 rows (30 KB of the 34.5 KB stage)
constexpr int kKVRows16 = 120;  // binary16 rows
constexpr int kMinAttnChunk = 60;
constexpr int kMaxAttnChunk = 1020;
constexpr int kMaxUnits = 256;         // attention units (kv head x chunk); units <= CTAs
constexpr int kHeadsPerKV = 4;         // query heads per KV head (SmolLM3-3B: 16 / 4)
constexpr int kRowsPerLane = 4;        // GEMV rows per lane per stage (both tile widths)
// shared scratch (floats): XS = inputs of this CTA's GEMV (pre-scaled by 2^64); B = x
// copy / cross-warp reduction / down-tile slice; Y = a segment's reduced sums; MISC =
// small reductions; TAB = split-K slots per tile; FIN = residual values of the columns
// this CTA finishes (its o_proj columns, its slice of a down tile)
constexpr int kXsCap = 2048;
constexpr int kOffB = kXsCap;
constexpr int kBFloats = kCW * 256;
constexpr int kOffY = kOffB + kBFloats;
constexpr int kOffMisc = kOffY + 256;
constexpr int kOffTab = kOffMisc + 64;
constexpr int kMaxTabTiles = 128;
constexpr int kOffFin = kOffTab + kMaxTabTiles;
constexpr int kFinCap = 256;
constexpr int kOffPlan = kOffFin + kFinCap;  // this CTA's plan for the launch (ints, see make_plan)
constexpr int kPlanInts = 64;
constexpr int kScratchFloats = kOffPlan + kPlanInts;
// attention (overlaps XS and B): q [4][128] | scores [4][kMaxAttnChunk] | (m,l) [4][2] |
// 1/l [4] | the new position's k and v rows [2][128] in the cache's element type
constexpr int kAttQ = 0, kAttS = 512, kAttML = kAttS + 4 * kMaxAttnChunk, kAttInv = kAttML + 8, kAttKV = kAttInv + 4;
// attention merge staging (XS and B, once the unit's own partials are out): the slice's
// o values [nch][slice], chunk (m, l) [nch][heads][2], weights [heads][nch], 1/l [heads]
constexpr int kMgO = 0, kMgML = 1024, kMgW = kMgML + 2 * kHeadsPerKV * kMaxUnits, kMgInv = kMgW + kHeadsPerKV * kMaxUnits;
static_assert(kAttKV + 256 <= kOffY, "attention scratch");
static_assert(kMgO + kHeadsPerKV * kHeadDim + kMaxUnits <= kMgML && kMgInv + kHeadsPerKV <= kOffY, "merge staging");
constexpr float kTwo64 = 18446744073709551616.0f;
constexpr int kPairsMax = (kXsCap / 2 + kCT - 1) / kCT;  // tagged word pairs per thread of a vector (3)
constexpr unsigned kPollSleepNs = 0;  // pause between re-reads of words that are not there yet (0: none)

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
  uint64_t* dn_part;          // tagged down split-K partials [tiles][slots][256]
  uint64_t* att_o;            // tagged [kMaxUnits][4][128]
  uint64_t* att_ml;           // tagged [kMaxUnits][4][2]
  uint64_t* att_fin;          // tagged [nh][128] merged attention output of the layer
  unsigned* epoch;            // launches so far (the tag base); advanced by the last CTA
  unsigned* cnt;              // arrival counters (the step's final one at c_lm), zero between launches
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
// [5] token, [6] spare, [7] current layer, [8] tag base (epoch * 64)

// Trace layout: per CTA kTracePerCta u64 globaltimer stamps written by consumer thread 0:
// [0] start, [1] after embedding, then per layer L at 2 + 8L + {0: x ready (QKV CTAs),
// 1: QKV done, 2: attention done, 3: attention output ready (O CTAs), 4: O done,
// 5: x_mid ready, 6: GU done, 7: DOWN done}, then [2+8*kTraceLayers] lm start, [+1] end.
// Then, per CTA, one stamp per layer when the producer has issued that layer's last
// copy; then kTraceFine spare words per CTA.
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

// the step's final arrival counter (the last CTA to arrive finishes the argmax)
QORA_DEV int c_lm(const Args& a) { return a.L * a.cpl; }

// ---- split-K geometry (32-bit: the host checks set size x tiles x K < 2^31)
// CTA lc of a g-CTA set owns rows [lc*T/g, (lc+1)*T/g) of the tiles*K flattened rows
QORA_DEV int owner32(unsigned p, unsigned total, unsigned g) { return (int)(((p + 1u) * g - 1u) / total); }

// Tile-aligned split-K (down_proj): tile t of T runs on CTAs [al_first(t), al_first(t+1))
// of a g-CTA set (g >= T, so every tile gets floor or ceil of g/T CTAs), and CTA j of
// the n on tile t owns its rows [j*K/n, (j+1)*K/n). No CTA crosses a tile boundary, so
// none streams two partial segments, and the n CTAs of a tile finish it together (each
// one slice of its columns).
// (32-bit: the host checks tiles * g and g * K below 2^31)
__host__ __device__ inline int al_first(int t, int g, int T) { return (int)((unsigned)(t * g) / (unsigned)T); }
__host__ __device__ inline int al_tile(int lc, int g, int T) {  // the tile CTA lc works on
  int t = (int)((unsigned)(lc * T) / (unsigned)g);
  while (t + 1 < T && al_first(t + 1, g, T) <= lc) ++t;
  while (t > 0 && al_first(t, g, T) > lc) --t;
  return t;
}

// CTA lc's span of the tile-aligned matrix: first flattened row, rows, first CTA of its tile
__host__ __device__ __forceinline__ void al_span(const Args& a, int m, int lc, int* out) {  // out: lin0, n, first CTA of the tile
  const int g = a.subn[m], T = a.tiles[m], K = a.K[m], t = al_tile(lc, g, T);
  const int f0 = al_first(t, g, T), n = al_first(t + 1, g, T) - f0, j = lc - f0;
  const int r0 = (int)((unsigned)(j * K) / (unsigned)n), r1 = (int)((unsigned)((j + 1) * K) / (unsigned)n);
  out[0] = t * K + r0;
  out[1] = r1 - r0;
  out[2] = f0;
}

QORA_DEV int nslots(const Args& a, int m, int t) {
  if (m == DOWN) return al_first(t + 1, a.subn[m], a.tiles[m]) - al_first(t, a.subn[m], a.tiles[m]);
  const unsigned K = (unsigned)a.K[m], total = (unsigned)a.tiles[m] * K, g = (unsigned)a.subn[m];
  return owner32((unsigned)(t + 1) * K - 1u, total, g) - owner32((unsigned)t * K, total, g) + 1;
}

QORA_DEV int row_bytes(int m) { return m < GU ? 18 : 144; }

// ---- the CTA's plan for one launch, computed once at kernel start (make_plan) so that
// no phase, and not the producer, repeats the integer divisions of the split geometry
// in every layer. Ints in shared memory:
//   [10 m ..]  matrix m: rows of the span, segments (<= 2), then per segment
//              (tile, first row, end row, split-K slot)
//   [40 ..]    attention unit: has a unit, kv head, chunk index, first position, end
//              position, end of the cached rows (the new position excluded), chunks per
//              KV head, holds the new position
//   [48 ..]    its merge slice: first output, end output, first head, heads
//   [52 ..]    down finish: tile, first column, end column, split-K slots of the tile
constexpr int kPlMat = 10, kPlAtt = 40, kPlMerge = 48, kPlDown = 52;
QORA_DEV int* plan_w() { return reinterpret_cast<int*>(sm_scratch() + kOffPlan); }
QORA_DEV const int* plan() { return reinterpret_cast<const int*>(sm_scratch() + kOffPlan); }
QORA_DEV const int* mat_plan(int m) { return plan() + kPlMat * m; }

// matrix m's span of CTA c (one thread per matrix, kernel start)
__device__ __noinline__ void make_mat_plan(const Args& a, int m, int c) {
  int* P = plan_w() + kPlMat * m;
  P[0] = P[1] = 0;
  const int lc = c - a.sub0[m], g = a.subn[m], K = a.K[m];
  if (lc < 0 || lc >= g) return;
  if (m == DOWN) {  // tile-aligned: one segment, and this CTA's slice of the tile's columns
    int sp[3];
    al_span(a, DOWN, lc, sp);
    const int t = sp[0] / K, j = lc - sp[2], ns = al_first(t + 1, g, a.tiles[m]) - sp[2];
    P[0] = sp[1];
    P[1] = sp[1] > 0 ? 1 : 0;
    P[2] = t;
    P[3] = sp[0] - t * K;
    P[4] = P[3] + sp[1];
    P[5] = j;
    int* D = plan_w() + kPlDown;
    D[0] = t;
    D[1] = j * kTileCols / ns;
    D[2] = (j + 1) * kTileCols / ns;
    D[3] = ns;
    return;
  }
  // CTA lc of the g-CTA set owns rows [lc*T/g, (lc+1)*T/g) of the tiles*K flattened rows
  const unsigned total = (unsigned)a.tiles[m] * (unsigned)K;
  const int l0 = (int)((unsigned)lc * total / (unsigned)g), l1 = (int)((unsigned)(lc + 1) * total / (unsigned)g);
  P[0] = l1 - l0;
  int ns = 0;
  for (int p = l0; p < l1 && ns < 2; ++ns) {
    const int t = p / K, pe = min(l1, (t + 1) * K);
    P[2 + 4 * ns] = t;
    P[3 + 4 * ns] = p - t * K;
    P[4 + 4 * ns] = pe - t * K;
    P[5 + 4 * ns] = lc - owner32((unsigned)t * (unsigned)K, total, (unsigned)g);
    p = pe;
  }
  P[1] = ns;
}

// the attention unit of CTA c for a cache of len positions (the new one at len - 1):
// (kv head, chunk of `chunk` positions), about one unit per CTA, on the CTAs from the end
// of the grid (the q|k|v CTAs) so that the o_proj CTAs at the front keep their o_proj
// weights queued in the ring behind nothing
__device__ __noinline__ void make_att_plan(const Args& a, int c, int G, int pos) {
  int* P = plan_w() + kPlAtt;
  P[0] = 0;
  if (pos < 0 || pos >= a.max_pos) return;  // rejected at kernel start: no unit, no cache write
  const int len = pos + 1;
  int csz = (len * a.nkvh + G - 1) / G;
  csz = max(kMinAttnChunk, min(kMaxAttnChunk, csz));
  csz = (csz + 59) / 60 * 60;  // whole stages of either cache type (<= kMaxAttnChunk: a multiple of 60)
  const int nch = (len + csz - 1) / csz, u = G - 1 - c;
  P[0] = u < a.nkvh * nch ? 1 : 0;
  if (!P[0]) return;
  const int g = u % a.nkvh, k = u / a.nkvh, s0 = k * csz, s1 = min(len, s0 + csz);
  P[1] = g;
  P[2] = k;
  P[3] = s0;
  P[4] = s1;
  P[5] = min(s1, pos);
  P[6] = nch;
  P[7] = pos < s1 ? 1 : 0;
  int* M = plan_w() + kPlMerge;  // outputs [r0, r1) of the head's hpk * 128
  const int nout = a.hpk * kHeadDim, r0 = k * nout / nch, r1 = (k + 1) * nout / nch;
  M[0] = r0;
  M[1] = r1;
  M[2] = r0 / kHeadDim;
  M[3] = (r1 - 1) / kHeadDim + 1 - r0 / kHeadDim;
}

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
  const int* P = mat_plan(m);
#pragma unroll 1
  for (int sg = 0; sg < P[1]; ++sg) {
    const int t = P[2 + 4 * sg], r1 = P[4 + 4 * sg];
#pragma unroll 1
    for (int r = P[3 + 4 * sg]; r < r1; r += rps)
      chunk = issue(base + ((long long)t * K + r) * rb, (uint32_t)(min(rps, r1 - r) * rb), chunk);
  }
  return chunk;
}

// the cached K rows, then V rows, of this CTA's attention unit (if it has one)
__device__ __noinline__ uint32_t produce_kv(int L, uint32_t chunk) {
  const Args& a = *sm_args();
  const int* P = plan() + kPlAtt;
  if (!P[0]) return chunk;
  const int g = P[1], s0 = P[3], sc1 = P[5];
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
  uint32_t stage_idx;     // chunk % kStages and the phase parity of chunk, kept incrementally
  uint32_t parity;
  bool stage_ok;          // warp-uniform: the current stage landed and the CTA is healthy

  QORA_DEV const Args& a() const { return *ap; }
  QORA_DEV int ns(int m, int t) const {  // split-K slots of tile t (GU, DOWN)
    return reinterpret_cast<const int*>(scratch + kOffTab)[(m == GU ? 0 : ap->tiles[GU]) + t];
  }
  // this thread's view; a decision that gates a barrier goes through bar_or()
  QORA_DEV bool aborted() const { return flags[0] != 0; }
  // uniform within the calling warp at any point
  QORA_DEV bool aborted_w() const { return __shfl_sync(0xffffffffu, flags[0] != 0, 0); }

  QORA_DEV void bar() const { ptx::named_bar(kBar, kCT); }
  // barrier that also tells every consumer thread whether any of them saw an abort
  QORA_DEV bool bar_aborted() const { return ptx::named_bar_or(kBar, kCT, flags[0] != 0); }

  QORA_DEV void stamp(int idx) {
    if (ap->trace && tid == 0) ap->trace[(long long)c * kTracePerCta + idx] = ptx::globaltimer();
  }

  // next stage of the ring (every consumer warp calls this for every chunk, in order).
  // Once the CTA has aborted, stages are skipped without waiting (see drain()).
  QORA_DEV const uint8_t* acquire_stage();

  QORA_DEV void release_stage() {
    __syncwarp();
    if (lane == 0 && stage_ok) ptx::mbar_arrive(&empty[stage_idx]);
    ++chunk;
    if (++stage_idx == (uint32_t)kStages) {
      stage_idx = 0;
      parity ^= 1u;
    }
  }
};

// The slow path of a stage acquisition (the stage had not landed when first tested):
// wait (bounded) for ring slot s to complete the phase with the given parity; true
// (warp-uniform) once it has, false if the CTA has aborted or the wait timed out
// (recorded). Once the CTA has aborted, stages are skipped without waiting (drain()).
__device__ __noinline__ bool stage_wait_slow(uint32_t s, uint32_t parity) {
  volatile int* flags = sm_flags();
  uint64_t* bar = sm_full() + s;
  bool timed_out = false;
  const uint64_t t0 = ptx::globaltimer();
  while (!ptx::mbar_try_wait(bar, parity)) {
    if (flags[0] != 0 || ptx::globaltimer() - t0 > sm_args()->timeout_ns) {
      timed_out = true;
      break;
    }
  }
  const bool ok = __all_sync(0xffffffffu, !timed_out);
  if (!ok && (threadIdx.x & 31) == 0 && flags[0] == 0) {
    flags[0] = 1;
    atomicExch(&sm_args()->st->error, 2);
  }
  return ok;
}

// Fast path inline (one test of the full barrier and a warp vote: a landed stage costs
// no call, no division and no abort check; a stage only completes while the CTA is
// healthy or its copy was issued before an abort, which the drain waits for anyway).
QORA_DEV const uint8_t* Cons::acquire_stage() {
  stage_ok = __all_sync(0xffffffffu, ptx::mbar_try_wait(&full[stage_idx], parity)) ||
             stage_wait_slow(stage_idx, parity);
  return ring + (size_t)stage_idx * kStageBytes;
}

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
  C.stage_idx = chunk % kStages;
  C.parity = (chunk / kStages) & 1u;
  C.stage_ok = false;
  return C;
}

// ---- tagged hand-off values: (tag << 32) | f32 bits
QORA_DEV uint32_t tag_of(const Cons& C, int L) { return (uint32_t)C.flags[8] + (uint32_t)L + 1u; }
QORA_DEV void st_tagged(uint64_t* p, float v, uint32_t tag) {
  ptx::st_relaxed_b64(p, ((uint64_t)tag << 32) | __float_as_uint(v));
}
QORA_DEV bool tag_ok(uint64_t w, uint32_t tag) { return (uint32_t)(w >> 32) == tag; }
QORA_DEV float tag_val(uint64_t w) { return __uint_as_float((uint32_t)w); }

// Retry control for tagged loads that found a stale tag (the producer's store had not
// arrived yet), called with it = 0, 1, 2, ... for the failed attempts of one wait:
// true = give up (this CTA or the grid aborted, or the wait timed out).
__device__ __noinline__ bool retry_stop(uint64_t& t0, int it) {
  const Args& a = *sm_args();
  volatile int* flags = sm_flags();
  if (it == 0) {
    t0 = ptx::globaltimer();
    return false;
  }
  if (flags[0] != 0) return true;
  const uint64_t dt = ptx::globaltimer() - t0;
  if (dt > a.timeout_ns) {
    flags[0] = 1;
    atomicExch(&a.st->error, 2);
    return true;
  }
  if (dt > kGridCheckNs && grid_failed(a)) {  // another CTA gave up: its code stands
    flags[0] = 1;
    return true;
  }
  if (kPollSleepNs) __nanosleep(kPollSleepNs);
  return false;
}

// one tagged value, re-read until it carries `tag` (bounded)
QORA_DEV float ld_checked(const uint64_t* p, uint32_t tag) {
  uint64_t w, t0 = 0;
#pragma unroll 1
  for (int it = 0;; ++it) {
    w = ptx::ld_relaxed_b64(p);
    if (tag_ok(w, tag) || retry_stop(t0, it)) break;
  }
  return tag_val(w);
}

// n tagged words (n even, n <= 2 * kPairsMax * kCT) -> dst[i] = value * mul (shared).
// Each thread loads its own pairs and re-reads only the stale ones until every word
// carries `tag` (bounded). The caller's barrier publishes dst. Returns the sum of squares
// of this thread's values (before `mul`), accumulated in a fixed order.
__device__ __noinline__ float poll_vec(const uint64_t* src, int n, uint32_t tag, float* dst, float mul) {
  const int tid = threadIdx.x, np = n >> 1;
  uint32_t todo = 0;
#pragma unroll
  for (int j = 0; j < kPairsMax; ++j)
    if (tid + j * kCT < np) todo |= 1u << j;
  uint64_t t0 = 0;
  float v[kPairsMax][2];
#pragma unroll 1
  for (int it = 0; todo != 0u; ++it) {
    uint64_t w[kPairsMax][2];
#pragma unroll
    for (int j = 0; j < kPairsMax; ++j)
      if (todo & (1u << j)) ptx::ld_relaxed_v2_b64(src + 2 * (tid + j * kCT), w[j][0], w[j][1]);
#pragma unroll
    for (int j = 0; j < kPairsMax; ++j)
      if ((todo & (1u << j)) && tag_ok(w[j][0], tag) && tag_ok(w[j][1], tag)) {
        v[j][0] = tag_val(w[j][0]);
        v[j][1] = tag_val(w[j][1]);
        todo &= ~(1u << j);
      }
    if (todo != 0u && retry_stop(t0, it)) break;
  }
  float ss = 0.0f;
#pragma unroll
  for (int j = 0; j < kPairsMax; ++j) {
    const int b = tid + j * kCT;
    if (b < np && !(todo & (1u << j))) {
      dst[2 * b] = __fmul_rn(v[j][0], mul);
      dst[2 * b + 1] = __fmul_rn(v[j][1], mul);
      ss = __fmaf_rn(v[j][0], v[j][0], ss);
      ss = __fmaf_rn(v[j][1], v[j][1], ss);
    }
  }
  return ss;
}

// block sum over consumer threads (fixed order), result in every thread
// Sum of kCW values in a fixed tree order (all loads first; no long dependent chain)
QORA_DEV float sum15(const float* p, int stride) {
  float v[kCW];
#pragma unroll
  for (int w = 0; w < kCW; ++w) v[w] = p[w * stride];
#pragma unroll
  for (int w = 0; w < 7; ++w) v[w] = __fadd_rn(v[2 * w], v[2 * w + 1]);  // 7 pairs, v[14] kept
  v[7] = v[14];
#pragma unroll
  for (int w = 0; w < 4; ++w) v[w] = __fadd_rn(v[2 * w], v[2 * w + 1]);
  return __fadd_rn(__fadd_rn(v[0], v[1]), __fadd_rn(v[2], v[3]));
}

// Block sum of the consumer threads' v in two halves around a barrier the caller has
// anyway (the one that publishes the polled vector): csum_put before it, csum_get after.
// The warp sums sit in MISC[0, 15) until the next barrier after csum_get (every caller
// has one before MISC is written again).
__device__ __forceinline__ void csum_put(float v) {
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) sm_scratch()[kOffMisc + (threadIdx.x >> 5)] = v;
}
__device__ __forceinline__ float csum_get() { return sum15(sm_scratch() + kOffMisc, 1); }

__device__ __forceinline__ float rms_inv_from(float sumsq, int H) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sumsq, (float)H), 1e-6f)));
}

// Input row of entry i of matrix m's span (its segments' rows back to back)
QORA_DEV int span_row(const int* P, int i) {
  const int n0 = P[4] - P[3];
  return i < n0 ? P[3] + i : P[7] + (i - n0);
}
// Norm gains gamma[row] of matrix m's span copied into xs asynchronously: issued before
// the wait for the activations, used after it.
__device__ __forceinline__ void stage_gains(const float* gamma, int m) {
  float* xs = sm_scratch();
  const int* P = mat_plan(m);
#pragma unroll 1
  for (int i = threadIdx.x; i < P[0]; i += kCT) ptx::cp_async_4(xs + i, gamma + span_row(P, i));
}
// xs[i] = x[row] * inv * gamma[row] * 2^64 (gamma from stage_gains, this thread's own
// copies)
__device__ __forceinline__ void fill_norm_inputs(const float* x, float inv, int m) {
  float* xs = sm_scratch();
  const int* P = mat_plan(m);
  ptx::cp_async_wait_all();
  constexpr int kPer = (kXsCap + kCT - 1) / kCT;  // entries per thread (5): independent, unrolled
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = threadIdx.x + j * kCT;
    if (i < P[0]) xs[i] = __fmul_rn(__fmul_rn(x[span_row(P, i)], inv), xs[i]) * kTwo64;
  }
}

// Tensor parallelism: this rank's partial value v of column `col` goes to every rank's
// receive buffer bufs[p][(L*tp + rank)*H + col]; the sum over ranks (rank order, the same
// on every rank) comes back once all tp partials of the column have arrived (bounded).
QORA_DEV void tp_push(const Args& a, uint64_t* const* bufs, int L, int col, float v, uint32_t tag) {
  const long long o = ((long long)L * a.tp + a.rank) * a.H + col;
  const uint64_t w = ((uint64_t)tag << 32) | __float_as_uint(v);
  for (int p = 0; p < a.tp; ++p) ptx::st_relaxed_sys_b64(bufs[p] + o, w);
}
__device__ __noinline__ float tp_sum(const uint64_t* own, int L, int col, uint32_t tag) {
  const Args& a = *sm_args();
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
    if (ok || retry_stop(t0, it)) break;
  }
  return s;
}

// ------------------------------------------------------------------ the GEMV
// A finished segment's sums (Y) go out tagged: q|k|v values; x_mid = x + o for o_proj
// columns (residual values from FIN); gate/up and down split-K partials.
__device__ __forceinline__ void seg_store(int m, int L, int t, int slot) {
  const Cons C = make_cons(0);
  const Args& a = C.a();
  const float* y = C.scratch + kOffY;
  const uint32_t tag = tag_of(C, L);
  if (m == QKV) {
    if (C.tid < kGroup) st_tagged(a.qkv + t * kGroup + C.tid, y[C.tid], tag);
  } else if (m == OPR) {
    if (C.tid < kGroup) {
      const int col = t * kGroup + C.tid;
      float o = y[C.tid];
      if (a.tp > 1) {  // row-split o_proj: sum the ranks' partials of this column
        tp_push(a, a.peer_o, L, col, o, tag);
        o = tp_sum(a.peer_o[a.rank], L, col, tag);
      }
      st_tagged(a.xmid + (long long)L * a.H + col, __fadd_rn(C.scratch[kOffFin + C.tid], o), tag);
    }
  } else if (C.tid < kTileCols) {
    const long long o = ((long long)t * a.slots[m] + slot) * kTileCols + C.tid;
    st_tagged((m == GU ? a.gu_part : a.dn_part) + o, y[C.tid], tag);
  }
}

// Stream this CTA's segments of matrix m through the ring, reduce each segment's sums
// into Y and store them (seg_store). Eight-group tiles (gate/up, down; T8): lane (sub,
// gi) takes group gi of 4 rows per warp pass; one-group tiles (q|k|v, o_proj): lane i
// takes row i of 32 per warp pass. Both read one 16-byte chunk of a 144-byte block per
// row and give every lane kRowsPerLane rows per stage; xs holds the (pre-scaled) inputs
// of all segments back to back. The tile width is a template parameter: the inner loop
// is bound by the ALU pipe (the nibble masks), and index arithmetic that depends on a
// runtime width measured 7 % of the whole step.
template <bool T8>
__device__ __noinline__ uint32_t gemv_run(int m, int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  constexpr bool t8 = T8;
  const int W = t8 ? 4 : 32;                       // rows per warp pass
  const int RPS = kStageBytes / (t8 ? 144 : 18);    // rows per stage (240 | 1920)
  const int NO = t8 ? kTileCols : kGroup;          // outputs per segment
  const int gi = t8 ? (C.lane & 7) : 0, sub = t8 ? (C.lane >> 3) : C.lane;
  const float* xs = C.scratch;
  float* red = C.scratch + kOffB;
  float* y = C.scratch + kOffY;
  const int* P = mat_plan(m);
  // this lane's rows of a stage (i = warp*W + sub + k*kCW*W, always inside the stage)
  // and the byte offsets of their 16-byte chunks, the same for every stage
  int row[kRowsPerLane], boff[kRowsPerLane], soff[kRowsPerLane];
#pragma unroll
  for (int k = 0; k < kRowsPerLane; ++k) {
    row[k] = C.warp * W + sub + k * kCW * W;
    const int blk = (t8 ? row[k] : (row[k] >> 3)) * 144, q = t8 ? gi : (row[k] & 7);
    boff[k] = blk + q * 16;
    soff[k] = blk + 128 + q * 2;
  }
  const int base = C.warp * W;
  int off = 0;
#pragma unroll 1
  for (int sg = 0; sg < P[1]; ++sg) {
    const int r0 = P[3 + 4 * sg], r1 = P[4 + 4 * sg];
    float2 acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = make_float2(0.0f, 0.0f);
    float cs = 0.0f;
#pragma unroll 1
    for (int cr = r0; cr < r1; cr += RPS) {
      const uint8_t* stg = C.acquire_stage();
      const int R = min(RPS, r1 - cr);
      if (C.stage_ok) {
        const float* xr = xs + off + (cr - r0);
        uint4 w[kRowsPerLane];
        float cf[kRowsPerLane];
#pragma unroll
        for (int k = 0; k < kRowsPerLane; ++k) {  // all loads issued before the math
          // rows past R of a partial stage read stale stage bytes and get a zero factor
          w[k] = *reinterpret_cast<const uint4*>(stg + boff[k]);
          const uint16_t sv = *reinterpret_cast<const uint16_t*>(stg + soff[k]);
          const float xv = xr[row[k]];
          cf[k] = row[k] < R ? __half2float(__ushort_as_half(sv)) * xv : 0.0f;
        }
#pragma unroll
        for (int k = 0; k < kRowsPerLane; ++k) {
          if (base + k * kCW * W < R) {  // passes past the stage's end are skipped (warp-uniform)
            cs += cf[k];
            q4_fma_chunk(w[k], cf[k], acc);
          }
        }
      }
      C.release_stage();
    }
    off += r1 - r0;

    // this lane's 32 outputs, then a transposing reduction over the lanes holding the
    // same outputs (masks 16, 8; one-group tiles also 4, 2, 1): afterwards lane (sub, gi)
    // holds outputs sub*8 + [0, 8) of group gi (eight-group) or output `lane` (one-group)
    const float bias = cs * 4.3368086899420177e-19f;  // 8 * 2^-64
    float v[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      v[2 * i] = __fmaf_rn(acc[i].x, q4_scale_of_pos((2 * i) & 7), -bias);
      v[2 * i + 1] = __fmaf_rn(acc[i].y, q4_scale_of_pos((2 * i + 1) & 7), -bias);
    }
#pragma unroll
    for (int msk = 16; msk >= (t8 ? 8 : 1); msk >>= 1) {
      const bool hi = (C.lane & msk) != 0;
#pragma unroll
      for (int e2 = 0; e2 < msk; ++e2) {
        const float send = hi ? v[e2] : v[msk + e2];
        const float keep = hi ? v[msk + e2] : v[e2];
        v[e2] = keep + __shfl_xor_sync(0xffffffffu, send, msk);
      }
    }
    // warp w's sums at red[w][e2][lane] (consecutive lanes, consecutive words): output
    // o = gi*32 + sub*8 + e2 of an eight-group tile sits at e2*32 + sub*8 + gi, output
    // `lane` of a one-group tile at lane
#pragma unroll
    for (int e2 = 0; e2 < (t8 ? 8 : 1); ++e2) red[C.warp * NO + e2 * 32 + C.lane] = v[e2];
    C.bar();
    if (C.tid < NO) {
      const int o = C.tid;
      y[o] = sum15(red + (t8 ? (o & 7) * 32 + ((o >> 3) & 3) * 8 + (o >> 5) : o), NO);
    }
    C.bar();
    seg_store(m, L, P[2 + 4 * sg], P[5 + 4 * sg]);
  }
  return C.chunk;
}

// ------------------------------------------------------------------ phases
// QKV: RMSNorm(x) . W for this CTA's 32-column group, all rows
__device__ __noinline__ uint32_t qkv_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  if (mat_plan(QKV)[0] == 0) return chunk;
  const int H = a.H;
  float* sB = C.scratch + kOffB;
  stage_gains(a.layers[L].g_in, QKV);
  float ss = 0.0f;
  if (L > 0) {
    ss = poll_vec(a.xbuf + (long long)L * H, H, tag_of(C, L), sB, 1.0f);
  } else {  // x_0 (the embedding row) is already in sB
#pragma unroll 1
    for (int i = C.tid; i < H; i += kCT) ss = __fmaf_rn(sB[i], sB[i], ss);
  }
  csum_put(ss);
  C.bar();
  C.stamp(2 + 8 * min(L, kTraceLayers - 1) + 0);
  const float inv = rms_inv_from(csum_get(), H);
  fill_norm_inputs(sB, inv, QKV);
  C.bar();
  return gemv_run<false>(QKV, L, C.chunk);
}

// O: the merged attention output of every head, GEMV over all rows for this CTA's 32
// columns, x_mid = x + o (the residual x of the columns is read first: it is ready)
__device__ __noinline__ uint32_t o_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const int* P = mat_plan(OPR);
  if (P[0] == 0) return chunk;
  const uint32_t tag = tag_of(C, L);
  if (C.tid < kGroup) C.scratch[kOffFin + C.tid] = ld_checked(a.xbuf + (long long)L * a.H + P[2] * kGroup + C.tid, tag);
  poll_vec(a.att_fin, a.K[OPR], tag, C.scratch, kTwo64);
  C.bar();
  C.stamp(2 + 8 * min(L, kTraceLayers - 1) + 3);
  return gemv_run<false>(OPR, L, C.chunk);
}

// GU (all): RMSNorm(x_mid) . [gate|up] -> split-K partials per tile
__device__ __noinline__ uint32_t gu_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const int H = a.H;
  float* sB = C.scratch + kOffB;
  stage_gains(a.layers[L].g_post, GU);
  const float ss = poll_vec(a.xmid + (long long)L * H, H, tag_of(C, L), sB, 1.0f);
  csum_put(ss);
  C.bar();
  C.stamp(2 + 8 * min(L, kTraceLayers - 1) + 5);
  if (mat_plan(DOWN)[0] > 0) {  // keep x_mid of the down columns this CTA finishes (sB is reused below)
    const int* D = plan() + kPlDown;
    if (C.tid < D[2] - D[1]) C.scratch[kOffFin + C.tid] = sB[D[0] * kTileCols + D[1] + C.tid];
  }
  const float inv = rms_inv_from(csum_get(), H);
  fill_norm_inputs(sB, inv, GU);
  C.bar();
  return gemv_run<true>(GU, L, C.chunk);
}

// silu(g) * u with silu(g) = g / (1 + exp(-g)) (src/gemv.rs:494-500)
__device__ __forceinline__ float swiglu(float g, float u) {
  return __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
}

// DOWN (all): SwiGLU of the rows it needs from the gate/up partials (src/gemv.rs:412-502),
// split-K GEMV, then this CTA's slice of its tile: x_{L+1} = x_mid + the sum of the tile's
// partials in slot order
__device__ __noinline__ uint32_t down_phase(int L, uint32_t chunk) {
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const int* P = mat_plan(DOWN);
  const int n = P[0];
  if (n == 0) return chunk;
  const int S = a.slots[GU];
  constexpr int kHalfTile = kTileCols / 2;  // gate (then up) outputs per gate/up tile
  const uint32_t tag = tag_of(C, L);
  {  // rows i = tid, tid + kCT: both rows' gate and up partials (4 slots each) in flight
    float* xs = C.scratch;
#pragma unroll 1
    for (int i = C.tid; i < n; i += 2 * kCT) {
      const int r = P[3] + i, r2 = r + kCT;  // one segment: rows P[3] + i
      const bool two = i + kCT < n;
      const int t1 = r / kHalfTile, t2 = r2 / kHalfTile;
      const int n1 = C.ns(GU, t1), n2 = two ? C.ns(GU, t2) : 0;
      const uint64_t* p1 = a.gu_part + (long long)t1 * S * kTileCols + r % kHalfTile;
      const uint64_t* p2 = a.gu_part + (long long)t2 * S * kTileCols + r2 % kHalfTile;
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
            v[0][k] = ok1 ? ptx::ld_relaxed_b64(p1 + (k0 + k) * kTileCols) : 0ull;
            v[1][k] = ok1 ? ptx::ld_relaxed_b64(p1 + (k0 + k) * kTileCols + kHalfTile) : 0ull;
            v[2][k] = ok2 ? ptx::ld_relaxed_b64(p2 + (k0 + k) * kTileCols) : 0ull;
            v[3][k] = ok2 ? ptx::ld_relaxed_b64(p2 + (k0 + k) * kTileCols + kHalfTile) : 0ull;
            ok &= (!ok1 || (tag_ok(v[0][k], tag) & tag_ok(v[1][k], tag))) &&
                  (!ok2 || (tag_ok(v[2][k], tag) & tag_ok(v[3][k], tag)));
          }
          if (ok || retry_stop(t0, it)) break;
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
      xs[i] = swiglu(g1, u1) * kTwo64;
      if (two) xs[i + kCT] = swiglu(g2, u2) * kTwo64;
    }
  }
  C.bar();
  chunk = gemv_run<true>(DOWN, L, C.chunk);
  // this CTA's slice [c0, c1) of tile t: entry i = (slot i / nc, column c0 + i % nc)
  const int* D = plan() + kPlDown;
  const int t = D[0], c0 = D[1], ns = D[3], nc = D[2] - D[1];
  float* fin = C.scratch + kOffB;  // [ns][nc]
  const uint64_t* base = a.dn_part + (long long)t * a.slots[DOWN] * kTileCols + c0;
#pragma unroll 1
  for (int i = C.tid; i < ns * nc; i += kCT) fin[i] = ld_checked(base + (long long)(i / nc) * kTileCols + i % nc, tag);
  C.bar();
  if (C.tid < nc) {
    float d = 0.0f;
#pragma unroll 1
    for (int s = 0; s < ns; ++s) d = __fadd_rn(d, fin[s * nc + C.tid]);
    const int col = t * kTileCols + c0 + C.tid;
    if (a.tp > 1) {  // row-split down: sum the ranks' partials of this column
      tp_push(a, a.peer_d, L, col, d, tag);
      d = tp_sum(a.peer_d[a.rank], L, col, tag);
    }
    // x_{L+1} carries layer L+1's tag
    st_tagged(a.xbuf + (long long)(L + 1) * a.H + col, __fadd_rn(C.scratch[kOffFin + C.tid], d), tag + 1u);
  }
  C.bar();  // the slice table (B) is read before the next phase reuses it
  return chunk;
}

// ---- attention
// Scores of the 4 query heads (q in shared memory) against nr K rows at `rows`, written
// to sc[h * kMaxAttnChunk + idx0 + i] scaled by 1/sqrt(128). A row is taken by 8 lanes,
// each lane group NU rows per pass (rows 4w + g and, binary16, 60 later: a whole stage of
// 60 f32 or 120 binary16 rows in one pass, the q loads shared by the rows); lane li holds dims
// {4 li + 32 j + c} (j, c < 4), so the 8 lanes of a row read 128 contiguous bytes per load
// (conflict-free; the 4 rows of a warp fill the 4 wavefronts a 16-byte warp load needs)
// and q is a broadcast. The 4 heads accumulate in independent FMA chains. KV: float or
// __half rows.
template <class KV>
__device__ __noinline__ void score_rows(const KV* rows, int nr, int idx0) {
  const float* sq = sm_scratch() + kAttQ;
  float* sc = sm_scratch() + kAttS;
  const int lane = threadIdx.x & 31, li = lane & 7;
  const float scale = 0.08838834764831845f;  // 1/sqrt(128): the f32 quotient of 1 and f32 sqrt(128)
  constexpr int NU = sizeof(KV) == 4 ? 1 : 2;
  static_assert(kCW * 4 * NU == (sizeof(KV) == 4 ? kKVRows : kKVRows16), "one pass per stage");
#pragma unroll 1
  for (int rb = 0; rb < nr; rb += kCW * 4 * NU) {  // a whole stage per pass
    int ir[2];
    ir[0] = rb + (threadIdx.x >> 5) * 4 + (lane >> 3);
    ir[1] = ir[0] + kCW * 4;
    float kf[2][16];
#pragma unroll
    for (int u = 0; u < NU; ++u) {
      const KV* krow = rows + (long long)min(ir[u], nr - 1) * kHeadDim;
      if constexpr (sizeof(KV) == 4) {  // 4 x 16 bytes: dims 4 li + 32 j .. + 3
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 k4 = *reinterpret_cast<const float4*>(krow + 4 * li + 32 * j);
          kf[u][4 * j] = k4.x;
          kf[u][4 * j + 1] = k4.y;
          kf[u][4 * j + 2] = k4.z;
          kf[u][4 * j + 3] = k4.w;
        }
      } else {  // 2 x 16 bytes of halves: dims 8 li + 64 j .. + 7
#pragma unroll
        for (int j = 0; j < 2; ++j) {
          const uint4 raw = *reinterpret_cast<const uint4*>(krow + 8 * li + 64 * j);
          const uint32_t wv[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&wv[q]));
            kf[u][8 * j + 2 * q] = f.x;
            kf[u][8 * j + 2 * q + 1] = f.y;
          }
        }
      }
    }
    float d[2][kHeadsPerKV] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // the q dims matching kf[u][4j .. 4j+3]
      const int dim = sizeof(KV) == 4 ? 4 * li + 32 * j : 8 * li + 64 * (j >> 1) + 4 * (j & 1);
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h) {
        const float4 q4 = *reinterpret_cast<const float4*>(sq + h * kHeadDim + dim);
#pragma unroll
        for (int u = 0; u < NU; ++u) {
          d[u][h] = __fmaf_rn(q4.x, kf[u][4 * j], d[u][h]);
          d[u][h] = __fmaf_rn(q4.y, kf[u][4 * j + 1], d[u][h]);
          d[u][h] = __fmaf_rn(q4.z, kf[u][4 * j + 2], d[u][h]);
          d[u][h] = __fmaf_rn(q4.w, kf[u][4 * j + 3], d[u][h]);
        }
      }
    }
#pragma unroll
    for (int u = 0; u < NU; ++u)
#pragma unroll
      for (int h = 0; h < kHeadsPerKV; ++h) {
        float v = d[u][h];
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        v += __shfl_xor_sync(0xffffffffu, v, 4);
        if (ir[u] < nr && li == 0) sc[h * kMaxAttnChunk + idx0 + ir[u]] = __fmul_rn(v, scale);
      }
  }
}

// one cached V element as f32
QORA_DEV float kv_elem(const float* p) { return *p; }
QORA_DEV float kv_elem(const __half* p) { return __half2float(*p); }

// P.V over nr V rows at `rows` for the 4 heads, added to o: thread (grp, d) of three
// 128-thread groups takes blocks of 4 consecutive rows (block b to group b % 3), the
// block's four V loads in flight and its probabilities sc[h * kMaxAttnChunk + idx0 + i]
// read as one float4 per head. The accumulators travel in registers (argument and
// result).
template <class KV>
__device__ __noinline__ float4 pv_rows(const KV* rows, int nr, int idx0, int grp, int dd, float4 o) {
  const float* sc = sm_scratch() + kAttS + idx0;
  const KV* vr = rows + dd;
  // blocks of 4 consecutive rows, block b to group b % 3; a full block's probabilities
  // are one float4 per head (idx0 is a multiple of 4 for the streamed stages)
  int b = grp;
#pragma unroll 1
  for (; 4 * b + 3 < nr; b += 3) {
    const int i = 4 * b;
    float v[4];
#pragma unroll
    for (int r = 0; r < 4; ++r) v[r] = kv_elem(vr + (long long)(i + r) * kHeadDim);
    const float4 p0 = *reinterpret_cast<const float4*>(sc + i);
    const float4 p1 = *reinterpret_cast<const float4*>(sc + kMaxAttnChunk + i);
    const float4 p2 = *reinterpret_cast<const float4*>(sc + 2 * kMaxAttnChunk + i);
    const float4 p3 = *reinterpret_cast<const float4*>(sc + 3 * kMaxAttnChunk + i);
    o.x = __fmaf_rn(p0.x, v[0], o.x);
    o.y = __fmaf_rn(p1.x, v[0], o.y);
    o.z = __fmaf_rn(p2.x, v[0], o.z);
    o.w = __fmaf_rn(p3.x, v[0], o.w);
    o.x = __fmaf_rn(p0.y, v[1], o.x);
    o.y = __fmaf_rn(p1.y, v[1], o.y);
    o.z = __fmaf_rn(p2.y, v[1], o.z);
    o.w = __fmaf_rn(p3.y, v[1], o.w);
    o.x = __fmaf_rn(p0.z, v[2], o.x);
    o.y = __fmaf_rn(p1.z, v[2], o.y);
    o.z = __fmaf_rn(p2.z, v[2], o.z);
    o.w = __fmaf_rn(p3.z, v[2], o.w);
    o.x = __fmaf_rn(p0.w, v[3], o.x);
    o.y = __fmaf_rn(p1.w, v[3], o.y);
    o.z = __fmaf_rn(p2.w, v[3], o.z);
    o.w = __fmaf_rn(p3.w, v[3], o.w);
  }
  if (4 * b < nr) {  // the partial last block (also the new position's single row)
#pragma unroll 1
    for (int i = 4 * b; i < nr; ++i) {
      const float v = kv_elem(vr + (long long)i * kHeadDim);
      o.x = __fmaf_rn(sc[i], v, o.x);
      o.y = __fmaf_rn(sc[kMaxAttnChunk + i], v, o.y);
      o.z = __fmaf_rn(sc[2 * kMaxAttnChunk + i], v, o.z);
      o.w = __fmaf_rn(sc[3 * kMaxAttnChunk + i], v, o.w);
    }
  }
  return o;
}

// Attention merge of KV head g (nch chunks): this unit (chunk k) produces outputs
// [r0, r1) of the head's hpk * 128: per query head h, M = max_ch m, w_ch = exp(m_ch - M),
// l = sum_ch l_ch w_ch (chunk order), out = (sum_ch o_ch w_ch, chunk order) * (1 / l),
// published tagged for o_proj. Every unit of the head reads all chunks' partials of its
// slice directly: one L2 round trip once they are there, no arrival counter.
__device__ __noinline__ void attn_merge(int L, int g, int nch) {
  const Cons C = make_cons(0);
  const Args& a = C.a();
  const int nout = a.hpk * kHeadDim;
  const int* M = plan() + kPlMerge;
  const int r0 = M[0], nr = M[1] - M[0], h0 = M[2], nh = M[3];  // the slice and its heads
  const uint32_t tag = tag_of(C, L);
  float* so = C.scratch + kMgO;      // [nch][nr]
  float* sml = C.scratch + kMgML;    // [nch][nh][2]
  float* mw = C.scratch + kMgW;      // [nh][nch]
  float* invl = C.scratch + kMgInv;  // [nh]
  const int nml = nch * nh * 2;
#pragma unroll 1
  for (int i = C.tid; i < nml + nch * nr; i += kCT) {
    if (i < nml) {  // (m, l) of chunk ch, head h0 + (i % (2 nh)) / 2
      const int ch = i / (2 * nh), rest = i % (2 * nh);
      sml[i] = ld_checked(a.att_ml + ((long long)(ch * a.nkvh + g) * kHeadsPerKV + h0 + rest / 2) * 2 + (rest & 1), tag);
    } else {  // o of chunk ch, output r0 + r
      const int j = i - nml, ch = j / nr, r = j % nr;
      so[j] = ld_checked(a.att_o + (long long)(ch * a.nkvh + g) * kHeadsPerKV * kHeadDim + r0 + r, tag);
    }
  }
  C.bar();
  if (C.tid < nh) {
    const int h = C.tid;
    float mx = -INFINITY;
#pragma unroll 1
    for (int ch = 0; ch < nch; ++ch) mx = fmaxf(mx, sml[(ch * nh + h) * 2]);
    float l = 0.0f;
#pragma unroll 1
    for (int ch = 0; ch < nch; ++ch) {
      const float w = expf(sml[(ch * nh + h) * 2] - mx);
      mw[h * nch + ch] = w;
      l = __fmaf_rn(sml[(ch * nh + h) * 2 + 1], w, l);
    }
    invl[h] = __fdiv_rn(1.0f, l);
  }
  C.bar();
  if (C.tid < nr) {
    const int r = r0 + C.tid, h = r / kHeadDim - h0;
    float acc = 0.0f;
#pragma unroll 1
    for (int ch = 0; ch < nch; ++ch) acc = __fmaf_rn(so[ch * nr + C.tid], mw[h * nch + ch], acc);
    st_tagged(a.att_fin + (long long)g * nout + r, __fmul_rn(acc, invl[h]), tag);
  }
  C.bar();  // the staging (XS, B) is read until here; the next phase writes it at once
}

// ATTN: unit u = c = (kv head g = u % nkvh, chunk u / nkvh) for the hpk query heads of g
// (src/gemv.rs:914-989, softmax_raw :782-793; RoPE src/gemv.rs:757-778). KV is float
// (the reference's f32 cache) or __half (the opt-in binary16 cache: the new k and v are
// rounded to nearest-even as they enter the cache, and the new position's score and P.V
// use the rounded values, exactly as if they were read back from it). The new
// position's k and v rows are kept in shared memory in the cache's element type, so the
// same routines score and weigh them as the cached rows streamed through the ring.
template <class KV>
__device__ __noinline__ uint32_t attention_phase_t(int L, uint32_t chunk) {
  constexpr int kRows = sizeof(KV) == 2 ? kKVRows16 : kKVRows;
  Cons C = make_cons(chunk);
  const Args& a = C.a();
  const int pos = C.pos, tid = C.tid;
  const int* P = plan() + kPlAtt;
  if (!P[0]) return chunk;
  const int g = P[1], kch = P[2], s0 = P[3], n = P[4] - P[3], sc1 = P[5], nch = P[6];
  const int u = kch * a.nkvh + g;
  const bool has_pos = P[7] != 0;
  const Layer& ly = a.layers[L];
  float* sq = C.scratch + kAttQ;
  float* sc = C.scratch + kAttS;
  float* sml = C.scratch + kAttML;
  float* sinv = C.scratch + kAttInv;
  KV* skv = reinterpret_cast<KV*>(C.scratch + kAttKV);  // [k row | v row]
  const int hpk = a.hpk;
  const uint32_t tag = tag_of(C, L);
  // RoPE pairs (d, d+64): threads 0..64*hpk-1 the query heads of g, 256..319 k (new
  // position's chunk only); 320..447 copy v
  if (tid < 64 * hpk || (has_pos && tid >= 256 && tid < 448)) {
    const bool isv = tid >= 320, isk = tid >= 256 && !isv;
    const int hh = (tid >> 6) & 3, d = isv ? tid - 320 : tid & 63;
    const bool rot = ly.rope && !isv;
    float cs = 1.0f, sn = 0.0f;
    if (rot) {  // the tables do not depend on this step's activations: read before the wait
      cs = __ldg(a.cos_t + (long long)pos * kHalfDim + d);
      sn = __ldg(a.sin_t + (long long)pos * kHalfDim + d);
    }
    const uint64_t* src = (isv ? a.qkv + a.nq + a.nkvw + g * kHeadDim
                               : isk ? a.qkv + a.nq + g * kHeadDim : a.qkv + (g * hpk + hh) * kHeadDim) + d;
    uint64_t w1, w2, t0 = 0;
#pragma unroll 1
    for (int it = 0;; ++it) {
      w1 = ptx::ld_relaxed_b64(src);
      w2 = ptx::ld_relaxed_b64(src + (isv ? 0 : kHalfDim));
      if ((tag_ok(w1, tag) & tag_ok(w2, tag)) || retry_stop(t0, it)) break;
    }
    float x1 = tag_val(w1), x2 = tag_val(w2);
    if (rot) {  // split-half rotation with the table row of this position
      const float y1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
      x2 = __fadd_rn(__fmul_rn(x2, cs), __fmul_rn(x1, sn));
      x1 = y1;
    }
    if (!isk && !isv) {
      sq[hh * kHeadDim + d] = x1;
      sq[hh * kHeadDim + d + kHalfDim] = x2;
    } else {  // append to the cache and keep the row (as stored) for this step
      KV* cache = reinterpret_cast<KV*>(isv ? ly.vc : ly.kc) + g * a.head_stride + (long long)pos * kHeadDim;
      KV* row = skv + (isv ? kHeadDim : 0);
      const KV e1 = (KV)x1;  // binary16: round to nearest even
      row[d] = e1;
      cache[d] = e1;
      if (!isv) {
        const KV e2 = (KV)x2;
        row[d + kHalfDim] = e2;
        cache[d + kHalfDim] = e2;
      }
    }
  }
  C.bar();
  // scores of the cached rows (streamed through the ring), then of the new position
#pragma unroll 1
  for (int s = s0; s < sc1; s += kRows) {
    const uint8_t* stg = C.acquire_stage();
    if (C.stage_ok) score_rows<KV>(reinterpret_cast<const KV*>(stg), min(kRows, sc1 - s), s - s0);
    C.release_stage();
  }
  if (has_pos && C.warp == 0 && !C.aborted_w()) score_rows<KV>(skv, 1, pos - s0);
  C.bar();
  // chunk softmax numerators, one warp per query head
  if (C.warp < hpk && !C.aborted_w()) {
    float* row = sc + C.warp * kMaxAttnChunk;
    float mx = -INFINITY;
#pragma unroll 1
    for (int i = C.lane; i < n; i += 32) mx = fmaxf(mx, row[i]);
    mx = warp_max(mx);
    float l = 0.0f;
#pragma unroll 1
    for (int i = C.lane; i < n; i += 32) {
      const float e = expf(row[i] - mx);
      row[i] = e;
      l += e;
    }
    l = warp_sum(l);
    if (C.lane == 0) {
      sml[C.warp * 2] = mx;
      sml[C.warp * 2 + 1] = l;
      sinv[C.warp] = __fdiv_rn(1.0f, l);
    }
  }
  C.bar();
  // P.V: three groups of 128 threads; thread d of a group accumulates dim d of the 4
  // heads over its rows; the groups' sums are added in group order
  const int grp = tid >> 7, dd = tid & (kHeadDim - 1);
  float4 o = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
#pragma unroll 1
  for (int s = s0; s < sc1; s += kRows) {
    const uint8_t* stg = C.acquire_stage();
    if (C.stage_ok && grp < 3) o = pv_rows<KV>(reinterpret_cast<const KV*>(stg), min(kRows, sc1 - s), s - s0, grp, dd, o);
    C.release_stage();
  }
  if (has_pos && grp == 0) o = pv_rows<KV>(skv + kHeadDim, 1, pos - s0, 0, dd, o);
  C.bar();  // every read of the probabilities is done: groups 1 and 2 park their sums there
  if ((grp == 1 || grp == 2) && !C.aborted()) {
    float* park = sc + (grp - 1) * kHeadsPerKV * kHeadDim + dd;
    park[0] = o.x;
    park[kHeadDim] = o.y;
    park[2 * kHeadDim] = o.z;
    park[3 * kHeadDim] = o.w;
  }
  C.bar();
  if (tid < kHeadDim && !C.aborted()) {
    const float ov[kHeadsPerKV] = {o.x, o.y, o.z, o.w};
#pragma unroll
    for (int h = 0; h < kHeadsPerKV; ++h) {
      if (h >= hpk) break;
      const float oh = __fadd_rn(__fadd_rn(ov[h], sc[h * kHeadDim + tid]), sc[kHeadsPerKV * kHeadDim + h * kHeadDim + tid]);
      if (nch == 1)  // the whole context: publish o / l (exp(m - max) = 1 for the one chunk)
        st_tagged(a.att_fin + (long long)(g * hpk + h) * kHeadDim + tid, __fmul_rn(oh, sinv[h]), tag);
      else
        st_tagged(a.att_o + ((long long)u * kHeadsPerKV + h) * kHeadDim + tid, oh, tag);
    }
    if (nch > 1 && tid < 2 * hpk) st_tagged(a.att_ml + (long long)u * 2 * kHeadsPerKV + tid, sml[tid], tag);
  }
  const bool ab = C.bar_aborted();  // the merge's barriers: every thread decides alike
  if (nch > 1 && !ab) attn_merge(L, g, nch);
  return C.chunk;
}

__device__ __forceinline__ uint32_t attention_phase(int L, uint32_t chunk) {
  return sm_args()->kv16 ? attention_phase_t<__half>(L, chunk) : attention_phase_t<float>(L, chunk);
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
  const float ss = poll_vec(a.xbuf + (long long)a.L * H, H, tag_of(C, a.L), sB, 1.0f);
  csum_put(ss);
  C.bar();
  C.stamp(2 + 8 * kTraceLayers);
  const float inv = rms_inv_from(csum_get(), H);
  // normed x into a padded copy (element i at i + i / 64: the 64-element block of lane l
  // starts at bank l, so the lanes' loads below do not conflict)
  float* sX = C.scratch;  // XS and the start of B (x is read into registers first)
  constexpr int kPer = (kXsCap + kCT - 1) / kCT;
  float xn[kPer];
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = C.tid + j * kCT;
    xn[j] = i < H ? __fmul_rn(__fmul_rn(sB[i], inv), a.final_gamma[i]) : 0.0f;
  }
  C.bar();
#pragma unroll
  for (int j = 0; j < kPer; ++j) {
    const int i = C.tid + j * kCT;
    if (i < H) sX[i + (i >> 6)] = xn[j];
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
      const int xi = lane * EPL + g * 32 + e;
      const float v = sX[xi + (xi >> 6)];
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
  __syncthreads();  // the shared copy of the arguments is complete
  const Args& a = *sa;
  {  // split-K slots per tile of gate/up, then down; this CTA's plan for the launch (built
     // from the shared copy: the parameter struct itself is never addressed)
    int* tab = reinterpret_cast<int*>(scratch + kOffTab);
    for (int t = tid; t < a.tiles[GU]; t += kThreads) tab[t] = nslots(a, GU, t);
    for (int t = tid; t < a.tiles[DOWN]; t += kThreads) tab[a.tiles[GU] + t] = nslots(a, DOWN, t);
    if (warp < 4 && lane == 0) make_mat_plan(a, warp, c);
    if (warp == 4 && lane == 0) make_att_plan(a, c, G, flags[2]);
  }
  __syncthreads();  // last block-wide barrier: the producer warp leaves below
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
          if ((tag_ok(wv, tag) & tag_ok(wi, tag)) || retry_stop(t0, it)) break;
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
