// qora_engine.cu — libqora_cuda.so: the C ABI of include/qora_cuda.h over the sm_100a
// kernels (q4_gemv.cuh, attention.cuh, lm_head.cuh, small_kernels.cuh).
//
// Device layout (HBM), per engine:
//   per layer   q|k|v fused Q4 matrix, o, gate/up fused (interleaved per 128 outputs) and
//               down, each re-tiled "tile-major": for column tile t (8 groups = 256
//               outputs) and row r, 144 contiguous bytes = 8 x 16 packed bytes followed
//               by the 8 f16 scales. A tile is one contiguous stream of K*144 bytes.
//               Dequantised values are unchanged (same nibbles, same f16 scales).
//               Norm gains as f32 (exact widening of the f16 values).
//   embedding   Q4 [vocab][hidden] as in the file (row-dot lm_head + row lookup).
//   RoPE tables f32 [rows][64] as in the file.
//   KV cache    per layer f32 [max_seq][kv_heads*128] (token-major like RawKvCache).
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

#include <cudaTypedefs.h>

#include "../../include/qora_cuda.h"
#include "attention.cuh"
#include "common.cuh"
#include "f16_batch.cuh"
#include "lm_head.cuh"
#include "umma_gemm.cuh"
#include "megakernel.cuh"
#include "q4_gemv.cuh"
#include "q4_gemv_tma.cuh"
#include "sampling.cuh"
#include "small_kernels.cuh"

using namespace qora;

namespace {

thread_local std::string g_last_error;

qora_status fail(qora_status st, const char* fmt, ...) {
  char buf[1024];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

#define QCUDA(call)                                                                   \
  do {                                                                                \
    cudaError_t e_ = (call);                                                          \
    if (e_ != cudaSuccess)                                                            \
      return fail(e_ == cudaErrorMemoryAllocation ? QORA_ERR_OOM : QORA_ERR_CUDA,     \
                  "%s failed: %s (%s:%d)", #call, cudaGetErrorString(e_), __FILE__, __LINE__); \
  } while (0)

#define QCHECK(expr)                 \
  do {                               \
    qora_status s_ = (expr);         \
    if (s_ != QORA_OK) return s_;    \
  } while (0)

int sm_count(int dev) {
  int n = 0;
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

// ------------------------------------------------------------------ GEMV planning
struct GemvShape {
  int K = 0, tiles = 0;
  SplitPlan plan{};
  int seg_cap = 0;  // floats of dynamic shared memory
};

GemvShape plan_gemv(int K, int tiles, int ctas_wanted) {
  GemvShape s;
  s.K = K;
  s.tiles = tiles;
  const long long total = (long long)tiles * K;
  const int ctas = (int)std::min<long long>(ctas_wanted, total);
  s.plan.ctas = ctas;
  s.plan.total = total;
  auto owner = [&](long long p) { return (int)(((p + 1) * (long long)ctas - 1) / total); };
  int mx = 1;
  for (int t = 0; t < tiles; ++t)
    mx = std::max(mx, owner((long long)(t + 1) * K - 1) - owner((long long)t * K) + 1);
  s.plan.max_slots = mx;
  s.seg_cap = (int)((total + ctas - 1) / ctas) + 1;
  return s;
}

size_t partial_floats(const GemvShape& s) {
  return (size_t)s.tiles * s.plan.max_slots * kTileCols;
}

template <class Pro, class Epi>
qora_status launch_gemv(const Q4Src& src, const GemvShape& sh, float* partials, unsigned* counters,
                        const Pro& pro, const Epi& epi, cudaStream_t stream) {
  SplitPlan plan = sh.plan;
  plan.partials = partials;
  plan.counters = counters;
  const size_t smem = (size_t)sh.seg_cap * sizeof(float);
  auto kern = q4_gemv_kernel<Pro, Epi>;
  if (smem > 48 * 1024) {
    if (smem > 200 * 1024) return fail(QORA_ERR_INVALID, "GEMV segment too long (%zu B)", smem);
    QCUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  }
  kern<<<plan.ctas, kGemvThreads, smem, stream>>>(src, plan, pro, epi);
  QCUDA(cudaGetLastError());
  return QORA_OK;
}

// ------------------------------------------------------------------ host-side re-tiling
struct GroupRef {
  const qora_matrix_view* m;  // nullptr: zero padding
  int g;
};

// Tile-major Q4 bytes for fused group list `refs` (all sources share K rows). tg == 8:
// tiles of 8 groups, each 144-byte tile row = 8 groups' 16 nibble bytes then their 8
// f16 scales. tg == 1: one group per tile, stored as 144-byte blocks of 8 consecutive
// rows (8 x 16 nibble bytes, then the 8 rows' scales; K % 8 == 0), which keeps every
// 16-byte row load aligned. Either way a tile row costs 18 bytes per group.
std::vector<uint8_t> build_tiled(int K, const std::vector<GroupRef>& refs, int tg = kTileGroups,
                                 int row0 = 0) {
  const int G = (int)refs.size();
  const int tiles = (G + tg - 1) / tg;
  std::vector<uint8_t> buf((size_t)tiles * K * tg * 18, 0);
  for (int r = 0; r < K; ++r) {
    for (int f = 0; f < tiles * tg; ++f) {
      const int t = f / tg, gi = f % tg;
      uint8_t* blk;  // 144-byte block holding this (group, row)
      int slot;      // 16-byte slot within the block
      if (tg == 1) {
        blk = buf.data() + ((size_t)t * K + (r & ~7)) * 18;
        slot = r & 7;
      } else {
        blk = buf.data() + ((size_t)t * K + r) * kTiledRowBytes;
        slot = gi;
      }
      if (f >= G || refs[f].m == nullptr) continue;  // zeros: scale 0 -> contributes 0
      const qora_matrix_view* m = refs[f].m;
      const size_t gpr = m->n / kGroup;
      const size_t sr = (size_t)(row0 + r);  // source row (row-split shards start at row0)
      std::memcpy(blk + slot * 16, m->packed + (sr * gpr + refs[f].g) * 16, 16);
      std::memcpy(blk + 128 + slot * 2, m->scales + sr * gpr + refs[f].g, 2);
    }
  }
  return buf;
}

struct DevQ4 {
  uint8_t* buf = nullptr;
  int K = 0, G = 0, tiles = 0;
  Q4Src src() const {
    Q4Src s{};
    s.p[0] = s.p[1] = buf;
    s.s[0] = s.s[1] = buf + kTileGroups * 16;
    s.tile_stride_p = s.tile_stride_s = (long long)K * kTiledRowBytes;
    s.row_stride_p = s.row_stride_s = kTiledRowBytes;
    s.split = 0;
    s.K = K;
    s.G = G;
    s.tiles = tiles;
    return s;
  }
};

// Q4Src over the reference F1 layout (packed [K][n/2], scales [K][n/32]) on the device.
Q4Src f1_src(const uint8_t* packed, const uint16_t* scales, int K, int n) {
  Q4Src s{};
  const int G = n / kGroup;
  s.p[0] = s.p[1] = packed;
  s.s[0] = s.s[1] = reinterpret_cast<const uint8_t*>(scales);
  s.tile_stride_p = kTileGroups * 16;
  s.tile_stride_s = kTileGroups * 2;
  s.row_stride_p = (long long)G * 16;
  s.row_stride_s = (long long)G * 2;
  s.split = 0;
  s.K = K;
  s.G = G;
  s.tiles = (G + kTileGroups - 1) / kTileGroups;
  return s;
}

// gate/up given as two F1 matrices: tile t = gate groups 4t..4t+3 | up groups 4t..4t+3.
Q4Src f1_pair_src(const uint8_t* gp, const uint16_t* gs, const uint8_t* upk, const uint16_t* us,
                  int K, int n) {
  Q4Src s{};
  const int G = n / kGroup;
  s.p[0] = gp;
  s.p[1] = upk;
  s.s[0] = reinterpret_cast<const uint8_t*>(gs);
  s.s[1] = reinterpret_cast<const uint8_t*>(us);
  s.tile_stride_p = (kTileGroups / 2) * 16;
  s.tile_stride_s = (kTileGroups / 2) * 2;
  s.row_stride_p = (long long)G * 16;
  s.row_stride_s = (long long)G * 2;
  s.split = kTileGroups / 2;
  s.K = K;
  s.G = G;
  s.tiles = (G + kTileGroups / 2 - 1) / (kTileGroups / 2);
  return s;
}

std::vector<float> f16_to_f32(const uint16_t* h, size_t n) {
  std::vector<float> out(n);
  for (size_t i = 0; i < n; ++i) {
    __half_raw r;
    r.x = h[i];
    out[i] = __half2float(__half(r));
  }
  return out;
}

struct LayerDev {
  DevQ4 qkv, o, gu, down;
  DevQ4 qkv1, o1;  // one-group tiles of q|k|v and o_proj for the persistent kernel
  float* g_in = nullptr;
  float* g_post = nullptr;
  int rope = 0;
  int nq = 0, nkv = 0;
};

// F16 weights (format 0) for the batched path, re-tiled for the tensor cores
// (umma_gemm.cuh: [N/128 tiles][K/64 chunks][16 KB]); q|k|v and gate|up are joined
// along n so one GEMM serves each group. Values are the file's f16 bits, unchanged.
struct F16Layer {
  uint8_t* wqkv = nullptr;   // n = nq + 2 nkv*128, k = hidden
  uint8_t* wo = nullptr;     // n = hidden, k = nq
  uint8_t* wgu = nullptr;    // n = 2 I (gate channels then up channels), k = hidden
  uint8_t* wdown = nullptr;  // n = hidden, k = I
  float* g_in = nullptr;
  float* g_post = nullptr;
  float gmax_in = 0.0f, gmax_post = 0.0f;  // max |gamma| (operand row-scale bounds)
  int rope = 0;
};

}  // namespace

// ================================================================== engine / kv objects
struct qora_engine {
  int device = 0;
  int sms = 148;
  cudaStream_t stream = nullptr;
  uint32_t format = QORA_FORMAT_Q4;
  uint32_t num_layers = 0, vocab = 0, hidden = 0, inter = 0;
  uint32_t nh = 0, nkv = 0, rope_rows = 0;  // nkv: KV heads this engine's caches hold
  uint32_t nkv_total = 0;                    // KV heads of the model
  // tensor parallelism: this engine is rank `rank` of `tp` (1 = whole model)
  int tp = 1, rank = 0;
  int nh_l = 0, nkv_l = 0, kv0 = 0, inter_l = 0;  // local q heads, kv heads, first kv head, MLP width
  uint8_t* tp_region = nullptr;                   // receive buffers peers write into (IPC-exported)
  size_t tp_region_bytes = 0, tp_off_d = 0, tp_off_lm = 0, tp_off_logits = 0;
  uint8_t* tp_peer[8] = {};                       // every rank's region (own included), after connect
  bool tp_connected = false;
  std::vector<void*> tp_opened;                   // IPC mappings to close
  std::vector<LayerDev> layers;
  // F16 weights: batched per-op path (f16_batch.cuh). Q4 weights: the same path serves
  // the prompt pass, its projections held again as Q4 chunks of the dequantising GEMM
  std::vector<F16Layer> fl;
  bool want_q4p = true;            // not disabled by QORA_FLAG_TOKEN_PREFILL
  bool q4p = false;                // Q4 prompt pass on the tensor cores available
  std::string q4p_why;             // why not
  uint8_t* f_lm = nullptr;         // tiled embedding (n = vocab, k = hidden): lookup + tied lm_head
  int f_nqkv = 0;                  // q|k|v columns
  float *f_x = nullptr, *f_qkv = nullptr, *f_attn = nullptr, *f_h = nullptr;  // [rows][...]
  float *f_logits = nullptr, *f_part = nullptr;
  size_t f_part_floats = 0;
  uint8_t* f_xt = nullptr;         // GEMM operand: activations as tiled f16 hi | lo rows
  float *f_xss = nullptr, *f_xmx = nullptr;  // statistics of f_x rows [hidden/128][128]
  float* f_hmx = nullptr;          // max |h| [I/64][128]
  float* f_amx = nullptr;          // max |attention out| [kv heads][128]
  float *f_att_part = nullptr, *f_att_ml = nullptr;  // split attention chunk partials
  unsigned* f_att_cnt = nullptr;
  unsigned* f_tcnt = nullptr;      // per-tile arrival counters of the fused GEMMs
  unsigned* f_sync = nullptr;      // grid barrier + finished-tile counter
  unsigned long long* f_amkey = nullptr;  // [128] greedy argmax keys
  float f_gmax_final = 0.0f;
  int f_it = 0;                    // gate/up channels of this rank (before padding to inter_l)
  int f_vt0 = 0, f_vt1 = 0;        // this rank's lm_head vocab tiles [f_vt0, f_vt1)
  unsigned* f_epoch = nullptr;     // forward passes (tensor-parallel exchange tags)
  int* f_err = nullptr;            // set by a GEMM whose bounded wait timed out
  // on-device sampling scratch (allocated on first use)
  float* smp_work = nullptr;       // [vocab] penalised logits
  unsigned* smp_hist = nullptr;    // history tokens
  size_t smp_hist_cap = 0;
  smp::Out* smp_out = nullptr;
  smp::Out* smp_out_host = nullptr;  // pinned
  uint8_t* lm_table = nullptr;   // embedding rows: hidden/2 packed bytes | hidden/32 f16 scales
  long long lm_row_bytes = 0;
  float* final_gamma = nullptr;
  float* rope_cos = nullptr;
  float* rope_sin = nullptr;
  // activations
  float *x = nullptr, *q = nullptr, *attn = nullptr, *h = nullptr, *logits = nullptr;
  // GEMV scratch
  GemvShape sh_qkv, sh_o, sh_gu, sh_down;
  float* partials = nullptr;
  unsigned* counters = nullptr;
  int max_tiles = 0;
  // lm_head scratch
  int lm_ctas = 0;
  float* lm_part_v = nullptr;
  unsigned* lm_part_i = nullptr;
  unsigned* lm_counter = nullptr;
  // persistent decode megakernel (shared buffers; per-cache parts live in qora_kv)
  bool mk_ok = false;
  std::string mk_why;
  int mk_G = 0;
  int mk_slots[4] = {0, 0, 0, 0};
  int mk_sub0[4] = {0, 0, 0, 0}, mk_subn[4] = {0, 0, 0, 0};
  uint32_t mk_max_seq = 0;
  uint64_t* mk_xmid = nullptr;  // tagged hand-off buffers: (tag << 32) | f32 bits
  uint64_t* mk_qkv = nullptr;
  uint64_t* mk_gu_part = nullptr;
  uint64_t* mk_dn_part = nullptr;  // tagged
  unsigned* mk_epoch = nullptr;
  int mk_cpl = 0, mk_ncnt = 0;
  uint64_t* mk_xbuf = nullptr;
  unsigned* mk_cnt = nullptr;
  float* mk_lm_v = nullptr;
  unsigned* mk_lm_i = nullptr;
  unsigned long long* mk_trace = nullptr;
  size_t mk_trace_n = 0;
  bool use_mega = true;
  std::vector<void*> allocs;
  uint64_t device_bytes = 0;
  std::vector<qora_kv*> kvs;  // live caches; detached (device state freed) on destroy

  template <typename T>
  qora_status alloc(T** p, size_t count) {
    void* d = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t e = cudaMalloc(&d, bytes);
    if (e != cudaSuccess)
      return fail(QORA_ERR_OOM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(e));
    allocs.push_back(d);
    device_bytes += bytes;
    *p = static_cast<T*>(d);
    return QORA_OK;
  }
  ~qora_engine();
};

struct qora_kv {
  qora_engine* e = nullptr;
  uint32_t max_seq = 0;
  uint32_t batch = 1;  // independent sequences
  uint32_t dtype = QORA_KV_F32;
  float* k = nullptr;  // [layers][batch][nkv][max_seq][128] f32, or binary16 (QORA_KV_F16)
  float* v = nullptr;
  std::vector<uint32_t> len;  // [batch][layers] positions filled
  int* rows = nullptr;        // F16 path: row table (f16b::RowInfo)
  int* rows_host = nullptr;   // pinned staging of the row table
  unsigned* f_argmax = nullptr;  // [batch]
  cudaGraphExec_t f_graph = nullptr;  // one batched F16 decode step
  StepState* st = nullptr;
  StepState* st_host = nullptr;  // pinned staging
  unsigned* ring = nullptr;      // greedy output ring [max_seq]
  uint32_t* ids = nullptr;       // prefill ids [max_seq]
  int attn_nc = 0;
  float* attn_o = nullptr;
  float* attn_ml = nullptr;
  unsigned* attn_counters = nullptr;
  cudaGraphExec_t graph = nullptr;
  bool mk_ready = false;
  mk::Args mk_args{};
  mk::Layer* mk_layers = nullptr;
  uint64_t* mk_att_o = nullptr;  // tagged
  uint64_t* mk_att_ml = nullptr;
  uint64_t* mk_att_fin = nullptr;  // tagged merged attention output [nh][128]
  std::vector<void*> allocs;
  // free the device-side state (the engine's stream must be idle or synchronised)
  void release_device() {
    if (graph) cudaGraphExecDestroy(graph);
    graph = nullptr;
    if (f_graph) cudaGraphExecDestroy(f_graph);
    f_graph = nullptr;
    if (rows_host) cudaFreeHost(rows_host);
    rows_host = nullptr;
    for (void* p : allocs) cudaFree(p);
    allocs.clear();
    if (st_host) cudaFreeHost(st_host);
    st_host = nullptr;
  }
  ~qora_kv() {
    if (e) {
      cudaSetDevice(e->device);
      cudaStreamSynchronize(e->stream);
      auto& v = e->kvs;
      v.erase(std::remove(v.begin(), v.end(), this), v.end());
    }
    release_device();
  }
  template <typename T>
  qora_status alloc(T** p, size_t count) {
    void* d = nullptr;
    const size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    cudaError_t err = cudaMalloc(&d, bytes);
    if (err != cudaSuccess)
      return fail(QORA_ERR_OOM, "cudaMalloc(%zu) failed: %s", bytes, cudaGetErrorString(err));
    allocs.push_back(d);
    *p = static_cast<T*>(d);
    return QORA_OK;
  }
  size_t seq_stride() const { return (size_t)max_seq * e->nkv * kHeadDim; }  // elements
  size_t layer_stride() const { return batch * seq_stride(); }
  size_t esz() const { return dtype == QORA_KV_F16 ? 2 : 4; }
  // base of layer li's keys (values) in the cache's element type
  void* k_layer(size_t li) const { return reinterpret_cast<uint8_t*>(k) + li * layer_stride() * esz(); }
  void* v_layer(size_t li) const { return reinterpret_cast<uint8_t*>(v) + li * layer_stride() * esz(); }
  uint32_t& lenof(uint32_t seq, uint32_t layer) { return len[(size_t)seq * (len.size() / batch) + layer]; }
};

qora_engine::~qora_engine() {
  if (stream) cudaStreamSynchronize(stream);
  for (qora_kv* kv : kvs) {  // caches outliving their engine become inert shells
    kv->release_device();
    kv->e = nullptr;
  }
  kvs.clear();
  if (!tp_opened.empty()) cudaSetDevice(device);
  for (void* p : tp_opened) cudaIpcCloseMemHandle(p);
  if (smp_out_host) cudaFreeHost(smp_out_host);
  for (void* p : allocs) cudaFree(p);
  if (stream) cudaStreamDestroy(stream);
}

namespace {

qora_status validate_view(const qora_weights_view* w) {
  if (!w) return fail(QORA_ERR_INVALID, "weights view is NULL");
  if (w->format != QORA_FORMAT_Q4 && w->format != QORA_FORMAT_F16)
    return fail(QORA_ERR_INVALID, "unknown format %u", w->format);
  const bool q4 = w->format == QORA_FORMAT_Q4;
  auto present = [q4](const qora_matrix_view& m) { return q4 ? (m.packed && m.scales) : m.data != nullptr; };
  if (w->num_layers == 0 || !w->layers) return fail(QORA_ERR_INVALID, "no layers");
  if (w->hidden == 0 || w->hidden % 1024 != 0 || w->hidden > 4096)
    return fail(QORA_ERR_UNSUPPORTED, "hidden=%u must be a multiple of 1024 up to 4096", w->hidden);
  if (w->rope_half_dim != kHalfDim)
    return fail(QORA_ERR_UNSUPPORTED, "rope_half_dim=%u, only 64 supported", w->rope_half_dim);
  if (w->vocab == 0 || w->vocab > (1u << 24)) return fail(QORA_ERR_UNSUPPORTED, "vocab %u (1 .. 2^24)", w->vocab);
  if (w->num_layers > 4096) return fail(QORA_ERR_UNSUPPORTED, "num_layers %u", w->num_layers);
  if (w->embed.k != w->vocab || w->embed.n != w->hidden || !present(w->embed))
    return fail(QORA_ERR_INVALID, "embedding must be [vocab][hidden] in the model's format");
  if (!q4 && w->vocab % 128 != 0)
    return fail(QORA_ERR_UNSUPPORTED, "F16 weights: vocab %u must be a multiple of 128", w->vocab);
  if (!w->final_norm_gamma || !w->no_rope_layers || !w->rope_cos || !w->rope_sin)
    return fail(QORA_ERR_INVALID, "missing final norm / rope tables / no_rope_layers");
  const qora_layer_view& L0 = w->layers[0];
  for (uint32_t i = 0; i < w->num_layers; ++i) {
    const qora_layer_view& L = w->layers[i];
    if (L.head_dim != kHeadDim) return fail(QORA_ERR_UNSUPPORTED, "layer %u head_dim=%u", i, L.head_dim);
    if (L.num_kv_heads == 0 || L.num_heads != L.num_kv_heads * kGrp || L.num_kv_groups != kGrp)
      return fail(QORA_ERR_UNSUPPORTED, "layer %u: heads %u/%u groups %u (need 4 query heads per KV head)",
                  i, L.num_heads, L.num_kv_heads, L.num_kv_groups);
    if (L.num_heads != L0.num_heads || L.num_kv_heads != L0.num_kv_heads || L.gate_proj.n != L0.gate_proj.n)
      return fail(QORA_ERR_UNSUPPORTED, "layer %u geometry differs from layer 0", i);
    const uint64_t H = w->hidden, nq = (uint64_t)L.num_heads * kHeadDim, nk = (uint64_t)L.num_kv_heads * kHeadDim;
    const uint64_t I = L.gate_proj.n;
    struct { const qora_matrix_view* m; uint64_t k, n; const char* name; } want[7] = {
        {&L.q_proj, H, nq, "q_proj"}, {&L.k_proj, H, nk, "k_proj"}, {&L.v_proj, H, nk, "v_proj"},
        {&L.o_proj, nq, H, "o_proj"}, {&L.gate_proj, H, I, "gate_proj"}, {&L.up_proj, H, I, "up_proj"},
        {&L.down_proj, I, H, "down_proj"}};
    for (auto& wm : want) {
      if (wm.m->k != wm.k || wm.m->n != wm.n || !present(*wm.m))
        return fail(QORA_ERR_INVALID, "layer %u %s: shape %llux%llu, expected %llux%llu (%s)", i, wm.name,
                    (unsigned long long)wm.m->k, (unsigned long long)wm.m->n,
                    (unsigned long long)wm.k, (unsigned long long)wm.n, q4 ? "Q4" : "F16");
    }
    if (I % 128 != 0 || I == 0 || I > (1u << 20))
      return fail(QORA_ERR_UNSUPPORTED, "intermediate %llu not a multiple of 128 up to 2^20", (unsigned long long)I);
    if (!L.input_norm_gamma || !L.post_attn_norm_gamma) return fail(QORA_ERR_INVALID, "layer %u norms missing", i);
  }
  return QORA_OK;
}

// The tensor-parallel shard of rank r of T (both formats): q heads split evenly; KV heads
// split while they divide, else each rank keeps the KV head its q heads use; gate/up
// columns and down rows [r*I/T, +I/T) (F16: padded to whole 64-channel tile halves);
// lm_head rows split evenly (F16: by 128-row tiles).
qora_status tp_plan(uint32_t format, uint32_t nh, uint32_t nkvh, uint32_t I, uint32_t V, int T, int r,
                    qora_tp_shard* o) {
  if (T != 1 && T != 2 && T != 4 && T != 8) return fail(QORA_ERR_INVALID, "tp_size %d (1, 2, 4 or 8)", T);
  if (r < 0 || r >= T) return fail(QORA_ERR_INVALID, "tp_rank %d of %d", r, T);
  if (nh == 0 || nkvh == 0 || nh % T != 0 || (nkvh % T != 0 && T % nkvh != 0))
    return fail(QORA_ERR_UNSUPPORTED, "tp_size %d does not divide heads %u/%u", T, nh, nkvh);
  o->q_heads = nh / T;
  o->q_head0 = r * o->q_heads;
  o->kv_heads = nkvh % T == 0 ? nkvh / T : 1;
  o->kv_head0 = nkvh % T == 0 ? r * o->kv_heads : r / (T / nkvh);
  if (o->q_heads % o->kv_heads != 0 || o->q_heads / o->kv_heads > (uint32_t)kGrp)
    return fail(QORA_ERR_UNSUPPORTED, "tp_size %d: %u query heads over %u kv heads per rank", T, o->q_heads,
                o->kv_heads);
  if (format == QORA_FORMAT_Q4) {
    if ((I / kGroup) % T != 0)
      return fail(QORA_ERR_UNSUPPORTED, "tp_size %d does not divide the %u MLP groups", T, I / kGroup);
    o->mlp_n = I / T;
    o->mlp_padded = o->mlp_n;
    o->vocab0 = (uint32_t)((uint64_t)r * V / T);
    o->vocab_n = (uint32_t)((uint64_t)(r + 1) * V / T) - o->vocab0;
  } else {
    if (I % T != 0 || (I / T) % 8 != 0)
      return fail(QORA_ERR_UNSUPPORTED, "tp_size %d does not divide the MLP width %u in multiples of 8", T, I);
    o->mlp_n = I / T;
    o->mlp_padded = (o->mlp_n + 63) / 64 * 64;
    const uint32_t vt = V / 128;
    o->vocab0 = (uint32_t)((uint64_t)r * vt / T) * 128;
    o->vocab_n = (uint32_t)((uint64_t)(r + 1) * vt / T) * 128 - o->vocab0;
  }
  o->mlp0 = r * o->mlp_n;
  return QORA_OK;
}

qora_status upload(qora_engine* /*e*/, void* dst, const void* src, size_t bytes) {
  QCUDA(cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice));
  return QORA_OK;
}

qora_status upload_q4(qora_engine* e, int K, const std::vector<GroupRef>& refs, DevQ4& out,
                      int tg = kTileGroups, int row0 = 0) {
  if (tg != kTileGroups && (tg != 1 || K % 8 != 0)) return fail(QORA_ERR_UNSUPPORTED, "tile shape");
  out.K = K;
  out.G = (int)refs.size();
  out.tiles = (out.G + tg - 1) / tg;
  std::vector<uint8_t> host = build_tiled(K, refs, tg, row0);
  QCHECK(e->alloc(&out.buf, host.size()));
  return upload(e, out.buf, host.data(), host.size());
}

// Layer i of this engine: the whole layer, or rank `rank`'s tensor-parallel shard of it
// (q heads [rank*nh_l, +nh_l) with their kv heads; o_proj rows of those heads; gate/up
// columns and down rows [rank*I_l, +I_l)).
qora_status build_layer(qora_engine* e, const qora_weights_view* w, uint32_t i) {
  const qora_layer_view& L = w->layers[i];
  LayerDev& d = e->layers[i];
  const int H = (int)w->hidden;
  const int nh_l = e->nh_l, nkv_l = e->nkv_l, h0 = e->rank * nh_l;
  std::vector<GroupRef> refs;
  auto add_groups = [&](const qora_matrix_view& m, int g0, int ng) {
    for (int g = g0; g < g0 + ng; ++g) refs.push_back({&m, g});
  };
  constexpr int kGpH = kHeadDim / kGroup;  // groups per head
  refs.clear();
  add_groups(L.q_proj, h0 * kGpH, nh_l * kGpH);
  add_groups(L.k_proj, e->kv0 * kGpH, nkv_l * kGpH);
  add_groups(L.v_proj, e->kv0 * kGpH, nkv_l * kGpH);
  QCHECK(upload_q4(e, H, refs, d.qkv));
  QCHECK(upload_q4(e, H, refs, d.qkv1, 1));
  refs.clear();
  add_groups(L.o_proj, 0, (int)(L.o_proj.n / kGroup));
  QCHECK(upload_q4(e, nh_l * kHeadDim, refs, d.o, kTileGroups, h0 * kHeadDim));
  QCHECK(upload_q4(e, nh_l * kHeadDim, refs, d.o1, 1, h0 * kHeadDim));
  refs.clear();
  // gate/up tiles: 4 gate groups then the same 4 up groups (zero-padded at the end)
  const int gI_l = e->inter_l / kGroup, gi0 = e->rank * gI_l;
  for (int t = 0; t < (gI_l + 3) / 4; ++t) {
    for (int j = 0; j < 4; ++j) refs.push_back({4 * t + j < gI_l ? &L.gate_proj : nullptr, gi0 + 4 * t + j});
    for (int j = 0; j < 4; ++j) refs.push_back({4 * t + j < gI_l ? &L.up_proj : nullptr, gi0 + 4 * t + j});
  }
  QCHECK(upload_q4(e, H, refs, d.gu));
  refs.clear();
  add_groups(L.down_proj, 0, (int)(L.down_proj.n / kGroup));
  QCHECK(upload_q4(e, e->inter_l, refs, d.down, kTileGroups, e->rank * e->inter_l));
  std::vector<float> g1 = f16_to_f32(L.input_norm_gamma, H), g2 = f16_to_f32(L.post_attn_norm_gamma, H);
  QCHECK(e->alloc(&d.g_in, H));
  QCHECK(e->alloc(&d.g_post, H));
  QCHECK(upload(e, d.g_in, g1.data(), H * 4));
  QCHECK(upload(e, d.g_post, g2.data(), H * 4));
  d.rope = w->no_rope_layers[i] ? 1 : 0;
  d.nq = nh_l * kHeadDim;
  d.nkv = nkv_l * kHeadDim;
  return QORA_OK;
}

qora_status mega_init(qora_engine* e);
qora_status q4_prefill_init(qora_engine* e, const qora_weights_view* w);

qora_status engine_init(qora_engine* e, const qora_weights_view* w) {
  const qora_layer_view& L0 = w->layers[0];
  e->format = w->format;
  e->num_layers = w->num_layers;
  e->vocab = w->vocab;
  e->hidden = w->hidden;
  e->inter = (uint32_t)L0.gate_proj.n;
  e->nh = L0.num_heads;
  e->nkv_total = L0.num_kv_heads;
  e->rope_rows = (uint32_t)w->rope_rows;
  {
    qora_tp_shard sh{};
    QCHECK(tp_plan(QORA_FORMAT_Q4, e->nh, e->nkv_total, e->inter, e->vocab, e->tp, e->rank, &sh));
    e->nh_l = (int)sh.q_heads;
    e->nkv_l = (int)sh.kv_heads;
    e->kv0 = (int)sh.kv_head0;
    e->inter_l = (int)sh.mlp_n;
    e->nkv = (uint32_t)e->nkv_l;  // KV heads held by this engine's caches
  }
  e->sms = sm_count(e->device);
  QCUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  e->layers.resize(w->num_layers);

  // layers re-tiled on host worker threads (allocation + upload per layer)
  {
    const unsigned nthreads = std::max(1u, std::min(8u, std::thread::hardware_concurrency()));
    std::vector<qora_status> st(w->num_layers, QORA_OK);
    std::vector<std::string> errs(w->num_layers);
    std::mutex alloc_mu;
    std::vector<std::thread> pool;
    std::atomic<uint32_t> next{0};
    for (unsigned t = 0; t < nthreads; ++t) {
      pool.emplace_back([&] {
        cudaSetDevice(e->device);
        for (;;) {
          const uint32_t i = next.fetch_add(1);
          if (i >= w->num_layers) break;
          // allocation bookkeeping is not thread-safe: build into a private engine shell
          qora_engine tmp;
          tmp.device = e->device;
          tmp.tp = e->tp;
          tmp.rank = e->rank;
          tmp.nh_l = e->nh_l;
          tmp.nkv_l = e->nkv_l;
          tmp.kv0 = e->kv0;
          tmp.inter_l = e->inter_l;
          tmp.layers.resize(w->num_layers);
          st[i] = build_layer(&tmp, w, i);
          if (st[i] != QORA_OK) errs[i] = g_last_error;
          std::lock_guard<std::mutex> lk(alloc_mu);
          e->layers[i] = tmp.layers[i];
          e->allocs.insert(e->allocs.end(), tmp.allocs.begin(), tmp.allocs.end());
          e->device_bytes += tmp.device_bytes;
          tmp.allocs.clear();
        }
      });
    }
    for (auto& th : pool) th.join();
    for (uint32_t i = 0; i < w->num_layers; ++i)
      if (st[i] != QORA_OK) return fail(st[i], "layer %u: %s", i, errs[i].c_str());
  }

  const size_t H = w->hidden, V = w->vocab;
  {
    // row-interleaved copy: one contiguous row per token serves both the embedding lookup
    // and the row-dot lm_head stream (same nibbles and f16 scales as the file)
    e->lm_row_bytes = (long long)(H / 2 + H / kGroup * 2);
    std::vector<uint8_t> host((size_t)V * e->lm_row_bytes);
    for (size_t v = 0; v < V; ++v) {
      uint8_t* dst = host.data() + v * e->lm_row_bytes;
      std::memcpy(dst, w->embed.packed + v * (H / 2), H / 2);
      std::memcpy(dst + H / 2, w->embed.scales + v * (H / kGroup), H / kGroup * 2);
    }
    QCHECK(e->alloc(&e->lm_table, host.size()));
    QCHECK(upload(e, e->lm_table, host.data(), host.size()));
  }
  std::vector<float> fg = f16_to_f32(w->final_norm_gamma, H);
  QCHECK(e->alloc(&e->final_gamma, H));
  QCHECK(upload(e, e->final_gamma, fg.data(), H * 4));
  const size_t rt = (size_t)w->rope_rows * kHalfDim;
  QCHECK(e->alloc(&e->rope_cos, rt));
  QCHECK(e->alloc(&e->rope_sin, rt));
  QCHECK(upload(e, e->rope_cos, w->rope_cos, rt * 4));
  QCHECK(upload(e, e->rope_sin, w->rope_sin, rt * 4));

  const int nq = (int)(e->nh * kHeadDim);
  QCHECK(e->alloc(&e->x, H));
  QCHECK(e->alloc(&e->q, nq));
  QCHECK(e->alloc(&e->attn, nq));
  QCHECK(e->alloc(&e->h, e->inter));
  QCHECK(e->alloc(&e->logits, V));

  const int ctas = 2 * e->sms;
  const LayerDev& d0 = e->layers[0];
  e->sh_qkv = plan_gemv(d0.qkv.K, d0.qkv.tiles, ctas);
  e->sh_o = plan_gemv(d0.o.K, d0.o.tiles, ctas);
  e->sh_gu = plan_gemv(d0.gu.K, d0.gu.tiles, ctas);
  e->sh_down = plan_gemv(d0.down.K, d0.down.tiles, ctas);
  size_t pf = 0;
  for (const GemvShape* s : {&e->sh_qkv, &e->sh_o, &e->sh_gu, &e->sh_down}) {
    pf = std::max(pf, partial_floats(*s));
    e->max_tiles = std::max(e->max_tiles, s->tiles);
  }
  QCHECK(e->alloc(&e->partials, pf));
  QCHECK(e->alloc(&e->counters, e->max_tiles));
  QCUDA(cudaMemset(e->counters, 0, e->max_tiles * sizeof(unsigned)));

  e->lm_ctas = 2 * e->sms;
  QCHECK(e->alloc(&e->lm_part_v, e->lm_ctas));
  QCHECK(e->alloc(&e->lm_part_i, e->lm_ctas));
  QCHECK(e->alloc(&e->lm_counter, 1));
  QCUDA(cudaMemset(e->lm_counter, 0, sizeof(unsigned)));
  QCHECK(mega_init(e));
  QCHECK(q4_prefill_init(e, w));
  QCUDA(cudaDeviceSynchronize());
  return QORA_OK;
}

// ------------------------------------------------------------------ megakernel set-up
template <int GPL>
qora_status mega_occupancy(int* blocks) {
  auto kern = mk::decode_megakernel<GPL>;
  QCUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)mk::smem_bytes()));
  QCUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(blocks, kern, mk::kThreads, mk::smem_bytes()));
  return QORA_OK;
}

// Decide whether the persistent kernel can run this geometry and allocate its buffers.
// q|k|v runs on the last gq CTAs and o_proj on the go CTAs before them, so that their
// few split-K partials can be summed directly by the consumers; gate/up and down run on
// every CTA.
qora_status mega_init(qora_engine* e) {
  e->mk_ok = false;
  const int H = (int)e->hidden, G = e->sms;
  const LayerDev& d0 = e->layers[0];
  const int nh = e->nh_l, nkvh = e->nkv_l;  // this engine's (shard's) heads
  auto no = [&](const char* why) {
    e->mk_why = why;
    return QORA_OK;
  };
  if (H != 1024 && H != 2048) return no("hidden must be 1024 or 2048");
  if (nh % nkvh != 0 || nh / nkvh > mk::kHeadsPerKV || nh > 16)
    return no("needs at most 4 query heads per KV head and at most 16 heads");
  if (G < 16 || G > mk::kMaxUnits) return no("SM count outside the supported range");
  // q|k|v and o_proj: one CTA per 32-column group (q|k|v on the last CTAs, o_proj on the
  // first); gate/up and down: split-K over all CTAs
  const DevQ4* mats[4] = {&d0.qkv1, &d0.o1, &d0.gu, &d0.down};
  if (d0.qkv1.G > G || d0.o1.G > G) return no("more q|k|v or o_proj column groups than SMs");
  const int sub0[4] = {G - d0.qkv1.G, 0, 0, 0};
  const int subn[4] = {d0.qkv1.G, d0.o1.G, G, G};
  for (int m = 0; m < 4; ++m) {
    const long long total = (long long)mats[m]->tiles * mats[m]->K;
    if ((m < mk::GU && mats[m]->K > mk::kXsCap) || (total + subn[m] - 1) / subn[m] > mk::kXsCap)
      return no("per-CTA rows exceed the shared input buffer");
    if (total * subn[m] >= (1ll << 31)) return no("matrix too large for 32-bit split-K indexing");
    if ((total + subn[m] - 1) / subn[m] > mats[m]->K) return no("a CTA's rows would span more than two tiles");
    e->mk_sub0[m] = sub0[m];
    e->mk_subn[m] = subn[m];
  }
  if (d0.gu.tiles + d0.down.tiles + 3 > mk::kMaxTabTiles) return no("too many gate/up and down tiles");
  if (H > mk::kBFloats) return no("hidden larger than the shared x buffer");

  if (e->lm_row_bytes > mk::kStageBytes) return no("embedding row larger than a stage");
  if ((long long)G * e->vocab >= (1ll << 31)) return no("vocab split outside 32-bit arithmetic");
  int blocks = 0;
  if (H == 2048) QCHECK(mega_occupancy<2>(&blocks)); else QCHECK(mega_occupancy<1>(&blocks));
  if (blocks < 1) return no("megakernel does not fit one CTA per SM");
  e->mk_G = G;
  // longest cache whose attention units (kv head x chunk of <= kMaxAttnChunk) fit the grid
  e->mk_max_seq = (uint32_t)mk::kMaxAttnChunk * (uint32_t)(G / nkvh);
  if (e->num_layers > 62) return no("more than 62 layers (hand-off tags hold layer + 1 in 6 bits)");
  {
    GemvShape sh = plan_gemv(mats[mk::GU]->K, mats[mk::GU]->tiles, subn[mk::GU]);
    e->mk_slots[mk::GU] = sh.plan.max_slots;
  }
  // down_proj: tile-aligned split (mk::al_first), at most ceil(G / tiles) CTAs per tile
  const int dt = mats[mk::DOWN]->tiles;
  if (dt > subn[mk::DOWN]) return no("more down_proj tiles than CTAs");
  if ((long long)dt * subn[mk::DOWN] >= (1ll << 31) || (long long)subn[mk::DOWN] * mats[mk::DOWN]->K >= (1ll << 31))
    return no("down_proj split outside 32-bit arithmetic");
  e->mk_slots[mk::DOWN] = 0;
  for (int t = 0; t < dt; ++t) {
    const int n = mk::al_first(t + 1, subn[mk::DOWN], dt) - mk::al_first(t, subn[mk::DOWN], dt);
    e->mk_slots[mk::DOWN] = std::max(e->mk_slots[mk::DOWN], n);
    if ((mats[mk::DOWN]->K + n - 1) / n > mk::kXsCap) return no("per-CTA down_proj rows exceed the shared input buffer");
  }
  const size_t np_gu = (size_t)d0.gu.tiles * e->mk_slots[2] * kTileCols;
  const size_t np_dn = (size_t)d0.down.tiles * e->mk_slots[3] * kTileCols;
  e->mk_cpl = d0.down.tiles + nkvh;  // per layer: down tile arrivals, then attention arrivals per KV head
  e->mk_ncnt = (int)e->num_layers * e->mk_cpl + 2;
  QCHECK(e->alloc(&e->mk_cnt, e->mk_ncnt));
  QCUDA(cudaMemset(e->mk_cnt, 0, (size_t)e->mk_ncnt * sizeof(unsigned)));
  QCHECK(e->alloc(&e->mk_epoch, 1));
  QCUDA(cudaMemset(e->mk_epoch, 0, sizeof(unsigned)));
  // tagged buffers start at tag 0, which no launch uses
  auto alloc_tagged = [&](uint64_t** p, size_t n) -> qora_status {
    QCHECK(e->alloc(p, n));
    QCUDA(cudaMemset(*p, 0, n * sizeof(uint64_t)));
    return QORA_OK;
  };
  QCHECK(alloc_tagged(&e->mk_xbuf, (size_t)(e->num_layers + 1) * H));
  QCHECK(alloc_tagged(&e->mk_xmid, (size_t)e->num_layers * H));
  QCHECK(alloc_tagged(&e->mk_qkv, (size_t)d0.qkv1.G * kGroup));
  QCHECK(alloc_tagged(&e->mk_gu_part, np_gu));
  QCHECK(alloc_tagged(&e->mk_dn_part, np_dn));
  if (e->tp > 1) {
    // receive buffers the peers write into: o and down partials [L][tp][H] (tagged), the
    // ranks' lm_head bests [tp][2] (tagged), the full logits [vocab]
    const size_t L = e->num_layers, T = e->tp;
    e->tp_off_d = L * T * H * 8;
    e->tp_off_lm = 2 * L * T * H * 8;
    e->tp_off_logits = (e->tp_off_lm + T * 16 + 255) / 256 * 256;
    e->tp_region_bytes = e->tp_off_logits + (size_t)e->vocab * 4;
    QCHECK(e->alloc(&e->tp_region, e->tp_region_bytes));
    QCUDA(cudaMemset(e->tp_region, 0, e->tp_region_bytes));
    e->logits = reinterpret_cast<float*>(e->tp_region + e->tp_off_logits);
  }
  QCHECK(e->alloc(&e->mk_lm_v, G));
  QCHECK(e->alloc(&e->mk_lm_i, G));
  e->mk_ok = true;
  return QORA_OK;
}

qora_status mega_prepare(qora_engine* e, qora_kv* kv) {
  if (kv->mk_ready) return QORA_OK;
  const int L = (int)e->num_layers, G = e->mk_G;
  std::vector<mk::Layer> hl(L);
  for (int i = 0; i < L; ++i) {
    const LayerDev& d = e->layers[i];
    hl[i].w[0] = d.qkv1.buf;
    hl[i].w[1] = d.o1.buf;
    hl[i].w[2] = d.gu.buf;
    hl[i].w[3] = d.down.buf;
    hl[i].g_in = d.g_in;
    hl[i].g_post = d.g_post;
    hl[i].kc = static_cast<float*>(kv->k_layer(i));
    hl[i].vc = static_cast<float*>(kv->v_layer(i));
    hl[i].rope = d.rope;
  }
  QCHECK(kv->alloc(&kv->mk_layers, L));
  QCUDA(cudaMemcpy(kv->mk_layers, hl.data(), L * sizeof(mk::Layer), cudaMemcpyHostToDevice));
  QCHECK(kv->alloc(&kv->mk_att_o, (size_t)G * mk::kHeadsPerKV * kHeadDim));
  QCHECK(kv->alloc(&kv->mk_att_ml, (size_t)G * mk::kHeadsPerKV * 2));
  QCUDA(cudaMemset(kv->mk_att_o, 0, (size_t)G * mk::kHeadsPerKV * kHeadDim * sizeof(uint64_t)));
  QCUDA(cudaMemset(kv->mk_att_ml, 0, (size_t)G * mk::kHeadsPerKV * 2 * sizeof(uint64_t)));
  QCHECK(kv->alloc(&kv->mk_att_fin, (size_t)e->nh_l * kHeadDim));
  QCUDA(cudaMemset(kv->mk_att_fin, 0, (size_t)e->nh_l * kHeadDim * sizeof(uint64_t)));
  mk::Args& a = kv->mk_args;
  a = mk::Args{};
  a.layers = kv->mk_layers;
  a.L = L;
  const LayerDev& d0 = e->layers[0];
  const DevQ4* mats[4] = {&d0.qkv1, &d0.o1, &d0.gu, &d0.down};
  for (int m = 0; m < 4; ++m) {
    a.K[m] = mats[m]->K;
    a.tiles[m] = mats[m]->tiles;
    a.slots[m] = e->mk_slots[m];
    a.sub0[m] = e->mk_sub0[m];
    a.subn[m] = e->mk_subn[m];
  }
  a.H = (int)e->hidden;
  a.nq = d0.nq;
  a.nkvw = d0.nkv;
  a.nh = e->nh_l;
  a.nkvh = e->nkv_l;
  a.vocab = (int)e->vocab;
  a.lm_row_bytes = (int)e->lm_row_bytes;
  {
    // embedding rows per stage: as many as fit, a multiple of the consumer warps if possible
    int rows = (int)(mk::kStageBytes / e->lm_row_bytes);
    if (rows >= mk::kCW) rows -= rows % mk::kCW;
    a.lm_rows_per_stage = rows;
  }
  a.head_stride = (long long)kv->max_seq * kHeadDim;
  a.kv16 = kv->dtype == QORA_KV_F16 ? 1 : 0;
  a.lm = e->lm_table;
  a.final_gamma = e->final_gamma;
  a.cos_t = e->rope_cos;
  a.sin_t = e->rope_sin;
  bool any_rope = false;
  for (auto& Ld : e->layers) any_rope |= (Ld.rope != 0);
  a.max_pos = (int)std::min<uint32_t>(kv->max_seq, any_rope ? e->rope_rows : kv->max_seq);
  a.xbuf = e->mk_xbuf;
  a.xmid = e->mk_xmid;
  a.qkv = e->mk_qkv;
  a.gu_part = e->mk_gu_part;
  a.dn_part = e->mk_dn_part;
  a.epoch = e->mk_epoch;
  a.logits = e->logits;
  a.att_o = kv->mk_att_o;
  a.att_ml = kv->mk_att_ml;
  a.att_fin = kv->mk_att_fin;
  a.cnt = e->mk_cnt;
  a.cpl = e->mk_cpl;
  a.n_cnt = e->mk_ncnt;
  a.lm_v = e->mk_lm_v;
  a.lm_i = e->mk_lm_i;
  a.st = kv->st;
  a.ring = kv->ring;
  a.ring_cap = (int)kv->max_seq;
  a.timeout_ns = 2000000000ull;
  a.trace = e->mk_trace;
  a.tp = e->tp;
  a.rank = e->rank;
  a.hpk = e->nh_l / e->nkv_l;
  a.want_logits = 1;
  a.v0 = (int)((long long)e->rank * e->vocab / e->tp);
  a.v1 = (int)((long long)(e->rank + 1) * e->vocab / e->tp);
  for (int p = 0; p < e->tp && e->tp > 1; ++p) {
    uint8_t* base = e->tp_peer[p];
    a.peer_o[p] = reinterpret_cast<uint64_t*>(base);
    a.peer_d[p] = reinterpret_cast<uint64_t*>(base + e->tp_off_d);
    a.peer_lm[p] = reinterpret_cast<uint64_t*>(base + e->tp_off_lm);
    a.peer_logits[p] = reinterpret_cast<float*>(base + e->tp_off_logits);
  }
  kv->mk_ready = true;
  return QORA_OK;
}

qora_status launch_mega(qora_engine* e, qora_kv* kv, bool want_logits) {
  kv->mk_args.want_logits = want_logits ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(e->mk_G);
  cfg.blockDim = dim3(mk::kThreads);
  cfg.dynamicSmemBytes = mk::smem_bytes();
  cfg.stream = e->stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (e->hidden == 2048) {
    QCUDA(cudaLaunchKernelEx(&cfg, mk::decode_megakernel<2>, kv->mk_args));
  } else {
    QCUDA(cudaLaunchKernelEx(&cfg, mk::decode_megakernel<1>, kv->mk_args));
  }
  return QORA_OK;
}

// ------------------------------------------------------------------ step launches
qora_status launch_lm_head(int hidden, const LmArgs& a, int ctas, cudaStream_t s) {
  switch (hidden) {
    case 1024: lm_head_kernel<1><<<ctas, kLmThreads, 0, s>>>(a); break;
    case 2048: lm_head_kernel<2><<<ctas, kLmThreads, 0, s>>>(a); break;
    case 3072: lm_head_kernel<3><<<ctas, kLmThreads, 0, s>>>(a); break;
    case 4096: lm_head_kernel<4><<<ctas, kLmThreads, 0, s>>>(a); break;
    default: return fail(QORA_ERR_UNSUPPORTED, "lm_head: hidden %d", hidden);
  }
  QCUDA(cudaGetLastError());
  return QORA_OK;
}

qora_status launch_layer(qora_engine* e, qora_kv* kv, uint32_t li) {
  const LayerDev& d = e->layers[li];
  cudaStream_t s = e->stream;
  float* kc = kv->k + li * kv->layer_stride();
  float* vc = kv->v + li * kv->layer_stride();
  EpiQKV eq{e->q, kc, vc, (long long)kv->max_seq * kHeadDim, kv->st, e->rope_cos, e->rope_sin, d.nq, d.nkv, d.rope,
            (int)std::min<uint32_t>(kv->max_seq, d.rope ? e->rope_rows : kv->max_seq)};
  QCHECK(launch_gemv(d.qkv.src(), e->sh_qkv, e->partials, e->counters,
                     ProNorm{e->x, d.g_in, (int)e->hidden}, eq, s));
  AttnArgs aa{};
  aa.q = e->q;
  aa.kc = kc;
  aa.vc = vc;
  aa.hs = (long long)kv->max_seq * kHeadDim;
  aa.out = e->attn;
  aa.st = kv->st;
  aa.nkv = (int)e->nkv;
  aa.nc = kv->attn_nc;
  aa.scale = 1.0f / std::sqrt((float)kHeadDim);
  aa.part_o = kv->attn_o;
  aa.part_ml = kv->attn_ml;
  aa.counters = kv->attn_counters;
  attn_decode_kernel<<<dim3(e->nkv, kv->attn_nc), kAttnThreads, 0, s>>>(aa);
  QCUDA(cudaGetLastError());
  QCHECK(launch_gemv(d.o.src(), e->sh_o, e->partials, e->counters, ProPlain{e->attn},
                     EpiResidual{e->x, (int)e->hidden}, s));
  QCHECK(launch_gemv(d.gu.src(), e->sh_gu, e->partials, e->counters,
                     ProNorm{e->x, d.g_post, (int)e->hidden}, EpiSwiGLU{e->h, (int)e->inter}, s));
  QCHECK(launch_gemv(d.down.src(), e->sh_down, e->partials, e->counters, ProPlain{e->h},
                     EpiResidual{e->x, (int)e->hidden}, s));
  return QORA_OK;
}

// the whole decode step (what the CUDA graph holds)
qora_status launch_step(qora_engine* e, qora_kv* kv, int* launches) {
  cudaStream_t s = e->stream;
  embed_q4_kernel<<<1, 256, 0, s>>>(e->lm_table, e->lm_row_bytes, (int)e->vocab,
                                    (int)e->hidden, kv->st, e->x);
  QCUDA(cudaGetLastError());
  int n = 1;
  for (uint32_t li = 0; li < e->num_layers; ++li) {
    QCHECK(launch_layer(e, kv, li));
    n += 5;
  }
  LmArgs la{};
  la.x = e->x;
  la.gamma = e->final_gamma;
  la.packed = e->lm_table;
  la.scales = e->lm_table + e->hidden / 2;
  la.row_stride_p = la.row_stride_s = e->lm_row_bytes;
  la.vocab = (int)e->vocab;
  la.logits = e->logits;
  la.argmax_out = &kv->st->argmax;
  la.part_v = e->lm_part_v;
  la.part_i = e->lm_part_i;
  la.counter = e->lm_counter;
  QCHECK(launch_lm_head((int)e->hidden, la, e->lm_ctas, s));
  advance_kernel<<<1, 1, 0, s>>>(kv->st, kv->ring, (int)kv->max_seq);
  QCUDA(cudaGetLastError());
  n += 2;
  if (launches) *launches = n;
  return QORA_OK;
}

qora_status ensure_graph(qora_engine* e, qora_kv* kv) {
  if (kv->graph) return QORA_OK;
  cudaGraph_t g = nullptr;
  QCUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  qora_status st = launch_step(e, kv, nullptr);
  cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (st != QORA_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (ce != cudaSuccess) return fail(QORA_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
  ce = cudaGraphInstantiate(&kv->graph, g, 0);
  cudaGraphDestroy(g);
  if (ce != cudaSuccess) return fail(QORA_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ce));
  return QORA_OK;
}

// prepare whichever decode path this engine uses (graph of per-op kernels, or the
// persistent megakernel)
bool kv_uses_mega(const qora_engine* e, const qora_kv* kv) {
  return e->mk_ok && e->use_mega && kv->max_seq <= e->mk_max_seq;
}

qora_status step_prepare(qora_engine* e, qora_kv* kv) {
  if (e->tp > 1 && !e->tp_connected)
    return fail(QORA_ERR_UNSUPPORTED, "tensor-parallel engine: call qora_tp_connect first");
  if (e->tp > 1 && !kv_uses_mega(e, kv))
    return fail(QORA_ERR_UNSUPPORTED, "tensor-parallel engines need caches of at most %u positions", e->mk_max_seq);
  if (kv_uses_mega(e, kv)) return mega_prepare(e, kv);
  return ensure_graph(e, kv);
}

// want_logits = false: the caller reads only the argmax of this step (greedy loops, the
// prompt tokens before the last), so tensor-parallel ranks exchange only their candidates
qora_status step_launch(qora_engine* e, qora_kv* kv, bool want_logits = true) {
  if (kv_uses_mega(e, kv)) return launch_mega(e, kv, want_logits);
  QCUDA(cudaGraphLaunch(kv->graph, e->stream));
  return QORA_OK;
}

qora_status check_uniform_len(const qora_kv* kv, uint32_t* len) {
  const uint32_t l = kv->len[0];
  for (uint32_t x : kv->len)
    if (x != l) return fail(QORA_ERR_INVALID, "KV layers have different lengths (layer_step use?)");
  *len = l;
  return QORA_OK;
}

qora_status set_state(qora_engine* e, qora_kv* kv, int pos, int token, int step) {
  kv->st_host->pos = pos;
  kv->st_host->token = token;
  kv->st_host->argmax = 0;
  kv->st_host->step = step;
  kv->st_host->error = 0;
  QCUDA(cudaMemcpyAsync(kv->st, kv->st_host, sizeof(StepState), cudaMemcpyHostToDevice, e->stream));
  return QORA_OK;
}

qora_status check_step_error(qora_engine* e, qora_kv* kv) {
  QCUDA(cudaMemcpyAsync(kv->st_host, kv->st, sizeof(StepState), cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaStreamSynchronize(e->stream));
  if (kv->st_host->error == 2) return fail(QORA_ERR_TIMEOUT, "a bounded device-side wait timed out");
  if (kv->st_host->error) return fail(QORA_ERR_RANGE, "device rejected a token id");
  return QORA_OK;
}

// ------------------------------------------------------------------ F16 weights: batched path
// Every F16 forward pass runs M rows (f16_batch.cuh): one row per sequence in a batched
// decode step, one row per prompt token in a prefill chunk.

// Persistent CTAs and partial slots per CTA of one tcgen05 GEMM (umma_gemm.cuh).
struct UmmaPlan {
  int G = 1, maxseg = 1;
};
UmmaPlan umma_plan(int sms, int tiles, int chunks) {
  UmmaPlan p;
  const long long T = (long long)tiles * chunks;
  p.G = (int)std::min<long long>(sms, T);
  p.maxseg = 1;
  for (int c = 0; c < p.G; ++c) {
    const long long b0 = umma::range_begin(c, T, p.G), b1 = umma::range_begin(c + 1, T, p.G);
    if (b1 > b0) p.maxseg = std::max(p.maxseg, (int)((b1 - 1) / chunks - b0 / chunks + 1));
  }
  return p;
}

// Device scratch shared by the fused tensor-core GEMMs of one engine (or one call).
struct UmmaCtx {
  int sms;
  cudaStream_t stream;
  uint8_t* xt;
  float* part;
  size_t part_floats;
  unsigned* tcnt;
  size_t ntcnt;
  unsigned* sync;
  int* err;
  bool q4 = false;  // weights are Q4 chunks (the dequantising kernel)
};

// Operand source of one fused GEMM: rows xin [M][ldx], RMSNorm with gamma when set, and
// the producer's statistics [st_n][128].
struct UmmaIn {
  const float* xin;
  int ldx;
  const float* gamma;
  float gmax;
  const float* st_ss;
  const float* st_mx;
  int st_n;
};

// One fused GEMM (umma::fused_gemm_kernel): N outputs over K, M rows, epilogue in `ep`
// (its output fields filled by the caller), cooperative launch on u.stream.
qora_status umma_fused(const UmmaCtx& u, const uint8_t* wt, int N, int K, int M, const UmmaIn& in,
                       umma::FusedArgs ep) {
  const int R = (M + 7) / 8 * 8, tiles = N / umma::kTileN, chunks = K / umma::kChunkK;
  const UmmaPlan p = umma_plan(u.sms, tiles, chunks);
  if ((size_t)p.G * p.maxseg * R * umma::kTileN > u.part_floats || (size_t)tiles > u.ntcnt || p.G > umma::kMaxContrib)
    return fail(QORA_ERR_INVALID, "GEMM plan exceeds the scratch (%d x %d x %d, %d tiles)", p.G, p.maxseg, R, tiles);
  umma::FusedArgs a = ep;
  a.w = wt;
  a.tiles = tiles;
  a.chunks = chunks;
  a.M = M;
  a.R = R;
  a.stages = umma::gemm_stages(R, u.q4);
  a.maxseg = p.maxseg;
  a.xin = in.xin;
  a.ldx = in.ldx;
  a.gamma = in.gamma;
  a.gmax = in.gmax;
  a.st_ss = in.st_ss;
  a.st_mx = in.st_mx;
  a.st_n = in.st_n;
  a.xt = u.xt;
  a.part = u.part;
  a.tile_cnt = u.tcnt;
  a.sync = u.sync;
  a.err = u.err;
  a.timeout_ns = 2000000000ull;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(p.G);
  cfg.blockDim = dim3(u.q4 ? umma::kQ4Threads : umma::kThreads);
  cfg.dynamicSmemBytes = umma::gemm_smem(R, a.stages, u.q4);
  cfg.stream = u.stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (u.q4) {
    QCUDA(cudaLaunchKernelEx(&cfg, umma::fused_gemm_kernel<true>, a));
  } else {
    QCUDA(cudaLaunchKernelEx(&cfg, umma::fused_gemm_kernel<false>, a));
  }
  return QORA_OK;
}

// opt the GEMM kernel in to its largest shared-memory footprint and check that one CTA
// fits on every SM (the cooperative launch needs all CTAs resident)
qora_status umma_attrs(bool q4 = false) {
  int maxsm = 0;
  for (int r = 8; r <= umma::kMaxRows; r += 8)
    maxsm = std::max(maxsm, (int)umma::gemm_smem(r, umma::gemm_stages(r, q4), q4));
  const void* fn = q4 ? (const void*)umma::fused_gemm_kernel<true> : (const void*)umma::fused_gemm_kernel<false>;
  QCUDA(cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, maxsm));
  int blocks = 0;
  QCUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks, fn, q4 ? umma::kQ4Threads : umma::kThreads, maxsm));
  if (blocks < 1) return fail(QORA_ERR_UNSUPPORTED, "tensor-core GEMM does not fit on an SM");
  return QORA_OK;
}

UmmaCtx umma_ctx(const qora_engine* e) {
  const int V = (int)e->vocab;
  return UmmaCtx{e->sms,  e->stream, e->f_xt, e->f_part, e->f_part_floats, e->f_tcnt,
                 (size_t)std::max(V, 2 * e->inter_l) / umma::kTileN + 1, e->f_sync, e->f_err,
                 e->format == QORA_FORMAT_Q4};
}

// Copy rows [r0, r0 + K) of an f16 matrix view to the device and re-tile them: for a
// projection ([k][n]) its columns [col0, col0 + N) become channels, for the embedding
// (kmajor, [vocab][hidden]) its rows do (then K = hidden, r0 = 0). Channel n goes to tile
// t0 + n / group, row o0 + n % group, of dst (`chunks` chunks of 64 k per tile).
qora_status f16_tile_upload(qora_engine* e, const qora_matrix_view& m, bool kmajor, uint64_t r0, int K, int col0,
                            int N, int t0, int group, int o0, int chunks, uint8_t* dst, __half* tmp) {
  const size_t rows = kmajor ? m.k : (size_t)K;
  QCUDA(cudaMemcpy(tmp, m.data + (kmajor ? 0 : r0 * m.n), rows * m.n * 2, cudaMemcpyHostToDevice));
  const long long units = (long long)N * (K / 8);
  const int blocks = (int)std::min<long long>((units + 255) / 256, 16LL * e->sms);
  umma::tile_weights_kernel<<<blocks, 256>>>(tmp, (long long)m.n, kmajor ? 1 : 0, K, N, kmajor ? 0 : col0, t0, group,
                                             o0, chunks, dst);
  QCUDA(cudaGetLastError());
  QCUDA(cudaDeviceSynchronize());
  return QORA_OK;
}

float max_abs_f16(const uint16_t* h, size_t n) {
  float m = 0.0f;
  for (float v : f16_to_f32(h, n)) m = std::max(m, std::fabs(v));
  return m;
}

// Row scratch of the batched tensor-core path (activations, GEMM operand and partial
// slots, statistics, attention partials, counters) for f16b::kMaxRows rows; lmN: lm_head
// columns run as a fused GEMM (0 when a Q4 engine runs its lm_head as row dots).
qora_status batched_scratch(qora_engine* e, int lmN) {
  const int H = (int)e->hidden, V = (int)e->vocab, nq = e->nh_l * kHeadDim, Il = e->inter_l;
  const size_t R = f16b::kMaxRows;
  size_t slots = 0;  // partial slots of the largest GEMM plan, in [R][128] blocks
  const int gn[5] = {e->f_nqkv, H, 2 * Il, H, lmN}, gk[5] = {H, nq, H, Il, H};
  for (int j = 0; j < 5; ++j) {
    const UmmaPlan p = umma_plan(e->sms, gn[j] / umma::kTileN, gk[j] / umma::kChunkK);
    slots = std::max(slots, (size_t)p.G * p.maxseg);
  }
  const size_t kmax = (size_t)std::max(std::max(H, nq), Il);
  e->f_part_floats = slots * R * umma::kTileN;
  QCHECK(e->alloc(&e->f_part, e->f_part_floats));
  QCHECK(e->alloc(&e->f_x, R * H));
  QCHECK(e->alloc(&e->f_qkv, R * e->f_nqkv));
  QCHECK(e->alloc(&e->f_attn, R * nq));
  QCHECK(e->alloc(&e->f_h, R * Il));
  QCHECK(e->alloc(&e->f_xt, kmax * R * 2 * 2));
  QCHECK(e->alloc(&e->f_xss, (size_t)(H / umma::kTileN) * R));
  QCHECK(e->alloc(&e->f_xmx, (size_t)(H / umma::kTileN) * R));
  QCHECK(e->alloc(&e->f_hmx, (size_t)(Il / 64) * R));
  QCHECK(e->alloc(&e->f_amx, (size_t)e->nkv * R));
  QCHECK(e->alloc(&e->f_att_part, R * e->nkv * f16b::kAttSplits * 4 * kHeadDim));
  QCHECK(e->alloc(&e->f_att_ml, R * e->nkv * f16b::kAttSplits * 4 * 2));
  QCHECK(e->alloc(&e->f_att_cnt, R * e->nkv));
  QCUDA(cudaMemset(e->f_att_cnt, 0, R * e->nkv * sizeof(unsigned)));
  const size_t ntc = (size_t)std::max(V, 2 * Il) / umma::kTileN + 1;
  QCHECK(e->alloc(&e->f_tcnt, ntc));
  QCUDA(cudaMemset(e->f_tcnt, 0, ntc * sizeof(unsigned)));
  QCHECK(e->alloc(&e->f_sync, 4));
  QCUDA(cudaMemset(e->f_sync, 0, 4 * sizeof(unsigned)));
  QCHECK(e->alloc(&e->f_amkey, R));
  QCUDA(cudaMemset(e->f_amkey, 0, R * sizeof(unsigned long long)));
  QCHECK(e->alloc(&e->f_err, 1));
  QCUDA(cudaMemset(e->f_err, 0, sizeof(int)));
  QCHECK(e->alloc(&e->f_epoch, 1));
  QCUDA(cudaMemset(e->f_epoch, 0, sizeof(unsigned)));
  return QORA_OK;
}

// Upload the F16 weights (exact copies; q|k|v and gate|up joined along n) and size the
// activation scratch for f16b::kMaxRows rows.
qora_status f16_engine_init(qora_engine* e, const qora_weights_view* w) {
  const qora_layer_view& L0 = w->layers[0];
  e->format = w->format;
  e->num_layers = w->num_layers;
  e->vocab = w->vocab;
  e->hidden = w->hidden;
  e->inter = (uint32_t)L0.gate_proj.n;
  e->nh = L0.num_heads;
  e->nkv_total = L0.num_kv_heads;
  e->rope_rows = (uint32_t)w->rope_rows;
  const int T = e->tp, r = e->rank;
  const int H = (int)e->hidden, I = (int)e->inter, V = (int)e->vocab;
  {
    qora_tp_shard sh{};
    QCHECK(tp_plan(QORA_FORMAT_F16, e->nh, e->nkv_total, (uint32_t)I, (uint32_t)V, T, r, &sh));
    e->nh_l = (int)sh.q_heads;
    e->nkv_l = (int)sh.kv_heads;
    e->kv0 = (int)sh.kv_head0;
    e->inter_l = (int)sh.mlp_padded;
    e->f_it = (int)sh.mlp_n;
    e->f_vt0 = (int)(sh.vocab0 / umma::kTileN);
    e->f_vt1 = (int)((sh.vocab0 + sh.vocab_n) / umma::kTileN);
  }
  e->nkv = (uint32_t)e->nkv_l;
  e->sms = sm_count(e->device);
  e->mk_ok = false;
  e->mk_why = "F16 weights run the batched path";
  QCUDA(cudaStreamCreateWithFlags(&e->stream, cudaStreamNonBlocking));
  const int nq = e->nh_l * kHeadDim, nkvw = e->nkv_l * kHeadDim, Il = e->inter_l, IT = e->f_it;
  const int h0 = r * e->nh_l;
  e->f_nqkv = nq + 2 * nkvw;
  e->fl.resize(e->num_layers);
  // staging buffer for one source matrix (freed at the end of the load)
  size_t tmp_elems = (size_t)V * H;
  tmp_elems = std::max(tmp_elems, (size_t)H * I);
  tmp_elems = std::max(tmp_elems, (size_t)H * e->nh * kHeadDim);
  __half* tmp = nullptr;
  QCUDA(cudaMalloc(&tmp, tmp_elems * 2));
  struct TmpFree {
    __half* p;
    ~TmpFree() { cudaFree(p); }
  } tmp_free{tmp};
  constexpr int TN = umma::kTileN, CK = umma::kChunkK;
  for (uint32_t i = 0; i < e->num_layers; ++i) {
    const qora_layer_view& L = w->layers[i];
    F16Layer& d = e->fl[i];
    QCHECK(e->alloc(&d.wqkv, (size_t)H * e->f_nqkv * 2));
    QCHECK(f16_tile_upload(e, L.q_proj, false, 0, H, h0 * kHeadDim, nq, 0, TN, 0, H / CK, d.wqkv, tmp));
    QCHECK(f16_tile_upload(e, L.k_proj, false, 0, H, e->kv0 * kHeadDim, nkvw, nq / TN, TN, 0, H / CK, d.wqkv, tmp));
    QCHECK(f16_tile_upload(e, L.v_proj, false, 0, H, e->kv0 * kHeadDim, nkvw, (nq + nkvw) / TN, TN, 0, H / CK,
                           d.wqkv, tmp));
    QCHECK(e->alloc(&d.wo, (size_t)nq * H * 2));
    QCHECK(f16_tile_upload(e, L.o_proj, false, (uint64_t)h0 * kHeadDim, nq, 0, H, 0, TN, 0, nq / CK, d.wo, tmp));
    // gate|up interleaved per tile: rows 0-63 gate channels 64t.., rows 64-127 the same up
    // channels, so one tile holds both operands of its 64 SwiGLU outputs (padding: zero)
    QCHECK(e->alloc(&d.wgu, (size_t)H * 2 * Il * 2));
    QCUDA(cudaMemset(d.wgu, 0, (size_t)H * 2 * Il * 2));
    QCHECK(f16_tile_upload(e, L.gate_proj, false, 0, H, r * IT, IT, 0, 64, 0, H / CK, d.wgu, tmp));
    QCHECK(f16_tile_upload(e, L.up_proj, false, 0, H, r * IT, IT, 0, 64, 64, H / CK, d.wgu, tmp));
    QCHECK(e->alloc(&d.wdown, (size_t)Il * H * 2));
    QCUDA(cudaMemset(d.wdown, 0, (size_t)Il * H * 2));
    QCHECK(f16_tile_upload(e, L.down_proj, false, (uint64_t)r * IT, IT, 0, H, 0, TN, 0, Il / CK, d.wdown, tmp));
    std::vector<float> g1 = f16_to_f32(L.input_norm_gamma, H), g2 = f16_to_f32(L.post_attn_norm_gamma, H);
    QCHECK(e->alloc(&d.g_in, H));
    QCHECK(e->alloc(&d.g_post, H));
    QCHECK(upload(e, d.g_in, g1.data(), (size_t)H * 4));
    QCHECK(upload(e, d.g_post, g2.data(), (size_t)H * 4));
    d.gmax_in = max_abs_f16(L.input_norm_gamma, H);
    d.gmax_post = max_abs_f16(L.post_attn_norm_gamma, H);
    d.rope = w->no_rope_layers[i] ? 1 : 0;
  }
  // the whole table: any token's embedding row; lm_head reads this rank's tiles
  QCHECK(e->alloc(&e->f_lm, (size_t)V * H * 2));
  QCHECK(f16_tile_upload(e, w->embed, true, 0, H, 0, V, 0, TN, 0, H / CK, e->f_lm, tmp));
  e->f_gmax_final = max_abs_f16(w->final_norm_gamma, H);
  std::vector<float> fg = f16_to_f32(w->final_norm_gamma, H);
  QCHECK(e->alloc(&e->final_gamma, H));
  QCHECK(upload(e, e->final_gamma, fg.data(), (size_t)H * 4));
  const size_t rt = (size_t)w->rope_rows * kHalfDim;
  QCHECK(e->alloc(&e->rope_cos, rt));
  QCHECK(e->alloc(&e->rope_sin, rt));
  QCHECK(upload(e, e->rope_cos, w->rope_cos, rt * 4));
  QCHECK(upload(e, e->rope_sin, w->rope_sin, rt * 4));

  QCHECK(batched_scratch(e, (e->f_vt1 - e->f_vt0) * TN));
  const size_t R = f16b::kMaxRows;
  if (T > 1) {
    // receive region (IPC-exported): o_proj and down partial tiles of every rank, the
    // ranks' lm_head candidates, and the full logits
    const size_t xr = (size_t)T * (H / TN) * R * TN * sizeof(uint64_t);
    e->tp_off_d = xr;
    e->tp_off_lm = 2 * xr;
    e->tp_off_logits = e->tp_off_lm + (size_t)T * R * 2 * sizeof(uint64_t);
    e->tp_region_bytes = e->tp_off_logits + R * (size_t)V * sizeof(float);
    QCHECK(e->alloc(&e->tp_region, e->tp_region_bytes));
    QCUDA(cudaMemset(e->tp_region, 0, e->tp_region_bytes));
    e->f_logits = reinterpret_cast<float*>(e->tp_region + e->tp_off_logits);
  } else {
    QCHECK(e->alloc(&e->f_logits, R * V));
  }
  e->logits = e->f_logits;
  QCHECK(umma_attrs());
  QCUDA(cudaDeviceSynchronize());
  return QORA_OK;
}

// Rows [r0, r0 + K) of a Q4 matrix view to the device (tmp_p / tmp_s), re-tiled as
// dequantisation chunks: column col0 + n -> tile t0 + n / group, channel o0 + n % group.
qora_status q4_chunk_upload(const qora_matrix_view& m, uint64_t r0, int K, int col0, int N, int t0, int group,
                            int o0, int chunks, uint8_t* dst, uint8_t* tmp_p, uint16_t* tmp_s, int sms) {
  QCUDA(cudaMemcpy(tmp_p, m.packed + r0 * (m.n / 2), (size_t)K * (m.n / 2), cudaMemcpyHostToDevice));
  QCUDA(cudaMemcpy(tmp_s, m.scales + r0 * (m.n / kGroup), (size_t)K * (m.n / kGroup) * 2, cudaMemcpyHostToDevice));
  const long long units = (long long)N * (K / 8);
  const int blocks = (int)std::min<long long>((units + 255) / 256, 16LL * sms);
  umma::tile_q4_kernel<<<blocks, 256>>>(tmp_p, tmp_s, (long long)m.n, K, N, col0, t0, group, o0, chunks, dst);
  QCUDA(cudaGetLastError());
  QCUDA(cudaDeviceSynchronize());
  return QORA_OK;
}

// The Q4 prompt pass on the tensor cores (raw_prefill, src/gemv.rs:1027-1190, with
// gemm_q4 :680-706): the batched path's layer loop over all prompt rows, each projection
// a dequantising tcgen05 GEMM over a second, chunked copy of its Q4 weights (0.5625 B per
// weight, 1.6 GB for SmolLM3-3B), the lm_head the decode step's row-dot kernel on the last
// row. Not set up (prompts then run as decode steps) for tensor-parallel shards, on
// request (QORA_FLAG_TOKEN_PREFILL), when the shapes do not tile, or when a scale times 8
// would overflow binary16.
qora_status q4_prefill_init(qora_engine* e, const qora_weights_view* w) {
  e->q4p = false;
  const int H = (int)e->hidden, I = (int)e->inter, nq = (int)e->nh * kHeadDim, nkvw = (int)e->nkv_total * kHeadDim;
  if (!e->want_q4p) {
    e->q4p_why = "disabled by QORA_FLAG_TOKEN_PREFILL";
    return QORA_OK;
  }
  if (e->tp > 1) {
    e->q4p_why = "tensor-parallel shard";
    return QORA_OK;
  }
  if (H % umma::kTileN || I % 64 || nq % umma::kTileN || nq > 8192 || I > 65536 ||
      (H != 1024 && H != 2048 && H != 3072 && H != 4096)) {
    e->q4p_why = "shapes do not tile";
    return QORA_OK;
  }
  // |q - 8| * |s| <= 8 |s| must stay finite in binary16: |s| <= 8188 (bits <= 0x6FFF)
  for (uint32_t i = 0; i < e->num_layers; ++i) {
    const qora_layer_view& L = w->layers[i];
    for (const qora_matrix_view* m : {&L.q_proj, &L.k_proj, &L.v_proj, &L.o_proj, &L.gate_proj, &L.up_proj,
                                      &L.down_proj}) {
      const size_t ns = (size_t)m->k * (m->n / kGroup);
      for (size_t j = 0; j < ns; ++j)
        if ((m->scales[j] & 0x7FFFu) > 0x6FFFu) {
          e->q4p_why = "a Q4 scale beyond 8188";
          return QORA_OK;
        }
    }
  }
  constexpr int TN = umma::kTileN, CK = umma::kChunkK;
  const size_t CH = umma::kQ4Chunk;
  const size_t maxk = (size_t)std::max(H, std::max(nq, I)), maxn = (size_t)std::max(std::max(H, nq), I);
  uint8_t* tmp_p = nullptr;
  uint16_t* tmp_s = nullptr;
  QCUDA(cudaMalloc(&tmp_p, maxk * maxn / 2));
  QCUDA(cudaMalloc(&tmp_s, maxk * (maxn / kGroup) * 2));
  struct TmpFree {
    void *a, *b;
    ~TmpFree() {
      cudaFree(a);
      cudaFree(b);
    }
  } tmp_free{tmp_p, tmp_s};
  e->f_nqkv = nq + 2 * nkvw;
  e->fl.assign(e->num_layers, F16Layer{});
  for (uint32_t i = 0; i < e->num_layers; ++i) {
    const qora_layer_view& L = w->layers[i];
    F16Layer& d = e->fl[i];
    const LayerDev& ld = e->layers[i];
    QCHECK(e->alloc(&d.wqkv, (size_t)(e->f_nqkv / TN) * (H / CK) * CH));
    QCHECK(q4_chunk_upload(L.q_proj, 0, H, 0, nq, 0, TN, 0, H / CK, d.wqkv, tmp_p, tmp_s, e->sms));
    QCHECK(q4_chunk_upload(L.k_proj, 0, H, 0, nkvw, nq / TN, TN, 0, H / CK, d.wqkv, tmp_p, tmp_s, e->sms));
    QCHECK(q4_chunk_upload(L.v_proj, 0, H, 0, nkvw, (nq + nkvw) / TN, TN, 0, H / CK, d.wqkv, tmp_p, tmp_s, e->sms));
    QCHECK(e->alloc(&d.wo, (size_t)(H / TN) * (nq / CK) * CH));
    QCHECK(q4_chunk_upload(L.o_proj, 0, nq, 0, H, 0, TN, 0, nq / CK, d.wo, tmp_p, tmp_s, e->sms));
    // gate|up per tile: channels 0-63 gate 64t.., 64-127 the same up columns
    QCHECK(e->alloc(&d.wgu, (size_t)(I / 64) * (H / CK) * CH));
    QCHECK(q4_chunk_upload(L.gate_proj, 0, H, 0, I, 0, 64, 0, H / CK, d.wgu, tmp_p, tmp_s, e->sms));
    QCHECK(q4_chunk_upload(L.up_proj, 0, H, 0, I, 0, 64, 64, H / CK, d.wgu, tmp_p, tmp_s, e->sms));
    QCHECK(e->alloc(&d.wdown, (size_t)(H / TN) * (I / CK) * CH));
    QCHECK(q4_chunk_upload(L.down_proj, 0, I, 0, H, 0, TN, 0, I / CK, d.wdown, tmp_p, tmp_s, e->sms));
    d.g_in = ld.g_in;
    d.g_post = ld.g_post;
    d.gmax_in = max_abs_f16(L.input_norm_gamma, H);
    d.gmax_post = max_abs_f16(L.post_attn_norm_gamma, H);
    d.rope = ld.rope;
  }
  QCHECK(batched_scratch(e, 0));
  QCHECK(umma_attrs(true));
  e->q4p = true;
  return QORA_OK;
}

// Launch count of f16_forward (reported as the engine's launches per step).
int f16_launches(const qora_engine* e, bool lm) {
  // embedding; per layer the q|k|v, o, gate|up and down GEMMs and attention; lm_head
  return 1 + 5 * (int)e->num_layers + (lm ? 1 : 0);
}

// The layer stack over the M rows of kv's row table, then (rows [lm0, M) only) the final
// RMSNorm, the tied lm_head into f_logits rows [0, M - lm0) and the greedy argmax.
// Mirrors forward_decode_raw / raw_prefill (src/gemv.rs:872-1019, :1027-1190) per row.
// Tensor-parallel exchange fields of one fused GEMM (every rank's receive region): the
// residual GEMMs use the partial-tile block at `xr_off`, lm_head the candidate slots and
// the full logits.
void f16_tp_args(const qora_engine* e, umma::FusedArgs& a, int tag_slot, size_t xr_off) {
  a.tp = e->tp;
  a.rank = e->rank;
  a.epoch = e->f_epoch;
  a.tag_slot = tag_slot;
  if (e->tp < 2) return;
  for (int p = 0; p < e->tp; ++p) {
    uint8_t* base = e->tp_peer[p];
    a.xr_peer[p] = reinterpret_cast<unsigned long long*>(base + xr_off);
    a.lg_peer[p] = reinterpret_cast<float*>(base + e->tp_off_logits);
    a.key_peer[p] = reinterpret_cast<unsigned long long*>(base + e->tp_off_lm);
  }
}

qora_status f16_forward(qora_engine* e, qora_kv* kv, int M, int lm0) {
  const int H = (int)e->hidden, nq = e->nh_l * kHeadDim, I = e->inter_l;
  const int V = (int)e->vocab, NQKV = e->f_nqkv, R = f16b::kMaxRows;
  const f16b::RowInfo ri = f16b::row_info(kv->rows);
  cudaStream_t s = e->stream;
  const UmmaCtx u = umma_ctx(e);
  const int xt_n = H / umma::kTileN;
  const bool q4 = e->format == QORA_FORMAT_Q4;
  if (q4) {
    f16b::embed_rows_q4_kernel<<<dim3(xt_n, M), 128, 0, s>>>(e->lm_table, e->lm_row_bytes, H, V, ri, e->f_x, e->f_xss,
                                                              e->f_xmx, e->f_epoch);
  } else {
    f16b::embed_rows_kernel<<<dim3(xt_n, M), 128, 0, s>>>(e->f_lm, H, V, ri, e->f_x, e->f_xss, e->f_xmx, e->f_epoch);
  }
  QCUDA(cudaGetLastError());
  const long long hs = (long long)kv->max_seq * kHeadDim, ss = (long long)kv->seq_stride();
  for (uint32_t li = 0; li < e->num_layers; ++li) {
    const F16Layer& d = e->fl[li];
    float* kc = kv->k + li * kv->layer_stride();
    float* vc = kv->v + li * kv->layer_stride();
    // RMSNorm + q|k|v + RoPE + KV append (q rows to f_qkv)
    umma::FusedArgs a{};
    a.ep = umma::kEpQKV;
    a.y = e->f_qkv;
    a.ldy = nq;
    a.q_tiles = nq / umma::kTileN;
    a.k_tiles = e->nkv_l;
    a.rope = d.rope;
    a.cos_t = e->rope_cos;
    a.sin_t = e->rope_sin;
    a.rows = ri;
    a.kc = kc;
    a.vc = vc;
    a.seq_stride = ss;
    a.head_stride = hs;
    QCHECK(umma_fused(u, d.wqkv, NQKV, H, M, UmmaIn{e->f_x, H, d.g_in, d.gmax_in, e->f_xss, e->f_xmx, xt_n}, a));
    {
      f16b::AttnRowsArgs at{};
      at.q = e->f_qkv;
      at.nq = nq;
      at.nkv = (int)e->nkv;
      at.hpk = e->nh_l / e->nkv_l;
      at.rows = ri;
      at.kc = kc;
      at.vc = vc;
      at.seq_stride = ss;
      at.head_stride = hs;
      at.out = e->f_attn;
      at.st_mx = e->f_amx;
      at.o_part = e->f_att_part;
      at.ml_part = e->f_att_ml;
      at.cnt = e->f_att_cnt;
      f16b::attention_split_kernel<<<dim3(e->nkv, M, f16b::kAttSplits), f16b::kAttThreads, 0, s>>>(at);
      QCUDA(cudaGetLastError());
    }
    // o_proj + residual (and the statistics of the new x)
    a = umma::FusedArgs{};
    a.ep = umma::kEpResidual;
    a.y = e->f_x;
    a.res = e->f_x;
    a.ldy = H;
    a.o_ss = e->f_xss;
    a.o_mx = e->f_xmx;
    f16_tp_args(e, a, 2 * (int)li + 1, 0);  // o_proj partials: block at offset 0
    QCHECK(umma_fused(u, d.wo, H, nq, M, UmmaIn{e->f_attn, nq, nullptr, 0.0f, nullptr, e->f_amx, (int)e->nkv}, a));
    // RMSNorm + gate|up + SwiGLU
    a = umma::FusedArgs{};
    a.ep = umma::kEpSwiGLU;
    a.y = e->f_h;
    a.ldy = I;
    a.o_mx = e->f_hmx;
    QCHECK(umma_fused(u, d.wgu, 2 * I, H, M, UmmaIn{e->f_x, H, d.g_post, d.gmax_post, e->f_xss, e->f_xmx, xt_n}, a));
    // down_proj + residual
    a = umma::FusedArgs{};
    a.ep = umma::kEpResidual;
    a.y = e->f_x;
    a.res = e->f_x;
    a.ldy = H;
    a.o_ss = e->f_xss;
    a.o_mx = e->f_xmx;
    f16_tp_args(e, a, 2 * (int)li + 2, e->tp_off_d);
    QCHECK(umma_fused(u, d.wdown, H, I, M, UmmaIn{e->f_h, I, nullptr, 0.0f, nullptr, e->f_hmx, I / 64}, a));
  }
  if (lm0 < M && q4) {
    // Q4 (prompt pass): final RMSNorm + tied lm_head + greedy argmax of the last row, the
    // decode step's kernel over the Q4 table
    if (lm0 != M - 1) return fail(QORA_ERR_INVALID, "Q4 prompt pass: logits of the last row only");
    LmArgs la{};
    la.x = e->f_x + (size_t)(M - 1) * H;
    la.gamma = e->final_gamma;
    la.packed = e->lm_table;
    la.scales = e->lm_table + H / 2;
    la.row_stride_p = la.row_stride_s = e->lm_row_bytes;
    la.vocab = V;
    la.logits = e->logits;
    la.argmax_out = &kv->st->argmax;
    la.part_v = e->lm_part_v;
    la.part_i = e->lm_part_i;
    la.counter = e->lm_counter;
    QCHECK(launch_lm_head(H, la, e->lm_ctas, s));
  } else if (lm0 < M) {
    // final RMSNorm + tied lm_head + greedy argmax for rows [lm0, M)
    umma::FusedArgs a{};
    a.ep = umma::kEpLogits;
    a.y = e->f_logits;
    a.ldy = V;
    a.am_key = e->f_amkey;
    a.am_out = kv->f_argmax;
    a.col0 = e->f_vt0 * umma::kTileN;
    f16_tp_args(e, a, 127, 0);
    const uint8_t* lmw = e->f_lm + (size_t)e->f_vt0 * (H / umma::kChunkK) * umma::kATile;
    QCHECK(umma_fused(u, lmw, (e->f_vt1 - e->f_vt0) * umma::kTileN, H, M - lm0,
                      UmmaIn{e->f_x + (size_t)lm0 * H, H, e->final_gamma, e->f_gmax_final, e->f_xss + lm0,
                             e->f_xmx + lm0, xt_n},
                      a));
  }
  (void)R;
  return QORA_OK;
}

// The batched decode step of all kv->batch rows as one CUDA graph (captured once per
// cache; the row table it reads stays at a fixed address).
qora_status f16_ensure_graph(qora_engine* e, qora_kv* kv) {
  if (kv->f_graph) return QORA_OK;
  cudaGraph_t g = nullptr;
  QCUDA(cudaStreamBeginCapture(e->stream, cudaStreamCaptureModeThreadLocal));
  const qora_status st = f16_forward(e, kv, (int)kv->batch, 0);
  const cudaError_t ce = cudaStreamEndCapture(e->stream, &g);
  if (st != QORA_OK) {
    if (g) cudaGraphDestroy(g);
    return st;
  }
  if (ce != cudaSuccess) return fail(QORA_ERR_CUDA, "graph capture: %s", cudaGetErrorString(ce));
  const cudaError_t ie = cudaGraphInstantiate(&kv->f_graph, g, 0);
  cudaGraphDestroy(g);
  if (ie != cudaSuccess) return fail(QORA_ERR_CUDA, "graph instantiate: %s", cudaGetErrorString(ie));
  return QORA_OK;
}

// Host lengths of every sequence (uniform over layers), as positions of the next row.
qora_status f16_seq_lens(qora_kv* kv, std::vector<uint32_t>& lens) {
  const uint32_t L = (uint32_t)(kv->len.size() / kv->batch);
  lens.resize(kv->batch);
  for (uint32_t b = 0; b < kv->batch; ++b) {
    lens[b] = kv->lenof(b, 0);
    for (uint32_t l = 1; l < L; ++l)
      if (kv->lenof(b, l) != lens[b])
        return fail(QORA_ERR_INVALID, "sequence %u: KV layers have different lengths", b);
  }
  return QORA_OK;
}

// Row table of a decode step: row b = sequence b at its current length with tokens[b].
qora_status f16_stage_decode_rows(qora_engine* e, qora_kv* kv, const uint32_t* tokens,
                                  const std::vector<uint32_t>& lens) {
  int* h = kv->rows_host;
  for (uint32_t b = 0; b < kv->batch; ++b) {
    h[b] = (int)b;
    h[f16b::kMaxRows + b] = (int)lens[b];
    h[2 * f16b::kMaxRows + b] = (int)tokens[b];
  }
  h[3 * f16b::kMaxRows] = 0;      // greedy step
  h[3 * f16b::kMaxRows + 1] = 0;  // error
  QCUDA(cudaMemcpyAsync(kv->rows, h, f16b::kRowInts * sizeof(int), cudaMemcpyHostToDevice, e->stream));
  return QORA_OK;
}

qora_status f16_check_error(qora_engine* e, qora_kv* kv) {
  int* h = kv->rows_host + 3 * f16b::kMaxRows;
  QCUDA(cudaMemcpyAsync(h + 1, kv->rows + 3 * f16b::kMaxRows + 1, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaMemcpyAsync(h, e->f_err, sizeof(int), cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaStreamSynchronize(e->stream));
  if (h[0]) {
    cudaMemsetAsync(e->f_err, 0, sizeof(int), e->stream);
    return fail(QORA_ERR_TIMEOUT, "a bounded wait in the tensor-core GEMM timed out");
  }
  if (h[1]) return fail(QORA_ERR_RANGE, "device rejected a token id");
  return QORA_OK;
}

qora_status f16_tp_ready(const qora_engine* e) {
  if (e->tp > 1 && !e->tp_connected)
    return fail(QORA_ERR_UNSUPPORTED, "tensor-parallel engine: call qora_tp_connect first");
  return QORA_OK;
}

qora_status f16_decode_step(qora_engine* e, qora_kv* kv, const uint32_t* tokens, float* logits, uint32_t* argmax) {
  QCHECK(f16_tp_ready(e));
  for (uint32_t b = 0; b < kv->batch; ++b)
    if (tokens[b] >= e->vocab) return fail(QORA_ERR_RANGE, "token %u (row %u) >= vocab %u", tokens[b], b, e->vocab);
  std::vector<uint32_t> lens;
  QCHECK(f16_seq_lens(kv, lens));
  for (uint32_t b = 0; b < kv->batch; ++b)
    if (lens[b] >= kv->max_seq) return fail(QORA_ERR_RANGE, "sequence %u: KV cache full (%u positions)", b, kv->max_seq);
  QCUDA(cudaSetDevice(e->device));
  QCHECK(f16_ensure_graph(e, kv));
  QCHECK(f16_stage_decode_rows(e, kv, tokens, lens));
  QCUDA(cudaGraphLaunch(kv->f_graph, e->stream));
  if (logits)
    QCUDA(cudaMemcpyAsync(logits, e->f_logits, (size_t)kv->batch * e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
  if (argmax) QCUDA(cudaMemcpyAsync(argmax, kv->f_argmax, kv->batch * 4, cudaMemcpyDeviceToHost, e->stream));
  QCHECK(f16_check_error(e, kv));
  for (uint32_t b = 0; b < kv->batch; ++b)
    for (uint32_t l = 0; l < e->num_layers; ++l) kv->lenof(b, l) = lens[b] + 1;
  return QORA_OK;
}

// Greedy generation for every sequence of the cache: n_tokens batched steps on the
// device, each feeding its argmax back (f16b::advance_rows_kernel). out: [n_tokens][batch].
qora_status f16_generate(qora_engine* e, qora_kv* kv, const uint32_t* first, uint32_t n_tokens, uint32_t* out,
                         float* device_ms) {
  QCHECK(f16_tp_ready(e));
  for (uint32_t b = 0; b < kv->batch; ++b)
    if (first[b] >= e->vocab) return fail(QORA_ERR_RANGE, "token %u (row %u) >= vocab %u", first[b], b, e->vocab);
  std::vector<uint32_t> lens;
  QCHECK(f16_seq_lens(kv, lens));
  for (uint32_t b = 0; b < kv->batch; ++b)
    if ((uint64_t)lens[b] + n_tokens > kv->max_seq)
      return fail(QORA_ERR_RANGE, "sequence %u: %u tokens after %u positions exceed max_seq %u", b, n_tokens,
                  lens[b], kv->max_seq);
  if (n_tokens == 0) return QORA_OK;
  QCUDA(cudaSetDevice(e->device));
  QCHECK(f16_ensure_graph(e, kv));
  QCHECK(f16_stage_decode_rows(e, kv, first, lens));
  const f16b::RowInfo ri = f16b::row_info(kv->rows);
  cudaEvent_t a = nullptr, b = nullptr;
  if (device_ms) {
    QCUDA(cudaEventCreate(&a));
    QCUDA(cudaEventCreate(&b));
    QCUDA(cudaEventRecord(a, e->stream));
  }
  qora_status st = QORA_OK;
  for (uint32_t i = 0; i < n_tokens && st == QORA_OK; ++i) {
    cudaError_t ce = cudaGraphLaunch(kv->f_graph, e->stream);
    if (ce == cudaSuccess) {
      f16b::advance_rows_kernel<<<1, f16b::kMaxRows, 0, e->stream>>>((int)kv->batch, ri, kv->f_argmax, kv->ring,
                                                                   (int)kv->max_seq);
      ce = cudaGetLastError();
    }
    if (ce != cudaSuccess) st = fail(QORA_ERR_CUDA, "greedy step %u: %s", i, cudaGetErrorString(ce));
  }
  if (device_ms) {
    cudaEventRecord(b, e->stream);
    cudaError_t ce = cudaEventSynchronize(b);
    float ms = 0.0f;
    if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, a, b);
    cudaEventDestroy(a);
    cudaEventDestroy(b);
    if (st == QORA_OK && ce != cudaSuccess) st = fail(QORA_ERR_CUDA, "event timing: %s", cudaGetErrorString(ce));
    *device_ms = ms;
  }
  QCHECK(st);
  QCUDA(cudaMemcpyAsync(out, kv->ring, (size_t)n_tokens * kv->batch * 4, cudaMemcpyDeviceToHost, e->stream));
  QCHECK(f16_check_error(e, kv));
  for (uint32_t r = 0; r < kv->batch; ++r)
    for (uint32_t l = 0; l < e->num_layers; ++l) kv->lenof(r, l) = lens[r] + n_tokens;
  return QORA_OK;
}

__global__ void f16_prompt_rows_kernel(int* rows, const uint32_t* ids, int n, int seq, int pos0) {
  const f16b::RowInfo ri = f16b::row_info(rows);
  for (int m = threadIdx.x; m < n; m += blockDim.x) {
    ri.seq[m] = seq;
    ri.pos[m] = pos0 + m;
    ri.token[m] = (int)ids[m];
  }
  if (threadIdx.x == 0) *ri.error = 0;
}

// Prompt pass of one sequence in chunks of up to f16b::kMaxRows rows.
qora_status f16_prefill(qora_engine* e, qora_kv* kv, const uint32_t* ids, uint32_t n, uint32_t seq, float* logits,
                        uint32_t* argmax) {
  QCHECK(f16_tp_ready(e));
  std::vector<uint32_t> lens;
  QCHECK(f16_seq_lens(kv, lens));
  const uint32_t len = lens[seq];
  if ((uint64_t)len + n > kv->max_seq)
    return fail(QORA_ERR_RANGE, "prompt of %u after %u positions exceeds max_seq %u", n, len, kv->max_seq);
  QCUDA(cudaSetDevice(e->device));
  QCUDA(cudaMemcpyAsync(kv->ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
  for (uint32_t c0 = 0; c0 < n; c0 += f16b::kMaxRows) {
    const int c = (int)std::min<uint32_t>(f16b::kMaxRows, n - c0);
    f16_prompt_rows_kernel<<<1, f16b::kMaxRows, 0, e->stream>>>(kv->rows, kv->ids + c0, c, (int)seq, (int)(len + c0));
    QCUDA(cudaGetLastError());
    QCHECK(f16_forward(e, kv, c, c0 + c == n ? c - 1 : c));
  }
  if (logits) QCUDA(cudaMemcpyAsync(logits, e->f_logits, (size_t)e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
  if (argmax) QCUDA(cudaMemcpyAsync(argmax, kv->f_argmax, 4, cudaMemcpyDeviceToHost, e->stream));
  QCHECK(f16_check_error(e, kv));
  for (uint32_t l = 0; l < e->num_layers; ++l) kv->lenof(seq, l) = len + n;
  return QORA_OK;
}

// Q4 prompt of n >= 2 tokens on the tensor cores (q4_prefill_init): chunks of up to
// f16b::kMaxRows rows through the batched layer loop; the lm_head runs on the prompt's last
// row only. Leaves the step state as the token-by-token prefill does (pos = len + n,
// argmax = the greedy next token).
qora_status q4_prefill(qora_engine* e, qora_kv* kv, const uint32_t* ids, uint32_t n, float* logits,
                       uint32_t* argmax) {
  uint32_t len = 0;
  QCHECK(check_uniform_len(kv, &len));
  if ((uint64_t)len + n > kv->max_seq)
    return fail(QORA_ERR_RANGE, "prompt of %u after %u positions exceeds max_seq %u", n, len, kv->max_seq);
  QCUDA(cudaSetDevice(e->device));
  if (!kv->rows) {
    QCHECK(kv->alloc(&kv->rows, f16b::kRowInts));
    QCUDA(cudaMemset(kv->rows, 0, f16b::kRowInts * sizeof(int)));
    QCUDA(cudaMallocHost(&kv->rows_host, f16b::kRowInts * sizeof(int)));
    std::memset(kv->rows_host, 0, f16b::kRowInts * sizeof(int));
  }
  QCUDA(cudaMemcpyAsync(kv->ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
  QCHECK(set_state(e, kv, (int)(len + n), (int)ids[n - 1], 0));
  for (uint32_t c0 = 0; c0 < n; c0 += f16b::kMaxRows) {
    const int c = (int)std::min<uint32_t>(f16b::kMaxRows, n - c0);
    f16_prompt_rows_kernel<<<1, f16b::kMaxRows, 0, e->stream>>>(kv->rows, kv->ids + c0, c, 0, (int)(len + c0));
    QCUDA(cudaGetLastError());
    QCHECK(f16_forward(e, kv, c, c0 + c == n ? c - 1 : c));
  }
  QCUDA(cudaMemcpyAsync(kv->st_host, kv->st, sizeof(StepState), cudaMemcpyDeviceToHost, e->stream));
  if (logits) QCUDA(cudaMemcpyAsync(logits, e->logits, (size_t)e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
  QCHECK(f16_check_error(e, kv));
  if (argmax) *argmax = kv->st_host->argmax;
  for (auto& l : kv->len) l = len + n;
  return QORA_OK;
}

struct EntryScratch {
  float* partials = nullptr;
  size_t partial_floats = 0;
  unsigned* counters = nullptr;
  size_t ncounters = 0;
  uint64_t* tagged = nullptr;  // tagged split-K partials of the TMA GEMV (zero between launches)
  size_t ntagged = 0;
  float* lm_v = nullptr;
  unsigned* lm_i = nullptr;
  unsigned* lm_c = nullptr;
  int lm_n = 0;
  float* smp_work = nullptr;  // qora_sample_logits: [vocab] work row and the result slot
  size_t smp_n = 0;
  smp::Out* smp_out = nullptr;
};
std::mutex g_entry_mu;
std::map<int, EntryScratch> g_entry;

qora_status entry_scratch(int dev, size_t pf, size_t nc, int lm_n, EntryScratch** out, size_t nt = 0) {
  EntryScratch& s = g_entry[dev];
  if (s.ntagged < nt) {
    if (s.tagged) cudaFree(s.tagged);
    s.tagged = nullptr;
    QCUDA(cudaMalloc(&s.tagged, nt * sizeof(uint64_t)));
    QCUDA(cudaMemset(s.tagged, 0, nt * sizeof(uint64_t)));
    QCUDA(cudaDeviceSynchronize());  // zero before any stream's first launch (growth only)
    s.ntagged = nt;
  }
  if (s.partial_floats < pf) {
    if (s.partials) cudaFree(s.partials);
    s.partials = nullptr;
    QCUDA(cudaMalloc(&s.partials, pf * sizeof(float)));
    s.partial_floats = pf;
  }
  if (s.ncounters < nc) {
    if (s.counters) cudaFree(s.counters);
    s.counters = nullptr;
    QCUDA(cudaMalloc(&s.counters, nc * sizeof(unsigned)));
    QCUDA(cudaMemset(s.counters, 0, nc * sizeof(unsigned)));
    s.ncounters = nc;
  }
  if (s.lm_n < lm_n) {
    if (s.lm_v) cudaFree(s.lm_v);
    if (s.lm_i) cudaFree(s.lm_i);
    if (s.lm_c) cudaFree(s.lm_c);
    s.lm_v = nullptr;
    s.lm_i = nullptr;
    s.lm_c = nullptr;
    QCUDA(cudaMalloc(&s.lm_v, lm_n * sizeof(float)));
    QCUDA(cudaMalloc(&s.lm_i, lm_n * sizeof(unsigned)));
    QCUDA(cudaMalloc(&s.lm_c, sizeof(unsigned)));
    QCUDA(cudaMemset(s.lm_c, 0, sizeof(unsigned)));
    s.lm_n = lm_n;
  }
  *out = &s;
  return QORA_OK;
}


// ------------------------------------------------------------------ .qora reader
// load_model (src/save.rs:154-210) into host vectors, then the borrowed view.
// The file is memory-mapped read-only; the large arrays (Q4 nibbles, F16 weights) are
// used in place (they are only copied byte-wise: to the device, or into the re-tiling),
// the small ones (scales, norms, RoPE tables) are copied out aligned.
struct MappedFile {
  int fd = -1;
  const uint8_t* base = nullptr;
  size_t size = 0;
  ~MappedFile() {
    if (base) munmap(const_cast<uint8_t*>(base), size);
    if (fd >= 0) close(fd);
  }
};

struct FileMat {
  uint64_t k = 0, n = 0;
  const uint8_t* packed = nullptr;   // in the mapping
  std::vector<uint16_t> scales;
  const uint16_t* data = nullptr;    // in the mapping (read byte-wise only)
};
struct FileModel {
  MappedFile map;
  uint8_t format = 0;
  uint32_t num_layers = 0, vocab = 0, hidden = 0, half = 0;
  std::vector<uint8_t> no_rope;
  struct Layer {
    FileMat m[7];
    std::vector<uint16_t> g1, g2;
    uint32_t nh = 0, nkv = 0, hd = 0, grp = 0;
  };
  std::vector<Layer> layers;
  FileMat embed;
  std::vector<uint16_t> final_norm;
  std::vector<float> cos_t, sin_t;
};

struct FileReader {
  const uint8_t* p = nullptr;
  size_t left = 0;
  std::string err;
  bool ok = true;
  const uint8_t* take(size_t n) {  // n bytes at the cursor, or nullptr (short file)
    if (!ok) return nullptr;
    if (n > left) {
      ok = false;
      err = "short read";
      return nullptr;
    }
    const uint8_t* q = p;
    p += n;
    left -= n;
    return q;
  }
  template <typename T>
  T scalar() {
    T v{};
    if (const uint8_t* q = take(sizeof(T))) std::memcpy(&v, q, sizeof(T));
    return v;
  }
  uint32_t u32() { return scalar<uint32_t>(); }
  uint64_t u64() { return scalar<uint64_t>(); }
  uint8_t u8() { return scalar<uint8_t>(); }
  // length-prefixed array: its place in the mapping
  template <typename T>
  const uint8_t* span(uint64_t& len) {
    len = u64();
    if (!ok) return nullptr;
    if (len > (1ull << 36)) {
      ok = false;
      err = "implausible vector length";
      return nullptr;
    }
    return take(len * sizeof(T));
  }
  template <typename T>
  void vec(std::vector<T>& out) {
    uint64_t len = 0;
    const uint8_t* q = span<T>(len);
    if (!q) return;
    out.resize(len);
    if (len) std::memcpy(out.data(), q, len * sizeof(T));
  }
  void mat(uint8_t fmt, FileMat& m) {
    m.k = u64();
    m.n = u64();
    // bound the shape before any product of it (a wrapped k*n could match the stored size)
    if (ok && (m.k >= (1ull << 32) || m.n >= (1ull << 32) || m.k * m.n > (1ull << 40))) {
      ok = false;
      err = "implausible matrix shape";
      return;
    }
    if (fmt == 1) {
      uint64_t np = 0;
      m.packed = span<uint8_t>(np);
      vec(m.scales);
      if (ok && (m.n % kGroup || np != m.k * m.n / 2 || m.scales.size() != m.k * m.n / kGroup)) {
        ok = false;
        err = "q4 weight size mismatch";
      }
    } else if (fmt == 0) {
      uint64_t nd = 0;
      m.data = reinterpret_cast<const uint16_t*>(span<uint16_t>(nd));
      if (ok && nd != m.k * m.n) {
        ok = false;
        err = "f16 weight size mismatch";
      }
    } else {
      ok = false;
      err = "Unknown format id " + std::to_string(fmt);
    }
  }
};

qora_status read_qora_file(const char* path, FileModel& fm) {
  fm.map.fd = open(path, O_RDONLY);
  if (fm.map.fd < 0) return fail(QORA_ERR_IO, "cannot open %s", path);
  struct stat st{};
  if (fstat(fm.map.fd, &st) != 0) return fail(QORA_ERR_IO, "cannot stat %s", path);
  fm.map.size = (size_t)st.st_size;
  if (fm.map.size > 0) {
    void* base = mmap(nullptr, fm.map.size, PROT_READ, MAP_PRIVATE, fm.map.fd, 0);
    if (base == MAP_FAILED) return fail(QORA_ERR_IO, "cannot map %s", path);
    fm.map.base = static_cast<const uint8_t*>(base);
    madvise(base, fm.map.size, MADV_SEQUENTIAL);
  }
  FileReader r;
  r.p = fm.map.base;
  r.left = fm.map.size;
  const uint8_t* magic = r.take(4);
  if (r.ok && std::memcmp(magic, "QOR3", 4) != 0) { r.ok = false; r.err = "Invalid magic bytes"; }
  const uint32_t version = r.u32();
  if (r.ok && version != 1) { r.ok = false; r.err = "Unsupported version " + std::to_string(version) + ", expected 1"; }
  fm.format = r.u8();
  fm.num_layers = r.u32();
  fm.vocab = r.u32();
  fm.hidden = r.u32();
  fm.half = r.u32();
  r.vec(fm.no_rope);
  if (r.ok && fm.num_layers > 4096) { r.ok = false; r.err = "implausible layer count"; }
  if (r.ok) fm.layers.resize(fm.num_layers);
  for (uint32_t i = 0; r.ok && i < fm.num_layers; ++i) {
    auto& L = fm.layers[i];
    for (int w = 0; w < 7 && r.ok; ++w) r.mat(fm.format, L.m[w]);
    r.vec(L.g1);
    r.vec(L.g2);
    L.nh = r.u32();
    L.nkv = r.u32();
    L.hd = r.u32();
    L.grp = r.u32();
  }
  if (r.ok) r.mat(fm.format, fm.embed);
  r.vec(fm.final_norm);
  r.vec(fm.cos_t);
  r.vec(fm.sin_t);
  const bool io_short = !r.ok && r.err == "short read";
  if (!r.ok) return fail(io_short ? QORA_ERR_IO : QORA_ERR_INVALID, "%s: %s", path, r.err.c_str());
  if (fm.no_rope.size() != fm.num_layers) return fail(QORA_ERR_INVALID, "no_rope_layers length != num_layers");
  for (uint32_t i = 0; i < fm.num_layers; ++i) {
    if (fm.layers[i].g1.size() != fm.hidden || fm.layers[i].g2.size() != fm.hidden)
      return fail(QORA_ERR_INVALID, "layer %u norm length != hidden", i);
  }
  if (fm.final_norm.size() != fm.hidden) return fail(QORA_ERR_INVALID, "final norm length != hidden");
  if (fm.cos_t.size() != fm.sin_t.size() || fm.half == 0 || fm.cos_t.size() % fm.half)
    return fail(QORA_ERR_INVALID, "RoPE tables malformed");
  return QORA_OK;
}

qora_matrix_view mview(const FileMat& m) {
  qora_matrix_view v{};
  v.packed = m.packed;
  v.scales = m.scales.empty() ? nullptr : m.scales.data();
  v.data = m.data;
  v.k = m.k;
  v.n = m.n;
  return v;
}

}  // namespace

// ================================================================== C ABI
extern "C" {

const char* qora_last_error(void) { return g_last_error.c_str(); }

const char* qora_version(void) { return "qora-b200 0.1.0 (sm_100a)"; }

qora_status qora_engine_create(const qora_weights_view* weights, const qora_engine_options* opts,
                               qora_engine** out) {
  if (!out) return fail(QORA_ERR_INVALID, "out is NULL");
  *out = nullptr;
  QCHECK(validate_view(weights));
  const int n_gpus = opts ? opts->n_gpus : 1;
  if (n_gpus > 1)
    return fail(QORA_ERR_UNSUPPORTED,
                "single-process multi-GPU engines (n_gpus=%d) are not in this build; use tp_size/tp_rank with "
                "one engine per GPU",
                n_gpus);
  if (opts && (opts->flags & ~(QORA_FLAG_PER_OP_KERNELS | QORA_FLAG_TOKEN_PREFILL)))
    return fail(QORA_ERR_INVALID, "unknown option flags 0x%x", opts->flags);
  const int tp = (opts && opts->tp_size > 1) ? opts->tp_size : 1, rank = (opts && tp > 1) ? opts->tp_rank : 0;
  if (tp != 1 && tp != 2 && tp != 4 && tp != 8) return fail(QORA_ERR_INVALID, "tp_size %d (1, 2, 4 or 8)", tp);
  if (rank < 0 || rank >= tp) return fail(QORA_ERR_INVALID, "tp_rank %d of %d", rank, tp);
  if (tp > 1 && opts && (opts->flags & QORA_FLAG_PER_OP_KERNELS))
    return fail(QORA_ERR_UNSUPPORTED, "tensor-parallel engines run the persistent kernel only");
  int ndev = 0;
  QCUDA(cudaGetDeviceCount(&ndev));
  const int dev = opts ? opts->first_device : 0;
  if (dev < 0 || dev >= ndev) return fail(QORA_ERR_INVALID, "device %d out of range (%d devices)", dev, ndev);
  QCUDA(cudaSetDevice(dev));
  std::unique_ptr<qora_engine> e(new qora_engine());
  e->device = dev;
  e->tp = tp;
  e->rank = rank;
  e->use_mega = !(opts && (opts->flags & QORA_FLAG_PER_OP_KERNELS));
  e->want_q4p = !(opts && (opts->flags & QORA_FLAG_TOKEN_PREFILL));
  if (weights->format == QORA_FORMAT_F16)
    QCHECK(f16_engine_init(e.get(), weights));
  else
    QCHECK(engine_init(e.get(), weights));
  if (tp > 1 && weights->format == QORA_FORMAT_Q4 && !e->mk_ok)
    return fail(QORA_ERR_UNSUPPORTED, "tensor-parallel shard has no persistent kernel: %s", e->mk_why.c_str());
  *out = e.release();
  return QORA_OK;
}

qora_status qora_engine_create_from_file(const char* qora_path, const qora_engine_options* opts,
                                         qora_engine** out) {
  if (!qora_path || !out) return fail(QORA_ERR_INVALID, "NULL argument");
  *out = nullptr;
  FileModel fm;
  QCHECK(read_qora_file(qora_path, fm));
  std::vector<qora_layer_view> lv(fm.num_layers);
  for (uint32_t i = 0; i < fm.num_layers; ++i) {
    auto& L = fm.layers[i];
    qora_layer_view& v = lv[i];
    v.q_proj = mview(L.m[0]);
    v.k_proj = mview(L.m[1]);
    v.v_proj = mview(L.m[2]);
    v.o_proj = mview(L.m[3]);
    v.gate_proj = mview(L.m[4]);
    v.up_proj = mview(L.m[5]);
    v.down_proj = mview(L.m[6]);
    v.input_norm_gamma = L.g1.data();
    v.post_attn_norm_gamma = L.g2.data();
    v.num_heads = L.nh;
    v.num_kv_heads = L.nkv;
    v.head_dim = L.hd;
    v.num_kv_groups = L.grp;
  }
  qora_weights_view w{};
  w.format = fm.format;
  w.num_layers = fm.num_layers;
  w.vocab = fm.vocab;
  w.hidden = fm.hidden;
  w.rope_half_dim = fm.half;
  w.no_rope_layers = fm.no_rope.data();
  w.layers = lv.data();
  w.embed = mview(fm.embed);
  w.final_norm_gamma = fm.final_norm.data();
  w.rope_cos = fm.cos_t.data();
  w.rope_sin = fm.sin_t.data();
  w.rope_rows = fm.cos_t.size() / fm.half;
  return qora_engine_create(&w, opts, out);
}

void qora_engine_destroy(qora_engine* engine) {
  if (!engine) return;
  cudaSetDevice(engine->device);
  delete engine;
}

namespace {
struct TpBlob {  // what one rank hands to the others
  uint32_t magic, tp, rank, pad;
  uint64_t region_bytes;
  cudaIpcMemHandle_t handle;
};
constexpr uint32_t kTpMagic = 0x51545031u;  // "QTP1"
}  // namespace

qora_status qora_tp_export(qora_engine* e, void* buf, size_t cap, size_t* len) {
  if (!e || !len) return fail(QORA_ERR_INVALID, "NULL argument");
  if (e->tp < 2) return fail(QORA_ERR_INVALID, "not a tensor-parallel engine");
  *len = sizeof(TpBlob);
  if (!buf) return QORA_OK;
  if (cap < sizeof(TpBlob)) return fail(QORA_ERR_INVALID, "buffer of %zu bytes, need %zu", cap, sizeof(TpBlob));
  QCUDA(cudaSetDevice(e->device));
  TpBlob b{};
  b.magic = kTpMagic;
  b.tp = (uint32_t)e->tp;
  b.rank = (uint32_t)e->rank;
  b.region_bytes = e->tp_region_bytes;
  QCUDA(cudaIpcGetMemHandle(&b.handle, e->tp_region));
  std::memcpy(buf, &b, sizeof(b));
  return QORA_OK;
}

qora_status qora_tp_connect(qora_engine* e, const void* handles, size_t len_per_rank) {
  if (!e || !handles) return fail(QORA_ERR_INVALID, "NULL argument");
  if (e->tp < 2) return fail(QORA_ERR_INVALID, "not a tensor-parallel engine");
  if (e->tp_connected) return fail(QORA_ERR_INVALID, "already connected");
  if (len_per_rank != sizeof(TpBlob)) return fail(QORA_ERR_INVALID, "handle size %zu, expected %zu", len_per_rank,
                                                   sizeof(TpBlob));
  QCUDA(cudaSetDevice(e->device));
  std::vector<TpBlob> bs(e->tp);
  std::memcpy(bs.data(), handles, sizeof(TpBlob) * e->tp);
  for (int p = 0; p < e->tp; ++p)
    if (bs[p].magic != kTpMagic || (int)bs[p].tp != e->tp || (int)bs[p].rank != p ||
        bs[p].region_bytes != e->tp_region_bytes)
      return fail(QORA_ERR_INVALID, "handle %d is not rank %d of this %d-way group", p, p, e->tp);
  std::vector<void*> opened;
  for (int p = 0; p < e->tp; ++p) {
    if (p == e->rank) {
      e->tp_peer[p] = e->tp_region;
      continue;
    }
    void* ptr = nullptr;
    const cudaError_t ce = cudaIpcOpenMemHandle(&ptr, bs[p].handle, cudaIpcMemLazyEnablePeerAccess);
    if (ce != cudaSuccess) {
      for (void* q : opened) cudaIpcCloseMemHandle(q);
      return fail(QORA_ERR_CUDA, "opening rank %d's buffers: %s", p, cudaGetErrorString(ce));
    }
    opened.push_back(ptr);
    e->tp_peer[p] = static_cast<uint8_t*>(ptr);
  }
  e->tp_opened = opened;
  e->tp_connected = true;
  for (qora_kv* kv : e->kvs) kv->mk_ready = false;  // rebuild kernel arguments with the peers
  return QORA_OK;
}

qora_status qora_tp_plan(uint32_t format, uint32_t num_heads, uint32_t num_kv_heads, uint32_t intermediate,
                         uint32_t vocab, int32_t tp_size, int32_t tp_rank, qora_tp_shard* out) {
  if (!out) return fail(QORA_ERR_INVALID, "NULL argument");
  if (format != QORA_FORMAT_Q4 && format != QORA_FORMAT_F16) return fail(QORA_ERR_INVALID, "format %u", format);
  return tp_plan(format, num_heads, num_kv_heads, intermediate, vocab, tp_size, tp_rank, out);
}

qora_status qora_engine_info(const qora_engine* e, uint32_t* num_layers, uint32_t* vocab,
                             uint32_t* hidden, uint32_t* format, uint64_t* device_bytes) {
  if (!e) return fail(QORA_ERR_INVALID, "engine is NULL");
  if (num_layers) *num_layers = e->num_layers;
  if (vocab) *vocab = e->vocab;
  if (hidden) *hidden = e->hidden;
  if (format) *format = e->format;
  if (device_bytes) *device_bytes = e->device_bytes;
  return QORA_OK;
}

qora_status qora_kv_create(qora_engine* e, uint32_t max_seq, uint32_t batch, qora_kv** out) {
  return qora_kv_create_ex(e, max_seq, batch, QORA_KV_F32, out);
}

qora_status qora_kv_create_ex(qora_engine* e, uint32_t max_seq, uint32_t batch, uint32_t kv_dtype, qora_kv** out) {
  if (!e || !out) return fail(QORA_ERR_INVALID, "NULL argument");
  *out = nullptr;
  const bool f16 = e->format == QORA_FORMAT_F16;
  if (kv_dtype != QORA_KV_F32 && kv_dtype != QORA_KV_F16) return fail(QORA_ERR_INVALID, "kv_dtype %u", kv_dtype);
  if (batch == 0) return fail(QORA_ERR_INVALID, "batch must be > 0");
  if (!f16 && batch != 1) return fail(QORA_ERR_UNSUPPORTED, "batch=%u: Q4 engines decode batch 1", batch);
  if (batch > (uint32_t)f16b::kMaxRows)
    return fail(QORA_ERR_UNSUPPORTED, "batch=%u: at most %d sequences", batch, f16b::kMaxRows);
  if (max_seq == 0) return fail(QORA_ERR_INVALID, "max_seq must be > 0");
  if (kv_dtype == QORA_KV_F16 && (f16 || !e->use_mega || !e->mk_ok || e->tp > 1 || max_seq > e->mk_max_seq))
    return fail(QORA_ERR_UNSUPPORTED,
                "binary16 KV caches need a Q4 engine on the persistent step, tp_size 1 and max_seq <= %u",
                e->mk_max_seq);
  bool any_rope = false;
  for (auto& L : e->layers) any_rope |= (L.rope != 0);
  for (auto& L : e->fl) any_rope |= (L.rope != 0);
  if (any_rope && max_seq > e->rope_rows)
    return fail(QORA_ERR_RANGE, "max_seq %u exceeds the %u RoPE table rows", max_seq, e->rope_rows);
  QCUDA(cudaSetDevice(e->device));
  std::unique_ptr<qora_kv> kv(new qora_kv());
  kv->e = e;
  kv->max_seq = max_seq;
  kv->batch = batch;
  kv->dtype = kv_dtype;
  kv->len.assign((size_t)batch * e->num_layers, 0);
  const size_t per = (kv->layer_stride() * e->num_layers * kv->esz() + 3) / 4;  // in floats
  QCHECK(kv->alloc(&kv->k, per));
  QCHECK(kv->alloc(&kv->v, per));
  QCHECK(kv->alloc(&kv->st, 1));
  QCHECK(kv->alloc(&kv->ring, (size_t)max_seq * batch));
  QCHECK(kv->alloc(&kv->ids, max_seq));
  QCUDA(cudaMallocHost(&kv->st_host, sizeof(StepState)));
  if (f16) {
    QCHECK(kv->alloc(&kv->rows, f16b::kRowInts));
    QCHECK(kv->alloc(&kv->f_argmax, f16b::kMaxRows));
    QCUDA(cudaMemset(kv->rows, 0, f16b::kRowInts * sizeof(int)));
    QCUDA(cudaMallocHost(&kv->rows_host, f16b::kRowInts * sizeof(int)));
    std::memset(kv->rows_host, 0, f16b::kRowInts * sizeof(int));
    QCUDA(cudaMemset(kv->st, 0, sizeof(StepState)));
    QCUDA(cudaDeviceSynchronize());
    e->kvs.push_back(kv.get());
    *out = kv.release();
    return QORA_OK;
  }
  kv->attn_nc = std::max<int>(std::max(1, e->sms / (int)e->nkv), (int)((max_seq + kAttnMaxChunk - 1) / kAttnMaxChunk));
  QCHECK(kv->alloc(&kv->attn_o, (size_t)e->nkv * kv->attn_nc * kGrp * kHeadDim));
  QCHECK(kv->alloc(&kv->attn_ml, (size_t)e->nkv * kv->attn_nc * kGrp * 2));
  QCHECK(kv->alloc(&kv->attn_counters, e->nkv));
  QCUDA(cudaMemset(kv->attn_counters, 0, e->nkv * sizeof(unsigned)));
  QCUDA(cudaMemset(kv->st, 0, sizeof(StepState)));
  QCUDA(cudaDeviceSynchronize());
  e->kvs.push_back(kv.get());
  *out = kv.release();
  return QORA_OK;
}

void qora_kv_destroy(qora_kv* kv) { delete kv; }

qora_status qora_kv_length(const qora_kv* kv, uint32_t seq_idx, uint32_t* len) {
  if (!kv || !len) return fail(QORA_ERR_INVALID, "NULL argument");
  if (seq_idx >= kv->batch) return fail(QORA_ERR_RANGE, "seq_idx %u of %u sequences", seq_idx, kv->batch);
  *len = kv->len[(size_t)seq_idx * (kv->len.size() / kv->batch)];
  return QORA_OK;
}

qora_status qora_kv_reset(qora_kv* kv, uint32_t seq_idx) {
  if (!kv) return fail(QORA_ERR_INVALID, "NULL kv");
  if (seq_idx >= kv->batch) return fail(QORA_ERR_RANGE, "seq_idx %u of %u sequences", seq_idx, kv->batch);
  const size_t L = kv->len.size() / kv->batch;
  std::fill(kv->len.begin() + seq_idx * L, kv->len.begin() + (seq_idx + 1) * L, 0u);
  return QORA_OK;
}

// Import (to_device) or export one layer of a binary16 cache through an f32 device
// staging buffer of the host rows [seq_len][nkv_total*128]; the conversion kernels round
// to nearest even on the way in and widen exactly on the way out.
static qora_status kv_f16_transfer(qora_kv* kv, uint32_t layer, float* k, float* v, uint32_t seq_len,
                                   uint32_t seq_idx, bool to_device) {
  if (seq_len == 0) return QORA_OK;
  qora_engine* e = kv->e;
  const size_t row_floats = (size_t)e->nkv_total * kHeadDim, n = (size_t)seq_len * row_floats;
  float* tmp = nullptr;
  cudaError_t err = cudaMalloc(&tmp, n * sizeof(float));
  if (err != cudaSuccess) return fail(QORA_ERR_OOM, "cudaMalloc(%zu) failed: %s", n * 4, cudaGetErrorString(err));
  std::unique_ptr<float, decltype(&cudaFree)> guard(tmp, &cudaFree);
  const long long hs = (long long)kv->max_seq * kHeadDim;
  const size_t off = seq_idx * kv->seq_stride();  // elements, within the layer
  const int grid = e->sms * 4;
  for (int side = 0; side < 2; ++side) {
    float* host = side ? v : k;
    __half* dev = static_cast<__half*>(side ? kv->v_layer(layer) : kv->k_layer(layer)) + off;
    if (to_device) {
      QCUDA(cudaMemcpy(tmp, host, n * sizeof(float), cudaMemcpyHostToDevice));
      kv_pack_f16_kernel<<<grid, 256>>>(tmp, (int)row_floats, (int)e->kv0, (int)e->nkv, (int)seq_len, dev, hs);
      QCUDA(cudaGetLastError());
      QCUDA(cudaDeviceSynchronize());
    } else {  // the rank's own heads' columns of the host rows
      kv_unpack_f16_kernel<<<grid, 256>>>(dev, hs, (int)e->nkv, (int)seq_len, tmp);
      QCUDA(cudaGetLastError());
      const size_t lb = (size_t)e->nkv * kHeadDim * sizeof(float);
      QCUDA(cudaMemcpy2D(host + (size_t)e->kv0 * kHeadDim, row_floats * sizeof(float), tmp, lb, lb, seq_len,
                         cudaMemcpyDeviceToHost));
    }
  }
  return QORA_OK;
}

qora_status qora_kv_import(qora_kv* kv, uint32_t layer, const float* k, const float* v,
                           uint32_t seq_len, uint32_t seq_idx) {
  if (!kv || (!k && seq_len) || (!v && seq_len)) return fail(QORA_ERR_INVALID, "NULL argument");
  if (!kv->e) return fail(QORA_ERR_INVALID, "the KV cache's engine was destroyed");
  if (seq_idx >= kv->batch) return fail(QORA_ERR_RANGE, "seq_idx %u of %u sequences", seq_idx, kv->batch);
  if (layer >= kv->e->num_layers) return fail(QORA_ERR_RANGE, "layer %u", layer);
  if (seq_len > kv->max_seq) return fail(QORA_ERR_RANGE, "seq_len %u > max_seq %u", seq_len, kv->max_seq);
  QCUDA(cudaSetDevice(kv->e->device));
  if (kv->dtype == QORA_KV_F16) {
    QCHECK(kv_f16_transfer(kv, layer, const_cast<float*>(k), const_cast<float*>(v), seq_len, seq_idx, true));
    kv->lenof(seq_idx, layer) = seq_len;
    return QORA_OK;
  }
  // host rows [seq][all kv heads*128] -> device head-major [local kv heads][max_seq][128]
  // (a tensor-parallel rank keeps heads kv0 .. kv0 + nkv - 1)
  const size_t row = (size_t)kv->e->nkv_total * kHeadDim * sizeof(float), hb = kHeadDim * sizeof(float);
  for (uint32_t j = 0; seq_len && j < kv->e->nkv; ++j) {
    const size_t off = layer * kv->layer_stride() + seq_idx * kv->seq_stride() + (size_t)j * kv->max_seq * kHeadDim;
    const size_t src = (size_t)(kv->e->kv0 + j) * kHeadDim;
    QCUDA(cudaMemcpy2D(kv->k + off, hb, k + src, row, hb, seq_len, cudaMemcpyHostToDevice));
    QCUDA(cudaMemcpy2D(kv->v + off, hb, v + src, row, hb, seq_len, cudaMemcpyHostToDevice));
  }
  kv->lenof(seq_idx, layer) = seq_len;
  return QORA_OK;
}

qora_status qora_kv_export(const qora_kv* kv, uint32_t layer, float* k, float* v, uint32_t seq_len,
                           uint32_t seq_idx) {
  if (!kv || !k || !v) return fail(QORA_ERR_INVALID, "NULL argument");
  if (!kv->e) return fail(QORA_ERR_INVALID, "the KV cache's engine was destroyed");
  if (seq_idx >= kv->batch) return fail(QORA_ERR_RANGE, "seq_idx %u of %u sequences", seq_idx, kv->batch);
  if (layer >= kv->e->num_layers) return fail(QORA_ERR_RANGE, "layer %u", layer);
  const uint32_t have = kv->len[(size_t)seq_idx * (kv->len.size() / kv->batch) + layer];
  if (seq_len > have) return fail(QORA_ERR_RANGE, "seq_len %u > length %u", seq_len, have);
  QCUDA(cudaSetDevice(kv->e->device));
  QCUDA(cudaStreamSynchronize(kv->e->stream));
  if (kv->dtype == QORA_KV_F16) return kv_f16_transfer(const_cast<qora_kv*>(kv), layer, k, v, seq_len, seq_idx, false);
  const size_t row = (size_t)kv->e->nkv_total * kHeadDim * sizeof(float), hb = kHeadDim * sizeof(float);
  for (uint32_t j = 0; seq_len && j < kv->e->nkv; ++j) {  // a rank fills only its own heads' columns
    const size_t off = layer * kv->layer_stride() + seq_idx * kv->seq_stride() + (size_t)j * kv->max_seq * kHeadDim;
    const size_t dst = (size_t)(kv->e->kv0 + j) * kHeadDim;
    QCUDA(cudaMemcpy2D(k + dst, row, kv->k + off, hb, hb, seq_len, cudaMemcpyDeviceToHost));
    QCUDA(cudaMemcpy2D(v + dst, row, kv->v + off, hb, hb, seq_len, cudaMemcpyDeviceToHost));
  }
  return QORA_OK;
}

qora_status qora_decode_step(qora_engine* e, qora_kv* kv, const uint32_t* tokens,
                             float* logits_or_null, uint32_t* argmax_out) {
  if (!e || !kv || !tokens || kv->e != e) return fail(QORA_ERR_INVALID, "bad engine/kv/tokens");
  if (e->format == QORA_FORMAT_F16) return f16_decode_step(e, kv, tokens, logits_or_null, argmax_out);
  if (tokens[0] >= e->vocab) return fail(QORA_ERR_RANGE, "token %u >= vocab %u", tokens[0], e->vocab);
  uint32_t len = 0;
  QCHECK(check_uniform_len(kv, &len));
  if (len >= kv->max_seq) return fail(QORA_ERR_RANGE, "KV cache full (%u positions)", kv->max_seq);
  QCUDA(cudaSetDevice(e->device));
  QCHECK(step_prepare(e, kv));
  QCHECK(set_state(e, kv, (int)len, (int)tokens[0], 0));
  QCHECK(step_launch(e, kv));
  QCUDA(cudaMemcpyAsync(kv->st_host, kv->st, sizeof(StepState), cudaMemcpyDeviceToHost, e->stream));
  if (logits_or_null)
    QCUDA(cudaMemcpyAsync(logits_or_null, e->logits, (size_t)e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaStreamSynchronize(e->stream));
  if (kv->st_host->error == 2) return fail(QORA_ERR_TIMEOUT, "a bounded device-side wait timed out");
  if (kv->st_host->error) return fail(QORA_ERR_RANGE, "device rejected token id");
  if (argmax_out) argmax_out[0] = kv->st_host->argmax;
  for (auto& l : kv->len) l = len + 1;
  return QORA_OK;
}

qora_status qora_prefill(qora_engine* e, qora_kv* kv, const uint32_t* ids, uint32_t n,
                         uint32_t seq_idx, float* logits_or_null, uint32_t* argmax_out) {
  if (!e || !kv || kv->e != e || (!ids && n)) return fail(QORA_ERR_INVALID, "bad arguments");
  if (seq_idx >= kv->batch) return fail(QORA_ERR_RANGE, "seq_idx %u of %u sequences", seq_idx, kv->batch);
  if (n == 0) return fail(QORA_ERR_INVALID, "empty prompt");
  for (uint32_t i = 0; i < n; ++i)
    if (ids[i] >= e->vocab) return fail(QORA_ERR_RANGE, "token %u at %u >= vocab %u", ids[i], i, e->vocab);
  if (e->format == QORA_FORMAT_F16) return f16_prefill(e, kv, ids, n, seq_idx, logits_or_null, argmax_out);
  if (e->q4p && n >= 2 && kv->dtype == QORA_KV_F32) return q4_prefill(e, kv, ids, n, logits_or_null, argmax_out);
  uint32_t len = 0;
  QCHECK(check_uniform_len(kv, &len));
  if ((uint64_t)len + n > kv->max_seq)
    return fail(QORA_ERR_RANGE, "prompt of %u after %u positions exceeds max_seq %u", n, len, kv->max_seq);
  QCUDA(cudaSetDevice(e->device));
  QCHECK(step_prepare(e, kv));
  QCUDA(cudaMemcpyAsync(kv->ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, e->stream));
  QCHECK(set_state(e, kv, (int)len, (int)ids[0], 0));
  for (uint32_t i = 0; i < n; ++i) {
    QCUDA(cudaMemcpyAsync(&kv->st->token, kv->ids + i, 4, cudaMemcpyDeviceToDevice, e->stream));
    QCHECK(step_launch(e, kv, i + 1 == n));
  }
  QCUDA(cudaMemcpyAsync(kv->st_host, kv->st, sizeof(StepState), cudaMemcpyDeviceToHost, e->stream));
  if (logits_or_null)
    QCUDA(cudaMemcpyAsync(logits_or_null, e->logits, (size_t)e->vocab * 4, cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaStreamSynchronize(e->stream));
  if (kv->st_host->error == 2) return fail(QORA_ERR_TIMEOUT, "a bounded device-side wait timed out");
  if (kv->st_host->error) return fail(QORA_ERR_RANGE, "device rejected token id");
  if (argmax_out) *argmax_out = kv->st_host->argmax;
  for (auto& l : kv->len) l = len + n;
  return QORA_OK;
}

qora_status qora_generate_greedy(qora_engine* e, qora_kv* kv, uint32_t first_token,
                                 uint32_t n_tokens, uint32_t* out_tokens) {
  if (!e || !kv || kv->e != e || (!out_tokens && n_tokens)) return fail(QORA_ERR_INVALID, "bad arguments");
  if (first_token >= e->vocab) return fail(QORA_ERR_RANGE, "token %u >= vocab", first_token);
  if (kv->batch != 1) return fail(QORA_ERR_INVALID, "batched cache: use qora_generate_greedy_batch");
  if (e->format == QORA_FORMAT_F16) return f16_generate(e, kv, &first_token, n_tokens, out_tokens, nullptr);
  uint32_t len = 0;
  QCHECK(check_uniform_len(kv, &len));
  if ((uint64_t)len + n_tokens > kv->max_seq)
    return fail(QORA_ERR_RANGE, "%u tokens after %u positions exceed max_seq %u", n_tokens, len, kv->max_seq);
  if (n_tokens == 0) return QORA_OK;
  QCUDA(cudaSetDevice(e->device));
  QCHECK(step_prepare(e, kv));
  QCHECK(set_state(e, kv, (int)len, (int)first_token, 0));
  for (uint32_t i = 0; i < n_tokens; ++i) QCHECK(step_launch(e, kv, false));
  QCUDA(cudaMemcpyAsync(out_tokens, kv->ring, (size_t)n_tokens * 4, cudaMemcpyDeviceToHost, e->stream));
  QCHECK(check_step_error(e, kv));
  for (auto& l : kv->len) l = len + n_tokens;
  return QORA_OK;
}

qora_status qora_layer_step(qora_engine* e, qora_kv* kv, uint32_t layer, float* x_inout) {
  if (!e || !kv || kv->e != e || !x_inout) return fail(QORA_ERR_INVALID, "bad arguments");
  if (e->format != QORA_FORMAT_Q4) return fail(QORA_ERR_UNSUPPORTED, "qora_layer_step runs Q4 engines");
  if (kv->dtype != QORA_KV_F32) return fail(QORA_ERR_UNSUPPORTED, "qora_layer_step runs f32 KV caches");
  if (layer >= e->num_layers) return fail(QORA_ERR_RANGE, "layer %u", layer);
  const uint32_t len = kv->len[layer];
  if (len >= kv->max_seq) return fail(QORA_ERR_RANGE, "KV cache full");
  QCUDA(cudaSetDevice(e->device));
  QCUDA(cudaMemcpyAsync(e->x, x_inout, (size_t)e->hidden * 4, cudaMemcpyHostToDevice, e->stream));
  QCHECK(set_state(e, kv, (int)len, 0, 0));
  QCHECK(launch_layer(e, kv, layer));
  QCUDA(cudaMemcpyAsync(x_inout, e->x, (size_t)e->hidden * 4, cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaStreamSynchronize(e->stream));
  kv->len[layer] = len + 1;
  return QORA_OK;
}

qora_status qora_generate_greedy_timed(qora_engine* e, qora_kv* kv, uint32_t first_token,
                                       uint32_t n_tokens, uint32_t* out_tokens, float* device_ms) {
  if (!e || !kv || kv->e != e || (!out_tokens && n_tokens) || !device_ms)
    return fail(QORA_ERR_INVALID, "bad arguments");
  if (first_token >= e->vocab) return fail(QORA_ERR_RANGE, "token %u >= vocab", first_token);
  if (kv->batch != 1) return fail(QORA_ERR_INVALID, "batched cache: use qora_generate_greedy_batch");
  if (e->format == QORA_FORMAT_F16) return f16_generate(e, kv, &first_token, n_tokens, out_tokens, device_ms);
  uint32_t len = 0;
  QCHECK(check_uniform_len(kv, &len));
  if ((uint64_t)len + n_tokens > kv->max_seq)
    return fail(QORA_ERR_RANGE, "%u tokens after %u positions exceed max_seq %u", n_tokens, len, kv->max_seq);
  QCUDA(cudaSetDevice(e->device));
  QCHECK(step_prepare(e, kv));
  QCHECK(set_state(e, kv, (int)len, (int)first_token, 0));
  cudaEvent_t a = nullptr, b = nullptr;
  QCUDA(cudaEventCreate(&a));
  QCUDA(cudaEventCreate(&b));
  cudaEventRecord(a, e->stream);
  for (uint32_t i = 0; i < n_tokens; ++i) {
    const qora_status ls = step_launch(e, kv, false);
    if (ls != QORA_OK) {
      cudaEventDestroy(a);
      cudaEventDestroy(b);
      return ls;
    }
  }
  cudaEventRecord(b, e->stream);
  cudaError_t ce = cudaEventSynchronize(b);
  float ms = 0.0f;
  if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  if (ce != cudaSuccess) return fail(QORA_ERR_CUDA, "event timing: %s", cudaGetErrorString(ce));
  *device_ms = ms;
  if (n_tokens)
    QCUDA(cudaMemcpyAsync(out_tokens, kv->ring, (size_t)n_tokens * 4, cudaMemcpyDeviceToHost, e->stream));
  QCHECK(check_step_error(e, kv));
  for (auto& l : kv->len) l = len + n_tokens;
  return QORA_OK;
}

qora_status qora_engine_time_kernel(qora_engine* e, qora_kv* kv, int kernel, uint32_t reps,
                                    float* ms_per_launch, uint64_t* bytes_per_launch,
                                    uint32_t* launches) {
  if (!e || !kv || kv->e != e || !ms_per_launch || reps == 0) return fail(QORA_ERR_INVALID, "bad arguments");
  if (e->format != QORA_FORMAT_Q4) return fail(QORA_ERR_UNSUPPORTED, "kernel timing runs Q4 engines");
  if (kv->dtype != QORA_KV_F32) return fail(QORA_ERR_UNSUPPORTED, "kernel timing runs f32 KV caches");
  if (kernel < QORA_KERNEL_QKV || kernel > QORA_KERNEL_LM_HEAD) return fail(QORA_ERR_INVALID, "kernel %d", kernel);
  uint32_t len = 0;
  QCHECK(check_uniform_len(kv, &len));
  if (len >= kv->max_seq) return fail(QORA_ERR_RANGE, "KV cache full");
  QCUDA(cudaSetDevice(e->device));
  QCHECK(set_state(e, kv, (int)len, 0, 0));
  const uint64_t H = e->hidden, I = e->inter, nq = (uint64_t)e->nh * kHeadDim, nk = (uint64_t)e->nkv * kHeadDim;
  auto q4b = [](uint64_t k, uint64_t n) { return k * n / 2 + k * n / kGroup * 2; };
  uint64_t bytes = 0;
  switch (kernel) {
    case QORA_KERNEL_QKV: bytes = q4b(H, nq + 2 * nk) + 2 * H * 4 + (nq + 2 * nk) * 4; break;
    case QORA_KERNEL_ATTENTION: bytes = (uint64_t)(len + 1) * 2 * nk * 4 + 2 * nq * 4; break;
    case QORA_KERNEL_O: bytes = q4b(nq, H) + nq * 4 + 2 * H * 4; break;
    case QORA_KERNEL_GATE_UP: bytes = 2 * q4b(H, I) + 2 * H * 4 + I * 4; break;
    case QORA_KERNEL_DOWN: bytes = q4b(I, H) + I * 4 + 2 * H * 4; break;
    case QORA_KERNEL_LM_HEAD: bytes = q4b(e->vocab, H) + 2 * H * 4 + (uint64_t)e->vocab * 4; break;
  }
  auto run_once = [&](uint32_t li) -> qora_status {
    const LayerDev& d = e->layers[li];
    cudaStream_t s = e->stream;
    float* kc = kv->k + li * kv->layer_stride();
    float* vc = kv->v + li * kv->layer_stride();
    switch (kernel) {
      case QORA_KERNEL_QKV: {
        EpiQKV eq{e->q, kc, vc, (long long)kv->max_seq * kHeadDim, kv->st, e->rope_cos, e->rope_sin, d.nq, d.nkv, d.rope,
                  (int)std::min<uint32_t>(kv->max_seq, d.rope ? e->rope_rows : kv->max_seq)};
        return launch_gemv(d.qkv.src(), e->sh_qkv, e->partials, e->counters,
                           ProNorm{e->x, d.g_in, (int)e->hidden}, eq, s);
      }
      case QORA_KERNEL_ATTENTION: {
        AttnArgs aa{};
        aa.q = e->q; aa.kc = kc; aa.vc = vc; aa.hs = (long long)kv->max_seq * kHeadDim;
        aa.out = e->attn; aa.st = kv->st;
        aa.nkv = (int)e->nkv; aa.nc = kv->attn_nc; aa.scale = 1.0f / std::sqrt((float)kHeadDim);
        aa.part_o = kv->attn_o; aa.part_ml = kv->attn_ml; aa.counters = kv->attn_counters;
        attn_decode_kernel<<<dim3(e->nkv, kv->attn_nc), kAttnThreads, 0, s>>>(aa);
        QCUDA(cudaGetLastError());
        return QORA_OK;
      }
      case QORA_KERNEL_O:
        return launch_gemv(d.o.src(), e->sh_o, e->partials, e->counters, ProPlain{e->attn},
                           EpiResidual{e->x, (int)e->hidden}, s);
      case QORA_KERNEL_GATE_UP:
        return launch_gemv(d.gu.src(), e->sh_gu, e->partials, e->counters,
                           ProNorm{e->x, d.g_post, (int)e->hidden}, EpiSwiGLU{e->h, (int)e->inter}, s);
      case QORA_KERNEL_DOWN:
        return launch_gemv(d.down.src(), e->sh_down, e->partials, e->counters, ProPlain{e->h},
                           EpiResidual{e->x, (int)e->hidden}, s);
      default: {
        LmArgs la{};
        la.x = e->x; la.gamma = e->final_gamma; la.packed = e->lm_table; la.scales = e->lm_table + e->hidden / 2;
        la.row_stride_p = la.row_stride_s = e->lm_row_bytes;
        la.vocab = (int)e->vocab; la.logits = e->logits; la.argmax_out = &kv->st->argmax;
        la.part_v = e->lm_part_v; la.part_i = e->lm_part_i; la.counter = e->lm_counter;
        return launch_lm_head((int)e->hidden, la, e->lm_ctas, s);
      }
    }
  };
  const uint32_t per_rep = (kernel == QORA_KERNEL_LM_HEAD) ? 1 : e->num_layers;
  for (uint32_t li = 0; li < per_rep; ++li) QCHECK(run_once(li));  // warm-up pass
  cudaEvent_t a = nullptr, b = nullptr;
  QCUDA(cudaEventCreate(&a));
  QCUDA(cudaEventCreate(&b));
  cudaEventRecord(a, e->stream);
  qora_status st = QORA_OK;
  for (uint32_t r = 0; r < reps && st == QORA_OK; ++r)
    for (uint32_t li = 0; li < per_rep && st == QORA_OK; ++li) st = run_once(li);
  cudaEventRecord(b, e->stream);
  cudaError_t ce = cudaEventSynchronize(b);
  float ms = 0.0f;
  if (ce == cudaSuccess) ce = cudaEventElapsedTime(&ms, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  QCHECK(st);
  if (ce != cudaSuccess) return fail(QORA_ERR_CUDA, "event timing: %s", cudaGetErrorString(ce));
  *ms_per_launch = ms / (float)(reps * per_rep);
  if (bytes_per_launch) *bytes_per_launch = bytes;
  if (launches) *launches = reps * per_rep;
  return QORA_OK;
}

qora_status qora_engine_set_trace(qora_engine* e, int enable) {
  if (!e) return fail(QORA_ERR_INVALID, "NULL engine");
  if (!e->mk_ok) return fail(QORA_ERR_UNSUPPORTED, "no persistent decode kernel: %s", e->mk_why.c_str());
  QCUDA(cudaSetDevice(e->device));
  if (enable && !e->mk_trace) {
    e->mk_trace_n = (size_t)e->mk_G * (mk::kTracePerCta + mk::kTraceLayers + mk::kTraceFine);
    QCHECK(e->alloc(&e->mk_trace, e->mk_trace_n));
    QCUDA(cudaMemset(e->mk_trace, 0, e->mk_trace_n * 8));
  }
  unsigned long long* t = enable ? e->mk_trace : nullptr;
  for (qora_kv* kv : e->kvs) kv->mk_args.trace = t;
  return QORA_OK;
}

qora_status qora_engine_get_trace(qora_engine* e, uint64_t* out, size_t cap, size_t* n) {
  if (!e || !n) return fail(QORA_ERR_INVALID, "NULL argument");
  *n = e->mk_trace ? e->mk_trace_n : 0;
  if (!e->mk_trace || !out) return QORA_OK;
  QCUDA(cudaSetDevice(e->device));
  QCUDA(cudaStreamSynchronize(e->stream));
  QCUDA(cudaMemcpy(out, e->mk_trace, std::min(cap, e->mk_trace_n) * 8, cudaMemcpyDeviceToHost));
  return QORA_OK;
}

qora_status qora_engine_launches_per_step(const qora_engine* e, uint32_t* launches) {
  if (!e || !launches) return fail(QORA_ERR_INVALID, "NULL argument");
  if (e->format == QORA_FORMAT_F16)
    *launches = (uint32_t)f16_launches(e, true);
  else
    *launches = (e->mk_ok && e->use_mega) ? 1u : 1 + 5 * e->num_layers + 2;
  return QORA_OK;
}

qora_status qora_engine_prompt_path(const qora_engine* e, uint32_t* path) {
  if (!e || !path) return fail(QORA_ERR_INVALID, "NULL argument");
  *path = (e->format == QORA_FORMAT_F16 || e->q4p) ? QORA_PROMPT_TENSOR_CORES : QORA_PROMPT_TOKEN_STEPS;
  return QORA_OK;
}

qora_status qora_generate_greedy_batch(qora_engine* e, qora_kv* kv, const uint32_t* first_tokens,
                                       uint32_t n_tokens, uint32_t* out_tokens, float* device_ms) {
  if (!e || !kv || kv->e != e || !first_tokens || (!out_tokens && n_tokens))
    return fail(QORA_ERR_INVALID, "bad arguments");
  if (e->format == QORA_FORMAT_F16) return f16_generate(e, kv, first_tokens, n_tokens, out_tokens, device_ms);
  if (device_ms) return qora_generate_greedy_timed(e, kv, first_tokens[0], n_tokens, out_tokens, device_ms);
  return qora_generate_greedy(e, kv, first_tokens[0], n_tokens, out_tokens);
}

// ------------------------------------------------------------------ kernel-level entries
}  // extern "C"

// cuTensorMapEncodeTiled through the runtime's driver entry point (no libcuda link)
static PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q{};
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D row-major tensor map over [rows][cols] elements of `esz` bytes, boxes of
// box_cols x box_rows elements (no swizzle; rows past the end read as zero)
static qora_status encode_2d(CUtensorMap* m, const void* base, CUtensorMapDataType type, int esz, uint64_t cols,
                             uint64_t rows, uint32_t box_cols, uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return fail(QORA_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * (cuuint64_t)esz};
  const cuuint32_t box[2] = {box_cols, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  const CUresult r = enc(m, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                         CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(QORA_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", (int)r);
  return QORA_OK;
}

// The TMA GEMV (q4_gemv_tma.cuh) for shapes it takes: 256-column tiles, 16-byte-aligned
// rows of both arrays, whole boxes of rows per CTA (k a multiple of the box height, at
// least one and at most kMaxBoxes boxes per CTA); *used = false otherwise.
static qora_status q4_gemv_tma(const float* d_x, const uint8_t* d_packed, const uint16_t* d_scales, int k, int n,
                               float* d_y, cudaStream_t stream, int dev, bool* used) {
  *used = false;
  const int G = sm_count(dev);
  if (!g1::shape_ok(k, n, G) || ((uintptr_t)d_packed | (uintptr_t)d_scales) % 16) return QORA_OK;
  const long long tiles = n / kTileCols, boxes = tiles * (long long)(k / g1::kBoxRows);
  static std::once_flag attr_once;
  static cudaError_t attr_err = cudaSuccess;
  std::call_once(attr_once, [] {
    attr_err = cudaFuncSetAttribute(g1::q4_gemv_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    (int)g1::kSmemBytes);
    if (attr_err == cudaSuccess)  // room for two CTAs per SM
      attr_err = cudaFuncSetAttribute(g1::q4_gemv_tma_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                      cudaSharedmemCarveoutMaxShared);
  });
  QCUDA(attr_err);
  CUtensorMap mp, ms;
  QCHECK(encode_2d(&mp, d_packed, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, (uint64_t)n / 2, (uint64_t)k, 128, g1::kBoxRows));
  QCHECK(encode_2d(&ms, d_scales, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (uint64_t)n / kGroup, (uint64_t)k, 8, g1::kBoxRows));
  // CTAs touching one tile: every CTA owns at least floor(boxes / G) boxes of the range
  const int slots = g1::slots_bound(k, boxes, G);
  std::lock_guard<std::mutex> lk(g_entry_mu);
  EntryScratch* sc = nullptr;
  QCHECK(entry_scratch(dev, 0, 0, 0, &sc, (size_t)tiles * slots * kTileCols));
  g1::Args a{d_x, d_y, sc->tagged, k, n, (int)tiles, slots};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(G);
  cfg.blockDim = dim3(g1::kThreads);
  cfg.dynamicSmemBytes = g1::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  QCUDA(cudaLaunchKernelEx(&cfg, g1::q4_gemv_tma_kernel, mp, ms, a));
  *used = true;
  return QORA_OK;
}

extern "C" {

qora_status qora_q4_gemv(const float* d_x, const uint8_t* d_packed, const uint16_t* d_scales,
                         uint64_t k, uint64_t n, float* d_y, void* stream) {
  if (!d_x || !d_packed || !d_scales || !d_y) return fail(QORA_ERR_INVALID, "NULL pointer");
  if (k == 0 || n == 0 || n % kGroup || k > (1u << 30) || n > (1u << 30))
    return fail(QORA_ERR_INVALID, "bad shape k=%llu n=%llu", (unsigned long long)k, (unsigned long long)n);
  int dev = 0;
  QCUDA(cudaGetDevice(&dev));
  bool used = false;
  QCHECK(q4_gemv_tma(d_x, d_packed, d_scales, (int)k, (int)n, d_y, (cudaStream_t)stream, dev, &used));
  if (used) return QORA_OK;
  const Q4Src src = f1_src(d_packed, d_scales, (int)k, (int)n);
  const GemvShape sh = plan_gemv((int)k, src.tiles, 2 * sm_count(dev));
  std::lock_guard<std::mutex> lk(g_entry_mu);
  EntryScratch* sc = nullptr;
  QCHECK(entry_scratch(dev, partial_floats(sh), sh.tiles, 0, &sc));
  return launch_gemv(src, sh, sc->partials, sc->counters, ProPlain{d_x}, EpiStore{d_y, (int)n},
                     (cudaStream_t)stream);
}

// Scratch of qora_q4_gemv_static: QORA_GEMV_STATIC_FLOATS split-K partials followed by
// QORA_GEMV_STATIC_TILES arrival counters (zero-initialised at module load; every
// launch's last arriver of a tile puts its counter back to zero).
static __device__ __align__(256) float g_gemv_static_scratch[QORA_GEMV_STATIC_FLOATS + QORA_GEMV_STATIC_TILES];
constexpr int kStaticMaxDevices = 64;
static std::mutex g_static_mu;
static void* g_static_addr[kStaticMaxDevices] = {};

qora_status qora_q4_gemv_static(const float* d_x, const uint8_t* d_packed, const uint16_t* d_scales,
                                uint64_t k, uint64_t n, float* d_y, void* stream) {
  if (!d_x || !d_packed || !d_scales || !d_y) return fail(QORA_ERR_INVALID, "NULL pointer");
  if (k == 0 || n == 0 || n % kGroup || k > (1u << 30) || n > (1u << 30))
    return fail(QORA_ERR_INVALID, "bad shape k=%llu n=%llu", (unsigned long long)k, (unsigned long long)n);
  int dev = 0;
  QCUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= kStaticMaxDevices) return fail(QORA_ERR_UNSUPPORTED, "device ordinal %d", dev);
  const Q4Src src = f1_src(d_packed, d_scales, (int)k, (int)n);
  const GemvShape sh = plan_gemv((int)k, src.tiles, 2 * sm_count(dev));
  if ((size_t)sh.tiles > QORA_GEMV_STATIC_TILES || partial_floats(sh) > QORA_GEMV_STATIC_FLOATS)
    return fail(QORA_ERR_UNSUPPORTED,
                "k=%llu n=%llu needs %zu partial floats and %d tile counters; the static scratch "
                "holds %u and %u",
                (unsigned long long)k, (unsigned long long)n, partial_floats(sh), sh.tiles,
                QORA_GEMV_STATIC_FLOATS, QORA_GEMV_STATIC_TILES);
  void* base = nullptr;
  {
    std::lock_guard<std::mutex> lk(g_static_mu);
    if (!g_static_addr[dev]) {
      // one-time per device, with `dev` current: resolve the array's device address
      void* p = nullptr;
      const cudaError_t ce = cudaGetSymbolAddress(&p, g_gemv_static_scratch);
      if (ce != cudaSuccess || !p)
        return fail(QORA_ERR_CUDA, "cudaGetSymbolAddress: %s", cudaGetErrorString(ce));
      g_static_addr[dev] = p;
    }
    base = g_static_addr[dev];
  }
  float* partials = static_cast<float*>(base);
  unsigned* counters = reinterpret_cast<unsigned*>(partials + QORA_GEMV_STATIC_FLOATS);
  const qora_status ls = launch_gemv(src, sh, partials, counters, ProPlain{d_x}, EpiStore{d_y, (int)n},
                                     (cudaStream_t)stream);
  // a launch that failed may have left arrival counts behind (the next call would then
  // sum stale partials): put the counters of this plan back to zero (no allocation)
  if (ls != QORA_OK) cudaMemsetAsync(counters, 0, (size_t)sh.tiles * sizeof(unsigned), (cudaStream_t)stream);
  return ls;
}

qora_status qora_q4_dequant(const uint8_t* d_packed, const uint16_t* d_scales, uint64_t n,
                            uint64_t row0, uint64_t rows, float* d_out, void* stream) {
  if (!d_packed || !d_scales || !d_out) return fail(QORA_ERR_INVALID, "NULL pointer");
  if (n == 0 || n % kGroup) return fail(QORA_ERR_INVALID, "n=%llu must be a multiple of 32", (unsigned long long)n);
  if (rows == 0) return QORA_OK;
  const long long total = (long long)(rows * n);
  const int blocks = (int)std::min<long long>((total + 255) / 256, 4096);
  dequant_q4_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(d_packed, d_scales, (long long)n,
                                                               (long long)row0, (long long)rows, d_out);
  QCUDA(cudaGetLastError());
  return QORA_OK;
}

qora_status qora_q4_gate_up(const float* d_x, const uint8_t* d_gate_packed,
                            const uint16_t* d_gate_scales, const uint8_t* d_up_packed,
                            const uint16_t* d_up_scales, uint64_t k, uint64_t n, float* d_out,
                            void* stream) {
  if (!d_x || !d_gate_packed || !d_gate_scales || !d_up_packed || !d_up_scales || !d_out)
    return fail(QORA_ERR_INVALID, "NULL pointer");
  if (k == 0 || n == 0 || n % 128 || k > (1u << 30) || n > (1u << 30))
    return fail(QORA_ERR_INVALID, "bad shape k=%llu n=%llu (n must be a multiple of 128)",
                (unsigned long long)k, (unsigned long long)n);
  int dev = 0;
  QCUDA(cudaGetDevice(&dev));
  const Q4Src src = f1_pair_src(d_gate_packed, d_gate_scales, d_up_packed, d_up_scales, (int)k, (int)n);
  const GemvShape sh = plan_gemv((int)k, src.tiles, 2 * sm_count(dev));
  std::lock_guard<std::mutex> lk(g_entry_mu);
  EntryScratch* sc = nullptr;
  QCHECK(entry_scratch(dev, partial_floats(sh), sh.tiles, 0, &sc));
  return launch_gemv(src, sh, sc->partials, sc->counters, ProPlain{d_x}, EpiSwiGLU{d_out, (int)n},
                     (cudaStream_t)stream);
}

qora_status qora_q4_lm_head(const float* d_x, const uint8_t* d_packed, const uint16_t* d_scales,
                            uint64_t vocab, uint64_t hidden, float* d_logits, uint32_t* d_argmax,
                            void* stream) {
  if (!d_x || !d_packed || !d_scales || !d_argmax) return fail(QORA_ERR_INVALID, "NULL pointer");
  if (vocab == 0 || vocab > (1u << 30)) return fail(QORA_ERR_INVALID, "bad vocab");
  int dev = 0;
  QCUDA(cudaGetDevice(&dev));
  const int ctas = (int)std::min<uint64_t>(2 * sm_count(dev), vocab);
  std::lock_guard<std::mutex> lk(g_entry_mu);
  EntryScratch* sc = nullptr;
  QCHECK(entry_scratch(dev, 0, 0, ctas, &sc));
  LmArgs a{};
  a.x = d_x;
  a.gamma = nullptr;
  a.packed = d_packed;
  a.scales = reinterpret_cast<const uint8_t*>(d_scales);
  a.row_stride_p = (long long)(hidden / 2);
  a.row_stride_s = (long long)(hidden / kGroup * 2);
  a.vocab = (int)vocab;
  a.logits = d_logits;
  a.argmax_out = d_argmax;
  a.part_v = sc->lm_v;
  a.part_i = sc->lm_i;
  a.counter = sc->lm_c;
  return launch_lm_head((int)hidden, a, ctas, (cudaStream_t)stream);
}

namespace {
qora_status sample_params(const qora_sampling* p, uint32_t vocab, smp::Params* out) {
  if (!p) return fail(QORA_ERR_INVALID, "NULL sampling parameters");
  if (vocab == 0 || vocab > (uint32_t)smp::kMaxVocabBits)
    return fail(QORA_ERR_UNSUPPORTED, "vocab %u (at most %d for on-device sampling)", vocab, smp::kMaxVocabBits);
  if (p->temperature > 0.0f && (p->top_k == 0 || p->top_k > (uint32_t)smp::kMaxTopK))
    return fail(QORA_ERR_UNSUPPORTED, "top_k %u: on-device sampling takes 1..%d", p->top_k, smp::kMaxTopK);
  out->temperature = p->temperature;
  out->top_p = p->top_p;
  out->top_k = (int)std::min<uint32_t>(p->top_k, vocab);
  out->repetition_penalty = p->repetition_penalty;
  out->presence_penalty = p->presence_penalty;
  out->ban = p->ban_token;
  return QORA_OK;
}
}  // namespace

qora_status qora_sample(qora_engine* e, uint32_t row, const uint32_t* history, uint32_t n_history,
                        const qora_sampling* params, uint64_t* rng_state, uint32_t* token_out) {
  if (!e || !rng_state || !token_out || (!history && n_history)) return fail(QORA_ERR_INVALID, "NULL argument");
  smp::Params sp{};
  QCHECK(sample_params(params, e->vocab, &sp));
  const uint32_t rows = e->format == QORA_FORMAT_F16 ? (uint32_t)f16b::kMaxRows : 1u;
  if (row >= rows) return fail(QORA_ERR_RANGE, "logits row %u", row);
  QCUDA(cudaSetDevice(e->device));
  if (!e->smp_work) {
    QCHECK(e->alloc(&e->smp_work, e->vocab));
    QCHECK(e->alloc(&e->smp_out, 1));
    QCUDA(cudaMallocHost(&e->smp_out_host, sizeof(smp::Out)));
  }
  if (n_history > e->smp_hist_cap) {
    const size_t cap = std::max<size_t>(n_history, 4096);
    QCHECK(e->alloc(&e->smp_hist, cap));
    e->smp_hist_cap = cap;
  }
  if (n_history)
    QCUDA(cudaMemcpyAsync(e->smp_hist, history, (size_t)n_history * 4, cudaMemcpyHostToDevice, e->stream));
  const float* logits = e->logits + (size_t)row * e->vocab;
  smp::sample_kernel<<<1, smp::kThreads, 0, e->stream>>>(logits, (int)e->vocab, e->smp_hist, (int)n_history, sp,
                                                        (unsigned long long)*rng_state, e->smp_work, e->smp_out);
  QCUDA(cudaGetLastError());
  QCUDA(cudaMemcpyAsync(e->smp_out_host, e->smp_out, sizeof(smp::Out), cudaMemcpyDeviceToHost, e->stream));
  QCUDA(cudaStreamSynchronize(e->stream));
  *token_out = e->smp_out_host->token;
  *rng_state = e->smp_out_host->state;
  return QORA_OK;
}

qora_status qora_sample_logits(const float* d_logits, uint32_t vocab, const uint32_t* d_history,
                               uint32_t n_history, const qora_sampling* params, uint64_t* rng_state,
                               uint32_t* token_out, void* stream) {
  if (!d_logits || !rng_state || !token_out || (!d_history && n_history))
    return fail(QORA_ERR_INVALID, "NULL argument");
  smp::Params sp{};
  QCHECK(sample_params(params, vocab, &sp));
  const cudaStream_t s = (cudaStream_t)stream;
  int dev = 0;
  QCUDA(cudaGetDevice(&dev));
  // the work row and result slot are cached per device (grown on demand) and used under
  // the entry lock until this call's result is back on the host, so calls never share them
  std::lock_guard<std::mutex> lk(g_entry_mu);
  EntryScratch& es = g_entry[dev];
  if (es.smp_n < vocab) {
    if (es.smp_work) cudaFree(es.smp_work);
    es.smp_work = nullptr;
    es.smp_n = 0;
    QCUDA(cudaMalloc(&es.smp_work, (size_t)vocab * 4));
    es.smp_n = vocab;
  }
  if (!es.smp_out) QCUDA(cudaMalloc(&es.smp_out, sizeof(smp::Out)));
  smp::sample_kernel<<<1, smp::kThreads, 0, s>>>(d_logits, (int)vocab, d_history, (int)n_history, sp,
                                                (unsigned long long)*rng_state, es.smp_work, es.smp_out);
  cudaError_t ce = cudaGetLastError();
  smp::Out h{};
  if (ce == cudaSuccess) ce = cudaMemcpyAsync(&h, es.smp_out, sizeof(h), cudaMemcpyDeviceToHost, s);
  if (ce == cudaSuccess) ce = cudaStreamSynchronize(s);
  if (ce != cudaSuccess) return fail(QORA_ERR_CUDA, "sampling: %s", cudaGetErrorString(ce));
  *token_out = h.token;
  *rng_state = h.state;
  return QORA_OK;
}

qora_status qora_f16_gemm(const float* d_x, const uint16_t* d_w, uint64_t m, uint64_t k, uint64_t n,
                          float* d_y, void* stream) {
  if (!d_x || !d_w || !d_y) return fail(QORA_ERR_INVALID, "NULL pointer");
  if (m == 0 || k == 0 || n == 0) return fail(QORA_ERR_INVALID, "empty GEMM");
  if (k % umma::kChunkK || n % umma::kTileN || k > (1u << 16) || n > (1u << 20))
    return fail(QORA_ERR_UNSUPPORTED, "k=%llu must be a multiple of 64 (<= 65536), n=%llu of 128", (unsigned long long)k,
                (unsigned long long)n);
  int dev = 0;
  QCUDA(cudaGetDevice(&dev));
  const cudaStream_t s = (cudaStream_t)stream;
  const int K = (int)k, N = (int)n, sms = sm_count(dev), R = umma::kMaxRows;
  const UmmaPlan p = umma_plan(sms, N / umma::kTileN, K / umma::kChunkK);
  struct Scratch {
    std::vector<void*> ptrs;
    ~Scratch() {
      for (void* q : ptrs) cudaFree(q);
    }
  } sc;
  auto grab = [&](size_t bytes, void** out) -> qora_status {
    QCUDA(cudaMalloc(out, std::max<size_t>(bytes, 16)));
    QCUDA(cudaMemset(*out, 0, std::max<size_t>(bytes, 16)));
    sc.ptrs.push_back(*out);
    return QORA_OK;
  };
  void *wt = nullptr, *xt = nullptr, *mx = nullptr, *part = nullptr, *tcnt = nullptr, *sync = nullptr, *err = nullptr;
  const size_t tiles = (size_t)N / umma::kTileN;
  QCHECK(grab((size_t)K * N * 2, &wt));
  QCHECK(grab((size_t)K * R * 4, &xt));
  QCHECK(grab((size_t)R * 4, &mx));
  const size_t part_floats = (size_t)p.G * p.maxseg * R * umma::kTileN;
  QCHECK(grab(part_floats * 4, &part));
  QCHECK(grab(tiles * 4, &tcnt));
  QCHECK(grab(16, &sync));
  QCHECK(grab(sizeof(int), &err));
  QCHECK(umma_attrs());
  const long long units = (long long)N * (K / 8);
  umma::tile_weights_kernel<<<(int)std::min<long long>((units + 255) / 256, 16LL * sms), 256, 0, s>>>(
      reinterpret_cast<const __half*>(d_w), N, 0, K, N, 0, 0, umma::kTileN, 0, K / umma::kChunkK,
      static_cast<uint8_t*>(wt));
  QCUDA(cudaGetLastError());
  const UmmaCtx u{sms, s, static_cast<uint8_t*>(xt), static_cast<float*>(part), part_floats,
                  static_cast<unsigned*>(tcnt), tiles, static_cast<unsigned*>(sync), static_cast<int*>(err)};
  for (uint64_t m0 = 0; m0 < m; m0 += umma::kMaxRows) {
    const int mb = (int)std::min<uint64_t>(umma::kMaxRows, m - m0);
    umma::row_max_kernel<<<mb, 256, 0, s>>>(d_x + m0 * k, K, static_cast<float*>(mx));
    QCUDA(cudaGetLastError());
    umma::FusedArgs a{};
    a.ep = umma::kEpStore;
    a.y = d_y + m0 * n;
    a.ldy = N;
    QCHECK(umma_fused(u, static_cast<uint8_t*>(wt), N, K, mb,
                      UmmaIn{d_x + m0 * k, K, nullptr, 0.0f, nullptr, static_cast<float*>(mx), 1}, a));
  }
  int herr = 0;
  QCUDA(cudaMemcpyAsync(&herr, err, sizeof(int), cudaMemcpyDeviceToHost, s));
  QCUDA(cudaStreamSynchronize(s));
  if (herr) return fail(QORA_ERR_TIMEOUT, "a bounded wait in the tensor-core GEMM timed out");
  return QORA_OK;
}

}  // extern "C"
