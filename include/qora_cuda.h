/*
 * qora_cuda.h — C ABI of libqora_cuda.so, the sm_100a decode engine that sits behind
 * QORA's SmolLM3-3B forward step.
 *
 * Every entry point returns a qora_status (0 = ok). No C++ exception or panic crosses
 * this boundary; the message of the last failure on the calling thread is available
 * from qora_last_error(). An engine is driven by one host thread at a time.
 *
 * The reference exposes the same path as plain Rust functions; each declaration below
 * names the reference interface it replaces (path:line inside the qora crate).
 */
#ifndef QORA_CUDA_H
#define QORA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int qora_status;

#define QORA_OK              0
#define QORA_ERR_INVALID     1  /* bad argument, shape or file contents              */
#define QORA_ERR_IO          2  /* file could not be opened / short read             */
#define QORA_ERR_CUDA        3  /* CUDA runtime error (message has the CUDA string)  */
#define QORA_ERR_OOM         4  /* device allocation failed                          */
#define QORA_ERR_RANGE       5  /* token id / position / sequence beyond capacity    */
#define QORA_ERR_TIMEOUT     6  /* a bounded device-side wait gave up                */
#define QORA_ERR_UNSUPPORTED 7  /* feature not available in this build / config      */
#define QORA_ERR_NCCL        8  /* collective failure (tensor-parallel engines)      */

#define QORA_FORMAT_F16 0u
#define QORA_FORMAT_Q4  1u

/* ------------------------------------------------------------------------------------
 * Borrowed host views of the weights (replace `WeightRef` / `GpuLayerRef` /
 * `DecodeWeights::layer_ref` / `embed_ref`, src/gemv.rs:66-96, :248-271).
 * Orientation (src/gemv.rs:23-38): projections are input-major [k = in][n = out];
 * Q4 groups of 32 run along n, a group is 16 packed bytes (low nibble = even element)
 * plus one f16 scale, value = (q - 8) * scale. The embedding is [k = vocab][n = hidden].
 * The engine copies (and may re-tile) what it needs and keeps no host pointer.
 * ---------------------------------------------------------------------------------- */
typedef struct qora_matrix_view {
    const uint8_t*  packed;  /* Q4: k*n/2 bytes, row ki at ki*(n/2)             */
    const uint16_t* scales;  /* Q4: k*n/32 f16 bit patterns, row ki at ki*(n/32) */
    const uint16_t* data;    /* F16: k*n f16 bit patterns, row-major [k][n]      */
    uint64_t k;
    uint64_t n;
} qora_matrix_view;

typedef struct qora_layer_view {
    qora_matrix_view q_proj, k_proj, v_proj, o_proj, gate_proj, up_proj, down_proj;
    const uint16_t* input_norm_gamma;      /* [hidden] f16 */
    const uint16_t* post_attn_norm_gamma;  /* [hidden] f16 */
    uint32_t num_heads, num_kv_heads, head_dim, num_kv_groups;
} qora_layer_view;

typedef struct qora_weights_view {
    uint32_t format;            /* QORA_FORMAT_F16 or QORA_FORMAT_Q4 (src/save.rs:170) */
    uint32_t num_layers;
    uint32_t vocab;
    uint32_t hidden;
    uint32_t rope_half_dim;
    const uint8_t* no_rope_layers;   /* [num_layers]; nonzero = APPLY RoPE (src/gemv.rs:885,903) */
    const qora_layer_view* layers;   /* [num_layers] */
    qora_matrix_view embed;          /* tied embedding / lm_head, k = vocab, n = hidden */
    const uint16_t* final_norm_gamma;/* [hidden] f16 */
    const float* rope_cos;           /* [rope_rows][rope_half_dim] f32 */
    const float* rope_sin;
    uint64_t rope_rows;              /* number of positions in the tables */
} qora_weights_view;

typedef struct qora_engine qora_engine;
typedef struct qora_kv qora_kv;

/* Engine options. Zero-initialise and set what you need.
 *
 * Tensor parallelism runs one engine per GPU, each in its own process (or thread):
 * set tp_size > 1 and this engine's tp_rank, create the engine on its device, pass every
 * rank's qora_tp_export() bytes to every rank's qora_tp_connect(), then drive all ranks
 * through the same sequence of calls (same tokens; each rank owns its own KV cache).
 * q|k|v and gate/up are column-split, o_proj and down row-split, lm_head split by vocab
 * (the reference itself has no tensor parallelism; its math is unchanged by the split). */
typedef struct qora_engine_options {
    int32_t  n_gpus;        /* single-process multi-GPU engines: must be 0 or 1     */
    int32_t  first_device;  /* CUDA ordinal this engine runs on                     */
    uint32_t flags;         /* QORA_FLAG_* bits                                     */
    int32_t  tp_size;       /* tensor-parallel degree: 0/1 (none), 2, 4 or 8         */
    int32_t  tp_rank;       /* this engine's rank in [0, tp_size)                   */
} qora_engine_options;

/* Run each decode step as a CUDA graph of per-operation kernels instead of the
 * persistent single-kernel step (diagnostics and cross-checking). */
#define QORA_FLAG_PER_OP_KERNELS 1u

/* Q4 engines: run a prompt as one decode step per token instead of the tensor-core
 * prompt pass (which holds a second copy of the projections, 0.5625 B per weight). */
#define QORA_FLAG_TOKEN_PREFILL 2u

/* Last error message of the calling thread ("" if none). */
const char* qora_last_error(void);

/* Library version string. */
const char* qora_version(void);

/* Load a .qora file and upload it. Replaces `save::load_model` (src/save.rs:154) +
 * the cortex upload `load_model_gpu` (src/gpu_loader.rs:134). */
qora_status qora_engine_create_from_file(const char* qora_path,
                                         const qora_engine_options* opts,
                                         qora_engine** out);

/* Upload borrowed host weights (the slices `DecodeWeights` holds, src/gemv.rs:195-206). */
qora_status qora_engine_create(const qora_weights_view* weights,
                               const qora_engine_options* opts,
                               qora_engine** out);

void qora_engine_destroy(qora_engine* engine);

/* Tensor-parallel set-up (no counterpart in the reference). qora_tp_export writes this
 * rank's opaque peer handle (an IPC handle of its receive buffers) to buf and its size to
 * *len (call with buf == NULL to query the size). qora_tp_connect takes all tp_size
 * ranks' handles concatenated in rank order and maps the peers' buffers; decode steps
 * are refused until it succeeds. All ranks must run on GPUs of one NVLink domain. */
qora_status qora_tp_export(qora_engine* engine, void* buf, size_t cap, size_t* len);

/* The shard rank tp_rank of a tp_size-way group holds (host-only arithmetic, no device
 * needed): query heads [q_head0, +q_heads), KV heads [kv_head0, +kv_heads) (split while
 * tp_size divides the KV heads, else the one KV head of the rank's query heads), gate/up
 * columns = down rows [mlp0, +mlp_n) (F16: computed as mlp_padded channels, the extra
 * ones zero), lm_head rows [vocab0, +vocab_n) (F16: whole 128-row tiles). */
typedef struct qora_tp_shard {
    uint32_t q_head0, q_heads;
    uint32_t kv_head0, kv_heads;
    uint32_t mlp0, mlp_n, mlp_padded;
    uint32_t vocab0, vocab_n;
} qora_tp_shard;
qora_status qora_tp_plan(uint32_t format, uint32_t num_heads, uint32_t num_kv_heads,
                         uint32_t intermediate, uint32_t vocab, int32_t tp_size,
                         int32_t tp_rank, qora_tp_shard* out);
qora_status qora_tp_connect(qora_engine* engine, const void* handles, size_t len_per_rank);

/* Geometry of a loaded engine. */
qora_status qora_engine_info(const qora_engine* engine, uint32_t* num_layers,
                             uint32_t* vocab, uint32_t* hidden, uint32_t* format,
                             uint64_t* device_bytes);

/* KV cache with capacity max_seq positions for `batch` independent sequences, f32.
 * Replaces `empty_kv_cache` (src/gemv.rs:159) / `RawKvCache` (src/gemv.rs:156), one per
 * sequence. Q4 engines take batch 1 (the batch-1 decode of the reference); F16 engines
 * take 1..128 sequences that decode together (each decode step advances all of them). */
qora_status qora_kv_create(qora_engine* engine, uint32_t max_seq, uint32_t batch,
                           qora_kv** out);

/* Element types of a KV cache. QORA_KV_F32 is the reference's cache. QORA_KV_F16 is the
 * opt-in lower-precision cache of long contexts (no counterpart in the reference): each
 * K and V value is rounded to IEEE binary16 (nearest even; beyond +-65504 it becomes
 * +-inf) when it enters the cache, by a decode step or by qora_kv_import, and attention
 * reads the rounded values, which halves the bytes a decode step streams per cached
 * position. Results then differ from the reference's f32 cache. Supported by Q4
 * engines on the persistent step with tp_size 1; anything else is QORA_ERR_UNSUPPORTED.
 * Import and export keep the f32 host layout. */
#define QORA_KV_F32 0u
#define QORA_KV_F16 1u

/* qora_kv_create with an element type (QORA_KV_*). */
qora_status qora_kv_create_ex(qora_engine* engine, uint32_t max_seq, uint32_t batch,
                              uint32_t kv_dtype, qora_kv** out);
void qora_kv_destroy(qora_kv* kv);

/* Current length (positions filled) of sequence seq_idx. */
qora_status qora_kv_length(const qora_kv* kv, uint32_t seq_idx, uint32_t* len);

/* Reset sequence seq_idx to empty (the reference builds a fresh RawKvCache). */
qora_status qora_kv_reset(qora_kv* kv, uint32_t seq_idx);

/* Import seq_len positions of one layer, token-major [seq_len][kv_heads][head_dim] f32
 * host arrays (the `(Vec<f32>, Vec<f32>, usize)` of RawKvCache, src/gemv.rs:156). After
 * importing every layer with the same seq_len, the sequence length becomes seq_len. */
qora_status qora_kv_import(qora_kv* kv, uint32_t layer, const float* k, const float* v,
                           uint32_t seq_len, uint32_t seq_idx);

/* Export the first seq_len positions of one layer to host arrays (same layout). */
qora_status qora_kv_export(const qora_kv* kv, uint32_t layer, float* k, float* v,
                           uint32_t seq_len, uint32_t seq_idx);

/* Prompt pass. Replaces `raw_prefill` (src/gemv.rs:1027): the n ids are appended at
 * positions len..len+n-1 of sequence seq_idx; the logits of the last id are written to
 * logits_or_null ([vocab] f32) if non-NULL, and its argmax (first maximum) to argmax_out
 * if non-NULL. */
qora_status qora_prefill(qora_engine* engine, qora_kv* kv, const uint32_t* ids,
                         uint32_t n, uint32_t seq_idx, float* logits_or_null,
                         uint32_t* argmax_out);

/* One decode step. Replaces `forward_decode_raw` (src/gemv.rs:872) followed by the
 * greedy branch of `sample_token_top_k` (src/generate.rs:346-352). tokens: [batch] host
 * ids; logits_or_null: [batch][vocab] host f32 (parity / sampling mode) or NULL (greedy
 * fast path: only argmax_out [batch] is read back). */
qora_status qora_decode_step(qora_engine* engine, qora_kv* kv, const uint32_t* tokens,
                             float* logits_or_null, uint32_t* argmax_out);

/* Greedy generation of n_tokens starting from `first_token` entirely on the device
 * (token feedback without host round trips; the loop of src/main.rs:105-117 and
 * src/generate.rs:299-331 with temperature 0 and no penalties / EOS stop). Writes
 * the n_tokens argmax ids to out_tokens. */
qora_status qora_generate_greedy(qora_engine* engine, qora_kv* kv, uint32_t first_token,
                                 uint32_t n_tokens, uint32_t* out_tokens);

/* Greedy generation for every sequence of a cache at once: first_tokens [batch], then
 * n_tokens batched decode steps on the device, each feeding its argmax back. out_tokens:
 * [n_tokens][batch]. device_ms (optional) receives the CUDA-event time of the steps.
 * The batched form of the loop of src/generate.rs:299-331 (temperature 0). */
qora_status qora_generate_greedy_batch(qora_engine* engine, qora_kv* kv,
                                       const uint32_t* first_tokens, uint32_t n_tokens,
                                       uint32_t* out_tokens, float* device_ms);

/* One decoder layer at batch 1 (the body of the layer loop, src/gemv.rs:883-1012):
 * x ([hidden] host f32) is the residual stream in and out; the layer's K/V row is
 * appended at the sequence's current length of that layer, which then grows by one. */
qora_status qora_layer_step(qora_engine* engine, qora_kv* kv, uint32_t layer,
                            float* x_inout);

/* ------------------------------------------------------------------------------------
 * Kernel-level entry points on DEVICE pointers (cudaStream_t passed as void*; NULL =
 * legacy default stream). Used for parity tests and the GEMV bandwidth benchmark.
 * ---------------------------------------------------------------------------------- */

/* Q4 GEMV in the reference layout: y[n] = x[k] . W[k][n] (replaces `gemv_q4`,
 * src/gemv.rs:646-675, and `gemv_q4_avx512`, src/simd.rs:44-83). packed/scales are the
 * F1-layout arrays as in the file; n % 32 == 0. Scratch for the split-K partial sums is
 * allocated (zeroed) on first use and cached by the library (per device); every call
 * leaves it zeroed again, and calls on one device share it, so calls that may run at the
 * same time on different streams must be ordered by the caller. Results are
 * deterministic (fixed summation order, no float atomics). */
qora_status qora_q4_gemv(const float* d_x, const uint8_t* d_packed,
                         const uint16_t* d_scales, uint64_t k, uint64_t n, float* d_y,
                         void* stream);

/* The same Q4 GEMV with no allocation at all (no counterpart in the reference, which
 * has no device memory): the split-K partial sums and arrival counters live in one
 * fixed-size file-scope device array of the library (QORA_GEMV_STATIC_FLOATS floats
 * of partials + QORA_GEMV_STATIC_TILES counters per device). For callers that must not
 * allocate: a host that owns every byte of device memory up front (a serving process
 * that pre-reserves HBM, an allocator-free embedding, code paths where a hidden
 * cudaMalloc would synchronise the device). Shapes whose plan needs more scratch than
 * the array holds are rejected with QORA_ERR_UNSUPPORTED. The first call on a device
 * looks up the array's address (a one-time set-up step; make it before any stream
 * capture). The address is kept for the life of the process: after a cudaDeviceReset
 * (which unloads the library's device code) the cached address is stale, so do not call
 * this entry again in that process. Every call shares the array: the counters start at
 * zero and each call leaves them at zero, so calls must not overlap in time (concurrent
 * calls on different streams of one device race on the shared partials). A call whose
 * launch fails puts the counters back to zero before it returns the error; a kernel that
 * faults mid-way loses the whole CUDA context, and with it every later call. */
#define QORA_GEMV_STATIC_FLOATS (512u * 1024u)
#define QORA_GEMV_STATIC_TILES 1024u
qora_status qora_q4_gemv_static(const float* d_x, const uint8_t* d_packed,
                                const uint16_t* d_scales, uint64_t k, uint64_t n,
                                float* d_y, void* stream);

/* Bit-exact dequantisation of rows [row0, row0+rows) of a Q4 matrix to f32
 * ((q-8)*f32(scale), src/gemv.rs:727-731). d_out: rows*n floats. */
qora_status qora_q4_dequant(const uint8_t* d_packed, const uint16_t* d_scales,
                            uint64_t n, uint64_t row0, uint64_t rows, float* d_out,
                            void* stream);

/* Fused gate/up: out[n] = silu(x.Wg) * (x.Wu) (replaces `fused_gate_up_q4`,
 * src/gemv.rs:412-502). */
qora_status qora_q4_gate_up(const float* d_x, const uint8_t* d_gate_packed,
                            const uint16_t* d_gate_scales, const uint8_t* d_up_packed,
                            const uint16_t* d_up_scales, uint64_t k, uint64_t n,
                            float* d_out, void* stream);

/* ------------------------------------------------------------------------------------
 * On-device sampling (the sampling step of src/generate.rs:216-235): penalties, then
 * sample_token_top_k (src/generate.rs:345-394) on the logits that stay on the device, so
 * that only the token crosses PCIe when temperature > 0.
 * ---------------------------------------------------------------------------------- */
typedef struct qora_sampling {
    float    temperature;         /* <= 0: greedy first maximum                        */
    float    top_p;               /* nucleus cut within the top_k                      */
    uint32_t top_k;               /* 1..1024 when temperature > 0                      */
    float    repetition_penalty;  /* applied when > 1: each occurrence among the last
                                     64 history tokens (apply_repetition_penalty)      */
    float    presence_penalty;    /* applied when > 0: once per distinct history token
                                     (apply_presence_penalty)                          */
    int32_t  ban_token;           /* set to -inf after the penalties; -1: none (the
                                     thinking branch bans EOS)                         */
} qora_sampling;

/* Sample from row `row` of the logits of the engine's last decode step or prefill
 * (Q4 engines: row 0; F16 engines: the sequence's row of the last batched step, row 0
 * after a prefill). history: host token ids (all generated tokens, oldest first).
 * rng_state: the reference's xorshift64 Rng state (src/generate.rs:38-61), advanced by
 * one draw only when the reference draws. Synchronises the engine's stream. */
qora_status qora_sample(qora_engine* engine, uint32_t row, const uint32_t* history,
                        uint32_t n_history, const qora_sampling* params,
                        uint64_t* rng_state, uint32_t* token_out);

/* The same on a caller's device logits [vocab] and device history (kernel level). */
qora_status qora_sample_logits(const float* d_logits, uint32_t vocab, const uint32_t* d_history,
                               uint32_t n_history, const qora_sampling* params,
                               uint64_t* rng_state, uint32_t* token_out, void* stream);

/* F16 GEMM y[m][n] = x[m][k] . W[k][n] on the tcgen05 tensor cores (replaces `gemm_f16`,
 * src/gemv.rs:571-588, and `gemv_f16` at m = 1, src/gemv.rs:534-567). W is the
 * reference's row-major [k][n] f16 bit patterns; k must be a multiple of 64 and n of 128.
 * Each call re-tiles W into device scratch (the engine does this once at load); x keeps
 * ~22 bits through an f16 hi + lo split. Synchronises the stream before returning. */
qora_status qora_f16_gemm(const float* d_x, const uint16_t* d_w, uint64_t m, uint64_t k,
                          uint64_t n, float* d_y, void* stream);

/* Row-dot Q4 lm_head + first-maximum argmax over rows (replaces `lm_head_parallel_q4`,
 * src/gemv.rs:825-864, and the greedy branch of src/generate.rs:346-352). d_logits may
 * be NULL; d_argmax receives one uint32. */
qora_status qora_q4_lm_head(const float* d_x, const uint8_t* d_packed,
                            const uint16_t* d_scales, uint64_t vocab, uint64_t hidden,
                            float* d_logits, uint32_t* d_argmax, void* stream);


/* ------------------------------------------------------------------------------------
 * Measurement entry points (no counterpart in the reference, which only times whole
 * calls with Instant, src/main.rs:105-117 and src/generate.rs:134-139, :255-260).
 * ---------------------------------------------------------------------------------- */

/* qora_generate_greedy, and *device_ms receives the time of the n_tokens decode steps
 * measured with CUDA events on the engine's stream. */
qora_status qora_generate_greedy_timed(qora_engine* engine, qora_kv* kv, uint32_t first_token,
                                       uint32_t n_tokens, uint32_t* out_tokens,
                                       float* device_ms);

#define QORA_KERNEL_QKV       0  /* RMSNorm + q|k|v GEMV + RoPE + KV append, per layer */
#define QORA_KERNEL_ATTENTION 1  /* split-KV decode attention, per layer               */
#define QORA_KERNEL_O         2  /* o_proj GEMV + residual, per layer                  */
#define QORA_KERNEL_GATE_UP   3  /* RMSNorm + gate/up GEMV + SwiGLU, per layer         */
#define QORA_KERNEL_DOWN      4  /* down_proj GEMV + residual, per layer               */
#define QORA_KERNEL_LM_HEAD   5  /* final RMSNorm + lm_head + argmax                   */

/* Launch one kernel family `reps` times over every layer in order (so consecutive
 * launches read different weights) between CUDA events on the engine's stream; returns
 * the mean device time of one launch and the algorithmic bytes one launch moves
 * (weights + input vector + output vector; for attention the K/V rows read). The KV
 * state of `kv` (its current length) sets the attention length. */
qora_status qora_engine_time_kernel(qora_engine* engine, qora_kv* kv, int kernel,
                                    uint32_t reps, float* ms_per_launch,
                                    uint64_t* bytes_per_launch, uint32_t* launches);

/* Diagnostics of the persistent decode kernel: when enabled, every CTA records
 * %globaltimer stamps at its phase boundaries during each step (overwritten by the next
 * step). get_trace copies up to `cap` u64 values and reports how many exist. */
qora_status qora_engine_set_trace(qora_engine* engine, int enable);
qora_status qora_engine_get_trace(qora_engine* engine, uint64_t* out, size_t cap, size_t* n);

/* Number of kernel launches one decode step makes (the captured graph's nodes). */
qora_status qora_engine_launches_per_step(const qora_engine* engine, uint32_t* launches);

/* How qora_prefill runs a prompt of two or more tokens on this engine:
 * QORA_PROMPT_TENSOR_CORES: all prompt rows at once, layer by layer, through tcgen05 GEMMs
 * (F16 engines; Q4 engines at tp_size 1 with a binary32 KV cache, unless created with
 * QORA_FLAG_TOKEN_PREFILL); QORA_PROMPT_TOKEN_STEPS: one decode step per token. */
#define QORA_PROMPT_TOKEN_STEPS 0u
#define QORA_PROMPT_TENSOR_CORES 1u
qora_status qora_engine_prompt_path(const qora_engine* engine, uint32_t* path);

#ifdef __cplusplus
}
#endif

#endif /* QORA_CUDA_H */
