/*
 * qora_oracle.h — TEST INFRASTRUCTURE ONLY.
 *
 * CPU restatement of the reference QORA CPU decode path (Rust crate `qora`):
 *   src/gemv.rs:380-1190  (GEMV/GEMM, RMSNorm, RoPE, softmax, attention, lm_head,
 *                          forward_decode_raw, raw_prefill)
 *   src/simd.rs:44-176    (AVX-512 kernels; Q4 results are identical to the scalar path)
 *   src/save.rs:154-262   (.qora reader)
 *   src/generate.rs:346-352 (greedy argmax)
 * used as the parity checker for libqora_cuda.so and as the timed CPU baseline.
 * Nothing in the shipped engine links or calls this library.
 *
 * Bit-exactness: compiled with -ffp-contract=off, so every multiply and add rounds
 * separately as in Rust; the one FMA the reference uses (_mm512_fmadd_ps in
 * gemv_f16_avx512, src/simd.rs:166) is kept. Results that the reference makes
 * dependent on rayon's thread count (the k-split of src/gemv.rs:650-674, :419-492,
 * :540-555) take the thread count T from orc_set_threads().
 *
 * Parity pins: the reference ships no tests, fixtures or golden vectors and cannot be
 * built here (no cargo), so this restatement is pinned by known-answer tests and a
 * float64 NumPy cross-check (tests/test_oracle.py), not by reference outputs.
 */
#ifndef QORA_ORACLE_H
#define QORA_ORACLE_H

#include <stddef.h>
#include <stdint.h>
#include "../include/qora_cuda.h"

#ifdef __cplusplus
extern "C" {
#endif

typedef struct orc_model orc_model;
typedef struct orc_kv orc_kv;

/* rayon::current_num_threads() stand-in (the T of the k-split). Default: 1. */
void orc_set_threads(int t);
int  orc_get_threads(void);
/* Select the arithmetic of the host the reference would run on: 1 = AVX-512 paths
 * (gemv_f16 uses FMA), 0 = scalar paths. Default: detected at load. */
void orc_set_avx512(int on);
int  orc_get_avx512(void);
int  orc_host_has_avx512(void);

/* ---- model ---- */
orc_model* orc_model_load(const char* path, char* err, size_t errlen);   /* src/save.rs:154 */
orc_model* orc_model_from_view(const qora_weights_view* v, char* err, size_t errlen);
void       orc_model_free(orc_model* m);
uint32_t   orc_model_vocab(const orc_model* m);
uint32_t   orc_model_hidden(const orc_model* m);
uint32_t   orc_model_layers(const orc_model* m);
uint32_t   orc_model_format(const orc_model* m);

/* ---- KV cache (RawKvCache, src/gemv.rs:154-166) ---- */
orc_kv*  orc_kv_new(const orc_model* m);
void     orc_kv_free(orc_kv* kv);
uint32_t orc_kv_len(const orc_kv* kv, uint32_t layer);
/* replace layer contents with seq_len token-major rows */
int      orc_kv_import(orc_kv* kv, uint32_t layer, const float* k, const float* v, uint32_t seq_len);
int      orc_kv_export(const orc_kv* kv, uint32_t layer, float* k, float* v, uint32_t seq_len);
/* Opt-in binary16 cache (no counterpart in the reference; the engine's QORA_KV_F16):
 * every K and V value is rounded to IEEE binary16 (nearest even) when it enters the cache
 * (decode append, prefill, import) and attention reads the rounded values. Only on an
 * empty cache; returns nonzero otherwise. */
int      orc_kv_set_f16(orc_kv* kv, int on);
/* out[i] = x[i] rounded to the nearest binary16 value (ties to even), as f32 */
void     orc_round_f16(const float* x, float* out, size_t n);

/* ---- primitive restatements ---- */
float orc_f16_to_f32(uint16_t h);
/* gemv_q4 (src/gemv.rs:646-675) incl. the 4,000,000 threshold and the T-way k-split */
void  orc_gemv_q4(const float* x, const uint8_t* packed, const uint16_t* scales,
                  size_t k, size_t n, float* y);
/* gemv_q4_inner over rows [k0,k1) (src/gemv.rs:596-641), y zero-initialised inside */
void  orc_gemv_q4_rows(const float* x, const uint8_t* packed, const uint16_t* scales,
                       size_t n, size_t k0, size_t k1, float* y);
/* fused_gate_up_q4 (src/gemv.rs:412-502) */
void  orc_fused_gate_up_q4(const float* x, const uint8_t* gp, const uint16_t* gs,
                           const uint8_t* up, const uint16_t* us, size_t k, size_t n,
                           float* out);
/* gemv_f16 (src/gemv.rs:534-567) */
void  orc_gemv_f16(const float* x, const uint16_t* w, size_t k, size_t n, float* y);
/* gemm dispatch for prefill (src/gemv.rs:506-511, :571-588, :680-706) */
void  orc_gemm_q4(const float* x, size_t seq, const uint8_t* packed, const uint16_t* scales,
                  size_t k, size_t n, float* y);
void  orc_gemm_f16(const float* x, size_t seq, const uint16_t* w, size_t k, size_t n, float* y);
/* embed_lookup_q4 (src/gemv.rs:710-736) */
void  orc_embed_q4(const uint8_t* packed, const uint16_t* scales, size_t n, size_t row, float* out);
void  orc_dequant_q4_rows(const uint8_t* packed, const uint16_t* scales, size_t n,
                          size_t row0, size_t rows, float* out);
/* rms_norm_f16 (src/gemv.rs:744-753), eps 1e-6 */
void  orc_rms_norm(const float* x, const uint16_t* gamma, size_t size, float* out);
/* apply_rope_raw (src/gemv.rs:757-778), in place */
void  orc_rope(float* data, size_t heads, size_t head_dim, const float* cos_t,
               const float* sin_t, size_t half_dim, size_t pos);
/* softmax_raw (src/gemv.rs:782-793), in place */
void  orc_softmax(float* s, size_t n);
/* lm_head_parallel_q4 / _f16 (src/gemv.rs:797-864) */
void  orc_lm_head_q4(const float* x, const uint8_t* packed, const uint16_t* scales,
                     size_t vocab, size_t hidden, float* logits);
void  orc_lm_head_f16(const float* x, const uint16_t* w, size_t vocab, size_t hidden,
                      float* logits);
/* greedy branch of sample_token_top_k (src/generate.rs:346-352) */
uint32_t orc_argmax(const float* logits, size_t n);
/* Rng::next_f32 (src/generate.rs:54-60) */
float orc_rng_next_f32(uint64_t* state);
/* apply_repetition_penalty / apply_presence_penalty (src/generate.rs:64-92), in place */
void orc_repetition_penalty(float* logits, size_t n, const uint32_t* hist, size_t nh, float penalty);
void orc_presence_penalty(float* logits, size_t n, const uint32_t* hist, size_t nh, float penalty);
/* sample_token_top_k (src/generate.rs:345-394) */
uint32_t orc_sample_top_k(const float* logits, size_t n, float temperature, float top_p, size_t top_k,
                          uint64_t* state);
/* penalties (repetition, presence, banned token) on a copy, then sample_token_top_k */
uint32_t orc_sample(const float* logits, size_t n, const uint32_t* hist, size_t nh, float temperature,
                    float top_p, size_t top_k, float repetition_penalty, float presence_penalty, int64_t ban,
                    uint64_t* state);

/* ---- model-level ---- */
/* forward_decode_raw (src/gemv.rs:872-1019); logits [vocab] */
int  orc_forward_decode(const orc_model* m, uint32_t token, orc_kv* kv, float* logits);
/* the body of the layer loop (src/gemv.rs:883-1012) for one layer */
int  orc_layer_forward(const orc_model* m, uint32_t layer, float* x, orc_kv* kv);
/* raw_prefill (src/gemv.rs:1027-1190); kv must be empty; logits [vocab] of the last id */
int  orc_prefill(const orc_model* m, const uint32_t* ids, size_t n, orc_kv* kv, float* logits);
/* harness loop of src/main.rs:105-117 style: prefill then n greedy steps. tokens[n]
 * receives the generated ids; margins[n] (optional) the top-1 minus top-2 logit of
 * each step's argmax. Returns 0 on success. */
int  orc_generate_greedy(const orc_model* m, const uint32_t* prompt, size_t n_prompt,
                         size_t n_new, orc_kv* kv, uint32_t* tokens, float* margins);

#ifdef __cplusplus
}
#endif
#endif
