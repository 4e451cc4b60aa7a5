// qora_host.hpp — C++17 host-side mirror of the reference's decode interface (the Rust
// crate `qora`), over the C ABI of include/qora_cuda.h. Header-only; link
// libqora_cuda.so.
//
// Reference interface (src/...)                 here
//   save::load_model(path) -> io::Result        qora::load_model(path)            (:154)
//   gemv::DecodeWeights                          qora::DecodeWeights               (gemv.rs:177-206)
//   gemv::empty_kv_cache(layers, kvh, hd)        qora::empty_kv_cache(w, max_seq)  (gemv.rs:159)
//   gemv::RawKvCache                             qora::RawKvCache                  (gemv.rs:154-166)
//   gemv::forward_decode_raw(&w, tok, &mut kv)   qora::forward_decode_raw(w, tok, kv) (gemv.rs:872)
//   gemv::raw_prefill(&w, &ids)                  qora::raw_prefill(w, ids)         (gemv.rs:1027)
//   generate::sample_token_top_k (greedy)        qora::greedy(logits)              (generate.rs:346-352)
//   generate::Rng + penalties + top-k/top-p      qora::Rng, qora::sample_next(...) (generate.rs:38-92, 345-394)
//
// Errors: the reference returns io::Error from load_model and panics on bad input in the
// forward functions; here every failing call throws qora::Error carrying the library's
// status code and message (nothing falls back to the CPU).
#pragma once

#include <cmath>
#include <cstdint>
#include <memory>
#include <stdexcept>
#include <string>
#include <utility>
#include <vector>

#include "../../include/qora_cuda.h"

namespace qora {

class Error : public std::runtime_error {
 public:
  Error(qora_status status, const std::string& what) : std::runtime_error(what), status_(status) {}
  qora_status status() const { return status_; }

 private:
  qora_status status_;
};

inline void check(qora_status st) {
  if (st != QORA_OK) throw Error(st, qora_last_error());
}

// The model resident on a GPU (or one tensor-parallel shard of it).
class DecodeWeights {
 public:
  static DecodeWeights load_model(const std::string& path, int device = 0) {
    qora_engine_options o{};
    o.first_device = device;
    qora_engine* e = nullptr;
    check(qora_engine_create_from_file(path.c_str(), &o, &e));
    return DecodeWeights(e);
  }
  static DecodeWeights from_view(const qora_weights_view& view, const qora_engine_options* opts = nullptr) {
    qora_engine* e = nullptr;
    check(qora_engine_create(&view, opts, &e));
    return DecodeWeights(e);
  }
  uint32_t num_layers() const { return info().num_layers; }
  uint32_t vocab() const { return info().vocab; }
  uint32_t hidden() const { return info().hidden; }
  uint32_t format() const { return info().format; }
  qora_engine* raw() const { return e_.get(); }

 private:
  struct Info {
    uint32_t num_layers, vocab, hidden, format;
  };
  explicit DecodeWeights(qora_engine* e) : e_(e, &qora_engine_destroy) {}
  Info info() const {
    Info i{};
    uint64_t bytes = 0;
    check(qora_engine_info(e_.get(), &i.num_layers, &i.vocab, &i.hidden, &i.format, &bytes));
    return i;
  }
  std::unique_ptr<qora_engine, void (*)(qora_engine*)> e_;
};

// A KV cache on the device: `batch` independent sequences of up to max_seq positions.
// kv_dtype QORA_KV_F16 is the opt-in binary16 cache (Q4 engines; results differ from the
// reference's f32 cache).
class RawKvCache {
 public:
  RawKvCache(const DecodeWeights& w, uint32_t max_seq, uint32_t batch = 1, uint32_t kv_dtype = QORA_KV_F32)
      : kv_(nullptr, &qora_kv_destroy) {
    qora_kv* kv = nullptr;
    check(qora_kv_create_ex(w.raw(), max_seq, batch, kv_dtype, &kv));
    kv_.reset(kv);
    batch_ = batch;
  }
  uint32_t len(uint32_t seq = 0) const {
    uint32_t n = 0;
    check(qora_kv_length(kv_.get(), seq, &n));
    return n;
  }
  void reset(uint32_t seq = 0) { check(qora_kv_reset(kv_.get(), seq)); }
  // token-major [seq_len][kv_heads*128] rows of one layer (the RawKvCache tuple)
  void import_layer(uint32_t layer, const std::vector<float>& k, const std::vector<float>& v, uint32_t seq_len,
                    uint32_t seq = 0) {
    check(qora_kv_import(kv_.get(), layer, k.data(), v.data(), seq_len, seq));
  }
  // the first seq_len rows of one layer, token-major [seq_len][kv_heads*128] (f32 whatever
  // the cache's element type)
  void export_layer(uint32_t layer, std::vector<float>& k, std::vector<float>& v, uint32_t seq_len, size_t kv_row,
                    uint32_t seq = 0) const {
    k.resize((size_t)seq_len * kv_row);
    v.resize((size_t)seq_len * kv_row);
    check(qora_kv_export(kv_.get(), layer, k.data(), v.data(), seq_len, seq));
  }
  uint32_t batch() const { return batch_; }
  qora_kv* raw() const { return kv_.get(); }

 private:
  std::unique_ptr<qora_kv, void (*)(qora_kv*)> kv_;
  uint32_t batch_ = 1;
};

inline RawKvCache empty_kv_cache(const DecodeWeights& w, uint32_t max_seq = 4096) { return RawKvCache(w, max_seq); }

// One decode step of sequence 0: appends one KV row, returns the logits [vocab].
inline std::vector<float> forward_decode_raw(const DecodeWeights& w, uint32_t token_id, RawKvCache& kv) {
  std::vector<float> logits(w.vocab());
  uint32_t am = 0;
  check(qora_decode_step(w.raw(), kv.raw(), &token_id, logits.data(), &am));
  return logits;
}

// Prompt pass into a fresh cache: (logits of the last id, the cache).
inline std::pair<std::vector<float>, RawKvCache> raw_prefill(const DecodeWeights& w, const std::vector<uint32_t>& ids,
                                                             uint32_t max_seq = 4096) {
  RawKvCache kv(w, max_seq);
  std::vector<float> logits(w.vocab());
  uint32_t am = 0;
  check(qora_prefill(w.raw(), kv.raw(), ids.data(), (uint32_t)ids.size(), 0, logits.data(), &am));
  return {std::move(logits), std::move(kv)};
}

// Greedy branch of sample_token_top_k: first maximum (index 0 if none).
inline uint32_t greedy(const std::vector<float>& logits) {
  uint32_t best = 0;
  float mx = -INFINITY;
  for (size_t i = 0; i < logits.size(); ++i)
    if (logits[i] > mx) {
      mx = logits[i];
      best = (uint32_t)i;
    }
  return best;
}

// n greedy tokens after `first`, on the device (token feedback without host round trips).
inline std::vector<uint32_t> generate_greedy(const DecodeWeights& w, RawKvCache& kv, uint32_t first, uint32_t n) {
  std::vector<uint32_t> out(n);
  check(qora_generate_greedy(w.raw(), kv.raw(), first, n, out.data()));
  return out;
}

// The reference's generator state (xorshift64); seed it like Rng::new (non-zero).
struct Rng {
  uint64_t state = 1;
};

// GenerateParams' sampling fields (src/generate.rs:8-35 defaults).
struct SamplingParams {
  float temperature = 0.6f;
  float top_p = 0.95f;
  uint32_t top_k = 20;
  float repetition_penalty = 1.1f;
  float presence_penalty = 1.5f;
  int32_t ban_token = -1;
};

// The next token from the last step's logits left on the device: penalties over the
// generated history, then sample_token_top_k; advances rng exactly as the reference.
inline uint32_t sample_next(const DecodeWeights& w, const std::vector<uint32_t>& history, const SamplingParams& p,
                            Rng& rng, uint32_t row = 0) {
  qora_sampling s{p.temperature, p.top_p, p.top_k, p.repetition_penalty, p.presence_penalty, p.ban_token};
  uint32_t tok = 0;
  check(qora_sample(w.raw(), row, history.data(), (uint32_t)history.size(), &s, &rng.state, &tok));
  return tok;
}

}  // namespace qora
