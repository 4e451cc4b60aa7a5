// Parity of the C++ host mirror (qora-llm_b200/host/qora_host.hpp) against the CPU
// oracle, written like the reference's own call sequence (src/generate.rs:135-145,
// :216-235): load_model, raw_prefill, greedy, forward_decode_raw step by step, the error
// behaviour of a bad token, and one sampling step on the device.
//
//   host_parity <model.qora> <n_steps> <prompt ids...>
// Exit status 0 when every check holds; the first failure is printed.
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <vector>

#include "qora_host.hpp"
#include "qora_oracle.h"

static double rel_l2(const std::vector<float>& a, const std::vector<float>& b) {
  double num = 0.0, den = 0.0;
  for (size_t i = 0; i < a.size(); ++i) {
    const double d = (double)a[i] - (double)b[i];
    num += d * d;
    den += (double)b[i] * b[i];
  }
  return std::sqrt(num / (den > 0 ? den : 1e-300));
}

#define CHECK(cond, ...)              \
  do {                                \
    if (!(cond)) {                    \
      std::fprintf(stderr, __VA_ARGS__); \
      std::fprintf(stderr, "\n");     \
      return 1;                       \
    }                                 \
  } while (0)

int main(int argc, char** argv) {
  if (argc < 4) {
    std::fprintf(stderr, "usage: %s model.qora n_steps ids...\n", argv[0]);
    return 2;
  }
  const char* path = argv[1];
  const int n_steps = std::atoi(argv[2]);
  std::vector<uint32_t> ids;
  for (int i = 3; i < argc; ++i) ids.push_back((uint32_t)std::strtoul(argv[i], nullptr, 10));
  try {
    qora::DecodeWeights w = qora::DecodeWeights::load_model(path);
    char err[256] = {0};
    orc_set_threads(8);
    orc_model* om = orc_model_load(path, err, sizeof(err));
    CHECK(om, "oracle load: %s", err);
    orc_kv* okv = orc_kv_new(om);
    const uint32_t V = w.vocab();
    std::vector<float> lo(V);

    auto pre = qora::raw_prefill(w, ids, 256);
    CHECK(orc_prefill(om, ids.data(), ids.size(), okv, lo.data()) == 0, "oracle prefill");
    double worst = rel_l2(pre.first, lo);
    CHECK(worst < 1e-3, "prefill logits rel-L2 %.3e", worst);
    uint32_t tok = qora::greedy(pre.first);
    CHECK(tok == orc_argmax(lo.data(), V), "prefill argmax %u vs %u", tok, orc_argmax(lo.data(), V));
    qora::RawKvCache& kv = pre.second;
    std::vector<uint32_t> history(ids);
    std::vector<float> last = pre.first;
    for (int s = 0; s < n_steps; ++s) {
      history.push_back(tok);
      std::vector<float> lg = qora::forward_decode_raw(w, tok, kv);
      last = lg;
      CHECK(orc_forward_decode(om, tok, okv, lo.data()) == 0, "oracle step");
      const double r = rel_l2(lg, lo);
      worst = r > worst ? r : worst;
      CHECK(r < 1e-3, "step %d logits rel-L2 %.3e", s, r);
      const uint32_t t = qora::greedy(lg), to = orc_argmax(lo.data(), V);
      CHECK(t == to, "step %d greedy %u vs oracle %u", s, t, to);
      tok = t;
    }
    CHECK(kv.len() == ids.size() + (size_t)n_steps, "cache length %u", kv.len());

    // one sampling step on the device-resident logits vs the oracle's restatement on the
    // same logits read back
    qora::SamplingParams sp;
    qora::Rng rng{0x853C49E6748FEA9Bull};
    uint64_t ostate = rng.state;
    const uint32_t sampled = qora::sample_next(w, history, sp, rng);
    const uint32_t osampled = orc_sample(last.data(), V, history.data(), history.size(), sp.temperature, sp.top_p,
                                         sp.top_k, sp.repetition_penalty, sp.presence_penalty, sp.ban_token, &ostate);
    CHECK(sampled == osampled && rng.state == ostate, "sampling %u vs %u", sampled, osampled);

    // error behaviour: a token id past the vocabulary is rejected (the reference panics)
    bool threw = false;
    try {
      qora::forward_decode_raw(w, V, kv);
    } catch (const qora::Error& e) {
      threw = e.status() == QORA_ERR_RANGE;
    }
    CHECK(threw, "an out-of-range token must raise QORA_ERR_RANGE");
    CHECK(kv.len() == ids.size() + (size_t)n_steps, "a rejected step must not advance the cache");

    orc_kv_free(okv);
    orc_model_free(om);
    std::printf("host parity ok: %d steps, worst logits rel-L2 %.3e\n", n_steps, worst);
    return 0;
  } catch (const qora::Error& e) {
    std::fprintf(stderr, "qora::Error %d: %s\n", (int)e.status(), e.what());
    return 1;
  }
}
