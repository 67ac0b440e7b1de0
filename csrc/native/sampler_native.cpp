// Native host-side sampler chain for the samplers the fused device sampler does not run:
// Mirostat v1 / v2, locally typical sampling and XTC, with the repetition / frequency / presence
// penalties, temperature, top-k, top-p and min-p around them.
//
// Parity: the reference's sampler set (sampling/src/lib.rs:54-65, penalties.rs:7-442; Rust).  The
// algorithms follow the published methods, as the Python chain in sampling/host_samplers.py does
// (that chain is the oracle of tests/test_sampler_native.py: identical kept-token sets and final
// distributions, sample frequencies within sampling error):
//   * Mirostat v1 / v2: Basu et al., "Mirostat: a neural text decoding algorithm that directly
//     controls perplexity" (ICLR 2021): Zipf exponent estimated from the top 100 probabilities (v1),
//     truncation at surprise <= mu (v2), mu -= eta * (observed surprise - tau).
//   * Locally typical sampling: Meister et al., "Locally Typical Sampling" (TACL 2022).
//   * XTC: with probability p, drop every token above the threshold except the least likely one.
// Order of the chain: penalties, temperature, top-k, typical, top-p, min-p, XTC, then a draw from
// the softmax over the kept tokens.
//
// Cost: the torch chain sorts the whole vocabulary row for top-p and typical; here the candidates
// are ordered by a partial sort over a prefix that grows 4x until the kept mass is reached, and the
// k-th largest logit comes from nth_element, so a 128k-token row costs a few linear passes.
#include <algorithm>
#include <cmath>
#include <cstdint>
#include <limits>
#include <numeric>
#include <random>
#include <stdexcept>
#include <tuple>
#include <unordered_map>
#include <vector>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

namespace py = pybind11;

namespace {

constexpr float kNegInf = -std::numeric_limits<float>::infinity();

struct SamplerParams {
  double temperature = 1.0;
  int top_k = 0;
  double top_p = 1.0, min_p = 0.0, typical_p = 1.0;
  double repetition = 1.0, frequency = 0.0, presence = 0.0;
  int mirostat = 0;
  double tau = 5.0, eta = 0.1;
  double xtc_probability = 0.0, xtc_threshold = 0.1;
};

class HostSampler {
 public:
  HostSampler(const SamplerParams& p, int vocab, uint64_t seed)
      : p_(p), vocab_(vocab), rng_(seed), mu_(2.0 * p.tau) {
    if (vocab <= 0) throw std::invalid_argument("HostSampler: vocab must be positive");
  }

  double mu() const { return mu_; }
  void set_mu(double m) { mu_ = m; }

  int sample(py::array_t<float, py::array::c_style | py::array::forcecast> logits, const std::vector<int>& history) {
    std::vector<float> lg = prepare(logits, history);
    if (p_.temperature <= 0.0) return argmax(lg);
    scale(lg);
    if (p_.mirostat == 1 || p_.mirostat == 2) {
      std::vector<int> ids;
      std::vector<double> probs, full;
      mirostat_candidates(lg, ids, probs, full);
      const int j = draw(probs);
      const double s = p_.mirostat == 1 ? -std::log2(std::max(1e-30, full[j])) : -std::log2(std::max(1e-30, probs[j]));
      mu_ -= p_.eta * (s - p_.tau);
      return ids[j];
    }
    std::vector<int> cand = chain(lg, true);
    std::vector<double> pr = softmax(lg, cand);
    return cand[draw(pr)];
  }

  // The distribution the next sample() draws from (no state change, XTC off): (ids, probabilities).
  std::pair<std::vector<int>, std::vector<double>> distribution(
      py::array_t<float, py::array::c_style | py::array::forcecast> logits, const std::vector<int>& history) {
    std::vector<float> lg = prepare(logits, history);
    if (p_.temperature <= 0.0) return {{argmax(lg)}, {1.0}};
    scale(lg);
    if (p_.mirostat == 1 || p_.mirostat == 2) {
      std::vector<int> ids;
      std::vector<double> probs, full;
      mirostat_candidates(lg, ids, probs, full);
      return {ids, probs};
    }
    std::vector<int> cand = chain(lg, false);
    std::vector<double> pr = softmax(lg, cand);
    return {cand, pr};
  }

 private:
  std::vector<float> prepare(const py::array_t<float, py::array::c_style | py::array::forcecast>& logits,
                             const std::vector<int>& history) const {
    if (logits.ndim() != 1 || logits.shape(0) < vocab_) throw std::invalid_argument("logits must be 1-D with >= vocab entries");
    const float* src = logits.data();
    std::vector<float> lg(src, src + vocab_);
    if (!history.empty() && (p_.repetition != 1.0 || p_.frequency != 0.0 || p_.presence != 0.0)) {
      std::unordered_map<int, int> counts;
      for (int t : history)
        if (t >= 0 && t < vocab_) ++counts[t];
      for (const auto& kv : counts) {
        float v = lg[kv.first];
        // float32 arithmetic, as the torch chain does it
        const float rep = (float)p_.repetition;
        if (p_.repetition != 1.0) v = v > 0 ? v / rep : v * rep;
        v = v - (float)kv.second * (float)p_.frequency - (float)p_.presence;
        lg[kv.first] = v;
      }
    }
    return lg;
  }

  void scale(std::vector<float>& lg) const {
    const float t = (float)p_.temperature;
    for (float& v : lg) v = v / t;
  }

  static int argmax(const std::vector<float>& lg) {
    return (int)(std::max_element(lg.begin(), lg.end()) - lg.begin());  // first maximum
  }

  // softmax of lg over the candidates, in candidate order
  static std::vector<double> softmax(const std::vector<float>& lg, const std::vector<int>& cand) {
    double mx = -std::numeric_limits<double>::infinity();
    for (int i : cand) mx = std::max(mx, (double)lg[i]);
    std::vector<double> pr(cand.size());
    double z = 0;
    for (size_t j = 0; j < cand.size(); ++j) z += pr[j] = std::exp((double)lg[cand[j]] - mx);
    for (double& v : pr) v /= z;
    return pr;
  }

  double uniform() { return (double)(rng_() >> 11) * (1.0 / 9007199254740992.0); }

  // inverse-CDF draw over probabilities that sum to one
  int draw(const std::vector<double>& pr) {
    const double u = uniform();
    double c = 0;
    for (size_t j = 0; j < pr.size(); ++j) {
      c += pr[j];
      if (u < c) return (int)j;
    }
    for (size_t j = pr.size(); j-- > 0;)  // rounding left u above the total: last non-zero entry
      if (pr[j] > 0) return (int)j;
    return 0;
  }

  // Order `cand` by `key` ascending over a prefix that grows until the running sum of `mass`
  // (indexed like lg) along that order reaches `target`; returns the length of the kept prefix:
  // every entry up to and including the one at which the sum first reaches the target.
  template <typename Key>
  static size_t ordered_prefix(std::vector<int>& cand, const std::vector<double>& mass, double target, Key key) {
    size_t m = std::min<size_t>(cand.size(), 256);
    for (;;) {
      std::partial_sort(cand.begin(), cand.begin() + m, cand.end(),
                        [&](int a, int b) { return key(a) < key(b); });
      double c = 0;
      for (size_t j = 0; j < m; ++j) {
        c += mass[cand[j]];
        if (c >= target) return j + 1;
      }
      if (m == cand.size()) return m;
      m = std::min(cand.size(), m * 4);
    }
  }

  // penalties and temperature already applied; masked entries of lg become -inf
  std::vector<int> chain(std::vector<float>& lg, bool allow_xtc) {
    const int V = vocab_;
    std::vector<int> cand(V);
    std::iota(cand.begin(), cand.end(), 0);
    // top-k: keep the logits >= the k-th largest
    if (p_.top_k > 0 && p_.top_k < V) {
      std::vector<float> tmp(lg);
      std::nth_element(tmp.begin(), tmp.begin() + (p_.top_k - 1), tmp.end(), std::greater<float>());
      const float th = tmp[p_.top_k - 1];
      cand.clear();
      for (int i = 0; i < V; ++i)
        if (lg[i] >= th) cand.push_back(i);
        else lg[i] = kNegInf;
    }
    std::vector<double> prob(V, 0.0);
    auto fill_prob = [&]() {
      const std::vector<double> pr = softmax(lg, cand);
      for (size_t j = 0; j < cand.size(); ++j) prob[cand[j]] = pr[j];
    };
    auto restrict_to = [&](size_t n_keep) {
      std::vector<char> keep(V, 0);
      for (size_t j = 0; j < n_keep; ++j) keep[cand[j]] = 1;
      std::vector<int> out;
      out.reserve(n_keep);
      for (int i : cand)
        if (keep[i]) out.push_back(i);
        else lg[i] = kNegInf;
      std::sort(out.begin(), out.end());
      cand.swap(out);
    };
    // locally typical: the tokens whose surprise is closest to the entropy, until mass >= p
    if (p_.typical_p < 1.0) {
      fill_prob();
      double ent = 0;
      for (int i : cand)
        if (prob[i] > 0) ent -= prob[i] * std::log(prob[i]);
      std::vector<double> shifted(V);
      for (int i : cand) shifted[i] = prob[i] > 0 ? std::fabs(-std::log(prob[i]) - ent) : HUGE_VAL;
      const size_t n = ordered_prefix(cand, prob, p_.typical_p, [&](int i) { return shifted[i]; });
      restrict_to(std::max<size_t>(1, n));
    }
    // top-p: the most likely tokens until the mass before the next one reaches p
    if (p_.top_p < 1.0) {
      fill_prob();
      const size_t n = ordered_prefix(cand, prob, p_.top_p, [&](int i) { return -(double)lg[i]; });
      restrict_to(std::max<size_t>(1, n));
    }
    // min-p: tokens at least p times as likely as the most likely one
    if (p_.min_p > 0.0) {
      fill_prob();
      double mx = 0;
      for (int i : cand) mx = std::max(mx, prob[i]);
      std::vector<int> out;
      for (int i : cand)
        if (prob[i] >= p_.min_p * mx) out.push_back(i);
        else lg[i] = kNegInf;
      cand.swap(out);
    }
    // XTC: with probability p, keep only the least likely of the tokens above the threshold
    if (allow_xtc && p_.xtc_probability > 0.0 && uniform() < p_.xtc_probability) {
      fill_prob();
      int keep = -1, n_above = 0;
      for (int i : cand)
        if (prob[i] > p_.xtc_threshold) {
          ++n_above;
          if (keep < 0 || prob[i] < prob[keep]) keep = i;
        }
      if (n_above >= 2) {
        std::vector<int> out;
        for (int i : cand)
          if (prob[i] > p_.xtc_threshold && i != keep) lg[i] = kNegInf;
          else out.push_back(i);
        cand.swap(out);
      }
    }
    return cand;
  }

  // Mirostat candidates (the k most likely ids, in no particular order), their renormalised
  // probabilities, and their probabilities under the full distribution
  void mirostat_candidates(const std::vector<float>& lg, std::vector<int>& ids, std::vector<double>& probs,
                           std::vector<double>& full) const {
    const int N = vocab_;
    double mx = -std::numeric_limits<double>::infinity();
    for (float v : lg) mx = std::max(mx, (double)v);
    double z = 0;
    for (float v : lg) z += std::exp((double)v - mx);
    auto prob = [&](int i) { return std::exp((double)lg[i] - mx) / z; };
    std::vector<int> order(N);
    std::iota(order.begin(), order.end(), 0);
    auto desc = [&](int a, int b) { return lg[a] > lg[b] || (lg[a] == lg[b] && a < b); };
    int k;
    if (p_.mirostat == 1) {
      const int n = std::min(100, N - 1);
      std::partial_sort(order.begin(), order.begin() + std::max(n, 1), order.end(), desc);
      double tb = 0, tt = 0;
      for (int i = 1; i < n; ++i) {
        const double t = std::log((double)(i + 1) / i);
        const double b = std::log(prob(order[i - 1]) / prob(order[i]));
        tb += t * b;
        tt += t * t;
      }
      const double s_hat = tt > 0 ? tb / tt : 1.0;
      const double e = s_hat - 1;
      double kf = N;
      if (e > 0) kf = std::pow((e * std::pow(2.0, mu_)) / (1 - std::pow((double)N, -e)), 1 / s_hat);
      kf = std::nearbyint(std::min((double)N, std::max(1.0, kf)));  // round half to even
      k = (int)kf;
    } else {
      k = 0;  // tokens with surprise <= mu, i.e. probability >= 2^-mu
      for (int i = 0; i < N; ++i)
        if (-std::log2(std::max(1e-30, prob(i))) <= mu_) ++k;
      k = std::max(1, k);
    }
    if (k < N) std::nth_element(order.begin(), order.begin() + (k - 1), order.end(), desc);  // the top k, unordered
    ids.assign(order.begin(), order.begin() + k);
    full.resize(k);
    probs.resize(k);
    double zk = 0;
    for (int j = 0; j < k; ++j) zk += full[j] = prob(ids[j]);
    for (int j = 0; j < k; ++j) probs[j] = full[j] / zk;
  }

  SamplerParams p_;
  int vocab_;
  std::mt19937_64 rng_;
  double mu_;
};

}  // namespace

void register_sampler(py::module_& m) {
  py::class_<HostSampler>(m, "HostSampler")
      .def(py::init([](int vocab, uint64_t seed, double temperature, int top_k, double top_p, double min_p,
                       double typical_p, double repetition, double frequency, double presence, int mirostat,
                       double tau, double eta, double xtc_probability, double xtc_threshold) {
             SamplerParams p;
             p.temperature = temperature, p.top_k = top_k, p.top_p = top_p, p.min_p = min_p;
             p.typical_p = typical_p, p.repetition = repetition, p.frequency = frequency, p.presence = presence;
             p.mirostat = mirostat, p.tau = tau, p.eta = eta;
             p.xtc_probability = xtc_probability, p.xtc_threshold = xtc_threshold;
             return HostSampler(p, vocab, seed);
           }),
           py::arg("vocab"), py::arg("seed"), py::arg("temperature"), py::arg("top_k"), py::arg("top_p"),
           py::arg("min_p"), py::arg("typical_p"), py::arg("repetition"), py::arg("frequency"), py::arg("presence"),
           py::arg("mirostat"), py::arg("tau"), py::arg("eta"), py::arg("xtc_probability"), py::arg("xtc_threshold"))
      .def("sample", &HostSampler::sample, py::arg("logits"), py::arg("history"))
      .def("distribution", &HostSampler::distribution, py::arg("logits"), py::arg("history"))
      .def_property("mu", &HostSampler::mu, &HostSampler::set_mu);
}
