// Native GBNF recognizer and per-step token masks (constrained generation: grammars, JSON mode).
//
// Parity: the reference's GrammarSampler (sampling/src/grammar_sampler.rs:20-320) masks tokens from
// a fixed root rule and never advances; this recognizer advances with every accepted token.  The
// grammar is parsed in Python (sampling/grammar.py) and handed over as rules -> alternatives ->
// elements; here it is flattened so that every alternative is a run of elements closed by END:
//
//   element = CHAR (code-point ranges, optionally negated) | REF (rule id) | END
//
// A parse stack is a vector of element indices: each entry is the element to match next in its
// alternative, the top one always a CHAR (after expansion) — an empty stack means "complete
// sentence".  A parse state is a sorted, de-duplicated set of stacks.  expand() follows REF and
// END entries to CHAR tops (with a visited set, so left recursion terminates); step() advances
// every stack whose top CHAR accepts a code point.  Masks walk a trie of the vocabulary's token
// strings with the state set and prune dead branches; masks are memoised per state set.  Same
// semantics and outputs as the Python recognizer (tested against it).

#include <algorithm>
#include <cstdint>
#include <functional>
#include <map>
#include <memory>
#include <set>
#include <string>
#include <unordered_map>
#include <vector>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

namespace py = pybind11;

namespace {

using Stack = std::vector<int32_t>;
using State = std::vector<Stack>;  // sorted, unique

struct VecHash {
  size_t operator()(const Stack& s) const {
    size_t h = 1469598103934665603ull;
    for (int32_t v : s) h = (h ^ static_cast<uint32_t>(v)) * 1099511628211ull;
    return h;
  }
};
struct StateHash {
  size_t operator()(const State& st) const {
    size_t h = 0x9e3779b97f4a7c15ull;
    VecHash vh;
    for (const Stack& s : st) h = (h ^ vh(s)) * 0x100000001b3ull + (h >> 7);
    return h;
  }
};

enum Kind : int32_t { END = 0, CHR = 1, REF = 2 };

struct Elem {
  int32_t kind;
  int32_t rule;         // REF
  int32_t r0, r1;       // CHR: ranges_[r0, r1)
  bool neg;
};

void normalize(State& st) {
  std::sort(st.begin(), st.end());
  st.erase(std::unique(st.begin(), st.end()), st.end());
}

class NativeTrie {
 public:
  explicit NativeTrie(const std::vector<py::object>& strings) {
    nodes_.emplace_back();
    token_cps_.resize(strings.size());
    for (size_t tid = 0; tid < strings.size(); ++tid) {
      if (strings[tid].is_none()) continue;
      std::u32string s = py::cast<std::u32string>(strings[tid]);
      if (s.empty()) continue;
      token_cps_[tid].assign(s.begin(), s.end());
      int node = 0;
      for (char32_t ch : s) {
        auto& ch_map = nodes_[node].children;
        auto it = ch_map.find(static_cast<int32_t>(ch));
        int nxt;
        if (it == ch_map.end()) {
          nxt = static_cast<int>(nodes_.size());
          ch_map.emplace(static_cast<int32_t>(ch), nxt);
          nodes_.emplace_back();
        } else {
          nxt = it->second;
        }
        node = nxt;
      }
      nodes_[node].tokens.push_back(static_cast<int32_t>(tid));
    }
    // children as sorted vectors for the walk
    for (auto& n : nodes_) n.kids.assign(n.children.begin(), n.children.end());
  }
  struct Node {
    std::map<int32_t, int> children;
    std::vector<std::pair<int32_t, int>> kids;
    std::vector<int32_t> tokens;
  };
  std::vector<Node> nodes_;
  std::vector<std::vector<int32_t>> token_cps_;
  size_t size() const { return nodes_.size(); }
};

class NativeGrammar {
 public:
  // rules[r][a] = list of elements: ("c", [(lo, hi), ...], negated) or ("r", rule_id)
  NativeGrammar(const py::list& rules, int root) : root_(root) {
    for (auto rule_h : rules) {
      std::vector<int32_t> starts;
      for (auto alt_h : py::cast<py::list>(rule_h)) {
        starts.push_back(static_cast<int32_t>(elems_.size()));
        for (auto el_h : py::cast<py::list>(alt_h)) {
          py::tuple el = py::cast<py::tuple>(el_h);
          std::string kind = py::cast<std::string>(el[0]);
          Elem e{};
          if (kind == "c") {
            e.kind = CHR;
            e.r0 = static_cast<int32_t>(ranges_.size());
            for (auto rg : py::cast<py::list>(el[1])) {
              py::tuple t = py::cast<py::tuple>(rg);
              ranges_.emplace_back(py::cast<int32_t>(t[0]), py::cast<int32_t>(t[1]));
            }
            e.r1 = static_cast<int32_t>(ranges_.size());
            e.neg = py::cast<bool>(el[2]);
          } else {
            e.kind = REF;
            e.rule = py::cast<int32_t>(el[1]);
          }
          elems_.push_back(e);
        }
        elems_.push_back(Elem{END, 0, 0, 0, false});
      }
      alts_.push_back(std::move(starts));
    }
    for (const Elem& e : elems_)
      if (e.kind == REF && (e.rule < 0 || e.rule >= static_cast<int32_t>(alts_.size())))
        throw py::value_error("grammar: reference to an undefined rule");
    if (root_ < 0 || root_ >= static_cast<int>(alts_.size())) throw py::value_error("grammar: bad root rule");
  }

  bool match(int32_t idx, int32_t c) const {
    const Elem& e = elems_[idx];
    bool hit = false;
    for (int32_t k = e.r0; k < e.r1 && !hit; ++k) hit = ranges_[k].first <= c && c <= ranges_[k].second;
    return hit != e.neg;
  }

  // all stacks reachable from `st` whose top is a CHR element (or that are empty), appended to out
  void expand(const Stack& st, State& out) {
    auto hit = expand_cache_.find(st);
    if (hit != expand_cache_.end()) {
      out.insert(out.end(), hit->second.begin(), hit->second.end());
      return;
    }
    State res;
    std::vector<Stack> todo{st};
    std::unordered_map<Stack, bool, VecHash> seen;
    while (!todo.empty()) {
      Stack s = std::move(todo.back());
      todo.pop_back();
      if (!seen.emplace(s, true).second) continue;
      if (s.empty()) {
        res.push_back(s);
        continue;
      }
      const int32_t top = s.back();
      const Elem& e = elems_[top];
      if (e.kind == END) {
        s.pop_back();
        todo.push_back(std::move(s));
      } else if (e.kind == CHR) {
        res.push_back(std::move(s));
      } else {
        s.back() = top + 1;  // continue after the reference once the rule is done
        for (int32_t start : alts_[e.rule]) {
          Stack n = s;
          n.push_back(start);
          todo.push_back(std::move(n));
        }
      }
    }
    normalize(res);
    if (expand_cache_.size() < 200000) expand_cache_.emplace(st, res);
    out.insert(out.end(), res.begin(), res.end());
  }

  State initial() {
    State out;
    for (int32_t start : alts_[root_]) expand(Stack{start}, out);
    normalize(out);
    return out;
  }

  State step(const State& st, int32_t c) {
    State out;
    for (const Stack& s : st) {
      if (s.empty() || !match(s.back(), c)) continue;
      Stack n = s;
      n.back() += 1;
      expand(n, out);
    }
    normalize(out);
    return out;
  }

  // allowed token ids for state `st` over `trie`, memoised per (trie, state)
  const std::vector<int32_t>& allowed(const NativeTrie& trie, const State& st, const std::vector<int32_t>& eos) {
    auto& cache = mask_cache_[&trie];
    auto hit = cache.find(st);
    if (hit != cache.end()) return hit->second;
    std::vector<int32_t> ids;
    std::vector<std::pair<int, State>> todo;
    todo.emplace_back(0, st);
    while (!todo.empty()) {
      auto [node, s] = std::move(todo.back());
      todo.pop_back();
      for (const auto& [ch, child] : trie.nodes_[node].kids) {
        State ns = step(s, ch);
        if (ns.empty()) continue;
        const auto& toks = trie.nodes_[child].tokens;
        ids.insert(ids.end(), toks.begin(), toks.end());
        todo.emplace_back(child, std::move(ns));
      }
    }
    bool complete = std::any_of(st.begin(), st.end(), [](const Stack& s) { return s.empty(); });
    if (complete) ids.insert(ids.end(), eos.begin(), eos.end());
    if (cache.size() >= 4096) cache.clear();
    return cache.emplace(st, std::move(ids)).first->second;
  }

  size_t n_elems() const { return elems_.size(); }

 private:
  int root_;
  std::vector<Elem> elems_;
  std::vector<std::pair<int32_t, int32_t>> ranges_;
  std::vector<std::vector<int32_t>> alts_;
  std::unordered_map<Stack, State, VecHash> expand_cache_;
  std::map<const NativeTrie*, std::unordered_map<State, std::vector<int32_t>, StateHash>> mask_cache_;
};

class NativeMatcher {
 public:
  NativeMatcher(std::shared_ptr<NativeGrammar> g, std::shared_ptr<NativeTrie> t, std::vector<int32_t> eos)
      : g_(std::move(g)), t_(std::move(t)), eos_(std::move(eos)) {
    st_ = g_->initial();
  }

  std::vector<int32_t> allowed_ids() { return g_->allowed(*t_, st_, eos_); }

  py::array_t<uint32_t> allowed_mask(int64_t words) {
    std::vector<int32_t> ids;
    {
      py::gil_scoped_release nogil;
      ids = g_->allowed(*t_, st_, eos_);
    }
    if (ids.empty()) ids = eos_;  // dead end: let the model finish instead of emitting garbage
    py::array_t<uint32_t> m(words);
    auto* p = m.mutable_data();
    std::fill(p, p + words, 0u);
    for (int32_t id : ids)
      if (id >= 0 && id < words * 32) p[id >> 5] |= 1u << (id & 31);  // bit i of word w: token 32w+i
    return m;
  }

  void accept(int32_t tid) {
    if (std::find(eos_.begin(), eos_.end(), tid) != eos_.end()) {
      st_.clear();
      return;
    }
    if (tid < 0 || tid >= static_cast<int32_t>(t_->token_cps_.size())) return;
    for (int32_t c : t_->token_cps_[tid]) {
      st_ = g_->step(st_, c);
      if (st_.empty()) break;
    }
  }

  void accept_text(const std::u32string& s) {
    for (char32_t c : s) {
      st_ = g_->step(st_, static_cast<int32_t>(c));
      if (st_.empty()) break;
    }
  }

  bool done() const {
    return !std::any_of(st_.begin(), st_.end(), [](const Stack& s) { return !s.empty(); });
  }
  bool complete() const {
    return std::any_of(st_.begin(), st_.end(), [](const Stack& s) { return s.empty(); });
  }
  size_t n_stacks() const { return st_.size(); }

 private:
  std::shared_ptr<NativeGrammar> g_;
  std::shared_ptr<NativeTrie> t_;
  std::vector<int32_t> eos_;
  State st_;
};

}  // namespace

void register_grammar(py::module_& m) {
  py::class_<NativeTrie, std::shared_ptr<NativeTrie>>(m, "NativeTrie")
      .def(py::init<const std::vector<py::object>&>())
      .def("__len__", &NativeTrie::size);
  py::class_<NativeGrammar, std::shared_ptr<NativeGrammar>>(m, "NativeGrammar")
      .def(py::init<const py::list&, int>())
      .def("n_elems", &NativeGrammar::n_elems);
  py::class_<NativeMatcher>(m, "NativeMatcher")
      .def(py::init<std::shared_ptr<NativeGrammar>, std::shared_ptr<NativeTrie>, std::vector<int32_t>>())
      .def("allowed_ids", &NativeMatcher::allowed_ids, py::call_guard<py::gil_scoped_release>())
      .def("allowed_mask", &NativeMatcher::allowed_mask)
      .def("accept", &NativeMatcher::accept)
      .def("accept_text", &NativeMatcher::accept_text)
      .def("done", &NativeMatcher::done)
      .def("complete", &NativeMatcher::complete)
      .def("n_stacks", &NativeMatcher::n_stacks);
}
