// Native merge loops of the GGUF tokenizers (the CPU hot path of long prompts).
//
// Parity: the reference's GgufTokenizer (vocab/src/gguf_tokenizer.rs): SentencePiece-style merging by
// vocabulary score for `llama` vocabularies and GPT-2 byte-level BPE by merge rank for `gpt2`
// ones.  Pre-tokenization (special-token split, the GPT-2 / Llama-3 regex, byte-to-unicode
// mapping) stays in Python; this file runs the merges:
//
// * spm(text): `text` is the prompt with spaces already replaced by U+2581.  Symbols start as
//   single UTF-8 code points in a doubly linked list; a heap holds candidate merges of adjacent
//   symbols whose concatenation is a vocabulary entry, ordered by higher score then lower left
//   position; stale candidates are skipped on pop.  Final symbols map to their ids, unknown ones
//   to their UTF-8 bytes' <0xNN> tokens.
// * bpe(words): each word (already byte-to-unicode mapped) is merged by lowest merge rank, ties
//   to the leftmost pair, with the same linked-list + heap scheme; whole-word vocabulary hits skip
//   the merge loop.
// Both produce exactly the ids of the Python implementation (tested against it).

#include <cstdint>
#include <queue>
#include <string>
#include <string_view>
#include <unordered_map>
#include <vector>

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

namespace py = pybind11;

namespace {

size_t utf8_len(unsigned char c) {
  if (c < 0x80) return 1;
  if ((c >> 5) == 0x6) return 2;
  if ((c >> 4) == 0xE) return 3;
  if ((c >> 3) == 0x1E) return 4;
  return 1;  // invalid lead byte: one byte per symbol (Python never produces this: input is str)
}

struct Sym {
  size_t off, len;
  int prev, next;
  bool alive;
};

class NativeTokenizer {
 public:
  NativeTokenizer(const std::vector<std::string>& tokens, const std::vector<double>& scores,
                  const std::vector<std::string>& merges, const std::vector<int>& byte_ids, int unk_id)
      : scores_(scores), byte_ids_(byte_ids), unk_(unk_id) {
    vocab_.reserve(tokens.size() * 2);
    for (size_t i = 0; i < tokens.size(); ++i) vocab_[tokens[i]] = static_cast<int>(i);  // last duplicate wins
    ranks_.reserve(merges.size() * 2);
    for (size_t r = 0; r < merges.size(); ++r) {
      const std::string& m = merges[r];
      size_t sp = m.find(' ');
      if (sp == std::string::npos) continue;
      // key: left + '\x01' + right (0x01 never occurs in byte-to-unicode mapped text)
      std::string key = m.substr(0, sp);
      key.push_back('\x01');
      key.append(m, sp + 1, std::string::npos);
      ranks_[std::move(key)] = static_cast<int>(r);  // a repeated merge keeps its last rank (dict semantics)
    }
    if (byte_ids_.size() != 256) byte_ids_.assign(256, -1);
  }

  std::vector<int> spm(const std::string& text) const {
    std::vector<int> out;
    std::vector<Sym> s = split(text);
    if (s.empty()) return out;
    struct Cand {
      double score;
      int left, right;
      size_t len;
    };
    auto worse = [](const Cand& a, const Cand& b) {  // max-heap on (score, -left)
      if (a.score != b.score) return a.score < b.score;
      return a.left > b.left;
    };
    std::priority_queue<Cand, std::vector<Cand>, decltype(worse)> heap(worse);
    auto push = [&](int i) {
      int j = s[i].next;
      if (j < 0) return;
      std::string_view cand(text.data() + s[i].off, s[i].len + s[j].len);
      auto it = vocab_.find(std::string(cand));
      if (it != vocab_.end()) heap.push({score(it->second), i, j, cand.size()});
    };
    for (int i = 0; i + 1 < static_cast<int>(s.size()); ++i) push(i);
    while (!heap.empty()) {
      Cand c = heap.top();
      heap.pop();
      if (!s[c.left].alive || !s[c.right].alive || s[c.left].next != c.right ||
          s[c.left].len + s[c.right].len != c.len)
        continue;
      s[c.left].len += s[c.right].len;
      s[c.right].alive = false;
      s[c.left].next = s[c.right].next;
      if (s[c.right].next >= 0) s[s[c.right].next].prev = c.left;
      if (s[c.left].prev >= 0) push(s[c.left].prev);
      push(c.left);
    }
    for (int i = 0; i >= 0; i = s[i].next) emit(text, s[i], out);
    return out;
  }

  std::vector<int> bpe(const std::vector<std::string>& words) const {
    std::vector<int> out;
    for (const std::string& w : words) {
      auto hit = vocab_.find(w);
      if (hit != vocab_.end()) {
        out.push_back(hit->second);
        continue;
      }
      std::vector<Sym> s = split(w);
      if (s.empty()) continue;
      struct Cand {
        int rank, left, right;
        size_t len;
      };
      auto worse = [](const Cand& a, const Cand& b) {  // min-heap on (rank, left)
        if (a.rank != b.rank) return a.rank > b.rank;
        return a.left > b.left;
      };
      std::priority_queue<Cand, std::vector<Cand>, decltype(worse)> heap(worse);
      std::string key;
      auto push = [&](int i) {
        int j = s[i].next;
        if (j < 0) return;
        key.assign(w, s[i].off, s[i].len);
        key.push_back('\x01');
        key.append(w, s[j].off, s[j].len);
        auto it = ranks_.find(key);
        if (it != ranks_.end()) heap.push({it->second, i, j, s[i].len + s[j].len});
      };
      for (int i = 0; i + 1 < static_cast<int>(s.size()); ++i) push(i);
      while (!heap.empty()) {
        Cand c = heap.top();
        heap.pop();
        if (!s[c.left].alive || !s[c.right].alive || s[c.left].next != c.right ||
            s[c.left].len + s[c.right].len != c.len)
          continue;
        s[c.left].len += s[c.right].len;
        s[c.right].alive = false;
        s[c.left].next = s[c.right].next;
        if (s[c.right].next >= 0) s[s[c.right].next].prev = c.left;
        if (s[c.left].prev >= 0) push(s[c.left].prev);
        push(c.left);
      }
      for (int i = 0; i >= 0; i = s[i].next) {
        std::string piece(w, s[i].off, s[i].len);
        auto it = vocab_.find(piece);
        if (it != vocab_.end()) {
          out.push_back(it->second);
        } else {  // every single mapped-byte character is in a byte-level vocabulary
          for (size_t k = 0; k < piece.size();) {
            size_t n = utf8_len(static_cast<unsigned char>(piece[k]));
            auto ch = vocab_.find(piece.substr(k, n));
            if (ch != vocab_.end()) out.push_back(ch->second);
            k += n;
          }
        }
      }
    }
    return out;
  }

  size_t size() const { return vocab_.size(); }

 private:
  double score(int id) const { return id < static_cast<int>(scores_.size()) ? scores_[id] : 0.0; }

  static std::vector<Sym> split(const std::string& t) {
    std::vector<Sym> s;
    for (size_t i = 0; i < t.size();) {
      size_t n = utf8_len(static_cast<unsigned char>(t[i]));
      if (i + n > t.size()) n = t.size() - i;
      int k = static_cast<int>(s.size());
      s.push_back({i, n, k - 1, k + 1, true});
      i += n;
    }
    if (!s.empty()) s.back().next = -1;
    return s;
  }

  void emit(const std::string& text, const Sym& sym, std::vector<int>& out) const {
    auto it = vocab_.find(text.substr(sym.off, sym.len));
    if (it != vocab_.end()) {
      out.push_back(it->second);
      return;
    }
    for (size_t k = 0; k < sym.len; ++k) {
      int b = static_cast<unsigned char>(text[sym.off + k]);
      out.push_back(byte_ids_[b] >= 0 ? byte_ids_[b] : unk_);
    }
  }

  std::unordered_map<std::string, int> vocab_;
  std::unordered_map<std::string, int> ranks_;
  std::vector<double> scores_;
  std::vector<int> byte_ids_;
  int unk_;
};

}  // namespace

void register_tokenizer(py::module_& m) {
  py::class_<NativeTokenizer>(m, "NativeTokenizer")
      .def(py::init<const std::vector<std::string>&, const std::vector<double>&, const std::vector<std::string>&,
                    const std::vector<int>&, int>(),
           py::arg("tokens"), py::arg("scores"), py::arg("merges"), py::arg("byte_ids"), py::arg("unk_id"))
      .def("spm", &NativeTokenizer::spm, py::call_guard<py::gil_scoped_release>())
      .def("bpe", &NativeTokenizer::bpe, py::call_guard<py::gil_scoped_release>())
      .def("__len__", &NativeTokenizer::size);
}
