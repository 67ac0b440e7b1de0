// Native continuous-batching scheduler core: waiting / running queues, chunked prefill under a
// per-step token budget, admission against free KV blocks with radix prefix-cache hits, sliding-
// window block release and preemption (recompute) of the youngest sequence.
//
// Parity: the reference's BatchScheduler (advanced/src/continuous_batching.rs:27-180: pending
// queue, admission up to max_sequences, fill_batch of prompts for new sequences and last tokens for
// running ones) and the batch engine around it (advanced/src/batch_engine.rs:72-191), both Rust.
// The paged-memory model (admission against the block pool, prefix reuse, preemption) is this
// framework's; engine/scheduler.py states the same policy in Python, and the tests drive both with
// the same random workloads and require identical plans, block tables and pool state.
//
// Ownership: the core holds every sequence's scheduling state (tokens, cached length, block table,
// queue position).  The Python Sequence objects mirror it: after each schedule() the binding
// returns the records of the sequences whose state changed, and after each engine step commit()
// hands back the cached lengths and sampled tokens.  Block ids come from the shared BlockPool, so
// the Python side and the core never disagree about ownership.
#include <algorithm>
#include <deque>
#include <stdexcept>
#include <string>
#include <tuple>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "kvcache_native.h"

namespace py = pybind11;

namespace barq_native {
namespace {

enum Status : int { kWaiting = 0, kRunning = 1, kFinished = 2 };

struct Seq {
  long id = 0;
  double arrival = 0;
  std::vector<int> tokens;  // prompt + output
  int n_cached = 0;
  std::vector<int> table;
  int window_freed = 0;
  long gen = 0;             // bumped when the table is replaced or rewritten (not when it grows)
  int n_preempted = 0;
  int prefix_hit = 0;
  bool embeds = false;      // prompt positions with given embeddings: no prefix-cache reuse
  int status = kWaiting;
  int n_tokens() const { return (int)tokens.size(); }
  int n_uncached() const { return n_tokens() - n_cached; }
};

class Scheduler {
 public:
  Scheduler(BlockPool& pool, RadixCache* cache, int max_num_seqs, int max_batched_tokens, bool chunked_prefill,
            int sliding_window)
      : pool_(pool), cache_(cache), max_seqs_(max_num_seqs), max_tokens_(max_batched_tokens),
        chunked_(chunked_prefill), window_(sliding_window) {
    if (max_num_seqs <= 0 || max_batched_tokens <= 0)
      throw std::invalid_argument("Scheduler: max_num_seqs and max_num_batched_tokens must be positive");
  }

  void add(long id, double arrival, const std::vector<int>& prompt, bool embeds) {
    if (seqs_.count(id)) throw std::invalid_argument("sequence " + std::to_string(id) + " already added");
    if (prompt.empty()) throw std::invalid_argument("empty prompt");
    Seq s;
    s.id = id, s.arrival = arrival, s.tokens = prompt, s.embeds = embeds;
    seqs_.emplace(id, std::move(s));
    waiting_.push_back(id);
    dirty_.insert(id);
  }

  // The engine ran a step: the new cached length of each listed sequence and the tokens appended
  // to it since the previous commit (flattened; `n_append[i]` of them belong to ids[i]).
  void commit(const std::vector<long>& ids, const std::vector<int>& n_cached, const std::vector<int>& n_append,
              const std::vector<int>& tokens) {
    if (ids.size() != n_cached.size() || ids.size() != n_append.size())
      throw std::invalid_argument("commit: ids, n_cached and n_append differ in length");
    size_t off = 0;
    for (size_t i = 0; i < ids.size(); ++i) {
      Seq& s = at(ids[i]);
      if (off + (size_t)n_append[i] > tokens.size()) throw std::invalid_argument("commit: too few tokens");
      s.tokens.insert(s.tokens.end(), tokens.begin() + off, tokens.begin() + off + n_append[i]);
      off += (size_t)n_append[i];
      if (n_cached[i] < 0 || n_cached[i] > s.n_tokens()) throw std::invalid_argument("commit: n_cached out of range");
      s.n_cached = n_cached[i];
    }
    if (off != tokens.size()) throw std::invalid_argument("commit: too many tokens");
  }

  void finish(long id) {
    Seq& s = at(id);
    s.status = kFinished;
    if (cache_ && !s.embeds && !s.window_freed)
      cache_->insert(std::vector<int>(s.tokens.begin(), s.tokens.begin() + s.n_cached), s.table);
    free_seq(s);
    erase(running_, id);
    auto w = std::find(waiting_.begin(), waiting_.end(), id);
    if (w != waiting_.end()) waiting_.erase(w);
    dirty_.insert(id);
  }

  bool abort(long id) {
    Seq& s = at(id);
    if (s.status == kFinished) return false;
    auto it = std::find(waiting_.begin(), waiting_.end(), id);
    if (it != waiting_.end()) {
      waiting_.erase(it);
      s.status = kFinished;
      free_seq(s);
      dirty_.insert(id);
      return true;
    }
    finish(id);
    return true;
  }

  // A finished sequence's record is no longer needed once the caller has read it.
  void forget(long id) {
    auto it = seqs_.find(id);
    if (it != seqs_.end() && it->second.status == kFinished) seqs_.erase(it), dirty_.erase(id);
  }

  // (kind: 0 none / 1 prefill / 2 decode, ids, new tokens per id)
  std::tuple<int, std::vector<long>, std::vector<int>> schedule() {
    if (window_ > 0)
      for (long id : running_) trim_window(at(id));
    std::vector<long> ids;
    std::vector<int> n_new;
    int budget = max_tokens_;
    // 1) continue the chunked prefills of running sequences
    std::vector<long> pre;
    for (long id : running_)
      if (at(id).n_uncached() > 1) pre.push_back(id);
    for (long id : pre) {
      Seq& s = at(id);
      if (s.status != kRunning) continue;  // preempted to make room for a chunk scheduled above
      const int n = std::min(s.n_uncached(), budget);
      if (n <= 0) break;
      std::vector<long> protect = ids;     // this step's plan is never preempted for a later entry
      protect.push_back(id);
      if (!reserve(s, s.n_cached + n, protect)) break;
      ids.push_back(id);
      n_new.push_back(n);
      budget -= n;
    }
    // 2) admit waiting sequences
    while (!waiting_.empty() && budget > 0 && (int)running_.size() < max_seqs_) {
      Seq& s = at(waiting_.front());
      if (cache_ && s.table.empty() && !s.embeds) {
        auto hit = cache_->match(std::vector<int>(s.tokens.begin(), s.tokens.end() - 1));
        if (!hit.first.empty()) {
          pool_.retain(hit.first);
          s.table = hit.first;
          ++s.gen;
          s.n_cached = hit.second;
          s.prefix_hit = hit.second;
          dirty_.insert(s.id);
        }
      }
      const int total = s.n_uncached();
      const int n = total <= budget ? total : (chunked_ ? budget : 0);
      if (n <= 0) break;
      const int need = pool_.blocks_for(s.n_cached + n) - (int)s.table.size();
      if (!pool_.can_allocate(need)) {
        if (cache_ && cache_->evict(need - pool_.n_free()) > 0) continue;
        if (!s.table.empty() && s.prefix_hit) free_seq(s);
        break;
      }
      waiting_.pop_front();
      grow(s, s.n_cached + n);
      s.status = kRunning;
      running_.push_back(s.id);
      ids.push_back(s.id);
      n_new.push_back(n);
      budget -= n;
    }
    if (!ids.empty()) return {1, ids, n_new};
    // 3) one token for every running sequence, oldest first
    if (running_.empty()) return {0, {}, {}};
    std::vector<long> order = running_;
    std::stable_sort(order.begin(), order.end(), [&](long a, long b) { return at(a).arrival < at(b).arrival; });
    const long p0 = n_preemptions_;
    const int cap = pool_.block_size();
    for (long id : order) {
      Seq& s = at(id);
      if (n_preemptions_ != p0 && s.status != kRunning) continue;
      if (s.n_tokens() <= (int)s.table.size() * cap || reserve(s, s.n_tokens(), {id})) ids.push_back(id);
    }
    if (n_preemptions_ != p0)
      ids.erase(std::remove_if(ids.begin(), ids.end(), [&](long id) { return at(id).status != kRunning; }), ids.end());
    if (ids.empty()) return {0, {}, {}};
    return {2, ids, std::vector<int>(ids.size(), 1)};
  }

  // (id, status, n_cached, window_freed, gen, n_preempted, prefix_hit, block table) of every
  // sequence changed since the previous call
  std::vector<std::tuple<long, int, int, int, long, int, int, std::vector<int>>> take_changes() {
    std::vector<std::tuple<long, int, int, int, long, int, int, std::vector<int>>> out;
    out.reserve(dirty_.size());
    for (long id : dirty_) {
      const Seq& s = at(id);
      out.emplace_back(id, s.status, s.n_cached, s.window_freed, s.gen, s.n_preempted, s.prefix_hit, s.table);
    }
    dirty_.clear();
    return out;
  }

  std::vector<long> waiting_ids() const { return {waiting_.begin(), waiting_.end()}; }
  const std::vector<long>& running_ids() const { return running_; }
  size_t n_waiting() const { return waiting_.size(); }
  size_t n_running() const { return running_.size(); }
  long n_preemptions() const { return n_preemptions_; }
  long n_window_freed() const { return n_window_freed_; }
  int dummy_block() const { return dummy_; }
  void set_dummy_block(int b) { dummy_ = b; }
  std::vector<int> table(long id) { return at(id).table; }

 private:
  Seq& at(long id) {
    auto it = seqs_.find(id);
    if (it == seqs_.end()) throw std::out_of_range("unknown sequence " + std::to_string(id));
    return it->second;
  }
  static void erase(std::vector<long>& v, long id) {
    auto it = std::find(v.begin(), v.end(), id);
    if (it != v.end()) v.erase(it);
  }

  void free_seq(Seq& s) {
    if (!s.table.empty()) pool_.release(std::vector<int>(s.table.begin() + s.window_freed, s.table.end()));
    s.table.clear();
    ++s.gen;
    s.n_cached = 0;
    s.window_freed = 0;
    dirty_.insert(s.id);
  }

  void grow(Seq& s, int n_tokens) {
    const int need = pool_.blocks_for(n_tokens) - (int)s.table.size();
    if (need <= 0) return;
    const std::vector<int> add = pool_.allocate(need);
    s.table.insert(s.table.end(), add.begin(), add.end());
    dirty_.insert(s.id);
  }

  // blocks wholly below the next query's window [n_cached - W + 1, n_cached] are dead
  void trim_window(Seq& s) {
    if (window_ <= 0 || dummy_ < 0) return;
    const int dead = std::min(std::max(0, s.n_cached - window_ + 1) / pool_.block_size(), (int)s.table.size());
    if (dead <= s.window_freed) return;
    pool_.release(std::vector<int>(s.table.begin() + s.window_freed, s.table.begin() + dead));
    n_window_freed_ += dead - s.window_freed;
    std::fill(s.table.begin() + s.window_freed, s.table.begin() + dead, dummy_);
    ++s.gen;
    s.window_freed = dead;
    dirty_.insert(s.id);
  }

  bool preempt_youngest(const std::vector<long>& protect) {
    long victim = -1;
    double best = 0;
    for (long id : running_) {  // the first of the latest arrivals, in running order
      if (std::find(protect.begin(), protect.end(), id) != protect.end()) continue;
      const double a = at(id).arrival;
      if (victim < 0 || a > best) victim = id, best = a;
    }
    if (victim < 0) return false;
    Seq& v = at(victim);
    erase(running_, victim);
    free_seq(v);
    v.status = kWaiting;
    ++v.n_preempted;
    ++n_preemptions_;
    waiting_.push_front(victim);
    return true;
  }

  bool reserve(Seq& s, int n_tokens, const std::vector<long>& protect) {
    const int need = pool_.blocks_for(n_tokens) - (int)s.table.size();
    while (need > pool_.n_free()) {
      if (cache_ && cache_->evict(need - pool_.n_free()) > 0) continue;
      if (!preempt_youngest(protect)) return false;
    }
    grow(s, n_tokens);
    return true;
  }

  BlockPool& pool_;
  RadixCache* cache_;
  int max_seqs_, max_tokens_;
  bool chunked_;
  int window_;
  int dummy_ = -1;
  std::unordered_map<long, Seq> seqs_;
  std::deque<long> waiting_;
  std::vector<long> running_;
  std::unordered_set<long> dirty_;
  long n_preemptions_ = 0, n_window_freed_ = 0;
};

}  // namespace
}  // namespace barq_native

void register_scheduler(py::module_& m) {
  using barq_native::Scheduler;
  py::class_<Scheduler>(m, "Scheduler")
      .def(py::init<barq_native::BlockPool&, barq_native::RadixCache*, int, int, bool, int>(), py::arg("pool"),
           py::arg("cache"), py::arg("max_num_seqs"), py::arg("max_num_batched_tokens"),
           py::arg("chunked_prefill"), py::arg("sliding_window"), py::keep_alive<1, 2>(), py::keep_alive<1, 3>())
      .def("add", &Scheduler::add)
      .def("commit", &Scheduler::commit)
      .def("finish", &Scheduler::finish)
      .def("abort", &Scheduler::abort)
      .def("forget", &Scheduler::forget)
      .def("schedule", &Scheduler::schedule)
      .def("take_changes", &Scheduler::take_changes)
      .def("waiting_ids", &Scheduler::waiting_ids)
      .def("running_ids", &Scheduler::running_ids)
      .def("table", &Scheduler::table)
      .def_property_readonly("n_waiting", &Scheduler::n_waiting)
      .def_property_readonly("n_running", &Scheduler::n_running)
      .def_property_readonly("n_preemptions", &Scheduler::n_preemptions)
      .def_property_readonly("n_window_freed", &Scheduler::n_window_freed)
      .def_property("dummy_block", &Scheduler::dummy_block, &Scheduler::set_dummy_block);
}
