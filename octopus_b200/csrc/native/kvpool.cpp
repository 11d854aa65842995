// Host-side KV memory manager of the rollout engine (module octopus_b200._native).
//
// SlotPool     page-size-1 KV slots with holder refcounts.  A slot returns to the free
//              list only when its last holder releases it, so a page shared by a radix
//              node, a cursor, a running request and any number of mounts is freed
//              exactly once ("owned" = no other holder).
// RadixCache   token-sequence -> slot-list prefix cache (compressed radix tree) with
//              per-node lock counts and LRU eviction of unlocked leaves.  Nodes are
//              namespaced by a 64-bit key (weight version / adapter), so the same tokens
//              under different weights never share KV.
//
// Reference parity (behaviour): SGLang's radix cache + token-to-KV pool as patched by
// `octopus/serving/kv_mount.py:460-550` (lend: shared-page holder refcounts; owned: free
// only pages with no other holder; stats) and the zero-copy fuzz invariants of
// `tests/test_sglang_mount.py:254-420` (pool balance, no double free, no freed-but-held
// slot).
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <list>
#include <map>
#include <memory>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace octo_native {

class SlotPool {
 public:
  // Free slots are kept as coalesced runs [start, start + len) ordered by address, and
  // alloc(n) takes the lowest-addressed run that holds all n (else the lowest runs in
  // turn), so a request's slots come out ascending and, while the pool is not fragmented,
  // consecutive: the decode kernels then stream a sequence's keys with tiled TMA copies.
  explicit SlotPool(int64_t capacity) : cap_(capacity), ref_(capacity, 0), free_n_(capacity) {
    if (capacity > 0) runs_.emplace(0, capacity);
  }
  int64_t capacity() const { return cap_; }
  int64_t free_count() const { return free_n_; }
  int64_t used_count() const { return cap_ - free_n_; }

  // Allocate n slots with refcount 1; returns an empty vector if not enough are free.
  std::vector<int64_t> alloc(int64_t n) {
    std::vector<int64_t> out;
    if (n <= 0 || n > free_n_) return out;
    out.reserve(n);
    auto it = runs_.begin();
    for (; it != runs_.end(); ++it)
      if (it->second >= n) break;
    if (it != runs_.end()) {
      take(it, n, out);
    } else {
      while (static_cast<int64_t>(out.size()) < n) take(runs_.begin(), n - static_cast<int64_t>(out.size()), out);
    }
    return out;
  }
  void incref(const int64_t* s, int64_t n) {
    for (int64_t i = 0; i < n; ++i) {
      check(s[i]);
      if (ref_[s[i]] <= 0) throw std::runtime_error("incref of a free slot " + std::to_string(s[i]));
      ++ref_[s[i]];
    }
  }
  // Returns how many slots became free.
  int64_t decref(const int64_t* s, int64_t n) {
    std::vector<int64_t> freed;
    for (int64_t i = 0; i < n; ++i) {
      check(s[i]);
      if (ref_[s[i]] <= 0) throw std::runtime_error("double free of slot " + std::to_string(s[i]));
      if (--ref_[s[i]] == 0) freed.push_back(s[i]);
    }
    std::sort(freed.begin(), freed.end());
    for (size_t i = 0; i < freed.size();) {  // consecutive freed slots go back as one run
      size_t j = i + 1;
      while (j < freed.size() && freed[j] == freed[j - 1] + 1) ++j;
      give(freed[i], static_cast<int64_t>(j - i));
      i = j;
    }
    return static_cast<int64_t>(freed.size());
  }
  int32_t refcount(int64_t s) const {
    check(s);
    return ref_[s];
  }
  // Invariant check: every slot is either free (ref 0, in exactly one run) or held, and
  // runs are disjoint, non-adjacent and counted.
  bool check_invariants() const {
    std::vector<uint8_t> seen(cap_, 0);
    int64_t total = 0, prev_end = -1;
    for (const auto& r : runs_) {
      if (r.second <= 0 || r.first < 0 || r.first + r.second > cap_ || r.first <= prev_end) return false;
      for (int64_t s = r.first; s < r.first + r.second; ++s) {
        if (seen[s] || ref_[s] != 0) return false;
        seen[s] = 1;
      }
      prev_end = r.first + r.second;
      total += r.second;
    }
    if (total != free_n_) return false;
    for (int64_t s = 0; s < cap_; ++s)
      if (!seen[s] && ref_[s] <= 0) return false;
    return true;
  }

 private:
  void check(int64_t s) const {
    if (s < 0 || s >= cap_) throw std::out_of_range("slot id out of range " + std::to_string(s));
  }
  // up to `want` slots from the front of run `it`
  void take(std::map<int64_t, int64_t>::iterator it, int64_t want, std::vector<int64_t>& out) {
    const int64_t start = it->first, len = it->second;
    const int64_t k = std::min(want, len);
    for (int64_t s = start; s < start + k; ++s) {
      ref_[s] = 1;
      out.push_back(s);
    }
    runs_.erase(it);
    if (k < len) runs_.emplace(start + k, len - k);
    free_n_ -= k;
  }
  // return [start, start + len) to the free runs, merging with its neighbours
  void give(int64_t start, int64_t len) {
    free_n_ += len;
    auto next = runs_.lower_bound(start);
    if (next != runs_.begin()) {
      auto prev = std::prev(next);
      if (prev->first + prev->second == start) {
        start = prev->first;
        len += prev->second;
        runs_.erase(prev);
      }
    }
    next = runs_.lower_bound(start);
    if (next != runs_.end() && next->first == start + len) {
      len += next->second;
      runs_.erase(next);
    }
    runs_.emplace(start, len);
  }
  int64_t cap_;
  std::vector<int32_t> ref_;
  std::map<int64_t, int64_t> runs_;  // free runs: start -> length
  int64_t free_n_;
};

struct RNode {
  std::vector<int32_t> key;   // edge tokens
  std::vector<int64_t> slots; // one per token, each holding one ref in the pool
  std::map<int32_t, RNode*> children;
  RNode* parent = nullptr;
  int64_t lock = 0;
  uint64_t last_use = 0;
  uint64_t ns = 0;
  std::list<RNode*>::iterator lru_it;
  bool in_lru = false;
};

class RadixCache {
 public:
  explicit RadixCache(SlotPool* pool) : pool_(pool) {}
  ~RadixCache() {
    for (auto& kv : roots_) destroy(kv.second.get(), false);
  }

  // Longest cached prefix of `tokens` under namespace ns: (matched length, slots, node id).
  py::tuple match(uint64_t ns, py::array_t<int32_t, py::array::c_style | py::array::forcecast> tokens) {
    auto buf = tokens.unchecked<1>();
    const int64_t n = buf.shape(0);
    RNode* node = root(ns);
    std::vector<int64_t> slots;
    int64_t i = 0;
    ++clock_;
    while (i < n) {
      auto it = node->children.find(buf(i));
      if (it == node->children.end()) break;
      RNode* c = it->second;
      int64_t j = 0;
      const int64_t m = static_cast<int64_t>(c->key.size());
      while (j < m && i + j < n && c->key[j] == buf(i + j)) ++j;
      if (j < m) {
        // partial edge match: split so the matched part becomes its own node
        c = split(c, j);
      }
      slots.insert(slots.end(), c->slots.begin(), c->slots.end());
      i += static_cast<int64_t>(c->key.size());
      node = c;
      touch(node);
      if (j < m) break;
    }
    const int64_t id = register_handle(node);
    return py::make_tuple(i, slots, id);
  }

  // Insert tokens[0:n] with their slots.  Tokens already cached keep their existing
  // slots (the caller's duplicate slots are NOT referenced); the returned int is the
  // number of tokens newly inserted; new suffix slots get one extra ref (the tree's).
  int64_t insert(uint64_t ns, py::array_t<int32_t, py::array::c_style | py::array::forcecast> tokens,
                 py::array_t<int64_t, py::array::c_style | py::array::forcecast> slots) {
    auto t = tokens.unchecked<1>();
    auto s = slots.unchecked<1>();
    const int64_t n = t.shape(0);
    if (s.shape(0) != n) throw std::invalid_argument("insert: tokens and slots differ in length");
    RNode* node = root(ns);
    int64_t i = 0;
    ++clock_;
    while (i < n) {
      auto it = node->children.find(t(i));
      if (it == node->children.end()) {
        auto* c = new RNode();
        c->parent = node;
        c->ns = ns;
        c->key.assign(t.data(i), t.data(i) + (n - i));
        c->slots.assign(s.data(i), s.data(i) + (n - i));
        pool_->incref(c->slots.data(), static_cast<int64_t>(c->slots.size()));
        node->children[t(i)] = c;
        touch(c);
        cached_tokens_ += n - i;
        return n - i;
      }
      RNode* c = it->second;
      int64_t j = 0;
      const int64_t m = static_cast<int64_t>(c->key.size());
      while (j < m && i + j < n && c->key[j] == t(i + j)) ++j;
      if (j < m) c = split(c, j);
      i += static_cast<int64_t>(c->key.size());
      node = c;
      touch(node);
    }
    return 0;
  }

  void lock(int64_t handle) {
    RNode* n = handle_node(handle);
    for (; n != nullptr && n->parent != nullptr; n = n->parent) {
      if (n->lock++ == 0 && n->in_lru) {
        lru_.erase(n->lru_it);
        n->in_lru = false;
      }
    }
  }
  void unlock(int64_t handle) {
    RNode* n = handle_node(handle);
    for (; n != nullptr && n->parent != nullptr; n = n->parent) {
      if (n->lock <= 0) throw std::runtime_error("radix unlock below zero");
      if (--n->lock == 0 && n->children.empty()) push_lru(n);
    }
  }
  void release_handle(int64_t handle) { handles_.erase(handle); }

  // Evict least-recently-used unlocked leaves until `want` slots became free in the
  // pool (or nothing evictable is left).  Returns slots freed.
  int64_t evict(int64_t want) {
    int64_t freed = 0;
    while (freed < want && !lru_.empty()) {
      RNode* n = lru_.front();
      lru_.pop_front();
      n->in_lru = false;
      if (n->lock > 0 || !n->children.empty()) continue;
      freed += pool_->decref(n->slots.data(), static_cast<int64_t>(n->slots.size()));
      cached_tokens_ -= static_cast<int64_t>(n->key.size());
      RNode* p = n->parent;
      p->children.erase(n->key[0]);
      drop_handles(n);
      delete n;
      if (p->parent != nullptr && p->children.empty() && p->lock == 0) push_lru(p);
    }
    return freed;
  }

  int64_t cached_tokens() const { return cached_tokens_; }
  int64_t evictable_tokens() const {
    int64_t t = 0;
    for (auto* n : lru_) t += static_cast<int64_t>(n->key.size());
    return t;
  }

 private:
  RNode* root(uint64_t ns) {
    auto& r = roots_[ns];
    if (!r) {
      r.reset(new RNode());
      r->ns = ns;
    }
    return r.get();
  }
  RNode* split(RNode* c, int64_t j) {
    // c = [0, j) + [j, m): the head keeps the parent link, the tail becomes its child
    auto* head = new RNode();
    head->parent = c->parent;
    head->ns = c->ns;
    head->key.assign(c->key.begin(), c->key.begin() + j);
    head->slots.assign(c->slots.begin(), c->slots.begin() + j);
    head->lock = c->lock;
    head->last_use = c->last_use;
    c->parent->children[head->key[0]] = head;
    c->key.erase(c->key.begin(), c->key.begin() + j);
    c->slots.erase(c->slots.begin(), c->slots.begin() + j);
    c->parent = head;
    head->children[c->key[0]] = c;
    return head;
  }
  void touch(RNode* n) {
    n->last_use = clock_;
    if (n->in_lru) {
      lru_.erase(n->lru_it);
      n->in_lru = false;
    }
    if (n->lock == 0 && n->children.empty()) push_lru(n);
  }
  void push_lru(RNode* n) {
    if (n->in_lru) lru_.erase(n->lru_it);
    lru_.push_back(n);
    n->lru_it = std::prev(lru_.end());
    n->in_lru = true;
  }
  int64_t register_handle(RNode* n) {
    const int64_t id = next_handle_++;
    handles_[id] = n;
    return id;
  }
  RNode* handle_node(int64_t h) {
    auto it = handles_.find(h);
    if (it == handles_.end()) throw std::out_of_range("unknown radix handle");
    return it->second;
  }
  void drop_handles(RNode* n) {
    for (auto it = handles_.begin(); it != handles_.end();) {
      if (it->second == n) it = handles_.erase(it);
      else ++it;
    }
  }
  void destroy(RNode* n, bool release) {
    for (auto& kv : n->children) {
      destroy(kv.second, release);
      delete kv.second;
    }
    n->children.clear();
  }

  SlotPool* pool_;
  std::unordered_map<uint64_t, std::unique_ptr<RNode>> roots_;
  std::list<RNode*> lru_;
  std::unordered_map<int64_t, RNode*> handles_;
  int64_t next_handle_ = 1;
  uint64_t clock_ = 0;
  int64_t cached_tokens_ = 0;
};

}  // namespace octo_native

PYBIND11_MODULE(_native, m) {
  using namespace octo_native;
  m.doc() = "octopus_b200 host-side KV manager (slot pool with holder refcounts, radix prefix cache)";
  py::class_<SlotPool>(m, "SlotPool")
      .def(py::init<int64_t>())
      .def_property_readonly("capacity", &SlotPool::capacity)
      .def("free_count", &SlotPool::free_count)
      .def("used_count", &SlotPool::used_count)
      .def("alloc",
           [](SlotPool& p, int64_t n) {
             auto v = p.alloc(n);
             return py::array_t<int64_t>(static_cast<py::ssize_t>(v.size()), v.data());
           })
      .def("incref",
           [](SlotPool& p, py::array_t<int64_t, py::array::c_style | py::array::forcecast> s) {
             p.incref(s.data(), s.size());
           })
      .def("decref",
           [](SlotPool& p, py::array_t<int64_t, py::array::c_style | py::array::forcecast> s) {
             return p.decref(s.data(), s.size());
           })
      .def("refcount", &SlotPool::refcount)
      .def("check_invariants", &SlotPool::check_invariants);
  py::class_<RadixCache>(m, "RadixCache")
      .def(py::init<SlotPool*>(), py::keep_alive<1, 2>())
      .def("match", &RadixCache::match)
      .def("insert", &RadixCache::insert)
      .def("lock", &RadixCache::lock)
      .def("unlock", &RadixCache::unlock)
      .def("release_handle", &RadixCache::release_handle)
      .def("evict", &RadixCache::evict)
      .def("cached_tokens", &RadixCache::cached_tokens)
      .def("evictable_tokens", &RadixCache::evictable_tokens);
}
