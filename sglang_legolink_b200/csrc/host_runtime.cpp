// Native runtime core (CPU): KV page allocator, LegoLink block registry and a
// paged radix prefix index.  These sit on the admission path of every
// Compile / Link / decode step, so they are C++ rather than Python.
//
// Reference behaviour (re-designed here for a paged pool, not copied):
//  * block registry: patched_sglang_files/python/sglang/srt/mem_cache/radix_cache.py
//    register_legolink_block :755-929, lookup_legolink_blocks :995-1244,
//    acquire/release :1246,:1330, pin/unpin :1370,:1401, unregister :1408,
//    clear :1449, legolink_stats :732-752, capacity eviction score :1937-1965.
//  * radix prefix cache: radix_cache.py match_prefix/insert/evict :1457,:1517,:1657.
#include <pybind11/pybind11.h>
#include <pybind11/numpy.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <chrono>
#include <cstdint>
#include <list>
#include <map>
#include <memory>
#include <optional>
#include <queue>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace {

double now_s() {
  using namespace std::chrono;
  return duration<double>(steady_clock::now().time_since_epoch()).count();
}

// ------------------------------------------------------------ PageAllocator
// Fixed pool of KV pages with reference counts.  A page is free when its
// count drops to zero.  `generation` increments on reset(); a block recorded
// under an older generation is stale.
class PageAllocator {
 public:
  explicit PageAllocator(int64_t num_pages) : refs_(num_pages, 0) {
    free_.reserve(num_pages);
    for (int64_t p = num_pages - 1; p >= 0; --p) free_.push_back((int32_t)p);
  }

  int64_t num_pages() const { return (int64_t)refs_.size(); }
  int64_t num_free() const { return (int64_t)free_.size(); }
  int64_t generation() const { return generation_; }

  // Returns exactly n pages or throws (caller checks capacity first).
  std::vector<int32_t> alloc(int64_t n) {
    if (n > (int64_t)free_.size()) throw std::runtime_error("KV pool out of pages");
    std::vector<int32_t> out(n);
    for (int64_t i = 0; i < n; ++i) {
      out[i] = free_.back();
      free_.pop_back();
      refs_[out[i]] = 1;
    }
    return out;
  }

  void incref(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      check(p);
      if (refs_[p] <= 0) throw std::runtime_error("incref of a free page");
      ++refs_[p];
    }
  }

  // Decrements; pages reaching zero return to the free list.  Returns the
  // number of pages freed.
  int64_t release(const std::vector<int32_t>& pages) {
    int64_t freed = 0;
    // Pushed in reverse so that a later alloc (which pops from the back)
    // hands the run out again in ascending order: ascending page runs let
    // the attention kernels load several pages with one TMA box.
    for (auto it = pages.rbegin(); it != pages.rend(); ++it) {
      const int32_t p = *it;
      check(p);
      if (refs_[p] <= 0) throw std::runtime_error("release of a free page");
      if (--refs_[p] == 0) {
        free_.push_back(p);
        ++freed;
      }
    }
    return freed;
  }

  int32_t refcount(int32_t p) const {
    check(p);
    return refs_[p];
  }

  void reset() {
    const int64_t n = (int64_t)refs_.size();
    std::fill(refs_.begin(), refs_.end(), 0);
    free_.clear();
    for (int64_t p = n - 1; p >= 0; --p) free_.push_back((int32_t)p);
    ++generation_;
  }

 private:
  void check(int32_t p) const {
    if (p < 0 || p >= (int32_t)refs_.size()) throw std::out_of_range("page id out of range");
  }
  std::vector<int32_t> refs_;
  std::vector<int32_t> free_;
  int64_t generation_ = 0;
};

// ------------------------------------------------------------ BlockRegistry
struct BlockEntry {
  std::string cache_key;
  std::string compat_key;   // serialized LegoLinkBlockKey minus the token hash
  std::string token_hash;   // sha256 of the compact token list
  std::vector<int64_t> token_ids;
  std::vector<int32_t> pages;
  int64_t token_count = 0;
  int64_t first_page_offset = 0;  // tokens start at this offset in pages[0]
  int64_t generation = 0;
  int64_t allocator_generation = 0;
  int64_t pin_count = 0;
  int64_t active_refs = 0;
  int64_t reuse_count = 0;
  int64_t recompute_saved_tokens = 0;
  int32_t residency = 0;  // device / replica id holding the pages
  double created_at = 0;
  double last_used = 0;
  std::string block_id;
};

class BlockRegistry {
 public:
  BlockRegistry(PageAllocator* alloc, int64_t max_blocks, int32_t residency)
      : alloc_(alloc), max_blocks_(max_blocks), residency_(residency) {}

  // Registers (or keeps) a compiled block.  `pages` are handed over: the
  // registry now owns one reference to each.  Returns "registered",
  // "duplicate" (existing identical block kept; the new pages are released)
  // or throws on a key collision with different content / compatibility.
  std::string register_block(const std::string& cache_key, const std::string& compat_key,
                             const std::string& token_hash, const std::vector<int64_t>& token_ids,
                             const std::vector<int32_t>& pages, int64_t first_page_offset,
                             const std::string& block_id) {
    ++stats_["register_calls"];
    auto it = blocks_.find(cache_key);
    if (it != blocks_.end()) {
      BlockEntry& e = it->second;
      const bool stale = e.generation != generation_ || e.allocator_generation != alloc_->generation();
      if (!stale) {
        if (e.token_hash != token_hash || e.compat_key != compat_key)
          throw std::invalid_argument("LegoLink block '" + cache_key +
                                      "' is already registered with different content");
        alloc_->release(pages);
        ++stats_["duplicate_registrations"];
        touch(e);
        return "duplicate";
      }
      drop(cache_key, /*evicted=*/false);
    }
    BlockEntry e;
    e.cache_key = cache_key;
    e.compat_key = compat_key;
    e.token_hash = token_hash;
    e.token_ids = token_ids;
    e.pages = pages;
    e.token_count = (int64_t)token_ids.size();
    e.first_page_offset = first_page_offset;
    e.generation = generation_;
    e.allocator_generation = alloc_->generation();
    e.residency = residency_;
    e.created_at = e.last_used = now_s();
    e.block_id = block_id;
    blocks_.emplace(cache_key, std::move(e));
    lru_.push_back(cache_key);
    ++stats_["registered"];
    while (max_blocks_ > 0 && (int64_t)blocks_.size() > max_blocks_) {
      if (!evict_one()) break;
    }
    return "registered";
  }

  // Classifies each key: found / missing / stale / incompatible.
  py::dict lookup(const std::vector<std::string>& keys, const std::string& compat_key) {
    ++stats_["lookups"];
    py::list found, missing, stale, incompatible;
    for (const auto& k : keys) {
      auto it = blocks_.find(k);
      if (it == blocks_.end()) {
        missing.append(k);
        ++stats_["misses"];
        continue;
      }
      BlockEntry& e = it->second;
      if (e.generation != generation_ || e.allocator_generation != alloc_->generation()) {
        stale.append(k);
        ++stats_["stale"];
        continue;
      }
      if (!compat_key.empty() && e.compat_key != compat_key) {
        incompatible.append(k);
        ++stats_["incompatible"];
        continue;
      }
      found.append(k);
      ++stats_["hits"];
    }
    py::dict d;
    d["found"] = found;
    d["missing"] = missing;
    d["stale"] = stale;
    d["incompatible"] = incompatible;
    d["ok"] = py::bool_(py::len(missing) == 0 && py::len(stale) == 0 && py::len(incompatible) == 0);
    return d;
  }

  void acquire(const std::vector<std::string>& keys) {
    for (const auto& k : keys) {
      BlockEntry& e = get(k);
      ++e.active_refs;
      touch(e);
    }
    ++stats_["acquires"];
  }

  void release(const std::vector<std::string>& keys) {
    for (const auto& k : keys) {
      auto it = blocks_.find(k);
      if (it == blocks_.end()) continue;  // unregistered while linked: nothing to release
      if (it->second.active_refs <= 0) throw std::runtime_error("release without acquire: " + k);
      --it->second.active_refs;
    }
    ++stats_["releases"];
  }

  void pin(const std::vector<std::string>& keys) {
    for (const auto& k : keys) ++get(k).pin_count;
    ++stats_["pins"];
  }

  void unpin(const std::vector<std::string>& keys) {
    for (const auto& k : keys) {
      auto it = blocks_.find(k);
      if (it == blocks_.end()) continue;
      if (it->second.pin_count <= 0) throw std::runtime_error("unpin without pin: " + k);
      --it->second.pin_count;
    }
  }

  void record_execution(const std::string& k, int64_t reused_tokens, int64_t recompute_tokens) {
    auto it = blocks_.find(k);
    if (it == blocks_.end()) return;
    ++it->second.reuse_count;
    it->second.recompute_saved_tokens += std::max<int64_t>(0, reused_tokens - recompute_tokens);
    stats_["reused_tokens"] += reused_tokens;
  }

  bool unregister(const std::string& k) {
    auto it = blocks_.find(k);
    if (it == blocks_.end()) return false;
    if (it->second.active_refs > 0 || it->second.pin_count > 0)
      throw std::runtime_error("cannot unregister a pinned or linked block: " + k);
    drop(k, false);
    return true;
  }

  // Invalidates every block (generation bump) and frees unreferenced pages.
  void clear() {
    ++generation_;
    std::vector<std::string> keys;
    for (auto& kv : blocks_)
      if (kv.second.active_refs == 0 && kv.second.pin_count == 0) keys.push_back(kv.first);
    for (auto& k : keys) drop(k, false);
  }

  // Pages that capacity eviction could free right now.
  int64_t capacity_evictable_pages() const {
    int64_t n = 0;
    for (const auto& kv : blocks_) {
      const BlockEntry& e = kv.second;
      if (e.active_refs == 0 && e.pin_count == 0) n += owned_pages(e);
    }
    return n;
  }

  // Frees blocks (lowest score first) until `pages_needed` pages are free in
  // the allocator or nothing evictable is left.  Returns pages freed.
  int64_t evict_for_capacity(int64_t pages_needed) {
    int64_t freed = 0;
    while (alloc_->num_free() < pages_needed) {
      const std::string* victim = nullptr;
      double best = 0;
      const double t = now_s();
      for (const auto& kv : blocks_) {
        const BlockEntry& e = kv.second;
        if (e.active_refs > 0 || e.pin_count > 0) continue;
        const double s = score(e, t);
        if (victim == nullptr || s < best) {
          victim = &kv.first;
          best = s;
        }
      }
      if (victim == nullptr) break;
      const std::string k = *victim;
      const int64_t before = alloc_->num_free();
      drop(k, true);
      freed += alloc_->num_free() - before;
    }
    return freed;
  }

  // Unreferenced blocks with at most `max_pins` pins, lowest keep-value
  // first, as (cache_key, owned pages).  A DP owner walks this list for
  // published blocks (pinned once by publication) it may withdraw.
  std::vector<std::pair<std::string, int64_t>> eviction_candidates(int64_t max_pins) const {
    std::vector<std::pair<double, const BlockEntry*>> v;
    const double t = now_s();
    for (const auto& kv : blocks_) {
      const BlockEntry& e = kv.second;
      if (e.active_refs > 0 || e.pin_count > max_pins) continue;
      v.emplace_back(score(e, t), &e);
    }
    std::sort(v.begin(), v.end(), [](const auto& a, const auto& b) {
      return a.first < b.first || (a.first == b.first && a.second->cache_key < b.second->cache_key);
    });
    std::vector<std::pair<std::string, int64_t>> out;
    out.reserve(v.size());
    for (const auto& p : v) out.emplace_back(p.second->cache_key, owned_pages(*p.second));
    return out;
  }

  // Keep-value of a block: (reuse x recomputation saved) / (residency x (age+1)).
  static double score(const BlockEntry& e, double t) {
    const double reuse = 1.0 + (double)e.reuse_count;
    const double saved = 1.0 + (double)e.recompute_saved_tokens + (double)e.token_count;
    const double resid = std::max<double>(1.0, (double)e.pages.size());
    const double age = std::max(0.0, t - e.last_used);
    return (reuse * saved) / (resid * (age + 1.0));
  }

  py::dict handle(const std::string& k) {
    const BlockEntry& e = get(k);
    py::dict d;
    d["cache_key"] = e.cache_key;
    d["compat_key"] = e.compat_key;
    d["token_hash"] = e.token_hash;
    d["token_count"] = e.token_count;
    d["pages"] = e.pages;
    d["first_page_offset"] = e.first_page_offset;
    d["generation"] = e.generation;
    d["allocator_generation"] = e.allocator_generation;
    d["pin_count"] = e.pin_count;
    d["active_refs"] = e.active_refs;
    d["reuse_count"] = e.reuse_count;
    d["residency"] = e.residency;
    d["block_id"] = e.block_id;
    d["stale"] = py::bool_(e.generation != generation_ || e.allocator_generation != alloc_->generation());
    return d;
  }

  std::optional<std::vector<int64_t>> tokens(const std::string& k) const {
    auto it = blocks_.find(k);
    if (it == blocks_.end()) return std::nullopt;
    return it->second.token_ids;
  }

  // Content hash of a registered block (None when absent): equal hashes mean
  // equal token ids, so a caller may keep a converted copy keyed by it.
  std::optional<std::string> token_hash(const std::string& k) const {
    auto it = blocks_.find(k);
    if (it == blocks_.end()) return std::nullopt;
    return it->second.token_hash;
  }

  bool contains(const std::string& k) const { return blocks_.count(k) != 0; }
  int64_t size() const { return (int64_t)blocks_.size(); }
  int64_t generation() const { return generation_; }
  std::vector<std::string> keys() const {
    std::vector<std::string> out;
    for (auto& kv : blocks_) out.push_back(kv.first);
    return out;
  }

  py::dict stats() const {
    py::dict d;
    for (auto& kv : stats_) d[py::str(kv.first)] = kv.second;
    d["blocks"] = (int64_t)blocks_.size();
    int64_t pinned = 0, linked = 0, tokens = 0;
    for (auto& kv : blocks_) {
      pinned += kv.second.pin_count > 0;
      linked += kv.second.active_refs > 0;
      tokens += kv.second.token_count;
    }
    d["pinned_blocks"] = pinned;
    d["linked_blocks"] = linked;
    d["resident_tokens"] = tokens;
    d["generation"] = generation_;
    return d;
  }

 private:
  static int64_t owned_pages(const BlockEntry& e) { return (int64_t)e.pages.size(); }

  BlockEntry& get(const std::string& k) {
    auto it = blocks_.find(k);
    if (it == blocks_.end()) throw std::out_of_range("LegoLink block is not registered: " + k);
    return it->second;
  }

  void touch(BlockEntry& e) {
    e.last_used = now_s();
    lru_.remove(e.cache_key);
    lru_.push_back(e.cache_key);
  }

  bool evict_one() {
    for (auto it = lru_.begin(); it != lru_.end(); ++it) {
      auto b = blocks_.find(*it);
      if (b != blocks_.end() && b->second.active_refs == 0 && b->second.pin_count == 0) {
        drop(*it, true);
        return true;
      }
    }
    return false;
  }

  void drop(const std::string& k, bool evicted) {
    auto it = blocks_.find(k);
    if (it == blocks_.end()) return;
    const bool stale_alloc = it->second.allocator_generation != alloc_->generation();
    if (!stale_alloc) alloc_->release(it->second.pages);
    if (evicted) {
      ++stats_["evicted_blocks"];
      stats_["evicted_tokens"] += it->second.token_count;
    }
    blocks_.erase(it);
    lru_.remove(k);
  }

  PageAllocator* alloc_;
  int64_t max_blocks_;
  int32_t residency_;
  int64_t generation_ = 0;
  std::unordered_map<std::string, BlockEntry> blocks_;
  std::list<std::string> lru_;
  std::map<std::string, int64_t> stats_;
};

// ------------------------------------------------------------ RadixIndex
// Prefix index at page granularity: an edge holds exactly one full page of
// tokens.  Roots are per namespace (extra_key), so requests under different
// namespaces never share KV.  Leaves with no lock are evicted LRU-first.
class RadixIndex {
  struct Node {
    std::vector<int64_t> tokens;  // page_size tokens
    int32_t page = -1;
    Node* parent = nullptr;
    std::map<std::vector<int64_t>, std::unique_ptr<Node>> children;
    int64_t lock = 0;
    double last_used = 0;
  };

 public:
  RadixIndex(PageAllocator* alloc, int64_t page_size) : alloc_(alloc), ps_(page_size) {}

  // Longest cached prefix of `tokens` (whole pages only).  Returns its pages;
  // the caller must incref them if it keeps them.
  std::vector<int32_t> match_prefix(const std::string& ns, const std::vector<int64_t>& tokens) {
    std::vector<int32_t> pages;
    Node* n = root(ns);
    const double t = now_s();
    for (size_t off = 0; off + ps_ <= tokens.size(); off += ps_) {
      std::vector<int64_t> key(tokens.begin() + off, tokens.begin() + off + ps_);
      auto it = n->children.find(key);
      if (it == n->children.end()) break;
      n = it->second.get();
      n->last_used = t;
      pages.push_back(n->page);
    }
    return pages;
  }

  // Inserts the full pages of `tokens`.  Each newly indexed page gets one
  // allocator reference held by the index.  Returns the number inserted.
  int64_t insert(const std::string& ns, const std::vector<int64_t>& tokens, const std::vector<int32_t>& pages) {
    Node* n = root(ns);
    int64_t added = 0;
    const double t = now_s();
    for (size_t i = 0; (i + 1) * ps_ <= tokens.size() && i < pages.size(); ++i) {
      std::vector<int64_t> key(tokens.begin() + i * ps_, tokens.begin() + (i + 1) * ps_);
      auto it = n->children.find(key);
      if (it == n->children.end()) {
        auto child = std::make_unique<Node>();
        child->tokens = key;
        child->page = pages[i];
        child->parent = n;
        child->last_used = t;
        alloc_->incref({pages[i]});
        Node* c = child.get();
        n->children.emplace(key, std::move(child));
        n = c;
        ++added;
        ++indexed_pages_;
      } else {
        n = it->second.get();
        n->last_used = t;
      }
    }
    return added;
  }

  // Frees up to `num_pages` pages held only by the index (LRU leaves first).
  int64_t evict(int64_t num_pages) {
    int64_t freed = 0;
    while (freed < num_pages) {
      Node* victim = nullptr;
      for (auto& kv : roots_) find_lru_leaf(kv.second.get(), &victim);
      if (victim == nullptr) break;
      const int32_t p = victim->page;
      Node* parent = victim->parent;
      const bool only_ref = alloc_->refcount(p) == 1;
      alloc_->release({p});
      --indexed_pages_;
      if (only_ref) ++freed;
      parent->children.erase(victim->tokens);
    }
    return freed;
  }

  int64_t evictable_pages() const {
    int64_t n = 0;
    for (auto& kv : roots_) n += count_sole(kv.second.get());
    return n;
  }

  int64_t indexed_pages() const { return indexed_pages_; }

  void reset() {
    roots_.clear();
    indexed_pages_ = 0;
  }

 private:
  Node* root(const std::string& ns) {
    auto it = roots_.find(ns);
    if (it == roots_.end()) it = roots_.emplace(ns, std::make_unique<Node>()).first;
    return it->second.get();
  }

  void find_lru_leaf(Node* n, Node** best) {
    for (auto& kv : n->children) {
      Node* c = kv.second.get();
      if (c->children.empty()) {
        if (c->lock == 0 && (*best == nullptr || c->last_used < (*best)->last_used)) *best = c;
      } else {
        find_lru_leaf(c, best);
      }
    }
  }

  int64_t count_sole(Node* n) const {
    int64_t c = 0;
    for (auto& kv : n->children) {
      Node* ch = kv.second.get();
      if (ch->page >= 0 && alloc_->refcount(ch->page) == 1) ++c;
      c += count_sole(ch);
    }
    return c;
  }

  PageAllocator* alloc_;
  int64_t ps_;
  std::map<std::string, std::unique_ptr<Node>> roots_;
  int64_t indexed_pages_ = 0;
};

// Makespan of list scheduling: items taken in the given order, each onto the
// worker that becomes free first.  With one CTA per SM this is how the
// GPU's block scheduler places the CTAs of one launch, so it models a
// kernel's duration from its per-CTA work (the prefill attention's split
// choice).
double list_schedule_makespan(py::array_t<double, py::array::c_style | py::array::forcecast> items, int workers) {
  if (workers <= 0) throw std::invalid_argument("workers must be positive");
  auto it = items.unchecked<1>();
  std::priority_queue<double, std::vector<double>, std::greater<double>> free_at;
  for (int i = 0; i < workers; ++i) free_at.push(0.0);
  double end = 0.0;
  for (py::ssize_t i = 0; i < it.shape(0); ++i) {
    const double w = it(i);
    const double t = free_at.top() + w;
    free_at.pop();
    free_at.push(t);
    end = std::max(end, t);
  }
  return end;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "LegoLink B200 runtime core: page allocator, block registry, radix prefix index";
  m.def("list_schedule_makespan", &list_schedule_makespan, py::arg("items"), py::arg("workers"));
  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int64_t>())
      .def_property_readonly("num_pages", &PageAllocator::num_pages)
      .def_property_readonly("num_free", &PageAllocator::num_free)
      .def_property_readonly("generation", &PageAllocator::generation)
      .def("alloc", &PageAllocator::alloc)
      .def("incref", &PageAllocator::incref)
      .def("release", &PageAllocator::release)
      .def("refcount", &PageAllocator::refcount)
      .def("reset", &PageAllocator::reset);
  py::class_<BlockRegistry>(m, "BlockRegistry")
      .def(py::init<PageAllocator*, int64_t, int32_t>(), py::keep_alive<1, 2>())
      .def("register_block", &BlockRegistry::register_block)
      .def("lookup", &BlockRegistry::lookup)
      .def("acquire", &BlockRegistry::acquire)
      .def("release", &BlockRegistry::release)
      .def("pin", &BlockRegistry::pin)
      .def("unpin", &BlockRegistry::unpin)
      .def("record_execution", &BlockRegistry::record_execution)
      .def("unregister", &BlockRegistry::unregister)
      .def("clear", &BlockRegistry::clear)
      .def("capacity_evictable_pages", &BlockRegistry::capacity_evictable_pages)
      .def("evict_for_capacity", &BlockRegistry::evict_for_capacity)
      .def("eviction_candidates", &BlockRegistry::eviction_candidates)
      .def("handle", &BlockRegistry::handle)
      .def("tokens", &BlockRegistry::tokens)
      .def("token_hash", &BlockRegistry::token_hash)
      .def("contains", &BlockRegistry::contains)
      .def("keys", &BlockRegistry::keys)
      .def("stats", &BlockRegistry::stats)
      .def_property_readonly("size", &BlockRegistry::size)
      .def_property_readonly("generation", &BlockRegistry::generation);
  py::class_<RadixIndex>(m, "RadixIndex")
      .def(py::init<PageAllocator*, int64_t>(), py::keep_alive<1, 2>())
      .def("match_prefix", &RadixIndex::match_prefix)
      .def("insert", &RadixIndex::insert)
      .def("evict", &RadixIndex::evict)
      .def("evictable_pages", &RadixIndex::evictable_pages)
      .def_property_readonly("indexed_pages", &RadixIndex::indexed_pages)
      .def("reset", &RadixIndex::reset);
}
