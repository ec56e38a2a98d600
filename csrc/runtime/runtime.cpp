// Native host runtime of sglang_neuron_b200 (module sglang_neuron_b200._runtime).
//
//  * PageAllocator: the paged KV-pool allocator. Frees can be staged behind a launch epoch and are only
//    returned to the free list once that epoch has retired, so a page that an in-flight step still reads
//    is never handed out again. Parity: NeuronPagedTokenToKVPoolAllocator and its staged frees
//    (sglang_neuron/mem_cache/allocator.py:172; docs/design/runtime.md:1252-1293 "held until the launches
//    that read them retire").
//  * RadixCache: a page-granular prefix tree (keys are token ids, one edge chunk per page) with
//    reference counts and LRU eviction of unreferenced leaves. Parity: SGLang's radix tree as the
//    reference drives it (ChunkKeyedRadixCache, sglang_neuron/mem_cache/chunk_keyed_tree.py:58, with the
//    page as its chunk so hits are bit-identical).
//  * build_page_table_rows: fills padded int32 block-table rows and slot mappings for a batch in one call.
//  * ShmReduce: element-wise MIN / MAX of a short int64 vector over the ranks of one node through a POSIX
//    shared-memory segment (no sockets, no pickling). Parity: the reference's NodeShmMin
//    (sglang_neuron/distributed/node_shm_min.py:68; docs/design/parallelism.md:940-989: spin, then short
//    naps, and a timeout), which backs its poll reduces.
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <atomic>
#include <cstring>
#include <chrono>
#include <string>
#include <thread>

#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <deque>
#include <list>
#include <map>
#include <memory>
#include <stdexcept>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

class PageAllocator {
 public:
  PageAllocator(int64_t num_pages, int64_t page_size, int64_t reserved)
      : num_pages_(num_pages), page_size_(page_size) {
    if (reserved < 0 || reserved >= num_pages) throw std::invalid_argument("bad reserved page count");
    free_.reserve(num_pages);
    for (int64_t p = num_pages - 1; p >= reserved; --p) free_.push_back((int32_t)p);
    reserved_ = reserved;
  }

  int64_t available() const { return (int64_t)free_.size(); }
  int64_t staged() const {
    int64_t n = 0;
    for (auto& kv : staged_) n += (int64_t)kv.second.size();
    return n;
  }
  int64_t num_pages() const { return num_pages_; }
  int64_t page_size() const { return page_size_; }

  // Returns n page ids, or an empty vector when fewer than n are free (nothing is taken then).
  std::vector<int32_t> alloc(int64_t n) {
    std::vector<int32_t> out;
    if (n <= 0) return out;
    if ((int64_t)free_.size() < n) return out;
    out.reserve(n);
    for (int64_t i = 0; i < n; ++i) {
      out.push_back(free_.back());
      free_.pop_back();
    }
    return out;
  }

  void free(const std::vector<int32_t>& pages) {
    for (int32_t p : pages) {
      if (p < reserved_ || p >= num_pages_) throw std::out_of_range("freeing an invalid page id");
      free_.push_back(p);
    }
  }

  // Stage frees until launch `epoch` retires.
  void free_after(const std::vector<int32_t>& pages, int64_t epoch) {
    auto& v = staged_[epoch];
    v.insert(v.end(), pages.begin(), pages.end());
  }

  // Every launch with epoch <= retired_epoch has completed on the device.
  int64_t retire(int64_t retired_epoch) {
    int64_t n = 0;
    while (!staged_.empty() && staged_.begin()->first <= retired_epoch) {
      auto& v = staged_.begin()->second;
      n += (int64_t)v.size();
      free(v);
      staged_.erase(staged_.begin());
    }
    return n;
  }

  void reset() {
    free_.clear();
    staged_.clear();
    for (int64_t p = num_pages_ - 1; p >= reserved_; --p) free_.push_back((int32_t)p);
  }

 private:
  int64_t num_pages_, page_size_, reserved_ = 1;
  std::vector<int32_t> free_;
  std::map<int64_t, std::vector<int32_t>> staged_;
};

// ---------------------------------------------------------------------------------------------------
// Radix prefix cache over pages.
// ---------------------------------------------------------------------------------------------------
struct RadixNode {
  std::vector<int32_t> key;    // tokens, a multiple of page_size
  std::vector<int32_t> pages;  // key.size() / page_size pages
  RadixNode* parent = nullptr;
  std::unordered_map<int64_t, std::unique_ptr<RadixNode>> children;  // keyed by a hash of the first page
  int64_t lock_ref = 0;
  uint64_t last_access = 0;
};

class RadixCache {
 public:
  explicit RadixCache(int64_t page_size) : page_size_(page_size), root_(new RadixNode()) {
    root_->lock_ref = 1;
  }

  int64_t page_size() const { return page_size_; }
  int64_t cached_pages() const { return cached_pages_; }
  int64_t evictable_pages() const { return evictable_pages_; }

  // Longest cached prefix of `tokens` in whole pages. Returns (matched_tokens, pages, node handle).
  py::tuple match_prefix(const std::vector<int32_t>& tokens) {
    std::vector<int32_t> pages;
    RadixNode* node = root_.get();
    size_t pos = 0;
    ++clock_;
    node->last_access = clock_;
    while (pos + page_size_ <= tokens.size()) {
      auto it = node->children.find(page_hash(tokens.data() + pos));
      if (it == node->children.end()) break;
      RadixNode* child = it->second.get();
      // compare page by page along the child's key
      size_t n = 0;
      const size_t klen = child->key.size();
      while (n < klen && pos + n + page_size_ <= tokens.size() &&
             std::equal(child->key.begin() + n, child->key.begin() + n + page_size_, tokens.begin() + pos + n)) {
        n += page_size_;
      }
      if (n == 0) break;
      if (n < klen) {
        child = split(child, n);
      }
      child->last_access = clock_;
      pages.insert(pages.end(), child->pages.begin(), child->pages.end());
      pos += n;
      node = child;
      if (n < klen) break;
    }
    return py::make_tuple((int64_t)pos, pages, reinterpret_cast<uintptr_t>(node));
  }

  // Insert a page-aligned prefix. Pages already present are returned in `duplicates` (the caller frees
  // them); the tree keeps its own copy.
  std::vector<int32_t> insert(const std::vector<int32_t>& tokens, const std::vector<int32_t>& pages) {
    std::vector<int32_t> duplicates;
    const size_t n_tok = (tokens.size() / page_size_) * page_size_;
    if (pages.size() * page_size_ < n_tok) throw std::invalid_argument("insert: not enough pages for tokens");
    RadixNode* node = root_.get();
    size_t pos = 0;
    ++clock_;
    while (pos < n_tok) {
      const int64_t h = page_hash(tokens.data() + pos);
      auto it = node->children.find(h);
      if (it == node->children.end()) {
        auto child = std::make_unique<RadixNode>();
        child->key.assign(tokens.begin() + pos, tokens.begin() + n_tok);
        child->pages.assign(pages.begin() + pos / page_size_, pages.begin() + n_tok / page_size_);
        child->parent = node;
        child->last_access = clock_;
        const int64_t np = (int64_t)child->pages.size();
        cached_pages_ += np;
        evictable_pages_ += np;
        if (node != root_.get() && node->children.empty() && node->lock_ref == 0) {
          // node stops being a leaf: its pages stay evictable through the subtree
        }
        node->children[h] = std::move(child);
        return duplicates;
      }
      RadixNode* child = it->second.get();
      size_t n = 0;
      const size_t klen = child->key.size();
      while (n < klen && pos + n < n_tok &&
             std::equal(child->key.begin() + n, child->key.begin() + n + page_size_, tokens.begin() + pos + n)) {
        n += page_size_;
      }
      if (n == 0) {
        // hash collision on a different first page: treat as a miss below this node
        return duplicates;
      }
      if (n < klen) child = split(child, n);
      for (size_t i = 0; i < n / page_size_; ++i) {
        const int32_t mine = pages[pos / page_size_ + i];
        if (mine != child->pages[i]) duplicates.push_back(mine);
      }
      child->last_access = clock_;
      pos += n;
      node = child;
    }
    return duplicates;
  }

  // Reference counting along the path from a node to the root (a running request pins its prefix).
  void inc_lock(uintptr_t handle) {
    for (RadixNode* n = reinterpret_cast<RadixNode*>(handle); n != nullptr && n != root_.get(); n = n->parent) {
      if (n->lock_ref == 0) evictable_pages_ -= (int64_t)n->pages.size();
      ++n->lock_ref;
    }
  }
  void dec_lock(uintptr_t handle) {
    for (RadixNode* n = reinterpret_cast<RadixNode*>(handle); n != nullptr && n != root_.get(); n = n->parent) {
      if (n->lock_ref <= 0) throw std::runtime_error("radix dec_lock below zero");
      --n->lock_ref;
      if (n->lock_ref == 0) evictable_pages_ += (int64_t)n->pages.size();
    }
  }

  // Evict least-recently-used unlocked leaves until `num_pages` pages are released; returns them.
  std::vector<int32_t> evict(int64_t num_pages) {
    std::vector<int32_t> freed;
    while ((int64_t)freed.size() < num_pages) {
      RadixNode* victim = nullptr;
      find_lru_leaf(root_.get(), victim);
      if (victim == nullptr) break;
      freed.insert(freed.end(), victim->pages.begin(), victim->pages.end());
      cached_pages_ -= (int64_t)victim->pages.size();
      evictable_pages_ -= (int64_t)victim->pages.size();
      RadixNode* parent = victim->parent;
      for (auto it = parent->children.begin(); it != parent->children.end(); ++it) {
        if (it->second.get() == victim) {
          parent->children.erase(it);
          break;
        }
      }
    }
    return freed;
  }

  std::vector<int32_t> reset() {
    std::vector<int32_t> all;
    collect(root_.get(), all);
    root_ = std::make_unique<RadixNode>();
    root_->lock_ref = 1;
    cached_pages_ = evictable_pages_ = 0;
    return all;
  }

 private:
  int64_t page_hash(const int32_t* t) const {
    uint64_t h = 1469598103934665603ull;
    for (int64_t i = 0; i < page_size_; ++i) {
      h ^= (uint64_t)(uint32_t)t[i];
      h *= 1099511628211ull;
    }
    return (int64_t)h;
  }

  RadixNode* split(RadixNode* child, size_t n) {
    // child -> [new_node (first n tokens)] -> child (rest)
    RadixNode* parent = child->parent;
    const int64_t h = page_hash(child->key.data());
    auto owned = std::move(parent->children[h]);
    auto mid = std::make_unique<RadixNode>();
    mid->key.assign(child->key.begin(), child->key.begin() + n);
    mid->pages.assign(child->pages.begin(), child->pages.begin() + n / page_size_);
    mid->parent = parent;
    mid->lock_ref = child->lock_ref;
    mid->last_access = child->last_access;
    child->key.erase(child->key.begin(), child->key.begin() + n);
    child->pages.erase(child->pages.begin(), child->pages.begin() + n / page_size_);
    child->parent = mid.get();
    RadixNode* mid_raw = mid.get();
    mid->children[page_hash(child->key.data())] = std::move(owned);
    parent->children[h] = std::move(mid);
    return mid_raw;
  }

  void find_lru_leaf(RadixNode* n, RadixNode*& best) {
    if (n != root_.get() && n->children.empty() && n->lock_ref == 0) {
      if (best == nullptr || n->last_access < best->last_access) best = n;
    }
    for (auto& kv : n->children) find_lru_leaf(kv.second.get(), best);
  }

  void collect(RadixNode* n, std::vector<int32_t>& out) {
    out.insert(out.end(), n->pages.begin(), n->pages.end());
    for (auto& kv : n->children) collect(kv.second.get(), out);
  }

  int64_t page_size_;
  std::unique_ptr<RadixNode> root_;
  uint64_t clock_ = 0;
  int64_t cached_pages_ = 0, evictable_pages_ = 0;
};

// Fill block-table rows [B, max_pages] (padded with `pad`) from per-request page lists.
void build_page_table_rows(py::array_t<int32_t> table, const std::vector<std::vector<int32_t>>& pages,
                           int32_t pad) {
  auto t = table.mutable_unchecked<2>();
  const int64_t B = t.shape(0), W = t.shape(1);
  if ((int64_t)pages.size() > B) throw std::invalid_argument("more requests than table rows");
  for (int64_t b = 0; b < B; ++b) {
    int64_t j = 0;
    if (b < (int64_t)pages.size()) {
      const auto& pl = pages[b];
      if ((int64_t)pl.size() > W) throw std::invalid_argument("page list longer than the table width");
      for (; j < (int64_t)pl.size(); ++j) t(b, j) = pl[j];
    }
    for (; j < W; ++j) t(b, j) = pad;
  }
}

// Slots (page * page_size + offset) for token positions [start, end) of a request.
std::vector<int64_t> slots_for_range(const std::vector<int32_t>& pages, int64_t page_size, int64_t start,
                                     int64_t end) {
  std::vector<int64_t> out;
  out.reserve(end > start ? end - start : 0);
  for (int64_t p = start; p < end; ++p) {
    const int64_t idx = p / page_size;
    if (idx >= (int64_t)pages.size()) throw std::out_of_range("position beyond allocated pages");
    out.push_back((int64_t)pages[idx] * page_size + p % page_size);
  }
  return out;
}

// Segment: per rank one 64-byte-aligned slot {atomic<uint64> epoch; int64 vals[2][width]}. Call e writes
// buffer (e & 1) of its own slot, publishes epoch e (release), waits until every slot shows >= e (acquire),
// and reduces buffer (e & 1) of all slots. Two buffers suffice: a rank can only start call e + 2 after every
// rank published e + 1, i.e. after every rank finished reading call e.
class ShmReduce {
 public:
  ShmReduce(const std::string& name, int64_t world, int64_t rank, int64_t width, bool create)
      : name_(name), world_(world), rank_(rank), width_(width) {
    if (world < 1 || rank < 0 || rank >= world || width < 1 || width > 4096)
      throw std::invalid_argument("ShmReduce: bad world / rank / width");
    slot_bytes_ = ((sizeof(uint64_t) + 2 * width * sizeof(int64_t)) + 63) / 64 * 64;
    bytes_ = slot_bytes_ * world;
    int fd = shm_open(name.c_str(), create ? (O_CREAT | O_RDWR) : O_RDWR, 0600);
    if (fd < 0) throw std::runtime_error("ShmReduce: shm_open failed for " + name);
    if (create && ftruncate(fd, (off_t)bytes_) != 0) {
      close(fd);
      throw std::runtime_error("ShmReduce: ftruncate failed");
    }
    void* p = mmap(nullptr, bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (p == MAP_FAILED) throw std::runtime_error("ShmReduce: mmap failed");
    base_ = static_cast<uint8_t*>(p);
    if (create) std::memset(base_, 0, bytes_);
    owner_ = create;
  }
  ~ShmReduce() {
    if (base_) munmap(base_, bytes_);
    if (owner_) shm_unlink(name_.c_str());
  }
  std::vector<int64_t> reduce(const std::vector<int64_t>& v, bool is_min, double timeout_s) {
    if ((int64_t)v.size() != width_) throw std::invalid_argument("ShmReduce: vector width");
    const uint64_t e = ++epoch_;
    const int buf = (int)(e & 1);
    int64_t* mine = vals(rank_, buf);
    for (int64_t i = 0; i < width_; ++i) mine[i] = v[i];
    epoch_of(rank_)->store(e, std::memory_order_release);
    const auto t0 = std::chrono::steady_clock::now();
    std::vector<int64_t> out(v);
    for (int64_t q = 0; q < world_; ++q) {
      if (q == rank_) continue;
      int spins = 0;
      long nap_ns = 20000;
      while (epoch_of(q)->load(std::memory_order_acquire) < e) {
        if (++spins < 64) continue;
        struct timespec ts{0, nap_ns};  // naps after the first polls: 20 us, doubling up to 1 ms
        nanosleep(&ts, nullptr);
        nap_ns = std::min(nap_ns * 2, 1000000L);
        const double dt = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
        if (dt > timeout_s)
          throw std::runtime_error("ShmReduce: rank " + std::to_string(q) + " did not arrive within the timeout");
      }
      const int64_t* other = vals(q, buf);
      for (int64_t i = 0; i < width_; ++i) out[i] = is_min ? std::min(out[i], other[i]) : std::max(out[i], other[i]);
    }
    return out;
  }
  int64_t world() const { return world_; }

 private:
  std::atomic<uint64_t>* epoch_of(int64_t r) { return reinterpret_cast<std::atomic<uint64_t>*>(base_ + r * slot_bytes_); }
  int64_t* vals(int64_t r, int buf) {
    return reinterpret_cast<int64_t*>(base_ + r * slot_bytes_ + sizeof(uint64_t)) + buf * width_;
  }
  std::string name_;
  int64_t world_, rank_, width_;
  size_t slot_bytes_ = 0, bytes_ = 0;
  uint8_t* base_ = nullptr;
  bool owner_ = false;
  uint64_t epoch_ = 0;
};

PYBIND11_MODULE(_runtime, m) {
  m.doc() = "sglang_neuron_b200 native host runtime";
  py::class_<PageAllocator>(m, "PageAllocator")
      .def(py::init<int64_t, int64_t, int64_t>(), py::arg("num_pages"), py::arg("page_size"), py::arg("reserved") = 1)
      .def("available", &PageAllocator::available)
      .def("staged", &PageAllocator::staged)
      .def("num_pages", &PageAllocator::num_pages)
      .def("page_size", &PageAllocator::page_size)
      .def("alloc", &PageAllocator::alloc, py::arg("n"))
      .def("free", &PageAllocator::free, py::arg("pages"))
      .def("free_after", &PageAllocator::free_after, py::arg("pages"), py::arg("epoch"))
      .def("retire", &PageAllocator::retire, py::arg("epoch"))
      .def("reset", &PageAllocator::reset);
  py::class_<RadixCache>(m, "RadixCache")
      .def(py::init<int64_t>())
      .def("page_size", &RadixCache::page_size)
      .def("cached_pages", &RadixCache::cached_pages)
      .def("evictable_pages", &RadixCache::evictable_pages)
      .def("match_prefix", &RadixCache::match_prefix, py::arg("tokens"))
      .def("insert", &RadixCache::insert, py::arg("tokens"), py::arg("pages"))
      .def("inc_lock", &RadixCache::inc_lock, py::arg("node"))
      .def("dec_lock", &RadixCache::dec_lock, py::arg("node"))
      .def("evict", &RadixCache::evict, py::arg("num_pages"))
      .def("reset", &RadixCache::reset);
  m.def("build_page_table_rows", &build_page_table_rows);
  m.def("slots_for_range", &slots_for_range);
  py::class_<ShmReduce>(m, "ShmReduce")
      .def(py::init<const std::string&, int64_t, int64_t, int64_t, bool>(), py::arg("name"), py::arg("world"),
           py::arg("rank"), py::arg("width"), py::arg("create"))
      .def("min", [](ShmReduce& s, const std::vector<int64_t>& v, double t) { return s.reduce(v, true, t); },
           py::arg("values"), py::arg("timeout_s") = 60.0, py::call_guard<py::gil_scoped_release>())
      .def("max", [](ShmReduce& s, const std::vector<int64_t>& v, double t) { return s.reduce(v, false, t); },
           py::arg("values"), py::arg("timeout_s") = 60.0, py::call_guard<py::gil_scoped_release>())
      .def("world", &ShmReduce::world);
}
