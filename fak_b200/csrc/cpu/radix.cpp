// Native page pool and radix-tree prefix cache of the KV engine.
//
// Same interface and semantics as fak_b200/kv/radix.py (its executable specification): pages are
// refcounted, the tree matches and stores whole pages, a page a live sequence holds has refcount
// >= 2 and is never evicted, eviction drops least-recently-used unlocked leaves.  Recency is a
// logical clock bumped by every operation.  Reference: PagedKVPool (internal/model/pagedkv.go:44-124)
// and radixkv.Tree (internal/radixkv/radixkv.go: Lookup :189, Insert :211, split :149, evictToBudget :252).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <memory>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace {

struct OutOfPagesError : std::runtime_error {
  using std::runtime_error::runtime_error;
};

class PagePool {
 public:
  PagePool(int n_pages, int reserve) : n_pages_(n_pages), reserve_(reserve), ref_(n_pages, 0) {
    if (reserve < 0 || reserve > n_pages) throw std::invalid_argument("PagePool: bad reserve");
    for (int p = n_pages - 1; p >= reserve; p--) free_.push_back(p);
  }
  int n_free() const { return (int)free_.size(); }
  int n_pages() const { return n_pages_; }
  int reserve() const { return reserve_; }
  std::vector<int> alloc(int n) {
    if (n > (int)free_.size())
      throw OutOfPagesError("need " + std::to_string(n) + " KV pages, " + std::to_string(free_.size()) + " free");
    std::vector<int> out;
    out.reserve(n);
    for (int i = 0; i < n; i++) {
      const int p = free_.back();
      free_.pop_back();
      ref_[p] = 1;
      out.push_back(p);
    }
    return out;
  }
  void retain(const std::vector<int>& pages) {
    for (int p : pages) {
      check(p);
      if (ref_[p] <= 0) throw std::runtime_error("retain of free page " + std::to_string(p));
      ref_[p]++;
    }
  }
  void release(const std::vector<int>& pages) {
    for (int p : pages) {
      check(p);
      const int r = ref_[p] - 1;
      if (r < 0) throw std::runtime_error("double release of page " + std::to_string(p));
      ref_[p] = r;
      if (r == 0) free_.push_back(p);
    }
  }
  int refcount(int p) const {
    check(p);
    return ref_[p];
  }
  const std::vector<int>& refs() const { return ref_; }

 private:
  void check(int p) const {
    if (p < 0 || p >= n_pages_) throw std::out_of_range("page id " + std::to_string(p));
  }
  int n_pages_, reserve_;
  std::vector<int> ref_;
  std::vector<int> free_;
};

struct Node {
  std::vector<int64_t> key;  // tokens on the edge into this node (a multiple of the page size)
  std::vector<int> pages;    // one page per page_size tokens of key
  std::unordered_map<std::string, std::unique_ptr<Node>> children;  // by the first page of tokens
  Node* parent = nullptr;
  uint64_t last_use = 0;
};

class RadixCache {
 public:
  RadixCache(std::shared_ptr<PagePool> pool, int page_size) : pool_(std::move(pool)), ps_(page_size) {
    if (page_size <= 0) throw std::invalid_argument("page size");
    root_ = std::make_unique<Node>();
  }

  // Longest cached whole-page prefix -> (tokens matched, pages).  Splits an edge that matches
  // only partly so the returned pages end on a node boundary.
  std::pair<int64_t, std::vector<int>> match(const std::vector<int64_t>& tokens) {
    std::vector<Node*> path;
    std::vector<int> pages;
    const int64_t i = walk(tokens, (int64_t)tokens.size(), &pages, &path);
    const uint64_t now = ++clock_;
    for (Node* nd : path) nd->last_use = now;
    return {i, pages};
  }

  std::pair<int64_t, std::vector<int>> lookup(const std::vector<int64_t>& tokens, py::object max_tokens) {
    int64_t limit = (int64_t)tokens.size();
    if (!max_tokens.is_none()) limit = std::min<int64_t>(limit, max_tokens.cast<int64_t>());
    std::vector<Node*> path;
    std::vector<int> pages;
    const int64_t n = walk(tokens, limit, &pages, &path);
    const uint64_t now = ++clock_;
    for (Node* nd : path) nd->last_use = now;
    lookup_tokens_ += (int64_t)tokens.size();
    hits_tokens_ += n;
    pool_->retain(pages);
    return {n, pages};
  }

  int64_t insert(const std::vector<int64_t>& tokens, const std::vector<int>& pages) {
    const int64_t n = std::min<int64_t>((int64_t)tokens.size() - (int64_t)tokens.size() % ps_,
                                        (int64_t)pages.size() * ps_);
    Node* node = root_.get();
    int64_t i = 0, added = 0;
    while (i < n) {
      const std::string k = chunk_key(tokens.data() + i);
      auto it = node->children.find(k);
      if (it == node->children.end()) {
        auto nn = std::make_unique<Node>();
        nn->key.assign(tokens.begin() + i, tokens.begin() + n);
        nn->pages.assign(pages.begin() + i / ps_, pages.begin() + n / ps_);
        nn->parent = node;
        nn->last_use = ++clock_;
        pool_->retain(nn->pages);
        n_cached_pages_ += (int64_t)nn->pages.size();
        added += n - i;
        node->children.emplace(k, std::move(nn));
        break;
      }
      Node* child = it->second.get();
      int64_t m = common(child->key, tokens, i, n);
      m -= m % ps_;
      if (m == 0) break;  // cannot happen: the first page matched by key
      if (m < (int64_t)child->key.size()) child = split(child, m);
      child->last_use = ++clock_;
      i += m;
      node = child;
    }
    return added;
  }

  // Free up to n_pages by dropping least-recently-used leaves no live sequence holds.
  int64_t evict(int64_t n_pages) {
    int64_t freed = 0;
    while (freed < n_pages) {
      Node* victim = nullptr;
      std::vector<Node*> stack{root_.get()};
      while (!stack.empty()) {
        Node* nd = stack.back();
        stack.pop_back();
        if (nd->children.empty() && nd != root_.get()) {
          bool unlocked = true;
          for (int p : nd->pages)
            if (pool_->refcount(p) != 1) {
              unlocked = false;
              break;
            }
          if (unlocked && (victim == nullptr || nd->last_use < victim->last_use)) victim = nd;
        }
        for (auto& kv : nd->children) stack.push_back(kv.second.get());
      }
      if (victim == nullptr) break;
      Node* parent = victim->parent;
      std::vector<int> pages = victim->pages;
      parent->children.erase(chunk_key(victim->key.data()));
      pool_->release(pages);
      n_cached_pages_ -= (int64_t)pages.size();
      freed += (int64_t)pages.size();
    }
    return freed;
  }

  // (tokens, pages) of every root-to-leaf path, sorted (a session checkpoint saves these)
  std::vector<std::pair<std::vector<int64_t>, std::vector<int>>> sequences() const {
    std::vector<std::pair<std::vector<int64_t>, std::vector<int>>> out;
    struct Item {
      const Node* nd;
      std::vector<int64_t> toks;
      std::vector<int> pages;
    };
    std::vector<Item> stack{{root_.get(), {}, {}}};
    while (!stack.empty()) {
      Item it = std::move(stack.back());
      stack.pop_back();
      it.toks.insert(it.toks.end(), it.nd->key.begin(), it.nd->key.end());
      it.pages.insert(it.pages.end(), it.nd->pages.begin(), it.nd->pages.end());
      if (it.nd->children.empty() && it.nd != root_.get()) out.emplace_back(it.toks, it.pages);
      for (auto& kv : it.nd->children) stack.push_back({kv.second.get(), it.toks, it.pages});
    }
    std::sort(out.begin(), out.end());
    return out;
  }

  py::dict stats() const {
    py::dict d;
    d["cached_pages"] = n_cached_pages_;
    d["hit_tokens"] = hits_tokens_;
    d["lookup_tokens"] = lookup_tokens_;
    d["hit_rate"] = lookup_tokens_ ? (double)hits_tokens_ / (double)lookup_tokens_ : 0.0;
    return d;
  }
  int64_t n_cached_pages() const { return n_cached_pages_; }
  std::shared_ptr<PagePool> pool() const { return pool_; }
  int page_size() const { return ps_; }

 private:
  std::string chunk_key(const int64_t* t) const {
    return std::string(reinterpret_cast<const char*>(t), sizeof(int64_t) * (size_t)ps_);
  }
  static int64_t common(const std::vector<int64_t>& key, const std::vector<int64_t>& tokens, int64_t i, int64_t n) {
    int64_t m = 0;
    const int64_t lim = std::min<int64_t>((int64_t)key.size(), n - i);
    while (m < lim && key[m] == tokens[i + m]) m++;
    return m;
  }
  int64_t walk(const std::vector<int64_t>& tokens, int64_t limit, std::vector<int>* pages, std::vector<Node*>* path) {
    Node* node = root_.get();
    int64_t i = 0;
    const int64_t n = limit - limit % ps_;
    while (i < n) {
      auto it = node->children.find(chunk_key(tokens.data() + i));
      if (it == node->children.end()) break;
      Node* child = it->second.get();
      int64_t m = common(child->key, tokens, i, n);
      m -= m % ps_;
      if (m == 0) break;
      if (m < (int64_t)child->key.size()) child = split(child, m);
      pages->insert(pages->end(), child->pages.begin(), child->pages.end());
      path->push_back(child);
      i += m;
      node = child;
    }
    return i;
  }
  // Split node's edge after m tokens; returns the new upper node.
  Node* split(Node* node, int64_t m) {
    Node* parent = node->parent;
    const std::string k = chunk_key(node->key.data());
    std::unique_ptr<Node> lower = std::move(parent->children[k]);
    auto upper = std::make_unique<Node>();
    upper->key.assign(lower->key.begin(), lower->key.begin() + m);
    upper->pages.assign(lower->pages.begin(), lower->pages.begin() + m / ps_);
    upper->parent = parent;
    upper->last_use = lower->last_use;
    lower->key.erase(lower->key.begin(), lower->key.begin() + m);
    lower->pages.erase(lower->pages.begin(), lower->pages.begin() + m / ps_);
    lower->parent = upper.get();
    Node* up = upper.get();
    up->children.emplace(chunk_key(lower->key.data()), std::move(lower));
    parent->children[k] = std::move(upper);
    return up;
  }

  std::shared_ptr<PagePool> pool_;
  int ps_;
  std::unique_ptr<Node> root_;
  uint64_t clock_ = 0;
  int64_t hits_tokens_ = 0, lookup_tokens_ = 0, n_cached_pages_ = 0;
};

}  // namespace

void register_radix(py::module& m) {
  py::register_exception_translator([](std::exception_ptr p) {
    try {
      if (p) std::rethrow_exception(p);
    } catch (const OutOfPagesError& e) {
      py::object kv = py::module_::import("fak_b200.kv.radix");
      PyErr_SetString(kv.attr("OutOfPages").ptr(), e.what());
    }
  });
  py::class_<PagePool, std::shared_ptr<PagePool>>(m, "PagePool")
      .def(py::init<int, int>(), py::arg("n_pages"), py::arg("reserve") = 1)
      .def("n_free", &PagePool::n_free)
      .def("alloc", &PagePool::alloc)
      .def("retain", &PagePool::retain)
      .def("release", &PagePool::release)
      .def("refcount", &PagePool::refcount)
      .def_property_readonly("ref", &PagePool::refs)
      .def_property_readonly("n_pages", &PagePool::n_pages)
      .def_property_readonly("reserve", &PagePool::reserve);
  py::class_<RadixCache>(m, "RadixCache")
      .def(py::init<std::shared_ptr<PagePool>, int>(), py::arg("pool"), py::arg("page_size") = 16)
      .def("match", &RadixCache::match)
      .def("lookup", &RadixCache::lookup, py::arg("tokens"), py::arg("max_tokens") = py::none())
      .def("insert", &RadixCache::insert)
      .def("evict", &RadixCache::evict)
      .def("stats", &RadixCache::stats)
      .def("sequences", &RadixCache::sequences)
      .def_property_readonly("n_cached_pages", &RadixCache::n_cached_pages)
      .def_property_readonly("pool", &RadixCache::pool)
      .def_property_readonly("ps", &RadixCache::page_size);
}
