// Radix prefix tree over token ids, kept entirely in host C++.
//
// Behaviour follows the reference's Python radix cache (python/minisgl/kvcache/radix_cache.py:
// match with page-aligned node split :205-231, insert :136-146, lock/unlock up the parent chain
// :113-130, LRU eviction of unreferenced leaves :148-175) and its C++ key compare
// (python/minisgl/kernel/csrc/src/radix.cpp:19-40). The data structure is this engine's own:
// nodes live in a vector with a free list and generation counters (stale handles are detected),
// children are bucketed by a hash of their first page, and every tree operation (walk, split,
// insert, evict, integrity check) runs in C++ so the scheduler's hot path never touches Python
// objects per node.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <queue>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;
using i32 = int32_t;
using i64 = int64_t;
using IntArray = py::array_t<i32, py::array::c_style | py::array::forcecast>;

namespace {

struct Node {
  std::vector<i32> key;    // token ids on the edge into this node
  std::vector<i32> value;  // KV slot index per token
  int parent = -1;
  i64 ref = 0;
  uint64_t stamp = 0;
  uint32_t gen = 0;
  bool alive = false;
  std::unordered_map<uint64_t, std::vector<int>> kids;  // first-page hash -> child ids
  size_t num_kids = 0;
};

class RadixTree {
 public:
  explicit RadixTree(int page_size) : page_(page_size) {
    if (page_size <= 0) throw std::invalid_argument("page_size must be positive");
    root_ = new_node();
    nodes_[root_].ref = 1;  // the root is never evictable
  }

  // Walk the tree along `tokens`; split a partially matched edge at a page boundary.
  // Returns (node handle, matched length). Mutates only timestamps and splits.
  py::tuple match(IntArray tokens) {
    auto buf = tokens.unchecked<1>();
    std::vector<i32> t(buf.data(0), buf.data(0) + buf.shape(0));
    auto [node, len] = walk(t.data(), (i64)t.size());
    return py::make_tuple(handle(node), len);
  }

  // Insert the page-aligned prefix of `tokens` with slot `indices`.
  // Returns (length that was already present, handle of the node ending the prefix).
  py::tuple insert(IntArray tokens, IntArray indices) {
    auto tb = tokens.unchecked<1>();
    auto ib = indices.unchecked<1>();
    if (tb.shape(0) != ib.shape(0)) throw std::invalid_argument("tokens/indices length differ");
    i64 n = tb.shape(0) - tb.shape(0) % page_;
    auto [node, prefix] = walk(tb.data(0), n);
    if (prefix < n) {
      int c = new_node();
      Node& nn = nodes_[c];
      nn.key.assign(tb.data(0) + prefix, tb.data(0) + n);
      nn.value.assign(ib.data(0) + prefix, ib.data(0) + n);
      nn.stamp = ++clock_;
      attach(c, node);
      evictable_ += n - prefix;
      node = c;
    }
    return py::make_tuple(prefix, handle(node));
  }

  void lock(i64 h) {
    for (int n = resolve(h); n != root_; n = nodes_[n].parent) {
      Node& x = nodes_[n];
      if (x.ref == 0) {
        evictable_ -= (i64)x.key.size();
        protected_ += (i64)x.key.size();
      }
      x.ref++;
    }
  }

  void unlock(i64 h) {
    for (int n = resolve(h); n != root_; n = nodes_[n].parent) {
      Node& x = nodes_[n];
      if (x.ref <= 0) throw std::runtime_error("radix: unlock of an unlocked node");
      if (--x.ref == 0) {
        evictable_ += (i64)x.key.size();
        protected_ -= (i64)x.key.size();
      }
    }
  }

  // Slot indices of the whole path root -> node.
  py::array_t<i32> indices(i64 h) {
    std::vector<int> path;
    for (int n = resolve(h); n != root_; n = nodes_[n].parent) path.push_back(n);
    size_t total = 0;
    for (int n : path) total += nodes_[n].value.size();
    py::array_t<i32> out((py::ssize_t)total);
    i32* p = out.mutable_data();
    for (auto it = path.rbegin(); it != path.rend(); ++it) {
      const auto& v = nodes_[*it].value;
      std::copy(v.begin(), v.end(), p);
      p += v.size();
    }
    return out;
  }

  i64 length_of(i64 h) {
    i64 len = 0;
    for (int n = resolve(h); n != root_; n = nodes_[n].parent) len += (i64)nodes_[n].key.size();
    return len;
  }

  // Free at least `size` tokens from least recently used unreferenced leaves.
  py::array_t<i32> evict(i64 size) {
    if (size <= 0) return py::array_t<i32>(0);
    if (size > evictable_)
      throw std::runtime_error("radix: cannot evict " + std::to_string(size) + ", only " +
                               std::to_string(evictable_) + " evictable");
    using Item = std::pair<uint64_t, int>;
    std::priority_queue<Item, std::vector<Item>, std::greater<Item>> heap;
    for (size_t i = 0; i < nodes_.size(); ++i) {
      const Node& x = nodes_[i];
      if (x.alive && (int)i != root_ && x.num_kids == 0 && x.ref == 0) heap.emplace(x.stamp, (int)i);
    }
    std::vector<i32> out;
    i64 freed = 0;
    while (freed < size) {
      if (heap.empty()) throw std::runtime_error("radix: eviction ran out of leaves");
      int n = heap.top().second;
      heap.pop();
      Node& x = nodes_[n];
      freed += (i64)x.key.size();
      evictable_ -= (i64)x.key.size();
      out.insert(out.end(), x.value.begin(), x.value.end());
      int p = x.parent;
      detach(n);
      free_node(n);
      Node& px = nodes_[p];
      if (p != root_ && px.num_kids == 0 && px.ref == 0) heap.emplace(px.stamp, p);
    }
    py::array_t<i32> arr((py::ssize_t)out.size());
    std::copy(out.begin(), out.end(), arr.mutable_data());
    return arr;
  }

  i64 evictable_size() const { return evictable_; }
  i64 protected_size() const { return protected_; }
  i64 num_nodes() const { return (i64)(nodes_.size() - free_.size()); }
  i64 root_handle() { return handle(root_); }

  // Recount sizes from scratch and verify structural invariants.
  void check_integrity() {
    i64 ev = 0, pr = 0;
    for (size_t i = 0; i < nodes_.size(); ++i) {
      const Node& x = nodes_[i];
      if (!x.alive || (int)i == root_) continue;
      if (x.key.size() != x.value.size() || x.key.empty())
        throw std::runtime_error("radix: bad node key/value");
      if (x.key.size() % page_ != 0) throw std::runtime_error("radix: node not page aligned");
      if (x.ref < 0) throw std::runtime_error("radix: negative ref");
      (x.ref == 0 ? ev : pr) += (i64)x.key.size();
      const Node& p = nodes_[x.parent];
      if (!p.alive) throw std::runtime_error("radix: dead parent");
      if (x.ref > p.ref && x.parent != root_) throw std::runtime_error("radix: child ref > parent");
      size_t cnt = 0;
      for (auto& kv : x.kids) cnt += kv.second.size();
      if (cnt != x.num_kids) throw std::runtime_error("radix: child count mismatch");
    }
    if (ev != evictable_ || pr != protected_)
      throw std::runtime_error("radix: size accounting mismatch");
  }

 private:
  int page_;
  int root_ = -1;
  uint64_t clock_ = 0;
  i64 evictable_ = 0, protected_ = 0;
  std::vector<Node> nodes_;
  std::vector<int> free_;

  uint64_t page_hash(const i32* t) const {
    uint64_t h = 1469598103934665603ull;  // FNV-1a over the first page
    for (int i = 0; i < page_; ++i) {
      h ^= (uint32_t)t[i];
      h *= 1099511628211ull;
    }
    return h;
  }

  int new_node() {
    int id;
    if (!free_.empty()) {
      id = free_.back();
      free_.pop_back();
    } else {
      id = (int)nodes_.size();
      nodes_.emplace_back();
    }
    Node& x = nodes_[id];
    uint32_t g = x.gen + 1;
    x = Node();
    x.gen = g;
    x.alive = true;
    return id;
  }

  void free_node(int n) {
    Node& x = nodes_[n];
    x.alive = false;
    x.key.clear();
    x.key.shrink_to_fit();
    x.value.clear();
    x.value.shrink_to_fit();
    x.kids.clear();
    free_.push_back(n);
  }

  i64 handle(int n) const { return ((i64)nodes_[n].gen << 32) | (uint32_t)n; }

  int resolve(i64 h) const {
    int n = (int)(uint32_t)(h & 0xffffffff);
    uint32_t g = (uint32_t)((uint64_t)h >> 32);
    if (n < 0 || n >= (int)nodes_.size() || !nodes_[n].alive || nodes_[n].gen != g)
      throw std::runtime_error("radix: stale or invalid handle");
    return n;
  }

  void attach(int c, int p) {
    nodes_[c].parent = p;
    nodes_[p].kids[page_hash(nodes_[c].key.data())].push_back(c);
    nodes_[p].num_kids++;
  }

  void detach(int c) {
    Node& p = nodes_[nodes_[c].parent];
    auto it = p.kids.find(page_hash(nodes_[c].key.data()));
    auto& v = it->second;
    v.erase(std::find(v.begin(), v.end(), c));
    if (v.empty()) p.kids.erase(it);
    p.num_kids--;
  }

  int find_child(int p, const i32* t) const {
    const Node& x = nodes_[p];
    auto it = x.kids.find(page_hash(t));
    if (it == x.kids.end()) return -1;
    for (int c : it->second)
      if (std::equal(t, t + page_, nodes_[c].key.data())) return c;
    return -1;
  }

  // Split node n so that its first `pos` tokens become a new parent. Returns the new parent.
  int split(int n, i64 pos) {
    int p = nodes_[n].parent;
    detach(n);
    int m = new_node();
    Node& nm = nodes_[m];
    Node& nn = nodes_[n];
    nm.key.assign(nn.key.begin(), nn.key.begin() + pos);
    nm.value.assign(nn.value.begin(), nn.value.begin() + pos);
    nm.ref = nn.ref;
    nm.stamp = nn.stamp;
    nn.key.erase(nn.key.begin(), nn.key.begin() + pos);
    nn.value.erase(nn.value.begin(), nn.value.begin() + pos);
    attach(m, p);
    attach(n, m);
    return m;
  }

  std::pair<int, i64> walk(const i32* t, i64 n) {
    uint64_t now = ++clock_;
    int node = root_;
    i64 done = 0;
    while (n - done >= page_) {
      int c = find_child(node, t + done);
      if (c < 0) break;
      const auto& key = nodes_[c].key;
      i64 lim = std::min<i64>((i64)key.size(), n - done);
      i64 m = std::mismatch(key.data(), key.data() + lim, t + done).first - key.data();
      m -= m % page_;
      nodes_[c].stamp = now;
      if (m < (i64)key.size()) {
        int s = split(c, m);
        nodes_[s].stamp = now;
        return {s, done + m};
      }
      done += m;
      node = c;
    }
    return {node, done};
  }
};

// First index where a and b differ (the reference's fast_compare_key).
i64 compare_key(IntArray a, IntArray b) {
  auto x = a.unchecked<1>();
  auto y = b.unchecked<1>();
  i64 n = std::min<i64>(x.shape(0), y.shape(0));
  return std::mismatch(x.data(0), x.data(0) + n, y.data(0)).first - x.data(0);
}

}  // namespace

PYBIND11_MODULE(_host, m) {
  m.doc() = "minisgl host-side runtime: radix prefix tree";
  py::class_<RadixTree>(m, "RadixTree")
      .def(py::init<int>(), py::arg("page_size"))
      .def("match", &RadixTree::match)
      .def("insert", &RadixTree::insert)
      .def("lock", &RadixTree::lock)
      .def("unlock", &RadixTree::unlock)
      .def("indices", &RadixTree::indices)
      .def("length_of", &RadixTree::length_of)
      .def("evict", &RadixTree::evict)
      .def("check_integrity", &RadixTree::check_integrity)
      .def("root_handle", &RadixTree::root_handle)
      .def_property_readonly("evictable_size", &RadixTree::evictable_size)
      .def_property_readonly("protected_size", &RadixTree::protected_size)
      .def_property_readonly("num_nodes", &RadixTree::num_nodes);
  m.def("compare_key", &compare_key);
}
