// Paged KV-cache block pool + per-sequence block tables + per-step batch-metadata builder (host C++).
//
// Replaces the reference's Java block managers (core/optimization/gollek-plugin-kv-cache/…/kvcache/
// PagedKVCacheManager.java:56-222: free deque, per-request block lists, allocate-for-prefill,
// append-token, free-request; prompt-prefix reuse core/optimization/gollek-plugin-prompt-cache/…/
// PagedKVCacheManagerExtension.java) with one native object the scheduler drives every step:
//
//   * BlockPool: LIFO free stack, reference counts, a hash -> block map of full prompt blocks
//     (prefix cache) and an LRU list of cached blocks whose refcount dropped to 0 (evicted only
//     when the free stack is empty).
//   * SeqTables: block list per sequence id; ensure_capacity() grows a sequence atomically
//     (all-or-nothing) so the scheduler can preempt when the pool is exhausted.
//   * build_batch(): writes positions, slot mapping, padded block tables, KV lengths and query
//     offsets for one engine step straight into (pinned) int32 tensors.
#include <algorithm>
#include <torch/extension.h>

#include <cstdint>
#include <list>
#include <stdexcept>
#include <unordered_map>
#include <vector>

class BlockPool {
 public:
  BlockPool(int64_t num_blocks, int64_t block_size)
      : num_blocks_(num_blocks), block_size_(block_size), ref_(num_blocks, 0), hash_(num_blocks, 0),
        has_hash_(num_blocks, 0), lru_pos_(num_blocks) {
    free_.reserve(num_blocks);
    for (int64_t b = num_blocks - 1; b >= 0; --b) free_.push_back((int32_t)b);
  }

  int64_t num_blocks() const { return num_blocks_; }
  int64_t block_size() const { return block_size_; }
  // blocks that can be handed out right now (free + evictable cached)
  int64_t num_free() const { return (int64_t)free_.size() + (int64_t)lru_.size(); }
  int64_t num_cached() const { return (int64_t)map_.size(); }
  int32_t refcount(int32_t b) const { return ref_.at(b); }

  int32_t alloc() {
    int32_t b;
    if (!free_.empty()) {
      b = free_.back();
      free_.pop_back();
    } else if (!lru_.empty()) {
      b = lru_.front();  // least recently released cached block
      lru_.pop_front();
      map_.erase(hash_[b]);
      has_hash_[b] = 0;
    } else {
      return -1;
    }
    ref_[b] = 1;
    return b;
  }

  void incref(int32_t b) {
    check(b);
    if (ref_[b] == 0 && has_hash_[b]) lru_.erase(lru_pos_[b]);
    ref_[b] += 1;
  }

  void decref(int32_t b) {
    check(b);
    if (ref_[b] <= 0) throw std::runtime_error("BlockPool: double free of block " + std::to_string(b));
    if (--ref_[b] == 0) {
      if (has_hash_[b]) {
        lru_.push_back(b);
        lru_pos_[b] = std::prev(lru_.end());
      } else {
        free_.push_back(b);
      }
    }
  }

  // Prefix-cache lookup: returns the block holding `h` (refcount incremented) or -1.
  int32_t lookup(int64_t h) {
    auto it = map_.find(h);
    if (it == map_.end()) return -1;
    incref(it->second);
    return it->second;
  }
  bool contains(int64_t h) const { return map_.count(h) != 0; }

  // Register a full block under hash h (no-op if the hash is already cached elsewhere).
  void insert(int32_t b, int64_t h) {
    check(b);
    if (map_.count(h) || has_hash_[b]) return;
    map_[h] = b;
    hash_[b] = h;
    has_hash_[b] = 1;
  }

  // Every cached (hash, block) pair (prefix-cache snapshot).
  std::vector<std::pair<int64_t, int32_t>> cached_items() const {
    return std::vector<std::pair<int64_t, int32_t>>(map_.begin(), map_.end());
  }

  // Take a free block, register it under `h` as a cached block with no owner (evictable, LRU
  // tail) and return it, so a snapshot's KV can be written into it; -1 if the hash is already
  // cached or no block is free (cached blocks are never evicted for this).
  int32_t adopt_cached(int64_t h) {
    if (map_.count(h) || free_.empty()) return -1;
    const int32_t b = free_.back();
    free_.pop_back();
    map_[h] = b;
    hash_[b] = h;
    has_hash_[b] = 1;
    ref_[b] = 0;
    lru_.push_back(b);
    lru_pos_[b] = std::prev(lru_.end());
    return b;
  }

  void reset_cache() {
    for (int32_t b : lru_) {
      has_hash_[b] = 0;
      free_.push_back(b);
    }
    lru_.clear();
    for (auto& kv : map_) has_hash_[kv.second] = 0;
    map_.clear();
  }

 private:
  void check(int32_t b) const {
    if (b < 0 || b >= num_blocks_) throw std::out_of_range("BlockPool: bad block id " + std::to_string(b));
  }
  int64_t num_blocks_, block_size_;
  std::vector<int32_t> free_;
  std::vector<int32_t> ref_;
  std::vector<int64_t> hash_;
  std::vector<uint8_t> has_hash_;
  std::list<int32_t> lru_;
  std::vector<std::list<int32_t>::iterator> lru_pos_;
  std::unordered_map<int64_t, int32_t> map_;
};

class SeqTables {
 public:
  explicit SeqTables(BlockPool* pool) : pool_(pool) {}

  void add(int64_t seq) {
    if (tables_.count(seq)) throw std::runtime_error("SeqTables: duplicate sequence " + std::to_string(seq));
    tables_[seq] = {};
  }
  bool has(int64_t seq) const { return tables_.count(seq) != 0; }

  void remove(int64_t seq) {
    auto it = tables_.find(seq);
    if (it == tables_.end()) return;
    for (int32_t b : it->second) pool_->decref(b);
    tables_.erase(it);
    dropped_.erase(seq);
  }

  // KV eviction: remove the blocks at table indices `idx` (sorted, unique, never the last block) and
  // release them. The sequence's later tokens keep their logical positions; their KV slots shift
  // down by the dropped tokens (`dropped`), so attention runs over the kept blocks only.
  int64_t drop(int64_t seq, std::vector<int64_t> idx) {
    auto& t = at(seq);
    std::sort(idx.begin(), idx.end());
    idx.erase(std::unique(idx.begin(), idx.end()), idx.end());
    for (int64_t i : idx)
      if (i < 0 || i + 1 >= (int64_t)t.size()) throw std::out_of_range("SeqTables.drop: bad block index");
    std::vector<int32_t> kept;
    kept.reserve(t.size() - idx.size());
    size_t k = 0;
    for (int64_t i = 0; i < (int64_t)t.size(); ++i) {
      if (k < idx.size() && idx[k] == i) {
        pool_->decref(t[i]);
        ++k;
      } else {
        kept.push_back(t[i]);
      }
    }
    t.swap(kept);
    dropped_[seq] += (int64_t)idx.size() * pool_->block_size();
    return (int64_t)idx.size();
  }
  int64_t dropped(int64_t seq) const {
    auto it = dropped_.find(seq);
    return it == dropped_.end() ? 0 : it->second;
  }

  void append_block(int64_t seq, int32_t b) { at(seq).push_back(b); }

  int64_t num_blocks(int64_t seq) const { return (int64_t)at_c(seq).size(); }
  std::vector<int32_t> blocks(int64_t seq) const { return at_c(seq); }

  // Make room for `total_tokens` tokens; allocates missing blocks all-or-nothing.
  bool ensure_capacity(int64_t seq, int64_t total_tokens) {
    auto& t = at(seq);
    total_tokens -= dropped(seq);
    const int64_t need = (total_tokens + pool_->block_size() - 1) / pool_->block_size();
    const int64_t have = (int64_t)t.size();
    if (need <= have) return true;
    if (need - have > pool_->num_free()) return false;
    for (int64_t i = have; i < need; ++i) {
      int32_t b = pool_->alloc();
      if (b < 0) {  // cannot happen after the num_free check; keep all-or-nothing anyway
        while ((int64_t)t.size() > have) {
          pool_->decref(t.back());
          t.pop_back();
        }
        return false;
      }
      t.push_back(b);
    }
    return true;
  }
  int64_t blocks_needed(int64_t seq, int64_t total_tokens) const {
    total_tokens -= dropped(seq);
    const int64_t need = (total_tokens + pool_->block_size() - 1) / pool_->block_size();
    return std::max<int64_t>(0, need - (int64_t)at_c(seq).size());
  }

  // One engine step. For sequence i: its new tokens occupy absolute positions
  // [start[i], start[i] + n_new[i]). Fills:
  //   positions[T], slots[T], block_tables[n, max_blocks] (padded with 0),
  //   seq_lens[n] = start + n_new, query_start[n + 1].
  // Returns the total number of tokens T.
  int64_t build_batch(torch::Tensor seq_ids, torch::Tensor start, torch::Tensor n_new, torch::Tensor positions,
                      torch::Tensor slots, torch::Tensor block_tables, torch::Tensor seq_lens,
                      torch::Tensor query_start) {
    const int64_t n = seq_ids.numel();
    const int64_t* ids = seq_ids.data_ptr<int64_t>();
    const int32_t* st = start.data_ptr<int32_t>();
    const int32_t* nn = n_new.data_ptr<int32_t>();
    int32_t* pos = positions.data_ptr<int32_t>();
    int32_t* sl = slots.data_ptr<int32_t>();
    int32_t* bt = block_tables.data_ptr<int32_t>();
    int32_t* lens = seq_lens.data_ptr<int32_t>();
    int32_t* qs = query_start.data_ptr<int32_t>();
    const int64_t max_blocks = block_tables.size(1), bt_stride = block_tables.stride(0);
    const int64_t bs = pool_->block_size();
    const int64_t cap_tokens = positions.numel();
    int64_t t = 0;
    qs[0] = 0;
    for (int64_t i = 0; i < n; ++i) {
      const auto& tab = at_c(ids[i]);
      const int64_t nb = (int64_t)tab.size();
      const int64_t dr = dropped(ids[i]);  // tokens evicted before this step's positions
      if (nb > max_blocks) throw std::runtime_error("build_batch: block table wider than buffer");
      if (st[i] < dr) throw std::runtime_error("build_batch: new tokens inside evicted blocks");
      if ((st[i] - dr + nn[i] + bs - 1) / bs > nb) throw std::runtime_error("build_batch: sequence lacks KV blocks");
      if (t + nn[i] > cap_tokens) throw std::runtime_error("build_batch: token buffer too small");
      int32_t* row = bt + i * bt_stride;
      for (int64_t j = 0; j < nb; ++j) row[j] = tab[j];
      for (int64_t j = nb; j < max_blocks; ++j) row[j] = 0;
      for (int64_t k = 0; k < nn[i]; ++k) {
        const int64_t p = st[i] + k, kp = p - dr;
        pos[t] = (int32_t)p;
        sl[t] = (int32_t)(tab[kp / bs] * bs + kp % bs);
        ++t;
      }
      lens[i] = (int32_t)(st[i] + nn[i] - dr);
      qs[i + 1] = (int32_t)t;
    }
    return t;
  }

 private:
  std::vector<int32_t>& at(int64_t seq) {
    auto it = tables_.find(seq);
    if (it == tables_.end()) throw std::runtime_error("SeqTables: unknown sequence " + std::to_string(seq));
    return it->second;
  }
  const std::vector<int32_t>& at_c(int64_t seq) const {
    auto it = tables_.find(seq);
    if (it == tables_.end()) throw std::runtime_error("SeqTables: unknown sequence " + std::to_string(seq));
    return it->second;
  }
  BlockPool* pool_;
  std::unordered_map<int64_t, std::vector<int32_t>> tables_;
  std::unordered_map<int64_t, int64_t> dropped_;
};

void register_block_allocator(pybind11::module& m) {
  namespace py = pybind11;
  py::class_<BlockPool>(m, "BlockPool")
      .def(py::init<int64_t, int64_t>())
      .def_property_readonly("num_blocks", &BlockPool::num_blocks)
      .def_property_readonly("block_size", &BlockPool::block_size)
      .def("num_free", &BlockPool::num_free)
      .def("num_cached", &BlockPool::num_cached)
      .def("refcount", &BlockPool::refcount)
      .def("alloc", &BlockPool::alloc)
      .def("incref", &BlockPool::incref)
      .def("decref", &BlockPool::decref)
      .def("lookup", &BlockPool::lookup)
      .def("contains", &BlockPool::contains)
      .def("insert", &BlockPool::insert)
      .def("reset_cache", &BlockPool::reset_cache)
      .def("cached_items", &BlockPool::cached_items)
      .def("adopt_cached", &BlockPool::adopt_cached);
  py::class_<SeqTables>(m, "SeqTables")
      .def(py::init<BlockPool*>(), py::keep_alive<1, 2>())
      .def("add", &SeqTables::add)
      .def("has", &SeqTables::has)
      .def("remove", &SeqTables::remove)
      .def("append_block", &SeqTables::append_block)
      .def("num_blocks", &SeqTables::num_blocks)
      .def("blocks", &SeqTables::blocks)
      .def("ensure_capacity", &SeqTables::ensure_capacity)
      .def("blocks_needed", &SeqTables::blocks_needed)
      .def("build_batch", &SeqTables::build_batch)
      .def("drop", &SeqTables::drop)
      .def("dropped", &SeqTables::dropped);
}
