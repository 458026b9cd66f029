// Paged-KV block manager (host side of the paged cache).
//
// Capabilities of the reference's BlockManager / PageTable / PagedKVCache /
// PrefixCache (openmini-server/src/hardware/kv_cache/block_manager.rs:33-280,
// page_table.rs:10-290, paged_cache.rs:110-435, prefix_cache.rs:14-862):
// ref-counted fixed-size blocks, per-sequence block tables, fork with
// copy-on-write, slot mapping for the device cache writer, and reuse of full
// prompt blocks through a chained token hash with LRU eviction of unreferenced
// cached blocks.
//
// The device cache itself is a flat [blocks, kv_heads, 16, head_dim] tensor per
// layer; this class only hands out block ids and slot numbers
// (slot = block * block_size + offset).
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>
#include <pybind11/numpy.h>

#include <cstdint>
#include <list>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace om_rt {

struct Seq {
  std::vector<int32_t> blocks;
  std::vector<int32_t> tokens;  // tokens whose KV is (or will be) in the cache
  std::vector<uint64_t> hashes; // chained hash of each full block (for the prefix cache)
};

static inline uint64_t mix(uint64_t h, uint64_t v) {
  // splitmix64-style combine
  h ^= v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2);
  h ^= h >> 30;
  h *= 0xBF58476D1CE4E5B9ull;
  h ^= h >> 27;
  h *= 0x94D049BB133111EBull;
  h ^= h >> 31;
  return h;
}

class BlockManager {
 public:
  BlockManager(int num_blocks, int block_size, bool prefix_cache)
      : nb_(num_blocks), bs_(block_size), prefix_(prefix_cache), ref_(num_blocks, 0),
        block_hash_(num_blocks, 0), lru_pos_(num_blocks) {
    if (num_blocks <= 0 || block_size <= 0) throw std::invalid_argument("num_blocks and block_size must be > 0");
    free_.reserve(num_blocks);
    for (int i = num_blocks - 1; i >= 0; --i) free_.push_back(i);
    in_lru_.assign(num_blocks, false);
  }

  int block_size() const { return bs_; }
  int num_blocks() const { return nb_; }
  int num_free() const { return (int)free_.size() + (int)lru_.size(); }
  double utilization() const { return 1.0 - (double)num_free() / nb_; }
  bool has(int64_t sid) const { return seqs_.count(sid) != 0; }

  int blocks_needed(int n_tokens) const { return (n_tokens + bs_ - 1) / bs_; }
  bool can_allocate(int n_tokens) const { return blocks_needed(n_tokens) <= num_free(); }

  // Register a new sequence holding `tokens`; returns the number of leading
  // tokens whose KV is already cached (prefix hit; always < len(tokens)).
  int allocate(int64_t sid, const std::vector<int32_t>& tokens) {
    if (seqs_.count(sid)) throw std::invalid_argument("sequence already allocated: " + std::to_string(sid));
    if (tokens.empty()) throw std::invalid_argument("empty sequence");
    Seq s;
    int cached = 0;
    const int n = (int)tokens.size();
    const int max_hit_blocks = (n - 1) / bs_;  // keep >= 1 token to compute
    uint64_t h = 0x51ED270B27EAFull;
    int hit_blocks = 0;
    if (prefix_) {
      for (int b = 0; b < max_hit_blocks; ++b) {
        uint64_t hb = h;
        for (int j = 0; j < bs_; ++j) hb = mix(hb, (uint32_t)tokens[b * bs_ + j]);
        auto it = cache_.find(hb);
        if (it == cache_.end()) break;
        const int blk = it->second;
        take_cached(blk);
        s.blocks.push_back(blk);
        s.hashes.push_back(hb);
        h = hb;
        ++hit_blocks;
      }
      cached = hit_blocks * bs_;
    }
    const int need = blocks_needed(n) - hit_blocks;
    if (need > num_free()) {
      for (int blk : s.blocks) release(blk);
      throw std::runtime_error("out of KV blocks");
    }
    for (int i = 0; i < need; ++i) s.blocks.push_back(alloc_block());
    s.tokens = tokens;
    seqs_.emplace(sid, std::move(s));
    rehash_full_blocks(sid);
    hits_ += cached;
    queries_ += n;
    return cached;
  }

  // Free blocks that appending n tokens takes: new blocks plus a copy of a shared,
  // partly filled last block (copy-on-write).
  int append_need(int64_t sid, int n) const {
    const Seq& s = get(sid);
    const int need = blocks_needed((int)s.tokens.size() + n) - (int)s.blocks.size();
    int cow = 0;
    if (!s.blocks.empty() && (s.tokens.size() % bs_) != 0 && ref_[s.blocks.back()] > 1) cow = 1;
    return std::max(need, 0) + cow;
  }

  bool can_append(int64_t sid, int n) const { return append_need(sid, n) <= num_free(); }

  // Append tokens to a sequence. Returns copy-on-write pairs (src, dst) that
  // the caller must apply to the device cache before writing new KV.
  std::vector<std::pair<int, int>> append(int64_t sid, const std::vector<int32_t>& toks) {
    Seq& s = getm(sid);
    std::vector<std::pair<int, int>> cow;
    if (toks.empty()) return cow;
    const size_t last = s.tokens.size() / bs_;  // block receiving the next token
    if ((s.tokens.size() % bs_) != 0 && last < s.blocks.size() && ref_[s.blocks[last]] > 1) {
      const int src = s.blocks[last];
      const int dst = alloc_block();
      release(src);
      s.blocks[last] = dst;
      cow.emplace_back(src, dst);
    }
    const int need = blocks_needed((int)(s.tokens.size() + toks.size())) - (int)s.blocks.size();
    if (need > num_free()) throw std::runtime_error("out of KV blocks");
    for (int i = 0; i < need; ++i) s.blocks.push_back(alloc_block());
    s.tokens.insert(s.tokens.end(), toks.begin(), toks.end());
    rehash_full_blocks(sid);
    return cow;
  }

  // Make sure blocks exist for `n` more tokens without registering tokens
  // (multi-step decode reserves slots before the tokens are known).
  void reserve(int64_t sid, int n) {
    Seq& s = getm(sid);
    const int need = blocks_needed((int)s.tokens.size() + n) - (int)s.blocks.size();
    if (need > num_free()) throw std::runtime_error("out of KV blocks");
    for (int i = 0; i < need; ++i) s.blocks.push_back(alloc_block());
  }

  // Child shares all of the parent's blocks (beam / group sampling).
  void fork(int64_t parent, int64_t child) {
    if (seqs_.count(child)) throw std::invalid_argument("child exists");
    Seq c = get(parent);
    for (int b : c.blocks) ref_[b]++;
    seqs_.emplace(child, std::move(c));
  }

  void free(int64_t sid) {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) return;
    for (int b : it->second.blocks) release(b);
    seqs_.erase(it);
  }

  std::vector<int32_t> block_table(int64_t sid) const { return get(sid).blocks; }
  int seq_len(int64_t sid) const { return (int)get(sid).tokens.size(); }

  // slots for tokens [start, end) of the sequence
  std::vector<int32_t> slots(int64_t sid, int start, int end) const {
    const Seq& s = get(sid);
    if (start < 0 || end > (int)s.blocks.size() * bs_ || start > end) throw std::out_of_range("slot range");
    std::vector<int32_t> out(end - start);
    for (int t = start; t < end; ++t) out[t - start] = s.blocks[t / bs_] * bs_ + (t % bs_);
    return out;
  }

  // Decode batch: the cache slot of position pos[i] of sequence sids[i] -> out[i].
  void decode_slots(const std::vector<int64_t>& sids, py::array_t<int32_t> pos, py::array_t<int32_t> out) const {
    auto p = pos.unchecked<1>();
    auto o = out.mutable_unchecked<1>();
    if ((size_t)p.shape(0) < sids.size() || (size_t)o.shape(0) < sids.size())
      throw std::out_of_range("decode_slots: arrays shorter than the batch");
    for (size_t i = 0; i < sids.size(); ++i) {
      const Seq& s = get(sids[i]);
      const int t = p(i);
      if (t < 0 || t >= (int)s.blocks.size() * bs_) throw std::out_of_range("decode_slots: position");
      o(i) = s.blocks[t / bs_] * bs_ + (t % bs_);
    }
  }

  // Fill a [len(sids), max_blocks] int32 numpy array (padded with 0).
  void fill_block_tables(const std::vector<int64_t>& sids, py::array_t<int32_t> out) const {
    auto buf = out.mutable_unchecked<2>();
    const int mb = (int)buf.shape(1);
    for (size_t i = 0; i < sids.size(); ++i) {
      const Seq& s = get(sids[i]);
      if ((int)s.blocks.size() > mb) throw std::out_of_range("block table wider than max_blocks");
      int j = 0;
      for (; j < (int)s.blocks.size(); ++j) buf(i, j) = s.blocks[j];
      for (; j < mb; ++j) buf(i, j) = 0;
    }
  }

  double prefix_hit_rate() const { return queries_ ? (double)hits_ / queries_ : 0.0; }
  int ref_count(int blk) const { return ref_.at(blk); }
  int num_cached_blocks() const { return (int)cache_.size(); }

  void reset_prefix_cache() {
    for (int b : lru_) {
      in_lru_[b] = false;
      block_hash_[b] = 0;
      free_.push_back(b);
    }
    lru_.clear();
    cache_.clear();
  }

 private:
  const Seq& get(int64_t sid) const {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) throw std::out_of_range("unknown sequence " + std::to_string(sid));
    return it->second;
  }
  Seq& getm(int64_t sid) {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) throw std::out_of_range("unknown sequence " + std::to_string(sid));
    return it->second;
  }

  int alloc_block() {
    int b;
    if (!free_.empty()) {
      b = free_.back();
      free_.pop_back();
    } else if (!lru_.empty()) {
      b = lru_.front();  // evict least recently used cached block
      lru_.pop_front();
      in_lru_[b] = false;
      cache_.erase(block_hash_[b]);
    } else {
      throw std::runtime_error("out of KV blocks");
    }
    block_hash_[b] = 0;
    ref_[b] = 1;
    return b;
  }
  void take_cached(int b) {
    if (in_lru_[b]) {
      lru_.erase(lru_pos_[b]);
      in_lru_[b] = false;
    }
    ref_[b]++;
  }
  void release(int b) {
    if (--ref_[b] > 0) return;
    ref_[b] = 0;
    auto it = block_hash_[b] ? cache_.find(block_hash_[b]) : cache_.end();
    if (prefix_ && it != cache_.end() && it->second == b) {
      lru_.push_back(b);
      lru_pos_[b] = std::prev(lru_.end());
      in_lru_[b] = true;
    } else {
      block_hash_[b] = 0;
      free_.push_back(b);
    }
  }
  void rehash_full_blocks(int64_t sid) {
    if (!prefix_) return;
    Seq& s = getm(sid);
    const int full = (int)s.tokens.size() / bs_;
    uint64_t h = s.hashes.empty() ? 0x51ED270B27EAFull : s.hashes.back();
    for (int b = (int)s.hashes.size(); b < full; ++b) {
      for (int j = 0; j < bs_; ++j) h = mix(h, (uint32_t)s.tokens[b * bs_ + j]);
      s.hashes.push_back(h);
      const int blk = s.blocks[b];
      if (!cache_.count(h) && block_hash_[blk] == 0) {
        cache_[h] = blk;
        block_hash_[blk] = h;
      }
    }
  }

  int nb_, bs_;
  bool prefix_;
  std::vector<int> ref_;
  std::vector<int> free_;
  std::vector<uint64_t> block_hash_;
  std::list<int> lru_;
  std::vector<std::list<int>::iterator> lru_pos_;
  std::vector<bool> in_lru_;
  std::unordered_map<uint64_t, int> cache_;
  std::unordered_map<int64_t, Seq> seqs_;
  int64_t hits_ = 0, queries_ = 0;
};

}  // namespace om_rt

void bind_block_manager(py::module_& m) {
  using om_rt::BlockManager;
  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, bool>(), py::arg("num_blocks"), py::arg("block_size") = 16,
           py::arg("prefix_cache") = true)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def_property_readonly("num_blocks", &BlockManager::num_blocks)
      .def("num_free", &BlockManager::num_free)
      .def("utilization", &BlockManager::utilization)
      .def("has", &BlockManager::has)
      .def("blocks_needed", &BlockManager::blocks_needed)
      .def("can_allocate", &BlockManager::can_allocate)
      .def("allocate", &BlockManager::allocate)
      .def("can_append", &BlockManager::can_append)
      .def("append_need", &BlockManager::append_need)
      .def("append", &BlockManager::append)
      .def("reserve", &BlockManager::reserve)
      .def("fork", &BlockManager::fork)
      .def("free", &BlockManager::free)
      .def("block_table", &BlockManager::block_table)
      .def("seq_len", &BlockManager::seq_len)
      .def("slots", &BlockManager::slots)
      .def("decode_slots", &BlockManager::decode_slots)
      .def("fill_block_tables", &BlockManager::fill_block_tables)
      .def("prefix_hit_rate", &BlockManager::prefix_hit_rate)
      .def("ref_count", &BlockManager::ref_count)
      .def("num_cached_blocks", &BlockManager::num_cached_blocks)
      .def("reset_prefix_cache", &BlockManager::reset_prefix_cache);
}
