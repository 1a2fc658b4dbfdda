// Paged KV block manager (host C++).
//
// Replaces the reference's dense slot-major cache bookkeeping
// (src/cache/parallel_cache_builder.rs:436-876: per-slot positions/indices, host masks) and
// the Fuel paged policies (src/model_fuel/policies.rs: PagedAdmission :330-390,
// BlockPrefixIndex :442-600 with chained per-block hashes and donor refcounts,
// ensure_writable_block COW in src/model_fuel/batched.rs:835-976).
//
// Model:
//  * a pool of `num_blocks` physical blocks of `block_size` token slots;
//  * each sequence owns a block table (vector of physical block ids) and a token count;
//  * blocks are reference counted; a block shared by several tables (prefix hit or fork)
//    is copied on the first write into it (copy-on-write) and the (src, dst) pair is
//    reported to the caller, which performs the device copy;
//  * full blocks are published in a prefix index keyed by a chained 64-bit hash of the
//    block's tokens and its predecessor's hash; the index verifies token contents on
//    lookup, so a hash collision can never splice a wrong prefix;
//  * blocks whose refcount drops to zero but which are in the prefix index stay cached and
//    are evicted least-recently-used when the free list runs dry.
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include <algorithm>
#include <cstdint>
#include <list>
#include <stdexcept>
#include <string>
#include <unordered_map>
#include <vector>

namespace py = pybind11;

namespace lbn {

static inline uint64_t mix64(uint64_t h, uint64_t v) {
  // 64-bit multiply-xorshift mixing (SplitMix64 finaliser applied to h ^ v).
  uint64_t z = h ^ (v + 0x9E3779B97F4A7C15ull + (h << 6) + (h >> 2));
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t hash_block(uint64_t parent, const int32_t* toks, int n) {
  uint64_t h = mix64(parent, 0xB10C5EEDull + static_cast<uint64_t>(n));
  for (int i = 0; i < n; ++i) h = mix64(h, static_cast<uint32_t>(toks[i]));
  return h;
}

struct CachedBlock {
  int block;
  uint64_t parent;
  std::vector<int32_t> tokens;
};

struct Sequence {
  std::vector<int> blocks;
  std::vector<int32_t> tokens;   // token ids written so far (for prefix publishing)
  int64_t num_tokens = 0;        // KV slots in use
  std::vector<uint64_t> hashes;  // chained hash of each full block
  bool no_publish = false;       // set after KV compaction: positions != token prefix
};

class BlockManager {
 public:
  BlockManager(int num_blocks, int block_size, bool enable_prefix)
      : num_blocks_(num_blocks), block_size_(block_size), prefix_(enable_prefix),
        ref_(num_blocks, 0), cached_key_(num_blocks, 0), is_cached_(num_blocks, 0) {
    if (num_blocks <= 0 || block_size <= 0) throw std::invalid_argument("bad geometry");
    free_.reserve(num_blocks);
    for (int b = num_blocks - 1; b >= 0; --b) free_.push_back(b);
  }

  int num_blocks() const { return num_blocks_; }
  int block_size() const { return block_size_; }
  int num_free_blocks() const { return static_cast<int>(free_.size() + lru_.size()); }
  int num_cached_blocks() const { return static_cast<int>(index_.size()); }
  double usage() const { return 1.0 - static_cast<double>(num_free_blocks()) / num_blocks_; }

  bool has_seq(int64_t sid) const { return seqs_.count(sid) != 0; }

  int blocks_needed(int64_t sid, int64_t new_tokens) const {
    auto it = seqs_.find(sid);
    const int64_t have = it == seqs_.end() ? 0 : it->second.num_tokens;
    const int64_t cap = it == seqs_.end() ? 0 : static_cast<int64_t>(it->second.blocks.size()) * block_size_;
    const int64_t need = have + new_tokens - cap;
    int extra = need > 0 ? static_cast<int>((need + block_size_ - 1) / block_size_) : 0;
    // A shared tail block will be copied on write: one more block.
    if (it != seqs_.end() && new_tokens > 0 && have % block_size_ != 0 && !it->second.blocks.empty() &&
        ref_[it->second.blocks.back()] > 1)
      extra += 1;
    return extra;
  }

  bool can_allocate(int64_t sid, int64_t new_tokens) const {
    return blocks_needed(sid, new_tokens) <= num_free_blocks();
  }

  // Admission for a batch: all-or-nothing (src/model_fuel/batched.rs:617-664).
  bool can_allocate_all(const std::vector<int64_t>& sids, const std::vector<int64_t>& n) const {
    int64_t need = 0;
    for (size_t i = 0; i < sids.size(); ++i) need += blocks_needed(sids[i], n[i]);
    return need <= num_free_blocks();
  }

  void add_sequence(int64_t sid) {
    if (seqs_.count(sid)) throw std::runtime_error("duplicate sequence id " + std::to_string(sid));
    seqs_[sid] = Sequence();
  }

  // Longest cached prefix of `tokens` (whole blocks only, leaving at least one token to
  // compute).  Adopts the blocks into `sid`'s table and returns the number of tokens reused.
  int64_t match_prefix(int64_t sid, const std::vector<int32_t>& tokens) {
    auto& s = get(sid);
    if (!prefix_ || !s.blocks.empty()) return 0;
    const int64_t max_full = (static_cast<int64_t>(tokens.size()) - 1) / block_size_;
    uint64_t parent = 0;
    int64_t matched = 0;
    for (int64_t b = 0; b < max_full; ++b) {
      const int32_t* tk = tokens.data() + b * block_size_;
      const uint64_t h = hash_block(parent, tk, block_size_);
      auto it = index_.find(h);
      if (it == index_.end()) break;
      const CachedBlock& cb = it->second;
      if (cb.parent != parent || !std::equal(cb.tokens.begin(), cb.tokens.end(), tk)) break;
      acquire(cb.block);
      s.blocks.push_back(cb.block);
      s.hashes.push_back(h);
      parent = h;
      ++matched;
    }
    s.num_tokens = matched * block_size_;
    s.tokens.assign(tokens.begin(), tokens.begin() + s.num_tokens);
    hits_tokens_ += s.num_tokens;
    query_tokens_ += static_cast<int64_t>(tokens.size());
    return s.num_tokens;
  }

  // Reserve slots for `new_tokens` more tokens of `sid` whose ids are `toks` (may be empty
  // when unknown yet).  Returns {slot mapping, copy-on-write pairs (src,dst) flattened}.
  std::pair<std::vector<int64_t>, std::vector<int>> append_slots(int64_t sid, int64_t new_tokens,
                                                                 const std::vector<int32_t>& toks) {
    auto& s = get(sid);
    if (blocks_needed(sid, new_tokens) > num_free_blocks())
      throw std::runtime_error("out of KV blocks");
    std::vector<int> cow;
    std::vector<int64_t> slots;
    slots.reserve(new_tokens);
    for (int64_t i = 0; i < new_tokens; ++i) {
      const int64_t pos = s.num_tokens;
      const int64_t bi = pos / block_size_;
      const int off = static_cast<int>(pos % block_size_);
      if (bi == static_cast<int64_t>(s.blocks.size())) {
        s.blocks.push_back(take_free());
      } else if (ref_[s.blocks[bi]] > 1) {
        // copy-on-write of a shared partially-filled block
        const int src = s.blocks[bi];
        const int dst = take_free();
        release(src);
        s.blocks[bi] = dst;
        cow.push_back(src);
        cow.push_back(dst);
      }
      slots.push_back(static_cast<int64_t>(s.blocks[bi]) * block_size_ + off);
      s.num_tokens += 1;
      if (i < static_cast<int64_t>(toks.size())) s.tokens.push_back(toks[i]);
      maybe_publish(s);
    }
    return {slots, cow};
  }

  // Record token ids for already-reserved slots (decode: the id is known after sampling).
  void set_tokens(int64_t sid, const std::vector<int32_t>& toks) {
    auto& s = get(sid);
    for (int32_t t : toks) {
      if (static_cast<int64_t>(s.tokens.size()) >= s.num_tokens) break;
      s.tokens.push_back(t);
    }
    maybe_publish(s);
  }

  // Fork: child shares all of parent's blocks (refcount++), COW on later writes.
  void fork(int64_t parent, int64_t child) {
    auto& p = get(parent);
    if (seqs_.count(child)) throw std::runtime_error("fork: child exists");
    Sequence c = p;
    for (int b : c.blocks) acquire(b);
    seqs_[child] = std::move(c);
  }

  // Keep the first `new_len` token slots of `sid` (speculative decoding rollback).
  void truncate(int64_t sid, int64_t new_len) {
    auto& s = get(sid);
    if (new_len >= s.num_tokens) return;
    const int64_t keep_blocks = (new_len + block_size_ - 1) / block_size_;
    while (static_cast<int64_t>(s.blocks.size()) > keep_blocks) {
      release(s.blocks.back());
      s.blocks.pop_back();
    }
    // A kept, partially truncated block will be written again: if it is published in the
    // prefix index (for the tokens that were cut), withdraw it so no later lookup splices
    // KV that is about to change.  A shared block is copied on write instead.
    if (new_len % block_size_ != 0 && !s.blocks.empty()) {
      const int b = s.blocks.back();
      if (is_cached_[b] && ref_[b] == 1) {
        index_.erase(cached_key_[b]);
        is_cached_[b] = 0;
      }
    }
    s.num_tokens = new_len;
    if (static_cast<int64_t>(s.tokens.size()) > new_len) s.tokens.resize(new_len);
    const int64_t full = new_len / block_size_;
    if (static_cast<int64_t>(s.hashes.size()) > full) s.hashes.resize(full);
  }

  // Fresh blocks owned by the caller (refcount 1), e.g. compaction targets.
  std::vector<int> alloc_blocks(int n) {
    if (n > num_free_blocks()) throw std::runtime_error("out of KV blocks");
    std::vector<int> out;
    for (int i = 0; i < n; ++i) out.push_back(take_free());
    return out;
  }

  // Return blocks from alloc_blocks that were never attached to a sequence (rollback).
  void free_blocks(const std::vector<int>& blocks) {
    for (int b : blocks) {
      if (b < 0 || b >= static_cast<int>(ref_.size()) || ref_[b] <= 0)
        throw std::runtime_error("free_blocks: block not held");
      release(b);
    }
  }

  // Replace the table of `sid` with a compacted list of kept logical blocks (KV eviction:
  // the caller has moved surviving slots); blocks not kept are released.
  void set_blocks(int64_t sid, const std::vector<int>& blocks, int64_t num_tokens) {
    auto& s = get(sid);
    std::unordered_map<int, int> keep;
    for (int b : blocks) keep[b]++;
    for (int b : s.blocks) {
      auto it = keep.find(b);
      if (it != keep.end() && it->second > 0) {
        it->second--;
      } else {
        release(b);
      }
    }
    s.blocks = blocks;
    s.num_tokens = num_tokens;
    s.tokens.clear();  // positions no longer map to a token prefix: never publish again
    s.hashes.assign(s.blocks.size() + 1, 0);
    s.no_publish = true;
  }

  void free_sequence(int64_t sid) {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) return;
    for (auto b = it->second.blocks.rbegin(); b != it->second.blocks.rend(); ++b) release(*b);
    seqs_.erase(it);
  }

  std::vector<int> block_table(int64_t sid) const { return getc(sid).blocks; }
  int64_t num_tokens(int64_t sid) const { return getc(sid).num_tokens; }

  // Fill a dense [len(sids), width] int32 table (pad with 0).
  void fill_block_tables(const std::vector<int64_t>& sids, py::buffer out, int width) const {
    py::buffer_info bi = out.request(true);
    if (bi.itemsize != 4) throw std::runtime_error("block table buffer must be int32");
    int32_t* p = static_cast<int32_t*>(bi.ptr);
    for (size_t r = 0; r < sids.size(); ++r) {
      const auto& s = getc(sids[r]);
      if (static_cast<int>(s.blocks.size()) > width) throw std::runtime_error("table too narrow");
      int32_t* row = p + r * width;
      std::copy(s.blocks.begin(), s.blocks.end(), row);
      std::fill(row + s.blocks.size(), row + width, 0);
    }
  }

  int refcount(int b) const { return ref_.at(b); }
  std::pair<int64_t, int64_t> prefix_stats() const { return {hits_tokens_, query_tokens_}; }
  void reset_prefix_cache() {
    for (int b : lru_) {
      is_cached_[b] = 0;
      free_.push_back(b);
    }
    lru_.clear();
    lru_pos_.clear();
    index_.clear();
    for (int b = 0; b < num_blocks_; ++b) is_cached_[b] = 0;
  }

  // Consistency check used by tests: every block is exactly one of free / cached-idle /
  // referenced, and refcounts equal table occurrences.
  bool check_invariants() const {
    std::vector<int> occ(num_blocks_, 0);
    for (auto& kv : seqs_)
      for (int b : kv.second.blocks) occ[b]++;
    std::vector<int> state(num_blocks_, 0);
    for (int b : free_) state[b] |= 1;
    for (int b : lru_) state[b] |= 2;
    for (int b = 0; b < num_blocks_; ++b) {
      if (occ[b] != ref_[b]) return false;
      const bool idle = ref_[b] == 0;
      if (idle && !(state[b] == 1 || state[b] == 2)) return false;
      if (!idle && state[b] != 0) return false;
    }
    return true;
  }

 private:
  Sequence& get(int64_t sid) {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) throw std::runtime_error("unknown sequence " + std::to_string(sid));
    return it->second;
  }
  const Sequence& getc(int64_t sid) const {
    auto it = seqs_.find(sid);
    if (it == seqs_.end()) throw std::runtime_error("unknown sequence " + std::to_string(sid));
    return it->second;
  }

  int take_free() {
    if (free_.empty()) evict_one();
    if (free_.empty()) throw std::runtime_error("out of KV blocks");
    const int b = free_.back();
    free_.pop_back();
    ref_[b] = 1;
    return b;
  }

  void evict_one() {
    if (lru_.empty()) return;
    const int b = lru_.front();
    lru_.pop_front();
    lru_pos_.erase(b);
    if (is_cached_[b]) {
      index_.erase(cached_key_[b]);
      is_cached_[b] = 0;
    }
    free_.push_back(b);
  }

  void acquire(int b) {
    if (ref_[b] == 0) {
      auto it = lru_pos_.find(b);
      if (it != lru_pos_.end()) {
        lru_.erase(it->second);
        lru_pos_.erase(it);
      }
    }
    ref_[b]++;
  }

  void release(int b) {
    if (--ref_[b] == 0) {
      if (is_cached_[b]) {
        lru_.push_back(b);
        lru_pos_[b] = std::prev(lru_.end());
      } else {
        free_.push_back(b);
      }
    }
  }

  void maybe_publish(Sequence& s) {
    if (!prefix_ || s.no_publish) return;
    const int64_t full_known = std::min<int64_t>(s.num_tokens, s.tokens.size()) / block_size_;
    while (static_cast<int64_t>(s.hashes.size()) < full_known) {
      const int64_t bi = s.hashes.size();
      const uint64_t parent = bi == 0 ? 0 : s.hashes[bi - 1];
      const int32_t* tk = s.tokens.data() + bi * block_size_;
      const uint64_t h = hash_block(parent, tk, block_size_);
      s.hashes.push_back(h);
      const int b = s.blocks[bi];
      if (!index_.count(h) && !is_cached_[b]) {
        index_[h] = CachedBlock{b, parent, std::vector<int32_t>(tk, tk + block_size_)};
        cached_key_[b] = h;
        is_cached_[b] = 1;
      }
    }
  }

  int num_blocks_, block_size_;
  bool prefix_;
  std::vector<int> ref_;
  std::vector<uint64_t> cached_key_;
  std::vector<char> is_cached_;
  std::vector<int> free_;
  std::list<int> lru_;
  std::unordered_map<int, std::list<int>::iterator> lru_pos_;
  std::unordered_map<uint64_t, CachedBlock> index_;
  std::unordered_map<int64_t, Sequence> seqs_;
  int64_t hits_tokens_ = 0, query_tokens_ = 0;
};

}  // namespace lbn

void register_block_manager(py::module_& m) {
  using lbn::BlockManager;
  py::class_<BlockManager>(m, "BlockManager")
      .def(py::init<int, int, bool>(), py::arg("num_blocks"), py::arg("block_size"),
           py::arg("enable_prefix") = true)
      .def_property_readonly("num_blocks", &BlockManager::num_blocks)
      .def_property_readonly("block_size", &BlockManager::block_size)
      .def("num_free_blocks", &BlockManager::num_free_blocks)
      .def("num_cached_blocks", &BlockManager::num_cached_blocks)
      .def("usage", &BlockManager::usage)
      .def("has_seq", &BlockManager::has_seq)
      .def("blocks_needed", &BlockManager::blocks_needed)
      .def("can_allocate", &BlockManager::can_allocate)
      .def("can_allocate_all", &BlockManager::can_allocate_all)
      .def("add_sequence", &BlockManager::add_sequence)
      .def("match_prefix", &BlockManager::match_prefix)
      .def("append_slots", &BlockManager::append_slots, py::arg("sid"), py::arg("n"),
           py::arg("tokens") = std::vector<int32_t>())
      .def("set_tokens", &BlockManager::set_tokens)
      .def("fork", &BlockManager::fork)
      .def("truncate", &BlockManager::truncate)
      .def("set_blocks", &BlockManager::set_blocks)
      .def("alloc_blocks", &BlockManager::alloc_blocks)
      .def("free_blocks", &BlockManager::free_blocks)
      .def("free_sequence", &BlockManager::free_sequence)
      .def("block_table", &BlockManager::block_table)
      .def("num_tokens", &BlockManager::num_tokens)
      .def("fill_block_tables", &BlockManager::fill_block_tables)
      .def("refcount", &BlockManager::refcount)
      .def("prefix_stats", &BlockManager::prefix_stats)
      .def("reset_prefix_cache", &BlockManager::reset_prefix_cache)
      .def("check_invariants", &BlockManager::check_invariants);
  m.def("hash_block", [](uint64_t parent, const std::vector<int32_t>& toks) {
    return lbn::hash_block(parent, toks.data(), static_cast<int>(toks.size()));
  });
}
