// Host-side block manager of the paged KV cache: slots, block tables, refcounts and
// the content-keyed prefix cache. C++ restatement of the bookkeeping half of
// PagedKVCache (engine/kv_cache.py:411-560) with identical results:
//
//  * free pool: least recently freed block first (engine/kv_cache.py:468-475);
//    a released block that holds a prefix key goes to the tail, one without a key
//    to the head (:482-488); sharing a free cached block takes it out of the pool (:477-480).
//  * prefix keys: block i of a prompt is keyed by (key of block i-1, its tokens)
//    (:490-497). The reference nests Python's hash() of the parent key; here the
//    parent is a 128-bit chain hash, so two keys agree exactly when the reference's
//    do, short of a hash collision in either.
//  * matching takes at most (len - 1) / block_size leading full blocks (:499-508).
//  * slot ids: lowest first, a freed id is the next one handed out (:431, :560).
//
// The free pool is an intrusive doubly linked list over block ids (O(1) for
// every operation above) and the key index is a hash map from key to block.
#include <algorithm>
#include <cstdint>
#include <cstring>
#include <new>
#include <unordered_map>
#include <vector>

#include "../../include/pkv.h"

namespace {

struct Hash128 {
  uint64_t lo = 0, hi = 0;
  bool operator==(const Hash128& o) const { return lo == o.lo && hi == o.hi; }
};

// SplitMix64 finaliser (Steele, Lea, Flood: "Fast splittable pseudorandom number
// generators", 2014) as the mixing step of a two-lane chain hash.
inline uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
  return z ^ (z >> 31);
}

Hash128 chain_hash(const Hash128& parent, bool has_parent, const int64_t* toks, int64_t n) {
  uint64_t a = 0x243f6a8885a308d3ULL ^ (has_parent ? mix64(parent.lo) : 0x13198a2e03707344ULL);
  uint64_t b = 0xa4093822299f31d0ULL ^ (has_parent ? mix64(parent.hi + 0x082efa98ec4e6c89ULL) : 0x452821e638d01377ULL);
  a = mix64(a ^ static_cast<uint64_t>(n));
  b = mix64(b + static_cast<uint64_t>(n) * 0x9e3779b97f4a7c15ULL);
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t t = static_cast<uint64_t>(toks[i]);
    a = mix64(a ^ (t + 0x9e3779b97f4a7c15ULL * static_cast<uint64_t>(i + 1)));
    b = mix64(b + (t ^ 0xc2b2ae3d27d4eb4fULL) * 0x165667b19e3779f9ULL);
  }
  return Hash128{a, b};
}

// Key of one block: (parent key, this block's tokens). The parent enters by its
// chain hash; has_parent distinguishes the first block (parent None).
struct BlockKey {
  Hash128 parent;
  bool has_parent = false;
  std::vector<int64_t> tokens;
  Hash128 self;  // chain hash of this key (what the next block's key holds as its parent)
  bool operator==(const BlockKey& o) const {
    return has_parent == o.has_parent && parent == o.parent && tokens == o.tokens;
  }
};

struct BlockKeyHash {
  size_t operator()(const BlockKey& k) const { return static_cast<size_t>(k.self.lo ^ (k.self.hi * 31)); }
};

// Iterates the keys of the first `count` blocks of a token sequence.
class KeyChain {
 public:
  KeyChain(const int64_t* toks, int64_t n, int32_t bs) : toks_(toks), n_(n), bs_(bs) {}
  BlockKey next() {
    BlockKey k;
    k.has_parent = has_prev_;
    k.parent = prev_;
    const int64_t a = std::min<int64_t>(static_cast<int64_t>(i_) * bs_, n_);
    const int64_t b = std::min<int64_t>(static_cast<int64_t>(i_ + 1) * bs_, n_);
    k.tokens.assign(toks_ + a, toks_ + b);
    k.self = chain_hash(k.parent, k.has_parent, k.tokens.data(), static_cast<int64_t>(k.tokens.size()));
    prev_ = k.self;
    has_prev_ = true;
    ++i_;
    return k;
  }

 private:
  const int64_t* toks_;
  int64_t n_;
  int32_t bs_;
  int32_t i_ = 0;
  Hash128 prev_;
  bool has_prev_ = false;
};

}  // namespace

struct pkv_block_manager {
  int32_t num_blocks, block_size, max_seqs, max_len;
  bool prefix_caching;
  // free pool as a linked list over block ids
  std::vector<int32_t> prev, next;
  std::vector<uint8_t> in_pool;
  int32_t head = -1, tail = -1, pool_size = 0;
  std::vector<int32_t> refs;
  // slots
  std::vector<int32_t> slot_stack;  // top = back
  std::vector<uint8_t> live;
  std::vector<std::vector<int32_t>> tables;
  std::vector<int64_t> lengths;
  // prefix cache
  std::vector<int32_t> key_slot;  // block -> index into keys, -1 if uncached
  std::vector<BlockKey> keys;     // storage; freed entries recycled via free_keys
  std::vector<int32_t> free_keys;
  std::unordered_map<BlockKey, int32_t, BlockKeyHash> index;
  int64_t prefix_hit_tokens = 0;
  // journal of table edits for a device mirror
  bool journal_on = false;
  bool journal_overflow = false;
  std::vector<int32_t> journal;

  static constexpr size_t kJournalCap = size_t(1) << 22;  // triples

  void push_back(int32_t b) {
    prev[b] = tail;
    next[b] = -1;
    if (tail >= 0) next[tail] = b; else head = b;
    tail = b;
    in_pool[b] = 1;
    ++pool_size;
  }
  void push_front(int32_t b) {
    prev[b] = -1;
    next[b] = head;
    if (head >= 0) prev[head] = b; else tail = b;
    head = b;
    in_pool[b] = 1;
    ++pool_size;
  }
  void unlink(int32_t b) {
    const int32_t p = prev[b], n = next[b];
    if (p >= 0) next[p] = n; else head = n;
    if (n >= 0) prev[n] = p; else tail = p;
    in_pool[b] = 0;
    --pool_size;
  }
  int64_t blocks_for(int64_t n) const { return (n + block_size - 1) / block_size; }
  bool can_allocate(int64_t n) const {
    return !slot_stack.empty() && n <= max_len && blocks_for(n) <= pool_size;
  }
  void record(int32_t slot, int32_t col, int32_t block) {
    if (!journal_on) return;
    if (journal.size() / 3 >= kJournalCap) { journal_overflow = true; return; }
    journal.push_back(slot);
    journal.push_back(col);
    journal.push_back(block);
  }
  void forget_key(int32_t b) {
    const int32_t ks = key_slot[b];
    if (ks < 0) return;
    index.erase(keys[ks]);
    keys[ks] = BlockKey();
    free_keys.push_back(ks);
    key_slot[b] = -1;
  }
  int32_t take_fresh() {  // engine/kv_cache.py:468-475
    const int32_t b = head;
    unlink(b);
    forget_key(b);
    refs[b] = 1;
    return b;
  }
  void add_ref(int32_t b) {  // engine/kv_cache.py:477-480
    if (refs[b] == 0) unlink(b);
    ++refs[b];
  }
  void drop_ref(int32_t b) {  // engine/kv_cache.py:482-488
    if (--refs[b] == 0) {
      if (key_slot[b] >= 0) push_back(b); else push_front(b);
    }
  }
  void set_key(int32_t b, BlockKey&& k) {
    int32_t ks;
    if (!free_keys.empty()) { ks = free_keys.back(); free_keys.pop_back(); keys[ks] = std::move(k); }
    else { ks = static_cast<int32_t>(keys.size()); keys.push_back(std::move(k)); }
    key_slot[b] = ks;
    index.emplace(keys[ks], b);
  }
  bool valid_slot(int32_t s) const { return s >= 0 && s < max_seqs && live[s]; }
};

extern "C" {

int pkv_bm_create(int32_t num_blocks, int32_t block_size, int32_t max_seqs, int32_t max_len,
                  int32_t enable_prefix_caching, pkv_block_manager** out) {
  if (!out || num_blocks < 0 || block_size <= 0 || max_seqs < 0) return PKV_ERR_INVALID_ARGUMENT;
  pkv_block_manager* bm = new (std::nothrow) pkv_block_manager();
  if (!bm) return PKV_ERR_INVALID_ARGUMENT;
  bm->num_blocks = num_blocks;
  bm->block_size = block_size;
  bm->max_seqs = max_seqs;
  bm->max_len = max_len;
  bm->prefix_caching = enable_prefix_caching != 0;
  bm->prev.assign(num_blocks, -1);
  bm->next.assign(num_blocks, -1);
  bm->in_pool.assign(num_blocks, 0);
  for (int32_t b = 0; b < num_blocks; ++b) bm->push_back(b);
  bm->refs.assign(num_blocks, 0);
  bm->key_slot.assign(num_blocks, -1);
  for (int32_t s = max_seqs - 1; s >= 0; --s) bm->slot_stack.push_back(s);
  bm->live.assign(max_seqs, 0);
  bm->tables.assign(max_seqs, {});
  bm->lengths.assign(max_seqs, 0);
  *out = bm;
  return PKV_OK;
}

void pkv_bm_destroy(pkv_block_manager* bm) { delete bm; }

int pkv_bm_can_allocate(const pkv_block_manager* bm, int64_t num_tokens, int32_t* out) {
  if (!bm || !out) return PKV_ERR_INVALID_ARGUMENT;
  *out = bm->can_allocate(num_tokens) ? 1 : 0;
  return PKV_OK;
}

int pkv_bm_allocate(pkv_block_manager* bm, int64_t num_tokens, const int64_t* token_ids, int64_t n_ids,
                    int32_t* out_slot) {
  if (!bm || !out_slot) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->can_allocate(num_tokens)) return PKV_ERR_NO_BLOCKS;
  std::vector<int32_t> shared;
  if (bm->prefix_caching && token_ids && n_ids > 0) {  // engine/kv_cache.py:499-508
    const int64_t usable = (n_ids - 1) / bm->block_size;
    KeyChain chain(token_ids, n_ids, bm->block_size);
    for (int64_t i = 0; i < usable; ++i) {
      auto it = bm->index.find(chain.next());
      if (it == bm->index.end()) break;
      shared.push_back(it->second);
    }
  }
  for (int32_t b : shared) bm->add_ref(b);
  const int32_t slot = bm->slot_stack.back();
  bm->slot_stack.pop_back();
  std::vector<int32_t>& table = bm->tables[slot];
  table = shared;
  const int64_t fresh = std::max<int64_t>(0, bm->blocks_for(num_tokens) - static_cast<int64_t>(shared.size()));
  for (int64_t i = 0; i < fresh; ++i) table.push_back(bm->take_fresh());
  for (size_t i = 0; i < table.size(); ++i) bm->record(slot, static_cast<int32_t>(i), table[i]);
  bm->live[slot] = 1;
  bm->lengths[slot] = static_cast<int64_t>(shared.size()) * bm->block_size;
  bm->prefix_hit_tokens += bm->lengths[slot];
  *out_slot = slot;
  return PKV_OK;
}

int pkv_bm_register_prefix(pkv_block_manager* bm, int32_t slot, const int64_t* token_ids, int64_t n_ids) {
  if (!bm) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->prefix_caching) return PKV_OK;  // engine/kv_cache.py:533-534
  if (!bm->valid_slot(slot)) return PKV_ERR_UNKNOWN_SLOT;
  if (n_ids > 0 && !token_ids) return PKV_ERR_INVALID_ARGUMENT;
  const std::vector<int32_t>& table = bm->tables[slot];
  const int64_t full = bm->lengths[slot] / bm->block_size;
  KeyChain chain(token_ids, n_ids, bm->block_size);
  for (int64_t i = 0; i < full; ++i) {
    BlockKey k = chain.next();
    if (i >= static_cast<int64_t>(table.size())) return PKV_ERR_OUT_OF_RANGE;  // the reference's IndexError
    const int32_t b = table[i];
    if (bm->index.find(k) == bm->index.end() && bm->key_slot[b] < 0) bm->set_key(b, std::move(k));
  }
  return PKV_OK;
}

int pkv_bm_ensure_capacity(pkv_block_manager* bm, int32_t slot, int64_t num_tokens, int32_t* out) {
  if (!bm || !out) return PKV_ERR_INVALID_ARGUMENT;
  if (num_tokens > bm->max_len) { *out = 0; return PKV_OK; }  // checked before the table lookup, as :545-546
  if (!bm->valid_slot(slot)) return PKV_ERR_UNKNOWN_SLOT;
  std::vector<int32_t>& table = bm->tables[slot];
  const int64_t missing = bm->blocks_for(num_tokens) - static_cast<int64_t>(table.size());
  if (missing > bm->pool_size) { *out = 0; return PKV_OK; }
  for (int64_t i = 0; i < missing; ++i) {
    table.push_back(bm->take_fresh());
    bm->record(slot, static_cast<int32_t>(table.size() - 1), table.back());
  }
  *out = 1;
  return PKV_OK;
}

int pkv_bm_free(pkv_block_manager* bm, int32_t slot) {
  if (!bm) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->valid_slot(slot)) return PKV_ERR_DOUBLE_FREE;
  std::vector<int32_t>& table = bm->tables[slot];
  for (auto it = table.rbegin(); it != table.rend(); ++it) bm->drop_ref(*it);
  table.clear();
  bm->live[slot] = 0;
  bm->lengths[slot] = 0;
  bm->slot_stack.push_back(slot);
  return PKV_OK;
}

int pkv_bm_fork(pkv_block_manager* bm, int32_t src_slot, int32_t* out_slot) {
  if (!bm || !out_slot) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->valid_slot(src_slot)) return PKV_ERR_UNKNOWN_SLOT;
  if (bm->slot_stack.empty()) return PKV_ERR_NO_BLOCKS;
  const int32_t slot = bm->slot_stack.back();
  bm->slot_stack.pop_back();
  std::vector<int32_t>& table = bm->tables[slot];
  table = bm->tables[src_slot];  // every block shared, a partially filled last one included
  for (size_t i = 0; i < table.size(); ++i) {
    bm->add_ref(table[i]);
    bm->record(slot, static_cast<int32_t>(i), table[i]);
  }
  bm->live[slot] = 1;
  bm->lengths[slot] = bm->lengths[src_slot];
  *out_slot = slot;
  return PKV_OK;
}

int pkv_bm_prepare_write(pkv_block_manager* bm, int32_t slot, int64_t first_pos, int64_t n_tokens, int32_t* pairs,
                         int32_t cap_pairs, int32_t* n_pairs) {
  if (!bm || !n_pairs || n_tokens < 0 || first_pos < 0 || (cap_pairs > 0 && !pairs)) return PKV_ERR_INVALID_ARGUMENT;
  *n_pairs = 0;
  if (!bm->valid_slot(slot)) return PKV_ERR_UNKNOWN_SLOT;
  if (n_tokens == 0) return PKV_OK;
  std::vector<int32_t>& table = bm->tables[slot];
  const int64_t b0 = first_pos / bm->block_size, b1 = (first_pos + n_tokens - 1) / bm->block_size;
  if (b1 >= static_cast<int64_t>(table.size())) return PKV_ERR_OUT_OF_RANGE;
  int32_t shared = 0;
  for (int64_t i = b0; i <= b1; ++i) shared += bm->refs[table[i]] > 1;
  if (shared > cap_pairs) return PKV_ERR_WORKSPACE;
  if (shared > bm->pool_size) return PKV_ERR_NO_BLOCKS;  // nothing changed
  for (int64_t i = b0; i <= b1; ++i) {
    const int32_t old = table[i];
    if (bm->refs[old] <= 1) continue;
    const int32_t fresh = bm->take_fresh();
    table[i] = fresh;
    bm->drop_ref(old);  // still held by the sequences it is shared with
    bm->record(slot, static_cast<int32_t>(i), fresh);
    pairs[2 * *n_pairs] = old;
    pairs[2 * *n_pairs + 1] = fresh;
    ++*n_pairs;
  }
  return PKV_OK;
}

int pkv_bm_decode_positions(const pkv_block_manager* bm, const int32_t* slots, int32_t n, int32_t* out) {
  if (!bm || n < 0 || (n > 0 && (!slots || !out))) return PKV_ERR_INVALID_ARGUMENT;
  for (int32_t i = 0; i < n; ++i) {
    const int32_t s = slots[i];
    if (!bm->valid_slot(s)) return PKV_ERR_UNKNOWN_SLOT;
    const int64_t p = bm->lengths[s];
    if (p < 0 || p / bm->block_size >= static_cast<int64_t>(bm->tables[s].size())) return PKV_ERR_OUT_OF_RANGE;
    out[i] = static_cast<int32_t>(p);
  }
  return PKV_OK;
}

int pkv_bm_commit_decode(pkv_block_manager* bm, const int32_t* slots, int32_t n) {
  if (!bm || n < 0 || (n > 0 && !slots)) return PKV_ERR_INVALID_ARGUMENT;
  for (int32_t i = 0; i < n; ++i)
    if (!bm->valid_slot(slots[i])) return PKV_ERR_UNKNOWN_SLOT;
  for (int32_t i = 0; i < n; ++i) ++bm->lengths[slots[i]];
  return PKV_OK;
}

int pkv_bm_get_length(const pkv_block_manager* bm, int32_t slot, int64_t* out) {
  if (!bm || !out) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->valid_slot(slot)) return PKV_ERR_UNKNOWN_SLOT;
  *out = bm->lengths[slot];
  return PKV_OK;
}

int pkv_bm_set_length(pkv_block_manager* bm, int32_t slot, int64_t value) {
  if (!bm) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->valid_slot(slot)) return PKV_ERR_UNKNOWN_SLOT;
  bm->lengths[slot] = value;
  return PKV_OK;
}

int pkv_bm_get_table(const pkv_block_manager* bm, int32_t slot, int32_t* out, int32_t cap, int32_t* out_len) {
  if (!bm || !out_len || (cap > 0 && !out)) return PKV_ERR_INVALID_ARGUMENT;
  if (!bm->valid_slot(slot)) return PKV_ERR_UNKNOWN_SLOT;
  const std::vector<int32_t>& t = bm->tables[slot];
  *out_len = static_cast<int32_t>(t.size());
  const int32_t n = std::min<int32_t>(cap, static_cast<int32_t>(t.size()));
  if (n > 0) std::memcpy(out, t.data(), sizeof(int32_t) * n);
  return PKV_OK;
}

int pkv_bm_live_slots(const pkv_block_manager* bm, int32_t* out, int32_t cap, int32_t* out_len) {
  if (!bm || !out_len || (cap > 0 && !out)) return PKV_ERR_INVALID_ARGUMENT;
  int32_t n = 0;
  for (int32_t s = 0; s < bm->max_seqs; ++s) {
    if (!bm->live[s]) continue;
    if (n < cap) out[n] = s;
    ++n;
  }
  *out_len = n;
  return PKV_OK;
}

int pkv_bm_num_free_blocks(const pkv_block_manager* bm, int32_t* out) {
  if (!bm || !out) return PKV_ERR_INVALID_ARGUMENT;
  *out = bm->pool_size;
  return PKV_OK;
}

int pkv_bm_num_free_slots(const pkv_block_manager* bm, int32_t* out) {
  if (!bm || !out) return PKV_ERR_INVALID_ARGUMENT;
  *out = static_cast<int32_t>(bm->slot_stack.size());
  return PKV_OK;
}

int pkv_bm_prefix_hit_tokens(const pkv_block_manager* bm, int64_t* out) {
  if (!bm || !out) return PKV_ERR_INVALID_ARGUMENT;
  *out = bm->prefix_hit_tokens;
  return PKV_OK;
}

int pkv_bm_free_order(const pkv_block_manager* bm, int32_t* out, int32_t cap, int32_t* out_len) {
  if (!bm || !out_len || (cap > 0 && !out)) return PKV_ERR_INVALID_ARGUMENT;
  int32_t n = 0;
  for (int32_t b = bm->head; b >= 0; b = bm->next[b]) {
    if (n < cap) out[n] = b;
    ++n;
  }
  *out_len = n;
  return PKV_OK;
}

int pkv_bm_ref_counts(const pkv_block_manager* bm, int32_t* out, int32_t cap) {
  if (!bm || (cap > 0 && !out)) return PKV_ERR_INVALID_ARGUMENT;
  const int32_t n = std::min(cap, bm->num_blocks);
  if (n > 0) std::memcpy(out, bm->refs.data(), sizeof(int32_t) * n);
  return PKV_OK;
}

int pkv_bm_cached_blocks(const pkv_block_manager* bm, int32_t* out, int32_t cap, int32_t* out_len) {
  if (!bm || !out_len || (cap > 0 && !out)) return PKV_ERR_INVALID_ARGUMENT;
  int32_t n = 0;
  for (int32_t b = 0; b < bm->num_blocks; ++b) {
    if (bm->key_slot[b] < 0) continue;
    if (n < cap) out[n] = b;
    ++n;
  }
  *out_len = n;
  return PKV_OK;
}

int pkv_bm_set_journal(pkv_block_manager* bm, int32_t enable) {
  if (!bm) return PKV_ERR_INVALID_ARGUMENT;
  bm->journal_on = enable != 0;
  if (!bm->journal_on) {
    bm->journal.clear();
    bm->journal_overflow = false;
  }
  return PKV_OK;
}

int pkv_bm_drain_table_edits(pkv_block_manager* bm, int32_t* out, int32_t cap_triples, int32_t* out_len,
                             int32_t* overflow) {
  if (!bm || !out_len || !overflow || (cap_triples > 0 && !out)) return PKV_ERR_INVALID_ARGUMENT;
  const int32_t have = static_cast<int32_t>(bm->journal.size() / 3);
  const int32_t n = std::min(have, cap_triples);
  if (n > 0) std::memcpy(out, bm->journal.data(), sizeof(int32_t) * 3 * static_cast<size_t>(n));
  *out_len = n;
  *overflow = (bm->journal_overflow || have > cap_triples) ? 1 : 0;
  bm->journal.clear();
  bm->journal_overflow = false;
  return PKV_OK;
}

}  // extern "C"
