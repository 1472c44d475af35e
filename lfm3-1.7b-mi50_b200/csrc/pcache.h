// Host-side prefix cache of the paged KV pool and the per-sequence block bookkeeping around it: the
// counterpart of internal/model/cache.go (the cache) and internal/model/generate.go:222-385 (reuse,
// ensureBlock, register / registerAt, release). Host code only: nothing here touches the GPU. The kernels
// read K/V through each sequence's logical -> physical block table, so a reused prefix is shared by
// pointing two tables at the same physical blocks; no KV byte moves.
//
// Full-attention blocks (32 tokens) are identified by a chain hash of the salt and every token up to and
// including the block (cache.go:137-154, FNV-1a 64 over the previous hash and the block's tokens, little
// endian), kept while a sequence references them and evicted least recently used once unreferenced
// (cache.go:48-101). Sliding-window blocks and conv-state checkpoints live in rings addressed by an ever
// increasing epoch: an entry is usable until the ring is about to overwrite it (cache.go:103-125).
#pragma once
#include <stdint.h>
#include <string.h>

#include <algorithm>
#include <unordered_map>
#include <vector>

namespace lfm3a {

// FNV-1a, 64-bit (the published offset basis and prime).
constexpr uint64_t kFnvOffset = 0xcbf29ce484222325ull;
constexpr uint64_t kFnvPrime = 0x100000001b3ull;
inline uint64_t fnv1a64(uint64_t h, const uint8_t* p, size_t n) {
  for (size_t i = 0; i < n; ++i) {
    h ^= p[i];
    h *= kFnvPrime;
  }
  return h;
}

// The chain's first link: FNV-1a of "prefix-v1" NUL then the salt's bytes (cache.go:138-143). Different
// salts give disjoint caches.
inline uint64_t prefix_salt_seed(const char* salt) {
  static const char tag[] = "prefix-v1";   // hashed with its terminating NUL: 10 bytes
  uint64_t h = fnv1a64(kFnvOffset, reinterpret_cast<const uint8_t*>(tag), sizeof(tag));
  return fnv1a64(h, reinterpret_cast<const uint8_t*>(salt), salt ? strlen(salt) : 0);
}

// Hash of one 32-token block given the hash of everything before it (cache.go:145-154): FNV-1a over the
// previous hash (8 bytes, little endian) followed by each token (4 bytes, little endian).
constexpr int kPrefixBlockTokens = 32;
inline uint64_t prefix_chain_hash(uint64_t prev, const int32_t* tokens) {
  uint8_t buf[8 + 4 * kPrefixBlockTokens];
  for (int i = 0; i < 8; ++i) buf[i] = (uint8_t)(prev >> (8 * i));
  for (int t = 0; t < kPrefixBlockTokens; ++t) {
    const uint32_t v = (uint32_t)tokens[t];
    for (int i = 0; i < 4; ++i) buf[8 + 4 * t + i] = (uint8_t)(v >> (8 * i));
  }
  return fnv1a64(kFnvOffset, buf, sizeof(buf));
}

// A cached full-attention block (cache.go:18-25).
struct PrefixEntry {
  uint64_t hash = 0;
  int32_t full = 0;
  int64_t slide_epoch = -1;   // ring epoch of the block's sliding-window copy, -1 if none
  int64_t conv_epoch = -1;    // ring epoch of the conv checkpoint taken at the block's end, -1 if none
  int refs = 0;
  PrefixEntry* newer = nullptr;   // LRU links while unreferenced
  PrefixEntry* older = nullptr;
  bool indexed = true;            // still reachable through the hash index (false after reset)
};

class PrefixPool {
 public:
  // A reused sliding block must stay out of the ring's overwrite path for as long as it can sit inside
  // the attention window of the sequence reusing it (cache.go:12-16).
  static constexpr int64_t kSlideReuseMargin = 128;

  PrefixPool(int full_blocks, int slide_blocks, int conv_slots)
      : slide_blocks_(slide_blocks), conv_slots_(conv_slots - 1) {
    free_.reserve(full_blocks);
    for (int b = full_blocks - 1; b >= 0; --b) free_.push_back(b);   // block 0 is handed out first
  }
  ~PrefixPool() {
    for (auto& kv : index_) delete kv.second;
    for (PrefixEntry* e : orphans_) delete e;
  }
  PrefixPool(const PrefixPool&) = delete;
  PrefixPool& operator=(const PrefixPool&) = delete;

  // A free full block, else the least recently used unreferenced cached one (dropped from the index).
  bool alloc_full(int32_t* block) {
    if (!free_.empty()) {
      *block = free_.back();
      free_.pop_back();
      return true;
    }
    PrefixEntry* v = coldest_;
    if (!v) return false;
    unlink(v);
    *block = v->full;
    drop(v);
    return true;
  }
  void pin(PrefixEntry* e) {
    if (e->refs == 0) unlink(e);
    ++e->refs;
  }
  void unpin(PrefixEntry* e) {
    if (--e->refs == 0) push_warm(e);
  }
  void give_back(int32_t block) { free_.push_back(block); }

  // Ring slots: slot = epoch mod ring size (the conv ring skips slot 0, which holds the running state).
  int32_t alloc_slide(int64_t* epoch) {
    *epoch = slide_next_++;
    return (int32_t)(*epoch % slide_blocks_);
  }
  bool slide_valid(int64_t ep) const { return ep >= 0 && slide_next_ - ep < slide_blocks_ - kSlideReuseMargin; }
  int32_t alloc_conv(int64_t* epoch) {
    *epoch = conv_next_++;
    return conv_slot_of(*epoch);
  }
  bool conv_valid(int64_t ep) const { return ep >= 0 && conv_next_ - ep < conv_slots_; }
  int32_t conv_slot_of(int64_t ep) const { return (int32_t)(ep % conv_slots_) + 1; }
  int64_t slide_blocks() const { return slide_blocks_; }

  PrefixEntry* find(uint64_t h) const {
    auto it = index_.find(h);
    return it == index_.end() ? nullptr : it->second;
  }
  // A new referenced entry in the index.
  PrefixEntry* insert(uint64_t h, int32_t full, int64_t slide_epoch) {
    PrefixEntry* e = new PrefixEntry;
    e->hash = h;
    e->full = full;
    e->slide_epoch = slide_epoch;
    e->refs = 1;
    index_[h] = e;
    return e;
  }

  // Forgets every cached prefix (cache.go:127-136): unreferenced blocks return to the free list; blocks a
  // live sequence still references stay with it and re-enter the LRU order when it lets go of them.
  // The reference appends the freed blocks in Go map order, which is unspecified; here they are appended
  // highest first, so the lowest-numbered freed block is handed out first, as from a new pool.
  void reset() {
    std::vector<int32_t> freed;
    for (auto& kv : index_) {
      PrefixEntry* e = kv.second;
      e->indexed = false;
      if (e->refs == 0) {
        freed.push_back(e->full);
        delete e;
      } else {
        orphans_.push_back(e);
      }
    }
    std::sort(freed.begin(), freed.end(), [](int32_t x, int32_t y) { return x > y; });
    free_.insert(free_.end(), freed.begin(), freed.end());
    index_.clear();
    warmest_ = coldest_ = nullptr;
  }

  int free_blocks() const { return (int)free_.size(); }
  int cached_entries() const { return (int)index_.size(); }

 private:
  void unlink(PrefixEntry* e) {
    if (e->newer) e->newer->older = e->older;
    else if (warmest_ == e) warmest_ = e->older;
    if (e->older) e->older->newer = e->newer;
    else if (coldest_ == e) coldest_ = e->newer;
    e->newer = e->older = nullptr;
  }
  void push_warm(PrefixEntry* e) {
    e->newer = nullptr;
    e->older = warmest_;
    if (warmest_) warmest_->newer = e;
    warmest_ = e;
    if (!coldest_) coldest_ = e;
  }
  // An evicted entry leaves the index (or the orphan list) and is freed: nothing references it.
  void drop(PrefixEntry* e) {
    if (e->indexed) {
      index_.erase(e->hash);
    } else {
      for (size_t i = 0; i < orphans_.size(); ++i)
        if (orphans_[i] == e) {
          orphans_[i] = orphans_.back();
          orphans_.pop_back();
          break;
        }
    }
    delete e;
  }

  std::unordered_map<uint64_t, PrefixEntry*> index_;
  std::vector<PrefixEntry*> orphans_;   // referenced entries dropped from the index by reset()
  std::vector<int32_t> free_;
  PrefixEntry* warmest_ = nullptr;      // most recently released
  PrefixEntry* coldest_ = nullptr;      // next to evict
  int64_t slide_blocks_, slide_next_ = 0;
  int64_t conv_slots_, conv_next_ = 0;  // checkpoint slots, excluding the running slot 0
};

// One sequence's blocks (generate.go:50-61): its chain hash so far, the cache entries it references,
// logical -> physical full and sliding blocks, and full blocks it owns privately.
struct PrefixSeq {
  uint64_t hash = 0;
  int registered = 0;   // complete blocks handed to the cache
  std::vector<PrefixEntry*> entries;
  std::vector<int32_t> priv;   // full blocks whose content is also cached under another block
  std::vector<int32_t> full, slide;
  std::vector<int64_t> slide_epoch;
  bool released = false;
};

// The longest usable cached prefix of `prompt` (generate.go:222-279): whole blocks only, at least one
// prompt token left to compute, the last reused block's conv checkpoint still in its ring, and every
// sliding block inside the attention window (window tokens) of the next token still in its ring. Maps
// the blocks into the sequence, pins them, and returns the reused tokens; *conv_slot is the checkpoint
// slot the caller restores into the running conv state (0 and no reuse when nothing qualifies).
// align: the reused block count is a multiple of it. MODE_F16 keeps an int8 copy of V per 64-token
// block, two pages: reusing an odd number of pages would let the reusing sequence's first append rewrite
// the int8 V of a shared page, so its callers pass 2 (the reference's per-token records need 1).
inline int prefix_reuse(PrefixPool& c, PrefixSeq& s, const int32_t* prompt, int n, int window, int align,
                        int32_t* conv_slot) {
  *conv_slot = 0;
  const int limit = n > 0 ? (n - 1) / kPrefixBlockTokens : 0;
  std::vector<PrefixEntry*> chain;
  uint64_t h = s.hash;
  for (int i = 0; i < limit; ++i) {
    h = prefix_chain_hash(h, prompt + i * kPrefixBlockTokens);
    PrefixEntry* e = c.find(h);
    if (!e) break;
    chain.push_back(e);
  }
  int hit = 0;
  for (int k = (int)chain.size(); k > 0; --k) {
    if (k % align != 0 || !c.conv_valid(chain[k - 1]->conv_epoch)) continue;
    const int first = k * kPrefixBlockTokens - window + 1 > 0 ? k * kPrefixBlockTokens - window + 1 : 0;
    bool ok = true;
    for (int b = first / kPrefixBlockTokens; b < k && ok; ++b) ok = c.slide_valid(chain[b]->slide_epoch);
    if (ok) {
      hit = k;
      break;
    }
  }
  for (int i = 0; i < hit; ++i) {
    PrefixEntry* e = chain[i];
    c.pin(e);
    s.entries.push_back(e);
    s.full.push_back(e->full);
    s.slide.push_back(e->slide_epoch >= 0 ? (int32_t)(e->slide_epoch % c.slide_blocks()) : 0);
    s.slide_epoch.push_back(e->slide_epoch);
    s.hash = e->hash;
  }
  if (hit > 0) {
    s.registered = hit;
    *conv_slot = c.conv_slot_of(chain[hit - 1]->conv_epoch);
  }
  return hit * kPrefixBlockTokens;
}

// Physical blocks for logical blocks up to `logical` (generate.go:281-295); false when the pool is
// exhausted (every full block referenced).
inline bool prefix_ensure(PrefixPool& c, PrefixSeq& s, int logical) {
  while ((int)s.full.size() <= logical) {
    int32_t f;
    if (!c.alloc_full(&f)) return false;
    int64_t ep;
    const int32_t sl = c.alloc_slide(&ep);
    s.full.push_back(f);
    s.slide.push_back(sl);
    s.slide_epoch.push_back(ep);
  }
  return true;
}

// Hands every newly complete block up to token `upto` to the cache (generate.go:346-373); the last of
// them owns the conv checkpoint `conv_epoch`. A block already cached under other physical pages keeps
// this sequence's pages (which become private) and takes this sequence's fresher sliding epoch.
// tokens: the sequence's tokens, at least `upto` of them. Blocks must have been ensured.
inline bool prefix_register(PrefixPool& c, PrefixSeq& s, const int32_t* tokens, int upto, int64_t conv_epoch) {
  const int n = upto / kPrefixBlockTokens;
  if (n > (int)s.full.size()) return false;
  for (int i = s.registered; i < n; ++i) {
    s.hash = prefix_chain_hash(s.hash, tokens + i * kPrefixBlockTokens);
    PrefixEntry* e = c.find(s.hash);
    if (e) {
      c.pin(e);
      if (e->full != s.full[i]) s.priv.push_back(s.full[i]);
      e->slide_epoch = s.slide_epoch[i];
    } else {
      e = c.insert(s.hash, s.full[i], s.slide_epoch[i]);
    }
    s.entries.push_back(e);
    if (i == n - 1) e->conv_epoch = conv_epoch;
  }
  if (n > s.registered) s.registered = n;
  return true;
}

// Returns the sequence's blocks (generate.go:376-385): cached ones become evictable once unreferenced;
// private blocks and an unregistered tail go back to the free list.
inline void prefix_release(PrefixPool& c, PrefixSeq& s) {
  if (s.released) return;
  for (PrefixEntry* e : s.entries) c.unpin(e);
  for (int32_t b : s.priv) c.give_back(b);
  for (size_t i = (size_t)s.registered; i < s.full.size(); ++i) c.give_back(s.full[i]);
  s.released = true;
}

}  // namespace lfm3a
