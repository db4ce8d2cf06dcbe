// Shard directory: the host-side index and slot allocator of the G1 KV pool.
//
// The G1 pool of one node is split into one shard per GPU. Shard s owns a device
// slab of `n_slots` fixed-size chunk slots (a chunk holds one KV page of 16 tokens
// for every layer, K and V, in the pool's storage format). A prefix is owned by the
// shard `prefix_key % world`. This directory records, for every shard, which slots
// are free and which prefix occupies which slots, so that ANY local rank can look
// up, pin, allocate and commit entries of ANY shard without a device round trip or
// a message to the owner: the directory lives in POSIX shared memory mapped by all
// ranks of the node, each shard guarded by a robust process-shared mutex (a rank
// that dies while holding it does not wedge the others).
//
// Reference behaviour this covers: CompressedVRAMPool's prefix index, allocator and
// reuse-score eviction (korith_vllm_ext/compressed_vram_pool.py:142-206, :612-726),
// extended from one process/GPU to a node-wide sharded pool. Eviction keeps the
// reference score  a*age_s + b/hits + c*size_MB - d*avg_savings_ms  (a=.3 b=.4 c=.1
// d=.2, evict the maximum) but never evicts an entry that some rank has pinned for
// an in-flight restore. Slots of an entry form a chain (next_slot[]), so allocation
// never needs a contiguous run and the pool cannot fragment.
#pragma once

#include <pthread.h>

#include <cstdint>
#include <string>
#include <vector>

namespace axr {

constexpr int kMaxRanks = 32;

enum class EntryPhase : std::uint32_t { kEmpty = 0, kWriting = 1, kReady = 2, kTomb = 3 };

struct DirEntry {
  std::uint64_t key;        // primary prefix key (64-bit), 0 = empty
  std::uint64_t key2;       // independent check hash (guards against key collisions)
  std::uint32_t phase;      // EntryPhase
  std::uint32_t n_tokens;
  std::uint32_t n_chunks;
  std::int32_t first_slot;
  std::int32_t writer;      // rank that allocated it
  std::uint32_t fmt;        // storage format id of the chunks
  std::uint64_t created_ns;
  std::uint64_t last_hit_ns;
  std::uint64_t phase_ns;   // when the phase last changed
  std::uint64_t hit_count;
  std::uint64_t nbytes;
  double avg_savings_ms;
  std::uint16_t pins[kMaxRanks];  // per-rank pin counts (in-flight restores)
};

struct ShardStats {
  std::uint64_t hits, misses, inserts, evictions, bytes_stored, bytes_evicted;
  std::uint64_t busy, alloc_failures, reclaimed;
};

struct ShardInfo {
  std::uint32_t n_slots;
  std::uint32_t free_slots;
  std::uint64_t chunk_bytes;
  std::uint32_t entries;
  std::uint32_t entry_cap;
  ShardStats stats;
};

struct LookupOut {
  bool found = false;
  std::uint32_t n_tokens = 0;
  std::uint32_t fmt = 0;
  std::vector<std::int32_t> slots;
};

enum class InsertStatus : int { kOk = 0, kExists = 1, kBusy = 2, kNoSpace = 3, kTooLarge = 4 };

class ShardDirectory {
 public:
  // Create (or, with attach=true, open) the directory. An empty name keeps it in
  // process-private memory (single-process use).
  ShardDirectory(const std::string& name, int world, const std::vector<std::uint32_t>& n_slots,
                 std::uint64_t chunk_bytes, std::uint32_t entry_cap, bool attach,
                 double lock_timeout_s = 5.0);
  ~ShardDirectory();
  ShardDirectory(const ShardDirectory&) = delete;
  ShardDirectory& operator=(const ShardDirectory&) = delete;

  int world() const;
  std::uint64_t chunk_bytes(int shard) const;

  LookupOut lookup(int shard, std::uint64_t key, std::uint64_t key2, int pin_rank);
  bool contains(int shard, std::uint64_t key, std::uint64_t key2);
  void unpin(int shard, std::uint64_t key, int rank);
  InsertStatus begin_insert(int shard, std::uint64_t key, std::uint64_t key2,
                            std::uint32_t n_chunks, std::uint32_t n_tokens, std::uint32_t fmt,
                            int writer, double savings_ms, std::vector<std::int32_t>* slots,
                            std::vector<std::uint64_t>* evicted);
  bool commit(int shard, std::uint64_t key);
  bool abort(int shard, std::uint64_t key);
  bool remove(int shard, std::uint64_t key);
  void clear(int shard);
  // Drop every pin held by `rank` and abort the entries it was writing (a rank failed).
  std::uint32_t release_rank(int rank);
  // Abort WRITING entries whose phase is older than `max_age_s` (a writer vanished).
  std::uint32_t reclaim_stale(int shard, double max_age_s);
  ShardInfo info(int shard);
  std::vector<DirEntry> entries(int shard);
  void note_savings(int shard, std::uint64_t key, double savings_ms);
  // Distinct token lengths of READY entries (all shards), longest first.
  std::vector<std::uint32_t> lengths();

 private:
  struct Layout;
  struct Guard;
  void lock(int shard);
  void unlock(int shard);
  DirEntry* find_locked(int shard, std::uint64_t key, std::uint64_t key2);
  DirEntry* slot_for_insert_locked(int shard, std::uint64_t key);
  void free_chain_locked(int shard, DirEntry* e);
  bool evict_one_locked(int shard, std::vector<std::uint64_t>* evicted);
  void note_len(std::uint32_t n_tokens, int delta);
  double score_locked(const DirEntry& e, std::uint64_t now_ns, std::uint64_t chunk_bytes) const;

  std::string name_;
  bool owner_ = false;
  void* base_ = nullptr;
  std::size_t bytes_ = 0;
  double lock_timeout_s_ = 5.0;
  Layout* lay_ = nullptr;
};

std::uint64_t mono_ns();

}  // namespace axr
