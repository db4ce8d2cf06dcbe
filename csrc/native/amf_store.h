// Persistent AMF disk store: the on-disk checkpoint tier of the framework.
//
// Behaviour parity with the reference AmfStore (core/amf_store.h:163-239,
// core/amf_store.cpp): keyed by the 9-field AmfKey, index file amf_index.bin
// (magic "AMF1", version 9, version 8 readable), entry files <basename>.kv/.tok,
// longest-prefix lookup verified against the .tok file, admission with disk guard
// and ROI gate, watermark eviction cold -> warm -> hot (hot only above the 0.98
// critical watermark) under an lru/lfu/roi policy, adaptive TTL, async prewarm.
//
// Implementation is new: entries live in a dense vector with O(1) swap-erase,
// lookups probe only the prefix lengths that exist in the index (instead of every
// length from n down to min_tokens), all public methods are mutex-protected so the
// store can be shared by the engine thread and server threads, and the index is
// serialised field by field in little-endian order (the byte layout is the format
// contract, not a C struct).
#pragma once

#include <atomic>
#include <cmath>
#include <cstdint>
#include <limits>
#include <map>
#include <mutex>
#include <string>
#include <thread>
#include <unordered_map>
#include <unordered_set>
#include <vector>

namespace axr {

struct AmfKey {
  std::uint64_t model_hash = 0;
  std::uint64_t tenant_hash = 0;
  std::uint64_t prefix_hash = 0;
  std::uint32_t n_ctx = 0;
  std::uint32_t kv_version = 0;
  std::uint32_t rope_base_bits = 0;
  std::uint32_t rope_scale_bits = 0;
  std::uint64_t sampling_hash = 0;
  std::uint64_t rng_hash = 0;
  bool operator==(const AmfKey& o) const {
    return model_hash == o.model_hash && tenant_hash == o.tenant_hash &&
           prefix_hash == o.prefix_hash && n_ctx == o.n_ctx && kv_version == o.kv_version &&
           rope_base_bits == o.rope_base_bits && rope_scale_bits == o.rope_scale_bits &&
           sampling_hash == o.sampling_hash && rng_hash == o.rng_hash;
  }
};

struct AmfKeyHasher {
  std::size_t operator()(const AmfKey& k) const noexcept;
};

// Everything in a key except the prefix hash.
struct AmfContext {
  std::uint64_t model_hash = 0;
  std::uint64_t tenant_hash = 0;
  std::uint32_t n_ctx = 0;
  std::uint32_t kv_version = 0;
  std::uint32_t rope_base_bits = 0;
  std::uint32_t rope_scale_bits = 0;
  std::uint64_t sampling_hash = 0;
  std::uint64_t rng_hash = 0;
  AmfKey key_for(std::uint64_t prefix_hash) const {
    AmfKey k;
    k.model_hash = model_hash;
    k.tenant_hash = tenant_hash;
    k.prefix_hash = prefix_hash;
    k.n_ctx = n_ctx;
    k.kv_version = kv_version;
    k.rope_base_bits = rope_base_bits;
    k.rope_scale_bits = rope_scale_bits;
    k.sampling_hash = sampling_hash;
    k.rng_hash = rng_hash;
    return k;
  }
};

constexpr double kNaN = std::numeric_limits<double>::quiet_NaN();

struct AmfEntry {
  AmfKey key{};
  std::uint64_t model_hash = 0;
  std::uint32_t prefix_len = 0;
  std::uint64_t seen_count = 0;
  std::uint64_t restore_count = 0;
  double ema_saved_ms = kNaN;
  double ema_restore_ms = kNaN;
  double ema_roi = kNaN;
  std::uint64_t failure_count = 0;
  std::uint64_t block_count = 0;
  std::uint64_t saved_ms = 0;
  std::uint64_t hit_count = 0;
  std::uint64_t last_used = 0;
  std::uint64_t last_hit_ms = 0;
  std::uint32_t low_roi_hits = 0;
  std::uint64_t kv_size = 0;
  std::uint64_t last_access_time_ms = 0;
  std::uint64_t access_count = 0;
  std::uint64_t stored_at_ms = 0;
  std::uint64_t expires_at_ms = 0;
  std::uint64_t size_bytes = 0;
  std::uint64_t kv_checksum = 0;
  std::uint8_t state = 0;
};

struct AmfStats {
  std::uint64_t hits = 0, misses = 0, tokens_saved = 0, ms_saved = 0, restore_ms = 0;
  double saved_ms_ema = kNaN, restore_ms_ema = kNaN;
  std::uint64_t failures = 0, blocks = 0, admissions = 0, admission_rejects = 0;
  std::uint64_t admission_bytes = 0, store_failures = 0, evictions = 0, evicted_bytes = 0;
  std::uint64_t entries = 0, bytes = 0;
};

struct AmfStorageStats {
  std::uint64_t total_bytes = 0, budget_bytes = 0;
  double utilization = 0.0;
  std::uint64_t hot_entries = 0, warm_entries = 0, cold_entries = 0;
  std::uint64_t disk_free_bytes = 0, disk_capacity_bytes = 0;
  double disk_free_ratio = 0.0;
  bool low_disk = false;
};

enum class Tier : std::uint8_t { kHot = 0, kWarm = 1, kCold = 2 };
enum class EvictionPolicy : std::uint8_t { kLru = 0, kLfu = 1, kRoi = 2 };
enum class EntryState : std::uint8_t { kCold = 0, kWarmPending = 1, kHot = 2 };
enum class DisableReason : std::uint8_t { kNone = 0, kEnvOff, kNoPath, kIoError, kStateApiMissing };
enum class Lookup : std::uint8_t {
  kHit = 0,
  kMissFirstRun,
  kMissShortPrefix,
  kMissHashMismatch,
  kMissTokenMismatch,
  kMissLoadFailed,
};

const char* disable_reason_name(DisableReason r);
const char* lookup_name(Lookup r);

// Index record sizes of the two readable on-disk versions.
constexpr std::size_t kIndexHeaderBytes = 24;
constexpr std::size_t kRecordBytesV9 = 232;
constexpr std::size_t kRecordBytesV8 = 224;
constexpr std::uint32_t kIndexMagic = 0x31464d41u;  // "AMF1" little-endian
constexpr std::uint32_t kIndexVersion = 9u;

// Serialise / parse one index record (exposed for format tests).
void encode_record_v9(const AmfEntry& e, std::uint8_t* out);
AmfEntry decode_record(const std::uint8_t* in, std::uint32_t version);

struct StoreConfig {
  std::size_t min_tokens = 64;
  double min_prompt_ms = 0.0;
  double min_roi = 0.0;
  double min_admit_roi = 0.0;
  std::uint64_t max_bytes = 512ull << 20;
  std::uint64_t storage_budget_bytes = 512ull << 20;
  double eviction_watermark = 0.90;
  double critical_watermark = 0.98;
  std::uint64_t hot_ttl_ms = 5ull * 60 * 1000;
  std::uint64_t warm_ttl_ms = 60ull * 60 * 1000;
  EvictionPolicy policy = EvictionPolicy::kLru;
  std::uint64_t max_age_ms = 0;
  std::uint64_t default_ttl_ms = 24ull * 3600 * 1000;
  std::uint64_t max_ttl_ms = 7ull * 24 * 3600 * 1000;
  bool model_version_check = true;
  std::uint32_t low_roi_hit_limit = 3;
  bool prewarm = false;
  std::uint32_t prewarm_top_k = 10;
  std::uint64_t prewarm_timeout_ms = 30000;
  std::uint64_t prewarm_wait_ms = 100;
  bool disk_guard = true;
  std::uint64_t min_free_disk_bytes = 0;
  double min_free_disk_ratio = 0.0;
};

// Parse every KORITH_AMF_* variable that configures the disk store.
// Returns false (with *enabled=false) when KORITH_ENABLE_AMF is unset/0.
bool store_config_from_env(StoreConfig* cfg, std::string* path, bool* enabled);

class AmfStore {
 public:
  AmfStore() = default;
  ~AmfStore();
  AmfStore(const AmfStore&) = delete;
  AmfStore& operator=(const AmfStore&) = delete;

  bool init_from_env();
  bool init(const std::string& path, const StoreConfig& cfg);

  bool enabled() const { return enabled_; }
  DisableReason disable_reason() const { return disable_reason_; }
  const StoreConfig& config() const { return cfg_; }
  std::string dir() const { return dir_; }

  Lookup find_longest_prefix(const AmfContext& ctx, const std::int32_t* toks, std::size_t n,
                             AmfEntry* out_entry, std::vector<std::int32_t>* out_tokens);
  bool load_kv(const AmfEntry& e, std::vector<std::uint8_t>* out) const;
  bool load_kv_into(const AmfEntry& e, void* buf, std::size_t cap, std::size_t* got) const;
  bool store_entry(const AmfContext& ctx, const std::int32_t* toks, std::size_t n,
                   const std::uint8_t* kv, std::size_t kv_size, std::uint64_t saved_ms);

  void note_hit(const AmfEntry& e, std::uint64_t tokens_saved, std::uint64_t restore_ms,
                std::uint64_t saved_ms);
  void note_failure(const AmfEntry& e);
  void note_block();
  void note_block(const AmfEntry& e);
  void note_miss();
  void evict_expired_entries(std::uint64_t now_ms);
  bool remove(const AmfKey& key);

  AmfStats stats() const;
  AmfStorageStats storage_stats(std::uint64_t now_ms) const;
  std::vector<AmfEntry> entries() const;
  std::uint64_t total_bytes() const;
  std::uint64_t entry_count() const;
  double eviction_pressure() const;
  double warm_ratio() const;
  bool prewarm_complete() const { return prewarm_complete_.load(); }
  std::uint64_t prewarm_loaded() const { return prewarm_loaded_.load(); }
  std::uint64_t prewarm_failed() const { return prewarm_failed_.load(); }
  std::uint64_t oldest_entry_age_ms(std::uint64_t now_ms) const;
  float reuse_score(std::size_t prompt_len, std::uint32_t prefix_len) const;
  float avg_prefix_length() const;
  float historical_accept_rate() const;
  float restore_cost_ms() const;

  void set_min_prompt_ms(double v);
  void set_min_admit_roi(double v);
  void set_eviction_pressure(double v);

  std::string basename_of(const AmfKey& k) const;
  std::string kv_path(const AmfKey& k) const;
  std::string tok_path(const AmfKey& k) const;
  bool flush();
  void shutdown();

 private:
  bool load_index_locked();
  bool flush_index_locked() const;
  Tier tier_of(const AmfEntry& e, std::uint64_t now_ms) const;
  std::uint64_t ttl_for(std::uint64_t access_count) const;
  void evict_at_locked(std::size_t idx, const char* reason);
  void erase_at_locked(std::size_t idx);
  void insert_locked(const AmfEntry& e);
  std::size_t pick_victim_locked(Tier tier, std::uint64_t now_ms) const;
  void evict_for_locked(std::uint64_t incoming);
  void refresh_pressure_locked();
  bool disk_allows(std::uint64_t incoming, std::uint64_t* avail, std::uint64_t* cap,
                   double* ratio) const;
  bool read_tokens(const AmfEntry& e, std::vector<std::int32_t>* out) const;
  bool is_prewarmed(const AmfKey& k) const;
  void start_prewarm_locked();
  void run_prewarm(std::vector<AmfEntry> ranked);

  mutable std::recursive_mutex mu_;
  StoreConfig cfg_{};
  std::string dir_;
  std::string index_path_;
  bool enabled_ = false;
  DisableReason disable_reason_ = DisableReason::kNone;
  std::uint64_t total_bytes_ = 0;
  double eviction_pressure_ = 1.0;
  std::uint32_t roi_decline_streak_ = 0;
  bool admissions_disabled_ = false;
  AmfStats stats_{};
  std::vector<AmfEntry> entries_;
  std::unordered_map<AmfKey, std::size_t, AmfKeyHasher> index_;
  std::map<std::uint32_t, std::uint32_t> len_counts_;  // prefix_len -> #entries

  mutable std::mutex prewarm_mu_;
  std::unordered_set<AmfKey, AmfKeyHasher> prewarmed_;
  std::thread prewarm_thread_;
  std::atomic<bool> prewarm_running_{false};
  std::atomic<bool> prewarm_complete_{true};
  std::atomic<bool> prewarm_cancel_{false};
  std::atomic<std::uint64_t> prewarm_loaded_{0};
  std::atomic<std::uint64_t> prewarm_failed_{0};
};

std::uint64_t now_epoch_ms();

}  // namespace axr
