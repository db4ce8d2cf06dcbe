// Persistent AMF disk store (see amf_store.h for the contract).
#include "amf_store.h"

#include <unistd.h>

#include <algorithm>
#include <cerrno>
#include <cstdarg>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <filesystem>
#include <fstream>

#include "fnv.h"

namespace fs = std::filesystem;

namespace axr {

namespace {

constexpr std::uint32_t kIndexVersionV8 = 8u;
constexpr std::uint32_t kRoiDeclineWarn = 3u;
constexpr std::uint32_t kRoiDeclineStop = 5u;
constexpr std::uint64_t kMaxRecords = 1ull << 20;
constexpr double kEmaAlpha = 0.2;

// ---- little-endian field codec -------------------------------------------------
struct Writer {
  std::uint8_t* p;
  void u8(std::uint8_t v) { *p++ = v; }
  void u32(std::uint32_t v) { std::memcpy(p, &v, 4); p += 4; }
  void u64(std::uint64_t v) { std::memcpy(p, &v, 8); p += 8; }
  void f64(double v) { std::memcpy(p, &v, 8); p += 8; }
  void pad(std::size_t n) { std::memset(p, 0, n); p += n; }
};
struct Reader {
  const std::uint8_t* p;
  std::uint8_t u8() { return *p++; }
  std::uint32_t u32() { std::uint32_t v; std::memcpy(&v, p, 4); p += 4; return v; }
  std::uint64_t u64() { std::uint64_t v; std::memcpy(&v, p, 8); p += 8; return v; }
  double f64() { double v; std::memcpy(&v, p, 8); p += 8; return v; }
  void skip(std::size_t n) { p += n; }
};
static_assert(sizeof(double) == 8, "double must be 64-bit");

void encode_header(std::uint8_t* out, std::uint32_t version, std::uint64_t count,
                   std::uint64_t checksum) {
  Writer w{out};
  w.u32(kIndexMagic);
  w.u32(version);
  w.u64(count);
  w.u64(checksum);
}

bool env_u64(const char* name, std::uint64_t* out) {
  const char* v = std::getenv(name);
  if (!v || !*v) return false;
  char* end = nullptr;
  errno = 0;
  unsigned long long x = std::strtoull(v, &end, 10);
  if (!end || end == v || *end != '\0' || errno == ERANGE) return false;
  *out = x;
  return true;
}

bool env_f64(const char* name, double* out) {
  const char* v = std::getenv(name);
  if (!v || !*v) return false;
  char* end = nullptr;
  double x = std::strtod(v, &end);
  if (!end || end == v || *end != '\0' || !std::isfinite(x)) return false;
  *out = x;
  return true;
}

bool env_bool(const char* name, bool dflt) {
  const char* v = std::getenv(name);
  if (!v || !*v) return dflt;
  std::string s(v);
  if (s == "1" || s == "true" || s == "TRUE" || s == "yes" || s == "on") return true;
  if (s == "0" || s == "false" || s == "FALSE" || s == "no" || s == "off") return false;
  return dflt;
}

double ema(double cur, double sample) {
  if (!std::isfinite(sample)) return cur;
  if (!std::isfinite(cur)) return sample;
  return cur * (1.0 - kEmaAlpha) + sample * kEmaAlpha;
}

std::uint64_t last_access(const AmfEntry& e) {
  return e.last_access_time_ms > 0 ? e.last_access_time_ms : e.last_used;
}

const char* tier_name(Tier t) {
  switch (t) {
    case Tier::kHot: return "hot";
    case Tier::kWarm: return "warm";
    default: return "cold";
  }
}

const char* policy_name(EvictionPolicy p) {
  switch (p) {
    case EvictionPolicy::kLru: return "lru";
    case EvictionPolicy::kLfu: return "lfu";
    case EvictionPolicy::kRoi: return "roi";
  }
  return "unknown";
}

void log_line(const char* fmt, ...) __attribute__((format(printf, 1, 2)));
void log_line(const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  std::vfprintf(stderr, fmt, ap);
  va_end(ap);
  std::fflush(stderr);
}

void log_store_fail(const char* stage, const char* reason, const std::string& path) {
  const int err = errno;
  log_line("[AMF_STORE_FAIL] stage=%s reason=%s path=%s errno=%d err=%s\n", stage, reason,
           path.c_str(), err, std::strerror(err));
}

bool read_file(const std::string& path, std::vector<std::uint8_t>* out) {
  out->clear();
  std::FILE* fp = std::fopen(path.c_str(), "rb");
  if (!fp) return false;
  if (std::fseek(fp, 0, SEEK_END) != 0) { std::fclose(fp); return false; }
  long sz = std::ftell(fp);
  if (sz <= 0) { std::fclose(fp); return false; }
  std::rewind(fp);
  out->resize(static_cast<std::size_t>(sz));
  const std::size_t got = std::fread(out->data(), 1, out->size(), fp);
  std::fclose(fp);
  return got == out->size();
}

bool write_file(const std::string& path, const void* data, std::size_t n) {
  std::FILE* fp = std::fopen(path.c_str(), "wb");
  if (!fp) return false;
  bool ok = n == 0 || std::fwrite(data, 1, n, fp) == n;
  ok = (std::fclose(fp) == 0) && ok;
  return ok;
}

}  // namespace

std::uint64_t now_epoch_ms() {
  using namespace std::chrono;
  return static_cast<std::uint64_t>(
      duration_cast<milliseconds>(system_clock::now().time_since_epoch()).count());
}

std::size_t AmfKeyHasher::operator()(const AmfKey& k) const noexcept {
  std::uint64_t h = kFnvOffset;
  auto mix = [&](std::uint64_t v) { h = (h ^ v) * kFnvPrime; };
  mix(k.model_hash);
  mix(k.tenant_hash);
  mix(k.prefix_hash);
  mix(k.n_ctx);
  mix(k.kv_version);
  mix(k.rope_base_bits);
  mix(k.rope_scale_bits);
  mix(k.sampling_hash);
  mix(k.rng_hash);
  return static_cast<std::size_t>(h);
}

const char* disable_reason_name(DisableReason r) {
  switch (r) {
    case DisableReason::kEnvOff: return "env_off";
    case DisableReason::kNoPath: return "no_path";
    case DisableReason::kIoError: return "io_error";
    case DisableReason::kStateApiMissing: return "state_api_missing";
    default: return "none";
  }
}

const char* lookup_name(Lookup r) {
  switch (r) {
    case Lookup::kHit: return "hit";
    case Lookup::kMissFirstRun: return "first_run";
    case Lookup::kMissShortPrefix: return "short_prefix";
    case Lookup::kMissHashMismatch: return "hash_mismatch";
    case Lookup::kMissTokenMismatch: return "token_mismatch";
    case Lookup::kMissLoadFailed: return "load_failed";
  }
  return "unknown";
}

// ---- record codec ---------------------------------------------------------------
void encode_record_v9(const AmfEntry& e, std::uint8_t* out) {
  Writer w{out};
  w.u64(e.key.model_hash);
  w.u64(e.key.tenant_hash);
  w.u64(e.key.prefix_hash);
  w.u32(e.key.n_ctx);
  w.u32(e.key.kv_version);
  w.u32(e.key.rope_base_bits);
  w.u32(e.key.rope_scale_bits);
  w.u64(e.key.sampling_hash);
  w.u64(e.key.rng_hash);
  w.u64(e.model_hash);
  w.u32(e.prefix_len);
  w.u32(0);
  w.u64(e.seen_count);
  w.u64(e.restore_count);
  w.f64(e.ema_saved_ms);
  w.f64(e.ema_restore_ms);
  w.f64(e.ema_roi);
  w.u64(e.failure_count);
  w.u64(e.block_count);
  w.u64(e.saved_ms);
  w.u64(e.hit_count);
  w.u64(e.last_used);
  w.u64(e.last_hit_ms);
  w.u32(e.low_roi_hits);
  w.u32(0);
  w.u64(e.kv_size);
  w.u64(e.last_access_time_ms);
  w.u64(e.access_count);
  w.u64(e.stored_at_ms);
  w.u64(e.expires_at_ms);
  w.u64(e.size_bytes);
  w.u64(e.kv_checksum);
  w.u8(e.state);
  w.pad(7);
}

AmfEntry decode_record(const std::uint8_t* in, std::uint32_t version) {
  Reader r{in};
  AmfEntry e;
  e.key.model_hash = r.u64();
  e.key.tenant_hash = (version >= kIndexVersion) ? r.u64() : 0;  // v8 keys have no tenant
  e.key.prefix_hash = r.u64();
  e.key.n_ctx = r.u32();
  e.key.kv_version = r.u32();
  e.key.rope_base_bits = r.u32();
  e.key.rope_scale_bits = r.u32();
  e.key.sampling_hash = r.u64();
  e.key.rng_hash = r.u64();
  e.model_hash = r.u64();
  e.prefix_len = r.u32();
  r.skip(4);
  e.seen_count = r.u64();
  e.restore_count = r.u64();
  e.ema_saved_ms = r.f64();
  e.ema_restore_ms = r.f64();
  e.ema_roi = r.f64();
  e.failure_count = r.u64();
  e.block_count = r.u64();
  e.saved_ms = r.u64();
  e.hit_count = r.u64();
  e.last_used = r.u64();
  e.last_hit_ms = r.u64();
  e.low_roi_hits = r.u32();
  r.skip(4);
  e.kv_size = r.u64();
  e.last_access_time_ms = r.u64();
  e.access_count = r.u64();
  e.stored_at_ms = r.u64();
  e.expires_at_ms = r.u64();
  e.size_bytes = r.u64();
  e.kv_checksum = r.u64();
  e.state = r.u8();
  return e;
}

// ---- configuration ---------------------------------------------------------------
bool store_config_from_env(StoreConfig* c, std::string* path, bool* enabled) {
  const char* en = std::getenv("KORITH_ENABLE_AMF");
  *enabled = !(en == nullptr || en[0] == '\0' || en[0] == '0');
  const char* p = std::getenv("KORITH_AMF_PATH");
  *path = (p && *p) ? p : "amf";
  std::uint64_t u = 0;
  double d = 0.0;
  if (env_u64("KORITH_AMF_MIN_TOKENS", &u) && u > 0) c->min_tokens = u;
  if (env_u64("KORITH_AMF_MAX_BYTES", &u) && u > 0) { c->max_bytes = u; c->storage_budget_bytes = u; }
  if (env_f64("KORITH_AMF_STORAGE_BUDGET_GB", &d) && d > 0.0) {
    long double b = static_cast<long double>(d) * 1024.0L * 1024.0L * 1024.0L;
    if (b > 0.0L && b <= static_cast<long double>(UINT64_MAX)) {
      c->storage_budget_bytes = static_cast<std::uint64_t>(b);
      c->max_bytes = c->storage_budget_bytes;
    }
  }
  if (env_f64("KORITH_AMF_EVICTION_WATERMARK", &d) && d > 0.0 && d <= 1.0) c->eviction_watermark = d;
  if (env_u64("KORITH_AMF_HOT_TTL_S", &u) && u > 0) c->hot_ttl_ms = u * 1000ull;
  if (env_u64("KORITH_AMF_WARM_TTL_S", &u) && u > 0) c->warm_ttl_ms = u * 1000ull;
  if (c->hot_ttl_ms > c->warm_ttl_ms) c->hot_ttl_ms = c->warm_ttl_ms;
  if (const char* pol = std::getenv("KORITH_AMF_EVICTION_POLICY")) {
    std::string s(pol);
    if (s == "lru") c->policy = EvictionPolicy::kLru;
    else if (s == "lfu") c->policy = EvictionPolicy::kLfu;
    else if (s == "roi") c->policy = EvictionPolicy::kRoi;
  }
  if (env_f64("KORITH_AMF_MIN_PROMPT_MS", &d) && d > 0.0) c->min_prompt_ms = d;
  if (env_f64("KORITH_AMF_MIN_ROI", &d) && d >= 0.0) c->min_roi = d;
  if (env_f64("KORITH_AMF_MIN_ADMIT_ROI", &d) && d >= 0.0) c->min_admit_roi = d;
  if (env_u64("KORITH_AMF_MAX_AGE_MS", &u)) c->max_age_ms = u;
  if (env_u64("KORITH_AMF_DEFAULT_TTL_S", &u) && u > 0) c->default_ttl_ms = u * 1000ull;
  if (env_u64("KORITH_AMF_MAX_TTL_S", &u) && u > 0) c->max_ttl_ms = u * 1000ull;
  if (c->max_ttl_ms < c->default_ttl_ms) c->max_ttl_ms = c->default_ttl_ms;
  c->model_version_check = env_bool("KORITH_AMF_MODEL_VERSION_CHECK", true);
  if (env_u64("KORITH_AMF_LOW_ROI_HITS", &u) && u > 0)
    c->low_roi_hit_limit = static_cast<std::uint32_t>(std::min<std::uint64_t>(u, UINT32_MAX));
  c->prewarm = env_bool("KORITH_AMF_PREWARM", false);
  if (env_u64("KORITH_AMF_PREWARM_TOP_K", &u) && u > 0)
    c->prewarm_top_k = static_cast<std::uint32_t>(std::min<std::uint64_t>(u, UINT32_MAX));
  if (env_u64("KORITH_AMF_PREWARM_TIMEOUT_S", &u)) c->prewarm_timeout_ms = u * 1000ull;
  c->disk_guard = env_bool("KORITH_AMF_DISK_GUARD", true);
  if (env_u64("KORITH_AMF_MIN_FREE_DISK_BYTES", &u)) c->min_free_disk_bytes = u;
  if (env_f64("KORITH_AMF_MIN_FREE_DISK_PCT", &d) && d >= 0.0 && d <= 1.0) c->min_free_disk_ratio = d;
  if (c->storage_budget_bytes == 0) c->storage_budget_bytes = c->max_bytes;
  if (c->max_bytes == 0) c->max_bytes = c->storage_budget_bytes;
  return *enabled;
}

// ---- lifecycle --------------------------------------------------------------------
AmfStore::~AmfStore() { shutdown(); }

bool AmfStore::init_from_env() {
  StoreConfig cfg;
  std::string path;
  bool en = false;
  store_config_from_env(&cfg, &path, &en);
  if (!en) {
    std::lock_guard<std::recursive_mutex> g(mu_);
    cfg_ = cfg;
    enabled_ = false;
    disable_reason_ = DisableReason::kEnvOff;
    return false;
  }
  return init(path, cfg);
}

bool AmfStore::init(const std::string& path, const StoreConfig& cfg) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  cfg_ = cfg;
  dir_ = path;
  if (dir_.empty()) {
    enabled_ = false;
    disable_reason_ = DisableReason::kNoPath;
    return false;
  }
  std::error_code ec;
  fs::create_directories(dir_, ec);
  if (ec) {
    enabled_ = false;
    disable_reason_ = DisableReason::kIoError;
    return false;
  }
  index_path_ = (fs::path(dir_) / "amf_index.bin").string();
  enabled_ = load_index_locked();
  if (!enabled_) return false;
  disable_reason_ = DisableReason::kNone;
  log_line("[AMF_PATH] dir=%s index=%s entries=%llu bytes=%llu\n", dir_.c_str(),
           index_path_.c_str(), (unsigned long long)entries_.size(),
           (unsigned long long)total_bytes_);
  if (cfg_.prewarm) start_prewarm_locked();
  return true;
}

void AmfStore::shutdown() {
  prewarm_cancel_.store(true);
  if (prewarm_thread_.joinable()) prewarm_thread_.join();
  prewarm_running_.store(false);
  prewarm_complete_.store(true);
  prewarm_cancel_.store(false);
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (!enabled_) return;
  flush_index_locked();
  log_line("[AMF_SHUTDOWN] entries_persisted=%llu bytes=%llu\n",
           (unsigned long long)entries_.size(), (unsigned long long)total_bytes_);
  enabled_ = false;
}

bool AmfStore::flush() {
  std::lock_guard<std::recursive_mutex> g(mu_);
  return enabled_ && flush_index_locked();
}

// ---- index persistence ------------------------------------------------------------
bool AmfStore::load_index_locked() {
  entries_.clear();
  index_.clear();
  len_counts_.clear();
  total_bytes_ = 0;
  stats_.entries = stats_.bytes = 0;
  roi_decline_streak_ = 0;
  admissions_disabled_ = false;
  prewarm_running_.store(false);
  prewarm_complete_.store(!cfg_.prewarm);
  prewarm_loaded_.store(0);
  prewarm_failed_.store(0);
  {
    std::lock_guard<std::mutex> pg(prewarm_mu_);
    prewarmed_.clear();
  }
  refresh_pressure_locked();

  std::vector<std::uint8_t> buf;
  std::error_code ec;
  if (!fs::exists(index_path_, ec)) return true;  // cold start
  if (!read_file(index_path_, &buf) || buf.size() < kIndexHeaderBytes) {
    disable_reason_ = DisableReason::kIoError;
    return false;
  }
  Reader hr{buf.data()};
  const std::uint32_t magic = hr.u32();
  const std::uint32_t version = hr.u32();
  const std::uint64_t count = hr.u64();
  const std::uint64_t checksum = hr.u64();
  if (magic != kIndexMagic) {
    disable_reason_ = DisableReason::kIoError;
    return false;
  }
  if (version != kIndexVersion && version != kIndexVersionV8) {
    fs::remove(index_path_, ec);
    if (ec) {
      disable_reason_ = DisableReason::kIoError;
      return false;
    }
    log_line("[AMF_INDEX_RESET] reason=version_mismatch found=%u expected=%u\n", version,
             kIndexVersion);
    return true;
  }
  if (count > kMaxRecords) {
    disable_reason_ = DisableReason::kIoError;
    return false;
  }
  const std::size_t rec_bytes = version == kIndexVersion ? kRecordBytesV9 : kRecordBytesV8;
  if (buf.size() < kIndexHeaderBytes + count * rec_bytes) {
    disable_reason_ = DisableReason::kIoError;
    return false;
  }
  std::uint8_t hdr0[kIndexHeaderBytes];
  encode_header(hdr0, version, count, 0);
  std::uint64_t h = fnv1a_bytes(kFnvOffset, hdr0, sizeof(hdr0));
  h = fnv1a_bytes(h, buf.data() + kIndexHeaderBytes, count * rec_bytes);
  if (h != checksum) {
    disable_reason_ = DisableReason::kIoError;
    return false;
  }
  const std::uint64_t now = now_epoch_ms();
  for (std::uint64_t i = 0; i < count; ++i) {
    AmfEntry e = decode_record(buf.data() + kIndexHeaderBytes + i * rec_bytes, version);
    if (e.model_hash == 0) e.model_hash = e.key.model_hash;
    if (e.size_bytes == 0) e.size_bytes = e.kv_size;
    if (e.last_access_time_ms == 0) e.last_access_time_ms = e.last_used;
    if (e.expires_at_ms == 0 && cfg_.default_ttl_ms > 0) {
      const std::uint64_t base = e.last_access_time_ms > 0 ? e.last_access_time_ms : now;
      e.expires_at_ms = base + ttl_for(e.access_count);
    }
    if (cfg_.prewarm) {
      e.state = static_cast<std::uint8_t>(EntryState::kWarmPending);
    } else {
      e.state = static_cast<std::uint8_t>(tier_of(e, now) == Tier::kHot ? EntryState::kHot
                                                                        : EntryState::kCold);
    }
    insert_locked(e);
  }
  refresh_pressure_locked();
  return true;
}

bool AmfStore::flush_index_locked() const {
  const std::string tmp = (fs::path(dir_) / "amf_index.tmp").string();
  std::vector<std::uint8_t> buf(kIndexHeaderBytes + entries_.size() * kRecordBytesV9);
  for (std::size_t i = 0; i < entries_.size(); ++i)
    encode_record_v9(entries_[i], buf.data() + kIndexHeaderBytes + i * kRecordBytesV9);
  encode_header(buf.data(), kIndexVersion, entries_.size(), 0);
  const std::uint64_t sum = fnv1a_bytes(kFnvOffset, buf.data(), buf.size());
  encode_header(buf.data(), kIndexVersion, entries_.size(), sum);

  errno = 0;
  std::FILE* fp = std::fopen(tmp.c_str(), "wb");
  if (!fp) { log_store_fail("flush_index_open", "open_failed", tmp); return false; }
  if (std::fwrite(buf.data(), 1, buf.size(), fp) != buf.size()) {
    std::fclose(fp);
    log_store_fail("flush_index_write", "write_failed", tmp);
    return false;
  }
  if (std::fflush(fp) != 0 || ::fsync(::fileno(fp)) != 0) {
    std::fclose(fp);
    log_store_fail("flush_index_fsync", "fsync_failed", tmp);
    return false;
  }
  if (std::fclose(fp) != 0) { log_store_fail("flush_index_close", "close_failed", tmp); return false; }
  std::error_code ec;
  fs::rename(tmp, index_path_, ec);
  if (ec) {
    log_line("[AMF_STORE_FAIL] stage=flush_index_rename reason=rename_failed path=%s ec=%d msg=%s\n",
             index_path_.c_str(), ec.value(), ec.message().c_str());
    fs::remove(tmp, ec);
    return false;
  }
  return true;
}

// ---- naming -------------------------------------------------------------------------
std::string AmfStore::basename_of(const AmfKey& k) const {
  char b[256];
  std::snprintf(b, sizeof(b), "amf_%016llx_%016llx_%016llx_%08x_%08x_%08x_%08x_%016llx_%016llx",
                (unsigned long long)k.model_hash, (unsigned long long)k.tenant_hash,
                (unsigned long long)k.prefix_hash, k.n_ctx, k.kv_version, k.rope_base_bits,
                k.rope_scale_bits, (unsigned long long)k.sampling_hash,
                (unsigned long long)k.rng_hash);
  return b;
}
std::string AmfStore::kv_path(const AmfKey& k) const {
  return (fs::path(dir_) / (basename_of(k) + ".kv")).string();
}
std::string AmfStore::tok_path(const AmfKey& k) const {
  return (fs::path(dir_) / (basename_of(k) + ".tok")).string();
}

// ---- entry bookkeeping ---------------------------------------------------------------
void AmfStore::insert_locked(const AmfEntry& e) {
  index_[e.key] = entries_.size();
  entries_.push_back(e);
  len_counts_[e.prefix_len] += 1;
  total_bytes_ += e.size_bytes;
  stats_.entries = entries_.size();
  stats_.bytes = total_bytes_;
}

void AmfStore::erase_at_locked(std::size_t idx) {
  const AmfEntry e = entries_[idx];
  auto lc = len_counts_.find(e.prefix_len);
  if (lc != len_counts_.end() && --lc->second == 0) len_counts_.erase(lc);
  index_.erase(e.key);
  const std::size_t last = entries_.size() - 1;
  if (idx != last) {
    entries_[idx] = entries_[last];
    index_[entries_[idx].key] = idx;
  }
  entries_.pop_back();
  const std::uint64_t b = e.size_bytes > 0 ? e.size_bytes : e.kv_size;
  total_bytes_ = b <= total_bytes_ ? total_bytes_ - b : 0;
  stats_.entries = entries_.size();
  stats_.bytes = total_bytes_;
  std::lock_guard<std::mutex> pg(prewarm_mu_);
  prewarmed_.erase(e.key);
}

void AmfStore::evict_at_locked(std::size_t idx, const char* reason) {
  if (idx >= entries_.size()) return;
  const AmfEntry e = entries_[idx];
  const Tier t = tier_of(e, now_epoch_ms());
  std::error_code ec;
  fs::remove(kv_path(e.key), ec);
  fs::remove(tok_path(e.key), ec);
  const std::uint64_t b = e.size_bytes > 0 ? e.size_bytes : e.kv_size;
  stats_.evictions += 1;
  stats_.evicted_bytes += b;
  erase_at_locked(idx);
  refresh_pressure_locked();
  log_line("[AMF_EVICT] hash=%016llx size=%llu tier=%s policy=%s reason=%s\n",
           (unsigned long long)e.key.prefix_hash, (unsigned long long)b, tier_name(t),
           policy_name(cfg_.policy), reason ? reason : "unknown");
  flush_index_locked();
}

bool AmfStore::remove(const AmfKey& key) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  auto it = index_.find(key);
  if (it == index_.end()) return false;
  evict_at_locked(it->second, "explicit");
  return true;
}

Tier AmfStore::tier_of(const AmfEntry& e, std::uint64_t now_ms) const {
  const std::uint64_t last = last_access(e);
  if (last == 0 || now_ms == 0 || now_ms < last) return Tier::kCold;
  const std::uint64_t age = now_ms - last;
  if (age <= cfg_.hot_ttl_ms) return Tier::kHot;
  if (age <= cfg_.warm_ttl_ms) return Tier::kWarm;
  return Tier::kCold;
}

std::uint64_t AmfStore::ttl_for(std::uint64_t access_count) const {
  if (cfg_.default_ttl_ms == 0) return 0;
  const double boost = 1.0 + std::log2(static_cast<double>(std::max<std::uint64_t>(1, access_count)));
  double ttl = static_cast<double>(cfg_.default_ttl_ms) * boost;
  if (!std::isfinite(ttl) || ttl < static_cast<double>(cfg_.default_ttl_ms))
    ttl = static_cast<double>(cfg_.default_ttl_ms);
  if (cfg_.max_ttl_ms > 0) ttl = std::min(ttl, static_cast<double>(cfg_.max_ttl_ms));
  return static_cast<std::uint64_t>(ttl);
}

void AmfStore::refresh_pressure_locked() {
  const std::uint64_t budget = cfg_.storage_budget_bytes > 0 ? cfg_.storage_budget_bytes : cfg_.max_bytes;
  if (budget == 0) { eviction_pressure_ = 0.0; return; }
  const double p = static_cast<double>(total_bytes_) / static_cast<double>(budget);
  eviction_pressure_ = std::isfinite(p) ? std::max(0.0, p) : 0.0;
}

std::size_t AmfStore::pick_victim_locked(Tier tier, std::uint64_t now_ms) const {
  auto roi = [](const AmfEntry& e) -> double {
    if (std::isfinite(e.ema_roi)) return e.ema_roi;
    if (std::isfinite(e.ema_restore_ms) && e.ema_restore_ms > 0.0 && std::isfinite(e.ema_saved_ms)) {
      const double r = e.ema_saved_ms / e.ema_restore_ms;
      return std::isfinite(r) ? r : 0.0;
    }
    return 0.0;
  };
  // Returns true when `a` is a better eviction victim than `b`.
  auto better = [&](const AmfEntry& a, const AmfEntry& b) -> bool {
    const std::uint64_t la = last_access(a), lb = last_access(b);
    switch (cfg_.policy) {
      case EvictionPolicy::kLru:
        if (la != lb) return la < lb;
        return a.access_count < b.access_count;
      case EvictionPolicy::kRoi: {
        const double ra = roi(a), rb = roi(b);
        if (ra != rb) return ra < rb;
        if (a.access_count != b.access_count) return a.access_count < b.access_count;
        return la < lb;
      }
      case EvictionPolicy::kLfu:
      default:
        if (a.access_count != b.access_count) return a.access_count < b.access_count;
        return la < lb;
    }
  };
  std::size_t best = SIZE_MAX;
  for (std::size_t i = 0; i < entries_.size(); ++i) {
    if (tier_of(entries_[i], now_ms) != tier) continue;
    if (best == SIZE_MAX || better(entries_[i], entries_[best])) best = i;
  }
  return best;
}

void AmfStore::evict_for_locked(std::uint64_t incoming) {
  const std::uint64_t budget = cfg_.storage_budget_bytes > 0 ? cfg_.storage_budget_bytes : cfg_.max_bytes;
  if (budget == 0 || incoming > budget) return;
  const long double wm = static_cast<long double>(budget) * cfg_.eviction_watermark;
  const long double crit = static_cast<long double>(budget) * cfg_.critical_watermark;
  auto projected = [&]() {
    return static_cast<long double>(total_bytes_) + static_cast<long double>(incoming);
  };
  while (projected() > wm && !entries_.empty()) {
    const std::uint64_t now = now_epoch_ms();
    std::size_t idx = pick_victim_locked(Tier::kCold, now);
    if (idx == SIZE_MAX) idx = pick_victim_locked(Tier::kWarm, now);
    if (idx == SIZE_MAX && projected() > crit) idx = pick_victim_locked(Tier::kHot, now);
    if (idx == SIZE_MAX) break;
    evict_at_locked(idx, "budget");
  }
  refresh_pressure_locked();
}

bool AmfStore::disk_allows(std::uint64_t incoming, std::uint64_t* avail, std::uint64_t* cap,
                           double* ratio) const {
  *avail = 0;
  *cap = 0;
  *ratio = 0.0;
  if (!cfg_.disk_guard) return true;
  std::error_code ec;
  const fs::space_info si = fs::space(dir_, ec);
  if (ec) return true;
  *avail = si.available;
  *cap = si.capacity;
  if (*cap > 0) *ratio = static_cast<double>(*avail) / static_cast<double>(*cap);
  if (cfg_.min_free_disk_bytes > 0 && *avail <= cfg_.min_free_disk_bytes) return false;
  if (cfg_.min_free_disk_ratio > 0.0 && *cap > 0 && *ratio <= cfg_.min_free_disk_ratio) return false;
  if (incoming > 0 && *avail <= incoming) return false;
  return true;
}

bool AmfStore::read_tokens(const AmfEntry& e, std::vector<std::int32_t>* out) const {
  out->clear();
  std::vector<std::uint8_t> raw;
  if (!read_file(tok_path(e.key), &raw) || raw.size() % 4 != 0) return false;
  out->resize(raw.size() / 4);
  std::memcpy(out->data(), raw.data(), raw.size());
  return true;
}

// ---- lookup ----------------------------------------------------------------------------
Lookup AmfStore::find_longest_prefix(const AmfContext& ctx, const std::int32_t* toks,
                                     std::size_t n, AmfEntry* out_entry,
                                     std::vector<std::int32_t>* out_tokens) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (!enabled_) return Lookup::kMissLoadFailed;
  if (n < cfg_.min_tokens) return Lookup::kMissShortPrefix;
  if (entries_.empty()) return Lookup::kMissFirstRun;

  // Only lengths that some entry actually has can match; probe them longest first.
  std::vector<std::uint32_t> lens;
  for (auto it = len_counts_.rbegin(); it != len_counts_.rend(); ++it) {
    if (it->first <= n && it->first >= cfg_.min_tokens) lens.push_back(it->first);
  }
  if (lens.empty()) return Lookup::kMissHashMismatch;
  std::vector<std::uint64_t> ph(lens.front());
  std::uint64_t h = kFnvOffset;
  for (std::size_t i = 0; i < lens.front(); ++i) {
    h = fnv1a_token(h, toks[i]);
    ph[i] = h;
  }
  const std::uint64_t now = now_epoch_ms();
  std::vector<std::int32_t> scratch;
  std::vector<std::int32_t>* tokbuf = out_tokens ? out_tokens : &scratch;
  for (std::uint32_t len : lens) {
    auto it = index_.find(ctx.key_for(ph[len - 1]));
    if (it == index_.end()) continue;
    const AmfEntry e = entries_[it->second];
    if (e.prefix_len != len) continue;
    if (cfg_.model_version_check && e.model_hash != 0 && e.model_hash != ctx.model_hash) {
      log_line("[AMF_MODEL_MISMATCH] hash=%016llx\n", (unsigned long long)e.key.prefix_hash);
      evict_at_locked(it->second, "model_mismatch");
      continue;
    }
    if (e.expires_at_ms > 0 && now > e.expires_at_ms) {
      const std::uint64_t age = now > e.stored_at_ms ? now - e.stored_at_ms : 0;
      log_line("[AMF_EXPIRED] hash=%016llx age_s=%llu\n", (unsigned long long)e.key.prefix_hash,
               (unsigned long long)(age / 1000));
      evict_at_locked(it->second, "ttl");
      continue;
    }
    if (cfg_.prewarm && e.state == static_cast<std::uint8_t>(EntryState::kWarmPending) &&
        !is_prewarmed(e.key) && prewarm_running_.load()) {
      std::this_thread::sleep_for(std::chrono::milliseconds(cfg_.prewarm_wait_ms));
      if (!is_prewarmed(e.key)) continue;
    }
    if (is_prewarmed(e.key)) {
      auto live = index_.find(e.key);
      if (live != index_.end()) entries_[live->second].state = static_cast<std::uint8_t>(EntryState::kHot);
    }
    if (!read_tokens(e, tokbuf)) return Lookup::kMissLoadFailed;
    if (tokbuf->size() != len) return Lookup::kMissTokenMismatch;
    if (!std::equal(tokbuf->begin(), tokbuf->end(), toks)) return Lookup::kMissTokenMismatch;
    if (out_entry) *out_entry = e;
    return Lookup::kHit;
  }
  return Lookup::kMissHashMismatch;
}

bool AmfStore::load_kv(const AmfEntry& e, std::vector<std::uint8_t>* out) const {
  if (!read_file(kv_path(e.key), out)) return false;
  if (e.kv_checksum > 0 && fnv1a_bytes(kFnvOffset, out->data(), out->size()) != e.kv_checksum)
    return false;
  return true;
}

bool AmfStore::load_kv_into(const AmfEntry& e, void* buf, std::size_t cap, std::size_t* got) const {
  *got = 0;
  const std::string path = kv_path(e.key);
  std::FILE* fp = std::fopen(path.c_str(), "rb");
  if (!fp) return false;
  std::fseek(fp, 0, SEEK_END);
  const long sz = std::ftell(fp);
  if (sz <= 0) { std::fclose(fp); return false; }
  const std::size_t n = static_cast<std::size_t>(sz);
  if (n > cap) {
    std::fclose(fp);
    log_line("[AMF_STORE] load_kv_into: buf too small (%zu < %zu)\n", cap, n);
    return false;
  }
  std::rewind(fp);
  const std::size_t r = std::fread(buf, 1, n, fp);
  std::fclose(fp);
  if (r != n) return false;
  if (e.kv_checksum > 0 && fnv1a_bytes(kFnvOffset, buf, n) != e.kv_checksum) {
    log_line("[AMF_STORE] load_kv_into: checksum mismatch\n");
    return false;
  }
  *got = n;
  return true;
}

// ---- admission -------------------------------------------------------------------------
bool AmfStore::store_entry(const AmfContext& ctx, const std::int32_t* toks, std::size_t n,
                           const std::uint8_t* kv, std::size_t kv_size, std::uint64_t saved_ms) {
  // The checksum of a multi-GB blob is the slow part: compute it before taking the lock.
  const std::uint64_t sum = (kv && kv_size) ? fnv1a_bytes(kFnvOffset, kv, kv_size) : 0;
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (!enabled_ || n < cfg_.min_tokens || kv_size == 0 || !kv) {
    stats_.admission_rejects += 1;
    return false;
  }
  const std::uint64_t budget = cfg_.storage_budget_bytes > 0 ? cfg_.storage_budget_bytes : cfg_.max_bytes;
  if (budget > 0 && kv_size > budget) {
    stats_.admission_rejects += 1;
    return false;
  }
  const AmfKey key = ctx.key_for(fnv1a_tokens(toks, n));
  auto it = index_.find(key);
  const bool existing = it != index_.end();
  const AmfEntry prev = existing ? entries_[it->second] : AmfEntry{};
  const std::uint64_t disk_incoming = existing ? (kv_size > prev.kv_size ? kv_size - prev.kv_size : 0) : kv_size;
  std::uint64_t avail = 0, cap = 0;
  double ratio = 0.0;
  if (!disk_allows(disk_incoming, &avail, &cap, &ratio)) {
    stats_.admission_rejects += 1;
    log_line("[AMF_ADMIT_REJECT] reason=disk_guard free_bytes=%llu free_pct=%.2f min_free_bytes=%llu min_free_pct=%.2f\n",
             (unsigned long long)avail, ratio * 100.0, (unsigned long long)cfg_.min_free_disk_bytes,
             cfg_.min_free_disk_ratio * 100.0);
    return false;
  }
  if (admissions_disabled_ && !existing) {
    stats_.admission_rejects += 1;
    log_line("[AMF_ADMIT_REJECT] reason=admissions_disabled\n");
    return false;
  }
  const bool ema_ready = existing && std::isfinite(prev.ema_roi);
  const bool bootstrap = !existing || (prev.restore_count == 0 && prev.seen_count == 0 && !ema_ready);
  if (cfg_.min_admit_roi > 0.0) {
    if (bootstrap) {
      log_line("[AMF_ADMIT_BOOTSTRAP] key=%016llx reason=first_restore\n",
               (unsigned long long)AmfKeyHasher{}(key));
    } else if (ema_ready && prev.ema_roi >= cfg_.min_admit_roi) {
      log_line("[AMF_ADMIT] reason=roi_pass roi=%.2f min=%.2f\n", prev.ema_roi, cfg_.min_admit_roi);
    } else {
      stats_.admission_rejects += 1;
      if (ema_ready) {
        log_line("[AMF_ADMIT_REJECT] reason=ema_roi roi=%.2f min=%.2f\n", prev.ema_roi, cfg_.min_admit_roi);
      } else {
        log_line("[AMF_ADMIT_REJECT] reason=ema_roi roi=nan min=%.2f\n", cfg_.min_admit_roi);
      }
      return false;
    }
  }

  const std::uint64_t now = now_epoch_ms();
  AmfEntry e;
  e.key = key;
  e.model_hash = ctx.model_hash;
  e.prefix_len = static_cast<std::uint32_t>(n);
  e.seen_count = existing ? prev.seen_count + 1 : 1;
  e.restore_count = existing ? prev.restore_count : 0;
  e.ema_saved_ms = existing ? prev.ema_saved_ms : kNaN;
  e.ema_restore_ms = existing ? prev.ema_restore_ms : kNaN;
  e.ema_roi = existing ? prev.ema_roi : kNaN;
  e.saved_ms = saved_ms;
  e.last_used = now;
  e.last_access_time_ms = now;
  e.stored_at_ms = now;
  e.expires_at_ms = cfg_.default_ttl_ms > 0 ? now + ttl_for(0) : 0;
  e.kv_size = kv_size;
  e.size_bytes = kv_size;
  e.kv_checksum = sum;
  e.state = static_cast<std::uint8_t>(EntryState::kHot);

  if (existing) {
    if (kv_size > prev.kv_size) evict_for_locked(kv_size - prev.kv_size);
  } else {
    evict_for_locked(kv_size);
  }
  // Eviction above may have moved entries; re-resolve the slot of an existing key.
  it = index_.find(key);
  const bool still_existing = it != index_.end();

  std::vector<std::uint8_t> tokbytes(n * 4);
  std::memcpy(tokbytes.data(), toks, n * 4);
  errno = 0;
  if (!write_file(tok_path(key), tokbytes.data(), tokbytes.size())) {
    log_store_fail("write_tokens", "write_failed", tok_path(key));
    stats_.store_failures += 1;
    return false;
  }
  if (!write_file(kv_path(key), kv, kv_size)) {
    log_store_fail("write_kv", "write_failed", kv_path(key));
    std::error_code ec;
    fs::remove(tok_path(key), ec);
    stats_.store_failures += 1;
    return false;
  }
  if (still_existing) {
    e.failure_count = prev.failure_count;
    e.block_count = prev.block_count;
    e.hit_count = prev.hit_count;
    e.last_hit_ms = prev.last_hit_ms;
    e.low_roi_hits = prev.low_roi_hits;
    e.last_access_time_ms = prev.last_access_time_ms;
    e.access_count = prev.access_count;
    e.stored_at_ms = prev.stored_at_ms;
    const std::uint64_t ttl = ttl_for(e.access_count);
    e.expires_at_ms = ttl > 0 ? now + ttl : prev.expires_at_ms;
    erase_at_locked(it->second);
  }
  insert_locked(e);
  stats_.admissions += 1;
  stats_.admission_bytes += kv_size;
  refresh_pressure_locked();
  if (!flush_index_locked()) {
    stats_.store_failures += 1;
    return false;
  }
  return true;
}

// ---- accounting --------------------------------------------------------------------------
void AmfStore::note_hit(const AmfEntry& entry, std::uint64_t tokens_saved,
                        std::uint64_t restore_ms, std::uint64_t saved_ms) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  stats_.hits += 1;
  stats_.tokens_saved += tokens_saved;
  stats_.ms_saved += saved_ms;
  stats_.restore_ms += restore_ms;
  const double s = static_cast<double>(saved_ms), r = static_cast<double>(restore_ms);
  const double roi = r > 0.0 ? s / r : 0.0;
  stats_.saved_ms_ema = ema(stats_.saved_ms_ema, s);
  stats_.restore_ms_ema = ema(stats_.restore_ms_ema, r);
  auto it = index_.find(entry.key);
  if (it == index_.end()) return;
  AmfEntry& e = entries_[it->second];
  const std::uint64_t now = now_epoch_ms();
  e.hit_count += 1;
  e.access_count += 1;
  e.restore_count += 1;
  e.last_used = e.last_access_time_ms = e.last_hit_ms = now;
  e.state = static_cast<std::uint8_t>(EntryState::kHot);
  const std::uint64_t ttl = ttl_for(e.access_count);
  if (ttl > 0) e.expires_at_ms = now + ttl;
  const double prev_roi = e.ema_roi;
  e.ema_restore_ms = ema(e.ema_restore_ms, r);
  e.ema_saved_ms = ema(e.ema_saved_ms, s);
  e.ema_roi = ema(e.ema_roi, roi);
  if (std::isfinite(prev_roi) && std::isfinite(e.ema_roi) && e.ema_roi < prev_roi) {
    if (roi_decline_streak_ < UINT32_MAX) roi_decline_streak_ += 1;
  } else {
    roi_decline_streak_ = 0;
  }
  if (roi_decline_streak_ == kRoiDeclineWarn) e.failure_count += 1;
  if (roi_decline_streak_ >= kRoiDeclineStop) admissions_disabled_ = true;
  if (cfg_.min_admit_roi > 0.0 && cfg_.low_roi_hit_limit > 0) {
    const double re = std::isfinite(e.ema_roi) ? e.ema_roi : 0.0;
    if (re < cfg_.min_admit_roi) {
      if (e.low_roi_hits < UINT32_MAX) e.low_roi_hits += 1;
    } else {
      e.low_roi_hits = 0;
    }
    if (e.low_roi_hits >= cfg_.low_roi_hit_limit) {
      evict_at_locked(it->second, "low_roi");
      return;
    }
  }
  flush_index_locked();
}

void AmfStore::note_failure(const AmfEntry& entry) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  stats_.failures += 1;
  auto it = index_.find(entry.key);
  if (it == index_.end()) return;
  AmfEntry& e = entries_[it->second];
  e.failure_count += 1;
  e.last_used = e.last_access_time_ms = now_epoch_ms();
  flush_index_locked();
}

void AmfStore::note_block() {
  std::lock_guard<std::recursive_mutex> g(mu_);
  stats_.blocks += 1;
}

void AmfStore::note_block(const AmfEntry& entry) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  stats_.blocks += 1;
  auto it = index_.find(entry.key);
  if (it == index_.end()) return;
  AmfEntry& e = entries_[it->second];
  e.block_count += 1;
  e.last_used = e.last_access_time_ms = now_epoch_ms();
  flush_index_locked();
}

void AmfStore::note_miss() {
  std::lock_guard<std::recursive_mutex> g(mu_);
  stats_.misses += 1;
}

void AmfStore::evict_expired_entries(std::uint64_t now_ms) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (!enabled_ || now_ms == 0 || entries_.empty()) return;
  // Swap-erase moves the last entry into the hole, so walk from the back.
  for (std::size_t i = entries_.size(); i-- > 0;) {
    if (i >= entries_.size()) continue;
    const AmfEntry& e = entries_[i];
    if (e.expires_at_ms > 0 && now_ms > e.expires_at_ms) {
      const std::uint64_t age = now_ms > e.stored_at_ms ? now_ms - e.stored_at_ms : 0;
      log_line("[AMF_EXPIRED] hash=%016llx age_s=%llu\n", (unsigned long long)e.key.prefix_hash,
               (unsigned long long)(age / 1000));
      evict_at_locked(i, "ttl");
      continue;
    }
    if (cfg_.max_age_ms == 0) continue;
    const std::uint64_t last = e.last_hit_ms > 0 ? e.last_hit_ms : e.last_used;
    if (last == 0 || now_ms <= last) continue;
    if (now_ms - last > cfg_.max_age_ms) evict_at_locked(i, "age");
  }
}

// ---- introspection -------------------------------------------------------------------------
AmfStats AmfStore::stats() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  return stats_;
}
std::vector<AmfEntry> AmfStore::entries() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  return entries_;
}
std::uint64_t AmfStore::total_bytes() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  return total_bytes_;
}
std::uint64_t AmfStore::entry_count() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  return entries_.size();
}
double AmfStore::eviction_pressure() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  return eviction_pressure_;
}
void AmfStore::set_min_prompt_ms(double v) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (std::isfinite(v) && v >= 0.0) cfg_.min_prompt_ms = v;
}
void AmfStore::set_min_admit_roi(double v) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (std::isfinite(v) && v >= 0.0) cfg_.min_admit_roi = v;
}
void AmfStore::set_eviction_pressure(double v) {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (std::isfinite(v) && v >= 0.0) eviction_pressure_ = v;
}

AmfStorageStats AmfStore::storage_stats(std::uint64_t now_ms) const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  AmfStorageStats o;
  o.total_bytes = total_bytes_;
  o.budget_bytes = cfg_.storage_budget_bytes > 0 ? cfg_.storage_budget_bytes : cfg_.max_bytes;
  if (o.budget_bytes > 0) {
    o.utilization = static_cast<double>(o.total_bytes) / static_cast<double>(o.budget_bytes);
    if (!std::isfinite(o.utilization) || o.utilization < 0.0) o.utilization = 0.0;
  }
  if (now_ms == 0) now_ms = now_epoch_ms();
  for (const AmfEntry& e : entries_) {
    switch (tier_of(e, now_ms)) {
      case Tier::kHot: o.hot_entries++; break;
      case Tier::kWarm: o.warm_entries++; break;
      default: o.cold_entries++; break;
    }
  }
  std::error_code ec;
  const fs::space_info si = fs::space(dir_.empty() ? "." : dir_, ec);
  if (!ec) {
    o.disk_free_bytes = si.available;
    o.disk_capacity_bytes = si.capacity;
    if (si.capacity > 0) o.disk_free_ratio = static_cast<double>(si.available) / static_cast<double>(si.capacity);
    if (cfg_.disk_guard) {
      o.low_disk = (cfg_.min_free_disk_bytes > 0 && o.disk_free_bytes <= cfg_.min_free_disk_bytes) ||
                   (cfg_.min_free_disk_ratio > 0.0 && o.disk_free_ratio <= cfg_.min_free_disk_ratio);
    }
  }
  return o;
}

std::uint64_t AmfStore::oldest_entry_age_ms(std::uint64_t now_ms) const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (entries_.empty() || now_ms == 0) return 0;
  std::uint64_t oldest = 0;
  for (const AmfEntry& e : entries_) {
    const std::uint64_t l = last_access(e);
    if (l != 0 && (oldest == 0 || l < oldest)) oldest = l;
  }
  return (oldest == 0 || now_ms <= oldest) ? 0 : now_ms - oldest;
}

float AmfStore::reuse_score(std::size_t prompt_len, std::uint32_t prefix_len) const {
  if (prompt_len == 0 || prefix_len == 0) return 0.0f;
  const double r = static_cast<double>(prefix_len) / static_cast<double>(prompt_len);
  return std::isfinite(r) ? static_cast<float>(std::clamp(r, 0.0, 1.0)) : 0.0f;
}
float AmfStore::avg_prefix_length() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (entries_.empty()) return 0.0f;
  std::uint64_t s = 0;
  for (const AmfEntry& e : entries_) s += e.prefix_len;
  return static_cast<float>(static_cast<double>(s) / static_cast<double>(entries_.size()));
}
float AmfStore::historical_accept_rate() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  const double d = static_cast<double>(stats_.hits + stats_.misses);
  if (d <= 0.0) return 0.0f;
  return static_cast<float>(std::clamp(static_cast<double>(stats_.hits) / d, 0.0, 1.0));
}
float AmfStore::restore_cost_ms() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (stats_.hits == 0) return 0.0f;
  return static_cast<float>(static_cast<double>(stats_.restore_ms) / static_cast<double>(stats_.hits));
}

double AmfStore::warm_ratio() const {
  std::lock_guard<std::recursive_mutex> g(mu_);
  if (entries_.empty()) return 1.0;
  std::uint64_t warm = 0;
  for (const AmfEntry& e : entries_) {
    const auto st = static_cast<EntryState>(e.state);
    if (st == EntryState::kHot || (st == EntryState::kWarmPending && is_prewarmed(e.key))) warm++;
  }
  return static_cast<double>(warm) / static_cast<double>(entries_.size());
}

// ---- prewarm -------------------------------------------------------------------------------
bool AmfStore::is_prewarmed(const AmfKey& k) const {
  std::lock_guard<std::mutex> pg(prewarm_mu_);
  return prewarmed_.count(k) > 0;
}

void AmfStore::start_prewarm_locked() {
  if (!enabled_ || !cfg_.prewarm || entries_.empty()) {
    prewarm_running_.store(false);
    prewarm_complete_.store(true);
    return;
  }
  if (prewarm_thread_.joinable()) {
    prewarm_cancel_.store(true);
    prewarm_thread_.join();
    prewarm_cancel_.store(false);
  }
  prewarm_loaded_.store(0);
  prewarm_failed_.store(0);
  prewarm_running_.store(true);
  prewarm_complete_.store(false);
  prewarm_thread_ = std::thread(&AmfStore::run_prewarm, this, entries_);
}

void AmfStore::run_prewarm(std::vector<AmfEntry> ranked) {
  const auto t0 = std::chrono::steady_clock::now();
  std::sort(ranked.begin(), ranked.end(), [](const AmfEntry& a, const AmfEntry& b) {
    if (a.access_count != b.access_count) return a.access_count > b.access_count;
    return last_access(a) > last_access(b);
  });
  if (ranked.size() > cfg_.prewarm_top_k) ranked.resize(cfg_.prewarm_top_k);
  std::uint64_t loaded = 0, failed = 0;
  std::vector<std::uint8_t> blob;
  for (const AmfEntry& e : ranked) {
    if (prewarm_cancel_.load() || cfg_.prewarm_timeout_ms == 0) break;
    const auto el = std::chrono::duration_cast<std::chrono::milliseconds>(
                        std::chrono::steady_clock::now() - t0).count();
    if (static_cast<std::uint64_t>(el) >= cfg_.prewarm_timeout_ms) break;
    bool ok = read_file(kv_path(e.key), &blob);
    if (ok && e.kv_checksum > 0) ok = fnv1a_bytes(kFnvOffset, blob.data(), blob.size()) == e.kv_checksum;
    if (ok) {
      std::lock_guard<std::mutex> pg(prewarm_mu_);
      prewarmed_.insert(e.key);
      loaded++;
    } else {
      failed++;
    }
  }
  prewarm_loaded_.store(loaded);
  prewarm_failed_.store(failed);
  prewarm_running_.store(false);
  prewarm_complete_.store(true);
  const auto ms = std::chrono::duration_cast<std::chrono::milliseconds>(
                      std::chrono::steady_clock::now() - t0).count();
  log_line("[AMF_PREWARM] loaded=%llu failed=%llu total_ms=%llu\n", (unsigned long long)loaded,
           (unsigned long long)failed, (unsigned long long)ms);
}

}  // namespace axr
