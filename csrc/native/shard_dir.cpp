// Shard directory implementation (see shard_dir.h).
#include "shard_dir.h"

#include <errno.h>
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <functional>
#include <chrono>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>

namespace axr {

namespace {
constexpr std::uint64_t kMagic = 0x52494453464d4158ull;  // "XAMFSDIR"
constexpr std::uint32_t kVersion = 1;
constexpr double kAlpha = 0.3, kBeta = 0.4, kGamma = 0.1, kDelta = 0.2;

std::size_t align64(std::size_t x) { return (x + 63) & ~std::size_t(63); }

std::uint64_t mix64(std::uint64_t x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return x;
}

constexpr int kMaxLens = 256;

struct GlobalHdr {
  std::uint64_t magic;
  std::uint32_t version;
  std::uint32_t world;
  std::uint32_t entry_cap;
  std::uint32_t ready;
  std::uint64_t total_bytes;
  std::uint64_t shard_off[kMaxRanks];
  // Distinct prefix lengths (tokens) of READY entries over all shards, with counts:
  // lookups probe only these lengths when searching the longest cached prefix.
  pthread_mutex_t len_mu;
  std::uint32_t n_lens;
  std::uint32_t len_val[kMaxLens];
  std::uint32_t len_cnt[kMaxLens];
};

struct ShardHdr {
  pthread_mutex_t mu;
  std::uint32_t n_slots;
  std::uint32_t free_top;
  std::uint64_t chunk_bytes;
  std::uint32_t entry_cap;
  std::uint32_t n_live;
  std::uint32_t n_tombs;
  std::uint32_t pad;
  ShardStats stats;
};

std::size_t shard_bytes(std::uint32_t n_slots, std::uint32_t cap) {
  return align64(sizeof(ShardHdr)) + 2 * align64(sizeof(std::int32_t) * n_slots) +
         align64(sizeof(DirEntry) * cap);
}

int pins_total(const DirEntry& e) {
  int t = 0;
  for (int r = 0; r < kMaxRanks; ++r) t += e.pins[r];
  return t;
}
}  // namespace

std::uint64_t mono_ns() {
  return static_cast<std::uint64_t>(std::chrono::duration_cast<std::chrono::nanoseconds>(
                                        std::chrono::steady_clock::now().time_since_epoch())
                                        .count());
}

struct ShardDirectory::Layout {
  GlobalHdr* g;
  ShardHdr* hdr[kMaxRanks];
  std::int32_t* free_stack[kMaxRanks];
  std::int32_t* next_slot[kMaxRanks];
  DirEntry* table[kMaxRanks];
};

struct ShardDirectory::Guard {
  ShardDirectory* d;
  int s;
  Guard(ShardDirectory* dir, int shard) : d(dir), s(shard) { d->lock(s); }
  ~Guard() { d->unlock(s); }
};

ShardDirectory::ShardDirectory(const std::string& name, int world,
                               const std::vector<std::uint32_t>& n_slots,
                               std::uint64_t chunk_bytes, std::uint32_t entry_cap, bool attach,
                               double lock_timeout_s)
    : name_(name), lock_timeout_s_(lock_timeout_s) {
  if (world <= 0 || world > kMaxRanks) throw std::invalid_argument("world must be in [1, 32]");
  std::uint32_t cap = 16;
  while (cap < entry_cap) cap <<= 1;
  if (!attach && static_cast<int>(n_slots.size()) != world)
    throw std::invalid_argument("n_slots must have one entry per shard");

  if (attach) {
    if (name.empty()) throw std::invalid_argument("attach needs a shared-memory name");
    int fd = -1;
    const auto deadline = std::chrono::steady_clock::now() + std::chrono::seconds(30);
    while ((fd = shm_open(name.c_str(), O_RDWR, 0600)) < 0) {
      if (std::chrono::steady_clock::now() > deadline)
        throw std::runtime_error("shard directory " + name + " not found (creator missing)");
      std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    struct stat st{};
    // The creator sizes the object before publishing `ready`; wait for a non-zero size.
    while (fstat(fd, &st) == 0 && st.st_size == 0) {
      if (std::chrono::steady_clock::now() > deadline) {
        close(fd);
        throw std::runtime_error("shard directory " + name + " never sized");
      }
      std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    bytes_ = static_cast<std::size_t>(st.st_size);
    base_ = mmap(nullptr, bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (base_ == MAP_FAILED) throw std::runtime_error("mmap of shard directory failed");
    auto* g = static_cast<GlobalHdr*>(base_);
    while (__atomic_load_n(&g->ready, __ATOMIC_ACQUIRE) == 0) {
      if (std::chrono::steady_clock::now() > deadline)
        throw std::runtime_error("shard directory " + name + " never became ready");
      std::this_thread::sleep_for(std::chrono::milliseconds(5));
    }
    if (g->magic != kMagic || g->version != kVersion)
      throw std::runtime_error("shard directory " + name + " has a foreign layout");
    world = static_cast<int>(g->world);
  } else {
    std::size_t total = align64(sizeof(GlobalHdr));
    std::vector<std::size_t> offs(world);
    for (int s = 0; s < world; ++s) {
      offs[s] = total;
      total += shard_bytes(n_slots[s], cap);
    }
    bytes_ = total;
    if (name.empty()) {
      base_ = mmap(nullptr, bytes_, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_ANONYMOUS, -1, 0);
    } else {
      shm_unlink(name.c_str());  // a stale object from a crashed job
      int fd = shm_open(name.c_str(), O_RDWR | O_CREAT | O_EXCL, 0600);
      if (fd < 0) throw std::runtime_error("shm_open(" + name + ") failed: " + std::strerror(errno));
      if (ftruncate(fd, static_cast<off_t>(bytes_)) != 0) {
        close(fd);
        shm_unlink(name.c_str());
        throw std::runtime_error("ftruncate of shard directory failed");
      }
      base_ = mmap(nullptr, bytes_, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
      close(fd);
    }
    if (base_ == MAP_FAILED) throw std::runtime_error("mmap of shard directory failed");
    owner_ = true;
    std::memset(base_, 0, bytes_);
    auto* g = static_cast<GlobalHdr*>(base_);
    g->magic = kMagic;
    g->version = kVersion;
    g->world = static_cast<std::uint32_t>(world);
    g->entry_cap = cap;
    g->total_bytes = bytes_;
    for (int s = 0; s < world; ++s) g->shard_off[s] = offs[s];
  }

  lay_ = new Layout{};
  lay_->g = static_cast<GlobalHdr*>(base_);
  auto* base = static_cast<std::uint8_t*>(base_);
  for (int s = 0; s < world; ++s) {
    std::uint8_t* p = base + lay_->g->shard_off[s];
    lay_->hdr[s] = reinterpret_cast<ShardHdr*>(p);
    const std::uint32_t ns = attach ? lay_->hdr[s]->n_slots : n_slots[s];
    p += align64(sizeof(ShardHdr));
    lay_->free_stack[s] = reinterpret_cast<std::int32_t*>(p);
    p += align64(sizeof(std::int32_t) * ns);
    lay_->next_slot[s] = reinterpret_cast<std::int32_t*>(p);
    p += align64(sizeof(std::int32_t) * ns);
    lay_->table[s] = reinterpret_cast<DirEntry*>(p);
  }
  if (!attach) {
    for (int s = 0; s < world; ++s) {
      ShardHdr* h = lay_->hdr[s];
      pthread_mutexattr_t a;
      pthread_mutexattr_init(&a);
      pthread_mutexattr_setpshared(&a, PTHREAD_PROCESS_SHARED);
      pthread_mutexattr_setrobust(&a, PTHREAD_MUTEX_ROBUST);
      pthread_mutex_init(&h->mu, &a);
      pthread_mutexattr_destroy(&a);
      h->n_slots = n_slots[s];
      h->chunk_bytes = chunk_bytes;
      h->entry_cap = cap;
      // Pop order: slot 0 first, so small pools fill from the start of the slab.
      h->free_top = n_slots[s];
      for (std::uint32_t i = 0; i < n_slots[s]; ++i)
        lay_->free_stack[s][i] = static_cast<std::int32_t>(n_slots[s] - 1 - i);
      for (std::uint32_t i = 0; i < n_slots[s]; ++i) lay_->next_slot[s][i] = -1;
    }
    {
      pthread_mutexattr_t a;
      pthread_mutexattr_init(&a);
      pthread_mutexattr_setpshared(&a, PTHREAD_PROCESS_SHARED);
      pthread_mutexattr_setrobust(&a, PTHREAD_MUTEX_ROBUST);
      pthread_mutex_init(&lay_->g->len_mu, &a);
      pthread_mutexattr_destroy(&a);
    }
    __atomic_store_n(&lay_->g->ready, 1u, __ATOMIC_RELEASE);
  }
}

void ShardDirectory::note_len(std::uint32_t n_tokens, int delta) {
  GlobalHdr* g = lay_->g;
  int rc = pthread_mutex_lock(&g->len_mu);
  if (rc == EOWNERDEAD) pthread_mutex_consistent(&g->len_mu);
  else if (rc != 0) return;
  int idx = -1;
  for (std::uint32_t i = 0; i < g->n_lens; ++i)
    if (g->len_val[i] == n_tokens) { idx = static_cast<int>(i); break; }
  if (delta > 0) {
    if (idx < 0 && g->n_lens < static_cast<std::uint32_t>(kMaxLens)) {
      idx = static_cast<int>(g->n_lens++);
      g->len_val[idx] = n_tokens;
      g->len_cnt[idx] = 0;
    }
    if (idx >= 0) g->len_cnt[idx] += 1;
  } else if (idx >= 0) {
    if (g->len_cnt[idx] > 0) g->len_cnt[idx] -= 1;
    if (g->len_cnt[idx] == 0) {  // swap-remove
      const std::uint32_t last = g->n_lens - 1;
      g->len_val[idx] = g->len_val[last];
      g->len_cnt[idx] = g->len_cnt[last];
      g->n_lens = last;
    }
  }
  pthread_mutex_unlock(&g->len_mu);
}

std::vector<std::uint32_t> ShardDirectory::lengths() {
  GlobalHdr* g = lay_->g;
  std::vector<std::uint32_t> out;
  int rc = pthread_mutex_lock(&g->len_mu);
  if (rc == EOWNERDEAD) pthread_mutex_consistent(&g->len_mu);
  else if (rc != 0) return out;
  out.assign(g->len_val, g->len_val + g->n_lens);
  pthread_mutex_unlock(&g->len_mu);
  std::sort(out.begin(), out.end(), std::greater<std::uint32_t>());
  return out;
}

ShardDirectory::~ShardDirectory() {
  delete lay_;
  if (base_ && base_ != MAP_FAILED) munmap(base_, bytes_);
  if (owner_ && !name_.empty()) shm_unlink(name_.c_str());
}

int ShardDirectory::world() const { return static_cast<int>(lay_->g->world); }
std::uint64_t ShardDirectory::chunk_bytes(int shard) const { return lay_->hdr[shard]->chunk_bytes; }

void ShardDirectory::lock(int s) {
  if (s < 0 || s >= world()) throw std::out_of_range("shard index out of range");
  timespec ts{};
  clock_gettime(CLOCK_REALTIME, &ts);
  const double secs = std::floor(lock_timeout_s_);
  ts.tv_sec += static_cast<time_t>(secs);
  ts.tv_nsec += static_cast<long>((lock_timeout_s_ - secs) * 1e9);
  if (ts.tv_nsec >= 1000000000L) { ts.tv_sec += 1; ts.tv_nsec -= 1000000000L; }
  const int rc = pthread_mutex_timedlock(&lay_->hdr[s]->mu, &ts);
  if (rc == EOWNERDEAD) {
    // The previous holder died mid-update; the shard's fields are each updated in a
    // single store, so the structure is usable — mark it consistent and go on.
    pthread_mutex_consistent(&lay_->hdr[s]->mu);
    return;
  }
  if (rc == ETIMEDOUT) throw std::runtime_error("shard directory lock timed out");
  if (rc != 0) throw std::runtime_error("shard directory lock failed");
}

void ShardDirectory::unlock(int s) { pthread_mutex_unlock(&lay_->hdr[s]->mu); }

DirEntry* ShardDirectory::find_locked(int s, std::uint64_t key, std::uint64_t key2) {
  const std::uint32_t cap = lay_->hdr[s]->entry_cap;
  DirEntry* t = lay_->table[s];
  std::uint32_t i = static_cast<std::uint32_t>(mix64(key)) & (cap - 1);
  for (std::uint32_t n = 0; n < cap; ++n, i = (i + 1) & (cap - 1)) {
    DirEntry& e = t[i];
    if (e.phase == static_cast<std::uint32_t>(EntryPhase::kEmpty)) return nullptr;
    if (e.phase != static_cast<std::uint32_t>(EntryPhase::kTomb) && e.key == key &&
        (key2 == 0 || e.key2 == key2))
      return &e;
  }
  return nullptr;
}

DirEntry* ShardDirectory::slot_for_insert_locked(int s, std::uint64_t key) {
  ShardHdr* h = lay_->hdr[s];
  const std::uint32_t cap = h->entry_cap;
  if (h->n_live + 1 > cap - cap / 8) return nullptr;  // keep probe chains short
  DirEntry* t = lay_->table[s];
  if (h->n_tombs > cap / 4) {
    // Rehash in place: collect live entries, clear, reinsert.
    std::vector<DirEntry> live;
    live.reserve(h->n_live);
    for (std::uint32_t i = 0; i < cap; ++i) {
      const auto ph = static_cast<EntryPhase>(t[i].phase);
      if (ph == EntryPhase::kWriting || ph == EntryPhase::kReady) live.push_back(t[i]);
    }
    std::memset(t, 0, sizeof(DirEntry) * cap);
    for (const DirEntry& e : live) {
      std::uint32_t i = static_cast<std::uint32_t>(mix64(e.key)) & (cap - 1);
      while (t[i].phase != 0) i = (i + 1) & (cap - 1);
      t[i] = e;
    }
    h->n_tombs = 0;
  }
  std::uint32_t i = static_cast<std::uint32_t>(mix64(key)) & (cap - 1);
  for (std::uint32_t n = 0; n < cap; ++n, i = (i + 1) & (cap - 1)) {
    const auto ph = static_cast<EntryPhase>(t[i].phase);
    if (ph == EntryPhase::kEmpty) return &t[i];
    if (ph == EntryPhase::kTomb) {
      h->n_tombs -= 1;
      return &t[i];
    }
  }
  return nullptr;
}

void ShardDirectory::free_chain_locked(int s, DirEntry* e) {
  ShardHdr* h = lay_->hdr[s];
  if (e->phase == static_cast<std::uint32_t>(EntryPhase::kReady)) note_len(e->n_tokens, -1);
  std::int32_t slot = e->first_slot;
  std::uint32_t n = 0;
  while (slot >= 0 && n < e->n_chunks) {
    const std::int32_t nxt = lay_->next_slot[s][slot];
    lay_->next_slot[s][slot] = -1;
    lay_->free_stack[s][h->free_top++] = slot;
    slot = nxt;
    ++n;
  }
  e->phase = static_cast<std::uint32_t>(EntryPhase::kTomb);
  e->key = 0;
  e->first_slot = -1;
  h->n_live -= 1;
  h->n_tombs += 1;
}

double ShardDirectory::score_locked(const DirEntry& e, std::uint64_t now_ns,
                                    std::uint64_t chunk_bytes) const {
  const double age_s = now_ns > e.last_hit_ns ? (now_ns - e.last_hit_ns) / 1e9 : 0.0;
  const double hits = e.hit_count > 0 ? static_cast<double>(e.hit_count) : 1.0;
  const double size_mb = static_cast<double>(e.n_chunks) * static_cast<double>(chunk_bytes) / (1 << 20);
  const double sav = e.avg_savings_ms > 0.0 ? e.avg_savings_ms : 0.0;
  return kAlpha * age_s + kBeta / hits + kGamma * size_mb - kDelta * sav;
}

bool ShardDirectory::evict_one_locked(int s, std::vector<std::uint64_t>* evicted) {
  ShardHdr* h = lay_->hdr[s];
  DirEntry* t = lay_->table[s];
  const std::uint64_t now = mono_ns();
  DirEntry* worst = nullptr;
  double worst_score = -INFINITY;
  for (std::uint32_t i = 0; i < h->entry_cap; ++i) {
    DirEntry& e = t[i];
    if (e.phase != static_cast<std::uint32_t>(EntryPhase::kReady) || pins_total(e) > 0) continue;
    const double sc = score_locked(e, now, h->chunk_bytes);
    if (sc > worst_score) {
      worst_score = sc;
      worst = &e;
    }
  }
  if (!worst) return false;
  if (evicted) evicted->push_back(worst->key);
  h->stats.evictions += 1;
  h->stats.bytes_evicted += worst->nbytes;
  free_chain_locked(s, worst);
  return true;
}

LookupOut ShardDirectory::lookup(int s, std::uint64_t key, std::uint64_t key2, int pin_rank) {
  Guard g(this, s);
  LookupOut out;
  DirEntry* e = find_locked(s, key, key2);
  ShardHdr* h = lay_->hdr[s];
  if (!e || e->phase != static_cast<std::uint32_t>(EntryPhase::kReady)) {
    h->stats.misses += 1;
    return out;
  }
  out.found = true;
  out.n_tokens = e->n_tokens;
  out.fmt = e->fmt;
  out.slots.reserve(e->n_chunks);
  std::int32_t slot = e->first_slot;
  for (std::uint32_t i = 0; i < e->n_chunks && slot >= 0; ++i) {
    out.slots.push_back(slot);
    slot = lay_->next_slot[s][slot];
  }
  e->hit_count += 1;
  e->last_hit_ns = mono_ns();
  h->stats.hits += 1;
  if (pin_rank >= 0 && pin_rank < kMaxRanks) e->pins[pin_rank] += 1;
  return out;
}

bool ShardDirectory::contains(int s, std::uint64_t key, std::uint64_t key2) {
  Guard g(this, s);
  DirEntry* e = find_locked(s, key, key2);
  return e && e->phase == static_cast<std::uint32_t>(EntryPhase::kReady);
}

void ShardDirectory::unpin(int s, std::uint64_t key, int rank) {
  Guard g(this, s);
  DirEntry* e = find_locked(s, key, 0);
  if (e && rank >= 0 && rank < kMaxRanks && e->pins[rank] > 0) e->pins[rank] -= 1;
}

InsertStatus ShardDirectory::begin_insert(int s, std::uint64_t key, std::uint64_t key2,
                                          std::uint32_t n_chunks, std::uint32_t n_tokens,
                                          std::uint32_t fmt, int writer, double savings_ms,
                                          std::vector<std::int32_t>* slots,
                                          std::vector<std::uint64_t>* evicted) {
  Guard g(this, s);
  ShardHdr* h = lay_->hdr[s];
  slots->clear();
  if (key == 0) throw std::invalid_argument("key 0 is reserved");
  if (n_chunks == 0 || n_chunks > h->n_slots) {
    h->stats.alloc_failures += 1;
    return InsertStatus::kTooLarge;
  }
  if (DirEntry* e = find_locked(s, key, key2)) {
    if (e->phase == static_cast<std::uint32_t>(EntryPhase::kReady)) return InsertStatus::kExists;
    h->stats.busy += 1;
    return InsertStatus::kBusy;
  }
  while (h->free_top < n_chunks) {
    if (!evict_one_locked(s, evicted)) {
      h->stats.alloc_failures += 1;
      return InsertStatus::kNoSpace;
    }
  }
  DirEntry* e = slot_for_insert_locked(s, key);
  if (!e) {
    if (!evict_one_locked(s, evicted) || !(e = slot_for_insert_locked(s, key))) {
      h->stats.alloc_failures += 1;
      return InsertStatus::kNoSpace;
    }
  }
  std::memset(e, 0, sizeof(DirEntry));
  slots->resize(n_chunks);
  std::int32_t prev = -1;
  for (std::uint32_t i = 0; i < n_chunks; ++i) {
    const std::int32_t sl = lay_->free_stack[s][--h->free_top];
    (*slots)[i] = sl;
    lay_->next_slot[s][sl] = -1;
    if (prev >= 0) lay_->next_slot[s][prev] = sl;
    else e->first_slot = sl;
    prev = sl;
  }
  const std::uint64_t now = mono_ns();
  e->key = key;
  e->key2 = key2;
  e->phase = static_cast<std::uint32_t>(EntryPhase::kWriting);
  e->n_tokens = n_tokens;
  e->n_chunks = n_chunks;
  e->writer = writer;
  e->fmt = fmt;
  e->created_ns = e->last_hit_ns = e->phase_ns = now;
  e->nbytes = static_cast<std::uint64_t>(n_chunks) * h->chunk_bytes;
  e->avg_savings_ms = savings_ms;
  h->n_live += 1;
  return InsertStatus::kOk;
}

bool ShardDirectory::commit(int s, std::uint64_t key) {
  Guard g(this, s);
  DirEntry* e = find_locked(s, key, 0);
  if (!e || e->phase != static_cast<std::uint32_t>(EntryPhase::kWriting)) return false;
  e->phase = static_cast<std::uint32_t>(EntryPhase::kReady);
  e->phase_ns = mono_ns();
  note_len(e->n_tokens, +1);
  ShardHdr* h = lay_->hdr[s];
  h->stats.inserts += 1;
  h->stats.bytes_stored += e->nbytes;
  return true;
}

bool ShardDirectory::abort(int s, std::uint64_t key) {
  Guard g(this, s);
  DirEntry* e = find_locked(s, key, 0);
  if (!e || e->phase != static_cast<std::uint32_t>(EntryPhase::kWriting)) return false;
  free_chain_locked(s, e);
  return true;
}

bool ShardDirectory::remove(int s, std::uint64_t key) {
  Guard g(this, s);
  DirEntry* e = find_locked(s, key, 0);
  if (!e || e->phase != static_cast<std::uint32_t>(EntryPhase::kReady) || pins_total(*e) > 0)
    return false;
  free_chain_locked(s, e);
  return true;
}

void ShardDirectory::clear(int s) {
  Guard g(this, s);
  ShardHdr* h = lay_->hdr[s];
  for (std::uint32_t i = 0; i < h->entry_cap; ++i) {
    DirEntry& e = lay_->table[s][i];
    if (e.phase == static_cast<std::uint32_t>(EntryPhase::kReady) && pins_total(e) == 0)
      free_chain_locked(s, &e);
  }
}

std::uint32_t ShardDirectory::release_rank(int rank) {
  std::uint32_t n = 0;
  for (int s = 0; s < world(); ++s) {
    Guard g(this, s);
    ShardHdr* h = lay_->hdr[s];
    for (std::uint32_t i = 0; i < h->entry_cap; ++i) {
      DirEntry& e = lay_->table[s][i];
      if (e.phase == static_cast<std::uint32_t>(EntryPhase::kEmpty) ||
          e.phase == static_cast<std::uint32_t>(EntryPhase::kTomb))
        continue;
      if (rank >= 0 && rank < kMaxRanks && e.pins[rank] > 0) {
        e.pins[rank] = 0;
        ++n;
      }
      if (e.phase == static_cast<std::uint32_t>(EntryPhase::kWriting) && e.writer == rank) {
        free_chain_locked(s, &e);
        h->stats.reclaimed += 1;
        ++n;
      }
    }
  }
  return n;
}

std::uint32_t ShardDirectory::reclaim_stale(int s, double max_age_s) {
  Guard g(this, s);
  ShardHdr* h = lay_->hdr[s];
  const std::uint64_t now = mono_ns();
  std::uint32_t n = 0;
  for (std::uint32_t i = 0; i < h->entry_cap; ++i) {
    DirEntry& e = lay_->table[s][i];
    if (e.phase == static_cast<std::uint32_t>(EntryPhase::kWriting) &&
        static_cast<double>(now - e.phase_ns) / 1e9 > max_age_s) {
      free_chain_locked(s, &e);
      h->stats.reclaimed += 1;
      ++n;
    }
  }
  return n;
}

ShardInfo ShardDirectory::info(int s) {
  Guard g(this, s);
  ShardHdr* h = lay_->hdr[s];
  ShardInfo o{};
  o.n_slots = h->n_slots;
  o.free_slots = h->free_top;
  o.chunk_bytes = h->chunk_bytes;
  o.entries = h->n_live;
  o.entry_cap = h->entry_cap;
  o.stats = h->stats;
  return o;
}

std::vector<DirEntry> ShardDirectory::entries(int s) {
  Guard g(this, s);
  std::vector<DirEntry> out;
  ShardHdr* h = lay_->hdr[s];
  for (std::uint32_t i = 0; i < h->entry_cap; ++i) {
    const DirEntry& e = lay_->table[s][i];
    if (e.phase == static_cast<std::uint32_t>(EntryPhase::kWriting) ||
        e.phase == static_cast<std::uint32_t>(EntryPhase::kReady))
      out.push_back(e);
  }
  return out;
}

void ShardDirectory::note_savings(int s, std::uint64_t key, double savings_ms) {
  Guard g(this, s);
  DirEntry* e = find_locked(s, key, 0);
  if (!e) return;
  // Running mean over hits (the reference keeps one per-entry average).
  const double n = static_cast<double>(e->hit_count > 0 ? e->hit_count : 1);
  e->avg_savings_ms += (savings_ms - e->avg_savings_ms) / n;
}

}  // namespace axr
