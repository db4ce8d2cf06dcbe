// Multi-threaded stress test of the host runtime, built with sanitizers by
// tests/test_native_sanitizers.py (AddressSanitizer + UndefinedBehaviorSanitizer, and
// ThreadSanitizer):
//
//   * ShardDirectory (process-private): 6 threads insert / commit / abort / look up
//     (pinned) / unpin / remove / reclaim on 2 shards; afterwards every READY entry's
//     slots are distinct across the shard and the free-slot count adds up.
//   * NgramTable: 4 threads each grow their own tables token by token and check every
//     proposal against a plain scan of the window.
//   * AmfStore (temporary directory): 4 threads store entries and look up prefixes of
//     shared and private token streams while a fifth thread flushes the index and
//     evicts expired entries; the index then reloads with the same entry count.
//
// Exit code 0 = every check held; the sanitizers abort the process on a data race,
// leak, overflow or undefined behaviour.
#include <algorithm>
#include <atomic>
#include <chrono>
#include <cstdio>
#include <cstdlib>
#include <random>
#include <set>
#include <string>
#include <thread>
#include <vector>

#include "../amf_store.h"
#include "../ngram.h"
#include "../shard_dir.h"

using namespace axr;

static std::atomic<int> g_fail{0};
#define CHECK(c)                                                          \
  do {                                                                    \
    if (!(c)) {                                                           \
      std::fprintf(stderr, "CHECK failed %s:%d: %s\n", __FILE__, __LINE__, #c); \
      g_fail.fetch_add(1);                                                \
    }                                                                     \
  } while (0)

static void shard_dir_stress() {
  const int world = 2;
  ShardDirectory dir("", world, {96, 96}, 4096, 256, false);
  std::atomic<int> ops{0};
  auto worker = [&](int tid) {
    std::mt19937_64 rng(1234 + tid);
    for (int it = 0; it < 4000; ++it) {
      const int shard = static_cast<int>(rng() % world);
      const std::uint64_t key = 1 + rng() % 48;
      const std::uint64_t key2 = key * 7919;
      switch (rng() % 6) {
        case 0:
        case 1: {
          std::vector<std::int32_t> slots;
          std::vector<std::uint64_t> evicted;
          const std::uint32_t n = 1 + static_cast<std::uint32_t>(rng() % 6);
          const InsertStatus st =
              dir.begin_insert(shard, key, key2, n, n * 16, 0, tid, 1.0, &slots, &evicted);
          if (st == InsertStatus::kOk) {
            CHECK(slots.size() == n);
            if (rng() % 5 == 0)
              dir.abort(shard, key);
            else
              dir.commit(shard, key);
          }
          break;
        }
        case 2: {
          LookupOut o = dir.lookup(shard, key, key2, tid);
          if (o.found) {
            CHECK(o.slots.size() * 16 == o.n_tokens);
            dir.unpin(shard, key, tid);
          }
          break;
        }
        case 3:
          dir.contains(shard, key, key2);
          break;
        case 4:
          dir.remove(shard, key);
          break;
        default:
          dir.reclaim_stale(shard, 10.0);
          dir.info(shard);
          break;
      }
      ops.fetch_add(1);
    }
  };
  std::vector<std::thread> ts;
  for (int t = 0; t < 6; ++t) ts.emplace_back(worker, t);
  for (auto& t : ts) t.join();
  for (int s = 0; s < world; ++s) {
    const ShardInfo inf = dir.info(s);
    std::set<std::int32_t> used;
    std::uint32_t n_used = 0;
    for (const DirEntry& e : dir.entries(s)) {
      if (e.phase != static_cast<std::uint32_t>(EntryPhase::kReady)) continue;
      LookupOut o = dir.lookup(s, e.key, e.key2, 99);
      CHECK(o.found);
      for (std::int32_t sl : o.slots) {
        CHECK(sl >= 0 && sl < static_cast<std::int32_t>(inf.n_slots));
        CHECK(used.insert(sl).second);  // no slot owned by two entries
      }
      n_used += static_cast<std::uint32_t>(o.slots.size());
      dir.unpin(s, e.key, 99);
    }
    CHECK(dir.info(s).free_slots + n_used <= inf.n_slots);
  }
  std::printf("shard_dir ops=%d\n", ops.load());
}

static void amf_store_stress(const std::string& root) {
  StoreConfig cfg;
  cfg.min_tokens = 16;
  cfg.max_bytes = 64ull << 20;
  cfg.storage_budget_bytes = 64ull << 20;
  cfg.disk_guard = false;
  std::uint64_t n_entries = 0;
  {
    AmfStore st;
    CHECK(st.init(root, cfg));
    AmfContext ctx;
    ctx.model_hash = 0x1234;
    ctx.tenant_hash = 0x99;
    ctx.n_ctx = 4096;
    ctx.kv_version = 1;
    std::vector<std::int32_t> shared(512);
    for (int i = 0; i < 512; ++i) shared[i] = 1000 + i;
    std::atomic<bool> stop{false};
    auto worker = [&](int tid) {
      std::mt19937 rng(77 + tid);
      std::vector<std::uint8_t> blob(8192);
      for (std::size_t i = 0; i < blob.size(); ++i) blob[i] = static_cast<std::uint8_t>(i * 31 + tid);
      for (int it = 0; it < 150; ++it) {
        std::vector<std::int32_t> toks;
        const bool use_shared = rng() % 2 == 0;
        const std::size_t n = 32 + (rng() % 16) * 16;
        for (std::size_t i = 0; i < n; ++i)
          toks.push_back(use_shared ? shared[i] : static_cast<std::int32_t>(tid * 100000 + it * 600 + i));
        AmfEntry e;
        std::vector<std::int32_t> got;
        const Lookup r = st.find_longest_prefix(ctx, toks.data(), toks.size(), &e, &got);
        if (r == Lookup::kHit) {
          std::vector<std::uint8_t> kv;
          if (st.load_kv(e, &kv)) st.note_hit(e, got.size(), 1, 5);
        } else {
          st.note_miss();
          st.store_entry(ctx, toks.data(), toks.size(), blob.data(), blob.size(), 20);
        }
      }
    };
    std::thread flusher([&] {
      while (!stop.load()) {
        st.flush();
        st.evict_expired_entries(0);
        st.stats();
        std::this_thread::sleep_for(std::chrono::milliseconds(2));
      }
    });
    std::vector<std::thread> ts;
    for (int t = 0; t < 4; ++t) ts.emplace_back(worker, t);
    for (auto& t : ts) t.join();
    stop.store(true);
    flusher.join();
    CHECK(st.flush());
    n_entries = st.entry_count();
    CHECK(n_entries > 0);
    st.shutdown();
  }
  AmfStore again;
  CHECK(again.init(root, cfg));
  CHECK(again.entry_count() == n_entries);
  std::printf("amf_store entries=%llu\n", static_cast<unsigned long long>(n_entries));
}

// Proposal by scanning the window (the definition the index must reproduce).
static std::vector<std::int32_t> scan_propose(const std::vector<std::int32_t>& all, int max_n, int min_n, int window,
                                              int k, int skip) {
  const long long L = static_cast<long long>(all.size()), lo = std::max(0LL, L - window);
  for (int n = max_n; n >= min_n; --n) {
    if (L - lo <= n) continue;
    int left = skip;
    for (long long i = L - n - 1; i >= lo; --i) {
      bool eq = true;
      for (int j = 0; j < n && eq; ++j) eq = all[i + j] == all[L - n + j];
      if (!eq) continue;
      if (left > 0) { --left; continue; }
      std::vector<std::int32_t> out(all.begin() + i + n, all.begin() + std::min(L, i + n + k));
      while (static_cast<int>(out.size()) < k) out.push_back(out.back());
      return out;
    }
  }
  return std::vector<std::int32_t>(k, L ? all.back() : 0);
}

static void ngram_stress() {
  std::vector<std::thread> ts;
  for (int t = 0; t < 4; ++t) {
    ts.emplace_back([t] {
      std::mt19937 rng(1234 + t);
      for (int trial = 0; trial < 20; ++trial) {
        const int vocab = 2 + static_cast<int>(rng() % 40), max_n = 1 + static_cast<int>(rng() % 5);
        const int min_n = 1 + static_cast<int>(rng() % max_n), window = 8 + static_cast<int>(rng() % 300);
        NgramTable tab(max_n, min_n, window);
        std::vector<std::int32_t> all;
        for (int step = 0; step < 300; ++step) {
          const int add = 1 + static_cast<int>(rng() % 4);
          std::vector<std::int32_t> fresh;
          for (int a = 0; a < add; ++a) fresh.push_back(static_cast<std::int32_t>(rng() % vocab));
          tab.extend(fresh.data(), fresh.size());
          all.insert(all.end(), fresh.begin(), fresh.end());
          const int k = 1 + static_cast<int>(rng() % 8), skip = static_cast<int>(rng() % 3);
          CHECK(tab.propose(k, skip) == scan_propose(all, max_n, min_n, window, k, skip));
        }
      }
    });
  }
  for (auto& th : ts) th.join();
}

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s <empty temp dir>\n", argv[0]);
    return 2;
  }
  shard_dir_stress();
  ngram_stress();
  amf_store_stress(argv[1]);
  if (g_fail.load() != 0) {
    std::fprintf(stderr, "%d check(s) failed\n", g_fail.load());
    return 1;
  }
  std::printf("native_stress ok\n");
  return 0;
}
