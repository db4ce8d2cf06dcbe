// Python bindings of the host-native runtime (no CUDA, no torch): AMF disk store,
// shard directory, hashing, and the runtime controllers.
#include <pybind11/numpy.h>
#include <pybind11/pybind11.h>
#include <pybind11/stl.h>

#include "amf_store.h"
#include "fnv.h"
#include "ngram.h"
#include "runtime.h"
#include "shard_dir.h"

namespace py = pybind11;
using namespace axr;

namespace {

using I32Array = py::array_t<std::int32_t, py::array::c_style | py::array::forcecast>;

py::dict entry_to_dict(const AmfEntry& e) {
  py::dict d;
  d["model_hash"] = e.key.model_hash;
  d["tenant_hash"] = e.key.tenant_hash;
  d["prefix_hash"] = e.key.prefix_hash;
  d["n_ctx"] = e.key.n_ctx;
  d["kv_version"] = e.key.kv_version;
  d["rope_base_bits"] = e.key.rope_base_bits;
  d["rope_scale_bits"] = e.key.rope_scale_bits;
  d["sampling_hash"] = e.key.sampling_hash;
  d["rng_hash"] = e.key.rng_hash;
  d["entry_model_hash"] = e.model_hash;
  d["prefix_len"] = e.prefix_len;
  d["seen_count"] = e.seen_count;
  d["restore_count"] = e.restore_count;
  d["ema_saved_ms"] = e.ema_saved_ms;
  d["ema_restore_ms"] = e.ema_restore_ms;
  d["ema_roi"] = e.ema_roi;
  d["failure_count"] = e.failure_count;
  d["block_count"] = e.block_count;
  d["saved_ms"] = e.saved_ms;
  d["hit_count"] = e.hit_count;
  d["last_used"] = e.last_used;
  d["last_hit_ms"] = e.last_hit_ms;
  d["low_roi_hits"] = e.low_roi_hits;
  d["kv_size"] = e.kv_size;
  d["last_access_time_ms"] = e.last_access_time_ms;
  d["access_count"] = e.access_count;
  d["stored_at_ms"] = e.stored_at_ms;
  d["expires_at_ms"] = e.expires_at_ms;
  d["size_bytes"] = e.size_bytes;
  d["kv_checksum"] = e.kv_checksum;
  d["state"] = e.state;
  return d;
}

AmfEntry entry_from_dict(const py::dict& d) {
  AmfEntry e;
  auto u64 = [&](const char* k, std::uint64_t dflt = 0) {
    return d.contains(k) ? d[k].cast<std::uint64_t>() : dflt;
  };
  auto f64 = [&](const char* k) { return d.contains(k) ? d[k].cast<double>() : kNaN; };
  e.key.model_hash = u64("model_hash");
  e.key.tenant_hash = u64("tenant_hash");
  e.key.prefix_hash = u64("prefix_hash");
  e.key.n_ctx = static_cast<std::uint32_t>(u64("n_ctx"));
  e.key.kv_version = static_cast<std::uint32_t>(u64("kv_version"));
  e.key.rope_base_bits = static_cast<std::uint32_t>(u64("rope_base_bits"));
  e.key.rope_scale_bits = static_cast<std::uint32_t>(u64("rope_scale_bits"));
  e.key.sampling_hash = u64("sampling_hash");
  e.key.rng_hash = u64("rng_hash");
  e.model_hash = u64("entry_model_hash", e.key.model_hash);
  e.prefix_len = static_cast<std::uint32_t>(u64("prefix_len"));
  e.seen_count = u64("seen_count");
  e.restore_count = u64("restore_count");
  e.ema_saved_ms = f64("ema_saved_ms");
  e.ema_restore_ms = f64("ema_restore_ms");
  e.ema_roi = f64("ema_roi");
  e.failure_count = u64("failure_count");
  e.block_count = u64("block_count");
  e.saved_ms = u64("saved_ms");
  e.hit_count = u64("hit_count");
  e.last_used = u64("last_used");
  e.last_hit_ms = u64("last_hit_ms");
  e.low_roi_hits = static_cast<std::uint32_t>(u64("low_roi_hits"));
  e.kv_size = u64("kv_size");
  e.last_access_time_ms = u64("last_access_time_ms");
  e.access_count = u64("access_count");
  e.stored_at_ms = u64("stored_at_ms");
  e.expires_at_ms = u64("expires_at_ms");
  e.size_bytes = u64("size_bytes");
  e.kv_checksum = u64("kv_checksum");
  e.state = static_cast<std::uint8_t>(u64("state"));
  return e;
}

AmfContext ctx_from_dict(const py::dict& d) {
  AmfContext c;
  auto u64 = [&](const char* k) { return d.contains(k) ? d[k].cast<std::uint64_t>() : 0ull; };
  c.model_hash = u64("model_hash");
  c.tenant_hash = u64("tenant_hash");
  c.n_ctx = static_cast<std::uint32_t>(u64("n_ctx"));
  c.kv_version = static_cast<std::uint32_t>(u64("kv_version"));
  c.rope_base_bits = static_cast<std::uint32_t>(u64("rope_base_bits"));
  c.rope_scale_bits = static_cast<std::uint32_t>(u64("rope_scale_bits"));
  c.sampling_hash = u64("sampling_hash");
  c.rng_hash = u64("rng_hash");
  return c;
}

py::dict stats_to_dict(const AmfStats& s) {
  py::dict d;
  d["hits"] = s.hits;
  d["misses"] = s.misses;
  d["tokens_saved"] = s.tokens_saved;
  d["ms_saved"] = s.ms_saved;
  d["restore_ms"] = s.restore_ms;
  d["saved_ms_ema"] = s.saved_ms_ema;
  d["restore_ms_ema"] = s.restore_ms_ema;
  d["failures"] = s.failures;
  d["blocks"] = s.blocks;
  d["admissions"] = s.admissions;
  d["admission_rejects"] = s.admission_rejects;
  d["admission_bytes"] = s.admission_bytes;
  d["store_failures"] = s.store_failures;
  d["evictions"] = s.evictions;
  d["evicted_bytes"] = s.evicted_bytes;
  d["entries"] = s.entries;
  d["bytes"] = s.bytes;
  return d;
}

py::dict dir_entry_to_dict(const DirEntry& e) {
  py::dict d;
  d["key"] = e.key;
  d["key2"] = e.key2;
  d["phase"] = e.phase;
  d["n_tokens"] = e.n_tokens;
  d["n_chunks"] = e.n_chunks;
  d["writer"] = e.writer;
  d["fmt"] = e.fmt;
  d["hit_count"] = e.hit_count;
  d["nbytes"] = e.nbytes;
  d["avg_savings_ms"] = e.avg_savings_ms;
  int pins = 0;
  for (int r = 0; r < kMaxRanks; ++r) pins += e.pins[r];
  d["pins"] = pins;
  return d;
}

StoreConfig cfg_from_kwargs(const py::dict& d) {
  StoreConfig c;
  if (d.contains("min_tokens")) c.min_tokens = d["min_tokens"].cast<std::size_t>();
  if (d.contains("min_prompt_ms")) c.min_prompt_ms = d["min_prompt_ms"].cast<double>();
  if (d.contains("min_roi")) c.min_roi = d["min_roi"].cast<double>();
  if (d.contains("min_admit_roi")) c.min_admit_roi = d["min_admit_roi"].cast<double>();
  if (d.contains("max_bytes")) c.max_bytes = d["max_bytes"].cast<std::uint64_t>();
  if (d.contains("storage_budget_bytes")) c.storage_budget_bytes = d["storage_budget_bytes"].cast<std::uint64_t>();
  if (d.contains("eviction_watermark")) c.eviction_watermark = d["eviction_watermark"].cast<double>();
  if (d.contains("hot_ttl_ms")) c.hot_ttl_ms = d["hot_ttl_ms"].cast<std::uint64_t>();
  if (d.contains("warm_ttl_ms")) c.warm_ttl_ms = d["warm_ttl_ms"].cast<std::uint64_t>();
  if (d.contains("policy")) {
    const std::string p = d["policy"].cast<std::string>();
    c.policy = p == "lfu" ? EvictionPolicy::kLfu : p == "roi" ? EvictionPolicy::kRoi : EvictionPolicy::kLru;
  }
  if (d.contains("max_age_ms")) c.max_age_ms = d["max_age_ms"].cast<std::uint64_t>();
  if (d.contains("default_ttl_ms")) c.default_ttl_ms = d["default_ttl_ms"].cast<std::uint64_t>();
  if (d.contains("max_ttl_ms")) c.max_ttl_ms = d["max_ttl_ms"].cast<std::uint64_t>();
  if (d.contains("model_version_check")) c.model_version_check = d["model_version_check"].cast<bool>();
  if (d.contains("low_roi_hit_limit")) c.low_roi_hit_limit = d["low_roi_hit_limit"].cast<std::uint32_t>();
  if (d.contains("prewarm")) c.prewarm = d["prewarm"].cast<bool>();
  if (d.contains("prewarm_top_k")) c.prewarm_top_k = d["prewarm_top_k"].cast<std::uint32_t>();
  if (d.contains("prewarm_timeout_ms")) c.prewarm_timeout_ms = d["prewarm_timeout_ms"].cast<std::uint64_t>();
  if (d.contains("disk_guard")) c.disk_guard = d["disk_guard"].cast<bool>();
  if (d.contains("min_free_disk_bytes")) c.min_free_disk_bytes = d["min_free_disk_bytes"].cast<std::uint64_t>();
  if (d.contains("min_free_disk_ratio")) c.min_free_disk_ratio = d["min_free_disk_ratio"].cast<double>();
  return c;
}

py::dict cfg_to_dict(const StoreConfig& c) {
  py::dict d;
  d["min_tokens"] = c.min_tokens;
  d["min_prompt_ms"] = c.min_prompt_ms;
  d["min_roi"] = c.min_roi;
  d["min_admit_roi"] = c.min_admit_roi;
  d["max_bytes"] = c.max_bytes;
  d["storage_budget_bytes"] = c.storage_budget_bytes;
  d["eviction_watermark"] = c.eviction_watermark;
  d["critical_watermark"] = c.critical_watermark;
  d["hot_ttl_ms"] = c.hot_ttl_ms;
  d["warm_ttl_ms"] = c.warm_ttl_ms;
  d["policy"] = c.policy == EvictionPolicy::kLfu ? "lfu" : c.policy == EvictionPolicy::kRoi ? "roi" : "lru";
  d["max_age_ms"] = c.max_age_ms;
  d["default_ttl_ms"] = c.default_ttl_ms;
  d["max_ttl_ms"] = c.max_ttl_ms;
  d["model_version_check"] = c.model_version_check;
  d["low_roi_hit_limit"] = c.low_roi_hit_limit;
  d["prewarm"] = c.prewarm;
  d["prewarm_top_k"] = c.prewarm_top_k;
  d["prewarm_timeout_ms"] = c.prewarm_timeout_ms;
  d["disk_guard"] = c.disk_guard;
  d["min_free_disk_bytes"] = c.min_free_disk_bytes;
  d["min_free_disk_ratio"] = c.min_free_disk_ratio;
  return d;
}

}  // namespace

PYBIND11_MODULE(_native, m) {
  m.doc() = "Host-native runtime of axropus_deploy_b200 (AMF store, shard directory, controllers)";

  m.attr("FNV_OFFSET") = kFnvOffset;
  m.attr("FNV_PRIME") = kFnvPrime;
  m.def("fnv1a_tokens", [](I32Array toks) {
    return fnv1a_tokens(toks.data(), static_cast<std::size_t>(toks.size()));
  });
  m.def("fnv1a_bytes", [](py::buffer b, std::uint64_t h) {
    py::buffer_info bi = b.request();
    const std::size_t n = static_cast<std::size_t>(bi.size * bi.itemsize);
    py::gil_scoped_release rel;
    return fnv1a_bytes(h, bi.ptr, n);
  }, py::arg("data"), py::arg("h") = kFnvOffset);
  m.def("fnv1a_ptr", [](std::uintptr_t ptr, std::size_t n, std::uint64_t h) {
    py::gil_scoped_release rel;
    return fnv1a_bytes(h, reinterpret_cast<const void*>(ptr), n);
  }, py::arg("ptr"), py::arg("n"), py::arg("h") = kFnvOffset);
  m.def("prefix_hashes", [](I32Array toks) {
    const auto n = static_cast<std::size_t>(toks.size());
    py::array_t<std::uint64_t> out(n);
    auto* o = out.mutable_data();
    std::uint64_t h = kFnvOffset;
    for (std::size_t i = 0; i < n; ++i) { h = fnv1a_token(h, toks.data()[i]); o[i] = h; }
    return out;
  });
  m.def("encode_record_v9", [](const py::dict& d) {
    std::string out(kRecordBytesV9, '\0');
    encode_record_v9(entry_from_dict(d), reinterpret_cast<std::uint8_t*>(&out[0]));
    return py::bytes(out);
  });
  m.def("decode_record", [](py::bytes b, std::uint32_t version) {
    std::string s = b;
    const std::size_t need = version >= 9 ? kRecordBytesV9 : kRecordBytesV8;
    if (s.size() < need) throw std::invalid_argument("record too short");
    return entry_to_dict(decode_record(reinterpret_cast<const std::uint8_t*>(s.data()), version));
  });
  m.def("store_config_from_env", []() {
    StoreConfig c;
    std::string path;
    bool en = false;
    store_config_from_env(&c, &path, &en);
    py::dict d = cfg_to_dict(c);
    d["path"] = path;
    d["enabled"] = en;
    return d;
  });
  m.def("lookup_name", [](int r) { return std::string(lookup_name(static_cast<Lookup>(r))); });

  py::class_<AmfStore>(m, "AmfStore")
      .def(py::init<>())
      .def("init_from_env", &AmfStore::init_from_env)
      .def("init", [](AmfStore& s, const std::string& path, const py::dict& cfg) {
        return s.init(path, cfg_from_kwargs(cfg));
      }, py::arg("path"), py::arg("config") = py::dict())
      .def_property_readonly("enabled", &AmfStore::enabled)
      .def_property_readonly("disabled_reason", [](const AmfStore& s) {
        return std::string(disable_reason_name(s.disable_reason()));
      })
      .def_property_readonly("dir", &AmfStore::dir)
      .def_property_readonly("config", [](const AmfStore& s) { return cfg_to_dict(s.config()); })
      .def("find_longest_prefix", [](AmfStore& s, const py::dict& ctx, I32Array toks) {
        AmfEntry e;
        std::vector<std::int32_t> out_toks;
        const AmfContext c = ctx_from_dict(ctx);
        Lookup r;
        {
          py::gil_scoped_release rel;
          r = s.find_longest_prefix(c, toks.data(), static_cast<std::size_t>(toks.size()), &e, &out_toks);
        }
        py::object entry = r == Lookup::kHit ? py::object(entry_to_dict(e)) : py::none();
        return py::make_tuple(std::string(lookup_name(r)), entry);
      })
      .def("load_kv", [](AmfStore& s, const py::dict& entry) -> py::object {
        std::vector<std::uint8_t> out;
        const AmfEntry e = entry_from_dict(entry);
        bool ok;
        {
          py::gil_scoped_release rel;
          ok = s.load_kv(e, &out);
        }
        if (!ok) return py::none();
        return py::bytes(reinterpret_cast<const char*>(out.data()), out.size());
      })
      .def("load_kv_into", [](AmfStore& s, const py::dict& entry, std::uintptr_t ptr, std::size_t cap) {
        std::size_t got = 0;
        const AmfEntry e = entry_from_dict(entry);
        bool ok;
        {
          py::gil_scoped_release rel;
          ok = s.load_kv_into(e, reinterpret_cast<void*>(ptr), cap, &got);
        }
        return ok ? static_cast<long long>(got) : -1LL;
      })
      .def("store_entry", [](AmfStore& s, const py::dict& ctx, I32Array toks, py::buffer kv,
                             std::uint64_t saved_ms) {
        py::buffer_info bi = kv.request();
        const AmfContext c = ctx_from_dict(ctx);
        py::gil_scoped_release rel;
        return s.store_entry(c, toks.data(), static_cast<std::size_t>(toks.size()),
                             static_cast<const std::uint8_t*>(bi.ptr),
                             static_cast<std::size_t>(bi.size * bi.itemsize), saved_ms);
      }, py::arg("ctx"), py::arg("tokens"), py::arg("kv"), py::arg("saved_ms") = 0)
      .def("store_entry_ptr", [](AmfStore& s, const py::dict& ctx, I32Array toks, std::uintptr_t ptr,
                                 std::size_t n, std::uint64_t saved_ms) {
        const AmfContext c = ctx_from_dict(ctx);
        py::gil_scoped_release rel;
        return s.store_entry(c, toks.data(), static_cast<std::size_t>(toks.size()),
                             reinterpret_cast<const std::uint8_t*>(ptr), n, saved_ms);
      })
      .def("note_hit", [](AmfStore& s, const py::dict& e, std::uint64_t tokens_saved,
                          std::uint64_t restore_ms, std::uint64_t saved_ms) {
        s.note_hit(entry_from_dict(e), tokens_saved, restore_ms, saved_ms);
      })
      .def("note_failure", [](AmfStore& s, const py::dict& e) { s.note_failure(entry_from_dict(e)); })
      .def("note_block", [](AmfStore& s, py::object e) {
        if (e.is_none()) s.note_block();
        else s.note_block(entry_from_dict(e.cast<py::dict>()));
      }, py::arg("entry") = py::none())
      .def("note_miss", &AmfStore::note_miss)
      .def("evict_expired_entries", &AmfStore::evict_expired_entries)
      .def("remove", [](AmfStore& s, const py::dict& e) { return s.remove(entry_from_dict(e).key); })
      .def("stats", [](const AmfStore& s) { return stats_to_dict(s.stats()); })
      .def("storage_stats", [](const AmfStore& s, std::uint64_t now_ms) {
        const AmfStorageStats o = s.storage_stats(now_ms);
        py::dict d;
        d["total_bytes"] = o.total_bytes;
        d["budget_bytes"] = o.budget_bytes;
        d["utilization"] = o.utilization;
        d["hot_entries"] = o.hot_entries;
        d["warm_entries"] = o.warm_entries;
        d["cold_entries"] = o.cold_entries;
        d["disk_free_bytes"] = o.disk_free_bytes;
        d["disk_capacity_bytes"] = o.disk_capacity_bytes;
        d["disk_free_ratio"] = o.disk_free_ratio;
        d["low_disk"] = o.low_disk;
        return d;
      }, py::arg("now_ms") = 0)
      .def("entries", [](const AmfStore& s) {
        py::list l;
        for (const auto& e : s.entries()) l.append(entry_to_dict(e));
        return l;
      })
      .def_property_readonly("total_bytes", &AmfStore::total_bytes)
      .def_property_readonly("entry_count", &AmfStore::entry_count)
      .def_property_readonly("eviction_pressure", &AmfStore::eviction_pressure)
      .def("warm_ratio", &AmfStore::warm_ratio)
      .def_property_readonly("prewarm_complete", &AmfStore::prewarm_complete)
      .def_property_readonly("prewarm_loaded", &AmfStore::prewarm_loaded)
      .def_property_readonly("prewarm_failed", &AmfStore::prewarm_failed)
      .def("oldest_entry_age_ms", &AmfStore::oldest_entry_age_ms)
      .def("reuse_score", &AmfStore::reuse_score)
      .def("avg_prefix_length", &AmfStore::avg_prefix_length)
      .def("historical_accept_rate", &AmfStore::historical_accept_rate)
      .def("restore_cost_ms", &AmfStore::restore_cost_ms)
      .def("set_min_prompt_ms", &AmfStore::set_min_prompt_ms)
      .def("set_min_admit_roi", &AmfStore::set_min_admit_roi)
      .def("set_eviction_pressure", &AmfStore::set_eviction_pressure)
      .def("basename", [](const AmfStore& s, const py::dict& e) { return s.basename_of(entry_from_dict(e).key); })
      .def("kv_path", [](const AmfStore& s, const py::dict& e) { return s.kv_path(entry_from_dict(e).key); })
      .def("tok_path", [](const AmfStore& s, const py::dict& e) { return s.tok_path(entry_from_dict(e).key); })
      .def("flush", &AmfStore::flush)
      .def("shutdown", &AmfStore::shutdown);

  py::enum_<InsertStatus>(m, "InsertStatus")
      .value("OK", InsertStatus::kOk)
      .value("EXISTS", InsertStatus::kExists)
      .value("BUSY", InsertStatus::kBusy)
      .value("NO_SPACE", InsertStatus::kNoSpace)
      .value("TOO_LARGE", InsertStatus::kTooLarge);

  py::class_<ShardDirectory>(m, "ShardDirectory")
      .def(py::init<const std::string&, int, const std::vector<std::uint32_t>&, std::uint64_t,
                    std::uint32_t, bool, double>(),
           py::arg("name"), py::arg("world"), py::arg("n_slots"), py::arg("chunk_bytes"),
           py::arg("entry_cap") = 4096, py::arg("attach") = false, py::arg("lock_timeout_s") = 5.0)
      .def_property_readonly("world", &ShardDirectory::world)
      .def("chunk_bytes", &ShardDirectory::chunk_bytes)
      .def("lookup", [](ShardDirectory& d, int shard, std::uint64_t key, std::uint64_t key2, int pin_rank) -> py::object {
        LookupOut o;
        {
          py::gil_scoped_release rel;
          o = d.lookup(shard, key, key2, pin_rank);
        }
        if (!o.found) return py::none();
        py::array_t<std::int32_t> slots(o.slots.size());
        std::copy(o.slots.begin(), o.slots.end(), slots.mutable_data());
        return py::make_tuple(o.n_tokens, o.fmt, slots);
      }, py::arg("shard"), py::arg("key"), py::arg("key2") = 0, py::arg("pin_rank") = -1)
      .def("contains", &ShardDirectory::contains, py::arg("shard"), py::arg("key"), py::arg("key2") = 0)
      .def("unpin", &ShardDirectory::unpin)
      .def("begin_insert", [](ShardDirectory& d, int shard, std::uint64_t key, std::uint64_t key2,
                              std::uint32_t n_chunks, std::uint32_t n_tokens, std::uint32_t fmt,
                              int writer, double savings_ms) {
        std::vector<std::int32_t> slots;
        std::vector<std::uint64_t> evicted;
        InsertStatus st;
        {
          py::gil_scoped_release rel;
          st = d.begin_insert(shard, key, key2, n_chunks, n_tokens, fmt, writer, savings_ms, &slots, &evicted);
        }
        py::array_t<std::int32_t> a(slots.size());
        std::copy(slots.begin(), slots.end(), a.mutable_data());
        return py::make_tuple(st, a, evicted);
      })
      .def("commit", &ShardDirectory::commit)
      .def("abort", &ShardDirectory::abort)
      .def("remove", &ShardDirectory::remove)
      .def("clear", &ShardDirectory::clear)
      .def("release_rank", &ShardDirectory::release_rank)
      .def("reclaim_stale", &ShardDirectory::reclaim_stale)
      .def("note_savings", &ShardDirectory::note_savings)
      .def("lengths", &ShardDirectory::lengths)
      .def("info", [](ShardDirectory& d, int shard) {
        const ShardInfo i = d.info(shard);
        py::dict o;
        o["n_slots"] = i.n_slots;
        o["free_slots"] = i.free_slots;
        o["chunk_bytes"] = i.chunk_bytes;
        o["entries"] = i.entries;
        o["entry_cap"] = i.entry_cap;
        o["hits"] = i.stats.hits;
        o["misses"] = i.stats.misses;
        o["inserts"] = i.stats.inserts;
        o["evictions"] = i.stats.evictions;
        o["bytes_stored"] = i.stats.bytes_stored;
        o["bytes_evicted"] = i.stats.bytes_evicted;
        o["busy"] = i.stats.busy;
        o["alloc_failures"] = i.stats.alloc_failures;
        o["reclaimed"] = i.stats.reclaimed;
        return o;
      })
      .def("entries", [](ShardDirectory& d, int shard) {
        py::list l;
        for (const auto& e : d.entries(shard)) l.append(dir_entry_to_dict(e));
        return l;
      });

  bind_runtime(m);
  bind_ngram(m);
}
