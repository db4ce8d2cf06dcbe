// Runtime helpers and controller bindings.
#include "runtime.h"

#include <pybind11/numpy.h>
#include <optional>
#include <chrono>

#include <cstdint>

#include "controllers.h"
#include <pybind11/stl.h>

namespace py = pybind11;

namespace axr {
namespace {

inline std::uint64_t mix64(std::uint64_t x) {
  x ^= x >> 30;
  x *= 0xbf58476d1ce4e5b9ull;
  x ^= x >> 27;
  x *= 0x94d049bb133111ebull;
  x ^= x >> 31;
  return x;
}

// Chained 128-bit content hashes of full 16-token blocks: block i's hash covers the
// hash of block i-1 and its own tokens, so equal hashes mean equal whole prefixes.
py::array_t<std::uint64_t> block_chain_hashes(py::array_t<std::int32_t, py::array::c_style | py::array::forcecast> toks,
                                              int page, long long n_blocks) {
  const long long n = toks.size();
  const long long nb = std::min<long long>(n_blocks < 0 ? n / page : n_blocks, n / page);
  py::array_t<std::uint64_t> out({nb, 2LL});
  auto* o = out.mutable_data();
  const std::int32_t* t = toks.data();
  std::uint64_t a = 0x6a09e667f3bcc908ull, b = 0xbb67ae8584caa73bull;
  {
    py::gil_scoped_release rel;
    for (long long i = 0; i < nb; ++i) {
      std::uint64_t ha = mix64(a ^ 0x3c6ef372fe94f82bull), hb = mix64(b + 0xa54ff53a5f1d36f1ull);
      for (int j = 0; j < page; ++j) {
        const std::uint64_t v = static_cast<std::uint32_t>(t[i * page + j]);
        ha = mix64(ha ^ (v * 0x9e3779b97f4a7c15ull + static_cast<std::uint64_t>(j)));
        hb = mix64(hb + v * 0xc2b2ae3d27d4eb4full + (ha << 1));
      }
      a = ha;
      b = hb;
      o[2 * i] = a;
      o[2 * i + 1] = b;
    }
  }
  return out;
}


MemoryFieldInput mf_input(const py::dict& d) {
  MemoryFieldInput i;
  auto g = [&](const char* k) { return d.contains(k) ? d[k].cast<std::uint64_t>() : 0ull; };
  i.now_ms = g("now_ms"); i.hits = g("hits"); i.misses = g("misses"); i.blocks = g("blocks");
  i.failures = g("failures"); i.tokens_saved = g("tokens_saved"); i.ms_saved = g("ms_saved");
  i.restore_ms = g("restore_ms"); i.admissions = g("admissions"); i.admission_rejects = g("admission_rejects");
  i.evictions = g("evictions"); i.evicted_bytes = g("evicted_bytes"); i.entries = g("entries"); i.bytes = g("bytes");
  i.max_bytes = g("max_bytes"); i.oldest_entry_age_ms = g("oldest_entry_age_ms");
  i.negative_roi_streak = g("negative_roi_streak");
  return i;
}

py::dict mf_out(const MemoryFieldOutput& o) {
  py::dict d;
  d["min_admit_roi"] = o.min_admit_roi;
  d["eviction_pressure"] = o.eviction_pressure;
  d["replay_disable_mask"] = o.replay_disable_mask;
  d["cooldown_ms"] = o.cooldown_ms;
  return d;
}

}  // namespace

void bind_runtime(py::module_& m) {
  m.def("block_chain_hashes", &block_chain_hashes, py::arg("tokens"), py::arg("page") = 16,
        py::arg("n_blocks") = -1);

  py::class_<SchedState>(m, "SchedulerState")
      .def(py::init<>())
      .def_readwrite("depth", &SchedState::depth)
      .def_readonly("ready", &SchedState::ready)
      .def_readonly("acceptance_ema", &SchedState::acc)
      .def_readonly("entropy_ema", &SchedState::ent)
      .def_readonly("tps_trend_ema", &SchedState::dtps)
      .def_readonly("step", &SchedState::step)
      .def_readonly("last_change", &SchedState::last_change)
      .def_readonly("miss_streak", &SchedState::miss_streak)
      .def_property_readonly("lane", [](const SchedState& s) { return std::string(lane_name(s.lane)); })
      .def_property_readonly("reason", [](const SchedState& s) { return std::string(s.reason); });
  m.def("schedule_step", [](SchedState& st, float acceptance, float entropy, float current_tps,
                            float engine_costs, float amf_reuse_score, float amf_avg_prefix_length,
                            float amf_accept_rate, float amf_restore_cost_ms, bool baseline_ready) {
    KorithScheduleInput in{acceptance, entropy, current_tps, engine_costs, amf_reuse_score, amf_avg_prefix_length,
                           amf_accept_rate, amf_restore_cost_ms, baseline_ready ? 1 : 0};
    const KorithScheduleOutput o = schedule(&st, in);
    py::dict d;
    d["desired_depth"] = o.desired_depth;
    d["stability_score"] = o.stability_score;
    d["throttle_flag"] = o.throttle_flag;
    d["lane"] = std::string(lane_name(st.lane));
    d["reason"] = std::string(st.reason);
    return d;
  }, py::arg("state"), py::arg("acceptance"), py::arg("entropy"), py::arg("current_tps") = 0.f,
     py::arg("engine_costs") = 0.f, py::arg("amf_reuse_score") = 0.f, py::arg("amf_avg_prefix_length") = 0.f,
     py::arg("amf_accept_rate") = 0.f, py::arg("amf_restore_cost_ms") = 0.f, py::arg("baseline_ready") = true);
  m.def("best_depth", &best_depth, py::arg("acceptance"), py::arg("draft_cost"), py::arg("cap"));

  py::class_<MemoryFieldState>(m, "MemoryFieldState")
      .def(py::init<>())
      .def_property_readonly("last", [](const MemoryFieldState& s) { return mf_out(s.last); })
      .def("to_json", [](const MemoryFieldState& s) { return memory_field_to_json(s); })
      .def("from_json", [](MemoryFieldState& s, const std::string& js) { return memory_field_from_json(js, &s); });
  m.def("memory_field_update", [](MemoryFieldState& s, const py::dict& in, bool log) {
    return mf_out(memory_field_update(&s, mf_input(in), log));
  }, py::arg("state"), py::arg("input"), py::arg("log") = false);

  py::class_<ThermoState>(m, "ThermoState")
      .def(py::init([](int max_depth) { ThermoState t; t.max_depth = max_depth; return t; }), py::arg("max_depth") = 12)
      .def_readonly("accept_ema", &ThermoState::accept_ema)
      .def_readonly("accept_var", &ThermoState::accept_var)
      .def_readonly("entropy", &ThermoState::entropy)
      .def_readonly("depth", &ThermoState::depth);
  m.def("thermo_next_depth", [](ThermoState& st, float accept,
                                 std::optional<py::array_t<float, py::array::c_style | py::array::forcecast>> logits) {
    if (logits) return thermo_next_depth(&st, accept, logits->data(), static_cast<int>(logits->size()));
    return thermo_next_depth(&st, accept, nullptr, 0);
  }, py::arg("state"), py::arg("accept"), py::arg("logits") = py::none());
  m.def("normalized_entropy", [](py::array_t<float, py::array::c_style | py::array::forcecast> l) {
    return normalized_entropy(l.data(), static_cast<int>(l.size()));
  });

  py::class_<HoloRing>(m, "HoloRing")
      .def(py::init<std::size_t>(), py::arg("capacity") = 50000)
      .def("record", [](HoloRing& r, int token, float accept, float entropy, int depth) {
        const auto ns = std::chrono::duration_cast<std::chrono::nanoseconds>(
            std::chrono::steady_clock::now().time_since_epoch()).count();
        r.record(HoloEvent{static_cast<std::uint64_t>(ns), token, accept, entropy, depth});
      })
      .def("__len__", &HoloRing::size)
      .def("future_safe", &HoloRing::future_safe, py::arg("window") = 256)
      .def("recent", [](const HoloRing& r, std::size_t n) {
        py::list l;
        for (const auto& e : r.recent(n)) l.append(py::make_tuple(e.token, e.accept, e.entropy, e.depth));
        return l;
      });

  py::class_<RollingMetrics>(m, "RollingMetrics")
      .def(py::init<double>(), py::arg("window_s") = 10.0)
      .def("record", &RollingMetrics::record)
      .def("tps", &RollingMetrics::tps)
      .def("tokens_per_joule", &RollingMetrics::tokens_per_joule)
      .def_property_readonly("total_tokens", &RollingMetrics::total_tokens);

  m.def("resolve_spec_plan", [](bool env_enabled, bool have_draft, bool paused, int scheduler_depth, int env_depth,
                                bool control_allow, float accept_ema, float min_accept, int max_depth) {
    const SpecPlan p = resolve_spec_plan(env_enabled, have_draft, paused, scheduler_depth, env_depth, control_allow,
                                         accept_ema, min_accept, max_depth);
    py::dict d;
    d["enabled"] = p.enabled;
    d["depth"] = p.depth;
    d["reason"] = std::string(spec_disable_reason_name(p.reason));
    return d;
  });
  m.def("collapse_decide", [](const std::vector<std::tuple<float, float, float, int>>& sig) {
    std::vector<EngineSignal> v;
    for (const auto& t : sig) v.push_back({std::get<0>(t), std::get<1>(t), std::get<2>(t), std::get<3>(t)});
    int chosen = -1;
    const bool commit = collapse_decide(v.data(), static_cast<int>(v.size()), &chosen);
    return py::make_tuple(commit, chosen);
  });
}

}  // namespace axr
