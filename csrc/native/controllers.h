// Host-native runtime controllers.
//
//  * Spec-depth scheduler with the C ABI `korith_schedule_step` (the reference's
//    Rust cdylib controller/ffi.rs:34-173 and controller/scheduler.rs:133-290, here
//    in C++ with the same structs, lane table and thresholds so an engine that
//    dlopens KORITH_SCHEDULER_LIB finds the same symbols and behaviour).
//  * Memory field (core/memory_field.h:10-66): bounded, cooldown-limited AMF policy
//    update (min_admit_roi, eviction_pressure, replay mask, cooldown) with JSON
//    snapshots.
//  * Thermo controller (core/thermo_controller.h:11-34): speculative depth from
//    acceptance EMA / variance / normalised logit entropy.
//  * Event ring (holographic/memory.h, ring_buffer.h): single-writer ring of decode
//    events with a "future safe" score mean(accept * exp(-entropy)).
//  * Rolling throughput / tokens-per-joule metrics (core/metrics.h).
//  * Spec plan resolution (core/spec_plan.h:5-124) and the collapse gate
//    (core/collapse_controller.h:9-66).
#pragma once

#include <atomic>
#include <cstdint>
#include <deque>
#include <mutex>
#include <string>
#include <vector>

extern "C" {
struct KorithSchedulerState {
  int speculative_depth;
  int batch_size;  // packed counters: step (16 bits) | last change (8) | miss streak (8)
  int baseline_ready;
};
struct KorithScheduleInput {
  float acceptance;
  float entropy;
  float current_tps;
  float engine_costs;
  float amf_reuse_score;
  float amf_avg_prefix_length;
  float amf_accept_rate;
  float amf_restore_cost_ms;
  int baseline_ready;
};
struct KorithScheduleOutput {
  int desired_depth;
  float stability_score;
  int throttle_flag;
};
KorithScheduleOutput korith_schedule_step(KorithSchedulerState* state, const KorithScheduleInput* input);
void korith_scheduler_reset(KorithSchedulerState* state);
int korith_scheduler_update(KorithSchedulerState* state, const KorithScheduleInput* input, int* out_depth);
}

namespace axr {

const char* last_lane_name();
const char* last_reason();

struct MemoryFieldInput {
  std::uint64_t now_ms = 0, hits = 0, misses = 0, blocks = 0, failures = 0, tokens_saved = 0, ms_saved = 0;
  std::uint64_t restore_ms = 0, admissions = 0, admission_rejects = 0, evictions = 0, evicted_bytes = 0;
  std::uint64_t entries = 0, bytes = 0, max_bytes = 0, oldest_entry_age_ms = 0, negative_roi_streak = 0;
};
struct MemoryFieldOutput {
  double min_admit_roi = 0.0;
  double eviction_pressure = 1.0;
  std::uint32_t replay_disable_mask = 0;
  std::uint64_t cooldown_ms = 0;
};
struct MemoryFieldState {
  std::uint64_t last_update_ms = 0, requests_since_update = 0, last_replay_flip_ms = 0;
  std::uint32_t replay_flip_count = 0;
  MemoryFieldOutput last{};
  MemoryFieldInput prev{};
  bool has_prev = false;
};
MemoryFieldOutput memory_field_update(MemoryFieldState* s, const MemoryFieldInput& in, bool log = true);
std::string memory_field_to_json(const MemoryFieldState& s);
bool memory_field_from_json(const std::string& js, MemoryFieldState* s);

struct ThermoState {
  float accept_ema = 0.f, accept_var = 0.f, entropy = 0.f;
  int depth = 1;
  int max_depth = 12;
};
float normalized_entropy(const float* logits, int n);
int thermo_next_depth(ThermoState* st, float accept, const float* logits, int n_vocab);

struct HoloEvent {
  std::uint64_t ts_ns;
  std::int32_t token;
  float accept;
  float entropy;
  std::int32_t depth;
};
class HoloRing {
 public:
  explicit HoloRing(std::size_t cap = 50000);
  void record(const HoloEvent& e);  // single writer
  std::size_t size() const;
  std::vector<HoloEvent> recent(std::size_t n) const;
  double future_safe(std::size_t window) const;

 private:
  std::vector<HoloEvent> buf_;
  std::atomic<std::uint64_t> head_{0};
};

class RollingMetrics {
 public:
  explicit RollingMetrics(double window_s = 10.0) : window_s_(window_s) {}
  void record(double now_s, std::uint64_t tokens, double watts);
  double tps(double now_s) const;
  double tokens_per_joule(double now_s) const;
  std::uint64_t total_tokens() const { return total_; }

 private:
  struct Sample { double t; std::uint64_t tokens; double watts; };
  std::deque<Sample> s_;
  double window_s_;
  std::uint64_t total_ = 0;
  mutable std::mutex mu_;
};

enum class SpecDisableReason : int { kNone = 0, kEnvOff, kNoDraft, kPaused, kSchedulerZero, kControlPlane, kLowAccept };
struct SpecPlan {
  bool enabled = false;
  int depth = 0;
  SpecDisableReason reason = SpecDisableReason::kNoDraft;
};
SpecPlan resolve_spec_plan(bool env_enabled, bool have_draft, bool paused, int scheduler_depth, int env_depth,
                           bool control_allow, float accept_ema, float min_accept, int max_depth);
const char* spec_disable_reason_name(SpecDisableReason r);

struct EngineSignal {
  float confidence;
  float cost_ms;
  float benefit_ms;
  int depth;
};
// Commit (true) when the expected benefit of the speculative branch beats its cost.
bool collapse_decide(const EngineSignal* signals, int n, int* chosen);

}  // namespace axr
