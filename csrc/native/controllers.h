// Host-native runtime controllers.
//
//  * Speculative-depth scheduler behind the C ABI `korith_schedule_step` /
//    `korith_scheduler_update` / `korith_scheduler_reset` (the symbols and structs of
//    the reference's controller/ffi.rs:30-175, so an engine that dlopens
//    KORITH_SCHEDULER_LIB finds them). The controller itself is this library's own: a
//    full state (`SchedState`), smoothed signals, a lane per step (SPEC_HIT / HIT /
//    MISS) and a depth chosen by the expected-tokens-per-cost model of speculative
//    decoding, with one-sided hysteresis and a starvation probe. Handles
//    (`korith_scheduler_create` / `_step_ex` / `_destroy`) give callers that run several
//    schedulers one state each; the reference-shaped calls share one process state.
//  * Memory field: AMF pool admission bar, eviction pressure and replay gate from the
//    windowed restore ROI and pool fill (core/memory_field.h:10-66 names the outputs).
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
// Caller-owned scheduler record of the reference ABI: the current depth, the
// recommended decode batch for that depth (output), and whether the engine's baseline
// throughput is stable.
struct KorithSchedulerState {
  int speculative_depth;
  int batch_size;
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
unsigned korith_scheduler_update(float entropy, float acceptance, float tps);
void korith_scheduler_reset(void);
void* korith_scheduler_create(void);
KorithScheduleOutput korith_scheduler_step_ex(void* handle, const KorithScheduleInput* input);
void korith_scheduler_destroy(void* handle);
}

namespace axr {

enum class Lane : int { kMiss = 1, kHit = 2, kSpecHit = 3 };
const char* lane_name(Lane l);

struct SchedConfig {
  float alpha = 0.3f;        // EMA weight of a new sample
  int max_depth = 16;
  int hold_up_steps = 24;    // steps between two increases of the depth
  int lane_debounce = 3;     // steps a better lane must persist before it is taken
  int starve_steps = 80;     // MISS steps before a starvation probe
  int probe_every = 48;      // depth-1 probe period
  float draft_cost = 0.08f;  // cost of one drafted token relative to one target step
};

struct SchedState {
  int depth = 1;
  bool ready = false;
  float acc = 0.f, ent = 1.f, dtps = 0.f;  // smoothed acceptance, entropy, throughput trend
  bool primed = false;
  std::uint64_t step = 0, last_change = 0;
  std::uint32_t miss_streak = 0, lane_age = 0, better_streak = 0;
  Lane lane = Lane::kMiss, pending = Lane::kMiss;
  const char* reason = "warmup";
};

// One decision. Deterministic in (state, input, config).
KorithScheduleOutput schedule(SchedState* st, const KorithScheduleInput& in, const SchedConfig& cfg = SchedConfig());
// Depth in [1, cap] that maximises expected accepted tokens per unit of step cost.
int best_depth(float acceptance, float draft_cost, int cap);

struct MemoryFieldInput {
  std::uint64_t now_ms = 0, hits = 0, misses = 0, blocks = 0, failures = 0, tokens_saved = 0, ms_saved = 0;
  std::uint64_t restore_ms = 0, admissions = 0, admission_rejects = 0, evictions = 0, evicted_bytes = 0;
  std::uint64_t entries = 0, bytes = 0, max_bytes = 0, oldest_entry_age_ms = 0, negative_roi_streak = 0;
};
struct MemoryFieldOutput {
  double min_admit_roi = 0.0;      // restores must save this many ms per ms they cost to be admitted
  double eviction_pressure = 1.0;  // multiplier on the pool's eviction score
  std::uint32_t replay_disable_mask = 0;
  std::uint64_t cooldown_ms = 0;   // time left before a disabled replay is tried again
};
struct MemoryFieldState {
  std::uint64_t last_update_ms = 0, requests_since_update = 0;
  bool has_prev = false;
  MemoryFieldInput prev{};
  double roi_ema = 1.0, hit_ema = 0.0, evidence = 0.0;  // smoothed window ROI, hit rate, recent hits
  bool roi_seen = false;
  std::uint64_t disabled_at_ms = 0, disable_until_ms = 0, last_disable_ms = 0;
  std::uint32_t backoff = 0;  // disables in a row (each doubles the next cooldown)
  MemoryFieldOutput last{};
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
