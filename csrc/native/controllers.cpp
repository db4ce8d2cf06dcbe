// Host-native runtime controllers (see controllers.h).
#include "controllers.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>

// ------------------------------------------------------------------ spec-depth scheduler
namespace axr {
namespace {

float unit_or(float v, float d) { return std::isfinite(v) ? std::min(1.f, std::max(0.f, v)) : d; }
float finite_or(float v, float d) { return std::isfinite(v) ? v : d; }

int lane_cap(Lane l, int max_depth) {
  const int c = l == Lane::kSpecHit ? 16 : l == Lane::kHit ? 10 : 3;
  return std::max(1, std::min(c, max_depth));
}

// The lane the smoothed signals point to. Quality q = acceptance x (1 - entropy) is the
// chance a drafted token survives; AMF reuse says the prefix was restored, i.e. the
// request replays a known context where drafts (n-gram or model) are usually right.
Lane lane_for(float acc, float ent, float dtps, float reuse) {
  const float q = acc * (1.f - ent);
  if (reuse >= 0.70f && q >= 0.35f && dtps >= -0.05f) return Lane::kSpecHit;
  if (reuse >= 0.70f || q >= 0.22f) return Lane::kHit;
  return Lane::kMiss;
}

}  // namespace

const char* lane_name(Lane l) { return l == Lane::kSpecHit ? "SPEC_HIT" : l == Lane::kHit ? "HIT" : "MISS"; }

// Expected tokens per verification step with k drafted tokens, each accepted with
// probability a (independently): 1 + a + ... + a^k = (1 - a^(k+1)) / (1 - a), against a
// step cost of 1 + c k (Leviathan, Kalman & Matias 2023, "Fast inference from
// transformers via speculative decoding", section 3).
int best_depth(float acceptance, float draft_cost, int cap) {
  const double a = std::min(0.98, std::max(0.0, static_cast<double>(acceptance)));
  const double c = std::min(1.0, std::max(0.005, static_cast<double>(draft_cost)));
  int best = 1;
  double best_v = -1.0;
  double pw = a;  // a^k
  for (int k = 1; k <= std::max(1, cap); ++k) {
    pw *= a;  // a^(k+1)
    const double tokens = a >= 0.999999 ? k + 1.0 : (1.0 - pw) / (1.0 - a);
    const double v = tokens / (1.0 + c * k);
    if (v > best_v + 1e-9) {
      best_v = v;
      best = k;
    }
  }
  return best;
}

KorithScheduleOutput schedule(SchedState* st, const KorithScheduleInput& in, const SchedConfig& cfg) {
  KorithScheduleOutput out{1, 0.f, static_cast<int>(Lane::kMiss)};
  st->step += 1;
  st->ready = in.baseline_ready != 0;
  if (!st->ready) {  // the engine's throughput baseline is not stable yet: no speculation
    st->depth = 1;
    st->lane = st->pending = Lane::kMiss;
    st->reason = "warmup";
    st->last_change = st->step;
    return out;
  }
  const float acc = unit_or(in.acceptance, 0.f), ent = unit_or(in.entropy, 1.f);
  const float dtps = std::max(-1.f, std::min(1.f, finite_or(in.current_tps, 0.f)));
  const float reuse = unit_or(in.amf_reuse_score, 0.f);
  if (!st->primed) {
    st->acc = acc;
    st->ent = ent;
    st->dtps = dtps;
    st->primed = true;
  } else {
    st->acc += cfg.alpha * (acc - st->acc);
    st->ent += cfg.alpha * (ent - st->ent);
    st->dtps += cfg.alpha * (dtps - st->dtps);
  }

  // lane: worse lanes are taken at once, better ones after lane_debounce steps in a row
  const Lane want = lane_for(st->acc, st->ent, st->dtps, reuse);
  if (static_cast<int>(want) < static_cast<int>(st->lane)) {
    st->lane = want;
    st->lane_age = 0;
    st->better_streak = 0;
  } else if (static_cast<int>(want) > static_cast<int>(st->lane)) {
    st->better_streak = st->pending == want ? st->better_streak + 1 : 1;
    st->pending = want;
    if (static_cast<int>(st->better_streak) >= cfg.lane_debounce) {
      st->lane = want;
      st->lane_age = 0;
      st->better_streak = 0;
    }
  } else {
    st->better_streak = 0;
  }
  st->lane_age += 1;
  st->miss_streak = st->lane == Lane::kMiss ? st->miss_streak + 1 : 0;

  const int cap = lane_cap(st->lane, cfg.max_depth);
  float cost = cfg.draft_cost;
  if (std::isfinite(in.engine_costs) && in.engine_costs > 0.f && in.engine_costs <= 1.f) cost = in.engine_costs;
  const int target = std::min(cap, best_depth(st->acc, cost, cap));
  int depth = std::max(1, st->depth);
  const char* reason = "hold";
  if (depth > cap || target < depth) {  // decreases are never held back
    depth = std::max(target, depth - 4);
    depth = std::min(depth, cap);
    reason = st->lane == Lane::kMiss ? "miss_down" : "down";
  } else if (target > depth && st->step - st->last_change >= static_cast<std::uint64_t>(cfg.hold_up_steps)) {
    depth = std::min(target, depth + 2);
    reason = "up";
  }
  // a long MISS stretch with usable acceptance: measure a deeper draft again
  if (st->lane == Lane::kMiss && st->miss_streak >= static_cast<std::uint32_t>(cfg.starve_steps) && st->acc >= 0.5f) {
    depth = std::min(lane_cap(Lane::kHit, cfg.max_depth), std::max(depth, 2) + 1);
    st->miss_streak = 0;
    reason = "starvation_probe";
  } else if (depth == 1 && st->step % static_cast<std::uint64_t>(std::max(1, cfg.probe_every)) == 0 &&
             st->dtps >= 0.f) {
    depth = 2;
    reason = "probe";
  }
  depth = std::max(1, std::min(cfg.max_depth, depth));
  if (depth != st->depth) st->last_change = st->step;
  st->depth = depth;
  st->reason = reason;
  out.desired_depth = depth;
  out.stability_score = std::min(1.f, std::max(0.f, st->acc * (1.f - st->ent)));
  out.throttle_flag = static_cast<int>(st->lane);
  if (std::getenv("KORITH_SCHED_LOG")) {
    std::fprintf(stderr, "[SCHEDULER_DECISION] depth=%d stability=%.3f throttle=%d lane=%s reason=%s\n", depth,
                 out.stability_score, out.throttle_flag, lane_name(st->lane), reason);
  }
  return out;
}

}  // namespace axr

namespace {
// The reference-shaped entry points keep one scheduler per process (the caller's record
// carries only the depth and the baseline flag).
std::mutex g_sched_mu;
axr::SchedState g_sched;

int batch_hint(int depth) { return std::max(1, 256 / (depth + 1)); }
}  // namespace

extern "C" {

__attribute__((visibility("default"))) KorithScheduleOutput korith_schedule_step(KorithSchedulerState* st,
                                                                                  const KorithScheduleInput* in) {
  KorithScheduleInput zero{};
  std::lock_guard<std::mutex> lk(g_sched_mu);
  if (st && st->speculative_depth >= 1) g_sched.depth = st->speculative_depth;
  const KorithScheduleOutput o = axr::schedule(&g_sched, in ? *in : zero);
  if (st) {
    st->speculative_depth = o.desired_depth;
    st->batch_size = batch_hint(o.desired_depth);
    st->baseline_ready = g_sched.ready ? 1 : 0;
  }
  return o;
}

__attribute__((visibility("default"))) unsigned korith_scheduler_update(float entropy, float acceptance, float tps) {
  KorithScheduleInput in{acceptance, entropy, tps, 0.f, 0.f, 0.f, 0.f, 0.f, 1};
  std::lock_guard<std::mutex> lk(g_sched_mu);
  const KorithScheduleOutput o = axr::schedule(&g_sched, in);
  return static_cast<unsigned>(std::max(1, o.desired_depth));
}

__attribute__((visibility("default"))) void korith_scheduler_reset(void) {
  std::lock_guard<std::mutex> lk(g_sched_mu);
  g_sched = axr::SchedState{};
}

__attribute__((visibility("default"))) void* korith_scheduler_create(void) { return new axr::SchedState(); }

__attribute__((visibility("default"))) KorithScheduleOutput korith_scheduler_step_ex(void* h,
                                                                                     const KorithScheduleInput* in) {
  KorithScheduleInput zero{};
  if (!h) return KorithScheduleOutput{1, 0.f, 1};
  return axr::schedule(static_cast<axr::SchedState*>(h), in ? *in : zero);
}

__attribute__((visibility("default"))) void korith_scheduler_destroy(void* h) { delete static_cast<axr::SchedState*>(h); }

}  // extern "C"

// ------------------------------------------------------------------ memory field
namespace axr {
namespace {
constexpr std::uint64_t kMinIntervalMs = 100, kMinRequests = 4;
constexpr std::uint64_t kBaseCooldownMs = 2000, kMaxCooldownMs = 60000, kBackoffForgetMs = 60000;
constexpr double kRoiMax = 10.0, kPressMin = 0.5, kPressMax = 3.0;
constexpr double kRoiSlew = 0.5, kPressSlew = 0.25;  // largest change of an output per update
constexpr double kRoiOff = 0.6, kEvidenceHits = 3.0;

std::uint64_t dlt(std::uint64_t a, std::uint64_t b) { return a >= b ? a - b : 0; }
double clamp(double v, double lo, double hi) { return std::isfinite(v) ? std::min(hi, std::max(lo, v)) : lo; }
double slew(double from, double to, double step) { return std::max(from - step, std::min(from + step, to)); }
double smoothstep(double e0, double e1, double x) {
  const double t = clamp((x - e0) / (e1 - e0), 0.0, 1.0);
  return t * t * (3.0 - 2.0 * t);
}
}  // namespace

// Outputs and how they move:
//  * min_admit_roi (admission bar of new AMF entries): 0 while the pool is below 60 %
//    full, rising linearly to 2 at 100 % full, plus 2 x (1 - ROI) while restores cost
//    more than they save, plus 0.5 per failed restore in the window; at most 0.5 of
//    change per update.
//  * eviction_pressure: 0.75 + 2.25 x smoothstep(fill from 50 % to 95 %), at most 0.25 of
//    change per update.
//  * replay gate (Schmitt trigger with exponential back-off): replay turns off when the
//    smoothed ROI falls below 0.6 with at least 3 hits of evidence; it turns back on
//    ("probation") once its cooldown has passed. Each off within 60 s of the previous one
//    doubles the cooldown (2 s, 4 s, ... up to 60 s), so an oscillating workload settles
//    with replay off for longer and longer stretches.
MemoryFieldOutput memory_field_update(MemoryFieldState* s, const MemoryFieldInput& in, bool log) {
  MemoryFieldState scratch;
  if (!s) s = &scratch;
  const MemoryFieldOutput last = s->last;
  if (s->has_prev) {
    s->requests_since_update += 1;
    if (dlt(in.now_ms, s->last_update_ms) < kMinIntervalMs && s->requests_since_update < kMinRequests) return last;
  }
  std::uint64_t dh = 0, dm = 0, df = 0, dsav = 0, drest = 0;
  if (s->has_prev) {
    dh = dlt(in.hits, s->prev.hits);
    dm = dlt(in.misses, s->prev.misses);
    df = dlt(in.failures, s->prev.failures);
    dsav = dlt(in.ms_saved, s->prev.ms_saved);
    drest = dlt(in.restore_ms, s->prev.restore_ms);
  }
  if (dh + dm) s->hit_ema = 0.7 * s->hit_ema + 0.3 * (double(dh) / double(dh + dm));
  if (drest) {
    const double roi = double(dsav) / double(drest);
    s->roi_ema = s->roi_seen ? 0.6 * s->roi_ema + 0.4 * roi : roi;
    s->roi_seen = true;
  }
  s->evidence = 0.5 * s->evidence + double(dh);
  const double fill = in.max_bytes ? clamp(double(in.bytes) / double(in.max_bytes), 0.0, 1.0) : 0.0;

  MemoryFieldOutput out = last;
  double bar = 5.0 * std::max(0.0, fill - 0.6);
  if (s->roi_seen && s->roi_ema < 1.0) bar += 2.0 * (1.0 - s->roi_ema);
  bar += 0.5 * std::min<std::uint64_t>(df, 8);
  out.min_admit_roi = clamp(slew(last.min_admit_roi, bar, kRoiSlew), 0.0, kRoiMax);
  const double press = 0.75 + 2.25 * smoothstep(0.5, 0.95, fill);
  out.eviction_pressure = clamp(slew(last.eviction_pressure, press, kPressSlew), kPressMin, kPressMax);

  const bool off = (last.replay_disable_mask & 1u) != 0;
  if (!off) {
    if (s->roi_seen && s->roi_ema < kRoiOff && s->evidence >= kEvidenceHits) {
      if (s->last_disable_ms && dlt(in.now_ms, s->last_disable_ms) <= kBackoffForgetMs) s->backoff += 1;
      else s->backoff = 0;
      const std::uint64_t cd = std::min(kMaxCooldownMs, kBaseCooldownMs << std::min<std::uint32_t>(s->backoff, 5));
      s->disabled_at_ms = in.now_ms;
      s->last_disable_ms = in.now_ms;
      s->disable_until_ms = in.now_ms + cd;
      out.replay_disable_mask = 1u;
    }
  } else if (in.now_ms >= s->disable_until_ms) {
    out.replay_disable_mask = 0u;  // probation: restores resume and the ROI is measured again
    s->roi_seen = false;
    s->evidence = 0.0;
  }
  out.cooldown_ms = (out.replay_disable_mask & 1u) ? dlt(s->disable_until_ms, in.now_ms) : 0;

  const bool changed = std::fabs(out.min_admit_roi - last.min_admit_roi) > 1e-6 ||
                       std::fabs(out.eviction_pressure - last.eviction_pressure) > 1e-6 ||
                       out.replay_disable_mask != last.replay_disable_mask;
  if (changed && log) {
    std::fprintf(stderr,
                 "[MF_POLICY] min_admit_roi=%.2f->%.2f evict_pressure=%.2f->%.2f replay_mask=0x%02x cooldown_ms=%llu "
                 "roi=%.2f hit_rate=%.2f fill=%.2f failures=%llu\n",
                 last.min_admit_roi, out.min_admit_roi, last.eviction_pressure, out.eviction_pressure,
                 out.replay_disable_mask, (unsigned long long)out.cooldown_ms, s->roi_ema, s->hit_ema, fill,
                 (unsigned long long)df);
    std::fflush(stderr);
  }
  s->last = out;
  s->prev = in;
  s->has_prev = true;
  s->last_update_ms = in.now_ms;
  s->requests_since_update = 0;
  return out;
}

std::string memory_field_to_json(const MemoryFieldState& s) {
  char b[768];
  std::snprintf(b, sizeof(b),
                "{\"min_admit_roi\":%.17g,\"eviction_pressure\":%.17g,\"replay_disable_mask\":%u,\"cooldown_ms\":%llu,"
                "\"roi_ema\":%.17g,\"hit_ema\":%.17g,\"roi_seen\":%d,\"disable_until_ms\":%llu,"
                "\"last_disable_ms\":%llu,\"backoff\":%u,\"last_update_ms\":%llu}",
                s.last.min_admit_roi, s.last.eviction_pressure, s.last.replay_disable_mask,
                (unsigned long long)s.last.cooldown_ms, s.roi_ema, s.hit_ema, s.roi_seen ? 1 : 0,
                (unsigned long long)s.disable_until_ms, (unsigned long long)s.last_disable_ms, s.backoff,
                (unsigned long long)s.last_update_ms);
  return b;
}

namespace {
bool json_num(const std::string& js, const char* key, double* out) {
  const std::string k = std::string("\"") + key + "\"";
  const std::size_t p = js.find(k);
  if (p == std::string::npos) return false;
  const std::size_t c = js.find(':', p + k.size());
  if (c == std::string::npos) return false;
  char* end = nullptr;
  const double v = std::strtod(js.c_str() + c + 1, &end);
  if (end == js.c_str() + c + 1 || !std::isfinite(v)) return false;
  *out = v;
  return true;
}
std::uint64_t u64(double v) { return static_cast<std::uint64_t>(std::max(0.0, v)); }
}  // namespace

bool memory_field_from_json(const std::string& js, MemoryFieldState* s) {
  if (!s) return false;
  double a, b, m, c;
  if (!json_num(js, "min_admit_roi", &a) || !json_num(js, "eviction_pressure", &b) ||
      !json_num(js, "replay_disable_mask", &m) || !json_num(js, "cooldown_ms", &c))
    return false;
  double roi = 1.0, hit = 0.0, seen = 0.0, until = 0.0, lastd = 0.0, bo = 0.0, upd = 0.0;
  json_num(js, "roi_ema", &roi);
  json_num(js, "hit_ema", &hit);
  json_num(js, "roi_seen", &seen);
  json_num(js, "disable_until_ms", &until);
  json_num(js, "last_disable_ms", &lastd);
  json_num(js, "backoff", &bo);
  json_num(js, "last_update_ms", &upd);
  s->last.min_admit_roi = clamp(a, 0.0, kRoiMax);
  s->last.eviction_pressure = clamp(b, kPressMin, kPressMax);
  s->last.replay_disable_mask = static_cast<std::uint32_t>(m) & 1u;
  s->last.cooldown_ms = std::min<std::uint64_t>(u64(c), kMaxCooldownMs);
  s->roi_ema = clamp(roi, 0.0, 1e6);
  s->hit_ema = clamp(hit, 0.0, 1.0);
  s->roi_seen = seen != 0.0;
  s->disable_until_ms = u64(until);
  s->last_disable_ms = u64(lastd);
  s->backoff = static_cast<std::uint32_t>(std::min(31.0, std::max(0.0, bo)));
  s->last_update_ms = u64(upd);
  return true;
}

// ------------------------------------------------------------------ thermo controller
float normalized_entropy(const float* logits, int n) {
  if (!logits || n <= 1) return 0.f;
  float mx = -std::numeric_limits<float>::infinity();
  for (int i = 0; i < n; ++i) mx = std::max(mx, logits[i]);
  if (!std::isfinite(mx)) return 0.f;
  double z = 0.0, zx = 0.0;
  for (int i = 0; i < n; ++i) {
    const double x = static_cast<double>(logits[i]) - mx;
    const double e = std::exp(x);
    z += e;
    zx += e * x;
  }
  if (!(z > 0.0)) return 0.f;
  const double h = (std::log(z) - zx / z) / std::log(static_cast<double>(n));
  return static_cast<float>(std::min(1.0, std::max(0.0, h)));
}

int thermo_next_depth(ThermoState* st, float accept, const float* logits, int n_vocab) {
  // EMA + EMA-variance of the acceptance rate; entropy from logits when given, else
  // 1 - acceptance as a proxy. Depth grows while acceptance is high and steady and the
  // distribution is sharp, and shrinks fast on an entropy spike or a volatile accept rate.
  const float a = std::isfinite(accept) ? std::min(1.f, std::max(0.f, accept)) : 0.f;
  const float alpha = 0.2f;
  const float prev = st->accept_ema;
  st->accept_ema = (1.f - alpha) * st->accept_ema + alpha * a;
  const float d = a - prev;
  st->accept_var = (1.f - alpha) * st->accept_var + alpha * d * d;
  const float h = logits ? normalized_entropy(logits, n_vocab) : 1.f - st->accept_ema;
  const bool spike = h > st->entropy + 0.10f;
  st->entropy = h;
  int depth = st->depth;
  if (spike || st->accept_ema < 0.4f || st->accept_var > 0.08f) depth = std::max(2, depth / 2);
  else if (st->accept_ema > 0.75f && h < 0.35f) depth += 1;
  else if (st->accept_ema < 0.55f) depth -= 1;
  st->depth = std::min(st->max_depth, std::max(1, depth));
  return st->depth;
}

// ------------------------------------------------------------------ event ring
HoloRing::HoloRing(std::size_t cap) : buf_(std::max<std::size_t>(1, cap)) {}

void HoloRing::record(const HoloEvent& e) {
  const std::uint64_t h = head_.load(std::memory_order_relaxed);
  buf_[h % buf_.size()] = e;
  head_.store(h + 1, std::memory_order_release);
}

std::size_t HoloRing::size() const {
  return static_cast<std::size_t>(std::min<std::uint64_t>(head_.load(std::memory_order_acquire), buf_.size()));
}

std::vector<HoloEvent> HoloRing::recent(std::size_t n) const {
  const std::uint64_t h = head_.load(std::memory_order_acquire);
  const std::uint64_t have = std::min<std::uint64_t>(h, buf_.size());
  n = static_cast<std::size_t>(std::min<std::uint64_t>(n, have));
  std::vector<HoloEvent> out(n);
  for (std::size_t i = 0; i < n; ++i) out[i] = buf_[(h - n + i) % buf_.size()];
  return out;
}

double HoloRing::future_safe(std::size_t window) const {
  const auto ev = recent(window);
  if (ev.empty()) return 0.0;
  double s = 0.0;
  for (const auto& e : ev) s += e.accept * std::exp(-static_cast<double>(e.entropy));
  return s / ev.size();
}

// ------------------------------------------------------------------ rolling metrics
void RollingMetrics::record(double now, std::uint64_t tokens, double watts) {
  std::lock_guard<std::mutex> g(mu_);
  s_.push_back({now, tokens, watts});
  total_ += tokens;
  while (!s_.empty() && now - s_.front().t > window_s_) s_.pop_front();
}

double RollingMetrics::tps(double now) const {
  std::lock_guard<std::mutex> g(mu_);
  std::uint64_t tok = 0;
  double t0 = now;
  for (const auto& x : s_) {
    if (now - x.t > window_s_) continue;
    tok += x.tokens;
    t0 = std::min(t0, x.t);
  }
  const double span = std::max(now - t0, 1e-3);
  return tok / span;
}

double RollingMetrics::tokens_per_joule(double now) const {
  std::lock_guard<std::mutex> g(mu_);
  std::uint64_t tok = 0;
  double joules = 0.0, prev_t = -1.0;
  for (const auto& x : s_) {
    if (now - x.t > window_s_) continue;
    tok += x.tokens;
    if (prev_t >= 0.0) joules += x.watts * (x.t - prev_t);
    prev_t = x.t;
  }
  return joules > 0.0 ? tok / joules : 0.0;
}

// ------------------------------------------------------------------ spec plan / collapse
SpecPlan resolve_spec_plan(bool env_enabled, bool have_draft, bool paused, int scheduler_depth, int env_depth,
                           bool control_allow, float accept_ema, float min_accept, int max_depth) {
  SpecPlan p;
  if (!env_enabled) { p.reason = SpecDisableReason::kEnvOff; return p; }
  if (!have_draft) { p.reason = SpecDisableReason::kNoDraft; return p; }
  if (paused) { p.reason = SpecDisableReason::kPaused; return p; }
  if (!control_allow) { p.reason = SpecDisableReason::kControlPlane; return p; }
  if (min_accept > 0.f && accept_ema < min_accept) { p.reason = SpecDisableReason::kLowAccept; return p; }
  const int d = env_depth > 0 ? env_depth : scheduler_depth;  // an explicit env depth overrides the scheduler
  if (d <= 0) { p.reason = SpecDisableReason::kSchedulerZero; return p; }
  p.enabled = true;
  p.depth = std::min(std::max(1, max_depth), d);
  p.reason = SpecDisableReason::kNone;
  return p;
}

const char* spec_disable_reason_name(SpecDisableReason r) {
  switch (r) {
    case SpecDisableReason::kNone: return "none";
    case SpecDisableReason::kEnvOff: return "env_off";
    case SpecDisableReason::kNoDraft: return "no_draft";
    case SpecDisableReason::kPaused: return "paused";
    case SpecDisableReason::kSchedulerZero: return "scheduler_zero";
    case SpecDisableReason::kControlPlane: return "control_plane";
    case SpecDisableReason::kLowAccept: return "low_accept";
  }
  return "unknown";
}

bool collapse_decide(const EngineSignal* sig, int n, int* chosen) {
  int best = -1;
  double best_gain = 0.0;
  for (int i = 0; i < n; ++i) {
    if (!std::isfinite(sig[i].confidence) || !std::isfinite(sig[i].cost_ms) || !std::isfinite(sig[i].benefit_ms)) continue;
    const double c = std::min(1.0, std::max(0.0, static_cast<double>(sig[i].confidence)));
    const double gain = c * sig[i].benefit_ms - sig[i].cost_ms;
    if (gain > best_gain || (best >= 0 && gain == best_gain && sig[i].depth < sig[best].depth)) {
      best_gain = gain;
      best = i;
    }
  }
  if (chosen) *chosen = best;
  return best >= 0;
}

}  // namespace axr
