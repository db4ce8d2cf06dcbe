// Host-native runtime controllers (see controllers.h).
#include "controllers.h"

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <limits>

namespace {

thread_local const char* g_lane = "MISS";
thread_local const char* g_reason = "warmup";

float unit_or(float v, float d) { return std::isfinite(v) ? std::min(1.f, std::max(0.f, v)) : d; }
float finite_or(float v, float d) { return std::isfinite(v) ? v : d; }

enum class Lane { kSpecHit, kHit, kMiss };

// Lane from the decode quality signals and the AMF reuse of the current prefix.
Lane lane_of(float acc, float ent, float dtps, float reuse) {
  const bool replay_local = reuse >= 0.70f;
  const bool stable = acc >= 0.78f && ent <= 0.58f && dtps >= -0.05f;
  if (replay_local && stable) return Lane::kSpecHit;
  if (replay_local || (acc >= 0.68f && ent <= 0.68f)) return Lane::kHit;
  return Lane::kMiss;
}

constexpr unsigned kProbeInterval = 64, kHysteresis = 32, kStarvation = 96;
constexpr int kMaxDepth = 16;

}  // namespace

extern "C" {

__attribute__((visibility("default"))) KorithScheduleOutput korith_schedule_step(KorithSchedulerState* st,
                                                                                  const KorithScheduleInput* in) {
  KorithScheduleOutput out{1, 0.f, 1};
  if (!st || !in) return out;
  st->baseline_ready = in->baseline_ready ? 1 : 0;
  if (!st->baseline_ready) {  // warm-up: miss budget until the baseline is stable
    st->speculative_depth = 1;
    g_lane = "MISS";
    g_reason = "warmup";
    return out;
  }
  const float acc = unit_or(in->acceptance, 0.f);
  const float ent = unit_or(in->entropy, 1.f);
  const float dtps = finite_or(in->current_tps, 0.f);
  const float reuse = unit_or(in->amf_reuse_score, 0.f);
  int depth = std::min(kMaxDepth, std::max(1, st->speculative_depth));
  const unsigned raw = static_cast<unsigned>(st->batch_size);
  unsigned step = ((raw & 0xFFFFu) + 1u) & 0xFFFFu;
  unsigned last_change = (raw >> 16) & 0xFFu;
  unsigned miss_streak = (raw >> 24) & 0xFFu;

  const Lane lane = lane_of(acc, ent, dtps, reuse);
  miss_streak = lane == Lane::kMiss ? std::min(255u, miss_streak + 1u) : 0u;
  const char* reason = "hold";
  bool force_down = false;
  int cap = 3, throttle = 1;
  switch (lane) {
    case Lane::kSpecHit:
      cap = 16;
      throttle = 3;
      if (acc >= 0.90f && ent <= 0.45f && dtps >= -0.02f) { depth += 2; reason = "spec_hit_up2"; }
      else if (acc >= 0.80f && ent <= 0.58f && dtps >= -0.05f) { depth += 1; reason = "spec_hit_up1"; }
      else if (acc < 0.62f || ent > 0.82f || dtps < -0.15f) { depth = std::max(2, depth - 2); force_down = true; reason = "spec_hit_down"; }
      g_lane = "SPEC_HIT";
      break;
    case Lane::kHit:
      cap = 12;
      throttle = 2;
      if (acc >= 0.82f && ent <= 0.62f && dtps >= -0.03f) { depth += 1; reason = "hit_up"; }
      else if (acc < 0.58f || ent > 0.84f || dtps < -0.14f) { depth = std::max(2, depth - 1); force_down = true; reason = "hit_down"; }
      g_lane = "HIT";
      break;
    case Lane::kMiss:
      if (acc < 0.50f || ent > 0.85f || dtps < -0.10f) { depth = 2; reason = "miss_cap"; }
      else { depth = std::min(depth, 3); reason = "miss_hold"; }
      if (miss_streak >= kStarvation && acc >= 0.60f && ent <= 0.70f) {  // starvation probe
        depth = 3;
        reason = "miss_probe";
        miss_streak = 0;
      }
      force_down = true;
      g_lane = "MISS";
      break;
  }
  depth = std::min(cap, std::max(1, depth));
  bool probed = false;
  if (depth == 1 && step % kProbeInterval == 0 && dtps >= 0.f) {  // periodic cold-start probe
    depth = 2;
    reason = "probe";
    probed = true;
    force_down = false;
  }
  depth = std::min(kMaxDepth, std::max(1, depth));
  if (depth != st->speculative_depth) {
    const unsigned s8 = step & 0xFFu;
    const unsigned since = (s8 - last_change) & 0xFFu;
    if (!probed && !force_down && since < kHysteresis) {
      depth = st->speculative_depth;
      reason = "hold";
    } else {
      last_change = s8;
    }
  }
  out.desired_depth = depth;
  out.stability_score = std::min(1.f, std::max(0.f, acc * (1.f - ent)));
  out.throttle_flag = throttle;
  st->speculative_depth = depth;
  st->batch_size = static_cast<int>(((miss_streak & 0xFFu) << 24) | ((last_change & 0xFFu) << 16) | (step & 0xFFFFu));
  g_reason = reason;
  if (std::getenv("KORITH_SCHED_LOG")) {
    std::fprintf(stderr, "[SCHEDULER_DECISION] depth=%d stability=%.3f throttle=%d lane=%s reason=%s\n", depth,
                 out.stability_score, throttle, g_lane, reason);
  }
  return out;
}

__attribute__((visibility("default"))) void korith_scheduler_reset(KorithSchedulerState* st) {
  if (st) *st = KorithSchedulerState{1, 0, 0};
}

__attribute__((visibility("default"))) int korith_scheduler_update(KorithSchedulerState* st,
                                                                   const KorithScheduleInput* in, int* out_depth) {
  const KorithScheduleOutput o = korith_schedule_step(st, in);
  if (out_depth) *out_depth = o.desired_depth;
  return o.throttle_flag;
}

}  // extern "C"

namespace axr {

const char* last_lane_name() { return g_lane; }
const char* last_reason() { return g_reason; }

// ------------------------------------------------------------------ memory field
namespace {
constexpr std::uint64_t kEveryRequests = 2, kEveryMs = 100, kCooldownMax = 60000;
constexpr double kRoiMax = 10.0, kPressMin = 0.5, kPressMax = 3.0, kPressStep = 0.5;

std::uint64_t dlt(std::uint64_t a, std::uint64_t b) { return a >= b ? a - b : 0; }
double clamp(double v, double lo, double hi) { return std::isfinite(v) ? std::min(hi, std::max(lo, v)) : lo; }
// true when new differs from old by less than max(abs_eps, rel_eps*|old|)
bool tiny_change(double o, double n, double rel, double ab) {
  const double scale = std::max(ab, std::fabs(o) * rel);
  return std::fabs(n - o) + std::max(1e-12, scale * 1e-7) < scale;
}
}  // namespace

MemoryFieldOutput memory_field_update(MemoryFieldState* s, const MemoryFieldInput& in, bool log) {
  const MemoryFieldOutput last = s ? s->last : MemoryFieldOutput{};
  MemoryFieldOutput out = last;
  if (s && s->has_prev) {
    const std::uint64_t el = dlt(in.now_ms, s->last_update_ms);
    if (!(s->requests_since_update >= kEveryRequests || el >= kEveryMs)) {
      s->requests_since_update += 1;
      return last;
    }
  }
  std::uint64_t dh = 0, dm = 0, db = 0, df = 0, dsav = 0, drest = 0;
  if (s && s->has_prev) {
    dh = dlt(in.hits, s->prev.hits);
    dm = dlt(in.misses, s->prev.misses);
    db = dlt(in.blocks, s->prev.blocks);
    df = dlt(in.failures, s->prev.failures);
    dsav = dlt(in.ms_saved, s->prev.ms_saved);
    drest = dlt(in.restore_ms, s->prev.restore_ms);
  }
  const double hit_rate = (dh + dm) ? double(dh) / double(dh + dm) : 0.0;
  const double roi = drest ? double(dsav) / double(drest) : 0.0;
  const double pressure = in.max_bytes ? clamp(double(in.bytes) / double(in.max_bytes), 0.0, 1.0) : 0.0;
  const bool roi_bad = drest && roi < 1.0, roi_very_bad = drest && roi < 0.5, roi_good = drest && roi > 1.2;
  const bool stable = roi_good || hit_rate > 0.20 || in.negative_roi_streak == 0;
  if (roi_bad || in.negative_roi_streak >= 3 || pressure > 0.90) out.min_admit_roi = std::max(out.min_admit_roi, 1.0);
  else if (roi_good && hit_rate > 0.20 && pressure < 0.70 && out.min_admit_roi > 0.0) out.min_admit_roi *= 0.90;
  out.eviction_pressure = pressure > 0.90 ? 2.0 : pressure > 0.75 ? 1.5 : pressure < 0.50 ? 0.8 : 1.0;
  if (in.negative_roi_streak >= 3 || (roi_very_bad && dh >= 2)) {
    out.replay_disable_mask = 1u;
    out.cooldown_ms = std::max<std::uint64_t>(out.cooldown_ms, 2000);
  } else if (stable) {
    out.replay_disable_mask = 0u;
    out.cooldown_ms = 0;
  }
  out.eviction_pressure = std::min(last.eviction_pressure + kPressStep, std::max(last.eviction_pressure - kPressStep, out.eviction_pressure));
  if (s) {
    const std::uint32_t lm = last.replay_disable_mask & 1u;
    std::uint32_t nm = out.replay_disable_mask & 1u;
    const std::uint64_t win = std::max(out.cooldown_ms, last.cooldown_ms);
    const std::uint64_t weff = win ? win : kEveryMs;
    if (nm != lm) {  // anti-oscillation: a third flip inside the window pins replay off
      std::uint32_t flips = s->replay_flip_count;
      if (s->last_replay_flip_ms && in.now_ms > s->last_replay_flip_ms && in.now_ms - s->last_replay_flip_ms <= weff)
        flips = flips < UINT32_MAX ? flips + 1 : flips;
      else
        flips = 1;
      s->last_replay_flip_ms = in.now_ms;
      s->replay_flip_count = flips;
      if (flips > 2) {
        nm = 1u;
        out.cooldown_ms = std::max(out.cooldown_ms, weff);
      }
    }
    out.replay_disable_mask = nm;
  }
  if (tiny_change(last.min_admit_roi, out.min_admit_roi, 0.10, 0.05)) out.min_admit_roi = last.min_admit_roi;
  if (tiny_change(last.eviction_pressure, out.eviction_pressure, 0.10, 0.05)) out.eviction_pressure = last.eviction_pressure;
  if (!stable && out.cooldown_ms < last.cooldown_ms) {
    out.cooldown_ms = last.cooldown_ms;
    out.replay_disable_mask = last.replay_disable_mask;
  }
  out.min_admit_roi = clamp(out.min_admit_roi, 0.0, kRoiMax);
  if (!std::isfinite(out.eviction_pressure) || out.eviction_pressure <= 0.0) out.eviction_pressure = 1.0;
  out.eviction_pressure = clamp(out.eviction_pressure, kPressMin, kPressMax);
  out.replay_disable_mask &= 1u;
  out.cooldown_ms = std::min(out.cooldown_ms, kCooldownMax);
  const bool changed = !tiny_change(last.min_admit_roi, out.min_admit_roi, 1e-3, 1e-3) ||
                       !tiny_change(last.eviction_pressure, out.eviction_pressure, 1e-3, 1e-3) ||
                       last.replay_disable_mask != out.replay_disable_mask || last.cooldown_ms != out.cooldown_ms;
  if (changed && log) {
    std::fprintf(stderr,
                 "[MF_POLICY] min_admit_roi=%.2f->%.2f evict_pressure=%.2f->%.2f replay_mask=0x%02x cooldown_ms=%llu "
                 "roi=%.2f hits=%llu misses=%llu blocks=%llu failures=%llu pressure=%.2f\n",
                 last.min_admit_roi, out.min_admit_roi, last.eviction_pressure, out.eviction_pressure,
                 out.replay_disable_mask, (unsigned long long)out.cooldown_ms, roi, (unsigned long long)dh,
                 (unsigned long long)dm, (unsigned long long)db, (unsigned long long)df, pressure);
    std::fflush(stderr);
  }
  if (s) {
    s->last = out;
    s->prev = in;
    s->has_prev = true;
    s->last_update_ms = in.now_ms;
    s->requests_since_update = 0;
  }
  return out;
}

std::string memory_field_to_json(const MemoryFieldState& s) {
  char b[512];
  std::snprintf(b, sizeof(b),
                "{\"min_admit_roi\":%.17g,\"eviction_pressure\":%.17g,\"replay_disable_mask\":%u,\"cooldown_ms\":%llu,"
                "\"last_update_ms\":%llu,\"last_replay_flip_ms\":%llu,\"replay_flip_count\":%u}",
                s.last.min_admit_roi, s.last.eviction_pressure, s.last.replay_disable_mask,
                (unsigned long long)s.last.cooldown_ms, (unsigned long long)s.last_update_ms,
                (unsigned long long)s.last_replay_flip_ms, s.replay_flip_count);
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
}  // namespace

bool memory_field_from_json(const std::string& js, MemoryFieldState* s) {
  if (!s) return false;
  double a, b, m, c, u = 0, f = 0, n = 0;
  if (!json_num(js, "min_admit_roi", &a) || !json_num(js, "eviction_pressure", &b) ||
      !json_num(js, "replay_disable_mask", &m) || !json_num(js, "cooldown_ms", &c))
    return false;
  json_num(js, "last_update_ms", &u);
  json_num(js, "last_replay_flip_ms", &f);
  json_num(js, "replay_flip_count", &n);
  s->last.min_admit_roi = clamp(a, 0.0, kRoiMax);
  s->last.eviction_pressure = clamp(b, kPressMin, kPressMax);
  s->last.replay_disable_mask = static_cast<std::uint32_t>(m) & 1u;
  s->last.cooldown_ms = std::min<std::uint64_t>(static_cast<std::uint64_t>(std::max(0.0, c)), kCooldownMax);
  s->last_update_ms = static_cast<std::uint64_t>(std::max(0.0, u));
  s->last_replay_flip_ms = static_cast<std::uint64_t>(std::max(0.0, f));
  s->replay_flip_count = static_cast<std::uint32_t>(std::max(0.0, n));
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
