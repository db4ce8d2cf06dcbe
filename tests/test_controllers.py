"""Native runtime controllers: spec-depth scheduler (Python binding and its C ABI),
memory field, thermo controller, event ring, rolling metrics, spec plan, collapse gate."""
import ctypes
import json

import numpy as np
import pytest

from axropus_deploy_b200._native_loader import native

n = native()


def test_scheduler_warmup_lanes_hysteresis():
    st = n.SchedulerState()
    o = n.schedule_step(st, 0.95, 0.2, baseline_ready=False)
    assert o["desired_depth"] == 1 and o["throttle_flag"] == 1 and o["reason"] == "warmup"
    # first change is blocked by hysteresis (step 1 is within 32 steps of step 0)
    o = n.schedule_step(st, 0.95, 0.2, amf_reuse_score=0.9)
    assert o["lane"] == "SPEC_HIT" and o["throttle_flag"] == 3 and o["desired_depth"] == 1
    for _ in range(40):
        o = n.schedule_step(st, 0.95, 0.2, amf_reuse_score=0.9)
    assert o["desired_depth"] > 1 and o["desired_depth"] <= 16
    # a miss lane forces the depth down immediately (no hysteresis on the way down)
    o = n.schedule_step(st, 0.3, 0.9)
    assert o["lane"] == "MISS" and o["desired_depth"] == 2 and o["reason"] == "miss_cap"
    o = n.schedule_step(st, 0.72, 0.6)
    assert o["lane"] == "HIT" and o["throttle_flag"] == 2
    assert 0.0 <= o["stability_score"] <= 1.0


def test_scheduler_c_abi():
    lib = ctypes.CDLL(n.__file__)

    class St(ctypes.Structure):
        _fields_ = [("speculative_depth", ctypes.c_int), ("batch_size", ctypes.c_int), ("baseline_ready", ctypes.c_int)]

    class In(ctypes.Structure):
        _fields_ = [(k, ctypes.c_float) for k in ("acceptance", "entropy", "current_tps", "engine_costs",
                                                  "amf_reuse_score", "amf_avg_prefix_length", "amf_accept_rate",
                                                  "amf_restore_cost_ms")] + [("baseline_ready", ctypes.c_int)]

    class Out(ctypes.Structure):
        _fields_ = [("desired_depth", ctypes.c_int), ("stability_score", ctypes.c_float),
                    ("throttle_flag", ctypes.c_int)]

    f = lib.korith_schedule_step
    f.restype = Out
    f.argtypes = [ctypes.POINTER(St), ctypes.POINTER(In)]
    st = St(1, 0, 0)
    for _ in range(40):
        out = f(ctypes.byref(st), ctypes.byref(In(0.95, 0.2, 0, 0, 0.9, 0, 0, 0, 1)))
    assert out.throttle_flag == 3 and out.desired_depth > 1 and st.speculative_depth == out.desired_depth
    lib.korith_scheduler_reset(ctypes.byref(st))
    assert (st.speculative_depth, st.batch_size, st.baseline_ready) == (1, 0, 0)


def test_memory_field_policy_and_snapshot():
    st = n.MemoryFieldState()
    base = {"now_ms": 1000, "max_bytes": 1000, "bytes": 100}
    n.memory_field_update(st, base)
    # bad ROI window with hits -> replay disabled with a cooldown, admission bar raised
    o = n.memory_field_update(st, dict(base, now_ms=1200, hits=4, misses=1, ms_saved=10, restore_ms=100))
    assert o["replay_disable_mask"] == 1 and o["cooldown_ms"] >= 2000 and o["min_admit_roi"] >= 1.0
    # high pressure -> eviction pressure rises by at most 0.5 per update
    o2 = n.memory_field_update(st, dict(base, now_ms=1400, bytes=990, hits=4, misses=1, ms_saved=10, restore_ms=100))
    assert o2["eviction_pressure"] <= o["eviction_pressure"] + 0.5 + 1e-9
    js = st.to_json()
    st2 = n.MemoryFieldState()
    assert st2.from_json(js) and st2.last == st.last
    assert json.loads(js)["cooldown_ms"] <= 60000
    assert not n.MemoryFieldState().from_json("{}")


def test_memory_field_cadence():
    st = n.MemoryFieldState()
    first = n.memory_field_update(st, {"now_ms": 0})
    a = n.memory_field_update(st, {"now_ms": 10, "max_bytes": 100, "bytes": 99})  # too soon: unchanged
    assert a == first
    n.memory_field_update(st, {"now_ms": 20, "max_bytes": 100, "bytes": 99})
    b = n.memory_field_update(st, {"now_ms": 30, "max_bytes": 100, "bytes": 99})  # after 2 skipped requests
    assert b["eviction_pressure"] > first["eviction_pressure"]


def test_thermo_ring_metrics_plan_collapse():
    t = n.ThermoState(8)
    for _ in range(20):
        d = n.thermo_next_depth(t, 0.95, np.array([10.0, 0.0, 0.0, 0.0], dtype=np.float32))
    assert d > 2 and t.accept_ema > 0.9
    d2 = n.thermo_next_depth(t, 0.0, np.zeros(1000, dtype=np.float32))  # entropy spike
    assert d2 <= d // 2 + 1
    assert abs(n.normalized_entropy(np.zeros(16, dtype=np.float32)) - 1.0) < 1e-6
    r = n.HoloRing(4)
    for i in range(6):
        r.record(i, 1.0, 0.0, 2)
    assert len(r) == 4 and [e[0] for e in r.recent(4)] == [2, 3, 4, 5]
    assert abs(r.future_safe(4) - 1.0) < 1e-9
    m = n.RollingMetrics(10.0)
    m.record(0.0, 100, 500.0)
    m.record(1.0, 100, 500.0)
    assert m.tps(1.0) == pytest.approx(200.0) and m.tokens_per_joule(1.0) == pytest.approx(200 / 500.0)
    assert n.resolve_spec_plan(False, True, False, 4, 0, True, 1, 0, 16)["reason"] == "env_off"
    assert n.resolve_spec_plan(True, True, False, 4, 0, True, 0.3, 0.5, 16)["reason"] == "low_accept"
    assert n.resolve_spec_plan(True, True, False, 4, 20, True, 1, 0, 16) == {"enabled": True, "depth": 16,
                                                                           "reason": "none"}
    assert n.collapse_decide([(0.9, 1.0, 10.0, 4), (0.5, 1.0, 10.0, 2)]) == (True, 0)
    assert n.collapse_decide([(0.1, 5.0, 10.0, 4)]) == (False, -1)
