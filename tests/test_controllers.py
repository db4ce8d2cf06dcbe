"""Native runtime controllers: spec-depth scheduler (Python binding and its C ABI),
memory field, thermo controller, event ring, rolling metrics, spec plan, collapse gate."""
import ctypes
import json

import numpy as np
import pytest

from axropus_deploy_b200._native_loader import native

n = native()


def _run(st, k, acc, ent, reuse=0.0, tps=0.0):
    o = None
    for _ in range(k):
        o = n.schedule_step(st, acc, ent, current_tps=tps, amf_reuse_score=reuse)
    return o


def test_best_depth_follows_the_speedup_model():
    # expected tokens / cost: a = 0 -> no speculation pays; high a -> deep drafts
    assert n.best_depth(0.0, 0.08, 16) == 1
    assert n.best_depth(0.95, 0.08, 16) >= 8
    assert n.best_depth(0.95, 0.5, 16) < n.best_depth(0.95, 0.05, 16)  # expensive drafts: shallower
    assert n.best_depth(0.99, 0.01, 4) == 4  # capped


def test_scheduler_warmup_and_lane_classification():
    st = n.SchedulerState()
    o = n.schedule_step(st, 0.95, 0.1, baseline_ready=False)
    assert o["desired_depth"] == 1 and o["lane"] == "MISS" and o["reason"] == "warmup"
    # replayed prefix + high quality -> SPEC_HIT, but only after the lane debounce (3 steps)
    o = n.schedule_step(st, 0.95, 0.1, amf_reuse_score=0.9)
    assert o["lane"] == "MISS"
    o = _run(st, 3, 0.95, 0.1, reuse=0.9)
    assert o["lane"] == "SPEC_HIT" and o["throttle_flag"] == 3
    # reuse alone -> HIT; a worse lane is taken at once
    st2 = n.SchedulerState()
    o = _run(st2, 4, 0.3, 0.8, reuse=0.9)
    assert o["lane"] == "HIT" and o["throttle_flag"] == 2
    o = _run(st2, 10, 0.1, 0.95, reuse=0.0)
    assert o["lane"] == "MISS" and o["desired_depth"] <= 3


def test_scheduler_hysteresis_up_slow_down_fast():
    st = n.SchedulerState()
    _run(st, 5, 0.95, 0.1, reuse=0.9)
    d0 = st.depth
    # increases wait hold_up_steps (24) between them and move by at most 2
    depths = [n.schedule_step(st, 0.95, 0.1, amf_reuse_score=0.9)["desired_depth"] for _ in range(100)]
    ups = [b - a for a, b in zip([d0] + depths, depths) if b > a]
    assert ups and max(ups) <= 2
    change_steps = [i for i in range(1, len(depths)) if depths[i] != depths[i - 1]]
    assert all(b - a >= 24 for a, b in zip(change_steps, change_steps[1:]))
    top = depths[-1]
    assert top > 4
    # a collapse of acceptance lowers the depth on the next steps without waiting
    o = n.schedule_step(st, 0.0, 1.0)
    assert o["desired_depth"] < top and o["reason"] in ("down", "miss_down")
    o = _run(st, 3, 0.0, 1.0)
    assert o["desired_depth"] <= 3


def test_scheduler_starvation_probe_and_periodic_probe():
    st = n.SchedulerState()
    reasons = [n.schedule_step(st, 0.55, 0.7)["reason"] for _ in range(200)]
    assert "starvation_probe" in reasons  # MISS lane with usable acceptance: a deeper draft is measured again
    st = n.SchedulerState()
    reasons = [n.schedule_step(st, 0.0, 1.0)["reason"] for _ in range(100)]
    assert "probe" in reasons and "starvation_probe" not in reasons  # no usable acceptance: only the depth-1 probe


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

    lib.korith_scheduler_reset.argtypes = []
    lib.korith_scheduler_reset()
    f = lib.korith_schedule_step
    f.restype = Out
    f.argtypes = [ctypes.POINTER(St), ctypes.POINTER(In)]
    st = St(1, 0, 0)
    for _ in range(80):
        out = f(ctypes.byref(st), ctypes.byref(In(0.95, 0.1, 0, 0, 0.9, 0, 0, 0, 1)))
    assert out.throttle_flag == 3 and out.desired_depth > 1 and st.speculative_depth == out.desired_depth
    assert st.batch_size == 256 // (out.desired_depth + 1) and st.baseline_ready == 1
    upd = lib.korith_scheduler_update
    upd.restype = ctypes.c_uint
    upd.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_float]
    assert upd(0.2, 0.9, 0.0) >= 1
    lib.korith_scheduler_reset()
    # handle API: independent states
    lib.korith_scheduler_create.restype = ctypes.c_void_p
    lib.korith_scheduler_step_ex.restype = Out
    lib.korith_scheduler_step_ex.argtypes = [ctypes.c_void_p, ctypes.POINTER(In)]
    lib.korith_scheduler_destroy.argtypes = [ctypes.c_void_p]
    h1, h2 = lib.korith_scheduler_create(), lib.korith_scheduler_create()
    for _ in range(60):
        a = lib.korith_scheduler_step_ex(h1, ctypes.byref(In(0.95, 0.1, 0, 0, 0.9, 0, 0, 0, 1)))
        b = lib.korith_scheduler_step_ex(h2, ctypes.byref(In(0.05, 0.95, 0, 0, 0.0, 0, 0, 0, 1)))
    assert a.desired_depth > b.desired_depth and a.throttle_flag == 3 and b.throttle_flag == 1
    lib.korith_scheduler_destroy(h1)
    lib.korith_scheduler_destroy(h2)


def _mf(st, now, **kw):
    d = {"now_ms": now, "max_bytes": 1000, "bytes": kw.pop("bytes", 100)}
    d.update(kw)
    return n.memory_field_update(st, d)


def test_memory_field_fill_drives_bar_and_pressure_with_slew():
    st = n.MemoryFieldState()
    o = _mf(st, 0)
    assert o["min_admit_roi"] == 0.0 and o["eviction_pressure"] == pytest.approx(0.75)
    outs = [_mf(st, 200 * (i + 1), bytes=990) for i in range(12)]
    steps = [b["eviction_pressure"] - a["eviction_pressure"] for a, b in zip([o] + outs, outs)]
    assert max(steps) <= 0.25 + 1e-9 and outs[-1]["eviction_pressure"] > 2.9
    assert outs[-1]["min_admit_roi"] == pytest.approx(5.0 * (0.99 - 0.6), abs=1e-6)
    assert max(b["min_admit_roi"] - a["min_admit_roi"] for a, b in zip([o] + outs, outs)) <= 0.5 + 1e-9


def test_memory_field_replay_gate_and_backoff():
    st = n.MemoryFieldState()
    _mf(st, 0)
    # restores that cost 10x what they save, with hits: replay off, 2 s cooldown
    o = _mf(st, 200, hits=4, misses=1, ms_saved=10, restore_ms=100)
    assert o["replay_disable_mask"] == 1 and 0 < o["cooldown_ms"] <= 2000
    assert _mf(st, 1200, hits=4, misses=1, ms_saved=10, restore_ms=100)["replay_disable_mask"] == 1
    # cooldown over: probation (replay on again, ROI measured afresh)
    o = _mf(st, 2300, hits=4, misses=1, ms_saved=10, restore_ms=100)
    assert o["replay_disable_mask"] == 0 and o["cooldown_ms"] == 0
    # still bad: off again within 60 s -> the cooldown doubles (anti-oscillation)
    o = _mf(st, 2500, hits=8, misses=2, ms_saved=20, restore_ms=200)
    assert o["replay_disable_mask"] == 1 and 2000 < o["cooldown_ms"] <= 4000
    js = st.to_json()
    st2 = n.MemoryFieldState()
    assert st2.from_json(js) and st2.last == st.last
    assert json.loads(js)["backoff"] == 1
    assert not n.MemoryFieldState().from_json("{}")


def test_memory_field_cadence():
    st = n.MemoryFieldState()
    first = _mf(st, 0)
    assert _mf(st, 10, bytes=990) == first  # too soon and too few requests: unchanged
    _mf(st, 20, bytes=990)
    _mf(st, 30, bytes=990)
    b = _mf(st, 40, bytes=990)  # fourth request since the last update
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
