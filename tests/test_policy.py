"""Policy layer on the CPU: state vector from a fake engine, hysteresis admission, UCB1
convergence to the best speculative depth, fail-closed execution and clamps, the endpoint
model against a fake OpenAI-compatible server, reward ledger, GAE against a hand-computed
case, PPO / REINFORCE learning a depth rule, FedAvg (direct and over the fake NATS server),
curricula, PID anti-windup, the batch controller over a fake NVML, and the worker hooks.

Reference: platform/reasoning (adaptive_engine, decision_executor, reward_calculator,
rollout_buffer, learning_loop, federated_loop) and python/power.py, controller.py.
"""
import json
import threading
import types
from http.server import BaseHTTPRequestHandler, ThreadingHTTPServer

import numpy as np
import pytest
import torch

from axropus_deploy_b200.policy import (REWARD_WEIGHTS, WIDTH, AdaptivePolicy, BatchController, Decision,
                                        DecisionExecutor, DepthPolicy, EndpointModel, FederatedAverager, Pid,
                                        PolicyOrchestrator, PowerSampler, RewardLedger, RolloutBuffer, Slot,
                                        StateCollector, curriculum, fedavg, power_fraction, ppo_update,
                                        read_decode_config, reinforce_update)
from axropus_deploy_b200.policy.decide import DEPTHS
from axropus_deploy_b200.cluster.runtime import SpecKController


def _vec(**kw):
    v = np.zeros(WIDTH, np.float32)
    for k, x in kw.items():
        v[getattr(Slot, k)] = x
    return v


def test_state_collector_from_fake_engine():
    eng = types.SimpleNamespace(stat={"decode_tokens": 0, "prefill_tokens": 0, "restored_tokens": 0},
                                amf=types.SimpleNamespace(stat={"hits_g1_raw": 0, "misses": 0, "restore_ms": 0.0,
                                                                "captures": 0, "capture_failures": 0}),
                                bm=types.SimpleNamespace(num_blocks=100, num_free=lambda: 25), _graphs=object())
    c = StateCollector(eng)
    c.sample()
    eng.amf.stat.update(hits_g1_raw=3, misses=1, restore_ms=21.0)
    eng.stat.update(decode_tokens=500, prefill_tokens=500, restored_tokens=8192)
    c.record_decode_step(drafted=10, accepted=8, depth=6, entropy=0.2)
    v = c.sample()
    assert v.shape == (WIDTH,) and v.dtype == np.float32
    assert v[Slot.HIT_RATE] == pytest.approx(0.75) and v[Slot.HIT_DELTA] == 3 and v[Slot.MISS_DELTA] == 1
    assert v[Slot.KV_CACHE_UTILIZATION] == pytest.approx(0.75) and v[Slot.CUDA_GRAPH_ACTIVE] == 1.0
    assert v[Slot.ACCEPTANCE_EMA] == pytest.approx(0.16) and v[Slot.CURRENT_SPEC_DEPTH] == pytest.approx(6 / 16)
    assert v[Slot.INSTANT_TPS_NORM] > 0
    assert np.array_equal(c.vector(), v)


def test_hysteresis_admission_does_not_flap():
    p = AdaptivePolicy()
    seq = []
    for roi in [0.5] * 30 + [0.25] * 40 + [0.0] * 40 + [0.33] * 40 + [0.6] * 40:
        seq.append(p.decide(_vec(ROI_EMA_NORM=roi / 10.0)).cache_admission)
    after = seq[29:]  # the ROI EMA starts at 0 and has warmed up by then
    flips = sum(1 for a, b in zip(after, after[1:]) if a != b)
    # 0.25 and 0.33 sit inside the band [0.22, 0.38]: the state set before them holds
    assert seq[29] and seq[69] and not seq[109] and not seq[149] and seq[-1] and flips == 2


def test_ucb1_finds_best_depth():
    p = AdaptivePolicy()
    rng = np.random.default_rng(0)
    best = 8
    picks = []
    for i in range(600):
        d = p.decide(_vec(HIT_RATE=0.9, ENTROPY_EMA=0.7))
        picks.append(d.spec_decode_depth)
        acc = float(np.clip(0.9 - abs(d.spec_decode_depth - best) * 0.08 + rng.normal(0, 0.05), 0, 1))
        p.record_outcome("pfx", spec_depth=d.spec_decode_depth, admitted=True, was_hit=rng.random() < 0.5,
                         acceptance_rate=acc)
    late = picks[-200:]
    assert max(set(late), key=late.count) == best
    assert p.tenant_stats()["arm_pulls"][best] > 100


def test_prewarm_and_model_band():
    calls = []

    class M:
        def decide(self, v):
            calls.append(1)
            return Decision(spec_decode_depth=12, is_fallback=False)

    p = AdaptivePolicy(model=M())
    for _ in range(4):
        p.record_outcome("hot", was_hit=True, admitted=True, acceptance_rate=0.9)
    p.record_outcome("cold", was_hit=True)
    d = p.decide(_vec(HIT_RATE=0.0))
    assert d.pre_warm_predictions == ["hot"] and not calls  # confident: rules
    for _ in range(30):
        d = p.decide(_vec(HIT_RATE=0.5))  # EMA climbs into the uncertainty band
    assert calls and d.spec_decode_depth == 12 and p.stat["model"] == len(calls)


def test_executor_clamps_and_fails_closed(tmp_path):
    spec = SpecKController(4)
    amf = types.SimpleNamespace(capture_enabled=True)
    cfg = str(tmp_path / "decode.json")
    ex = DecisionExecutor(spec, amf, config_path=cfg)
    r = ex.execute(Decision(spec_decode_depth=16, cache_admission=False, throttle_back_pressure=0.9))
    assert r["applied"] and spec.k == spec.MAX_K and r["clamped"] and not amf.capture_enabled
    assert ex.back_pressure == 0.5 and read_decode_config(cfg)["spec_depth"] == spec.MAX_K
    r = ex.execute(Decision(spec_decode_depth=8), _vec(ACCEPTANCE_EMA=0.1, CURRENT_SPEC_DEPTH=0.5))
    assert spec.k == 3 and r["spec_depth"] == 3 and r["clamped"]  # low acceptance caps depth at 3
    before = (spec.k, amf.capture_enabled, ex.back_pressure)
    r = ex.execute(Decision(spec_decode_depth=40, draft_temperature=float("nan"), cache_admission=True))
    assert not r["applied"] and len(r["reasons"]) == 2 and ex.stat["rejected"] == 1
    assert (spec.k, amf.capture_enabled, ex.back_pressure) == before


def test_endpoint_model_parses_and_falls_back():
    answers = [json.dumps({"decode": {"spec_decode_depth": 6, "draft_temperature": 0.4},
                           "prefill": {"cache_admission": False}}), "not json", json.dumps({"spec_decode_depth": 99})]

    class H(BaseHTTPRequestHandler):
        def log_message(self, *a):
            pass

        def do_POST(self):
            body = json.loads(self.rfile.read(int(self.headers["Content-Length"])))
            assert "HIT_RATE" in body["messages"][1]["content"]
            out = json.dumps({"choices": [{"message": {"content": "decision: " + answers.pop(0)}}]}).encode()
            self.send_response(200)
            self.send_header("Content-Length", str(len(out)))
            self.end_headers()
            self.wfile.write(out)

    srv = ThreadingHTTPServer(("127.0.0.1", 0), H)
    threading.Thread(target=srv.serve_forever, daemon=True).start()
    try:
        m = EndpointModel(f"http://127.0.0.1:{srv.server_address[1]}")
        d = m.decide(_vec(HIT_RATE=0.5))
        assert not d.is_fallback and d.spec_decode_depth == 6 and not d.cache_admission
        assert m.decide(_vec()).is_fallback and m.decide(_vec()).is_fallback
        assert EndpointModel("http://127.0.0.1:1", timeout_s=0.5).decide(_vec()).is_fallback
    finally:
        srv.shutdown()
        srv.server_close()


def test_reward_ledger_and_gae():
    led = RewardLedger()
    d1 = led.record_decision(Decision(spec_decode_depth=8), _vec(HIT_RATE=0.5))
    d2 = led.record_decision(Decision(spec_decode_depth=4), _vec())
    assert led.record_outcome(d1, "hit_admitted") == 1.0
    led.record_outcome(d1, "spec_depth_wasteful")
    with pytest.raises(ValueError):
        led.record_outcome(d2, "bogus")
    assert led.reward(d1) == pytest.approx(0.5) and REWARD_WEIGHTS["eviction_miss"] == -1.0
    s, a, r = led.unconsumed()
    assert s.shape == (1, WIDTH) and a.tolist() == [DEPTHS.index(8)] and r.tolist() == [0.5]
    assert len(led.unconsumed()[1]) == 0  # consumed once
    b = RolloutBuffer(4)
    for rew, val, done in [(1.0, 0.5, False), (0.0, 0.4, False), (2.0, 0.2, True)]:
        b.add(np.zeros(WIDTH), 0, 0.0, val, rew, done)
    adv, ret = b.gae(last_value=9.0, gamma=0.9, lam=0.8)
    d2_ = 2.0 - 0.2
    d1_ = 0.0 + 0.9 * 0.2 - 0.4
    d0_ = 1.0 + 0.9 * 0.4 - 0.5
    want = [d0_ + 0.72 * (d1_ + 0.72 * d2_), d1_ + 0.72 * d2_, d2_]
    assert np.allclose(adv, want) and np.allclose(ret, np.array(want) + [0.5, 0.4, 0.2])


@pytest.mark.parametrize("algo", ["ppo", "reinforce"])
def test_learned_depth_policy(algo):
    torch.manual_seed(0)
    rng = np.random.default_rng(0)
    pol = DepthPolicy()
    opt = torch.optim.Adam(pol.parameters(), lr=3e-3 if algo == "ppo" else 1e-2)

    def target(s):
        return DEPTHS.index(12) if s[Slot.ENTROPY_EMA] < 0.5 else DEPTHS.index(4)

    for _ in range(60 if algo == "ppo" else 200):
        states = np.zeros((64, WIDTH), np.float32)
        states[:, Slot.ENTROPY_EMA] = rng.random(64)
        if algo == "ppo":
            buf = RolloutBuffer(64)
            for s in states:
                a, lp, v = pol.act(s)
                buf.add(s, a, lp, v, 1.0 if a == target(s) else 0.0, True)
            ppo_update(pol, opt, buf, epochs=2)
        else:
            acts = np.array([pol.act(s)[0] for s in states])
            rew = np.array([1.0 if a == target(s) else 0.0 for s, a in zip(states, acts)], np.float32)
            reinforce_update(pol, opt, states, acts, rew)
    lo, hi = _vec(ENTROPY_EMA=0.1), _vec(ENTROPY_EMA=0.9)
    assert pol.depth(lo) == 12 and pol.depth(hi) == 4


def test_fedavg_and_over_nats():
    from tests.test_netstores import _fake_nats
    from axropus_deploy_b200.cluster.netqueues import NatsClient

    a = {"w": np.ones(3, np.float32)}
    b = {"w": np.full(3, 4.0, np.float32)}
    assert np.allclose(fedavg([(a, 1), (b, 3)])["w"], 3.25)
    srv = _fake_nats()
    url = f"nats://127.0.0.1:{srv.server_address[1]}"
    try:
        base = {"w": torch.zeros(3)}
        out = {}

        def node(name, delta, n):
            fa = FederatedAverager(NatsClient(url), name, quorum=2, timeout_s=10)
            ready.wait()
            out[name] = fa.round(1, delta, n, base)

        ready = threading.Barrier(2)
        ths = [threading.Thread(target=node, args=("n0", a, 1)), threading.Thread(target=node, args=("n1", b, 3))]
        [t.start() for t in ths]
        [t.join(20) for t in ths]
        for name in ("n0", "n1"):
            state, k = out[name]
            assert k == 2 and torch.allclose(state["w"], torch.full((3,), 3.25))
    finally:
        srv.shutdown()
        srv.server_close()


def test_curriculum_levels():
    easy, hard = curriculum(0, 200), curriculum(5, 200)
    assert easy.reuse > hard.reuse and easy.prefixes < hard.prefixes and easy.zipf > hard.zipf
    reuse_easy = np.mean([r["expect_hit"] for r in easy.requests])
    assert reuse_easy > 0.8 and len({r["tenant"] for r in hard.requests}) > 1
    assert curriculum(3, 10, seed=1).requests == curriculum(3, 10, seed=1).requests


def test_pid_antiwindup_and_batch_controller_on_fake_nvml():
    pid = Pid(1.0, 1.0, 0.0, setpoint=1.0, out_min=-1.0, out_max=1.0)
    for _ in range(50):
        pid.update(0.0, 1.0)  # saturated high: the integral must not keep growing
    assert pid.i <= 1.0
    watts = {"w": 1000.0}

    class FakeNvml:
        def nvmlInit(self):
            pass

        def nvmlShutdown(self):
            pass

        def nvmlDeviceGetHandleByIndex(self, i):
            return i

        def nvmlDeviceGetPowerUsage(self, h):
            return int(watts["w"] * 1000)

        def nvmlDeviceGetEnforcedPowerLimit(self, h):
            return 1000 * 1000

    t = {"now": 0.0}
    ps = PowerSampler(0, nvml=FakeNvml(), window_s=0.5, clock=lambda: t["now"])
    eng = types.SimpleNamespace(cfg=types.SimpleNamespace(max_batch=64))
    bc = BatchController(eng, power_fraction(ps), setpoint=0.9, min_batch=4, kp=40, ki=20,
                         clock=lambda: t["now"])
    for _ in range(40):  # toy plant: power follows the batch cap
        t["now"] += 1.0
        cap = bc.step()
        watts["w"] = 400 + 600 * cap / 64
    assert 4 <= cap < 64 and abs(watts["w"] / 1000 - 0.9) < 0.05
    assert ps.read()["limit_w"] == 1000.0


def test_orchestrator_hooks_fail_closed_and_train():
    col = StateCollector()
    spec = SpecKController(4)
    orch = PolicyOrchestrator(col, executor=DecisionExecutor(spec), rewards=RewardLedger(), learner=DepthPolicy())
    tok = orch.before_job({"org_id": "acme", "fingerprint_hash": "fp1"})
    assert tok is not None and orch.stat["decisions"] == 1
    orch.after_job(tok, {"amf": {"decision": "hit", "tier": "g1_raw", "saved_ms": 100.0},
                         "spec": {"drafted": 10, "accepted": 9}, "perf": {}}, mode="speculative")
    assert orch.stat["outcomes"] >= 2 and orch.train() is not None and orch.stat["train_steps"] == 1

    class Broken:
        def decide(self, *a):
            raise RuntimeError("boom")

    bad = PolicyOrchestrator(col, policy=Broken())
    assert bad.before_job({}) is None and bad.stat["hook_failures"] == 1
    bad.after_job(("x", None, "t", "p"), {})  # malformed token: swallowed
    assert bad.stat["hook_failures"] == 2


def test_dpo_prefers_chosen_depth():
    import copy

    from axropus_deploy_b200.policy import dpo_update

    torch.manual_seed(0)
    pol = DepthPolicy()
    ref = copy.deepcopy(pol)
    opt = torch.optim.Adam(pol.parameters(), lr=1e-2)
    rng = np.random.default_rng(0)
    for _ in range(150):
        s = np.zeros((32, WIDTH), np.float32)
        s[:, Slot.ENTROPY_EMA] = rng.random(32)
        low = s[:, Slot.ENTROPY_EMA] < 0.5
        chosen = np.where(low, DEPTHS.index(12), DEPTHS.index(4))
        rejected = np.where(low, DEPTHS.index(4), DEPTHS.index(12))
        dpo_update(pol, ref, opt, s, chosen, rejected, beta=0.5)
    assert pol.depth(_vec(ENTROPY_EMA=0.1)) == 12 and pol.depth(_vec(ENTROPY_EMA=0.9)) == 4


def test_adversarial_workloads_and_trace_replay():
    from axropus_deploy_b200.cluster.ledger import SqliteLedger
    from axropus_deploy_b200.engine.block_manager import block_hashes
    from axropus_deploy_b200.policy import adversarial, replay_trace

    th = adversarial("thrash", 300, pool_prefixes=8, prefix_len=64)
    keys = [tuple(r["prompt"][:64]) for r in th]
    assert len(set(keys)) == 16 and keys[0] == keys[16] and keys[0] != keys[8]
    nd = adversarial("near_duplicate", 8, prefix_len=256)
    h0 = block_hashes(np.asarray(nd[0]["prompt"][:256]), 16)
    h1 = block_hashes(np.asarray(nd[1]["prompt"][:256]), 16)
    assert h0[:15] == h1[:15] and h0[15] != h1[15]  # only the last block differs
    assert len({tuple(r["prompt"][:64]) for r in adversarial("one_shot", 20, prefix_len=64)}) == 20
    with pytest.raises(ValueError):
        adversarial("nope")
    led = SqliteLedger(":memory:")
    for i in range(3):
        led.insert_job(f"j{i}", f"2026-01-0{i + 1}T00:00:00Z", {"prompt": [1, 2, i], "max_tokens": 8}, {}, "p", f"f{i}",
                       None, "SUCCEEDED")
    tr = replay_trace(led)
    assert [r["prompt"] for r in tr] == [[1, 2, 0], [1, 2, 1], [1, 2, 2]] and tr[0]["max_tokens"] == 8


def test_policy_loop_example_drives_the_engine():
    import importlib.util
    import os

    path = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "examples", "policy_loop.py")
    spec = importlib.util.spec_from_file_location("policy_loop", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    out = mod.run(levels=(0,), n_requests=8)
    lv = out["levels"][0]
    assert lv["amf_hits"] >= 4 and lv["admit_now"] is True  # high reuse: restores happen, admission stays on
    assert out["rewards"]["hit_admitted"]["count"] == lv["amf_hits"]


def test_lowered_max_batch_caps_running_sequences():
    from axropus_deploy_b200.engine import EngineConfig, LLMEngine, SamplingParams
    from axropus_deploy_b200.models.config import get_config
    from axropus_deploy_b200.models.llama import LlamaModel

    eng = LLMEngine(LlamaModel(get_config("tiny"), "cpu", seed=0),
                    EngineConfig(num_blocks=128, max_model_len=256, max_batch=8))
    eng.cfg.max_batch = 2  # what BatchController does
    reqs = [eng.add_request(list(range(1, 20 + i)), SamplingParams(max_tokens=3)) for i in range(5)]
    peak = 0
    while eng.has_unfinished():
        eng.step()
        peak = max(peak, len(eng.running))
    assert peak == 2 and all(len(r.output) == 3 for r in reqs)
    eng.close()
