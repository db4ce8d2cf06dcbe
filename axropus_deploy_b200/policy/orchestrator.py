"""Wiring of the policy layer into a worker, and feedback controllers for batch size.

:class:`PolicyOrchestrator` is what a :class:`~axropus_deploy_b200.cluster.worker.ClusterWorker`
calls around each run (``policy=`` argument): :meth:`before_job` reads the state vector,
asks the policy for a decision, applies it through the executor and logs it in the reward
ledger; :meth:`after_job` turns the run's result into outcomes (hit on an admitted prefix,
speculative acceptance high / low, a wasteful depth) for the ledger and the bandit; and
:meth:`train` runs one REINFORCE step of a learned depth policy on the logged samples. Every
hook is fail-closed: an exception inside it is counted and swallowed, and the run goes ahead
with the settings it had, so the policy layer can never fail a job.

:class:`Pid` is a textbook PID controller with output clamping and integral anti-windup;
:class:`BatchController` uses one to hold a measured signal (board power as a fraction of the
enforced limit from :class:`~.state.PowerSampler`, or decode latency per token) at a set
point by moving the engine's running-batch cap between ``min_batch`` and the batch size the
engine was built with (it never raises the cap above that, so buffers sized at start-up stay
valid).

Reference: platform/reasoning/orchestrator.py:98 and dynamo_reasoning_bridge.py:115 (wiring,
fail-closed), python/controller.py, physics_controller.py, physics_control.py (batch
controllers driven by power and latency).
"""
from __future__ import annotations

import logging
import time
from typing import Any, Callable, Dict, Optional, Tuple

import torch

from .decide import AdaptivePolicy, Decision, DecisionExecutor
from .learn import DepthPolicy, RewardLedger, reinforce_update
from .state import StateCollector

log = logging.getLogger(__name__)


class PolicyOrchestrator:
    def __init__(self, collector: StateCollector, policy: Optional[AdaptivePolicy] = None,
                 executor: Optional[DecisionExecutor] = None, rewards: Optional[RewardLedger] = None,
                 learner: Optional[DepthPolicy] = None, node_id: str = "", lr: float = 1e-3):
        self.collector = collector
        self.policy = policy or AdaptivePolicy()
        self.executor = executor or DecisionExecutor()
        self.rewards = rewards
        self.learner = learner
        self.opt = torch.optim.Adam(learner.parameters(), lr=lr) if learner is not None else None
        self.node_id = node_id
        self.stat = {"decisions": 0, "outcomes": 0, "hook_failures": 0, "train_steps": 0}

    def before_job(self, job: Dict[str, Any]) -> Optional[Tuple[str, Decision, str, str]]:
        try:
            v = self.collector.vector()
            tenant = str(job.get("org_id") or job.get("tenant") or "default")
            prefix = str(job.get("fingerprint_hash") or job.get("prefix_hash") or "")
            d = self.policy.decide(v, tenant, prefix)
            if self.learner is not None:
                d.spec_decode_depth = self.learner.depth(v)
            res = self.executor.execute(d, v)
            if not res.get("applied"):
                return None
            did = self.rewards.record_decision(d, v, tenant, self.node_id) if self.rewards is not None else ""
            self.stat["decisions"] += 1
            return did, d, tenant, prefix
        except Exception as e:
            self.stat["hook_failures"] += 1
            log.warning("policy before_job failed (run continues unchanged): %s", e)
            return None

    def after_job(self, token, result: Dict[str, Any], mode: str = "") -> None:
        if token is None:
            return
        try:
            did, d, tenant, prefix = token
            amf = result.get("amf") or {}
            hit = amf.get("decision") == "hit"
            sp = result.get("spec") or {}
            drafted, accepted = int(sp.get("drafted", 0)), int(sp.get("accepted", 0))
            acc = accepted / drafted if drafted else 0.0
            outcomes = []
            if hit and d.cache_admission:
                outcomes.append("hit_admitted")
            if mode == "speculative" and drafted:
                outcomes.append("spec_high_acceptance" if acc >= 0.8 else "spec_low_acceptance" if acc < 0.4
                                else "spec_depth_optimal")
                if d.spec_decode_depth > 8 and acc < 0.6:
                    outcomes.append("spec_depth_wasteful")
            if self.rewards is not None and did:
                for o in outcomes:
                    self.rewards.record_outcome(did, o, {"acceptance": acc, "tier": amf.get("tier")})
            self.collector.record_lookup(hit, float(amf.get("saved_ms", 0.0)),
                                         float((result.get("perf") or {}).get("restore_ms", 0.0)))
            if drafted:
                self.collector.record_decode_step(drafted, accepted, d.spec_decode_depth)
            self.policy.record_outcome(prefix, tenant, d.spec_decode_depth, d.cache_admission, hit, acc)
            self.stat["outcomes"] += len(outcomes)
        except Exception as e:
            self.stat["hook_failures"] += 1
            log.warning("policy after_job failed: %s", e)

    def train(self, limit: int = 4096) -> Optional[float]:
        """One REINFORCE step of the learned depth policy on unconsumed logged samples."""
        if self.learner is None or self.rewards is None:
            return None
        s, a, r = self.rewards.unconsumed(limit)
        if len(a) == 0:
            return None
        loss = reinforce_update(self.learner, self.opt, s, a, r)
        self.stat["train_steps"] += 1
        return loss


class Pid:
    def __init__(self, kp: float, ki: float, kd: float, setpoint: float, out_min: float, out_max: float):
        self.kp, self.ki, self.kd, self.setpoint = kp, ki, kd, setpoint
        self.out_min, self.out_max = out_min, out_max
        self.i = 0.0
        self.prev_err: Optional[float] = None

    def update(self, measured: float, dt: float) -> float:
        err = self.setpoint - measured
        d = 0.0 if self.prev_err is None or dt <= 0 else (err - self.prev_err) / dt
        self.prev_err = err
        i_new = self.i + err * dt
        out = self.kp * err + self.ki * i_new + self.kd * d
        if self.out_min <= out <= self.out_max:
            self.i = i_new  # integrate only while unsaturated (anti-windup)
        return max(self.out_min, min(self.out_max, out))


class BatchController:
    """Moves ``engine.cfg.max_batch`` (the cap on running sequences) to hold ``read()`` at
    ``setpoint``. ``read`` returns the controlled signal, for example power / limit (higher
    batch, more power) or decode ms per token; ``sign=-1`` when a higher batch lowers it."""

    def __init__(self, engine, read: Callable[[], float], setpoint: float, min_batch: int = 1,
                 kp: float = 32.0, ki: float = 8.0, kd: float = 0.0, sign: float = 1.0,
                 clock: Callable[[], float] = time.monotonic):
        self.engine, self.read, self.clock, self.sign = engine, read, clock, sign
        self.max_batch = int(engine.cfg.max_batch)
        self.min_batch = max(1, int(min_batch))
        span = float(self.max_batch - self.min_batch)
        self.pid = Pid(kp, ki, kd, setpoint, -span, span)
        self.base = float(self.max_batch)
        self._t = clock()

    def step(self) -> int:
        now = self.clock()
        dt, self._t = now - self._t, now
        u = self.pid.update(self.read(), dt)
        cap = int(round(max(self.min_batch, min(self.max_batch, self.base + self.sign * u))))
        self.engine.cfg.max_batch = cap
        return cap


def power_fraction(sampler) -> Callable[[], float]:
    def f() -> float:
        p = sampler.read()
        return p["avg_watts"] / p["limit_w"] if p["limit_w"] > 0 else 0.0
    return f
