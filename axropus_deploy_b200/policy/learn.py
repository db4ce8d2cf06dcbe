"""Learning side of the policy layer: rewards, rollouts, policy updates, federation and
synthetic curricula.

* :class:`RewardLedger` -- every decision (its state vector and JSON) and every outcome
  observed for it, in SQLite; an outcome's reward comes from :data:`REWARD_WEIGHTS` (the
  reference's outcome names and weights, so reward logs stay comparable across the two);
  :meth:`RewardLedger.unconsumed` hands (state, action, reward) samples to training once.
* :class:`RolloutBuffer` -- fixed-capacity (state, action, log-prob, value, reward, done)
  storage with generalised advantage estimation (GAE, Schulman et al. 2016) and returns.
* :class:`DepthPolicy` + :func:`ppo_update` / :func:`reinforce_update` -- a small MLP over
  the state vector with a categorical head over the speculative depths and a value head,
  trained with the clipped PPO objective (Schulman et al. 2017) or plain REINFORCE with a
  baseline. It runs on the CPU or the GPU; its size (a few thousand parameters) keeps an
  update far below a decode step's cost, so it can run beside serving.
* :func:`fedavg` / :class:`FederatedAverager` -- sample-weighted averaging of parameter
  deltas from many nodes, carried over NATS (subject ``amf.federated.gradient``) with this
  framework's NATS client; each message is one node's delta as base64 ``.npz``.
* :func:`curriculum` -- synthetic serving workloads by difficulty level: prefix reuse, prefix
  length, Zipf skew, suffix length and tenant count grow with the level, for training the
  policy and for soak tests.

Reference: platform/reasoning/reward_calculator.py:98-196, rollout_buffer.py:46-206,
learning_loop.py:159 (PPO / DPO / REINFORCE loop; here over a small policy instead of a
LoRA of an 8B model), federated_loop.py:115-385 and gradient_aggregator.py:104 (FedAvg over
NATS), curriculum.py:73-841.
"""
from __future__ import annotations

import base64
import io
import json
import sqlite3
import threading
import time
import uuid
from dataclasses import dataclass
from typing import Any, Dict, List, Optional, Sequence, Tuple

import numpy as np
import torch

from .decide import DEPTHS, Decision
from .state import WIDTH

REWARD_WEIGHTS: Dict[str, float] = {
    "hit_admitted": 1.0, "miss_never_reused": -0.5, "eviction_miss": -1.0, "pre_warm_hit": 1.0,
    "pre_warm_miss": -0.3, "route_improvement": 0.5, "route_regression": -0.5, "spec_high_acceptance": 1.0,
    "spec_low_acceptance": -0.8, "spec_depth_optimal": 0.5, "spec_depth_wasteful": -0.5, "spec_mode_match": 0.3,
    "spec_mode_mismatch": -0.3, "kv_compress_saved_oom": 1.5, "kv_compress_unnecessary": -0.2,
    "decode_latency_improved": 0.5, "decode_latency_worsened": -0.5, "cuda_graph_speedup": 0.3,
    "early_stop_correct": 0.8, "early_stop_premature": -0.6, "replicate_hit": 0.7, "replicate_waste": -0.3,
    "evict_hint_correct": 0.4, "evict_hint_wrong": -0.8,
}


class RewardLedger:
    def __init__(self, path: str = ":memory:"):
        self._db = sqlite3.connect(path, check_same_thread=False)
        self._mu = threading.Lock()
        self._db.executescript(
            "CREATE TABLE IF NOT EXISTS decisions (decision_id TEXT PRIMARY KEY, ts REAL NOT NULL, tenant_id TEXT NOT "
            "NULL, node_id TEXT NOT NULL, action INTEGER NOT NULL, state BLOB NOT NULL, decision_json TEXT NOT NULL, "
            "consumed INTEGER NOT NULL DEFAULT 0);"
            "CREATE TABLE IF NOT EXISTS outcomes (decision_id TEXT NOT NULL, ts REAL NOT NULL, outcome TEXT NOT NULL, "
            "reward REAL NOT NULL, detail_json TEXT NOT NULL DEFAULT '{}');"
            "CREATE INDEX IF NOT EXISTS outcomes_d ON outcomes(decision_id);")

    def record_decision(self, d: Decision, state: np.ndarray, tenant_id: str = "default", node_id: str = "") -> str:
        did = uuid.uuid4().hex
        action = DEPTHS.index(d.spec_decode_depth) if d.spec_decode_depth in DEPTHS else -1
        with self._mu:
            self._db.execute("INSERT INTO decisions VALUES (?,?,?,?,?,?,?,0)",
                             (did, time.time(), tenant_id, node_id, action,
                              np.asarray(state, np.float32).tobytes(), json.dumps(d.to_dict())))
            self._db.commit()
        return did

    def record_outcome(self, decision_id: str, outcome: str, detail: Optional[Dict[str, Any]] = None) -> float:
        if outcome not in REWARD_WEIGHTS:
            raise ValueError(f"unknown outcome {outcome!r}")
        r = REWARD_WEIGHTS[outcome]
        with self._mu:
            self._db.execute("INSERT INTO outcomes VALUES (?,?,?,?,?)",
                             (decision_id, time.time(), outcome, r, json.dumps(detail or {})))
            self._db.commit()
        return r

    def reward(self, decision_id: str) -> float:
        with self._mu:
            row = self._db.execute("SELECT COALESCE(SUM(reward), 0) FROM outcomes WHERE decision_id=?",
                                   (decision_id,)).fetchone()
        return float(row[0])

    def unconsumed(self, limit: int = 4096) -> Tuple[np.ndarray, np.ndarray, np.ndarray]:
        """(states [n, WIDTH], actions [n], rewards [n]) of decisions with at least one outcome
        and a depth action, marked consumed."""
        with self._mu:
            rows = self._db.execute(
                "SELECT d.decision_id, d.state, d.action, SUM(o.reward) FROM decisions d JOIN outcomes o "
                "ON o.decision_id = d.decision_id WHERE d.consumed = 0 AND d.action >= 0 GROUP BY d.decision_id "
                "ORDER BY d.ts LIMIT ?", (int(limit),)).fetchall()
            self._db.executemany("UPDATE decisions SET consumed=1 WHERE decision_id=?", [(r[0],) for r in rows])
            self._db.commit()
        if not rows:
            return np.zeros((0, WIDTH), np.float32), np.zeros(0, np.int64), np.zeros(0, np.float32)
        s = np.stack([np.frombuffer(r[1], np.float32) for r in rows])
        return s, np.array([r[2] for r in rows], np.int64), np.array([r[3] for r in rows], np.float32)

    def scored(self, limit: int = 4096, consume: bool = True) -> List[Dict[str, Any]]:
        """Decisions with at least one outcome and not yet consumed, oldest first, as
        ``{decision_id, state, decision, reward}`` rows (``decision`` a :class:`Decision`);
        marked consumed unless ``consume`` is False."""
        with self._mu:
            rows = self._db.execute(
                "SELECT d.decision_id, d.state, d.decision_json, SUM(o.reward) FROM decisions d JOIN outcomes o "
                "ON o.decision_id = d.decision_id WHERE d.consumed = 0 GROUP BY d.decision_id ORDER BY d.ts LIMIT ?",
                (int(limit),)).fetchall()
            if consume:
                self._db.executemany("UPDATE decisions SET consumed=1 WHERE decision_id=?", [(r[0],) for r in rows])
                self._db.commit()
        return [{"decision_id": r[0], "state": np.frombuffer(r[1], np.float32).copy(),
                 "decision": Decision.from_dict(json.loads(r[2])), "reward": float(r[3])} for r in rows]

    def summary(self) -> Dict[str, Any]:
        with self._mu:
            rows = self._db.execute("SELECT outcome, COUNT(*), SUM(reward) FROM outcomes GROUP BY outcome").fetchall()
        return {o: {"count": n, "reward": r} for o, n, r in rows}


class RolloutBuffer:
    def __init__(self, capacity: int, width: int = WIDTH):
        self.cap = capacity
        self.s = np.zeros((capacity, width), np.float32)
        self.a = np.zeros(capacity, np.int64)
        self.logp = np.zeros(capacity, np.float32)
        self.v = np.zeros(capacity, np.float32)
        self.r = np.zeros(capacity, np.float32)
        self.done = np.zeros(capacity, np.float32)
        self.n = 0

    def add(self, s, a: int, logp: float, v: float, r: float, done: bool) -> None:
        if self.n >= self.cap:
            raise OverflowError("rollout buffer full")
        i = self.n
        self.s[i], self.a[i], self.logp[i], self.v[i], self.r[i], self.done[i] = s, a, logp, v, r, float(done)
        self.n += 1

    def gae(self, last_value: float = 0.0, gamma: float = 0.99, lam: float = 0.95) -> Tuple[np.ndarray, np.ndarray]:
        """Advantages and returns: delta_t = r_t + gamma V_{t+1} (1 - done_t) - V_t,
        A_t = delta_t + gamma lam (1 - done_t) A_{t+1}, return_t = A_t + V_t."""
        n = self.n
        adv = np.zeros(n, np.float32)
        nxt_v, run = last_value, 0.0
        for t in range(n - 1, -1, -1):
            live = 1.0 - self.done[t]
            delta = self.r[t] + gamma * nxt_v * live - self.v[t]
            run = delta + gamma * lam * live * run
            adv[t] = run
            nxt_v = self.v[t]
        return adv, adv + self.v[:n]

    def clear(self) -> None:
        self.n = 0


class DepthPolicy(torch.nn.Module):
    def __init__(self, width: int = WIDTH, hidden: int = 64, n_actions: int = len(DEPTHS)):
        super().__init__()
        self.body = torch.nn.Sequential(torch.nn.Linear(width, hidden), torch.nn.Tanh(),
                                        torch.nn.Linear(hidden, hidden), torch.nn.Tanh())
        self.pi = torch.nn.Linear(hidden, n_actions)
        self.value = torch.nn.Linear(hidden, 1)

    def forward(self, s: torch.Tensor) -> Tuple[torch.distributions.Categorical, torch.Tensor]:
        h = self.body(s)
        return torch.distributions.Categorical(logits=self.pi(h)), self.value(h).squeeze(-1)

    @torch.no_grad()
    def act(self, s: np.ndarray, greedy: bool = False) -> Tuple[int, float, float]:
        dist, v = self(torch.as_tensor(s, dtype=torch.float32).unsqueeze(0))
        a = int(dist.probs.argmax(-1)) if greedy else int(dist.sample())
        return a, float(dist.log_prob(torch.tensor([a]))), float(v)

    def depth(self, s: np.ndarray) -> int:
        return DEPTHS[self.act(s, greedy=True)[0]]


def ppo_update(policy: DepthPolicy, opt: torch.optim.Optimizer, buf: RolloutBuffer, epochs: int = 4,
               clip: float = 0.2, vf_coef: float = 0.5, ent_coef: float = 0.01, last_value: float = 0.0,
               minibatch: int = 64) -> Dict[str, float]:
    adv, ret = buf.gae(last_value)
    n = buf.n
    s = torch.as_tensor(buf.s[:n])
    a = torch.as_tensor(buf.a[:n])
    old = torch.as_tensor(buf.logp[:n])
    A = torch.as_tensor(adv)
    A = (A - A.mean()) / (A.std() + 1e-8) if n > 1 else A
    R = torch.as_tensor(ret)
    last = {}
    for _ in range(epochs):
        for idx in torch.randperm(n).split(minibatch):
            dist, v = policy(s[idx])
            ratio = torch.exp(dist.log_prob(a[idx]) - old[idx])
            pg = -torch.min(ratio * A[idx], ratio.clamp(1 - clip, 1 + clip) * A[idx]).mean()
            vf = torch.nn.functional.mse_loss(v, R[idx])
            ent = dist.entropy().mean()
            loss = pg + vf_coef * vf - ent_coef * ent
            opt.zero_grad()
            loss.backward()
            torch.nn.utils.clip_grad_norm_(policy.parameters(), 0.5)
            opt.step()
            last = {"loss": loss.item(), "policy": pg.item(), "value": vf.item(), "entropy": ent.item()}
    return last


def reinforce_update(policy: DepthPolicy, opt: torch.optim.Optimizer, states: np.ndarray, actions: np.ndarray,
                     rewards: np.ndarray) -> float:
    """One REINFORCE step with the value head as baseline, on logged (state, action, reward)."""
    s = torch.as_tensor(states)
    a = torch.as_tensor(actions)
    r = torch.as_tensor(rewards)
    dist, v = policy(s)
    adv = (r - v).detach()
    loss = -(dist.log_prob(a) * adv).mean() + 0.5 * torch.nn.functional.mse_loss(v, r)
    opt.zero_grad()
    loss.backward()
    opt.step()
    return loss.item()


def dpo_update(policy: DepthPolicy, ref: DepthPolicy, opt: torch.optim.Optimizer, states: np.ndarray,
               chosen: np.ndarray, rejected: np.ndarray, beta: float = 0.1) -> float:
    """One Direct Preference Optimization step (Rafailov et al. 2023) on (state, preferred
    depth, rejected depth) pairs -- for example the depth of the higher-reward of two logged
    decisions in the same state bucket: loss = -log sigmoid(beta * ((log pi(a_w) - log
    pi_ref(a_w)) - (log pi(a_l) - log pi_ref(a_l)))), ``ref`` frozen."""
    s = torch.as_tensor(states)
    w, l = torch.as_tensor(chosen), torch.as_tensor(rejected)
    dist, _ = policy(s)
    with torch.no_grad():
        rdist, _ = ref(s)
    margin = (dist.log_prob(w) - rdist.log_prob(w)) - (dist.log_prob(l) - rdist.log_prob(l))
    loss = -torch.nn.functional.logsigmoid(beta * margin).mean()
    opt.zero_grad()
    loss.backward()
    opt.step()
    return loss.item()


# ---------------------------------------------------------------------- federation
def state_delta(model: torch.nn.Module, base: Dict[str, torch.Tensor]) -> Dict[str, np.ndarray]:
    return {k: (v.detach().cpu() - base[k].cpu()).numpy() for k, v in model.state_dict().items()}


def fedavg(deltas: Sequence[Tuple[Dict[str, np.ndarray], int]]) -> Dict[str, np.ndarray]:
    """Average of per-node deltas weighted by each node's sample count."""
    total = sum(n for _, n in deltas)
    if total <= 0:
        raise ValueError("no samples to average")
    keys = deltas[0][0].keys()
    return {k: sum(d[k].astype(np.float64) * n for d, n in deltas).astype(np.float32) / total for k in keys}


def _pack(delta: Dict[str, np.ndarray], n: int, node: str, rnd: int) -> bytes:
    buf = io.BytesIO()
    np.savez(buf, **delta)
    return json.dumps({"node": node, "round": rnd, "samples": n,
                       "npz": base64.b64encode(buf.getvalue()).decode()}).encode()


def _unpack(data: bytes) -> Tuple[Dict[str, np.ndarray], int, str, int]:
    m = json.loads(data)
    z = np.load(io.BytesIO(base64.b64decode(m["npz"])))
    return {k: z[k] for k in z.files}, int(m["samples"]), m["node"], int(m["round"])


class FederatedAverager:
    """Every node publishes its delta for round ``r`` and collects the others'; once
    ``quorum`` nodes (itself included) have reported, or ``timeout_s`` passed with at least
    one, it applies the FedAvg of what it has to ``base`` and returns the new state."""

    SUBJECT = "amf.federated.gradient"

    def __init__(self, nats_client, node_id: str, quorum: int, timeout_s: float = 30.0):
        self.nc, self.node, self.quorum, self.timeout_s = nats_client, node_id, quorum, timeout_s
        self.sid = self.nc.subscribe(self.SUBJECT)
        self.nc.flush()
        self._early: Dict[int, Dict[str, Tuple[Dict[str, np.ndarray], int]]] = {}

    def round(self, rnd: int, delta: Dict[str, np.ndarray], n: int,
              base: Dict[str, torch.Tensor]) -> Tuple[Dict[str, torch.Tensor], int]:
        self.nc.publish(self.SUBJECT, _pack(delta, n, self.node, rnd))
        got = self._early.pop(rnd, {})
        got[self.node] = (delta, n)
        deadline = time.monotonic() + self.timeout_s
        while len(got) < self.quorum and time.monotonic() < deadline:
            data = self.nc.next_msg(self.sid, min(0.5, max(0.0, deadline - time.monotonic())))
            if data is None:
                continue
            d, k, node, r = _unpack(data)
            if r == rnd:
                got[node] = (d, k)
            elif r > rnd:
                self._early.setdefault(r, {})[node] = (d, k)
        avg = fedavg(list(got.values()))
        return {k: base[k] + torch.as_tensor(avg[k]).to(base[k].dtype) for k in base}, len(got)


# ---------------------------------------------------------------------- curriculum
@dataclass
class Workload:
    level: int
    requests: List[Dict[str, Any]]
    prefixes: int
    reuse: float
    zipf: float


def curriculum(level: int, n_requests: int = 256, vocab: int = 32000, seed: int = 0) -> Workload:
    """Level 0 is easy (few long shared prefixes, high reuse, one tenant); each level adds
    prefixes, lowers reuse, flattens the Zipf skew, lengthens suffixes and adds tenants."""
    lv = max(0, int(level))
    rng = np.random.default_rng(seed + lv)
    n_pref = 4 * (lv + 1)
    reuse = max(0.2, 0.95 - 0.12 * lv)
    zipf = max(1.05, 2.0 - 0.2 * lv)
    pref_len = 512 * (1 + lv % 4)
    suffix = 32 * (1 + lv)
    tenants = 1 + lv // 2
    prefixes = [rng.integers(0, vocab, pref_len).tolist() for _ in range(n_pref)]
    w = 1.0 / np.arange(1, n_pref + 1) ** zipf
    w /= w.sum()
    reqs = []
    for i in range(n_requests):
        fresh = rng.random() > reuse
        p = rng.integers(0, vocab, pref_len).tolist() if fresh else prefixes[int(rng.choice(n_pref, p=w))]
        reqs.append({"prompt": p + rng.integers(0, vocab, suffix).tolist(), "amf_prefix_len": pref_len,
                     "tenant": f"t{int(rng.integers(0, tenants))}", "max_tokens": 16 + 16 * (lv % 3),
                     "expect_hit": not fresh})
    return Workload(lv, reqs, n_pref, reuse, zipf)


def adversarial(kind: str, n_requests: int = 256, vocab: int = 32000, pool_prefixes: int = 64,
                prefix_len: int = 1024, seed: int = 0) -> List[Dict[str, Any]]:
    """Workloads that stress the cache policy:

    * ``thrash`` -- cycles through 2 x ``pool_prefixes`` prefixes in order, so an LRU pool
      sized for ``pool_prefixes`` misses every time (admission should back off);
    * ``near_duplicate`` -- prefixes that differ from one base in a single token near the end
      (block hashing must not confuse them; only the shared leading blocks may hit);
    * ``burst`` -- long runs of one prefix then a switch, to test hysteresis and pre-warming;
    * ``one_shot`` -- every prefix seen once (admission should turn off)."""
    rng = np.random.default_rng(seed)
    base = rng.integers(0, vocab, prefix_len).tolist()
    reqs: List[Dict[str, Any]] = []
    if kind == "thrash":
        pref = [rng.integers(0, vocab, prefix_len).tolist() for _ in range(2 * pool_prefixes)]
        seq = [pref[i % len(pref)] for i in range(n_requests)]
    elif kind == "near_duplicate":
        seq = []
        for i in range(n_requests):
            p = list(base)
            p[prefix_len - 1 - (i % 7)] = int((p[prefix_len - 1 - (i % 7)] + 1 + i) % vocab)
            seq.append(p)
    elif kind == "burst":
        pref = [rng.integers(0, vocab, prefix_len).tolist() for _ in range(max(1, n_requests // 32))]
        seq = [pref[(i // 32) % len(pref)] for i in range(n_requests)]
    elif kind == "one_shot":
        seq = [rng.integers(0, vocab, prefix_len).tolist() for _ in range(n_requests)]
    else:
        raise ValueError(f"unknown adversarial workload {kind!r}")
    for p in seq:
        reqs.append({"prompt": p + rng.integers(0, vocab, 32).tolist(), "amf_prefix_len": prefix_len,
                     "tenant": "t0", "max_tokens": 16})
    return reqs


def replay_trace(ledger, limit: int = 1000, org_id: Optional[str] = None) -> List[Dict[str, Any]]:
    """Requests of the most recent jobs in a ledger, oldest first, in the shape the
    curricula use -- to replay production traffic against a new policy offline."""
    out = []
    for j in reversed(ledger.list_jobs(limit, org_id=org_id)):
        spec = json.loads(j["jobspec_json"])
        out.append({"prompt": spec.get("prompt"), "amf_prefix_len": spec.get("amf_prefix_len"),
                    "tenant": j["org_id"], "max_tokens": int(spec.get("max_tokens", 16)),
                    "fingerprint_hash": j["fingerprint_hash"]})
    return out
