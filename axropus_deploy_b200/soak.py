"""Soak / chaos runner: serving nodes under repeated failures, on the host.

``python -m axropus_deploy_b200.soak --nodes 3 --jobs 60 --out DIR [--device cpu]``

Node processes (one engine each, with a G1 pool, the AMF disk store under
``DIR/amf_node<r>`` written on every capture, and a tiny random-init Llama) take jobs
from one durable SQLite queue (``cluster/queues.py``: a job taken by a node that dies
stays in flight and is handed out again after the visibility timeout) and record
every finished job in ``DIR/results.db``. The parent fills the queue, computes the
cold reference output of every job with its own engine, and injects failures while the
nodes serve -- one failure, then a batch of jobs that meets its effect, for every failure
in turn (``--rounds`` passes) -- logging each one to ``DIR/chaos_events.jsonl``:

* ``node_kill``      SIGKILL of a node, possibly in the middle of a job
* ``node_restart``   a killed node started again on its disk store (restart recovery)
* ``blob_corrupt``   bytes of a stored AMF blob flipped (its checksum must reject it)
* ``blob_truncate``  a stored blob cut short
* ``disk_full``      the disk store's writes fail with ENOSPC for a while (an injected
                     error of the write call), then recover (``disk_full_off``)
* ``g1_evict``       a node drops its G1 pool and live prefix cache (memory pressure)
* ``writer_lost``    a shard-directory insert whose writer vanishes mid-copy, reclaimed

At the end every job must have finished, each result must equal the cold reference
tokens, and each must have ended as a restore (``g1_raw`` / ``disk`` / ``apc``) or a
cold prefill. ``DIR/soak_report.json`` holds the counts, the tier mix, latencies and
the verdict. No GPU is faulted, trapped or hung: every failure is made on the host.

Reference counterpart: scripts/soak_chaos.py:846-916 (chaos loop: worker kills and
restarts, router restart, autoscaling, disk pressure, ``chaos_events.jsonl``).
"""
from __future__ import annotations

import argparse
import json
import os
import random
import signal
import sqlite3
import statistics
import sys
import time
from typing import Dict, List, Optional

EVENTS = ("node_kill", "blob_corrupt", "disk_full", "g1_evict", "node_restart", "blob_truncate", "writer_lost",
          "disk_full_off")
TIERS_OK = {"cold", "apc", "g1_raw", "g1_pool", "disk", "lmcache"}


# ----------------------------------------------------------------------------- node
def _node_main(rank: int, c: dict) -> None:
    import numpy as np  # noqa: F401
    import torch

    torch.set_num_threads(max(1, int(c.get("threads", 1))))
    from .amf.disk import DiskTier
    from .amf.manager import AmfManager
    from .amf.pool import G1Pool
    from .cluster.queues import SqliteQueue
    from .engine import EngineConfig, LLMEngine, SamplingParams
    from .models.config import get_config
    from .models.llama import LlamaModel

    out = c["out"]
    dev = torch.device(c["device"])
    cfg = get_config(c["model"])
    model = LlamaModel(cfg, dev, seed=0)
    pool = G1Pool(cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, "raw", c["g1_slots"], device=dev)
    disk = DiskTier(path=os.path.join(out, f"amf_node{rank}"))
    full_flag = os.path.join(out, "disk_full")
    real_save = disk.save

    def save(tokens, pages, saved_ms=0.0):  # the disk store's write, failing while the disk is "full"
        if os.path.exists(full_flag):
            raise OSError(28, "No space left on device (injected)")
        return real_save(tokens, pages, saved_ms)

    disk.save = save
    amf = AmfManager(raw_pool=pool, disk=disk, min_tokens=64, sync_save=True)
    eng = LLMEngine(model, EngineConfig(num_blocks=c["blocks"], max_model_len=c["max_len"], max_batch=2), amf)
    q = SqliteQueue(os.path.join(out, "queue.db"), "soak", visibility_s=c["visibility_s"])
    res = sqlite3.connect(os.path.join(out, "results.db"), timeout=30.0)
    hb = os.path.join(out, f"hb{rank}")
    ctl = os.path.join(out, f"ctl{rank}")
    stop = os.path.join(out, "stop")
    while True:
        with open(hb, "w") as f:
            f.write(str(time.time()))
        if os.path.exists(ctl):
            with open(ctl) as f:
                cmd = f.read().strip()
            os.remove(ctl)
            if cmd == "g1_evict":
                eng.evict_live_cache()
                pool.clear()
            elif cmd == "writer_lost":
                from .amf.keys import pool_key_int

                ghost = 7  # a writer rank that vanishes mid-copy
                key = pool_key_int("%032x" % random.getrandbits(128))
                pool.dir.begin_insert(0, key, 0, 2, 32, 0, ghost, 0.0)
                n = int(pool.dir.release_rank(ghost))
                with open(os.path.join(out, f"ctl{rank}.done"), "w") as f:
                    f.write(json.dumps({"reclaimed": n}))
        item = q.dequeue()
        if item is None:
            if os.path.exists(stop):
                break
            time.sleep(0.05)
            continue
        iid, job = item
        t0 = time.perf_counter()
        r = eng.add_request(job["prompt"], SamplingParams(max_tokens=job["max_tokens"]),
                            amf_prefix_len=job["prefix_len"])
        while eng.has_unfinished():
            eng.step()
        ms = (time.perf_counter() - t0) * 1e3
        res.execute("INSERT INTO results VALUES (?,?,?,?,?,?,?)",
                    (job["id"], rank, r.amf_tier, json.dumps(r.output), ms, r.restored_tokens, time.time()))
        res.commit()
        q.ack(iid)
    res.close()


# ----------------------------------------------------------------------------- parent
class Soak:
    def __init__(self, out: str, nodes: int = 3, jobs: int = 60, prefixes: int = 6, prefix_len: int = 256,
                 suffix_len: int = 24, max_tokens: int = 4, visibility_s: float = 4.0,
                 seed: int = 0, device: str = "cpu", model: str = "tiny", deadline_s: float = 600.0,
                 rounds: int = 1):
        self.out = out
        self.n_nodes, self.n_jobs = nodes, jobs
        self.prefixes, self.prefix_len, self.suffix_len = prefixes, prefix_len, suffix_len
        self.max_tokens, self.visibility_s = max_tokens, visibility_s
        self.rng = random.Random(seed)
        self.device, self.model, self.deadline_s = device, model, deadline_s
        self.rounds = rounds
        self.procs: Dict[int, Optional[object]] = {}
        self.dead_at: Dict[int, float] = {}
        self.chaos_path = os.path.join(out, "chaos_events.jsonl")

    # ---- setup
    def _jobs(self) -> List[dict]:
        vocab = 32000
        pref = [[self.rng.randrange(vocab) for _ in range(self.prefix_len)] for _ in range(self.prefixes)]
        jobs = []
        for j in range(self.n_jobs):
            p = pref[min(int(self.rng.paretovariate(1.2)) - 1, self.prefixes - 1)]
            suffix = [self.rng.randrange(vocab) for _ in range(self.suffix_len)]
            jobs.append({"id": j, "prompt": p + suffix, "prefix_len": self.prefix_len, "max_tokens": self.max_tokens})
        return jobs

    def _reference(self, jobs: List[dict]) -> Dict[int, List[int]]:
        import torch

        from .engine import EngineConfig, LLMEngine, SamplingParams
        from .models.config import get_config
        from .models.llama import LlamaModel

        model = LlamaModel(get_config(self.model), torch.device(self.device), seed=0)
        eng = LLMEngine(model, EngineConfig(num_blocks=256, max_model_len=1024, max_batch=2,
                                            enable_prefix_cache=False))
        ref = {}
        for jb in jobs:
            r = eng.add_request(jb["prompt"], SamplingParams(max_tokens=jb["max_tokens"]))
            while eng.has_unfinished():
                eng.step()
            ref[jb["id"]] = r.output
        return ref

    def _node_cfg(self) -> dict:
        return {"out": self.out, "device": self.device, "model": self.model, "g1_slots": 512, "blocks": 64,
                "max_len": 1024, "visibility_s": self.visibility_s, "threads": 1}

    def _spawn(self, rank: int) -> None:
        import multiprocessing as mp

        p = mp.get_context("spawn").Process(target=_node_main, args=(rank, self._node_cfg()), daemon=True)
        p.start()
        self.procs[rank] = p
        self.dead_at.pop(rank, None)

    def _log(self, event: str, **kw) -> None:
        rec = {"ts": time.time(), "event": event, **kw}
        with open(self.chaos_path, "a") as f:
            f.write(json.dumps(rec) + "\n")

    # ---- chaos
    def _live(self) -> List[int]:
        return [r for r, p in self.procs.items() if p is not None and p.is_alive()]

    def _blobs(self) -> List[str]:
        out = []
        for r in range(self.n_nodes):
            d = os.path.join(self.out, f"amf_node{r}")
            if os.path.isdir(d):
                out += [os.path.join(d, f) for f in sorted(os.listdir(d)) if f.endswith(".kv")]
        return out

    def _chaos(self, event: str) -> None:
        live = self._live()
        if event == "node_kill":
            if len(live) <= 1:
                return self._log(event, outcome="skipped: one node left")
            r = self.rng.choice(live)
            os.kill(self.procs[r].pid, signal.SIGKILL)
            self.procs[r].join(5)
            self.dead_at[r] = time.time()
            return self._log(event, node=r, outcome="killed")
        if event == "node_restart":
            dead = [r for r in self.procs if r not in live]
            if not dead:
                return self._log(event, outcome="skipped: none dead")
            r = dead[0]
            self._spawn(r)
            return self._log(event, node=r, outcome="restarted on its disk store")
        if event in ("blob_corrupt", "blob_truncate"):
            blobs = self._blobs()
            if not blobs:
                return self._log(event, outcome="skipped: no blob stored yet")
            path = self.rng.choice(blobs)
            size = os.path.getsize(path)
            if event == "blob_corrupt":
                with open(path, "r+b") as f:
                    for _ in range(8):
                        f.seek(self.rng.randrange(max(1, size)))
                        b = f.read(1)
                        f.seek(-1, 1)
                        f.write(bytes([(b[0] if b else 0) ^ 0xFF]))
            else:
                with open(path, "r+b") as f:
                    f.truncate(size // 2)
            return self._log(event, blob=os.path.basename(path), outcome="modified")
        if event == "disk_full":
            open(os.path.join(self.out, "disk_full"), "w").close()
            return self._log(event, outcome="disk writes fail with ENOSPC")
        if event == "disk_full_off":
            try:
                os.remove(os.path.join(self.out, "disk_full"))
            except FileNotFoundError:
                pass
            return self._log(event, outcome="disk writes recover")
        if event in ("g1_evict", "writer_lost"):
            if not live:
                return self._log(event, outcome="skipped: no live node")
            r = self.rng.choice(live)
            with open(os.path.join(self.out, f"ctl{r}"), "w") as f:
                f.write(event)
            return self._log(event, node=r, outcome="requested")
        raise ValueError(event)

    # ---- run
    def run(self) -> dict:
        from .cluster.queues import SqliteQueue

        os.makedirs(self.out, exist_ok=True)
        for f in ("queue.db", "results.db", "chaos_events.jsonl", "stop", "disk_full"):
            try:
                os.remove(os.path.join(self.out, f))
            except FileNotFoundError:
                pass
        jobs = self._jobs()
        ref = self._reference(jobs)
        db = sqlite3.connect(os.path.join(self.out, "results.db"), timeout=30.0)
        db.execute("CREATE TABLE results (job INTEGER, node INTEGER, tier TEXT, tokens TEXT, ms REAL, "
                   "restored INTEGER, ts REAL)")
        db.commit()
        q = SqliteQueue(os.path.join(self.out, "queue.db"), "soak", visibility_s=self.visibility_s)
        # Phased schedule: a batch of jobs after each failure, so every failure is followed by
        # traffic that meets its effect; batch 0 warms the nodes (and fills the tiers).
        n_batches = self.rounds * len(EVENTS) + 1
        batches = [jobs[i::n_batches] for i in range(n_batches)]
        t_start = time.time()
        for r in range(self.n_nodes):
            self._spawn(r)
        for b, batch in enumerate(batches):
            if b > 0:
                self._chaos(EVENTS[(b - 1) % len(EVENTS)])
            for jb in batch:
                q.enqueue(jb)
            want = {jb["id"] for jb in batch}
            while time.time() - t_start < self.deadline_s:
                done = {row[0] for row in db.execute("SELECT DISTINCT job FROM results")}
                if want <= done:
                    break
                if not self._live():  # never leave the queue without a consumer
                    r = min(self.procs)
                    self._spawn(r)
                    self._log("node_restart", node=r, outcome="restarted: no node was alive")
                time.sleep(0.05)
        open(os.path.join(self.out, "stop"), "w").close()
        for p in self.procs.values():
            if p is not None:
                p.join(30)
                if p.is_alive():
                    p.kill()
        return self._report(jobs, ref, db, time.time() - t_start)

    def _report(self, jobs, ref, db, wall_s) -> dict:
        rows = db.execute("SELECT job, node, tier, tokens, ms, restored FROM results").fetchall()
        by_job: Dict[int, list] = {}
        for job, node, tier, toks, ms, restored in rows:
            by_job.setdefault(job, []).append((node, tier, json.loads(toks), ms, restored))
        mismatches = [j for j, rs in by_job.items() if any(t != ref[j] for _, _, t, _, _ in rs)]
        bad_tiers = sorted({tier for rs in by_job.values() for _, tier, _, _, _ in rs} - TIERS_OK)
        missing = [jb["id"] for jb in jobs if jb["id"] not in by_job]
        tiers: Dict[str, int] = {}
        for rs in by_job.values():
            for _, tier, _, _, _ in rs:
                tiers[tier] = tiers.get(tier, 0) + 1
        events: Dict[str, int] = {}
        with open(self.chaos_path) as f:
            for line in f:
                e = json.loads(line)
                key = e["event"] + ("" if str(e.get("outcome", "")).startswith(("killed", "restarted", "modified",
                                                                                 "requested", "disk"))
                                    else ":skipped")
                events[key] = events.get(key, 0) + 1
        ms = sorted(x[3] for rs in by_job.values() for x in rs)
        rep = {
            "jobs": len(jobs), "finished": len(by_job), "missing": missing, "results": len(rows),
            "reruns": len(rows) - len(by_job), "mismatches": mismatches, "bad_tiers": bad_tiers, "tiers": tiers,
            "restored_results": sum(1 for rs in by_job.values() for x in rs if x[4] > 0),
            "latency_ms": {"p50": statistics.median(ms) if ms else None,
                           "p95": ms[min(len(ms) - 1, int(0.95 * len(ms)))] if ms else None},
            "chaos_events": events, "wall_s": round(wall_s, 1),
        }
        rep["ok"] = not missing and not mismatches and not bad_tiers
        with open(os.path.join(self.out, "soak_report.json"), "w") as f:
            json.dump(rep, f, indent=2)
        return rep


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--out", required=True)
    ap.add_argument("--nodes", type=int, default=3)
    ap.add_argument("--jobs", type=int, default=60)
    ap.add_argument("--prefixes", type=int, default=6)
    ap.add_argument("--rounds", type=int, default=1, help="passes over the failure list")
    ap.add_argument("--visibility", type=float, default=4.0)
    ap.add_argument("--device", default="cpu")
    ap.add_argument("--model", default="tiny")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--deadline", type=float, default=600.0)
    a = ap.parse_args(argv)
    rep = Soak(a.out, a.nodes, a.jobs, a.prefixes, visibility_s=a.visibility, seed=a.seed, device=a.device,
               model=a.model, deadline_s=a.deadline, rounds=a.rounds).run()
    print(json.dumps(rep))
    return 0 if rep["ok"] else 1


if __name__ == "__main__":
    sys.exit(main())
