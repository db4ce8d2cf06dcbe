"""Soak / chaos runner on CPU nodes (axropus_deploy_b200/soak.py): every failure of the
list is injected between batches of jobs, and every job must still finish with the cold
reference tokens, as a restore or a cold prefill."""
import json
import os

from axropus_deploy_b200.soak import EVENTS, Soak


def test_soak_every_failure_and_every_job_finishes(tmp_path):
    rep = Soak(str(tmp_path), nodes=3, jobs=45, prefixes=8, visibility_s=3.0, deadline_s=400.0).run()
    assert rep["ok"], rep
    assert rep["finished"] == 45 and not rep["missing"] and not rep["mismatches"]
    assert set(rep["tiers"]) <= {"cold", "apc", "g1_raw", "disk"}
    assert rep["tiers"].get("cold", 0) > 0 and rep["restored_results"] + rep["tiers"].get("apc", 0) > 0
    for ev in EVENTS:  # each failure happened (none was skipped)
        assert rep["chaos_events"].get(ev, 0) >= 1, (ev, rep["chaos_events"])
    lines = [json.loads(x) for x in open(os.path.join(tmp_path, "chaos_events.jsonl"))]
    assert {x["event"] for x in lines} >= set(EVENTS)
