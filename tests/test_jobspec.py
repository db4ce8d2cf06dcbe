"""korith.jobspec.v1 contract (cluster/jobspec.py) and its enforcement by the control plane."""
import pytest

from axropus_deploy_b200.cluster import jobspec as js


def _spec(**kw):
    s = {"schema_version": "korith.jobspec.v1", "backend_id": "axr_engine", "model": {"model_id": "tiny"},
         "prompt": "hello", "deterministic_cfg": {"seed": 1, "n_ctx": 2048, "n_batch": 512, "max_tokens": 4},
         "policy": {"allow_amf_reuse": True, "allow_spec": False}}
    s.update(kw)
    return s


def test_valid_spec_and_translation():
    s = _spec(owner={"org_id": "acme"}, idempotency_key="k1")
    assert js.validate(s) == []
    job = js.to_job(s)
    assert job["prompt"] == "hello" and job["max_tokens"] == 4 and job["org_id"] == "acme"
    assert job["deterministic"]["seed"] == 1 and job["deterministic"]["temperature"] == 0.0
    t = _spec(prompt_template="Summarise {doc} in {n} words")
    del t["prompt"]
    t["input"] = {"doc": "X", "n": 5}
    assert js.validate(t) == [] and js.to_job(t)["prompt"] == "Summarise X in 5 words"


@pytest.mark.parametrize("mutate, needle", [
    (lambda s: s.update(extra=1), "extra: not allowed"),
    (lambda s: s.update(schema_version="korith.jobspec.v2"), "schema_version"),
    (lambda s: s.pop("policy"), "policy: required"),
    (lambda s: s["policy"].pop("allow_spec"), "policy.allow_spec: required"),
    (lambda s: s["deterministic_cfg"].update(n_ctx=128), "n_ctx: below 256"),
    (lambda s: s["deterministic_cfg"].update(seed=True), "seed: wrong type"),
    (lambda s: s["model"].update(weights="x"), "model.weights: not allowed"),
    (lambda s: s.update(prompt_template="{a}"), "exactly one"),
    (lambda s: s.update(backend_id="vllm"), "model.endpoint"),
    (lambda s: s.update(backend_id="korith_cuda"), "model.model_path"),
    (lambda s: s.update(owner={"org_id": ""}), "owner.org_id: empty"),
])
def test_violations(mutate, needle):
    s = _spec()
    mutate(s)
    errs = js.validate(s)
    assert any(needle in e for e in errs), errs


def test_control_plane_enforces_v1():
    from axropus_deploy_b200.cluster.control import ControlPlane, JobError

    class _L:
        def find_job_by_idempotency(self, *a):
            return None

    cp = ControlPlane(_L(), {}, strict_jobspec=True)
    with pytest.raises(JobError, match="korith.jobspec.v1"):
        cp._validate({"prompt": "hi", "max_tokens": 4})  # short form refused in strict mode
    with pytest.raises(JobError, match="not allowed"):
        cp._validate(_spec(extra=True))
    job = cp._validate(_spec())
    assert job["prompt"] == "hello" and job["max_tokens"] == 4 and job["backend_id"] == "axr_engine"
    loose = ControlPlane(_L(), {}, strict_jobspec=False)
    assert loose._validate({"prompt": "hi", "max_tokens": 4})["prompt"] == "hi"
