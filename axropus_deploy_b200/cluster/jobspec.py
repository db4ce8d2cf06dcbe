"""The ``korith.jobspec.v1`` job contract: validation and translation.

The contract (platform/contracts/jobspec.schema.json in the reference; enforced by its
ClusterRouter._validate_jobspec, platform/runtime/cluster_router.py:1347) is kept field
for field, since clients written against the reference submit it: a JSON object with
no keys beyond the listed ones; ``schema_version`` == ``"korith.jobspec.v1"``;
``backend_id``; ``model.model_id``; ``deterministic_cfg`` with ``seed``, ``n_ctx``
(>= 256) and ``n_batch`` (>= 1); ``policy`` with ``allow_amf_reuse`` and ``allow_spec``;
exactly one of ``prompt`` / ``prompt_template`` (``input`` fills the template's
``{field}`` slots). Backends that need a path or an endpoint must name it.

:func:`validate` returns the list of violations (empty: valid); :func:`to_job` turns a
valid spec into the control plane's job dict.
"""
from __future__ import annotations

from typing import Any, Dict, List

SCHEMA_VERSION = "korith.jobspec.v1"

# field -> (types, required); nested objects carry their own field tables
_STR, _INT, _NUM, _BOOL, _OBJ = (str,), (int,), (int, float), (bool,), (dict,)
_OWNER = {"org_id": (_STR, False), "user_id": (_STR, False)}
_MODEL = {"model_id": (_STR, True), "model_path": (_STR, False), "endpoint": (_STR, False)}
_DET = {"seed": (_INT, True), "temperature": (_NUM, False), "top_p": (_NUM, False), "top_k": (_INT, False),
        "n_ctx": (_INT, True), "n_batch": (_INT, True), "max_tokens": (_INT, False)}
_POLICY = {"allow_amf_reuse": (_BOOL, True), "allow_spec": (_BOOL, True)}
_TOP = {"schema_version": (_STR, True), "job_id": (_STR, False), "parent_job_id": (_STR, False),
        "session_id": (_STR, False), "idempotency_key": (_STR, False), "owner": (_OBJ, False),
        "backend_id": (_STR, True), "model": (_OBJ, True), "prompt": (_STR, False),
        "prompt_template": (_STR, False), "input": (_OBJ, False), "deterministic_cfg": (_OBJ, True),
        "policy": (_OBJ, True)}
_NESTED = {"owner": _OWNER, "model": _MODEL, "deterministic_cfg": _DET, "policy": _POLICY}
_MINIMUM = {("deterministic_cfg", "n_ctx"): 256, ("deterministic_cfg", "n_batch"): 1,
            ("deterministic_cfg", "max_tokens"): 1}
_MIN_LEN = {("owner", "org_id"): 1, ("model", "model_id"): 1, ("", "backend_id"): 1}
_NEEDS_PATH = ("korith_local", "korith_cuda")
_NEEDS_ENDPOINT = ("openai_compatible", "vllm", "vllm_openai")


def _type_ok(v: Any, types) -> bool:
    if types is _INT:  # JSON integers only (a bool is not an integer here)
        return isinstance(v, int) and not isinstance(v, bool)
    if types is _NUM:
        return isinstance(v, (int, float)) and not isinstance(v, bool)
    return isinstance(v, types)


def _check_object(obj: Dict[str, Any], table, where: str, errs: List[str]) -> None:
    for k in obj:
        if k not in table:
            errs.append(f"{where}{k}: not allowed")
    for k, (types, required) in table.items():
        if k not in obj:
            if required:
                errs.append(f"{where}{k}: required")
            continue
        v = obj[k]
        if not _type_ok(v, types):
            errs.append(f"{where}{k}: wrong type {type(v).__name__}")
            continue
        scope = where.rstrip(".")
        lo = _MINIMUM.get((scope, k))
        if lo is not None and v < lo:
            errs.append(f"{where}{k}: below {lo}")
        ml = _MIN_LEN.get((scope, k))
        if ml is not None and len(v) < ml:
            errs.append(f"{where}{k}: empty")


def validate(spec: Any) -> List[str]:
    """Violations of the v1 contract (empty list: the spec is valid)."""
    if not isinstance(spec, dict):
        return ["jobspec: must be a JSON object"]
    errs: List[str] = []
    _check_object(spec, _TOP, "", errs)
    if "schema_version" in spec and spec["schema_version"] != SCHEMA_VERSION:
        errs.append(f"schema_version: must be {SCHEMA_VERSION}")
    for k, table in _NESTED.items():
        if isinstance(spec.get(k), dict):
            _check_object(spec[k], table, k + ".", errs)
    has_p, has_t = "prompt" in spec, "prompt_template" in spec
    if has_p == has_t:
        errs.append("prompt / prompt_template: exactly one is required")
    model = spec.get("model") if isinstance(spec.get("model"), dict) else {}
    backend = spec.get("backend_id")
    if backend in _NEEDS_PATH and not model.get("model_path"):
        errs.append(f"model.model_path: required for backend {backend}")
    if backend in _NEEDS_ENDPOINT and not model.get("endpoint"):
        errs.append(f"model.endpoint: required for backend {backend}")
    return errs


def render_prompt(spec: Dict[str, Any]) -> str:
    """The prompt text: ``prompt``, or ``prompt_template`` with ``input`` filled into its
    ``{field}`` slots (a template that does not format is used as written)."""
    if "prompt" in spec:
        return str(spec["prompt"])
    tmpl = str(spec.get("prompt_template", ""))
    try:
        return tmpl.format(**(spec.get("input") or {}))
    except (KeyError, IndexError, ValueError):
        return tmpl


def to_job(spec: Dict[str, Any]) -> Dict[str, Any]:
    """A valid v1 spec as the control plane's job dict."""
    det = spec["deterministic_cfg"]
    job: Dict[str, Any] = {
        "prompt": render_prompt(spec),
        "backend_id": spec["backend_id"],
        "model": dict(spec["model"]),
        "max_tokens": int(det.get("max_tokens", 64)),
        "deterministic": {k: det[k] for k in ("seed", "temperature", "top_p", "top_k", "n_ctx", "n_batch")
                          if k in det},
        "policy": dict(spec["policy"]),
        "schema_version": SCHEMA_VERSION,
    }
    job["deterministic"].setdefault("temperature", 0.0)
    for k in ("job_id", "parent_job_id", "session_id", "idempotency_key"):
        if k in spec:
            job[k] = spec[k]
    owner = spec.get("owner") or {}
    if owner.get("org_id"):
        job["org_id"] = owner["org_id"]
    return job
