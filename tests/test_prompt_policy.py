"""KORITH_AMF_* prompt policy: canonical text, prefix extraction at the last boundary,
tenant namespaces and shared-prefix patterns, template JSON canonicalisation."""
from axropus_deploy_b200.amf.keys import amf_hash_tenant_id
from axropus_deploy_b200.amf.prompt_policy import (amf_prefix_tokens, amf_tenant, canonicalize_prompt_text,
                                                   canonicalize_template_data, prepare_prompt)


def _bt(s):
    return list(s.encode("utf-8"))


def test_canonical_text(monkeypatch):
    assert canonicalize_prompt_text("a  \r\nb\t\r\n\n\n\nc ") == "a\nb\n\n\n\nc"
    monkeypatch.setenv("KORITH_AMF_PROMPT_COLLAPSE_BLANKS", "1")
    monkeypatch.setenv("KORITH_AMF_PROMPT_STRIP_OUTER", "1")
    monkeypatch.setenv("KORITH_AMF_NORMALIZE_WHITESPACE", "1")
    monkeypatch.setenv("KORITH_AMF_NORMALIZE_UNICODE", "1")
    assert canonicalize_prompt_text("  x \t y\n\n\n\nz  ") == "x y\n\nz"
    assert canonicalize_prompt_text("é") == "é"


def test_prefix_extraction_and_tenants(monkeypatch):
    text = "<|system|>rules<|user|>first question<|assistant|>answer<|user|>second"
    assert amf_prefix_tokens(_bt(text), _bt) is None  # off by default: the whole prompt
    monkeypatch.setenv("KORITH_AMF_PREFIX_EXTRACTION", "1")
    n = amf_prefix_tokens(_bt(text), _bt)
    assert bytes(_bt(text)[:n]).decode() == "<|system|>rules<|user|>first question<|assistant|>answer"
    assert amf_prefix_tokens(_bt("no boundary"), _bt) is None
    assert amf_tenant("acme", "hello") == 0  # one namespace unless isolation is on
    monkeypatch.setenv("KORITH_AMF_TENANT_ISOLATION", "1")
    assert amf_tenant("acme", "hello") == amf_hash_tenant_id("acme")
    monkeypatch.setenv("KORITH_AMF_SHARED_PREFIXES", "1")
    monkeypatch.setenv("KORITH_AMF_SHARED_PREFIX_PATTERNS", "<|system|>rules,SYS:")
    assert amf_tenant("acme", text) == amf_hash_tenant_id("__shared__")
    p = prepare_prompt(text + "  \r\n", _bt, "acme")
    assert p["text"] == text + "\n" and p["amf_prefix_len"] == n and p["tenant_hash"] == amf_hash_tenant_id("__shared__")


def test_template_json(monkeypatch):
    data = {"tools": {"b": 1, "a": [2, {"d": "x  ", "c": 3}]}, "name": "n  "}
    assert canonicalize_template_data(data)["tools"] == data["tools"]  # off by default
    monkeypatch.setenv("KORITH_AMF_CANONICALIZE_TEMPLATE_JSON", "1")
    out = canonicalize_template_data(data)
    assert out["tools"] == '{"a":[2,{"c":3,"d":"x  "}],"b":1}' and out["name"] == "n  "
    monkeypatch.setenv("KORITH_AMF_CANONICALIZE_TEMPLATE_JSON_RECURSIVE", "1")
    monkeypatch.setenv("KORITH_AMF_CANONICALIZE_TEMPLATE_STRINGS", "1")
    out = canonicalize_template_data(data)
    assert out["tools"] == '{"a":[2,{"c":3,"d":"x"}],"b":1}' and out["name"] == "n"
