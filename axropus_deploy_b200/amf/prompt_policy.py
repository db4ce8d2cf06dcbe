"""What part of a prompt the AMF tiers key on, and under which tenant.

Repeated prompts often differ in bytes that do not change their meaning (line endings,
trailing blanks, key order in a JSON tool schema) or share only a system part followed by
a user turn. Before lookup and capture the serving path therefore:

* canonicalises the text (:func:`canonicalize_prompt_text`): CRLF / CR to LF and trailing
  blanks of every line always; with ``KORITH_AMF_NORMALIZE_UNICODE`` Unicode NFC; with
  ``KORITH_AMF_NORMALIZE_WHITESPACE`` runs of spaces / tabs to one space; with
  ``KORITH_AMF_PROMPT_COLLAPSE_BLANKS`` three or more newlines to two; with
  ``KORITH_AMF_PROMPT_STRIP_OUTER`` leading / trailing whitespace removed;
* canonicalises template data (:func:`canonicalize_template_data`): with
  ``KORITH_AMF_CANONICALIZE_TEMPLATE_JSON`` dict / list values become compact JSON with
  sorted keys (``..._JSON_RECURSIVE`` also canonicalises the strings inside them,
  ``KORITH_AMF_CANONICALIZE_TEMPLATE_STRINGS`` the top-level strings);
* with ``KORITH_AMF_PREFIX_EXTRACTION`` keys on the tokens before the last occurrence of
  the boundary (``KORITH_AMF_PREFIX_BOUNDARY_TOKEN``, default ``<|user|>``) instead of the
  whole prompt (:func:`amf_prefix_tokens`), so every turn of a conversation with the same
  system part shares one entry;
* picks the tenant namespace (:func:`amf_tenant`): the hash of ``KORITH_TENANT_ID`` with
  ``KORITH_AMF_TENANT_ISOLATION``, else 0 (one namespace); prompts that start with one of
  ``KORITH_AMF_SHARED_PREFIX_PATTERNS`` (comma separated) go to the ``__shared__`` tenant
  when ``KORITH_AMF_SHARED_PREFIXES`` is on, whatever the caller's tenant.

Reference: platform/runtime/prompt_canonicalization.py:18-60 and core/engine.cpp:392-420,
:2475-2486, :2611-2636 (the variables and what each one changes).
"""
from __future__ import annotations

import json
import os
import re
import unicodedata
from typing import Any, Dict, List, Optional, Sequence

from .keys import amf_hash_tenant_id


def _on(name: str, default: bool = False) -> bool:
    v = os.environ.get(name)
    return default if v is None else v.strip().lower() in ("1", "true", "yes", "on")


def canonicalize_prompt_text(text: str) -> str:
    s = str(text or "").replace("\r\n", "\n").replace("\r", "\n")
    if _on("KORITH_AMF_NORMALIZE_UNICODE"):
        s = unicodedata.normalize("NFC", s)
    s = "\n".join(line.rstrip() for line in s.split("\n"))
    if _on("KORITH_AMF_NORMALIZE_WHITESPACE"):
        s = re.sub(r"[ \t]+", " ", s)
    if _on("KORITH_AMF_PROMPT_COLLAPSE_BLANKS"):
        s = re.sub(r"\n{3,}", "\n\n", s)
    if _on("KORITH_AMF_PROMPT_STRIP_OUTER"):
        s = s.strip()
    return s


def canonicalize_template_data(data: Dict[str, Any]) -> Dict[str, Any]:
    if not isinstance(data, dict):
        return {}
    strings = _on("KORITH_AMF_CANONICALIZE_TEMPLATE_STRINGS")
    as_json = _on("KORITH_AMF_CANONICALIZE_TEMPLATE_JSON")
    recursive = _on("KORITH_AMF_CANONICALIZE_TEMPLATE_JSON_RECURSIVE")

    def deep(v: Any) -> Any:
        if isinstance(v, str):
            return canonicalize_prompt_text(v)
        if isinstance(v, dict):
            return {str(k): deep(x) for k, x in v.items()}
        if isinstance(v, list):
            return [deep(x) for x in v]
        return v

    out: Dict[str, Any] = {}
    for k, v in data.items():
        if isinstance(v, str):
            out[str(k)] = canonicalize_prompt_text(v) if strings else v
        elif as_json and isinstance(v, (dict, list)):
            out[str(k)] = json.dumps(deep(v) if recursive else v, sort_keys=True, ensure_ascii=False,
                                     separators=(",", ":"))
        else:
            out[str(k)] = v
    return out


def _last_subsequence(hay: Sequence[int], needle: Sequence[int]) -> int:
    n, m = len(hay), len(needle)
    if m == 0 or m > n:
        return -1
    first = needle[0]
    for i in range(n - m, -1, -1):
        if hay[i] == first and list(hay[i:i + m]) == list(needle):
            return i
    return -1


def amf_prefix_tokens(tokens: Sequence[int], tokenize, boundary: Optional[str] = None) -> Optional[int]:
    """Number of leading tokens the AMF tiers key on, or None for "the whole prompt".
    ``tokenize`` maps text to token ids (the boundary is tokenised the same way)."""
    if not _on("KORITH_AMF_PREFIX_EXTRACTION"):
        return None
    b = boundary if boundary is not None else (os.environ.get("KORITH_AMF_PREFIX_BOUNDARY_TOKEN") or "<|user|>")
    at = _last_subsequence(tokens, tokenize(b))
    return at if at >= 0 else None


def amf_tenant(tenant_id: Optional[str], prompt_text: str = "") -> int:
    """Tenant hash of the AMF key namespace for this prompt."""
    if _on("KORITH_AMF_SHARED_PREFIXES"):
        pats = [p for p in (os.environ.get("KORITH_AMF_SHARED_PREFIX_PATTERNS") or "").split(",") if p]
        if any(prompt_text.startswith(p) for p in pats):
            return amf_hash_tenant_id("__shared__")
    if _on("KORITH_AMF_TENANT_ISOLATION"):
        t = (tenant_id or os.environ.get("KORITH_TENANT_ID") or "default").strip() or "default"
        return amf_hash_tenant_id(t)
    return 0


def prepare_prompt(text: str, tokenize, tenant_id: Optional[str] = None) -> Dict[str, Any]:
    """Canonical text, its tokens, the AMF prefix length (None: whole prompt) and tenant hash."""
    canon = canonicalize_prompt_text(text)
    toks: List[int] = list(tokenize(canon))
    return {"text": canon, "tokens": toks, "amf_prefix_len": amf_prefix_tokens(toks, tokenize),
            "tenant_hash": amf_tenant(tenant_id, canon)}
