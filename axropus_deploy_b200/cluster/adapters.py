"""Backend adapters: how a control-plane worker runs a job on some inference backend.

:class:`BackendAdapter` is the interface (fingerprint, capabilities, tokenize,
baseline / accelerated / speculative runs, draft, verify); :class:`Capabilities`
names what a backend supports. Three backends:

* :class:`EngineAdapter` (``axr_engine``) -- this framework's engine in the worker's
  process: the paged KV cache, the AMF tiers and the GPU kernels. ``run_baseline``
  prefills everything (no AMF lookup); ``run_accel`` restores the longest cached prefix
  (G1 pool, CPU tier, disk) and captures on a miss; ``run_speculative`` turns on the
  engine's draft + device-verify path with the policy's depth. A KV snapshot file (the
  AMFK format, e.g. fetched from another node) given as ``mf_snapshot_in`` is imported
  into the AMF tiers before the run; every accelerated run exports its prefix as a
  snapshot into the job's artifacts.
* :class:`CAbiAdapter` (``korith_capi``) -- the C ABI library (``libkorith_b200.so``)
  through :class:`~.engine_client.EngineClient`: one sequence, KV replay from
  snapshot files, logits, token verification.
* :class:`OpenAICompatibleAdapter` (``openai_compatible``) -- any server speaking
  ``POST /v1/completions`` (this framework's server among them), over HTTP;
  :class:`VllmOpenAIAdapter` (``vllm_openai``) adds vLLM's request extras (``vllm_xargs``,
  speculative tokens, ``kv_transfer_params`` pass-through).
* :class:`TransformersAdapter` (``hf_transformers``) -- a Hugging Face causal LM in process.

:class:`AdapterRegistry` builds adapters from a jobspec and caches them per
(backend, model).

Reference: platform/adapters/base.py:8-109 (interface, capability names),
platform/adapters/registry.py (cache per backend/model), korith_local.py,
openai_compatible.py, vllm_openai.py:388-425 (kv_transfer_params), transformers_local.py.
"""
from __future__ import annotations

import hashlib
import json
import time
import urllib.request
from dataclasses import dataclass
from pathlib import Path
from typing import Any, Dict, List, Optional


@dataclass(frozen=True)
class Capabilities:
    kv_replay: bool = False
    deterministic_seeding: bool = False
    streaming: bool = False
    batch_prefill: bool = False
    logits_access: bool = False
    verify_tokens: bool = False
    draft_supported: bool = False

    def as_dict(self) -> Dict[str, bool]:
        return {"KV_REPLAY": self.kv_replay, "DETERMINISTIC_SEEDING": self.deterministic_seeding,
                "STREAMING": self.streaming, "BATCH_PREFILL": self.batch_prefill,
                "LOGITS_ACCESS": self.logits_access, "VERIFY_TOKENS": self.verify_tokens,
                "DRAFT_SUPPORTED": self.draft_supported}


def byte_tokens(text: str) -> List[int]:
    return list(text.encode("utf-8"))


def detok(tokens: List[int]) -> str:
    return bytes(t & 0xFF for t in tokens).decode("utf-8", errors="replace")


class BackendAdapter:
    backend_id = "base"
    backend_version = "v0"

    def get_fingerprint(self) -> Dict[str, str]:
        raise NotImplementedError

    def get_capabilities(self) -> Capabilities:
        raise NotImplementedError

    def tokenize(self, prompt: str) -> int:
        raise NotImplementedError

    def run_baseline(self, prompt: str, max_tokens: int, deterministic_cfg: Dict, policy: Dict,
                     artifacts: Dict[str, Any], mf_snapshot_in: Optional[str]) -> Dict:
        raise NotImplementedError

    def run_accel(self, prompt: str, max_tokens: int, deterministic_cfg: Dict, policy: Dict,
                  artifacts: Dict[str, Any], mf_snapshot_in: Optional[str], engine_cfg: Optional[Dict] = None) -> Dict:
        return self.run_baseline(prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in)

    def run_speculative(self, prompt: str, max_tokens: int, deterministic_cfg: Dict, policy: Dict,
                        artifacts: Dict[str, Any], mf_snapshot_in: Optional[str], spec_cfg: Optional[Dict] = None,
                        engine_cfg: Optional[Dict] = None) -> Dict:
        return self.run_accel(prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, engine_cfg)

    def run_draft(self, prompt: str, deterministic_cfg: Dict, max_tokens: int, spec_cfg: Optional[Dict] = None) -> Dict:
        raise NotImplementedError

    def verify_tokens(self, prompt: str, draft_tokens: List[int], deterministic_cfg: Dict,
                      spec_cfg: Optional[Dict] = None) -> Dict:
        raise NotImplementedError


def _result(output: List[int], t0: float, ttft_ms: float, prefill_ms: float, amf: Dict[str, Any],
            spec: Optional[Dict[str, Any]] = None) -> Dict[str, Any]:
    total = (time.perf_counter() - t0) * 1e3
    return {"output_tokens": output, "output_text": detok(output), "tokens_out": len(output), "exit_code": 0,
            "perf": {"total_ms": total, "ttft_ms": ttft_ms, "prefill_ms": prefill_ms,
                     "decode_ms": max(0.0, total - ttft_ms),
                     "tok_s": len(output) / max(1e-9, (total - ttft_ms) / 1e3) if len(output) > 1 else 0.0},
            "amf": amf, "spec": spec or {}}


class EngineAdapter(BackendAdapter):
    """This framework's engine, in process. ``engine`` is an ``LLMEngine`` (with or
    without an ``AmfManager``); ``model_name`` only labels the fingerprint."""

    backend_id = "axr_engine"
    backend_version = "b200-v1"

    def __init__(self, engine, model_name: str = "", service=None):
        self.eng = engine
        self.model_name = model_name or engine.model.cfg.name
        self.cold_ms_per_token = 0.0  # measured on cold prefills, prices restored tokens
        # with an EngineService driving the engine from its own thread, concurrent jobs are
        # batched by the engine; every direct use of the engine then runs on that thread
        self.svc = service

    def _on_engine(self, fn, *args):
        if self.svc is None:
            return fn(*args)
        return self.svc.run_in_engine(lambda _eng: fn(*args)).result()

    def get_fingerprint(self) -> Dict[str, str]:
        c = self.eng.model.cfg
        shape = f"{c.name}:{c.num_layers}:{c.hidden}:{c.num_heads}:{c.num_kv_heads}:{c.head_dim}:{c.vocab}"
        return {"backend_id": self.backend_id, "backend_version": self.backend_version, "model": self.model_name,
                "model_hash": hashlib.sha256(shape.encode()).hexdigest()[:16], "tokenizer": "bytes-v1",
                "kv_layout": f"paged16:{self.eng.cache.fmt}"}

    def get_capabilities(self) -> Capabilities:
        return Capabilities(kv_replay=self.eng.amf is not None, deterministic_seeding=True, streaming=False,
                            batch_prefill=True, logits_access=True, verify_tokens=True, draft_supported=True)

    def tokenize(self, prompt: str) -> int:
        return len(byte_tokens(prompt))

    # ------------------------------------------------------------------ snapshots
    def import_snapshot(self, path: str) -> int:
        """Load an AMFK snapshot (``path`` + ``path.tok`` token ids) into the AMF tiers;
        returns the tokens made available."""
        return self._on_engine(self._import_snapshot, path)

    def _import_snapshot(self, path: str) -> int:
        import numpy as np
        import torch

        from ..amf.disk import amfk_to_pages
        from ..ops.kvcache import PAGE

        amf = self.eng.amf
        tok_path = Path(str(path) + ".tok")
        if amf is None or not Path(path).exists() or not tok_path.exists():
            return 0
        _, pages = amfk_to_pages(Path(path).read_bytes())
        toks = np.fromfile(tok_path, dtype=np.int32).astype(np.int64)
        n = min(pages.shape[0], len(toks) // PAGE)
        if n == 0 or pages.shape[1] != self.eng.model.num_layers or not self.eng.bm.can_allocate(n):
            return 0
        blocks = self.eng.bm.allocate(n)
        try:
            bt = torch.tensor(blocks, dtype=torch.int64)
            self.eng.cache.write_units(bt, pages[:n].to(self.eng.device))
            ok = amf.capture(toks[: n * PAGE], self.eng.cache, bt.to(torch.int32))
        finally:
            self.eng.bm.release(blocks)
        return n * PAGE if ok else 0

    def export_snapshot(self, tokens: List[int], path: str) -> int:
        """Write the cached KV of ``tokens``' longest AMF-held prefix as an AMFK file."""
        return self._on_engine(self._export_snapshot, tokens, path)

    def _export_snapshot(self, tokens: List[int], path: str) -> int:
        import numpy as np
        import torch

        from ..amf.disk import pages_to_amfk
        from ..amf.keys import amf_hash_tokens

        amf = self.eng.amf
        if amf is None:
            return 0
        hit = amf.lookup(np.asarray(tokens, dtype=np.int64))
        if hit is None:
            return 0
        n = hit.n_pages
        if not self.eng.bm.can_allocate(n):
            hit.release()
            return 0
        blocks = self.eng.bm.allocate(n)
        try:
            hit.restore(self.eng.cache, torch.tensor(blocks, dtype=torch.int32))
            pages = self.eng.cache.read_units(torch.tensor(blocks, dtype=torch.int64)).to(torch.bfloat16).cpu()
        finally:
            hit.release()
            self.eng.bm.release(blocks)
        toks = list(tokens[: hit.n_tokens])
        Path(path).write_bytes(pages_to_amfk(pages, len(toks), 0, amf_hash_tokens(toks)))
        np.asarray(toks, dtype=np.int32).tofile(str(path) + ".tok")
        return len(toks)

    # ------------------------------------------------------------------ runs
    def _run(self, prompt: str, max_tokens: int, det: Dict, use_amf: bool, spec_depth: int = 0,
             prefix_len: Optional[int] = None) -> Dict:
        from ..engine.engine import SamplingParams

        eng = self.eng
        toks = byte_tokens(prompt)
        sp = SamplingParams(max_tokens=max_tokens, temperature=float(det.get("temperature", 0.0)),
                            seed=det.get("seed"))
        before = None
        t0 = time.perf_counter()
        if self.svc is not None:
            # shared, batching engine: the engine's own speculative setting applies
            r = self.svc.submit(toks, sp, amf_prefix_len=prefix_len if use_amf else 0).result()
        else:
            saved_spec = eng.spec
            if spec_depth <= 0:
                eng.spec = None
            elif eng.spec is not None:
                eng.spec.depth = max(1, min(int(spec_depth), eng.spec.max_depth))
                before = dict(eng.spec.stat)
            try:
                r = eng.add_request(toks, sp, amf_prefix_len=prefix_len if use_amf else 0)
                while not r.output or r.state != "finished":
                    eng.step()
            finally:
                eng.spec = saved_spec
        ttft = (r.t_first_token - t0) * 1e3 if r.t_first_token else 0.0
        computed = len(toks) - r.restored_tokens - r.local_cached_tokens
        if r.amf_tier == "cold" and computed > 0:
            rate = ttft / computed
            self.cold_ms_per_token = rate if self.cold_ms_per_token == 0 else 0.8 * self.cold_ms_per_token + 0.2 * rate
        reused = r.restored_tokens + r.local_cached_tokens
        saved = max(0.0, reused * self.cold_ms_per_token - r.restore_ms)
        amf = {"decision": "hit" if r.amf_tier != "cold" else "miss", "tier": r.amf_tier,
               "restored_tokens": r.restored_tokens, "restore_ms": r.restore_ms, "saved_ms": saved,
               "local_cached_tokens": r.local_cached_tokens}
        if eng.amf is not None:
            sts = [p.stats() for p in eng.amf.pools]
            amf["cache_entries"] = sum(int(st.get("num_prefixes", 0)) for st in sts)
            amf["cache_bytes"] = sum(int(st.get("used_bytes", 0)) for st in sts)
        spec = {}
        if before is not None:
            spec = {k: eng.spec.stat[k] - before.get(k, 0) for k in ("steps", "drafted", "accepted", "emitted")}
            spec["acceptance"] = spec["accepted"] / spec["drafted"] if spec["drafted"] else 0.0
        return _result(list(r.output), t0, ttft, ttft, amf, spec)

    def run_baseline(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in):
        return self._run(prompt, max_tokens, deterministic_cfg or {}, use_amf=False)

    def run_accel(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, engine_cfg=None):
        imported = self.import_snapshot(mf_snapshot_in) if mf_snapshot_in else 0
        plen = (engine_cfg or {}).get("amf_prefix_len")
        out = self._run(prompt, max_tokens, deterministic_cfg or {}, use_amf=True, prefix_len=plen)
        out["amf"]["snapshot_imported_tokens"] = imported
        snap = (artifacts or {}).get("snapshot")
        # a prefix this run computed itself becomes a snapshot other nodes can fetch
        if snap and out["amf"]["tier"] == "cold" and (policy or {}).get("export_snapshot", True):
            toks = byte_tokens(prompt)
            out["snapshot_tokens"] = self.export_snapshot(toks[:plen] if plen else toks, str(snap))
            out["snapshot_path"] = str(snap) if out["snapshot_tokens"] else ""
        return out

    def run_speculative(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, spec_cfg=None,
                        engine_cfg=None):
        if self.eng.spec is None:
            return self.run_accel(prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, engine_cfg)
        if mf_snapshot_in:
            self.import_snapshot(mf_snapshot_in)
        k = int((spec_cfg or {}).get("k", 4))
        return self._run(prompt, max_tokens, deterministic_cfg or {}, use_amf=True, spec_depth=k,
                         prefix_len=(engine_cfg or {}).get("amf_prefix_len"))

    def run_draft(self, prompt, deterministic_cfg, max_tokens, spec_cfg=None):
        from ..engine.spec import NgramDrafter

        toks = byte_tokens(prompt)
        return {"draft_tokens": NgramDrafter().propose(toks, int(max_tokens))}

    def verify_tokens(self, prompt, draft_tokens, deterministic_cfg, spec_cfg=None):
        """Greedy verification: the longest prefix of ``draft_tokens`` the model itself
        would produce after ``prompt`` (one forward over prompt + draft)."""
        return self._on_engine(self._verify_tokens, prompt, draft_tokens)

    def _verify_tokens(self, prompt, draft_tokens):
        import torch

        from .. import ops
        from ..models.llama import AttnMeta
        from ..ops.kvcache import PAGE

        eng = self.eng
        toks = byte_tokens(prompt) + [int(t) for t in draft_tokens]
        n = len(toks)
        need = (n + PAGE - 1) // PAGE
        blocks = eng.bm.allocate(need)
        try:
            dev = eng.device
            bt = torch.tensor(blocks, dtype=torch.int32, device=dev)[None]
            pos = torch.arange(n, dtype=torch.int32, device=dev)
            slots = (bt[0].long()[pos.long() // PAGE] * PAGE + pos.long() % PAGE).to(torch.int32)
            k = len(draft_tokens)
            idx = torch.arange(n - k - 1, n, dtype=torch.int32, device=dev)
            meta = AttnMeta("prefill", pos, slots, bt, torch.tensor([n], dtype=torch.int32, device=dev),
                            cu_q=torch.tensor([0, n], dtype=torch.int32, device=dev), max_q=n, max_seq_len=n,
                            logits_idx=idx)
            logits = eng.model.forward(torch.tensor(toks, dtype=torch.int32, device=dev), meta, eng.cache)
            out = ops.spec_verify(logits[None].float(), torch.tensor([list(draft_tokens)], dtype=torch.int32,
                                                                       device=dev)).tolist()[0]
        finally:
            eng.bm.release(blocks)
        acc = int(out[0])
        return {"accepted": acc, "accepted_tokens": list(draft_tokens[:acc]), "next_token": int(out[1 + acc])
                if len(out) > 1 + acc else None}


class CAbiAdapter(BackendAdapter):
    """The C ABI library through ctypes (one sequence per adapter)."""

    backend_id = "korith_capi"
    backend_version = "capi-v1"

    def __init__(self, model_path: str, n_ctx: int = 4096, lib_path: Optional[str] = None):
        from .engine_client import EngineClient

        self.model_path = model_path
        self.n_ctx = n_ctx
        self.client = EngineClient(lib_path)
        if not self.client.init_model(model_path, n_ctx):
            raise RuntimeError(f"korith_engine_init_model failed: {self.client.last_error()}")

    def get_fingerprint(self) -> Dict[str, str]:
        return {"backend_id": self.backend_id, "backend_version": self.backend_version, "model": self.model_path,
                "model_hash": hashlib.sha256(self.model_path.encode()).hexdigest()[:16], "tokenizer": "bytes-v1",
                "kv_layout": "amfk-bf16"}

    def get_capabilities(self) -> Capabilities:
        return Capabilities(kv_replay=True, deterministic_seeding=True, logits_access=True, verify_tokens=True)

    def tokenize(self, prompt: str) -> int:
        return len(byte_tokens(prompt))

    def _reset(self) -> None:
        if not self.client.init_model(self.model_path, self.n_ctx):
            raise RuntimeError(self.client.last_error())

    def run_baseline(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in):
        self._reset()
        t0 = time.perf_counter()
        toks = byte_tokens(prompt)
        restored = 0
        if mf_snapshot_in and Path(mf_snapshot_in).exists() and self.client.import_snapshot(mf_snapshot_in):
            restored = self.client.metrics().get("restore_ms", 0.0) and len(toks) // 16 * 16
        if not self.client.prefill(toks):
            raise RuntimeError(self.client.last_error())
        ttft = (time.perf_counter() - t0) * 1e3
        out = []
        for _ in range(max(0, max_tokens - 1)):
            t = self.client.decode_step()
            if t is None:
                break
            out.append(t)
        snap = (artifacts or {}).get("snapshot")
        if snap:
            self.client.export_snapshot(str(snap))
        m = self.client.metrics()
        return _result(out, t0, ttft, m.get("prefill_ms", ttft),
                       {"decision": "hit" if restored else "miss", "tier": "snapshot" if restored else "cold",
                        "restored_tokens": restored, "restore_ms": m.get("restore_ms", 0.0), "saved_ms": 0.0})

    def verify_tokens(self, prompt, draft_tokens, deterministic_cfg, spec_cfg=None):
        self._reset()
        self.client.prefill(byte_tokens(prompt))
        return {"accepted": self.client.verify(list(draft_tokens))}


class OpenAICompatibleAdapter(BackendAdapter):
    """``POST {endpoint}/v1/completions`` with ``prompt``, ``max_tokens``, ``temperature``,
    ``seed`` (and ``amf_prefix_len`` = 0 for baseline runs, which this framework's
    server honours)."""

    backend_id = "openai_compatible"
    backend_version = "http-v1"

    def __init__(self, endpoint: str, model_id: str = "", api_key: str = "", timeout_s: float = 120.0):
        self.endpoint = endpoint.rstrip("/")
        self.model_id = model_id
        self.api_key = api_key
        self.timeout_s = timeout_s

    def get_fingerprint(self) -> Dict[str, str]:
        return {"backend_id": self.backend_id, "backend_version": self.backend_version, "model": self.model_id,
                "model_hash": hashlib.sha256(f"{self.endpoint}|{self.model_id}".encode()).hexdigest()[:16],
                "tokenizer": "remote", "kv_layout": "remote"}

    def get_capabilities(self) -> Capabilities:
        return Capabilities(deterministic_seeding=True, batch_prefill=True)

    def tokenize(self, prompt: str) -> int:
        return len(byte_tokens(prompt))

    def _post(self, body: Dict[str, Any]) -> Dict[str, Any]:
        req = urllib.request.Request(self.endpoint + "/v1/completions", data=json.dumps(body).encode(),
                                     method="POST", headers={"Content-Type": "application/json"})
        if self.api_key:
            req.add_header("Authorization", f"Bearer {self.api_key}")
        with urllib.request.urlopen(req, timeout=self.timeout_s) as resp:
            return json.loads(resp.read())

    def _run(self, prompt, max_tokens, det, use_amf: bool) -> Dict:
        t0 = time.perf_counter()
        body = {"model": self.model_id, "prompt": prompt, "max_tokens": int(max_tokens),
                "temperature": float((det or {}).get("temperature", 0.0)), "seed": (det or {}).get("seed")}
        if not use_amf:
            body["amf_prefix_len"] = 0
        r = self._post(body)
        ax = r.get("axropus", {})
        toks = r.get("token_ids") or byte_tokens(r["choices"][0]["text"])
        ttft = float(ax.get("ttft_ms", 0.0))
        return _result(list(toks), t0, ttft, ttft, {"decision": "hit" if ax.get("hit") else "miss",
                                                    "tier": ax.get("tier", "remote"),
                                                    "restored_tokens": ax.get("restored_tokens", 0), "saved_ms": 0.0})

    def run_baseline(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in):
        return self._run(prompt, max_tokens, deterministic_cfg, use_amf=False)

    def run_accel(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, engine_cfg=None):
        return self._run(prompt, max_tokens, deterministic_cfg, use_amf=True)


class VllmOpenAIAdapter(OpenAICompatibleAdapter):
    """A vLLM OpenAI server. On top of the plain completion call: the job's lane and policy
    travel as ``vllm_xargs`` (``KORITH_VLLM_*`` admission hints read by a decode-first
    scheduler), a speculative run asks for ``num_speculative_tokens`` (and a draft model when
    the policy names one), and ``kv_transfer_params`` returned by a KV connector are kept in
    the result so a later request can hand them back."""

    backend_id = "vllm_openai"
    backend_version = "vllm-openai-v1"

    @staticmethod
    def _xargs(policy: Dict[str, Any], lane: str) -> Dict[str, Any]:
        x: Dict[str, Any] = {"korith_lane": lane or "MISS"}
        for k in ("priority", "replay_state", "tenant_id"):
            v = (policy or {}).get(k)
            if isinstance(v, (str, int, float)) and not isinstance(v, bool):
                x[f"korith_{k}"] = v
        return x

    def _body(self, prompt, max_tokens, det, policy, use_amf: bool, spec_k: int = 0) -> Dict[str, Any]:
        body = {"model": self.model_id, "prompt": prompt, "max_tokens": int(max_tokens),
                "temperature": float((det or {}).get("temperature", 0.0)), "seed": (det or {}).get("seed"),
                "vllm_xargs": self._xargs(policy, (policy or {}).get("lane", ""))}
        if not use_amf:
            body["amf_prefix_len"] = 0
        if (policy or {}).get("kv_transfer_params"):
            body["kv_transfer_params"] = policy["kv_transfer_params"]
        if spec_k > 0:
            body["num_speculative_tokens"] = int(spec_k)
            if (policy or {}).get("draft_model"):
                body["speculative_model"] = policy["draft_model"]
        return body

    def _run_v(self, prompt, max_tokens, det, policy, use_amf: bool, spec_k: int = 0) -> Dict:
        t0 = time.perf_counter()
        r = self._post(self._body(prompt, max_tokens, det, policy, use_amf, spec_k))
        ax = r.get("axropus", {})
        text = (r.get("choices") or [{}])[0].get("text", "")
        toks = r.get("token_ids") or byte_tokens(text)
        ttft = float(ax.get("ttft_ms", 0.0))
        out = _result(list(toks), t0, ttft, ttft, {"decision": "hit" if ax.get("hit") else "miss",
                                                   "tier": ax.get("tier", "remote"),
                                                   "restored_tokens": ax.get("restored_tokens", 0), "saved_ms": 0.0})
        kvp = r.get("kv_transfer_params") or (r.get("usage") or {}).get("kv_transfer_params")
        if kvp:
            out["kv_transfer_params"] = kvp
        usage = r.get("usage") or {}
        acc, prop = usage.get("accepted_speculative_tokens"), usage.get("proposed_speculative_tokens")
        if spec_k > 0 and acc is not None and prop:
            out["spec"] = {"drafted": int(prop), "accepted": int(acc), "acceptance": int(acc) / int(prop)}
        return out

    def get_capabilities(self) -> Capabilities:
        return Capabilities(deterministic_seeding=True, batch_prefill=True, kv_replay=True, draft_supported=True)

    def run_baseline(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in):
        return self._run_v(prompt, max_tokens, deterministic_cfg, policy, use_amf=False)

    def run_accel(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, engine_cfg=None):
        return self._run_v(prompt, max_tokens, deterministic_cfg, policy, use_amf=True)

    def run_speculative(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in, spec_cfg=None,
                        engine_cfg=None):
        return self._run_v(prompt, max_tokens, deterministic_cfg, policy, use_amf=True,
                           spec_k=int((spec_cfg or {}).get("k", 4)))


class TransformersAdapter(BackendAdapter):
    """A Hugging Face ``transformers`` causal LM in this process (``model_path`` of a local
    checkpoint, or ``config`` -- a dict for ``LlamaConfig`` -- for a random-init model).
    Baseline runs only: the KV cache lives inside ``generate`` and is not replayed; logits
    and token verification are exposed. Text is tokenised byte-wise, as elsewhere here."""

    backend_id = "hf_transformers"
    backend_version = "transformers"

    def __init__(self, model_path: str = "", config: Optional[Dict[str, Any]] = None, device: str = "cpu",
                 seed: int = 0):
        import torch
        import transformers

        if model_path:
            self.model = transformers.AutoModelForCausalLM.from_pretrained(model_path)
        else:
            torch.manual_seed(seed)
            cfg = transformers.LlamaConfig(**(config or {"vocab_size": 256, "hidden_size": 64, "intermediate_size": 128,
                                                         "num_hidden_layers": 2, "num_attention_heads": 4,
                                                         "num_key_value_heads": 2}))
            self.model = transformers.LlamaForCausalLM(cfg)
        self.model = self.model.to(device).eval()
        self.device = device
        self.name = model_path or "random-llama"
        self.backend_version = f"transformers-{transformers.__version__}"

    def get_fingerprint(self) -> Dict[str, str]:
        c = self.model.config
        shape = f"{c.model_type}:{c.num_hidden_layers}:{c.hidden_size}:{c.vocab_size}"
        return {"backend_id": self.backend_id, "backend_version": self.backend_version, "model": self.name,
                "model_hash": hashlib.sha256(shape.encode()).hexdigest()[:16], "tokenizer": "bytes-v1",
                "kv_layout": "hf-dynamic"}

    def get_capabilities(self) -> Capabilities:
        return Capabilities(deterministic_seeding=True, logits_access=True, verify_tokens=True)

    def tokenize(self, prompt: str) -> int:
        return len(byte_tokens(prompt))

    def _ids(self, toks):
        import torch

        v = self.model.config.vocab_size
        return torch.tensor([[t % v for t in toks]], device=self.device)

    def run_baseline(self, prompt, max_tokens, deterministic_cfg, policy, artifacts, mf_snapshot_in):
        import torch

        t0 = time.perf_counter()
        ids = self._ids(byte_tokens(prompt))
        with torch.no_grad():
            first = self.model(ids).logits[0, -1].argmax().item()
            ttft = (time.perf_counter() - t0) * 1e3
            out = self.model.generate(ids, max_new_tokens=int(max_tokens), do_sample=False,
                                      pad_token_id=0)[0, ids.shape[1]:].tolist()
        if out and out[0] != first:
            out = [first] + out[1:]
        return _result(out, t0, ttft, ttft, {"decision": "miss", "tier": "cold", "restored_tokens": 0, "saved_ms": 0.0})

    def verify_tokens(self, prompt, draft_tokens, deterministic_cfg, spec_cfg=None):
        import torch

        toks = byte_tokens(prompt)
        ids = self._ids(toks + list(draft_tokens))
        with torch.no_grad():
            pred = self.model(ids).logits[0, len(toks) - 1:-1].argmax(-1).tolist()
        acc = 0
        for p, d in zip(pred, draft_tokens):
            if p != d % self.model.config.vocab_size:
                break
            acc += 1
        return {"accepted": acc, "accepted_tokens": list(draft_tokens[:acc])}


class AdapterRegistry:
    """Adapters by jobspec ``backend_id`` + ``model``; one instance per (backend, model)."""

    def __init__(self, engine=None, service=None):
        self.engine = engine  # the worker's in-process engine, for axr_engine jobs
        self.service = service  # optional EngineService driving that engine (batched jobs)
        self._cache: Dict[tuple, BackendAdapter] = {}

    def get_adapter(self, jobspec: Dict[str, Any]) -> BackendAdapter:
        bid = jobspec.get("backend_id", "axr_engine")
        model = jobspec.get("model") or {}
        key = (bid, str(model.get("model_path", "")), str(model.get("endpoint", "")), str(model.get("model_id", "")))
        a = self._cache.get(key)
        if a is not None:
            return a
        if bid == "axr_engine":
            if self.engine is None:
                raise ValueError("axr_engine jobs need a worker with an engine")
            a = EngineAdapter(self.engine, str(model.get("model_id", "")), self.service)
        elif bid == "korith_capi":
            a = CAbiAdapter(str(model["model_path"]), int(model.get("n_ctx", 4096)))
        elif bid == "openai_compatible":
            a = OpenAICompatibleAdapter(str(model["endpoint"]), str(model.get("model_id", "")),
                                        str(model.get("api_key", "")))
        elif bid in ("vllm", "vllm_openai"):
            a = VllmOpenAIAdapter(str(model["endpoint"]), str(model.get("model_id", "")), str(model.get("api_key", "")))
        elif bid == "hf_transformers":
            a = TransformersAdapter(str(model.get("model_path", "")), model.get("config"),
                                    str(model.get("device", "cpu")))
        else:
            raise ValueError(f"unknown backend_id {bid!r}")
        self._cache[key] = a
        return a
