"""Python side of the C ABI (``libkorith_b200.so``, ``csrc/capi/``).

The C entry points mirror the reference's two C surfaces -- the llama.cpp wrapper
``korith_init / korith_tokenize / korith_step / korith_shutdown``
(korith_c_api/korith.h:9-24) and the engine ABI ``korith_engine_*``
(platform/engine/cpp/korith_engine.h:12-43), whose reference implementation returns
fake timings -- and forward to one :class:`CSession` here: a single sequence on this
framework's model, paged KV cache and kernels, with real prefill, greedy decode,
logits, speculative verification, KV snapshots in the AMFK format and KV replay.

``model_path`` names a model preset (``llama3-8b``, ``tiny128``, ...; optionally
``preset:layers``) or a directory holding ``config.json`` with a ``preset`` field:
these boxes have no checkpoints, weights are random-initialised. Text is tokenised
byte-wise (one token per UTF-8 byte), like the reference server's fallback tokenizer.
"""
from __future__ import annotations

import json
import os
import time
from typing import List, Optional, Sequence

import numpy as np
import torch

from . import ops
from .models.config import get_config
from .models.llama import AttnMeta, LlamaModel
from .ops.kvcache import PAGE, KVCache

_SESSION: Optional["CSession"] = None


def _resolve_model(model_path: str):
    name, layers = model_path, None
    if os.path.isdir(model_path):
        with open(os.path.join(model_path, "config.json")) as f:
            c = json.load(f)
        name, layers = c.get("preset", "tiny128"), c.get("layers")
    elif ":" in model_path:
        name, n = model_path.rsplit(":", 1)
        layers = int(n)
    return get_config(name), layers


class CSession:
    def __init__(self, model_path: str, n_ctx: int, device: Optional[str] = None):
        cfg, layers = _resolve_model(model_path)
        dev = device or os.environ.get("AXR_DEVICE") or ("cuda" if torch.cuda.is_available() else "cpu")
        dtype = torch.bfloat16 if dev.startswith("cuda") else torch.float32
        self.model = LlamaModel(cfg, dev, dtype=dtype, seed=int(os.environ.get("AXR_SEED", "0")), layers=layers)
        self.model.ensure_positions(n_ctx + PAGE)
        self.dev = self.model.device
        self.n_ctx = n_ctx
        self.blocks = (n_ctx + PAGE - 1) // PAGE
        self.cache = KVCache(self.model.num_layers, self.blocks, cfg.num_kv_heads, cfg.head_dim, "bf16", self.dev)
        self.bt = torch.arange(self.blocks, dtype=torch.int32, device=self.dev)[None]
        self.tokens: List[int] = []
        self.logits: Optional[torch.Tensor] = None
        self.m = {"prefill_ms": 0.0, "decode_ms": 0.0, "total_ms": 0.0, "restore_ms": 0.0, "verify_ms": 0.0,
                  "draft_ms": 0.0, "tokens_out": 0, "accepted_tokens": 0, "rejected_tokens": 0}

    # ------------------------------------------------------------------ helpers
    def _sync(self):
        if self.dev.type == "cuda":
            torch.cuda.synchronize(self.dev)

    def _forward(self, toks: Sequence[int], start: int, all_logits: bool = False) -> torch.Tensor:
        n = len(toks)
        dev = self.dev
        pos = torch.arange(start, start + n, dtype=torch.int32, device=dev)
        idx = torch.arange(n, dtype=torch.int32, device=dev) if all_logits else \
            torch.tensor([n - 1], dtype=torch.int32, device=dev)
        meta = AttnMeta("prefill", pos, pos, self.bt, torch.tensor([start + n], dtype=torch.int32, device=dev),
                        cu_q=torch.tensor([0, n], dtype=torch.int32, device=dev), max_q=n, max_seq_len=start + n,
                        logits_idx=idx)
        return self.model.forward(torch.tensor(list(toks), dtype=torch.int32, device=dev), meta, self.cache)

    # ------------------------------------------------------------------ korith_*
    def tokenize(self, prompt: str) -> int:
        toks = list(prompt.encode("utf-8"))
        self.tokens = []
        return len(toks) if self.prefill(toks) else -1

    def prefill(self, toks: Sequence[int]) -> bool:
        toks = [int(t) for t in toks]
        if not toks or len(self.tokens) + len(toks) >= self.n_ctx:
            return False
        if any(t < 0 or t >= self.model.cfg.vocab for t in toks):
            return False
        t0 = time.perf_counter()
        self.logits = self._forward(toks, len(self.tokens))[0]
        self.tokens += toks
        self._sync()
        self.m["prefill_ms"] += (time.perf_counter() - t0) * 1e3
        self.m["total_ms"] += (time.perf_counter() - t0) * 1e3
        return True

    def step(self) -> int:
        """Greedy next token, appended and evaluated; -1 when the context is full."""
        if self.logits is None or len(self.tokens) + 1 >= self.n_ctx:
            return -1
        t0 = time.perf_counter()
        tok = int(ops.argmax(self.logits[None].float()).item())
        self.logits = self._forward([tok], len(self.tokens))[0]
        self.tokens.append(tok)
        self._sync()
        dt = (time.perf_counter() - t0) * 1e3
        self.m["decode_ms"] += dt
        self.m["total_ms"] += dt
        self.m["tokens_out"] += 1
        return tok

    def get_logits(self) -> Optional[np.ndarray]:
        return None if self.logits is None else self.logits.float().cpu().numpy()

    def verify(self, proposed: Sequence[int]) -> int:
        """Greedy verification of proposed continuation tokens (one forward, device
        verify kernel); the accepted prefix is appended to the sequence."""
        proposed = [int(t) for t in proposed]
        if self.logits is None or not proposed or len(self.tokens) + len(proposed) >= self.n_ctx:
            return 0
        t0 = time.perf_counter()
        start = len(self.tokens)
        # rows: logits after the current sequence, then after each proposed token
        rows = self._forward(proposed, start, all_logits=True)
        logits = torch.cat([self.logits[None].float(), rows.float()], 0)[None]  # [1, k+1, V]
        out = ops.spec_verify(logits, torch.tensor([proposed], dtype=torch.int32, device=logits.device)).tolist()[0]
        acc = int(out[0])
        self.tokens += proposed[:acc]
        self.logits = logits[0, acc].to(self.logits.dtype)
        self._sync()
        dt = (time.perf_counter() - t0) * 1e3
        self.m["verify_ms"] += dt
        self.m["total_ms"] += dt
        self.m["accepted_tokens"] += acc
        self.m["rejected_tokens"] += len(proposed) - acc
        return acc

    # ------------------------------------------------------------------ KV snapshots (AMFK)
    def _pages(self) -> torch.Tensor:
        n = len(self.tokens) // PAGE
        return self.cache.read_units(torch.arange(n, dtype=torch.int64)).to(torch.bfloat16)

    def export_snapshot(self, path: str) -> bool:
        from .amf.disk import pages_to_amfk
        from .amf.keys import amf_hash_tokens

        n = len(self.tokens) // PAGE * PAGE
        if n == 0:
            return False
        toks = self.tokens[:n]
        blob = pages_to_amfk(self._pages().cpu(), n, 0, amf_hash_tokens(toks))
        with open(path, "wb") as f:
            f.write(blob)
        np.asarray(toks, dtype=np.int32).tofile(path + ".tok")
        return True

    def apply_kv_replay(self, blob: bytes, tokens: Optional[Sequence[int]] = None) -> bool:
        """Write an AMFK blob's pages into the cache as the sequence's first pages."""
        from .amf.disk import amfk_to_pages

        t0 = time.perf_counter()
        hdr, pages = amfk_to_pages(blob)
        n = pages.shape[0]
        if n == 0 or n * PAGE >= self.n_ctx or pages.shape[1] != self.model.num_layers:
            return False
        self.cache.write_units(torch.arange(n, dtype=torch.int64), pages.to(self.dev))
        if tokens is None:
            # the blob carries K/V but not the token ids: the sequence now holds n pages
            # of context; the caller prefills what follows before stepping
            self.tokens = [0] * (n * PAGE)
            self.logits = None
        else:
            self.tokens = [int(t) for t in tokens][: n * PAGE]
            # logits of the last restored position: evaluate it again on top of the pages
            last = self.tokens[-1]
            self.tokens = self.tokens[:-1]
            self.logits = self._forward([last], len(self.tokens))[0]
            self.tokens.append(last)
        self._sync()
        self.m["restore_ms"] += (time.perf_counter() - t0) * 1e3
        return True

    def import_snapshot(self, path: str) -> bool:
        with open(path, "rb") as f:
            blob = f.read()
        toks = np.fromfile(path + ".tok", dtype=np.int32).tolist() if os.path.exists(path + ".tok") else None
        return self.apply_kv_replay(blob, toks)

    def metrics(self) -> dict:
        return dict(self.m)


# ---------------------------------------------------------------------- flat functions for C
def init(model_path: str, n_ctx: int) -> bool:
    global _SESSION
    _SESSION = CSession(model_path, int(n_ctx))
    return True


def session() -> CSession:
    if _SESSION is None:
        raise RuntimeError("korith: not initialised")
    return _SESSION


def shutdown() -> None:
    global _SESSION
    _SESSION = None
    if torch.cuda.is_available():
        torch.cuda.empty_cache()


def cuda_probe() -> bool:
    return bool(torch.cuda.is_available())
