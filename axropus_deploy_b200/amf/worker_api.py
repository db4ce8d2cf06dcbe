"""Worker API: ``amf_save_kv`` / ``amf_restore_kv``.

The reference documents these as the methods of a vLLM worker extension
(README.md:85, :207-212) that never shipped; the behaviour it describes is that of
``AmfKvManager.save_kv_state(prompt_tokens, block_table)`` and
``restore_kv_state(prompt_tokens, block_table) -> n_tokens``
(korith_vllm_ext/amf_kv_manager.py:262-535): save the KV blocks of a prompt under
its AMF key (VRAM snapshot tier + disk AMFK), and restore them into physical blocks,
returning the number of restored tokens (0 on a miss). An empty ``block_table``
on save means "the whole cache" in the reference; here it means "the blocks the
engine holds for this prompt in its prefix cache".

These methods run on the engine's worker (same process as the KV cache); the
``call`` dispatcher lets a driver invoke them by name, like a collective RPC.
"""
from __future__ import annotations

import time
from typing import Any, List, Optional, Sequence

import numpy as np
import torch

from ..ops.kvcache import PAGE


class AmfWorkerExtension:
    def __init__(self, engine):
        self.engine = engine
        self.stats = {"saves": 0, "save_failures": 0, "hits": 0, "misses": 0, "restore_ms": 0.0}

    def _blocks_for(self, tokens: np.ndarray) -> List[int]:
        from ..engine.block_manager import block_hashes

        eng = self.engine
        hs = block_hashes(tokens, len(tokens) // PAGE)
        blocks = [eng.bm.by_hash.get(h) for h in hs]
        out = []
        for b in blocks:
            if b is None:
                break
            out.append(b)
        return out

    def amf_save_kv(self, prompt_tokens: Sequence[int], block_table: Optional[Sequence[int]] = None,
                    savings_ms: float = 0.0) -> bool:
        eng = self.engine
        if eng.amf is None:
            return False
        toks = np.asarray(prompt_tokens, dtype=np.int64).astype(np.int32)
        blocks = list(block_table) if block_table else self._blocks_for(toks)
        n = min(len(blocks), len(toks) // PAGE)
        if n * PAGE < eng.amf.min_tokens:
            self.stats["save_failures"] += 1
            return False
        ok = eng.amf.capture(toks[: n * PAGE], eng.cache, torch.tensor(blocks[:n], dtype=torch.int32),
                             savings_ms=savings_ms)
        self.stats["saves" if ok else "save_failures"] += 1
        return ok

    def amf_restore_kv(self, prompt_tokens: Sequence[int], block_table: Sequence[int]) -> int:
        eng = self.engine
        if eng.amf is None or not block_table:
            return 0
        toks = np.asarray(prompt_tokens, dtype=np.int64).astype(np.int32)
        t0 = time.perf_counter()
        hit = eng.amf.lookup(toks, min(len(toks), len(block_table) * PAGE))
        if hit is None:
            self.stats["misses"] += 1
            return 0
        try:
            n = hit.restore(eng.cache, torch.tensor(list(block_table)[: hit.n_pages], dtype=torch.int32))
            if eng.device.type == "cuda":
                torch.cuda.current_stream().synchronize()
        finally:
            hit.release()
        ms = (time.perf_counter() - t0) * 1e3
        self.stats["hits"] += 1
        self.stats["restore_ms"] += ms
        eng.amf.note_restored(hit, ms, 0.0)
        return n * PAGE

    def call(self, method: str, *args: Any, **kwargs: Any) -> Any:
        """Dispatch by name (``collective_rpc``-style)."""
        if method not in ("amf_save_kv", "amf_restore_kv"):
            raise AttributeError(method)
        return getattr(self, method)(*args, **kwargs)
