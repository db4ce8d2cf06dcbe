"""Disk tier: AMFK snapshots in the AMF store directory (the checkpoint tier).

The native :class:`AmfStore` owns ``amf_index.bin`` and the ``.kv``/``.tok`` files
(admission, eviction, TTL, prewarm, checksums); this module turns a prefix's KV
pages into an AMFK blob and back (reference: core/amf_direct_kv.cu:158-460,
korith_vllm_ext/amf_kv_manager.py:262-535). Blobs are bf16 (dtype tag 2), K and V of
each layer as ``[n_pages, H, 16, D]``, which the reference's readers accept.
"""
from __future__ import annotations

import logging
import time
from typing import Optional, Sequence, Tuple

import numpy as np
import torch

from .._native_loader import native
from .formats import AMFK_HEADER, DTYPE_BF16, AmfkHeader, decode_amfk_header, encode_amfk_header
from .keys import AmfContext, amf_hash_tokens

log = logging.getLogger(__name__)


def pages_to_amfk(pages: torch.Tensor, n_tokens: int, model_hash: int, prefix_hash: int) -> bytes:
    """dense pages [n, L, 2, H, 16, D] bf16 -> AMFK blob bytes."""
    n, L, _, H, P, D = pages.shape
    payload = pages.permute(1, 2, 0, 3, 4, 5).contiguous().cpu()
    blob = n * H * P * D * 2
    layers = [(2 * l * blob, blob, (2 * l + 1) * blob, blob) for l in range(L)]
    hdr = AmfkHeader(L, n_tokens, H, D, DTYPE_BF16, 2 * L * blob, model_hash, prefix_hash, layers=layers)
    return encode_amfk_header(hdr) + payload.view(torch.uint8).numpy().tobytes()


def amfk_to_pages(blob: bytes, page: int = 16) -> Tuple[AmfkHeader, torch.Tensor]:
    """AMFK blob -> (header, dense pages [n, L, 2, H, 16, D] bf16). Accepts per-layer
    K/V blobs of ``[n_pages, H, 16, D]`` (this framework, AmfKvManager) in f16/bf16/f32."""
    h = decode_amfk_header(blob)
    if h.dtype not in (0, 1, 2):
        raise ValueError(f"AMFK dtype {h.dtype} cannot be restored into a bf16 cache")
    elt = 4 if h.dtype == 1 else 2
    npdt = {0: np.float16, 1: np.float32, 2: np.uint16}[h.dtype]
    base = h.payload_offset
    per = h.layers[0][1] // elt if h.layers else 0
    n_pages = per // (h.n_kv_heads * page * h.head_dim) if per else 0
    out = torch.empty(n_pages, h.n_layers, 2, h.n_kv_heads, page, h.head_dim, dtype=torch.bfloat16)
    for l, (ko, kb, vo, vb) in enumerate(h.layers):
        for kv, (off, nb) in enumerate(((ko, kb), (vo, vb))):
            a = np.frombuffer(blob, dtype=npdt, count=nb // elt, offset=base + off)
            t = torch.from_numpy(a.copy())
            t = t.view(torch.bfloat16) if h.dtype == 2 else t.to(torch.bfloat16)
            out[:, l, kv] = t.view(n_pages, h.n_kv_heads, page, h.head_dim)
    return h, out


class DiskTier:
    def __init__(self, path: Optional[str] = None, ctx: Optional[AmfContext] = None, config: Optional[dict] = None,
                 from_env: bool = False):
        self.store = native().AmfStore()
        if from_env:
            self.enabled = self.store.init_from_env()
        else:
            self.enabled = self.store.init(path or "amf", config or {})
        self.ctx = ctx or AmfContext()

    def save(self, tokens: Sequence[int], pages: torch.Tensor, saved_ms: float = 0.0) -> bool:
        if not self.enabled:
            return False
        toks = np.asarray(tokens, dtype=np.int32)
        blob = pages_to_amfk(pages, len(toks), self.ctx.model_hash, amf_hash_tokens(toks))
        return bool(self.store.store_entry(self.ctx.as_dict(), toks, blob, int(saved_ms)))

    def lookup(self, tokens: Sequence[int]):
        """Longest stored prefix of ``tokens``: (reason, entry dict or None)."""
        if not self.enabled:
            return "load_failed", None
        return self.store.find_longest_prefix(self.ctx.as_dict(), np.asarray(tokens, dtype=np.int32))

    def load(self, entry: dict) -> Optional[Tuple[AmfkHeader, torch.Tensor]]:
        blob = self.store.load_kv(entry)
        if blob is None:
            self.store.note_failure(entry)
            return None
        try:
            return amfk_to_pages(blob)
        except ValueError as exc:
            log.warning("AMFK blob rejected: %s", exc)
            self.store.note_failure(entry)
            return None

    def note_hit(self, entry: dict, tokens_saved: int, restore_ms: float, saved_ms: float) -> None:
        self.store.note_hit(entry, int(tokens_saved), int(round(restore_ms)), int(round(saved_ms)))

    def stats(self) -> dict:
        return {"enabled": self.enabled, **(self.store.stats() if self.enabled else {})}
