"""vLLM v1 KV connector over this framework's AMF prefix keys: a hot GPU tier for vLLM.

For deployments that keep vLLM as the serving engine: point ``vllm serve
--kv-transfer-config`` at ``{"kv_connector": "AMFKVConnector",
"kv_connector_module_path": "axropus_deploy_b200.amf.vllm_connector",
"kv_role": "kv_both", "kv_connector_extra_config": {"pool_gb": 8, "min_prefix_tokens": 64}}``
(the connector name of the reference, so existing configurations change one module path).

* Scheduler side. ``get_num_new_matched_tokens`` finds the longest block-aligned prefix of
  the prompt held by the store -- entries are whole prompts under :func:`~.keys.pool_key`
  (the G1 key of this framework), every block indexed by the chained hash of the tokens up to
  it, so a shared system prompt matches whatever follows it -- leaving at least one token to
  compute, and reports it as loadable synchronously; ``update_state_after_alloc`` records
  the blocks vLLM gave those tokens;
  ``build_connector_meta`` hands the step's loads to the workers together with the saves:
  every new request whose whole block-aligned prompt prefix is computed in this step and is
  not held yet.
* Worker side. ``register_kv_caches`` takes vLLM's per-layer paged caches (the
  ``[2, num_blocks, block_size, kv_heads, head_dim]`` layout of the flash-attention backends,
  or ``[num_blocks, 2, ...]``); ``start_load_kv`` copies a held prefix into the allocated
  blocks of every layer before the forward; ``save_kv_layer`` copies a finished prefix out of
  each layer as the forward goes, and ``wait_for_save`` commits the entries. Copies are
  gather / scatter of whole blocks on the GPU, no host round trip.
* Store. One process-wide store of whole-prefix entries in device memory, bounded by
  ``pool_gb``, least recently used out first. Scheduler and workers share it, so the
  connector serves vLLM's single-process executor (one GPU per engine, the data-parallel
  deployment of this framework); a tensor-parallel vLLM engine runs its workers in other
  processes and should use this framework's own engine instead.

Reference: korith_vllm_ext/amf_kv_connector.py:128 (the connector this replaces; its
configuration keys ``num_layers`` / ``default_format`` are accepted and ignored).
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Tuple

import numpy as np
import torch

from .keys import pool_key

try:  # vLLM is optional: the store and key logic work without it
    from vllm.distributed.kv_transfer.kv_connector.v1.base import (KVConnectorBase_V1, KVConnectorMetadata,
                                                                   KVConnectorRole)
except Exception:  # pragma: no cover - vLLM absent
    KVConnectorBase_V1 = object

    class KVConnectorMetadata:  # type: ignore[no-redef]
        pass

    KVConnectorRole = None


class PrefixStore:
    """Whole-prompt KV entries in device memory, LRU within a byte budget, found by their
    longest block-aligned common prefix: every block of a stored prompt is indexed by the
    chained hash of the tokens up to it, so a prompt that shares only its first blocks with a
    stored one (same system prompt, new question) still loads those blocks."""

    def __init__(self, capacity_bytes: int):
        self.capacity = int(capacity_bytes)
        self.entries: "OrderedDict[str, Tuple[int, Dict[str, torch.Tensor], List[bytes]]]" = OrderedDict()
        self.index: Dict[bytes, Tuple[str, int]] = {}  # chained block hash -> (entry key, blocks up to it)
        self.used = 0
        self.mu = threading.Lock()
        self.stat = {"hits": 0, "misses": 0, "saves": 0, "evictions": 0, "loaded_tokens": 0}

    @staticmethod
    def _nbytes(layers: Dict[str, torch.Tensor]) -> int:
        return sum(t.numel() * t.element_size() for t in layers.values())

    @staticmethod
    def hashes(tokens: List[int], n_blocks: int) -> List[bytes]:
        from ..engine.block_manager import block_hashes

        return list(block_hashes(np.asarray(tokens, dtype=np.int64), n_blocks))

    def longest(self, tokens: List[int], limit: int, block: int) -> Tuple[int, Optional[str]]:
        hs = self.hashes(tokens, limit // block)
        with self.mu:
            for i in range(len(hs) - 1, -1, -1):
                hit = self.index.get(hs[i])
                if hit is not None and hit[0] in self.entries:
                    self.entries.move_to_end(hit[0])
                    self.stat["hits"] += 1
                    return (i + 1) * block, hit[0]
            self.stat["misses"] += 1
            return 0, None

    def get(self, key: str) -> Optional[Tuple[int, Dict[str, torch.Tensor]]]:
        with self.mu:
            e = self.entries.get(key)
            return None if e is None else (e[0], e[1])

    def contains(self, key: str) -> bool:
        with self.mu:
            return key in self.entries

    def _drop_locked(self, key: str) -> None:
        n, layers, hs = self.entries.pop(key)
        self.used -= self._nbytes(layers)
        for h in hs:
            if self.index.get(h, (None,))[0] == key:
                del self.index[h]

    def put(self, key: str, n_tokens: int, layers: Dict[str, torch.Tensor], hashes: List[bytes]) -> bool:
        size = self._nbytes(layers)
        with self.mu:
            if key in self.entries or size > self.capacity:
                return False
            while self.entries and self.used + size > self.capacity:
                self._drop_locked(next(iter(self.entries)))
                self.stat["evictions"] += 1
            self.entries[key] = (n_tokens, layers, list(hashes))
            self.used += size
            for i, h in enumerate(hashes):
                self.index.setdefault(h, (key, i + 1))
            self.stat["saves"] += 1
            return True


_STORES: Dict[Tuple[str, int], PrefixStore] = {}


def shared_store(engine_id: str, capacity_bytes: int) -> PrefixStore:
    """The store both roles of one vLLM engine use (created by whichever comes first)."""
    k = (engine_id, capacity_bytes)
    if k not in _STORES:
        _STORES[k] = PrefixStore(capacity_bytes)
    return _STORES[k]


@dataclass
class _Load:
    req_id: str
    key: str
    first_block: int          # first block of the prefix that vLLM does not hold yet
    block_ids: List[int]      # vLLM blocks for prefix blocks [first_block, first_block + len)


@dataclass
class _Save:
    req_id: str
    key: str
    n_tokens: int
    block_ids: List[int]      # vLLM blocks of prefix blocks [0, n_tokens / block_size)
    hashes: List[bytes]       # chained hash of each of those blocks


@dataclass
class AmfConnectorMetadata(KVConnectorMetadata):
    loads: List[_Load] = field(default_factory=list)
    saves: List[_Save] = field(default_factory=list)


def _block_dim(t: torch.Tensor) -> int:
    """Which dimension of a vLLM paged cache indexes blocks: 1 for [2, blocks, ...], 0 for
    [blocks, 2, ...]."""
    return 1 if t.shape[0] == 2 else 0


class AmfB200Connector(KVConnectorBase_V1):
    def __init__(self, vllm_config, role, kv_cache_config=None):
        super().__init__(vllm_config, role, kv_cache_config)
        extra = dict(getattr(vllm_config.kv_transfer_config, "kv_connector_extra_config", None) or {})
        self.block_size = int(getattr(getattr(vllm_config, "cache_config", None), "block_size", 16) or 16)
        self.min_tokens = int(extra.get("min_prefix_tokens", 64))
        cap = int(float(extra.get("pool_gb", 8)) * (1 << 30))
        eid = str(getattr(vllm_config.kv_transfer_config, "engine_id", "") or "default")
        self.store = shared_store(eid, cap)
        self.kv_caches: Dict[str, torch.Tensor] = {}
        self._loads: Dict[str, _Load] = {}   # scheduler: allocated, not yet sent to the workers
        self._pending: Dict[str, Tuple[int, Dict[str, torch.Tensor], List[bytes]]] = {}  # worker: saves in flight

    # ------------------------------------------------------------------ scheduler side
    def _limit(self, n_prompt: int) -> int:
        return max(0, (n_prompt - 1) // self.block_size * self.block_size)  # keep >= 1 token to compute

    def get_num_new_matched_tokens(self, request, num_computed_tokens: int) -> Tuple[Optional[int], bool]:
        toks = list(request.prompt_token_ids)
        n, key = self.store.longest(toks, self._limit(len(toks)), self.block_size)
        if key is None or n <= num_computed_tokens or n < self.min_tokens:
            return 0, False
        request._amf_key = (key, n)
        return n - num_computed_tokens, False

    def update_state_after_alloc(self, request, blocks, num_external_tokens: int):
        if num_external_tokens <= 0 or not hasattr(request, "_amf_key"):
            return
        key, n = request._amf_key
        ids = list(blocks.get_block_ids()[0])
        first = (n - num_external_tokens) // self.block_size
        self._loads[request.request_id] = _Load(request.request_id, key, first, ids[first:n // self.block_size])

    def build_connector_meta(self, scheduler_output) -> AmfConnectorMetadata:
        meta = AmfConnectorMetadata(loads=list(self._loads.values()))
        self._loads.clear()
        for nr in scheduler_output.scheduled_new_reqs:
            toks = list(nr.prompt_token_ids or [])
            n = self._limit(len(toks))
            done = nr.num_computed_tokens + scheduler_output.num_scheduled_tokens.get(nr.req_id, 0)
            if n < self.min_tokens or done < n:
                continue
            key = pool_key(toks[:n])
            if self.store.contains(key):
                continue
            ids = list(nr.block_ids[0])[: n // self.block_size]
            meta.saves.append(_Save(nr.req_id, key, n, ids, self.store.hashes(toks, n // self.block_size)))
        return meta

    def request_finished(self, request, block_ids):
        return False, None

    # ------------------------------------------------------------------ worker side
    def register_kv_caches(self, kv_caches: Dict[str, torch.Tensor]):
        self.kv_caches = dict(kv_caches)

    def _meta(self) -> Optional[AmfConnectorMetadata]:
        try:
            m = self._get_connector_metadata()
        except Exception:
            return None
        return m if isinstance(m, AmfConnectorMetadata) else None

    def start_load_kv(self, forward_context, **kwargs) -> None:
        meta = self._meta()
        if meta is None:
            return
        for ld in meta.loads:
            got = self.store.get(ld.key)
            if got is None or not ld.block_ids:
                continue
            _, layers = got
            for name, kv in self.kv_caches.items():
                src = layers.get(name)
                if src is None:
                    continue
                d = _block_dim(kv)
                idx = torch.as_tensor(ld.block_ids, dtype=torch.long, device=kv.device)
                part = src.narrow(d, ld.first_block, len(ld.block_ids))
                kv.index_copy_(d, idx, part.to(kv.dtype))
            self.store.stat["loaded_tokens"] += len(ld.block_ids) * self.block_size

    def wait_for_layer_load(self, layer_name: str) -> None:
        return None  # loads are issued in start_load_kv on the forward's stream

    def save_kv_layer(self, layer_name: str, kv_layer: torch.Tensor, attn_metadata, **kwargs) -> None:
        meta = self._meta()
        if meta is None:
            return
        for sv in meta.saves:
            d = _block_dim(kv_layer)
            idx = torch.as_tensor(sv.block_ids, dtype=torch.long, device=kv_layer.device)
            entry = self._pending.setdefault(sv.key, (sv.n_tokens, {}, sv.hashes))
            entry[1][layer_name] = kv_layer.index_select(d, idx)

    def wait_for_save(self):
        for key, (n, layers, hashes) in self._pending.items():
            if not self.kv_caches or len(layers) == len(self.kv_caches):
                self.store.put(key, n, layers, hashes)
        self._pending.clear()


# the connector name of the reference, so existing --kv-transfer-config files keep working
AMFKVConnector = AmfB200Connector
