"""AMF KV materialisation: keys, on-disk formats, the sharded G1 pool, lower tiers,
the tiered router and the engine-facing manager."""
from .disk import DiskTier, amfk_to_pages, pages_to_amfk
from .keys import (AmfContext, amf_float_bits, amf_hash_tenant_id, amf_hash_tokens, amf_prefix_hashes,
                   entry_basename, owner_of, parse_basename, pool_key)
from .lmcache import LMCacheAdapter
from .manager import AmfHit, AmfManager
from .pool import DenseStore, G1Pool, PoolHit, PoolSlab
from .router import CacheTier, LookupResult, MissReason, TieredCacheRouter, WritePolicy, compute_prefix_hash

__all__ = [n for n in dir() if not n.startswith("_")]
