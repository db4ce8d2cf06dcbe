"""Paged attention ops: split-KV decode and causal varlen prefill.

CUDA tensors run the sm_100a kernels; CPU tensors run the fp32 PyTorch oracle
(gather the sequence's pages, dequantise, softmax attention)."""
from __future__ import annotations

import math
import os
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch

from ._ext import cuda_ext
from .gemm import error_flag
from .kvcache import BF16, KVCache

# prefill of bf16 pages on the tcgen05 kernel (False: the warp-level mma.sync kernel)
PREFILL_TC = [True]
# new tokens per sequence up to which the tcgen05 prefill packs the query heads of a KV head
# into one tile's rows (AXR_PREFILL_GQA_PACK_MAX_Q; 0 turns packing off)
GQA_PACK_MAX_Q = [int(os.environ.get("AXR_PREFILL_GQA_PACK_MAX_Q", "2048"))]

_SMS = {}


def _num_sms(device: torch.device) -> int:
    idx = device.index or 0
    if idx not in _SMS:
        _SMS[idx] = torch.cuda.get_device_properties(idx).multi_processor_count
    return _SMS[idx]


def gather_seq_kv(cache: KVCache, layer: int, block_row: torch.Tensor, seq_len: int):
    """fp32 K, V of one sequence: [seq_len, H, D] each (oracle helper)."""
    n_pages = (seq_len + 15) // 16
    ids = block_row[:n_pages].long()
    u = cache.read_units(ids)[:, layer]  # [n, 2, H, P, D]
    k = u[:, 0].permute(0, 2, 1, 3).reshape(n_pages * 16, cache.num_kv_heads, cache.head_dim)[:seq_len]
    v = u[:, 1].permute(0, 2, 1, 3).reshape(n_pages * 16, cache.num_kv_heads, cache.head_dim)[:seq_len]
    return k, v


def _ref_attn(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, q_pos0: int, scale: float) -> torch.Tensor:
    """q [n, Hq, D], k/v [S, Hkv, D] fp32; causal with query i at absolute q_pos0 + i."""
    hq, hkv = q.shape[1], k.shape[1]
    g = hq // hkv
    k = k.repeat_interleave(g, dim=1)
    v = v.repeat_interleave(g, dim=1)
    s = torch.einsum("nhd,shd->hns", q.float(), k) * scale
    n, S = q.shape[0], k.shape[0]
    qpos = torch.arange(n, device=q.device)[:, None] + q_pos0
    kpos = torch.arange(S, device=q.device)[None, :]
    s = s.masked_fill(kpos > qpos, float("-inf"))
    p = torch.softmax(s, dim=-1)
    return torch.einsum("hns,shd->nhd", p, v)


class DecodeWorkspace:
    """Scratch for split-KV decode: partial outputs and log-sum-exps."""

    def __init__(self):
        self.o = None
        self.lse = None

    def get(self, B: int, Hq: int, S: int, D: int, device) -> tuple:
        need = B * Hq * S
        if self.o is None or self.lse.numel() < need or self.o.device != device:
            self.o = torch.empty(need * D, dtype=torch.float32, device=device)
            self.lse = torch.empty(need, dtype=torch.float32, device=device)
        return self.o, self.lse


_WS = DecodeWorkspace()
_CASCADE_WS = DecodeWorkspace()


@dataclass
class CascadeMeta:
    """Shared-prefix decode of one step: sequences whose block tables start with the same
    pages form a group; the group's queries attend to those shared pages once (one pass
    over them for every query of the group, on the tensor cores) and each sequence then
    attends only to its own pages, the two partial results merged by log-sum-exp.

    Device tensors (int32): ``q_index`` [R] decode rows of the groups' members, grouped;
    ``cu_q`` [NG+1] group offsets into q_index; ``seq_lens`` [NG] shared tokens per group;
    ``block_table`` [NG, max_blocks] the shared pages; ``row_of`` [B] packed row of each
    sequence in q_index (-1: in no group); ``page_start`` [B] first page of each sequence's
    own pass. ``max_q``: largest group (padded for CUDA graphs), ``num_splits``: KV slices
    of the shared pass."""

    q_index: torch.Tensor
    cu_q: torch.Tensor
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    row_of: torch.Tensor
    page_start: torch.Tensor
    max_q: int
    num_splits: int


def cascade_groups(block_lists: Sequence[Sequence[int]], min_pages: int = 32,
                   max_pages: Optional[Sequence[int]] = None) -> List[tuple]:
    """Groups of batch rows that share leading pages: [(rows, shared_pages), ...] with at
    least two rows and ``min_pages`` shared pages each. Rows are grouped by their first
    block; the shared length is the longest common prefix of the group's block lists,
    capped by ``max_pages[b]`` (a row's pages that hold prompt tokens), so that the pages
    a sequence is still writing stay in its own pass."""
    by_first = {}
    for i, bl in enumerate(block_lists):
        if len(bl) >= min_pages:
            by_first.setdefault(bl[0], []).append(i)
    groups = []
    for rows in by_first.values():
        if len(rows) < 2:
            continue
        n = min(len(block_lists[r]) if max_pages is None else min(len(block_lists[r]), max_pages[r]) for r in rows)
        first = block_lists[rows[0]]
        lcp = 0
        while lcp < n and all(block_lists[r][lcp] == first[lcp] for r in rows[1:]):
            lcp += 1
        if lcp >= min_pages:
            groups.append((rows, lcp))
    return groups


def cascade_num_splits(n_groups: int, kv_heads: int, max_seq_len: int, device: torch.device) -> int:
    """KV slices of the shared pass: enough CTAs (groups x KV heads x slices) for a wave of
    SMs, each slice keeping at least 4 KV tiles of 128 tokens."""
    ctas = max(1, n_groups) * kv_heads
    tiles = max(1, -(-max_seq_len // 128))
    return int(max(1, min(16, -(-_num_sms(device) // ctas), tiles // 4)))


def decode_num_splits(batch: int, kv_heads: int, max_pages: int, device: torch.device, fmt: int = -1) -> int:
    return int(cuda_ext().decode_num_splits(batch, kv_heads, max_pages, _num_sms(device), fmt))


def cascade_supported(cache: KVCache, head_dim: int) -> bool:
    """The shared pass runs on the tcgen05 prefill kernel: bf16 pages, head_dim 128."""
    return cache.fmt == BF16 and head_dim == 128 and PREFILL_TC[0]


def decode_attention(q: torch.Tensor, cache: KVCache, layer: int, block_table: torch.Tensor, seq_lens: torch.Tensor,
                     scale: Optional[float] = None, max_seq_len: Optional[int] = None,
                     num_splits: Optional[int] = None, out: Optional[torch.Tensor] = None,
                     workspace: Optional[DecodeWorkspace] = None,
                     cascade: Optional[CascadeMeta] = None) -> torch.Tensor:
    """q [B, Hq, D] (rotated) -> out [B, Hq, D]; attends to seq_lens[b] cached tokens.
    With ``cascade`` the shared prefixes of grouped sequences are attended once per group
    (same result; see :class:`CascadeMeta`)."""
    B, Hq, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    if q.is_cuda:
        if max_seq_len is None:
            max_seq_len = int(seq_lens.max().item()) if B else 0
        max_pages = (max_seq_len + 15) // 16
        S = num_splits if num_splits is not None else decode_num_splits(B, cache.num_kv_heads, max_pages, q.device, cache.fmt)
        ws = workspace or _WS
        po, pl = ws.get(B, Hq, S, D, q.device) if (S > 1 or cascade is not None) else (out, out)
        k, v, km, vm, bs, hs, mbs, mhs = cache.layer_args(layer)
        C = cuda_ext()
        if cascade is None:
            C.decode_attention(q, k, v, km, vm, bs, hs, mbs, mhs, cache.fmt, block_table, seq_lens,
                               cache.num_kv_heads, scale, S, max_pages, out, po, pl, None, None, None, None, 0)
            return out
        S2 = cascade.num_splits
        R = cascade.q_index.numel()
        po2, pl2 = _CASCADE_WS.get(max(R, 1), Hq, S2, D, q.device)
        C.prefill_attention_tc(q, k, v, bs, hs, cache.num_blocks, cascade.block_table, cascade.cu_q,
                               cascade.seq_lens, cache.num_kv_heads, scale, cascade.max_q, out, error_flag(q.device),
                               S2, po2, pl2, Hq // cache.num_kv_heads, 1, cascade.q_index, 1)
        C.decode_attention(q, k, v, km, vm, bs, hs, mbs, mhs, cache.fmt, block_table, seq_lens, cache.num_kv_heads,
                           scale, S, max_pages, out, po, pl, cascade.page_start, po2, pl2, cascade.row_of, S2)
        return out
    for b in range(B):
        n = int(seq_lens[b])
        k, v = gather_seq_kv(cache, layer, block_table[b], n)
        out[b] = _ref_attn(q[b:b + 1].float(), k, v, n - 1, scale)[0].to(out.dtype)
    return out


def prefill_num_splits(batch: int, heads: int, max_q: int, max_seq_len: Optional[int], device,
                       q_tile: int = 64, kv_tile: int = 64, per_sm: int = 2) -> int:
    """KV slices per query tile so that a short suffix over a long prefix still fills
    the GPU (``per_sm`` resident CTAs per SM); 1 when the query tiles alone do. Each
    slice keeps at least 4 KV tiles (2 for the 128-token tiles of the tensor-core kernel)."""
    if not max_seq_len:
        return 1
    ctas = max(1, -(-max_q // q_tile)) * heads * max(1, batch)
    target = per_sm * _num_sms(device)
    if ctas >= target:
        return 1
    kv_tiles = -(-max_seq_len // kv_tile)
    if kv_tile == 64:
        return int(max(1, min(-(-target // ctas), kv_tiles // 4, 32)))
    # one CTA per SM: pick the split count with the least estimated time, waves x (tiles
    # per slice + a per-CTA overhead of about two tiles)
    best, best_t = 1, None
    for s in range(1, max(1, min(32, kv_tiles // 2)) + 1):
        t = -(-ctas * s // target) * (-(-kv_tiles // s) + 2)
        if best_t is None or t < best_t:
            best, best_t = s, t
    return best


_PREFILL_WS = DecodeWorkspace()
_CASCADE_WS = DecodeWorkspace()


@dataclass
class CascadeMeta:
    """Shared-prefix decode of one step: sequences whose block tables start with the same
    pages form a group; the group's queries attend to those shared pages once (one pass
    over them for every query of the group, on the tensor cores) and each sequence then
    attends only to its own pages, the two partial results merged by log-sum-exp.

    Device tensors (int32): ``q_index`` [R] decode rows of the groups' members, grouped;
    ``cu_q`` [NG+1] group offsets into q_index; ``seq_lens`` [NG] shared tokens per group;
    ``block_table`` [NG, max_blocks] the shared pages; ``row_of`` [B] packed row of each
    sequence in q_index (-1: in no group); ``page_start`` [B] first page of each sequence's
    own pass. ``max_q``: largest group (padded for CUDA graphs), ``num_splits``: KV slices
    of the shared pass."""

    q_index: torch.Tensor
    cu_q: torch.Tensor
    seq_lens: torch.Tensor
    block_table: torch.Tensor
    row_of: torch.Tensor
    page_start: torch.Tensor
    max_q: int
    num_splits: int


def cascade_groups(block_lists: Sequence[Sequence[int]], min_pages: int = 32,
                   max_pages: Optional[Sequence[int]] = None) -> List[tuple]:
    """Groups of batch rows that share leading pages: [(rows, shared_pages), ...] with at
    least two rows and ``min_pages`` shared pages each. Rows are grouped by their first
    block; the shared length is the longest common prefix of the group's block lists,
    capped by ``max_pages[b]`` (a row's pages that hold prompt tokens), so that the pages
    a sequence is still writing stay in its own pass."""
    by_first = {}
    for i, bl in enumerate(block_lists):
        if len(bl) >= min_pages:
            by_first.setdefault(bl[0], []).append(i)
    groups = []
    for rows in by_first.values():
        if len(rows) < 2:
            continue
        n = min(len(block_lists[r]) if max_pages is None else min(len(block_lists[r]), max_pages[r]) for r in rows)
        first = block_lists[rows[0]]
        lcp = 0
        while lcp < n and all(block_lists[r][lcp] == first[lcp] for r in rows[1:]):
            lcp += 1
        if lcp >= min_pages:
            groups.append((rows, lcp))
    return groups


def cascade_num_splits(n_groups: int, kv_heads: int, max_seq_len: int, device: torch.device) -> int:
    """KV slices of the shared pass: enough CTAs (groups x KV heads x slices) for a wave of
    SMs, each slice keeping at least 4 KV tiles of 128 tokens."""
    ctas = max(1, n_groups) * kv_heads
    tiles = max(1, -(-max_seq_len // 128))
    return int(max(1, min(16, -(-_num_sms(device) // ctas), tiles // 4)))


def prefill_attention(q: torch.Tensor, cache: KVCache, layer: int, block_table: torch.Tensor, cu_q: torch.Tensor,
                      seq_lens: torch.Tensor, max_q: int, scale: Optional[float] = None,
                      out: Optional[torch.Tensor] = None, max_seq_len: Optional[int] = None,
                      num_splits: Optional[int] = None) -> torch.Tensor:
    """q [T, Hq, D] packed new tokens of B sequences (cu_q offsets); seq_lens = total
    cached length per sequence including the new tokens. With ``max_seq_len`` (the
    longest seq_lens entry) the KV range is split when the query tiles are too few."""
    T, Hq, D = q.shape
    scale = scale if scale is not None else 1.0 / math.sqrt(D)
    if out is None:
        out = torch.empty_like(q)
    if q.is_cuda:
        k, v, km, vm, bs, hs, mbs, mhs = cache.layer_args(layer)
        G = Hq // cache.num_kv_heads
        pack = G > 1 and max_q <= GQA_PACK_MAX_Q[0]
        if cache.fmt == BF16 and D == 128 and PREFILL_TC[0] and max_q * (G if pack else 1) >= 64:
            # tensor-core (tcgen05 / TMEM) kernel on bf16 pages: 256-row tiles, one CTA per
            # SM; up to GQA_PACK_MAX_Q new tokens the G query heads of a KV head share the
            # tiles (rows = token x head), and short suffixes over long prefixes split the KV range
            rows, heads = (max_q * G, cache.num_kv_heads) if pack else (max_q, Hq)
            S = num_splits if num_splits is not None else prefill_num_splits(
                seq_lens.shape[0], heads, rows, max_seq_len, q.device, q_tile=256, kv_tile=128, per_sm=1)
            po, pl = _PREFILL_WS.get(T, Hq, S, D, q.device) if S > 1 else (None, None)
            cuda_ext().prefill_attention_tc(q, k, v, bs, hs, cache.num_blocks, block_table, cu_q, seq_lens,
                                            cache.num_kv_heads, scale, max_q, out, error_flag(q.device), S, po, pl,
                                            G if pack else 1, 0, None, 0)
            return out
        S = num_splits if num_splits is not None else prefill_num_splits(seq_lens.shape[0], Hq, max_q, max_seq_len,
                                                                          q.device)
        po, pl = _PREFILL_WS.get(T, Hq, S, D, q.device) if S > 1 else (None, None)
        cuda_ext().prefill_attention(q, k, v, km, vm, bs, hs, mbs, mhs, cache.fmt, block_table, cu_q, seq_lens,
                                     cache.num_kv_heads, scale, max_q, out, S, po, pl)
        return out
    cu = cu_q.tolist()
    for b in range(len(cu) - 1):
        s0, s1 = cu[b], cu[b + 1]
        if s1 == s0:
            continue
        n = int(seq_lens[b])
        k, v = gather_seq_kv(cache, layer, block_table[b], n)
        out[s0:s1] = _ref_attn(q[s0:s1].float(), k, v, n - (s1 - s0), scale).to(out.dtype)
    return out
