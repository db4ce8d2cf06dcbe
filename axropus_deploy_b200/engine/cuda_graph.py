"""CUDA-graph replay of the decode step (replaces the reference's llama_decode graph
cache, core/cuda_graph_decode.cu:132-350).

One graph per batch-size bucket, captured lazily on first use. Inputs live in static
device buffers that are refreshed before each replay with one pinned host->device
copy (tokens, positions, slots, lengths) and one device gather of the block-table
rows. Padding rows get length 0 and slot -1, which every kernel treats as "no work".
The split-KV decode kernel is captured with the engine's maximum context, so its
grid is fixed; splits past a sequence's last page exit immediately.

The greedy token of every row (argmax) is part of the graph and lands in ``tok_out``;
:meth:`DecodeGraphRunner.run` then starts one asynchronous copy of the tokens and the
kernels' error flag into pinned memory. The next step may take its input tokens from
``tok_out`` on the device (``dev_tokens``), so the engine can launch step t + 1 before
it reads step t's tokens (decode pipelining). Host staging is double-buffered: a
buffer is written again only two launches later, after the engine has waited for the
earlier one.
"""
from __future__ import annotations

import bisect
from typing import Dict, List, Optional

import torch

from ..models.llama import AttnMeta
from ..ops.attention import CascadeMeta, DecodeWorkspace, cascade_num_splits, decode_num_splits

BUCKETS = [1, 2, 4, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256]


class DecodeGraphRunner:
    def __init__(self, engine, max_graphs: int = 16):
        self.eng = engine
        dev = engine.device
        self.max_b = engine.cfg.max_batch
        self.buckets = [b for b in BUCKETS if b < self.max_b] + [self.max_b]
        mb = engine.max_blocks_per_seq
        self.ints = torch.zeros(4, self.max_b, dtype=torch.int32, device=dev)  # tok, pos, slot, len
        self.hosts = [torch.zeros(4, self.max_b, dtype=torch.int32).pin_memory() for _ in range(2)]
        self.bt = torch.zeros(self.max_b, mb, dtype=torch.int32, device=dev)
        self.rows = torch.zeros(self.max_b, dtype=torch.long, device=dev)
        self.rows_hosts = [torch.zeros(self.max_b, dtype=torch.long).pin_memory() for _ in range(2)]
        self.tok_out = torch.zeros(self.max_b, dtype=torch.int32, device=dev)  # greedy tokens of the last replay
        self.tok_host = torch.zeros(2, self.max_b + 1, dtype=torch.int32).pin_memory()  # tokens + error flag
        self.gather = torch.zeros(self.max_b, dtype=torch.long, device=dev)
        self.gather_host = [torch.zeros(self.max_b, dtype=torch.long).pin_memory() for _ in range(2)]
        self.events = [torch.cuda.Event(), torch.cuda.Event()]
        self.flip = 0
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.outs: Dict[int, torch.Tensor] = {}
        self.ws = DecodeWorkspace()
        self.pool = None
        self.max_seq = engine.cfg.max_model_len
        self.splits: Dict[int, int] = {}
        self.kernels: Dict[int, int] = {}
        # shared-prefix decode: every graph carries the grouped pass; a step without groups
        # replays it with zero groups (its CTAs return at once)
        self.cascade = bool(getattr(engine, "_cascade_on", False))
        self.ng_max = max(1, self.max_b // 2)
        self.cints = torch.zeros(3, self.max_b, dtype=torch.int32, device=dev)  # q_index, row_of, page_start
        self.cgrp = torch.zeros(2, self.ng_max + 1, dtype=torch.int32, device=dev)  # cu_q, shared lengths
        self.cbt = torch.zeros(self.ng_max, mb, dtype=torch.int32, device=dev)
        self.chost = torch.zeros(3, self.max_b, dtype=torch.int32).pin_memory()
        self.cgrp_host = torch.zeros(2, self.ng_max + 1, dtype=torch.int32).pin_memory()
        self.cplan = ()  # identity of the plan in the cascade buffers
        self.csplits: Dict[int, int] = {}

    def _cascade(self, b: int):
        if not self.cascade:
            return None
        ng = max(1, b // 2)
        return CascadeMeta(q_index=self.cints[0, :b], cu_q=self.cgrp[0, :ng + 1], seq_lens=self.cgrp[1, :ng],
                           block_table=self.cbt[:ng], row_of=self.cints[1, :b], page_start=self.cints[2, :b],
                           max_q=b, num_splits=self.csplits[b])

    def _meta(self, b: int) -> AttnMeta:
        return AttnMeta(mode="decode", positions=self.ints[1, :b], slots=self.ints[2, :b], block_table=self.bt[:b],
                        seq_lens=self.ints[3, :b], max_seq_len=self.max_seq, num_splits=self.splits[b],
                        cascade=self._cascade(b))

    def _load_plan(self, plan, n: int) -> None:
        """Cascade buffers for this batch: the plan's groups, or none (row_of = -1)."""
        ident = (plan["serial"] if plan is not None else 0, n)
        if self.cplan == ident:
            return
        h, hg = self.chost, self.cgrp_host
        h.zero_()
        hg.zero_()
        h[1].fill_(-1)
        if plan is not None:
            R, ng = len(plan["q_index"]), len(plan["seq_lens"])
            h[0, :R] = torch.tensor(plan["q_index"], dtype=torch.int32)
            h[1, :n] = torch.tensor(plan["row_of"], dtype=torch.int32)
            h[2, :n] = torch.tensor(plan["page_start"], dtype=torch.int32)
            hg[0, :ng + 1] = torch.tensor(plan["cu_q"], dtype=torch.int32)
            hg[0, ng + 1:] = plan["cu_q"][-1]
            hg[1, :ng] = torch.tensor(plan["seq_lens"], dtype=torch.int32)
            rows = torch.tensor(plan["bt_rows"], dtype=torch.long, device=self.cbt.device)
            self.cbt[:ng] = self.eng.block_table.index_select(0, rows)
        self.cints.copy_(h, non_blocking=True)
        self.cgrp.copy_(hg, non_blocking=True)
        self.cplan = ident

    def _capture(self, b: int) -> None:
        eng = self.eng
        cache = eng.cache
        self.splits[b] = decode_num_splits(b, cache.num_kv_heads, (self.max_seq + 15) // 16, eng.device, cache.fmt)
        self.csplits[b] = cascade_num_splits(max(1, b // 6), cache.num_kv_heads, self.max_seq, eng.device)
        # pre-size the split scratch for the largest bucket so every graph shares it
        from ..ops import attention as att

        D, Hq = eng.model.cfg.head_dim, getattr(eng.model, "hq", eng.model.cfg.num_heads)
        self.ws.get(self.max_b, Hq, max(self.splits[b], 64), D, eng.device)
        if self.cascade:
            att._CASCADE_WS.get(self.max_b, Hq, 16, D, eng.device)
            self._load_plan(None, b)
        prev = att._WS
        att._WS = self.ws
        try:
            self.ints[3, :b] = 0
            self.ints[2, :b] = -1
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(2):  # warm-up outside the graph (allocator, lazy init)
                    eng.model.forward(self.ints[0, :b], self._meta(b), cache)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            from ..ops._ext import LAUNCHES

            n0 = LAUNCHES[0]
            with torch.cuda.graph(g, pool=self.pool):
                out = eng.model.forward(self.ints[0, :b], self._meta(b), cache)
                from ..ops.layers import argmax

                argmax(out, out=self.tok_out[:b])
            self.kernels[b] = LAUNCHES[0] - n0
            LAUNCHES[0] = n0
            if self.pool is None:
                self.pool = g.pool()
        finally:
            att._WS = prev
        self.graphs[b] = g
        self.outs[b] = out

    def run(self, reqs, toks: Optional[List[int]], pos: List[int], slots: List[int], lens: List[int],
            plan=None, dev_tokens: Optional[List[int]] = None):
        """Replays the bucket's graph for ``reqs``. Input tokens come from ``toks`` (host)
        or, with ``dev_tokens``, from rows of the previous replay's ``tok_out``. Returns
        (logits [n, vocab], pinned slot of the tokens + error flag, event after their copy)."""
        n = len(reqs)
        b = self.buckets[bisect.bisect_left(self.buckets, n)]
        if b not in self.graphs:
            self._capture(b)
        if self.cascade:
            self._load_plan(plan, n)
        slot = self.flip
        self.flip ^= 1
        h = self.hosts[slot]
        if toks is not None:
            h[0, :n] = torch.tensor(toks, dtype=torch.int32)
        h[1, :n] = torch.tensor(pos, dtype=torch.int32)
        h[2, :n] = torch.tensor(slots, dtype=torch.int32)
        h[3, :n] = torch.tensor(lens, dtype=torch.int32)
        if b > n:
            h[0, n:b] = 0
            h[1, n:b] = 0
            h[2, n:b] = -1
            h[3, n:b] = 0
        if dev_tokens is None:
            self.ints[:, :b].copy_(h[:, :b], non_blocking=True)
        else:
            self.ints[1:, :b].copy_(h[1:, :b], non_blocking=True)
            if dev_tokens == list(range(n)):
                self.ints[0, :n].copy_(self.tok_out[:n])
            else:
                gh = self.gather_host[slot]
                gh[:n] = torch.tensor(dev_tokens, dtype=torch.long)
                self.gather[:n].copy_(gh[:n], non_blocking=True)
                self.ints[0, :n].copy_(self.tok_out.index_select(0, self.gather[:n]))
            if b > n:
                self.ints[0, n:b].zero_()
        rh = self.rows_hosts[slot]
        rh[:n] = torch.tensor([r.row for r in reqs], dtype=torch.long)
        self.rows[:n].copy_(rh[:n], non_blocking=True)
        self.bt[:n] = self.eng.block_table.index_select(0, self.rows[:n])
        self.graphs[b].replay()
        from ..ops._ext import LAUNCHES
        from ..ops.gemm import error_flag

        LAUNCHES[0] += self.kernels[b]
        th = self.tok_host[slot]
        th[:n].copy_(self.tok_out[:n], non_blocking=True)
        th[n:n + 1].copy_(error_flag(self.eng.device)[:1], non_blocking=True)
        ev = self.events[slot]
        ev.record()
        return self.outs[b][:n], slot, ev

    def close(self) -> None:
        self.graphs.clear()
        self.outs.clear()
        self.pool = None


PREFILL_BUCKETS = [64, 128, 256, 512]


class PrefillGraphRunner:
    """CUDA-graph replay of a one-sequence prefill of at most 512 new tokens -- the step
    that decides the TTFT of an AMF hit (a short suffix over a restored prefix), where a
    ~300-kernel forward of small GEMMs is bound by the host launching it.

    One graph per (token bucket, context bucket): the new tokens are padded up to the
    bucket with slot -1 (no KV write, rows never read back), the attention grids are
    sized for the bucket's query rows and the context bucket's longest KV range (split-
    KV slices past the sequence's real length find no keys and mark their partials
    empty), and the real lengths reach the kernels through device tensors refreshed
    with one pinned copy before each replay. On CPU, :meth:`run` executes the same
    padded step eagerly, which is how the padding is tested without a GPU.
    """

    def __init__(self, engine, max_tokens: int = 512, max_graphs: int = 24):
        self.eng = engine
        dev = engine.device
        self.buckets = [b for b in PREFILL_BUCKETS if b <= max_tokens] or [PREFILL_BUCKETS[0]]
        self.max_t = self.buckets[-1]
        self.max_graphs = max_graphs
        self.on_gpu = dev.type == "cuda"
        self.ints = torch.zeros(3, self.max_t, dtype=torch.int32, device=dev)   # tok, pos, slot
        self.small = torch.zeros(4, dtype=torch.int32, device=dev)               # seq_len, 0, n, n-1
        pin = self.on_gpu
        self.host = torch.zeros(3, self.max_t, dtype=torch.int32, pin_memory=pin)
        self.small_host = torch.zeros(4, dtype=torch.int32, pin_memory=pin)
        self.bt = torch.zeros(1, engine.max_blocks_per_seq, dtype=torch.int32, device=dev)
        self.graphs: Dict[tuple, torch.cuda.CUDAGraph] = {}
        self.outs: Dict[tuple, torch.Tensor] = {}
        self.kernels: Dict[tuple, int] = {}
        self.pool = None
        self.ws = DecodeWorkspace()
        self.stat = {"replays": 0, "captures": 0, "eager": 0}

    def ctx_bucket(self, seq_len: int) -> int:
        c = 2048
        while c < seq_len:
            c *= 2
        return min(c, max(seq_len, self.eng.cfg.max_model_len))

    def supports(self, reqs, n_tokens: int, seq_len: int) -> bool:
        return len(reqs) == 1 and 0 < n_tokens <= self.max_t and seq_len <= self.eng.cfg.max_model_len and \
            all(r.params.temperature <= 0 for r in reqs)

    def _meta(self, tb: int, cb: int) -> AttnMeta:
        return AttnMeta(mode="prefill", positions=self.ints[1, :tb], slots=self.ints[2, :tb], block_table=self.bt,
                        seq_lens=self.small[0:1], cu_q=self.small[1:3], max_q=tb, max_seq_len=cb,
                        logits_idx=self.small[3:4])

    def _capture(self, key: tuple) -> None:
        from ..ops import attention as att
        from ..ops._ext import LAUNCHES

        tb, cb = key
        eng = self.eng
        cfg = eng.model.cfg
        hq = getattr(eng.model, "hq", cfg.num_heads)
        # split scratch sized once for the largest bucket, shared by every graph
        self.ws.get(self.max_t, hq, 32, cfg.head_dim, eng.device)
        prev = att._PREFILL_WS
        att._PREFILL_WS = self.ws
        try:
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                eng.model.forward(self.ints[0, :tb], self._meta(tb, cb), eng.cache)  # warm-up (lazy init)
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            n0 = LAUNCHES[0]
            with torch.cuda.graph(g, pool=self.pool):
                out = eng.model.forward(self.ints[0, :tb], self._meta(tb, cb), eng.cache)
            self.kernels[key] = LAUNCHES[0] - n0
            LAUNCHES[0] = n0
            if self.pool is None:
                self.pool = g.pool()
        finally:
            att._PREFILL_WS = prev
        self.graphs[key] = g
        self.outs[key] = out
        self.stat["captures"] += 1

    def run(self, r, toks: List[int], pos: List[int], slots: List[int], seq_len: int) -> torch.Tensor:
        n = len(toks)
        tb = self.buckets[bisect.bisect_left(self.buckets, n)]
        cb = self.ctx_bucket(seq_len)
        h = self.host
        h[0, :n] = torch.tensor(toks, dtype=torch.int32)
        h[1, :n] = torch.tensor(pos, dtype=torch.int32)
        h[2, :n] = torch.tensor(slots, dtype=torch.int32)
        if tb > n:
            h[0, n:tb] = 0
            h[1, n:tb] = pos[-1]
            h[2, n:tb] = -1
        self.small_host[0], self.small_host[1], self.small_host[2], self.small_host[3] = seq_len, 0, n, n - 1
        self.ints[:, :tb].copy_(h[:, :tb], non_blocking=True)
        self.small.copy_(self.small_host, non_blocking=True)
        self.bt.copy_(self.eng.block_table[r.row:r.row + 1])
        key = (tb, cb)
        if not self.on_gpu:
            self.stat["eager"] += 1
            return self.eng.model.forward(self.ints[0, :tb], self._meta(tb, cb), self.eng.cache)
        if key not in self.graphs:
            if len(self.graphs) >= self.max_graphs:
                self.stat["eager"] += 1
                return self.eng.model.forward(self.ints[0, :tb], self._meta(tb, cb), self.eng.cache)
            self._capture(key)
        self.graphs[key].replay()
        from ..ops._ext import LAUNCHES

        LAUNCHES[0] += self.kernels[key]
        self.stat["replays"] += 1
        return self.outs[key]

    def close(self) -> None:
        self.graphs.clear()
        self.outs.clear()
        self.pool = None
