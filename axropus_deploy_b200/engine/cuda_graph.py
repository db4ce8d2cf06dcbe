"""CUDA-graph replay of the decode step (replaces the reference's llama_decode graph
cache, core/cuda_graph_decode.cu:132-350).

One graph per batch-size bucket, captured lazily on first use. Inputs live in static
device buffers that are refreshed before each replay with one pinned host->device
copy (tokens, positions, slots, lengths) and one device gather of the block-table
rows. Padding rows get length 0 and slot -1, which every kernel treats as "no work".
The split-KV decode kernel is captured with the engine's maximum context, so its
grid is fixed; splits past a sequence's last page exit immediately.
"""
from __future__ import annotations

import bisect
from typing import Dict, List

import torch

from ..models.llama import AttnMeta
from ..ops.attention import DecodeWorkspace, decode_num_splits

BUCKETS = [1, 2, 4, 8, 12, 16, 24, 32, 48, 64, 96, 128, 192, 256]


class DecodeGraphRunner:
    def __init__(self, engine, max_graphs: int = 16):
        self.eng = engine
        dev = engine.device
        self.max_b = engine.cfg.max_batch
        self.buckets = [b for b in BUCKETS if b < self.max_b] + [self.max_b]
        mb = engine.max_blocks_per_seq
        self.ints = torch.zeros(4, self.max_b, dtype=torch.int32, device=dev)  # tok, pos, slot, len
        self.host = torch.zeros(4, self.max_b, dtype=torch.int32).pin_memory()
        self.bt = torch.zeros(self.max_b, mb, dtype=torch.int32, device=dev)
        self.rows = torch.zeros(self.max_b, dtype=torch.long, device=dev)
        self.rows_host = torch.zeros(self.max_b, dtype=torch.long).pin_memory()
        self.graphs: Dict[int, torch.cuda.CUDAGraph] = {}
        self.outs: Dict[int, torch.Tensor] = {}
        self.ws = DecodeWorkspace()
        self.pool = None
        self.max_seq = engine.cfg.max_model_len
        self.splits: Dict[int, int] = {}
        self.kernels: Dict[int, int] = {}

    def _meta(self, b: int) -> AttnMeta:
        return AttnMeta(mode="decode", positions=self.ints[1, :b], slots=self.ints[2, :b], block_table=self.bt[:b],
                        seq_lens=self.ints[3, :b], max_seq_len=self.max_seq, num_splits=self.splits[b])

    def _capture(self, b: int) -> None:
        eng = self.eng
        cache = eng.cache
        self.splits[b] = decode_num_splits(b, cache.num_kv_heads, (self.max_seq + 15) // 16, eng.device, cache.fmt)
        # pre-size the split scratch for the largest bucket so every graph shares it
        from ..ops import attention as att

        D, Hq = eng.model.cfg.head_dim, getattr(eng.model, "hq", eng.model.cfg.num_heads)
        self.ws.get(self.max_b, Hq, max(self.splits[b], 64), D, eng.device)
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
            self.kernels[b] = LAUNCHES[0] - n0
            LAUNCHES[0] = n0
            if self.pool is None:
                self.pool = g.pool()
        finally:
            att._WS = prev
        self.graphs[b] = g
        self.outs[b] = out

    def run(self, reqs, toks: List[int], pos: List[int], slots: List[int], lens: List[int]) -> torch.Tensor:
        n = len(reqs)
        b = self.buckets[bisect.bisect_left(self.buckets, n)]
        if b not in self.graphs:
            self._capture(b)
        h = self.host
        h[0, :n] = torch.tensor(toks, dtype=torch.int32)
        h[1, :n] = torch.tensor(pos, dtype=torch.int32)
        h[2, :n] = torch.tensor(slots, dtype=torch.int32)
        h[3, :n] = torch.tensor(lens, dtype=torch.int32)
        if b > n:
            h[0, n:b] = 0
            h[1, n:b] = 0
            h[2, n:b] = -1
            h[3, n:b] = 0
        self.ints[:, :b].copy_(h[:, :b], non_blocking=True)
        self.rows_host[:n] = torch.tensor([r.row for r in reqs], dtype=torch.long)
        self.rows[:n].copy_(self.rows_host[:n], non_blocking=True)
        self.bt[:n] = self.eng.block_table.index_select(0, self.rows[:n])
        self.graphs[b].replay()
        from ..ops._ext import LAUNCHES

        LAUNCHES[0] += self.kernels[b]
        return self.outs[b][:n]

    def close(self) -> None:
        self.graphs.clear()
        self.outs.clear()
        self.pool = None
