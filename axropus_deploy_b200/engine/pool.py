"""Pool of draft engines and multi-draft speculative decoding over copy-on-write KV views.

Each step the drafters of a :class:`DraftPool` (n-gram lookups of different lengths, a
draft model) propose ``k`` tokens for every greedy sequence; distinct proposals become
*branches* of the sequence. Branch 0 writes into the sequence's own pages; every other
branch is a copy-on-write view (:func:`fork_kv`): it shares the sequence's full pages
(read, never written), gets a private copy of the partially filled page it writes into and
fresh pages after it. All branches of all sequences are verified in ONE target forward
(a varlen prefill of ``k + 1`` rows per branch: the shared prefix pages are read by every
branch of a sequence at the same time, so they come from HBM once and from L2 after), the
device verify kernel gives each branch's accepted length, and each sequence keeps its
longest-accepted branch: if that is not branch 0 its private pages replace the sequence's
pages for those positions (a block-table swap, no copy), and the other branches' pages are
freed. Greedy output is unchanged by construction: every emitted token is the target's
argmax at its position.

Reference counterparts: the speculative engine with its copy-on-write KV view and the pool
of engines run per step (core/speculative_engine.h:20-75, core/engine_pool.cpp:57-145,
``engine_pool_run`` / ``engine_pool_attach_draft``); there each pool engine runs a llama.cpp
draft context on a host copy of the KV buffer, here drafts are verified on the device
against paged views of the live cache.
"""
from __future__ import annotations

import time
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass
from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .. import ops
from ..models.llama import AttnMeta
from ..ops.kvcache import PAGE
from .spec import ModelDrafter, NgramDrafter, SpecDecoder


@dataclass
class EngineResult:
    """What one pool engine did in the last step (the reference's EngineResult fields plus
    the verification outcome)."""

    tokens_generated: int = 0
    execution_time_ns: int = 0
    branches: int = 0        # distinct proposals this engine contributed
    wins: int = 0            # sequences whose kept branch was this engine's
    accepted: int = 0        # draft tokens accepted on those


@dataclass
class KvBranch:
    """A copy-on-write view of sequence ``req``'s paged KV for positions from ``start``:
    ``blocks`` = the sequence's pages before ``first_page`` (shared) + ``private`` (owned by
    the branch, the first one a copy of the sequence's page ``first_page`` when that page
    already holds positions before ``start``)."""

    req: object
    start: int
    first_page: int
    private: List[int]
    blocks: List[int]

    def release(self, bm) -> None:
        if self.private:
            bm.release(self.private)
            self.private = []


def copy_pages(cache, src: Sequence[int], dst: Sequence[int]) -> None:
    """KV (and scale) contents of pages ``src`` copied into pages ``dst`` of the same cache,
    every layer, K and V."""
    if not src:
        return
    si = torch.tensor(list(src), dtype=torch.long, device=cache.data.device)
    di = torch.tensor(list(dst), dtype=torch.long, device=cache.data.device)
    cache.data.index_copy_(2, di, cache.data.index_select(2, si))
    if cache.meta is not None:
        cache.meta.index_copy_(2, di, cache.meta.index_select(2, si))


def fork_kv(eng, req, start: int, end: int) -> Optional[KvBranch]:
    """Copy-on-write view of ``req`` for writing positions [start, end); None when the
    cache has no room for its private pages."""
    p0, p1 = start // PAGE, (end - 1) // PAGE
    n = p1 - p0 + 1
    if not eng.bm.can_allocate(n):
        return None
    private = eng.bm.allocate(n)
    if start % PAGE:
        copy_pages(eng.cache, [req.blocks[p0]], [private[0]])
    return KvBranch(req, start, p0, private, list(req.blocks[:p0]) + private)


class DraftPool:
    """Draft engines run each step (host drafters concurrently on a thread pool)."""

    def __init__(self, drafters: Sequence[object], threads: int = 4):
        self.drafters = list(drafters)
        self.results = [EngineResult() for _ in self.drafters]
        self._exec = ThreadPoolExecutor(max_workers=max(1, threads)) if len(self.drafters) > 1 else None

    def propose(self, eng, reqs, k: int) -> List[List[List[int]]]:
        """drafts[d][i]: drafter d's k tokens for reqs[i]."""
        def run(d):
            t0 = time.perf_counter_ns()
            if isinstance(d, ModelDrafter):
                out = d.propose_batch(eng, reqs, k)
            elif isinstance(d, NgramDrafter):
                out = [d.propose_req(r, k) for r in reqs]
            else:
                out = [d.propose(r.prompt + r.output, k) for r in reqs]
            return out, time.perf_counter_ns() - t0

        host = [i for i, d in enumerate(self.drafters) if not isinstance(d, ModelDrafter)]
        dev = [i for i, d in enumerate(self.drafters) if isinstance(d, ModelDrafter)]
        outs: Dict[int, tuple] = {}
        futs = {i: self._exec.submit(run, self.drafters[i]) for i in host} if self._exec else {}
        for i in dev + ([] if self._exec else host):  # device drafters on this thread (one stream)
            outs[i] = run(self.drafters[i])
        for i, f in futs.items():
            outs[i] = f.result()
        drafts = []
        for i in range(len(self.drafters)):
            toks, ns = outs[i]
            self.results[i].tokens_generated = len(reqs) * k
            self.results[i].execution_time_ns = ns
            drafts.append(toks)
        return drafts

    def forget(self, req_id: str) -> None:
        for d in self.drafters:
            if hasattr(d, "forget"):
                d.forget(req_id)

    def rewind(self, req_id: str, pos: int) -> None:
        for d in self.drafters:
            if isinstance(d, ModelDrafter):
                d.rewind(req_id, pos)

    def close(self) -> None:
        if self._exec is not None:
            self._exec.shutdown(wait=False)
            self._exec = None


class PoolSpecDecoder(SpecDecoder):
    """Speculative decoding with a pool of drafters: every distinct proposal of a sequence
    is verified in one target forward on its own copy-on-write branch; the longest
    accepted one is kept."""

    def __init__(self, engine, max_depth: int = 8, pool: Optional[DraftPool] = None, max_branches: int = 4):
        super().__init__(engine, max_depth, None)
        self.pool = pool or DraftPool([NgramDrafter(3, 1), NgramDrafter(3, 1, skip=1), NgramDrafter(6, 4)])
        self.max_branches = max_branches
        self.stat.update({"branches": 0, "branch_wins": 0})

    def step(self, reqs) -> List:
        eng = self.eng
        dev = eng.device
        k = self.depth
        for r in reqs:
            k = min(k, r.params.max_tokens - len(r.output))
        k = max(1, min(k, 64))
        drafts = self.pool.propose(eng, reqs, k)
        # distinct proposals per sequence, in drafter order (branch 0 = the first drafter's)
        plans = []  # per sequence: list of (drafter index, tokens, KvBranch or None for branch 0)
        for i, r in enumerate(reqs):
            L = r.seq_len
            seen: Dict[tuple, int] = {}
            br = []
            for d in range(len(drafts)):
                t = tuple(int(x) for x in drafts[d][i])
                if t in seen or len(br) >= self.max_branches:
                    continue
                view = None
                if br:  # branches after the first write into copy-on-write views
                    view = fork_kv(eng, r, L - 1, L + k)
                    if view is None:
                        break
                seen[t] = d
                br.append((d, list(t), view))
            plans.append(br)
        # one varlen verify forward over every branch
        toks, pos, slots, cu, lens, tables = [], [], [], [0], [], []
        flat = []
        for r, br in zip(reqs, plans):
            L = r.seq_len
            p = np.arange(L - 1, L + k)
            for (d, t, view) in br:
                blocks = r.blocks if view is None else view.blocks
                b = np.asarray(blocks, dtype=np.int64)
                toks += [r.output[-1]] + t
                pos += p.tolist()
                slots += (b[p // PAGE] * PAGE + p % PAGE).tolist()
                cu.append(cu[-1] + k + 1)
                lens.append(L + k)
                tables.append(list(blocks[: (L + k - 1) // PAGE + 1]))
                flat.append((r, d, t, view))
        width = max(len(t) for t in tables)
        bt = torch.tensor([t + [0] * (width - len(t)) for t in tables], dtype=torch.int32).to(dev, non_blocking=True)
        host = torch.tensor([toks, pos, slots], dtype=torch.int32)
        dv = host.to(dev, non_blocking=True)
        meta = AttnMeta("prefill", dv[1], dv[2], bt, torch.tensor(lens, dtype=torch.int32).to(dev, non_blocking=True),
                        cu_q=torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True), max_q=k + 1,
                        max_seq_len=max(lens), logits_idx=torch.arange(len(toks), dtype=torch.int32, device=dev))
        nb = len(flat)
        logits = eng.model.forward(dv[0], meta, eng.cache).view(nb, k + 1, -1)
        res = ops.spec_verify(logits, torch.tensor([f[2] for f in flat], dtype=torch.int32, device=dev)).tolist()
        # keep the longest-accepted branch of every sequence
        done = []
        acc_total = 0
        j = 0
        for r, br in zip(reqs, plans):
            outs = res[j:j + len(br)]
            j += len(br)
            w = max(range(len(br)), key=lambda b: (outs[b][0], -b))
            acc, _first, tok = outs[w]
            d, t, view = br[w]
            if view is not None:  # the winner's pages take over those positions
                p0 = view.first_page
                n = len(view.private)
                old = r.blocks[p0:p0 + n]
                r.blocks[p0:p0 + n] = view.private
                view.private = []
                eng.bm.release(old)
                eng._set_rows([r])
                self.pool.rewind(r.req_id, p0 * PAGE)  # draft models wrote their K/V into the old pages
                self.stat["branch_wins"] += 1
            for b, (_, _, v) in enumerate(br):
                if v is not None:
                    v.release(eng.bm)
            self.pool.results[d].wins += 1
            self.pool.results[d].accepted += acc
            for (dd, _, _) in br:
                self.pool.results[dd].branches += 1
            acc_total += acc
            for x in t[:acc] + [tok]:
                if r.state != "running":
                    break
                eng._append(r, int(x), done)
            if r.state != "running":
                self.pool.forget(r.req_id)
        n = len(reqs)
        self.stat["steps"] += 1
        self.stat["seq_steps"] += n
        self.stat["drafted"] += n * k
        self.stat["accepted"] += acc_total
        self.stat["emitted"] += acc_total + n
        self.stat["branches"] += nb
        eng.stat["decode_tokens"] += acc_total + n
        self.depth = int(self._native.thermo_next_depth(self.state, acc_total / float(n * k)))
        return done

    def stats(self) -> Dict:
        s = super().stats()
        s["engines"] = [vars(x).copy() for x in self.pool.results]
        return s
