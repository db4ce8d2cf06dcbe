"""Speculative decoding: draft -> verify on the device -> accept / roll back.

The engine's decode step becomes, for greedy requests:

1. **Draft.** :class:`NgramDrafter` proposes ``k`` tokens per sequence by prompt lookup:
   the most recent earlier occurrence of the sequence's last ``n`` tokens (``n`` from
   3 down to 1) is found and the tokens that followed it are proposed. No second model
   is needed; repetitive contexts (code, agent traces, looping greedy outputs) accept
   most drafts. (:class:`ModelDrafter` runs a small draft model instead.)
2. **Verify.** One target forward over ``[last token, d_1 .. d_k]`` per sequence (a
   varlen prefill of ``k+1`` rows at positions ``L-1 .. L-1+k``), then the
   device-resident verify kernel (argmax of every row, first mismatch by ballot;
   ``csrc/kernels/sampling.cu``) gives the accepted count and the token to emit at
   the first mismatch (or the bonus token when every draft was accepted).
3. **Roll back.** Nothing to undo: K/V written for rejected positions lies beyond the
   sequence length, is never attended, and is overwritten by the next step.

The depth ``k`` follows the native thermo controller (acceptance EMA / variance;
``csrc/native/controllers.cpp``), between 1 and ``max_depth``.

Reference counterparts: the batch executor's draft -> verify -> rollback loop and
spec v2 (core/batch_executor.cpp:398-731, core/spec_v2.cpp:286-376), its fused GPU
verify (core/kernels/spec_verify.cu) and accept scan (core/kernels/accept_scan.cu),
and the thermo controller (core/thermo_controller.h:11-34).
"""
from __future__ import annotations

from typing import Dict, List, Optional, Sequence

import numpy as np
import torch

from .. import ops
from ..models.llama import AttnMeta
from ..ops.kvcache import PAGE


class NgramDrafter:
    """Prompt-lookup drafting over the last ``window`` tokens of a sequence. ``skip`` > 0
    proposes what followed an earlier occurrence of the tail instead of the most recent
    one (a second candidate for multi-draft verification).

    :meth:`propose_req` keeps one native incremental index per request
    (``csrc/native/ngram.cpp``: every appended token adds the n-grams ending at it, a
    proposal is a hash lookup) and feeds it only the tokens generated since the last call,
    so a step costs O(new tokens) instead of a scan of the window; it releases the GIL, so
    the drafters of a pool run in parallel threads. :meth:`propose` is the stateless scan
    (any token list) and the oracle of the index."""

    def __init__(self, max_n: int = 3, min_n: int = 1, window: int = 4096, skip: int = 0):
        self.max_n, self.min_n, self.window, self.skip = max_n, min_n, window, skip
        self._tables: Dict[str, object] = {}

    def propose_req(self, r, k: int) -> List[int]:
        """``propose(r.prompt + r.output, k)`` through the request's native index."""
        ent = self._tables.get(r.req_id)
        n_prompt, total = len(r.prompt), len(r.prompt) + len(r.output)
        if ent is None or ent[1] > total:
            from .._native_loader import native

            # only the tokens a proposal can still reach are indexed: the last window + max_n
            start = max(0, total - self.window - self.max_n)
            ent = self._tables[r.req_id] = [native().NgramTable(self.max_n, self.min_n, self.window), start]
        t, have = ent
        if have < n_prompt:
            t.extend(np.asarray(r.prompt[have:], dtype=np.int32))
            t.extend(np.asarray(r.output, dtype=np.int32))
        elif have < total:
            t.extend(np.asarray(r.output[have - n_prompt:], dtype=np.int32))
        ent[1] = total
        return t.propose(k, self.skip)

    def forget(self, req_id: str) -> None:
        self._tables.pop(req_id, None)

    def propose(self, tokens: Sequence[int], k: int) -> List[int]:
        toks = np.asarray(tokens[-self.window:], dtype=np.int64)
        L = toks.shape[0]
        for n in range(self.max_n, self.min_n - 1, -1):
            if L <= n:
                continue
            tail = toks[L - n:]
            # candidate starts: positions i with toks[i:i+n] == tail and i + n < L
            cand = np.flatnonzero(toks[: L - n] == tail[0])
            skip = self.skip
            for i in cand[::-1]:
                if i + n < L and np.array_equal(toks[i:i + n], tail):
                    if skip > 0:
                        skip -= 1
                        continue
                    nxt = toks[i + n:i + n + k].tolist()
                    if nxt:
                        return (nxt + [nxt[-1]] * k)[:k]
        return [int(toks[-1])] * k if L else [0] * k


class ModelDrafter:
    """Greedy drafts from a small model with its own paged KV cache (same block ids as
    the target's, so the block tables carry over)."""

    def __init__(self, model, num_blocks: int, kv_fmt: str = "bf16"):
        from ..ops.kvcache import KVCache

        self.model = model
        self.cache = KVCache(model.num_layers, num_blocks, model.cfg.num_kv_heads, model.cfg.head_dim, kv_fmt,
                             model.device)
        self.synced: Dict[str, int] = {}  # req id -> tokens whose draft K/V is written

    def propose_batch(self, eng, reqs, k: int) -> List[List[int]]:
        dev = self.model.device
        out: List[List[int]] = [[] for _ in reqs]
        # catch the draft cache up with every sequence (prompt + accepted outputs), then
        # decode k tokens greedily
        for i, r in enumerate(reqs):
            toks = r.prompt + r.output
            have = self.synced.get(r.req_id, 0)
            n = len(toks) - 1 - have
            if n > 0:
                pos = np.arange(have, have + n)
                b = np.asarray(r.blocks, dtype=np.int64)
                slots = (b[pos // PAGE] * PAGE + pos % PAGE)
                meta = AttnMeta("prefill", torch.tensor(pos, dtype=torch.int32, device=dev),
                                torch.tensor(slots, dtype=torch.int32, device=dev),
                                eng.block_table[r.row:r.row + 1], torch.tensor([have + n], dtype=torch.int32,
                                                                                device=dev),
                                cu_q=torch.tensor([0, n], dtype=torch.int32, device=dev), max_q=n,
                                max_seq_len=have + n,
                                logits_idx=torch.tensor([n - 1], dtype=torch.int32, device=dev))
                self.model.forward(torch.tensor(toks[have:have + n], dtype=torch.int32, device=dev), meta, self.cache)
                self.synced[r.req_id] = have + n
        cur = [r.output[-1] for r in reqs]
        for step in range(k):
            pos = [len(r.prompt) + len(r.output) - 1 + step for r in reqs]
            slots = [r.blocks[p // PAGE] * PAGE + p % PAGE for r, p in zip(reqs, pos)]
            rows = torch.tensor([r.row for r in reqs], dtype=torch.long, device=dev)
            meta = AttnMeta("decode", torch.tensor(pos, dtype=torch.int32, device=dev),
                            torch.tensor(slots, dtype=torch.int32, device=dev), eng.block_table.index_select(0, rows),
                            torch.tensor([p + 1 for p in pos], dtype=torch.int32, device=dev),
                            max_seq_len=max(pos) + 1)
            logits = self.model.forward(torch.tensor(cur, dtype=torch.int32, device=dev), meta, self.cache)
            cur = ops.argmax(logits).tolist()
            for i, t in enumerate(cur):
                out[i].append(int(t))
        for r in reqs:  # drafted positions past the accepted ones are rewritten next time
            self.synced[r.req_id] = len(r.prompt) + len(r.output) - 1
        return out

    def forget(self, req_id: str) -> None:
        self.synced.pop(req_id, None)

    def rewind(self, req_id: str, pos: int) -> None:
        """The sequence's pages from ``pos`` on were replaced (a speculative branch won):
        the draft K/V written there is recomputed on the next proposal."""
        if req_id in self.synced:
            self.synced[req_id] = min(self.synced[req_id], pos)


class SpecDecoder:
    def __init__(self, engine, max_depth: int = 8, drafter=None):
        from .._native_loader import native

        self.eng = engine
        self.drafter = drafter or NgramDrafter()
        self.state = native().ThermoState(max_depth)
        self.max_depth = max_depth
        self.depth = min(4, max_depth)
        self._native = native()
        self.stat = {"steps": 0, "seq_steps": 0, "drafted": 0, "accepted": 0, "emitted": 0}

    def step(self, reqs) -> List:
        eng = self.eng
        dev = eng.device
        # room left in each sequence's allocated blocks bounds the depth
        k = self.depth
        for r in reqs:
            k = min(k, len(r.prompt) + r.params.max_tokens - (len(r.prompt) + len(r.output)))
        k = max(1, min(k, 64))
        if isinstance(self.drafter, ModelDrafter):
            drafts = self.drafter.propose_batch(eng, reqs, k)
        elif isinstance(self.drafter, NgramDrafter):
            drafts = [self.drafter.propose_req(r, k) for r in reqs]
        else:
            drafts = [self.drafter.propose(r.prompt + r.output, k) for r in reqs]
        toks, pos, slots, cu, lens = [], [], [], [0], []
        for r, d in zip(reqs, drafts):
            L = len(r.prompt) + len(r.output)
            toks += [r.output[-1]] + d
            p = np.arange(L - 1, L + k)
            pos += p.tolist()
            b = np.asarray(r.blocks, dtype=np.int64)
            slots += (b[p // PAGE] * PAGE + p % PAGE).tolist()
            cu.append(cu[-1] + k + 1)
            lens.append(L + k)
        rows = torch.tensor([r.row for r in reqs], dtype=torch.long, device=dev)
        host = torch.tensor([toks, pos, slots], dtype=torch.int32)
        d = host.to(dev, non_blocking=True)
        meta = AttnMeta("prefill", d[1], d[2], eng.block_table.index_select(0, rows),
                        torch.tensor(lens, dtype=torch.int32).to(dev, non_blocking=True),
                        cu_q=torch.tensor(cu, dtype=torch.int32).to(dev, non_blocking=True), max_q=k + 1,
                        max_seq_len=max(lens), logits_idx=torch.arange(len(toks), dtype=torch.int32, device=dev))
        logits = eng.model.forward(d[0], meta, eng.cache).view(len(reqs), k + 1, -1)
        res = ops.spec_verify(logits, torch.tensor(drafts, dtype=torch.int32, device=dev)).tolist()
        done = []
        acc_total = 0
        for r, dr, (acc, _first, tok) in zip(reqs, drafts, res):
            emit = dr[:acc] + [tok]
            acc_total += acc
            for t in emit:
                if r.state != "running":
                    break
                eng._append(r, int(t), done)
            if r.state != "running" and hasattr(self.drafter, "forget"):
                self.drafter.forget(r.req_id)
        n = len(reqs)
        self.stat["steps"] += 1
        self.stat["seq_steps"] += n
        self.stat["drafted"] += n * k
        self.stat["accepted"] += acc_total
        self.stat["emitted"] += acc_total + n
        eng.stat["decode_tokens"] += acc_total + n
        rate = acc_total / float(n * k)
        self.depth = int(self._native.thermo_next_depth(self.state, rate))
        return done

    def stats(self) -> Dict:
        s = dict(self.stat, depth=self.depth)
        s["acceptance"] = s["accepted"] / s["drafted"] if s["drafted"] else 0.0
        s["tokens_per_seq_step"] = s["emitted"] / max(1, s["seq_steps"])
        return s
